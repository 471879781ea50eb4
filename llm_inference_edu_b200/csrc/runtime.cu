// Host runtime behind the C ABI: device-resident models (Decoder,
// src/model.rs:59-340), cached sessions (CachedSession, src/kv_cache.rs:
// 156-475) and greedy generation state (GenerationSession,
// src/generation.rs:98-338).
//
// A session owns its KV cache, activations, a device control block and a
// CUDA graph that replays one decode step (control copy in, the persistent
// decode kernel, result copy out).  Handles are opaque, never reused, and
// every entry point validates before it writes.
#include <math.h>
#include <string.h>

#include <algorithm>
#include <cmath>
#include <map>
#include <memory>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "decode.cuh"
#include "prefill.cuh"
#include "sampling.cuh"
#include "tc_gemm.cuh"
#include "tp.cuh"

namespace qb {
int decode_max_ctas(int wfmt, int tfmt, int kv_bf16, size_t smem);

// ------------------------------------------------------ conversions ----

__global__ void bf16_to_f32_kernel(const uint16_t *__restrict__ s, float *__restrict__ d, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        d[i] = bf16_to_f32(s[i]);
}

__global__ void f32_to_bf16_kernel(const float *__restrict__ s, uint16_t *__restrict__ d, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        d[i] = f32_to_bf16_rne(s[i]);
}

__global__ void nonfinite_any(const float *__restrict__ v, size_t n, unsigned long long *first) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        if (!isfinite(v[i])) atomicMin(first, (unsigned long long)i);
}

// Copies columns [c0, c0 + nc) of a row-major [rows, cols] FP32 matrix into
// a padded row-major destination in format `fmt` (FP32, BF16 or biased u8
// from int8 `q`).
__global__ void relayout_kernel(const float *__restrict__ srcf, const int8_t *__restrict__ srcq,
                                size_t rows, size_t cols, size_t c0, size_t nc, uint8_t *dst,
                                size_t dst_stride, int fmt) {
    size_t n = rows * nc;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        size_t r = i / nc, c = i % nc;
        size_t s = r * cols + c0 + c;
        uint8_t *row = dst + r * dst_stride;
        if (fmt == WF_F32) ((float *)row)[c] = srcf[s];
        else if (fmt == WF_BF16) ((uint16_t *)row)[c] = f32_to_bf16_rne(srcf[s]);
        else row[c] = (uint8_t)((int)srcq[s] + 128);
    }
}

__global__ void unbias_kernel(const uint8_t *__restrict__ src, size_t rows, size_t cols, size_t stride,
                              int8_t *__restrict__ dst) {
    size_t n = rows * cols;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        size_t r = i / cols, c = i % cols;
        dst[i] = (int8_t)((int)src[r * stride + c] - 128);
    }
}

static unsigned gridn(size_t n) {
    size_t b = (n + 255) / 256;
    return (unsigned)std::max<size_t>(1, std::min<size_t>(b, 16384));
}

static size_t round16(size_t b) { return (b + 15) & ~(size_t)15; }

// RAII device buffer.
struct DevBuf {
    void *p = nullptr;
    size_t bytes = 0;
    DevBuf() = default;
    DevBuf(const DevBuf &) = delete;
    DevBuf &operator=(const DevBuf &) = delete;
    DevBuf(DevBuf &&o) noexcept : p(o.p), bytes(o.bytes) { o.p = nullptr; o.bytes = 0; }
    DevBuf &operator=(DevBuf &&o) noexcept {
        if (this != &o) { release(); p = o.p; bytes = o.bytes; o.p = nullptr; o.bytes = 0; }
        return *this;
    }
    ~DevBuf() { release(); }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        bytes = 0;
    }
    uint32_t alloc(size_t n, bool zero = true) {
        release();
        if (n == 0) n = 16;
        QB_CUDA(cudaMalloc(&p, n));
        bytes = n;
        if (zero) QB_CUDA(cudaMemset(p, 0, n));
        return QB_OK;
    }
    template <class T> T *as() const { return (T *)p; }
};

// Makes `device` current for the scope.
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur;
        if (cudaGetDevice(&cur) == cudaSuccess && prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

// ------------------------------------------------------------ model ----

struct Linear {  // one device linear in the decode layout
    DevBuf w;       // padded rows
    DevBuf scales;  // [rows] (INT8)
    size_t rows = 0, cols = 0, stride = 0;
    bool set = false;
};

struct LayerStore {
    DevBuf wqkv, sqkv, bqkv, wo, so;
    DevBuf wgu, sgu;  // gate and up rows interleaved: row 2f = gate f, 2f + 1 = up f
    Linear down;
    DevBuf attn_norm, ffn_norm;
    bool q = false, k = false, v = false, o = false, an = false, fn = false, gate = false, up = false;
};

struct Model {
    qb_model_config c{};
    int device = 0;
    // Tensor-parallel shard (tp_size 1: the whole model): query heads
    // [head0, head0 + nq), KV heads [kv0, kv0 + nkv), FFN columns
    // [f0, f0 + nff) and LM-head rows [v0, v0 + nv); the embedding table and
    // the norms are whole on every rank.
    int tp_rank = 0, tp_size = 1;
    size_t head0 = 0, nq = 0, kv0 = 0, nkv = 0, f0 = 0, nff = 0, v0 = 0, nv = 0;
    uint32_t lin = QB_LINEAR_F32, tab = QB_TABLE_F32;
    size_t sh = 0, shd = 0, sff = 0, semb = 0;
    DevBuf emb, head, final_norm;
    bool emb_set = false, head_set = false, fn_set = false, finalized = false;
    std::vector<LayerStore> layers;
    DevBuf dlayers;  // DecodeLayer[L] (weights only; sessions add KV pointers)
    size_t logical_bytes = 0;
    int wf() const { return lin == QB_LINEAR_INT8_ROW ? WF_I8 : (lin == QB_LINEAR_BF16 ? WF_BF16 : WF_F32); }
    size_t esz() const { return lin == QB_LINEAR_INT8_ROW ? 1 : (lin == QB_LINEAR_BF16 ? 2 : 4); }
    size_t tesz() const { return tab == QB_TABLE_BF16 ? 2 : 4; }
    size_t kv() const { return nkv * c.head_dim; }   // this shard's K (or V) rows
    size_t qd() const { return nq * c.head_dim; }    // this shard's Q rows
};

// The shard of rank `rank` of `size`: KV heads split evenly when size <=
// kv_heads; beyond that each KV head (and its group of query heads) is
// replicated on size / kv_heads ranks that split the group's query heads
// (sizes differ by at most one, e.g. 4 and 3 of 7); FFN columns split
// evenly; LM-head rows split in whole 128-row tiles.  False when the shape
// does not split this way.
static bool tp_split(const qb_model_config &c, int rank, int size, Model &m) {
    const size_t qh = c.query_heads, kvh = c.kv_heads, grp = qh / kvh, ff = c.ff_dim, V = c.vocab_size;
    if (size < 1 || size > kMaxTp || rank < 0 || rank >= size) return false;
    const size_t S = (size_t)size, r = (size_t)rank;
    if (S <= kvh) {
        if (kvh % S) return false;
        m.nkv = kvh / S; m.kv0 = r * m.nkv; m.nq = m.nkv * grp; m.head0 = m.kv0 * grp;
    } else {
        if (S % kvh || S / kvh > grp) return false;
        const size_t per_g = S / kvh, g = r / per_g, j = r % per_g, base = grp / per_g, extra = grp % per_g;
        m.kv0 = g; m.nkv = 1;
        m.nq = base + (j < extra ? 1 : 0);
        m.head0 = g * grp + j * base + std::min(j, extra);
    }
    if (S > 1 && (ff % S || (ff / S) % 4)) return false;
    m.nff = ff / S; m.f0 = r * m.nff;
    const size_t tiles = (V + 127) / 128, per = tiles / S, extra = tiles % S;
    const size_t t0 = r * per + std::min(r, extra), nt = per + (r < extra ? 1 : 0);
    if (nt == 0) return false;
    m.v0 = t0 * 128;
    m.nv = std::min(V, (t0 + nt) * 128) - m.v0;
    m.tp_rank = rank;
    m.tp_size = size;
    return true;
}

static std::mutex g_mu;
static uint64_t g_next = 1;
static std::map<uint64_t, std::shared_ptr<Model>> g_models;
struct Session;
struct Generation;
static std::map<uint64_t, std::shared_ptr<Session>> g_sessions;
static std::map<uint64_t, std::shared_ptr<Generation>> g_generations;
struct Sampler;
static std::map<uint64_t, std::shared_ptr<Sampler>> g_samplers;

static std::shared_ptr<Model> find_model(uint64_t h) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_models.find(h);
    return it == g_models.end() ? nullptr : it->second;
}

// Converts a host tensor (FP32 or BF16) to a temporary device FP32 buffer.
static uint32_t upload_f32(const void *data, size_t n, uint32_t dtype, DevBuf &out) {
    uint32_t s = out.alloc(n * 4, false);
    if (s) return s;
    if (dtype == QB_HOST_F32) {
        QB_CUDA(cudaMemcpy(out.p, data, n * 4, cudaMemcpyHostToDevice));
    } else {
        DevBuf tmp;
        if ((s = tmp.alloc(n * 2, false))) return s;
        QB_CUDA(cudaMemcpy(tmp.p, data, n * 2, cudaMemcpyHostToDevice));
        bf16_to_f32_kernel<<<gridn(n), 256>>>(tmp.as<uint16_t>(), out.as<float>(), n);
        QB_CUDA(cudaGetLastError());
        QB_CUDA(cudaDeviceSynchronize());
    }
    return QB_OK;
}

static uint32_t check_finite_dev(const float *p, size_t n, size_t *index) {
    void *sp;
    uint32_t s = scratch_get(64, &sp);
    if (s) return s;
    unsigned long long *f = (unsigned long long *)sp;
    QB_CUDA(cudaMemset(f, 0xff, 8));
    nonfinite_any<<<gridn(n), 256>>>(p, n, f);
    unsigned long long h;
    QB_CUDA(cudaMemcpy(&h, f, 8, cudaMemcpyDeviceToHost));
    if (h != ~0ull) {
        *index = (size_t)h;
        return QB_NONFINITE;
    }
    return QB_OK;
}

// Stores FP32 source rows into `dst` (row r at dst + r * stride), quantizing
// per row for INT8 with the bit-exact scheme of qb_quantize_int8.  Row r's
// scale goes to scales[r * scale_stride].
static uint32_t store_linear(const Model &m, const float *src, size_t rows, size_t cols, uint8_t *dst,
                             size_t stride, float *scales, size_t scale_stride) {
    const int wf = m.wf();
    if (wf == WF_I8) {
        DevBuf q, sc;
        uint32_t s;
        if ((s = q.alloc(rows * cols, false)) || (s = sc.alloc(rows * 4, false))) return s;
        s = qb_quantize_int8(src, rows * cols, rows, cols, cols, q.as<int8_t>(), sc.as<float>(), nullptr);
        if (s) return s == QB_NONFINITE_WEIGHT ? QB_NONFINITE : s;
        relayout_kernel<<<gridn(rows * cols), 256>>>(nullptr, q.as<int8_t>(), rows, cols, 0, cols, dst, stride, WF_I8);
        QB_CUDA(cudaGetLastError());
        if (scale_stride == 1) QB_CUDA(cudaMemcpy(scales, sc.p, rows * 4, cudaMemcpyDeviceToDevice));
        else QB_CUDA(cudaMemcpy2D(scales, scale_stride * 4, sc.p, 4, 4, rows, cudaMemcpyDeviceToDevice));
    } else {
        size_t idx;
        uint32_t s = check_finite_dev(src, rows * cols, &idx);
        if (s) { set_detail(0, 0, 0, idx); return s; }
        relayout_kernel<<<gridn(rows * cols), 256>>>(src, nullptr, rows, cols, 0, cols, dst, stride, wf);
        QB_CUDA(cudaGetLastError());
    }
    QB_CUDA(cudaDeviceSynchronize());
    return QB_OK;
}

// Columns [c0, c0 + nc) of a row-major [rows, cols] FP32 source, each row
// quantized (INT8) over all its columns, as the whole matrix would be.
static uint32_t store_linear_cols(const Model &m, const float *src, size_t rows, size_t cols, size_t c0, size_t nc,
                                  uint8_t *dst, size_t stride, float *scales) {
    if (c0 == 0 && nc == cols) return store_linear(m, src, rows, cols, dst, stride, scales, 1);
    const int wf = m.wf();
    uint32_t s;
    if (wf == WF_I8) {
        DevBuf q, sc;
        if ((s = q.alloc(rows * cols, false)) || (s = sc.alloc(rows * 4, false))) return s;
        s = qb_quantize_int8(src, rows * cols, rows, cols, cols, q.as<int8_t>(), sc.as<float>(), nullptr);
        if (s) return s == QB_NONFINITE_WEIGHT ? QB_NONFINITE : s;
        relayout_kernel<<<gridn(rows * nc), 256>>>(nullptr, q.as<int8_t>(), rows, cols, c0, nc, dst, stride, WF_I8);
        QB_CUDA(cudaGetLastError());
        QB_CUDA(cudaMemcpy(scales, sc.p, rows * 4, cudaMemcpyDeviceToDevice));
    } else {
        size_t idx;
        if ((s = check_finite_dev(src, rows * cols, &idx))) { set_detail(0, 0, 0, idx); return s; }
        relayout_kernel<<<gridn(rows * nc), 256>>>(src, nullptr, rows, cols, c0, nc, dst, stride, wf);
        QB_CUDA(cudaGetLastError());
    }
    QB_CUDA(cudaDeviceSynchronize());
    return QB_OK;
}

// o_proj in head-blocked form: block i holds the columns of query head
// head0 + i ([hh*hd, (hh+1)*hd)) of every row, so one head's partial
// product streams a contiguous block; a shard keeps its own heads' blocks.
static uint32_t store_o_proj(Model &m, LayerStore &L, const float *src) {
    const size_t h = m.c.hidden_dim, hd = m.c.head_dim, qh = m.nq;
    const int wf = m.wf();
    uint32_t s;
    if (wf == WF_I8) {
        DevBuf q, sc;
        if ((s = q.alloc(h * h, false)) || (s = sc.alloc(h * 4, false))) return s;
        s = qb_quantize_int8(src, h * h, h, h, h, q.as<int8_t>(), sc.as<float>(), nullptr);
        if (s) return s == QB_NONFINITE_WEIGHT ? QB_NONFINITE : s;
        for (size_t hh = 0; hh < qh; ++hh)
            relayout_kernel<<<gridn(h * hd), 256>>>(nullptr, q.as<int8_t>(), h, h, (m.head0 + hh) * hd, hd,
                                                    L.wo.as<uint8_t>() + hh * h * m.shd, m.shd, WF_I8);
        QB_CUDA(cudaMemcpy(L.so.p, sc.p, h * 4, cudaMemcpyDeviceToDevice));
    } else {
        size_t idx;
        if ((s = check_finite_dev(src, h * h, &idx))) { set_detail(0, 0, 0, idx); return s; }
        for (size_t hh = 0; hh < qh; ++hh)
            relayout_kernel<<<gridn(h * hd), 256>>>(src, nullptr, h, h, (m.head0 + hh) * hd, hd,
                                                    L.wo.as<uint8_t>() + hh * h * m.shd, m.shd, wf);
    }
    QB_CUDA(cudaGetLastError());
    QB_CUDA(cudaDeviceSynchronize());
    return QB_OK;
}

static uint32_t host_vector_finite(const void *data, size_t n, uint32_t dtype, std::vector<float> &out) {
    out.resize(n);
    for (size_t i = 0; i < n; ++i) {
        float v;
        if (dtype == QB_HOST_F32) v = ((const float *)data)[i];
        else {
            uint32_t u = (uint32_t)((const uint16_t *)data)[i] << 16;
            memcpy(&v, &u, 4);
        }
        if (!isfinite(v)) {
            set_detail(0, 0, 0, i);
            return QB_NONFINITE;
        }
        out[i] = v;
    }
    return QB_OK;
}

// ---------------------------------------------------------- session ----

struct Session {
    std::shared_ptr<Model> m;
    int device = 0;
    size_t capacity = 0, processed = 0;
    bool valid = true;
    int kv_bf16 = 0;
    size_t logical_bytes = 0, workspace_bytes = 0;
    size_t kv_layer_bytes = 0;  // bytes of one layer's K (or V) page pool
    cudaStream_t stream = nullptr;
    DevBuf kv, ptab, rope, xch, logits, amax_v, amax_i, emitted, ctrl, dlayers, geom, apart, hbar;
    DecodeCtrl *hctrl = nullptr;  // pinned mirror
    std::vector<DecodeLayer> hlayers;  // host copy of the layer table (chunked prompt path)
    DevBuf pf;                         // chunked prompt workspace (allocated on first use)
    std::unique_ptr<TcMaps> tcm;       // its tensor maps (built with it)
    DecodeParams params{};
    int grid = 0;
    // One-step graphs: the decode kernel without, and with, the long-context
    // position-split attention.
    cudaGraphExec_t g_host = nullptr, g_host_split = nullptr;
    bool logits_valid = false;
    ~Session() {
        DeviceGuard dg(device);
        if (g_host) cudaGraphExecDestroy(g_host);
        if (g_host_split) cudaGraphExecDestroy(g_host_split);
        if (hctrl) cudaFreeHost(hctrl);
        if (stream) cudaStreamDestroy(stream);
    }
};

static std::shared_ptr<Session> find_session(uint64_t h) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_sessions.find(h);
    return it == g_sessions.end() ? nullptr : it->second;
}

// workspace_bytes, src/kv_cache.rs:114-127 (the reference's resident vector
// payload formula, kept so budgets and reports agree with the reference).
static size_t ref_workspace_bytes(const qb_model_config &c, size_t capacity) {
    return (c.hidden_dim * 8 + c.kv_heads * c.head_dim * 3 + c.ff_dim * 3 + capacity * 2) * 4;
}

// RoPE table [cap][hd/2] of (cos, sin): the reference's f32 powf/sin/cos per
// position (src/rope.rs:83-90), computed on the host with the C library.
static uint32_t build_rope(const qb_model_config &c, size_t cap, DevBuf &out) {
    const size_t half = c.head_dim / 2;
    std::vector<float> tab(cap * half * 2);
    std::vector<float> freq(half);
    for (size_t j = 0; j < half; ++j) freq[j] = powf(c.rope_base, -((float)(2 * j)) / (float)c.head_dim);
    for (size_t t = 0; t < cap; ++t) {
        float pos = (float)t;
        for (size_t j = 0; j < half; ++j) {
            float a = pos * freq[j];
            tab[(t * half + j) * 2] = cosf(a);
            tab[(t * half + j) * 2 + 1] = sinf(a);
        }
    }
    uint32_t st = out.alloc(tab.size() * 4, false);
    if (st) return st;
    QB_CUDA(cudaMemcpy(out.p, tab.data(), tab.size() * 4, cudaMemcpyHostToDevice));
    return QB_OK;
}

// The model-level fields of the multi-token arguments, for a cache of `cap`
// positions per sequence.
static void prefill_common(const Model &m, size_t cap, int kv_bf16, PrefillArgs &a) {
    const qb_model_config &c = m.c;
    a.V = (int)m.nv; a.L = (int)c.layers; a.h = (int)c.hidden_dim; a.qh = (int)m.nq;
    a.kvh = (int)m.nkv; a.hd = (int)c.head_dim; a.ff = (int)m.nff; a.cap = (int)cap;
    a.group = (int)(m.nq / m.nkv);
    a.qd = (int)m.qd(); a.v0 = (int)m.v0;
    a.wfmt = m.wf(); a.tfmt = m.tab == QB_TABLE_BF16 ? WF_BF16 : WF_F32; a.kv_bf16 = kv_bf16;
    a.eps = c.norm_epsilon; a.sqrt_hd = sqrtf((float)c.head_dim);
    a.sh = m.sh; a.shd = m.shd; a.sff = m.sff; a.semb = m.semb;
    a.emb = m.emb.as<uint8_t>();
    // A shard's LM head: its rows of the untied head, or of the tied table.
    a.head = m.head_set ? m.head.as<uint8_t>() : m.emb.as<uint8_t>() + m.v0 * m.semb;
    a.final_norm = m.final_norm.as<float>();
    a.tp = nullptr;
    a.tp_seq = nullptr;
    a.tp_timeout_ns = 2000000000ull;
    a.kv.kvh = (int)m.nkv;
    a.kv.hd = (int)c.head_dim;
}

// Carves the multi-token workspace for `chunk` rows out of one buffer
// (allocated on first use): activations, split-K partials, ids, positions,
// sequences, the error word and the BF16 input planes of the tensor-core
// GEMMs.
static uint32_t prefill_workspace(const Model &m, int chunk, DevBuf &ws, PrefillArgs &a) {
    const size_t h = m.c.hidden_dim, ff = m.nff, rq = m.qd() + 2 * m.kv(), ch = (size_t)chunk;
    const size_t part = 4 * ch * std::max(rq, h);
    const size_t floats = ch * (4 * h + rq + ff) + part + 3 * ch + 64;
    const size_t fbytes = round16(floats * 4);
    const size_t hp = round16((size_t)TC_NP * ch * h * 2), fp = round16((size_t)TC_NP * ch * ff * 2);
    // Attention split partials: every row's full-length splits plus room for
    // the extra splits of small row counts; greedy partials per 128-row tile.
    const size_t kvh = m.nkv, grp = m.nq / kvh, hd = m.c.head_dim;
    const size_t apart = (ch * kvh * ((a.cap + 1023) / 1024) + 600) * grp * (hd + 2);
    const size_t am = std::max<size_t>((m.nv + 127) / 128, tp_argmax_scratch(1)) * ch;  // tile or slice partials
    const size_t abytes = round16(apart * 4), ambytes = round16(am * 4);
    if (!ws.p) {
        uint32_t st = ws.alloc(fbytes + 2 * hp + fp + abytes + 2 * ambytes);
        if (st) return st;
    }
    float *f = ws.as<float>();
    a.chunk = chunk;
    a.x = f; a.xn = a.x + ch * h; a.h2 = a.xn + ch * h; a.ctx = a.h2 + ch * h;
    a.qkv = a.ctx + ch * h; a.act = a.qkv + ch * rq; a.part = a.act + ch * ff; a.part_floats = part;
    a.ids = (uint32_t *)(a.part + part); a.pos = (int *)(a.ids + ch); a.seq = a.pos + ch;
    a.err = (unsigned *)(a.seq + ch);
    uint8_t *pl = ws.as<uint8_t>() + fbytes;
    a.xnp = (uint16_t *)pl;
    a.ctxp = (uint16_t *)(pl + hp);
    a.actp = (uint16_t *)(pl + 2 * hp);
    a.apart = (float *)(pl + 2 * hp + fp);
    a.apart_floats = apart;
    a.amv = (float *)(pl + 2 * hp + fp + abytes);
    a.ami = (int *)(pl + 2 * hp + fp + abytes + ambytes);
    return QB_OK;
}

// Tensor maps of the tensor-core GEMMs over this workspace: the linears when
// they are INT8 (per-row scales) or BF16 and every shape suits TMA, the LM
// head when its table is BF16.  What is not covered runs on the CUDA cores.
static void tc_prepare(const Model &m, PrefillArgs &a, TcMaps &maps) {
    a.tc = nullptr;
    maps.layers.clear();
    maps.head.wf = -1;
    if (!tc_encode_planes(maps.xn, a.xnp, a.h, a.chunk) || !tc_encode_planes(maps.ctx, a.ctxp, a.qd, a.chunk) ||
        !tc_encode_planes(maps.act, a.actp, a.ff, a.chunk))
        return;
    const int wf = m.wf();
    if (wf == WF_I8 || wf == WF_BF16) {
        const size_t h = a.h, ff = a.ff, rq = (size_t)a.qd + 2 * (size_t)a.kvh * a.hd;
        maps.layers.resize(a.L);
        bool ok = true;
        for (int l = 0; l < a.L && ok; ++l) {
            const DecodeLayer &Ly = a.layers[l];
            TcLayerMaps &M = maps.layers[l];
            ok = tc_encode_weight(M.qkv, Ly.wqkv, wf, rq, h, a.sh, 1, 0) &&
                 tc_encode_weight(M.o, Ly.wo, wf, h, a.hd, a.shd, a.qh, h * a.shd) &&
                 tc_encode_weight(M.gu, Ly.wgu, wf, 2 * ff, h, a.sh, 1, 0) &&
                 tc_encode_weight(M.down, Ly.wd, wf, h, ff, a.sff, 1, 0);
        }
        if (!ok) maps.layers.clear();
    }
    if (a.tfmt == WF_BF16) tc_encode_weight(maps.head, a.head, WF_BF16, a.V, a.h, a.semb, 1, 0);
    a.tc = &maps;
}

// KV-cache pages of a cache of `cap` positions per sequence: 16 positions
// each, ceil(cap / 16) per sequence.
static size_t pages_per_seq(size_t cap) { return (cap + kPageTokens - 1) / kPageTokens; }

static uint32_t session_build(Session &s) {
    Model &m = *s.m;
    const qb_model_config &c = m.c;
    const size_t L = c.layers, kvh = c.kv_heads, hd = c.head_dim, cap = s.capacity;
    const size_t esz = s.kv_bf16 ? 2 : 4;
    // The KV cache is a pool of 16-position pages per layer (K and V pools),
    // each page [kv_heads][16][head_dim]; the session's page table maps its
    // page j (positions 16 j .. 16 j + 15) to a pool page.  The pool is
    // allocated whole at creation (the reference's capacity is fixed too)
    // and the table hands the pages out last to first, so every access goes
    // through the table.
    const size_t npages = pages_per_seq(cap);
    const size_t per = npages * kvh * kPageTokens * hd * esz;
    uint32_t st;
    QB_CUDA(cudaStreamCreateWithFlags(&s.stream, cudaStreamNonBlocking));
    s.kv_layer_bytes = round16(per);
    if ((st = s.kv.alloc(s.kv_layer_bytes * 2 * L))) return st;
    {
        std::vector<int> tab(npages);
        for (size_t j = 0; j < npages; ++j) tab[j] = (int)(npages - 1 - j);
        if ((st = s.ptab.alloc(npages * 4, false))) return st;
        QB_CUDA(cudaMemcpy(s.ptab.p, tab.data(), npages * 4, cudaMemcpyHostToDevice));
    }
    if ((st = build_rope(c, cap, s.rope))) return st;
    const size_t rqkv = c.hidden_dim + 2 * kvh * hd;
    int dev_sms = 0;
    QB_CUDA(cudaDeviceGetAttribute(&dev_sms, cudaDevAttrMultiProcessorCount, s.device));
    s.grid = dev_sms;
    // Exchange vectors: per layer qkv, per-head o_proj partials, SwiGLU
    // activations and the layer output, each 16-byte aligned, in two
    // parities, every word starting as kNotReady (all bits set).
    auto al4 = [](size_t v) { return (v + 3) & ~(size_t)3; };
    const size_t x_part = al4(rqkv), x_act = x_part + al4(c.query_heads * c.hidden_dim);
    const size_t x_hid = x_act + al4(c.ff_dim), xl = x_hid + al4(c.hidden_dim);
    if (2 * L * xl >= (1ull << 31)) return QB_UNSUPPORTED;
    if ((st = s.xch.alloc(2 * L * xl * 4, false))) return st;
    QB_CUDA(cudaMemset(s.xch.p, 0xff, s.xch.bytes));
    if ((st = s.logits.alloc(c.vocab_size * 4)) || (st = s.amax_v.alloc(s.grid * 4)) ||
        (st = s.amax_i.alloc(s.grid * 4)) || (st = s.emitted.alloc(cap * 4)) ||
        (st = s.ctrl.alloc(sizeof(DecodeCtrl))))
        return st;
    QB_CUDA(cudaMallocHost((void **)&s.hctrl, sizeof(DecodeCtrl)));
    memset(s.hctrl, 0, sizeof(DecodeCtrl));
    // Per-session layer table: the model's weights plus this session's KV.
    std::vector<DecodeLayer> dl(L);
    QB_CUDA(cudaMemcpy(dl.data(), m.dlayers.p, L * sizeof(DecodeLayer), cudaMemcpyDeviceToHost));
    for (size_t l = 0; l < L; ++l) {
        dl[l].kc = s.kv.as<uint8_t>() + round16(per) * (2 * l);
        dl[l].vc = s.kv.as<uint8_t>() + round16(per) * (2 * l + 1);
    }
    if ((st = s.dlayers.alloc(L * sizeof(DecodeLayer), false))) return st;
    QB_CUDA(cudaMemcpy(s.dlayers.p, dl.data(), L * sizeof(DecodeLayer), cudaMemcpyHostToDevice));
    s.hlayers = dl;

    DecodeParams &p = s.params;
    const int wf = m.wf();
    const int epc = wf == WF_I8 ? 16 : (wf == WF_BF16 ? 8 : 4);
    const int tepc = m.tab == QB_TABLE_BF16 ? 8 : 4;
    p.V = (int)c.vocab_size; p.L = (int)L; p.h = (int)c.hidden_dim; p.qh = (int)c.query_heads;
    p.kvh = (int)kvh; p.hd = (int)hd; p.ff = (int)c.ff_dim; p.cap = (int)cap;
    p.group = (int)(c.query_heads / kvh);
    p.wfmt = wf; p.tfmt = m.tab == QB_TABLE_BF16 ? WF_BF16 : WF_F32; p.kv_bf16 = s.kv_bf16;
    p.eps = c.norm_epsilon;
    p.sqrt_hd = sqrtf((float)hd);
    p.sh = m.sh; p.shd = m.shd; p.sff = m.sff; p.semb = m.semb;
    p.ch = (int)(m.sh / 16); p.chd = (int)(m.shd / 16); p.cff = (int)(m.sff / 16); p.cemb = (int)(m.semb / 16);
    p.rqkv = (int)rqkv;
    p.ptab = s.ptab.as<int>();
    const int s_o = std::max(1, std::min(kMaxSplits, s.grid / std::max(1, p.qh)));  // CTAs per query head
    p.emb = m.emb.as<uint8_t>();
    p.head = m.head_set ? m.head.as<uint8_t>() : m.emb.as<uint8_t>();
    p.final_norm = m.final_norm.as<float>();
    p.layers = s.dlayers.as<DecodeLayer>();
    p.rope = s.rope.as<float2>();
    p.xch = s.xch.as<float>();
    p.xl = (int)xl; p.x_qkv = 0; p.x_part = (int)x_part; p.x_act = (int)x_act; p.x_hid = (int)x_hid;
    p.logits = s.logits.as<float>();
    p.amax_v = s.amax_v.as<float>(); p.amax_i = s.amax_i.as<int>(); p.emitted = s.emitted.as<int>();
    p.ctrl = s.ctrl.as<DecodeCtrl>();
    p.timeout_ns = 2000000000ull;
    p.prefetch = 1;
    // Three phases are prefetched ahead: each may hold 24 MB of L2 across
    // the grid, so larger blocks (the 7B shape's gate/up and down) are
    // prefetched only in part instead of evicting themselves before their
    // copies read them.
    p.pf_cap = (24ull << 20) / (unsigned long long)std::max(1, s.grid);
    p.withhold = 0;
    // Rows each CTA owns in every phase (floor(n * b / G) splits), and its
    // attention items: (query head, o_proj row range) pairs wi = b + m * G.
    std::vector<CtaGeom> geo(s.grid);
    auto lo = [&](long long n, int b) { return (int)(n * b / s.grid); };
    int max_qkv = 0, max_gu = 0, max_dn = 0, max_lm = 0, max_att = 0;
    for (int b = 0; b < s.grid; ++b) {
        CtaGeom &g = geo[b];
        memset(&g, 0, sizeof(g));
        g.qkv_r0 = lo(p.rqkv, b); g.qkv_n = lo(p.rqkv, b + 1) - g.qkv_r0;
        g.gu_f0 = lo(p.ff, b); g.gu_n = lo(p.ff, b + 1) - g.gu_f0;
        g.dn_r0 = lo(p.h, b); g.dn_n = lo(p.h, b + 1) - g.dn_r0;
        g.lm_v0 = lo(p.V, b); g.lm_n = lo(p.V, b + 1) - g.lm_v0;
        for (int wi = b; wi < p.qh * s_o; wi += s.grid) {
            if (g.natt == kMaxAttItems) return QB_UNSUPPORTED;
            const int sp = wi % s_o;
            const int r0 = (int)((long long)p.h * sp / s_o), r1 = (int)((long long)p.h * (sp + 1) / s_o);
            g.att_hh[g.natt] = wi / s_o;
            g.att_sp[g.natt] = sp;
            g.att_r0[g.natt] = r0;
            g.att_n[g.natt] = r1 - r0;
            max_att = std::max(max_att, r1 - r0);
            ++g.natt;
        }
        max_qkv = std::max(max_qkv, g.qkv_n); max_gu = std::max(max_gu, g.gu_n);
        max_dn = std::max(max_dn, g.dn_n); max_lm = std::max(max_lm, g.lm_n);
    }
    if ((size_t)p.V * s.grid >= (1ull << 31)) return QB_UNSUPPORTED;
    // Position-split attention for long contexts: each head's s_o CTAs take
    // a range of positions and combine through a per-head barrier.  Only
    // when every CTA has at most one attention item (no CTA waits on a head
    // whose other members are busy with another head) and the key rows
    // suit the vectorised path.
    {
        const size_t row_bytes = hd * (s.kv_bf16 ? 2 : 4), nc = row_bytes / 16;
        const bool vec = row_bytes % 16 == 0 && nc <= 32 && (nc & (nc - 1)) == 0;
        p.att_splits = (p.qh * s_o <= s.grid && s_o > 1 && vec) ? s_o : 1;
        p.att_split_min = 512;
        if ((st = s.apart.alloc((size_t)p.qh * s_o * (hd + 2) * 4, false)) ||
            (st = s.hbar.alloc((size_t)p.qh * 4)))
            return st;
        p.apart = s.apart.as<float>();
        p.hbar = s.hbar.as<unsigned>();
    }
    if ((st = s.geom.alloc(geo.size() * sizeof(CtaGeom), false))) return st;
    QB_CUDA(cudaMemcpy(s.geom.p, geo.data(), geo.size() * sizeof(CtaGeom), cudaMemcpyHostToDevice));
    p.geom = s.geom.as<CtaGeom>();

    // Shared-memory carve-up (floats).
    auto r4 = [](long long v) { return (int)((v + 3) & ~3LL); };
    const int xs = r4(std::max({(long long)p.ch * epc, (long long)p.chd * epc, (long long)p.cff * epc,
                                (long long)p.cemb * tepc}));
    const int h4 = r4(p.h);
    const int rv = r4(std::max({2 * max_qkv, 2 * max_gu, max_dn, max_att}) + 4);
    const int sc = r4(std::max({(int)cap, max_lm, 64}));
    const int q = r4(3 * p.hd);
    const int red = r4(std::max(64, 2 * 16 + 16 * p.hd));  // softmax partials, then [warp][hd] context partials
    const int lay = r4((long long)(L * sizeof(DecodeLayer) / 4));
    const int ptb = r4((long long)pages_per_seq(cap + 1));  // staged page table (one int per page)
    p.sm_xs = 0; p.sm_h2 = xs; p.sm_gain = p.sm_h2 + h4; p.sm_rv = p.sm_gain + 2 * h4;
    p.sm_gain_n = h4; p.sm_rv_n = rv;
    p.sm_sc = p.sm_rv + 2 * rv; p.sm_q = p.sm_sc + sc; p.sm_red = p.sm_q + q; p.sm_lay = p.sm_red + red;
    p.sm_ptab = p.sm_lay + lay;
    // Weight ring: slots of at least 16 KB holding whole rows (and whole
    // gate/up pairs), as many as fit the remaining shared memory (at most
    // 16), 128-byte aligned; the full/empty mbarriers (2 per slot, 8 bytes
    // each) precede it.
    size_t max_row = std::max({2 * m.sh, m.shd, m.sff, 2 * m.semb});  // gate/up and LM-head rows go in pairs
    p.slot_bytes = (int)std::max<size_t>(16384, (max_row + 127) & ~(size_t)127);
    p.sm_bar = (p.sm_ptab + ptb + 3) & ~3;
    p.sm_ring = (p.sm_bar + 2 * 2 * 16 + 31) & ~31;
    const size_t budget = 227 * 1024 - 1024;  // CTA limit less the static shared memory
    const size_t used = (size_t)p.sm_ring * 4;
    int nslot = used < budget ? (int)((budget - used) / p.slot_bytes) : 0;
    if (nslot > 16) nslot = 16;
    if (nslot < 2) return QB_UNSUPPORTED;
    p.nslot = nslot;
    p.sm_total = p.sm_ring + nslot * p.slot_bytes / 4;
    // Per-kind geometry of the streamed blocks.  The team size G = 2^lgG
    // minimises the critical path: rounds of units times (chunk products per
    // lane plus a fixed cost per round for the butterfly and epilogue).
    const size_t strides[NKIND] = {m.sh, m.shd, m.sh, m.sff, m.semb};
    const int rows_max[NKIND] = {max_qkv, max_att, 2 * max_gu, max_dn, max_lm};
    for (int k = 0; k < NKIND; ++k) {
        KindGeom &g = p.kind[k];
        g.stride = (int)strides[k];
        g.C = (int)(strides[k] / 16);
        // Row pairs (gate/up pairs; elsewhere two rows sharing the activation
        // loads) where two rows fit a slot, else single rows.
        g.U = (k == K_GU || k == K_LM || 2 * strides[k] <= (size_t)p.slot_bytes) ? 2 : 1;
        g.rpc = std::max(g.U, (p.slot_bytes / g.stride) / g.U * g.U);
        g.rpc_magic = g.rpc > 1 ? (unsigned)(((1ull << 32) + g.rpc - 1) / g.rpc) : 0u;  // rpc == 1 divides directly
        if ((size_t)g.rpc * strides[k] > (size_t)p.slot_bytes) return QB_UNSUPPORTED;  // a slot's rows must fit it
        const int block_slots = std::max(1, (rows_max[k] + g.rpc - 1) / g.rpc);
        // A per-layer block is consumed in one wave (its weights are already
        // resident); a longer stream (the LM head) in waves of a third of the
        // ring (at most three slots), so the rest keeps copies in flight.
        g.wave = block_slots <= nslot / 2 ? block_slots : std::max(1, std::min(3, nslot / 3));
        const int units = std::max(1, (std::min(rows_max[k], g.wave * g.rpc) + g.U - 1) / g.U);
        if (k == K_LM) {
            long long best = -1;
            for (int lg = 2; lg <= 5; ++lg) {  // team sizes 4 .. 32 (a run-time value on the device)
                const int G = 1 << lg, teams = kDecodeThreads / G;
                const long long rounds = (units + teams - 1) / teams;
                const long long cost = rounds * ((long long)((g.C + G - 1) / G) * 4 * g.U + 20 + 2 * lg);
                if (best < 0 || cost < best) { best = cost; g.lgG = lg; }
            }
        } else {
            // Per-layer blocks: the fewest rounds, then the most lanes with
            // chunks to multiply (one warp per SM sub-partition leaves its
            // dependent chains exposed; more busy warps hide them), then the
            // smaller team.  Teams of 64 or 128 threads span warps and meet
            // at a named barrier.
            long long best_rounds = -1, best_busy = -1;
            for (int lg = 2; lg <= 7; ++lg) {
                const int G = 1 << lg, teams = kDecodeThreads / G;
                const long long rounds = (units + teams - 1) / teams;
                const long long busy = (long long)std::min(units, teams) * std::min(G, g.C);
                if (best_rounds < 0 || rounds < best_rounds || (rounds == best_rounds && busy > best_busy)) {
                    best_rounds = rounds;
                    best_busy = busy;
                    g.lgG = lg;
                }
            }
        }
    }
    size_t smem = decode_smem_bytes(p);
    if (smem > 227 * 1024) return QB_UNSUPPORTED;
    int maxc = decode_max_ctas(wf, p.tfmt, s.kv_bf16, smem);
    if (maxc < s.grid) return QB_UNSUPPORTED;

    // Graphs: control block in, one decode step, result out.
    for (int split = 0; split < 2; ++split) {
        cudaGraphExec_t &gx = split ? s.g_host_split : s.g_host;
        cudaGraph_t g = nullptr;
        QB_CUDA(cudaStreamBeginCapture(s.stream, cudaStreamCaptureModeThreadLocal));
        cudaError_t e1 = cudaMemcpyAsync(s.ctrl.p, s.hctrl, 16, cudaMemcpyHostToDevice, s.stream);
        cudaError_t e2 = decode_launch(p, s.grid, s.stream, split != 0);
        cudaError_t e3 =
            cudaMemcpyAsync((char *)s.hctrl + 16, (char *)s.ctrl.p + 16, 8, cudaMemcpyDeviceToHost, s.stream);
        cudaError_t e4 = cudaStreamEndCapture(s.stream, &g);
        if (e1 == cudaSuccess && e2 == cudaSuccess && e3 == cudaSuccess && e4 == cudaSuccess) {
            cudaError_t e5 = cudaGraphInstantiate(&gx, g, 0);
            if (e5 != cudaSuccess) gx = nullptr;
        } else {
            gx = nullptr;
            cudaGetLastError();
        }
        if (g) cudaGraphDestroy(g);
    }
    s.logical_bytes = kvh * cap * hd * 2 * L * 4;  // the reference's FP32 KV count
    s.workspace_bytes = ref_workspace_bytes(c, cap);
    return QB_OK;
}

// Whether the step at cached position `pos` takes the decode kernel with the
// position-split attention (from att_split_min cached positions on).
static bool split_at(const Session &s, size_t pos) {
    return s.params.att_splits > 1 && pos + 1 >= (size_t)s.params.att_split_min;
}

// One decode step with a host-supplied token (graph replay).
static uint32_t session_launch(Session &s, uint32_t token, bool want_logits) {
    s.hctrl->token = (int)token;
    s.hctrl->pos = (int)s.processed;
    s.hctrl->write_logits = want_logits ? 1 : 0;
    const bool split = split_at(s, s.processed);
    cudaGraphExec_t gx = split ? s.g_host_split : s.g_host;
    if (gx) {
        QB_CUDA(cudaGraphLaunch(gx, s.stream));
    } else {
        QB_CUDA(cudaMemcpyAsync(s.ctrl.p, s.hctrl, 16, cudaMemcpyHostToDevice, s.stream));
        QB_CUDA(decode_launch(s.params, s.grid, s.stream, split));
        QB_CUDA(cudaMemcpyAsync((char *)s.hctrl + 16, (char *)s.ctrl.p + 16, 8, cudaMemcpyDeviceToHost, s.stream));
    }
    return QB_OK;
}

// Execution error: invalidate (src/kv_cache.rs:335-345) and clear the
// device control block and the exchange so the next step starts clean.
static uint32_t session_fail(Session &s, uint32_t status) {
    s.valid = false;
    s.processed = 0;
    s.logits_valid = false;
    cudaMemsetAsync(s.ctrl.p, 0, sizeof(DecodeCtrl), s.stream);
    if (s.hbar.p) cudaMemsetAsync(s.hbar.p, 0, s.hbar.bytes, s.stream);
    // Epoch 0 again: both parities of the exchange start not ready.
    if (s.xch.p) cudaMemsetAsync(s.xch.p, 0xff, s.xch.bytes, s.stream);
    cudaStreamSynchronize(s.stream);
    memset(s.hctrl, 0, sizeof(DecodeCtrl));
    return status;
}

static uint32_t session_finish(Session &s, float *logits, uint32_t *argmax) {
    cudaError_t e = cudaStreamSynchronize(s.stream);
    if (e != cudaSuccess) return session_fail(s, cuda_status(e));
    unsigned err = s.hctrl->error;
    if (err) return session_fail(s, (err & ERR_TIMEOUT) ? QB_DEVICE_TIMEOUT : QB_NONFINITE);
    if (logits) {
        e = cudaMemcpy(logits, s.logits.p, s.m->c.vocab_size * 4, cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) return session_fail(s, cuda_status(e));
    }
    if (argmax) *argmax = (uint32_t)s.hctrl->next_token;
    s.processed += 1;
    return QB_OK;
}

static uint32_t session_step(Session &s, uint32_t token, float *logits, size_t logits_len,
                             uint32_t *argmax, bool keep_logits) {
    if (!s.valid) return QB_INVALID_STATE;
    if (logits && logits_len != s.m->c.vocab_size) return QB_INVALID_OUTPUT_LENGTH;
    if (token >= s.m->c.vocab_size) return QB_INVALID_TOKEN;
    if (s.processed == s.capacity) return QB_FULL;
    DeviceGuard dg(s.device);
    uint32_t st = session_launch(s, token, logits != nullptr || keep_logits);
    if (st) return session_fail(s, st);
    st = session_finish(s, logits, argmax);
    if (!st) s.logits_valid = logits != nullptr || keep_logits;
    return st;
}

// --------------------------------------------------------- sampler ----

// Sampler (src/sampling.rs:19-110): the policy, the host generator and the
// device buffers of the selection kernel.
struct Sampler {
    int device = 0;
    SamplePolicy policy;
    uint64_t seed = 0;
    ChaCha8Rng rng;
    DevBuf scratch, staged, result;
    int scratch_n = 0;
    size_t staged_n = 0;
    uint32_t *hres = nullptr;  // pinned copy of the result words
    cudaStream_t stream = nullptr;
    std::mutex mu;
    ~Sampler() {
        DeviceGuard dg(device);
        if (hres) cudaFreeHost(hres);
        if (stream) cudaStreamDestroy(stream);
    }
};

// Sampler::new, src/sampling.rs:24-42.
static bool policy_ok(const qb_sampling *p) {
    if (!p || p->kind == QB_SAMPLING_GREEDY) return true;
    return p->kind == QB_SAMPLING_TEMPERATURE && std::isfinite(p->temperature) && p->temperature > 0.0f &&
           p->top_k != 0;
}

static uint32_t sampler_init(const qb_sampling *p, int device, Sampler &sp) {
    if (!policy_ok(p)) return QB_INVALID_PARAMETERS;
    const bool greedy = !p || p->kind == QB_SAMPLING_GREEDY;
    sp.device = device;
    sp.policy.greedy = greedy;
    sp.policy.temperature = greedy ? 1.0f : p->temperature;
    sp.policy.top_k = greedy ? 1 : (size_t)p->top_k;
    sp.seed = greedy ? 0 : p->seed;
    sp.rng.seed_from_u64(sp.seed);
    DeviceGuard dg(device);
    QB_CUDA(cudaMallocHost((void **)&sp.hres, 8));
    return sp.result.alloc(8);
}

// validate_vocab, src/sampling.rs:43-49.
static bool sampler_vocab_ok(const Sampler &sp, size_t vocab) {
    return vocab != 0 && (sp.policy.greedy || sp.policy.top_k <= vocab);
}

// Sampler::sample, src/sampling.rs:57-110, over device logits on `st` (the
// sampler's device current).  The reference's checks in its order: empty,
// non-finite (found by the kernel), top_k > n; on any error the stream is
// left where it was.
static uint32_t sampler_run(Sampler &sp, const float *logits, size_t n, cudaStream_t st, uint32_t *id) {
    if (n == 0) return QB_EMPTY_LOGITS;
    if (n > (size_t)INT32_MAX) return QB_INVALID_PARAMETERS;
    if (sp.scratch_n < (int)n) {
        uint32_t e = sp.scratch.alloc(sample_scratch_bytes((int)n), false);
        if (e) return e;
        sp.scratch_n = (int)n;
    }
    const bool vocab_ok = sampler_vocab_ok(sp, n);
    SamplePolicy pol = sp.policy;
    if (!vocab_ok) pol.greedy = true;  // only the finiteness check runs
    const ChaCha8Rng saved = sp.rng;
    const double u = pol.greedy ? 0.0 : sp.rng.next_f64();
    cudaError_t e = sample_launch(logits, (int)n, pol, u, sp.scratch.p, sp.result.as<uint32_t>(), st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(sp.hres, sp.result.p, 8, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
        sp.rng = saved;
        return cuda_status(e);
    }
    if (sp.hres[1] != 0) {
        sp.rng = saved;
        return sp.hres[1];
    }
    if (!vocab_ok) return QB_INVALID_PARAMETERS;
    *id = sp.hres[0];
    return QB_OK;
}

// ------------------------------------------------------- generation ----

struct Generation {
    std::shared_ptr<Session> cache;
    std::unique_ptr<Sampler> sampler;  // null: greedy through the fused argmax
    std::vector<uint32_t> history;
    std::vector<uint32_t> stops;
    size_t max_new = 0, generated = 0;
    int stop = QB_STOP_NONE;
    bool logits_ready = false;
    uint32_t last_argmax = 0;
    uint32_t vocab = 0;
};

static std::shared_ptr<Generation> find_generation(uint64_t h) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_generations.find(h);
    return it == g_generations.end() ? nullptr : it->second;
}

static bool cancelled(const volatile int32_t *c) { return c && *c != 0; }

// Chunked evaluation of a run of prompt tokens (all but the last of an
// append); fills the cache and advances `processed`.  Shapes the chunked
// kernels do not cover return QB_UNSUPPORTED without touching the session.
static constexpr int kPrefillChunk = 512;

static uint32_t session_prefill_chunked(Session &s, const uint32_t *tokens, size_t n) {
    const Model &m = *s.m;
    PrefillArgs a{};
    prefill_common(m, s.capacity, s.kv_bf16, a);
    a.layers = s.hlayers.data();
    a.rope = s.rope.as<float2>();
    a.kv.pool = s.kv.as<uint8_t>();
    a.kv.layer_bytes = s.kv_layer_bytes;
    a.kv.ptab = s.ptab.as<int>();
    a.kv.pps = (int)pages_per_seq(s.capacity);
    a.chunk = kPrefillChunk;
    if (!prefill_supported(a)) return QB_UNSUPPORTED;
    uint32_t st = prefill_workspace(m, kPrefillChunk, s.pf, a);
    if (st) return st;
    if (!s.tcm) {
        s.tcm.reset(new TcMaps());
        tc_prepare(m, a, *s.tcm);
    }
    a.tc = s.tcm.get();
    bool bad = false;
    cudaError_t e = prefill_kv(a, tokens, (int)n, (int)s.processed, s.stream, &bad);
    if (e != cudaSuccess) return session_fail(s, cuda_status(e));
    if (bad) return session_fail(s, QB_NONFINITE);
    s.processed += n;
    s.logits_valid = false;
    return QB_OK;
}

// evaluate_pending, src/generation.rs:258-274.
static uint32_t evaluate_pending(Generation &g, const volatile int32_t *cancel) {
    Session &s = *g.cache;
    // Without a cancel flag nothing can interrupt the evaluation between
    // tokens, so all pending tokens but the last go through the chunked path.
    if (!cancel && g.history.size() - s.processed >= 2) {
        DeviceGuard dg(s.device);
        const size_t n = g.history.size() - s.processed - 1;
        const uint32_t st = session_prefill_chunked(s, g.history.data() + s.processed, n);
        if (st != QB_OK && st != QB_UNSUPPORTED) return st;
        if (st == QB_OK) g.logits_ready = false;
    }
    while (s.processed < g.history.size()) {
        if (cancelled(cancel)) return QB_CANCELLED;
        uint32_t token = g.history[s.processed];
        g.logits_ready = false;
        uint32_t am = 0;
        uint32_t st = session_step(s, token, nullptr, 0, &am, true);
        if (st) return st;
        g.last_argmax = am;
        g.logits_ready = true;
    }
    if (cancelled(cancel)) return QB_CANCELLED;
    return QB_OK;
}

static void generation_reset(Generation &g) {
    if (g.sampler) g.sampler->rng.seed_from_u64(g.sampler->seed);
    g.cache->processed = 0;
    g.cache->valid = true;
    g.cache->logits_valid = false;
    g.history.clear();
    g.logits_ready = false;
    g.generated = 0;
    g.stop = QB_STOP_NONE;
}


// ------------------------------------------------------ tp communicator ----

// One rank's exchange buffer and its view of every rank's (CUDA IPC).
struct Comm {
    int device = 0, rank = 0, size = 1, rows = 0, h = 0;
    DevBuf buf;
    void *peer_base[kMaxTp] = {};  // opened IPC mappings (null for this rank)
    bool connected = false;
    TpPeers view{};
    unsigned seq = 0;  // exchange calls made (every rank makes the same ones)
    ~Comm() {
        DeviceGuard dg(device);
        for (int r = 0; r < kMaxTp; ++r)
            if (peer_base[r]) cudaIpcCloseMemHandle(peer_base[r]);
    }
};

static std::map<uint64_t, std::shared_ptr<Comm>> g_comms;

static std::shared_ptr<Comm> find_comm(uint64_t h) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_comms.find(h);
    return it == g_comms.end() ? nullptr : it->second;
}

// ----------------------------------------------------------- batch ----

// B independent sequences decoded in lockstep with the multi-token kernels
// (one row per sequence per step).  Each sequence has its own KV cache of
// `capacity` positions; all advance together.
struct Batch {
    std::shared_ptr<Model> m;
    int device = 0;
    size_t nseq = 0, capacity = 0, processed = 0;
    bool valid = true;
    int kv_bf16 = 0;
    cudaStream_t stream = nullptr;
    DevBuf kv, ptab, rope, ws, logits, amax, hist;
    std::vector<DecodeLayer> hlayers;
    TcMaps tcm;
    PrefillArgs a{};
    bool logits_valid = false;
    std::shared_ptr<Comm> comm;  // tensor-parallel batches
    ~Batch() {
        DeviceGuard dg(device);
        if (stream) cudaStreamDestroy(stream);
    }
};

static std::map<uint64_t, std::shared_ptr<Batch>> g_batches;

static std::shared_ptr<Batch> find_batch(uint64_t h) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_batches.find(h);
    return it == g_batches.end() ? nullptr : it->second;
}

static uint32_t batch_fail(Batch &b, uint32_t status) {
    b.valid = false;
    b.processed = 0;
    b.logits_valid = false;
    cudaStreamSynchronize(b.stream);
    return status;
}

// Runs n rows already in b.a.ids / pos / seq; checks the error word.
static uint32_t batch_forward(Batch &b, int n, int max_pos, bool lm_head) {
    cudaError_t e = forward_tokens(b.a, n, max_pos, lm_head, b.stream);
    if (e != cudaSuccess) return batch_fail(b, cuda_status(e));
    return QB_OK;
}

static uint32_t batch_check(Batch &b) {
    unsigned herr = 0;
    cudaError_t e = cudaMemcpyAsync(&herr, b.a.err, sizeof(unsigned), cudaMemcpyDeviceToHost, b.stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(b.stream);
    if (e != cudaSuccess) return batch_fail(b, cuda_status(e));
    if (herr) return batch_fail(b, (herr & ERR_TIMEOUT) ? QB_DEVICE_TIMEOUT : QB_NONFINITE);
    return QB_OK;
}

}  // namespace qb

using namespace qb;

extern "C" {

// ---------------------------------------------------------------- model ----

static uint32_t model_create(const qb_model_config *cfg, uint32_t linear_format, uint32_t table_format,
                             int device, int tp_rank, int tp_size, uint64_t *out) {
    clear_detail();
    if (!cfg || !out) return QB_INVALID_PARAMETERS;
    const qb_model_config c = *cfg;
    // Decoder::new admission, src/model.rs:191-230.
    if (!c.vocab_size || !c.layers || !c.hidden_dim || !c.query_heads || !c.kv_heads || !c.head_dim ||
        !c.ff_dim || !c.max_tokens)
        return QB_INVALID_CONFIG;
    if (c.head_dim % 2 || c.query_heads % c.kv_heads) return QB_INVALID_CONFIG;
    size_t qd;
    if (mul_ovf(c.query_heads, c.head_dim, &qd)) return QB_DIMENSION_OVERFLOW;
    if (qd != c.hidden_dim) return QB_INVALID_CONFIG;
    if (!isfinite(c.rope_base) || c.rope_base <= 0 || !isfinite(c.norm_epsilon) || c.norm_epsilon <= 0)
        return QB_INVALID_CONFIG;
    if (c.max_tokens > ((size_t)1 << 24)) return QB_INVALID_CONFIG;
    if (linear_format > QB_LINEAR_INT8_ROW || table_format > QB_TABLE_BF16) return QB_INVALID_PARAMETERS;
    if (c.vocab_size > 0x7fffffff || c.hidden_dim > 0xffffff || c.ff_dim > 0xffffff || c.head_dim > 512)
        return QB_UNSUPPORTED;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
        cudaGetLastError();
        return QB_CUDA_ERROR;
    }
    auto m = std::make_shared<Model>();
    m->c = c;
    if (!tp_split(c, tp_rank, tp_size, *m)) return QB_UNSUPPORTED;
    m->device = device;
    m->lin = linear_format;
    m->tab = table_format;
    m->sh = round16(c.hidden_dim * m->esz());
    m->shd = round16(c.head_dim * m->esz());
    m->sff = round16(m->nff * m->esz());
    m->semb = round16(c.hidden_dim * m->tesz());
    m->layers.resize(c.layers);
    DeviceGuard dg(device);
    const size_t h = c.hidden_dim, kv = m->kv(), ff = m->nff, rq = m->qd() + 2 * kv;
    uint32_t s;
    for (auto &L : m->layers) {
        if ((s = L.wqkv.alloc(rq * m->sh)) || (s = L.sqkv.alloc(rq * 4)) || (s = L.bqkv.alloc(rq * 4)) ||
            (s = L.wo.alloc(m->nq * h * m->shd)) || (s = L.so.alloc(h * 4)) ||
            (s = L.wgu.alloc(2 * ff * m->sh)) || (s = L.sgu.alloc(2 * ff * 4)) ||
            (s = L.down.w.alloc(h * m->sff)) || (s = L.down.scales.alloc(h * 4)) ||
            (s = L.attn_norm.alloc(h * 4)) || (s = L.ffn_norm.alloc(h * 4)))
            return s == QB_CUDA_ERROR ? QB_ALLOCATION : s;
    }
    if ((s = m->emb.alloc(c.vocab_size * m->semb)) || (s = m->final_norm.alloc(h * 4)))
        return s == QB_CUDA_ERROR ? QB_ALLOCATION : s;
    std::lock_guard<std::mutex> lk(g_mu);
    uint64_t id = g_next++;
    g_models[id] = m;
    *out = id;
    return QB_OK;
}

uint32_t qb_model_create(const qb_model_config *cfg, uint32_t linear_format, uint32_t table_format,
                         int device, uint64_t *out) {
    return model_create(cfg, linear_format, table_format, device, 0, 1, out);
}

uint32_t qb_model_create_tp(const qb_model_config *cfg, uint32_t linear_format, uint32_t table_format,
                            int device, int tp_rank, int tp_size, uint64_t *out) {
    return model_create(cfg, linear_format, table_format, device, tp_rank, tp_size, out);
}

uint32_t qb_tp_shard_of(const qb_model_config *cfg, int tp_rank, int tp_size, qb_tp_shard *out) {
    if (!cfg || !out) return QB_INVALID_PARAMETERS;
    if (!cfg->query_heads || !cfg->kv_heads || cfg->query_heads % cfg->kv_heads || !cfg->vocab_size)
        return QB_INVALID_CONFIG;
    Model m;
    if (!tp_split(*cfg, tp_rank, tp_size, m)) return QB_UNSUPPORTED;
    out->rank = m.tp_rank; out->size = m.tp_size;
    out->head0 = m.head0; out->heads = m.nq; out->kv_head0 = m.kv0; out->kv_heads = m.nkv;
    out->ff0 = m.f0; out->ff = m.nff; out->vocab0 = m.v0; out->vocab = m.nv;
    return QB_OK;
}

uint32_t qb_model_tp_info(uint64_t model, qb_tp_shard *out) {
    auto m = find_model(model);
    if (!m) return QB_INVALID_HANDLE;
    if (!out) return QB_INVALID_PARAMETERS;
    out->rank = m->tp_rank; out->size = m->tp_size;
    out->head0 = m->head0; out->heads = m->nq; out->kv_head0 = m->kv0; out->kv_heads = m->nkv;
    out->ff0 = m->f0; out->ff = m->nff; out->vocab0 = m->v0; out->vocab = m->nv;
    return QB_OK;
}

uint32_t qb_model_set_tensor(uint64_t model, int64_t layer, uint32_t tensor, uint32_t dtype,
                             const void *data, size_t n) {
    clear_detail();
    auto m = find_model(model);
    if (!m) return QB_INVALID_HANDLE;
    if (m->finalized) return QB_INVALID_STATE;
    if (!data || (dtype != QB_HOST_F32 && dtype != QB_HOST_BF16)) return QB_INVALID_PARAMETERS;
    const qb_model_config &c = m->c;
    // Full tensors are passed (every rank of a sharded model reads the same
    // ones); each stores its shard: kvf / ff / V are the full sizes, qd / kv
    // / nff / nv the shard's.
    const size_t h = c.hidden_dim, hd = c.head_dim, kvf = c.kv_heads * hd, ff = c.ff_dim, V = c.vocab_size;
    const size_t qd = m->qd(), kv = m->kv(), q0 = m->head0 * hd, k0 = m->kv0 * hd;
    DeviceGuard dg(m->device);
    size_t expected = 0;
    bool global = tensor <= QB_T_FINAL_NORM;
    if (global != (layer < 0)) return QB_INVALID_PARAMETERS;
    if (!global && (size_t)layer >= c.layers) return QB_INVALID_LAYER_COUNT;
    switch (tensor) {
    case QB_T_EMBEDDING: case QB_T_LM_HEAD: expected = V * h; break;
    case QB_T_FINAL_NORM: case QB_T_ATTN_NORM: case QB_T_FFN_NORM: case QB_T_Q_BIAS: expected = h; break;
    case QB_T_K_BIAS: case QB_T_V_BIAS: expected = kvf; break;
    case QB_T_Q: case QB_T_O: expected = h * h; break;
    case QB_T_K: case QB_T_V: expected = kvf * h; break;
    case QB_T_GATE: case QB_T_UP: case QB_T_DOWN: expected = ff * h; break;
    default: return QB_INVALID_PARAMETERS;
    }
    if (n != expected) {
        set_detail(tensor, expected, n);
        return QB_INVALID_LENGTH;
    }
    uint32_t s;
    std::vector<float> hv;
    if (tensor == QB_T_FINAL_NORM || tensor == QB_T_ATTN_NORM || tensor == QB_T_FFN_NORM ||
        tensor == QB_T_Q_BIAS || tensor == QB_T_K_BIAS || tensor == QB_T_V_BIAS) {
        if ((s = host_vector_finite(data, n, dtype, hv))) return s;
        float *dst = nullptr;
        size_t from = 0, cnt = n;  // the shard's part of a bias
        if (tensor == QB_T_FINAL_NORM) { dst = m->final_norm.as<float>(); m->fn_set = true; }
        else {
            LayerStore &L = m->layers[layer];
            if (tensor == QB_T_ATTN_NORM) { dst = L.attn_norm.as<float>(); L.an = true; }
            else if (tensor == QB_T_FFN_NORM) { dst = L.ffn_norm.as<float>(); L.fn = true; }
            else if (tensor == QB_T_Q_BIAS) { dst = L.bqkv.as<float>(); from = q0; cnt = qd; }
            else if (tensor == QB_T_K_BIAS) { dst = L.bqkv.as<float>() + qd; from = k0; cnt = kv; }
            else { dst = L.bqkv.as<float>() + qd + kv; from = k0; cnt = kv; }
        }
        QB_CUDA(cudaMemcpy(dst, hv.data() + from, cnt * 4, cudaMemcpyHostToDevice));
        return QB_OK;
    }
    DevBuf src;
    if ((s = upload_f32(data, n, dtype, src))) return s;
    if (tensor == QB_T_EMBEDDING || tensor == QB_T_LM_HEAD) {
        size_t idx;
        if ((s = check_finite_dev(src.as<float>(), n, &idx))) { set_detail(tensor, 0, 0, idx); return s; }
        DevBuf *dst = tensor == QB_T_EMBEDDING ? &m->emb : &m->head;
        // The embedding is whole; an untied head keeps the shard's rows.
        const size_t r0 = tensor == QB_T_LM_HEAD ? m->v0 : 0, nr = tensor == QB_T_LM_HEAD ? m->nv : V;
        if (tensor == QB_T_LM_HEAD && (s = m->head.alloc(nr * m->semb))) return s;
        relayout_kernel<<<gridn(nr * h), 256>>>(src.as<float>() + r0 * h, nullptr, nr, h, 0, h, dst->as<uint8_t>(),
                                                m->semb, m->tab == QB_TABLE_BF16 ? WF_BF16 : WF_F32);
        QB_CUDA(cudaGetLastError());
        QB_CUDA(cudaDeviceSynchronize());
        if (tensor == QB_T_EMBEDDING) m->emb_set = true; else m->head_set = true;
        return QB_OK;
    }
    LayerStore &L = m->layers[layer];
    switch (tensor) {
    case QB_T_Q:
        s = store_linear(*m, src.as<float>() + q0 * h, qd, h, L.wqkv.as<uint8_t>(), m->sh, L.sqkv.as<float>(), 1);
        if (!s) L.q = true;
        break;
    case QB_T_K:
        s = store_linear(*m, src.as<float>() + k0 * h, kv, h, L.wqkv.as<uint8_t>() + qd * m->sh, m->sh,
                         L.sqkv.as<float>() + qd, 1);
        if (!s) L.k = true;
        break;
    case QB_T_V:
        s = store_linear(*m, src.as<float>() + k0 * h, kv, h, L.wqkv.as<uint8_t>() + (qd + kv) * m->sh, m->sh,
                         L.sqkv.as<float>() + qd + kv, 1);
        if (!s) L.v = true;
        break;
    case QB_T_O:
        s = store_o_proj(*m, L, src.as<float>());
        if (!s) L.o = true;
        break;
    case QB_T_GATE:
        s = store_linear(*m, src.as<float>() + m->f0 * h, m->nff, h, L.wgu.as<uint8_t>(), 2 * m->sh,
                         L.sgu.as<float>(), 2);
        if (!s) L.gate = true;
        break;
    case QB_T_UP:
        s = store_linear(*m, src.as<float>() + m->f0 * h, m->nff, h, L.wgu.as<uint8_t>() + m->sh, 2 * m->sh,
                         L.sgu.as<float>() + 1, 2);
        if (!s) L.up = true;
        break;
    case QB_T_DOWN:
        s = store_linear_cols(*m, src.as<float>(), h, ff, m->f0, m->nff, L.down.w.as<uint8_t>(), m->sff,
                              L.down.scales.as<float>());
        if (!s) L.down.set = true;
        break;
    }
    if (s == QB_NONFINITE) set_detail(tensor, 0, 0, 0);
    return s;
}

uint32_t qb_model_finalize(uint64_t model) {
    clear_detail();
    auto m = find_model(model);
    if (!m) return QB_INVALID_HANDLE;
    if (m->finalized) return QB_OK;
    if (!m->emb_set || !m->fn_set) return QB_INVALID_STATE;
    for (auto &L : m->layers)
        if (!(L.q && L.k && L.v && L.o && L.an && L.fn && L.gate && L.up && L.down.set))
            return QB_INVALID_STATE;
    DeviceGuard dg(m->device);
    const bool i8 = m->wf() == WF_I8;
    std::vector<DecodeLayer> dl(m->c.layers);
    for (size_t l = 0; l < m->c.layers; ++l) {
        LayerStore &L = m->layers[l];
        DecodeLayer &d = dl[l];
        d.wqkv = L.wqkv.as<uint8_t>(); d.sqkv = i8 ? L.sqkv.as<float>() : nullptr; d.bqkv = L.bqkv.as<float>();
        d.wo = L.wo.as<uint8_t>(); d.so = i8 ? L.so.as<float>() : nullptr;
        d.wgu = L.wgu.as<uint8_t>(); d.sgu = i8 ? L.sgu.as<float>() : nullptr;
        d.wd = L.down.w.as<uint8_t>(); d.sd = i8 ? L.down.scales.as<float>() : nullptr;
        d.attn_norm = L.attn_norm.as<float>(); d.ffn_norm = L.ffn_norm.as<float>();
        d.kc = d.vc = nullptr;
    }
    uint32_t s;
    if ((s = m->dlayers.alloc(dl.size() * sizeof(DecodeLayer), false))) return s;
    QB_CUDA(cudaMemcpy(m->dlayers.p, dl.data(), dl.size() * sizeof(DecodeLayer), cudaMemcpyHostToDevice));
    // Logical payload: matrices at their stored width (FP32 4 B, BF16 2 B,
    // INT8 1 B + 4 B per row scale), plus FP32 norms and biases; the tied
    // table counts once (src/model.rs:347-385).
    const qb_model_config &c = m->c;
    // (the whole model's payload, also for a shard)
    const size_t h = c.hidden_dim, kv = c.kv_heads * c.head_dim, ff = c.ff_dim;
    size_t mats = h * h * 2 + kv * h * 2 + ff * h * 3;
    size_t rows = h + 2 * kv + h + 2 * ff + h;
    size_t per = i8 ? mats + rows * 4 : mats * m->esz();
    per += 2 * h * 4 + (h + 2 * kv) * 4;
    size_t table = c.vocab_size * h * m->tesz();
    m->logical_bytes = table * (m->head_set ? 2 : 1) + h * 4 + per * c.layers;
    m->finalized = true;
    return QB_OK;
}

uint32_t qb_model_logical_weight_bytes(uint64_t model, size_t *out) {
    auto m = find_model(model);
    if (!m) return QB_INVALID_HANDLE;
    if (!m->finalized) return QB_INVALID_STATE;
    *out = m->logical_bytes;
    return QB_OK;
}

uint32_t qb_model_read_int8(uint64_t model, int64_t layer, uint32_t tensor, int8_t *values, size_t vl,
                            float *scales, size_t sl) {
    clear_detail();
    auto m = find_model(model);
    if (!m) return QB_INVALID_HANDLE;
    if (m->wf() != WF_I8) return QB_UNSUPPORTED;
    if (layer < 0 || (size_t)layer >= m->c.layers) return QB_INVALID_LAYER_COUNT;
    const size_t h = m->c.hidden_dim, kv = m->kv(), ff = m->c.ff_dim;
    LayerStore &L = m->layers[layer];
    const uint8_t *src = nullptr;
    const float *sc = nullptr;
    size_t rows = 0, cols = h, stride = m->sh, sstride = 1;
    switch (tensor) {
    case QB_T_Q: src = L.wqkv.as<uint8_t>(); sc = L.sqkv.as<float>(); rows = h; break;
    case QB_T_K: src = L.wqkv.as<uint8_t>() + h * m->sh; sc = L.sqkv.as<float>() + h; rows = kv; break;
    case QB_T_V: src = L.wqkv.as<uint8_t>() + (h + kv) * m->sh; sc = L.sqkv.as<float>() + h + kv; rows = kv; break;
    case QB_T_GATE: src = L.wgu.as<uint8_t>(); sc = L.sgu.as<float>(); rows = ff; stride = 2 * m->sh; sstride = 2; break;
    case QB_T_UP:
        src = L.wgu.as<uint8_t>() + m->sh; sc = L.sgu.as<float>() + 1; rows = ff; stride = 2 * m->sh; sstride = 2;
        break;
    case QB_T_DOWN: src = L.down.w.as<uint8_t>(); sc = L.down.scales.as<float>(); rows = h; cols = ff; stride = m->sff; break;
    case QB_T_O: rows = h; sc = L.so.as<float>(); break;
    default: return QB_INVALID_PARAMETERS;
    }
    if (vl != rows * cols) { set_detail(0, rows * cols, vl); return QB_INVALID_LENGTH; }
    if (sl != rows) { set_detail(1, rows, sl); return QB_INVALID_LENGTH; }
    DeviceGuard dg(m->device);
    DevBuf tmp;
    uint32_t s;
    if ((s = tmp.alloc(rows * cols, false))) return s;
    if (tensor == QB_T_O) {
        const size_t hd = m->c.head_dim;
        std::vector<int8_t> blk(h * hd), out(h * h);
        DevBuf b1;
        if ((s = b1.alloc(h * hd, false))) return s;
        for (size_t hh = 0; hh < m->c.query_heads; ++hh) {
            unbias_kernel<<<gridn(h * hd), 256>>>(L.wo.as<uint8_t>() + hh * h * m->shd, h, hd, m->shd, b1.as<int8_t>());
            QB_CUDA(cudaMemcpy(blk.data(), b1.p, h * hd, cudaMemcpyDeviceToHost));
            for (size_t r = 0; r < h; ++r) memcpy(&out[r * h + hh * hd], &blk[r * hd], hd);
        }
        memcpy(values, out.data(), h * h);
    } else {
        unbias_kernel<<<gridn(rows * cols), 256>>>(src, rows, cols, stride, tmp.as<int8_t>());
        QB_CUDA(cudaGetLastError());
        QB_CUDA(cudaMemcpy(values, tmp.p, rows * cols, cudaMemcpyDeviceToHost));
    }
    QB_CUDA(cudaMemcpy2D(scales, 4, sc, sstride * 4, 4, rows, cudaMemcpyDeviceToHost));
    return QB_OK;
}

uint32_t qb_model_free(uint64_t model) {
    std::shared_ptr<Model> m;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto it = g_models.find(model);
        if (it == g_models.end()) return QB_INVALID_HANDLE;
        m = it->second;
        g_models.erase(it);
    }
    DeviceGuard dg(m->device);
    m.reset();  // sessions hold their own reference
    return QB_OK;
}

// -------------------------------------------------------------- session ----

static uint32_t session_create(uint64_t model, size_t capacity, uint32_t kv_dtype, size_t budget,
                               std::shared_ptr<Session> &out) {
    auto m = find_model(model);
    if (!m) return QB_INVALID_HANDLE;
    if (!m->finalized) return QB_INVALID_STATE;
    if (m->tp_size > 1) return QB_UNSUPPORTED;  // shards decode through qb_batch_create_tp
    const qb_model_config &c = m->c;
    if (capacity == 0 || capacity > c.max_tokens) return QB_INVALID_CAPACITY;
    if (kv_dtype > QB_KV_BF16) return QB_INVALID_PARAMETERS;
    size_t per, logical;
    if (mul_ovf(c.kv_heads, capacity, &per) || mul_ovf(per, c.head_dim, &per) || mul_ovf(per, 2, &logical) ||
        mul_ovf(logical, c.layers, &logical) || mul_ovf(logical, 4, &logical))
        return QB_DIMENSION_OVERFLOW;
    size_t ws = ref_workspace_bytes(c, capacity);
    if (budget && (logical > SIZE_MAX - ws || logical + ws > budget)) return QB_RESOURCE_BUDGET;
    auto s = std::make_shared<Session>();
    s->m = m;
    s->device = m->device;
    s->capacity = capacity;
    s->kv_bf16 = kv_dtype == QB_KV_BF16;
    DeviceGuard dg(m->device);
    uint32_t st = session_build(*s);
    if (st) return st == QB_CUDA_ERROR ? QB_ALLOCATION : st;
    out = s;
    return QB_OK;
}

uint32_t qb_session_create(uint64_t model, size_t capacity, uint32_t kv_dtype, size_t budget, uint64_t *out) {
    clear_detail();
    if (!out) return QB_INVALID_PARAMETERS;
    std::shared_ptr<Session> s;
    uint32_t st = session_create(model, capacity, kv_dtype, budget, s);
    if (st) return st;
    std::lock_guard<std::mutex> lk(g_mu);
    uint64_t id = g_next++;
    g_sessions[id] = s;
    *out = id;
    return QB_OK;
}

uint32_t qb_session_step(uint64_t session, uint32_t token, float *logits, size_t logits_len, uint32_t *argmax) {
    clear_detail();
    auto s = find_session(session);
    if (!s) return QB_INVALID_HANDLE;
    return session_step(*s, token, logits, logits_len, argmax, false);
}

uint32_t qb_session_append(uint64_t session, const uint32_t *tokens, size_t n, float *logits,
                           size_t logits_len, uint32_t *argmax, int32_t require_empty) {
    clear_detail();
    auto s = find_session(session);
    if (!s) return QB_INVALID_HANDLE;
    Session &S = *s;
    // append_into admission, src/kv_cache.rs:255-279.
    if (!S.valid) return QB_INVALID_STATE;
    if (require_empty && S.processed != 0) return QB_NOT_EMPTY;
    if (n == 0 || !tokens) return QB_EMPTY_INPUT;
    if (logits && logits_len != S.m->c.vocab_size) return QB_INVALID_OUTPUT_LENGTH;
    for (size_t i = 0; i < n; ++i)
        if (tokens[i] >= S.m->c.vocab_size) return QB_INVALID_TOKEN;
    if (S.processed + n > S.capacity) return QB_FULL;
    size_t i0 = 0;
    if (n >= 2) {
        DeviceGuard dg(S.device);
        const uint32_t st = session_prefill_chunked(S, tokens, n - 1);
        if (st == QB_OK) i0 = n - 1;
        else if (st != QB_UNSUPPORTED) return st;
    }
    for (size_t i = i0; i < n; ++i) {
        bool last = i + 1 == n;
        uint32_t st = session_step(S, tokens[i], last ? logits : nullptr, logits_len, last ? argmax : nullptr, last);
        if (st) return st;
    }
    return QB_OK;
}

uint32_t qb_session_step_profiled(uint64_t session, uint32_t token, float *logits, size_t logits_len,
                                  uint32_t *argmax, uint64_t *stamps, size_t stamps_len, size_t *needed) {
    clear_detail();
    auto sp = find_session(session);
    if (!sp) return QB_INVALID_HANDLE;
    Session &s = *sp;
    const size_t nb = 4 * s.m->c.layers;
    const size_t need = 2 * nb * (size_t)s.grid + 2;
    if (needed) *needed = need;
    if (!stamps || stamps_len < need) {
        set_detail(5, need, stamps_len);
        return QB_INVALID_LENGTH;
    }
    if (!s.valid) return QB_INVALID_STATE;
    if (logits && logits_len != s.m->c.vocab_size) return QB_INVALID_OUTPUT_LENGTH;
    if (token >= s.m->c.vocab_size) return QB_INVALID_TOKEN;
    if (s.processed == s.capacity) return QB_FULL;
    DeviceGuard dg(s.device);
    DevBuf tr;
    uint32_t st = tr.alloc(need * 8);
    if (st) return st;
    DecodeParams p = s.params;
    p.trace = tr.as<unsigned long long>();
    s.hctrl->token = (int)token;
    s.hctrl->pos = (int)s.processed;
    s.hctrl->write_logits = 1;
    cudaError_t e = cudaMemcpyAsync(s.ctrl.p, s.hctrl, 16, cudaMemcpyHostToDevice, s.stream);
    if (e == cudaSuccess) e = decode_launch(p, s.grid, s.stream, split_at(s, s.processed));
    if (e == cudaSuccess)
        e = cudaMemcpyAsync((char *)s.hctrl + 16, (char *)s.ctrl.p + 16, 8, cudaMemcpyDeviceToHost, s.stream);
    if (e != cudaSuccess) return session_fail(s, cuda_status(e));
    st = session_finish(s, logits, argmax);
    if (st) return st;
    s.logits_valid = true;
    QB_CUDA(cudaMemcpy(stamps, tr.p, need * 8, cudaMemcpyDeviceToHost));
    return QB_OK;
}

uint32_t qb_session_step_withheld(uint64_t session, uint32_t token, uint64_t timeout_ns) {
    clear_detail();
    auto sp = find_session(session);
    if (!sp) return QB_INVALID_HANDLE;
    Session &s = *sp;
    if (!s.valid) return QB_INVALID_STATE;
    if (token >= s.m->c.vocab_size) return QB_INVALID_TOKEN;
    if (s.processed == s.capacity) return QB_FULL;
    if (timeout_ns == 0 || timeout_ns > 2000000000ull) {
        set_detail(0, 2000000000ull, (size_t)timeout_ns);
        return QB_INVALID_PARAMETERS;
    }
    DeviceGuard dg(s.device);
    DecodeParams p = s.params;
    p.withhold = 1;
    p.timeout_ns = timeout_ns;
    s.hctrl->token = (int)token;
    s.hctrl->pos = (int)s.processed;
    s.hctrl->write_logits = 0;
    cudaError_t e = cudaMemcpyAsync(s.ctrl.p, s.hctrl, 16, cudaMemcpyHostToDevice, s.stream);
    if (e == cudaSuccess) e = decode_launch(p, s.grid, s.stream, split_at(s, s.processed));
    if (e == cudaSuccess)
        e = cudaMemcpyAsync((char *)s.hctrl + 16, (char *)s.ctrl.p + 16, 8, cudaMemcpyDeviceToHost, s.stream);
    if (e != cudaSuccess) return session_fail(s, cuda_status(e));
    return session_finish(s, nullptr, nullptr);
}

uint32_t qb_session_reset(uint64_t session) {
    auto s = find_session(session);
    if (!s) return QB_INVALID_HANDLE;
    s->processed = 0;
    s->valid = true;
    s->logits_valid = false;
    return QB_OK;
}

uint32_t qb_session_info_get(uint64_t session, qb_session_info *out) {
    auto s = find_session(session);
    if (!s) return QB_INVALID_HANDLE;
    if (!out) return QB_INVALID_PARAMETERS;
    out->processed = s->processed;
    out->capacity = s->capacity;
    out->logical_bytes = s->logical_bytes;
    out->workspace_bytes = s->workspace_bytes;
    out->valid = s->valid ? 1 : 0;
    return QB_OK;
}

uint32_t qb_session_decode_greedy(uint64_t session, uint32_t token, size_t steps, uint32_t *ids) {
    clear_detail();
    auto sp = find_session(session);
    if (!sp) return QB_INVALID_HANDLE;
    Session &s = *sp;
    if (!s.valid) return QB_INVALID_STATE;
    if (steps == 0 || !ids) return QB_EMPTY_INPUT;
    if (token >= s.m->c.vocab_size) return QB_INVALID_TOKEN;
    if (s.processed + steps > s.capacity) return QB_FULL;
    DeviceGuard dg(s.device);
    const size_t start = s.processed;
    // The first launch takes the host token; each step then feeds its own
    // argmax to the next through the device control block.
    s.hctrl->token = (int)token;
    s.hctrl->pos = (int)start;
    s.hctrl->write_logits = 0;
    cudaError_t e = cudaMemcpyAsync(s.ctrl.p, s.hctrl, 16, cudaMemcpyHostToDevice, s.stream);
    for (size_t i = 0; i < steps && e == cudaSuccess; ++i)
        e = decode_launch(s.params, s.grid, s.stream, split_at(s, start + i));
    if (e == cudaSuccess)
        e = cudaMemcpyAsync((char *)s.hctrl + 16, (char *)s.ctrl.p + 16, 8, cudaMemcpyDeviceToHost, s.stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s.stream);
    if (e != cudaSuccess) return session_fail(s, cuda_status(e));
    if (s.hctrl->error) return session_fail(s, (s.hctrl->error & ERR_TIMEOUT) ? QB_DEVICE_TIMEOUT : QB_NONFINITE);
    std::vector<int> out(steps);
    e = cudaMemcpy(out.data(), s.emitted.as<int>() + start, steps * 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return session_fail(s, cuda_status(e));
    for (size_t i = 0; i < steps; ++i) ids[i] = (uint32_t)out[i];
    s.processed += steps;
    s.logits_valid = false;
    return QB_OK;
}

uint32_t qb_session_stream(uint64_t session, void **stream) {
    auto s = find_session(session);
    if (!s) return QB_INVALID_HANDLE;
    *stream = (void *)s->stream;
    return QB_OK;
}

uint32_t qb_session_free(uint64_t session) {
    std::shared_ptr<Session> s;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto it = g_sessions.find(session);
        if (it == g_sessions.end()) return QB_INVALID_HANDLE;
        s = it->second;
        g_sessions.erase(it);
    }
    return QB_OK;
}

// ----------------------------------------------------------- generation ----

static uint32_t generation_create(uint64_t model, size_t capacity, const qb_sampling *policy, const uint32_t *stops,
                                  size_t nstops, size_t max_new, uint32_t kv_dtype, size_t budget, uint64_t *out) {
    clear_detail();
    if (!out) return QB_INVALID_PARAMETERS;
    auto m = find_model(model);
    if (!m) return QB_INVALID_HANDLE;
    // GenerationSession::new, src/generation.rs:111-138.
    if (max_new == 0 || max_new >= capacity) return QB_INVALID_PARAMETERS;
    for (size_t i = 0; i < nstops; ++i)
        if (stops[i] >= m->c.vocab_size) return QB_INVALID_PARAMETERS;
    std::unique_ptr<Sampler> sampler;
    if (policy && policy->kind != QB_SAMPLING_GREEDY) {
        sampler.reset(new Sampler());
        uint32_t st = sampler_init(policy, m->device, *sampler);
        if (st) return st;
        if (!sampler_vocab_ok(*sampler, m->c.vocab_size)) return QB_INVALID_PARAMETERS;
    }
    std::shared_ptr<Session> s;
    uint32_t st = session_create(model, capacity, kv_dtype, budget, s);
    if (st) return st;
    auto g = std::make_shared<Generation>();
    g->cache = s;
    g->sampler = std::move(sampler);
    g->stops.assign(stops, stops + nstops);
    g->max_new = max_new;
    g->vocab = (uint32_t)m->c.vocab_size;
    g->history.reserve(capacity);
    std::lock_guard<std::mutex> lk(g_mu);
    uint64_t id = g_next++;
    g_generations[id] = g;
    *out = id;
    return QB_OK;
}

uint32_t qb_generation_create(uint64_t model, size_t capacity, const uint32_t *stops, size_t nstops,
                              size_t max_new, uint32_t kv_dtype, size_t budget, uint64_t *out) {
    return generation_create(model, capacity, nullptr, stops, nstops, max_new, kv_dtype, budget, out);
}

uint32_t qb_generation_create_sampled(uint64_t model, size_t capacity, const qb_sampling *policy,
                                      const uint32_t *stops, size_t nstops, size_t max_new, uint32_t kv_dtype,
                                      size_t budget, uint64_t *out) {
    return generation_create(model, capacity, policy, stops, nstops, max_new, kv_dtype, budget, out);
}

uint32_t qb_generation_start(uint64_t gen, const uint32_t *prompt, size_t n, const volatile int32_t *cancel) {
    clear_detail();
    auto gp = find_generation(gen);
    if (!gp) return QB_INVALID_HANDLE;
    Generation &g = *gp;
    // start_with_cancel, src/generation.rs:145-170.
    if (!g.history.empty()) return QB_ALREADY_STARTED;
    if (n == 0 || !prompt) return QB_INVALID_PARAMETERS;
    for (size_t i = 0; i < n; ++i)
        if (prompt[i] >= g.vocab) return QB_INVALID_PARAMETERS;
    if (n > SIZE_MAX - g.max_new || n + g.max_new > g.cache->capacity) return QB_INVALID_PARAMETERS;
    if (cancelled(cancel)) return QB_CANCELLED;
    if (!g.cache->valid) return QB_INVALID_STATE;
    g.history.insert(g.history.end(), prompt, prompt + n);
    return evaluate_pending(g, cancel);
}

uint32_t qb_generation_next_token(uint64_t gen, const volatile int32_t *cancel, uint32_t *token, int32_t *has) {
    clear_detail();
    auto gp = find_generation(gen);
    if (!gp) return QB_INVALID_HANDLE;
    Generation &g = *gp;
    if (has) *has = 0;
    // next_token, src/generation.rs:307-337.
    if (cancelled(cancel)) return QB_CANCELLED;
    if (!g.cache->valid) return QB_INVALID_STATE;
    if (g.history.empty()) return QB_NOT_STARTED;
    if (g.stop != QB_STOP_NONE) return QB_OK;
    uint32_t st = evaluate_pending(g, cancel);
    if (st) return st;
    if (!g.logits_ready) return QB_NOT_STARTED;
    uint32_t next = g.last_argmax;
    if (g.sampler) {
        // The temperature policy samples the last token's logits, still on
        // the device (the decode step kept them).
        Session &s = *g.cache;
        DeviceGuard dg(s.device);
        st = sampler_run(*g.sampler, s.logits.as<float>(), s.m->c.vocab_size, s.stream, &next);
        if (st) return st;
    }
    g.history.push_back(next);
    g.generated += 1;
    g.logits_ready = false;
    if (std::find(g.stops.begin(), g.stops.end(), next) != g.stops.end()) g.stop = QB_STOP_TOKEN;
    else if (g.generated == g.max_new) g.stop = QB_STOP_OUTPUT_LIMIT;
    if (token) *token = next;
    if (has) *has = 1;
    return QB_OK;
}

uint32_t qb_generation_append_context(uint64_t gen, const uint32_t *suffix, size_t n, size_t max_new,
                                      const volatile int32_t *cancel) {
    clear_detail();
    auto gp = find_generation(gen);
    if (!gp) return QB_INVALID_HANDLE;
    Generation &g = *gp;
    const size_t cap = g.cache->capacity;
    // admit_context, src/generation.rs:183-218.
    bool bad = g.history.empty() || g.stop == QB_STOP_NONE || n == 0 || !suffix || max_new == 0 || max_new >= cap;
    if (!bad)
        for (size_t i = 0; i < n; ++i)
            if (suffix[i] >= g.vocab) bad = true;
    if (!bad && (g.history.size() > SIZE_MAX - n || g.history.size() + n > SIZE_MAX - max_new ||
                 g.history.size() + n + max_new > cap))
        bad = true;
    if (bad) return QB_INVALID_PARAMETERS;
    if (!g.cache->valid) return QB_INVALID_STATE;
    if (cancelled(cancel)) return QB_CANCELLED;
    g.history.insert(g.history.end(), suffix, suffix + n);
    g.max_new = max_new;
    g.generated = 0;
    g.stop = QB_STOP_NONE;
    return evaluate_pending(g, cancel);
}

uint32_t qb_generation_replay_history(uint64_t gen, const uint32_t *hist, size_t n, size_t max_new,
                                      const volatile int32_t *cancel) {
    clear_detail();
    auto gp = find_generation(gen);
    if (!gp) return QB_INVALID_HANDLE;
    Generation &g = *gp;
    const size_t cap = g.cache->capacity;
    // admit_replay, src/generation.rs:228-257.
    bool bad = n == 0 || !hist || max_new == 0 || max_new >= cap;
    if (!bad)
        for (size_t i = 0; i < n; ++i)
            if (hist[i] >= g.vocab) bad = true;
    if (!bad && (n > SIZE_MAX - max_new || n + max_new > cap)) bad = true;
    if (bad) return QB_INVALID_PARAMETERS;
    if (cancelled(cancel)) return QB_CANCELLED;
    std::vector<uint32_t> copy(hist, hist + n);  // `hist` may alias our history
    generation_reset(g);
    g.max_new = max_new;
    g.history = copy;
    return evaluate_pending(g, cancel);
}

uint32_t qb_generation_reset(uint64_t gen) {
    auto gp = find_generation(gen);
    if (!gp) return QB_INVALID_HANDLE;
    generation_reset(*gp);
    return QB_OK;
}

uint32_t qb_generation_info_get(uint64_t gen, qb_generation_info *out) {
    auto gp = find_generation(gen);
    if (!gp) return QB_INVALID_HANDLE;
    if (!out) return QB_INVALID_PARAMETERS;
    out->processed = gp->cache->processed;
    out->history_len = gp->history.size();
    out->generated = gp->generated;
    out->max_new = gp->max_new;
    out->stop_reason = gp->stop;
    out->valid = gp->cache->valid ? 1 : 0;
    out->logits_ready = gp->logits_ready ? 1 : 0;
    return QB_OK;
}

uint32_t qb_generation_history(uint64_t gen, uint32_t *ids, size_t cap, size_t *len) {
    auto gp = find_generation(gen);
    if (!gp) return QB_INVALID_HANDLE;
    size_t n = gp->history.size();
    if (len) *len = n;
    if (ids) memcpy(ids, gp->history.data(), std::min(n, cap) * 4);
    return QB_OK;
}

uint32_t qb_generation_prefix_logits(uint64_t gen, float *logits, size_t n) {
    clear_detail();
    auto gp = find_generation(gen);
    if (!gp) return QB_INVALID_HANDLE;
    Session &s = *gp->cache;
    // prefix_logits, src/generation.rs:281-283: valid cache and processed > 0.
    if (!s.valid || s.processed == 0 || !s.logits_valid) return QB_NOT_STARTED;
    if (n != s.m->c.vocab_size) return QB_INVALID_OUTPUT_LENGTH;
    DeviceGuard dg(s.device);
    QB_CUDA(cudaMemcpy(logits, s.logits.p, n * 4, cudaMemcpyDeviceToHost));
    return QB_OK;
}

uint32_t qb_generation_free(uint64_t gen) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_generations.find(gen);
    if (it == g_generations.end()) return QB_INVALID_HANDLE;
    g_generations.erase(it);
    return QB_OK;
}


// -------------------------------------------------------- sampler ABI ----

static std::shared_ptr<Sampler> find_sampler(uint64_t h) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_samplers.find(h);
    return it == g_samplers.end() ? nullptr : it->second;
}

uint32_t qb_sampler_create(const qb_sampling *policy, int device, uint64_t *out) {
    clear_detail();
    if (!policy || !out || !policy_ok(policy)) return QB_INVALID_PARAMETERS;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) return QB_INVALID_PARAMETERS;
    auto sp = std::make_shared<Sampler>();
    uint32_t st = sampler_init(policy, device, *sp);
    if (st) return st;
    DeviceGuard dg(device);
    QB_CUDA(cudaStreamCreateWithFlags(&sp->stream, cudaStreamNonBlocking));
    std::lock_guard<std::mutex> lk(g_mu);
    uint64_t id = g_next++;
    g_samplers[id] = sp;
    *out = id;
    return QB_OK;
}

uint32_t qb_sampler_validate_vocab(uint64_t h, size_t vocab) {
    auto sp = find_sampler(h);
    if (!sp) return QB_INVALID_HANDLE;
    return sampler_vocab_ok(*sp, vocab) ? QB_OK : QB_INVALID_PARAMETERS;
}

uint32_t qb_sampler_reset(uint64_t h) {
    auto sp = find_sampler(h);
    if (!sp) return QB_INVALID_HANDLE;
    std::lock_guard<std::mutex> lk(sp->mu);
    sp->rng.seed_from_u64(sp->seed);
    return QB_OK;
}

uint32_t qb_sampler_sample(uint64_t h, const float *logits, size_t n, uint32_t *out) {
    clear_detail();
    auto sp = find_sampler(h);
    if (!sp) return QB_INVALID_HANDLE;
    if (!out || (n && !logits)) return QB_INVALID_PARAMETERS;
    if (n == 0) return QB_EMPTY_LOGITS;
    std::lock_guard<std::mutex> lk(sp->mu);
    DeviceGuard dg(sp->device);
    if (sp->staged_n < n) {
        uint32_t e = sp->staged.alloc(n * 4, false);
        if (e) return e;
        sp->staged_n = n;
    }
    QB_CUDA(cudaMemcpyAsync(sp->staged.p, logits, n * 4, cudaMemcpyHostToDevice, sp->stream));
    return sampler_run(*sp, sp->staged.as<float>(), n, sp->stream, out);
}

uint32_t qb_sampler_sample_device(uint64_t h, const float *logits, size_t n, uint32_t *out) {
    clear_detail();
    auto sp = find_sampler(h);
    if (!sp) return QB_INVALID_HANDLE;
    if (!out || (n && !logits)) return QB_INVALID_PARAMETERS;
    std::lock_guard<std::mutex> lk(sp->mu);
    DeviceGuard dg(sp->device);
    // The caller's logits may come from another stream: order after all of it.
    QB_CUDA(cudaDeviceSynchronize());
    return sampler_run(*sp, logits, n, sp->stream, out);
}

uint32_t qb_sampler_free(uint64_t h) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_samplers.find(h);
    if (it == g_samplers.end()) return QB_INVALID_HANDLE;
    g_samplers.erase(it);
    return QB_OK;
}

// ----------------------------------------------------------- batch ABI ----

static uint32_t batch_create(uint64_t model, uint64_t comm, size_t sequences, size_t capacity, uint32_t kv_dtype,
                             uint64_t *out) {
    clear_detail();
    auto m = find_model(model);
    if (!m) return QB_INVALID_HANDLE;
    if (!m->finalized) return QB_INVALID_STATE;
    if (!out) return QB_INVALID_PARAMETERS;
    std::shared_ptr<Comm> cm;
    if (comm) {
        cm = find_comm(comm);
        if (!cm) return QB_INVALID_HANDLE;
        if (!cm->connected || cm->rank != m->tp_rank || cm->size != m->tp_size || cm->device != m->device ||
            cm->h != (int)m->c.hidden_dim)
            return QB_INVALID_PARAMETERS;
    } else if (m->tp_size > 1) {
        return QB_INVALID_PARAMETERS;  // a shard decodes only with its communicator
    }
    if (sequences == 0 || capacity == 0 || capacity > m->c.max_tokens) return QB_INVALID_CAPACITY;
    if (kv_dtype > QB_KV_BF16) return QB_INVALID_PARAMETERS;
    auto b = std::make_shared<Batch>();
    b->m = m;
    b->device = m->device;
    b->nseq = sequences;
    b->capacity = capacity;
    b->kv_bf16 = kv_dtype == QB_KV_BF16;
    DeviceGuard dg(b->device);
    PrefillArgs &a = b->a;
    prefill_common(*m, capacity, b->kv_bf16, a);
    const int chunk = (int)std::max<size_t>(sequences, 256);
    a.chunk = chunk;
    if (!prefill_supported(a) || sequences > (1u << 20)) return QB_UNSUPPORTED;
    if (cm && cm->rows < chunk) return QB_INVALID_PARAMETERS;
    // One page pool per layer for all sequences; the table interleaves the
    // sequences' pages (sequence s's page j is pool page j B + s).
    const size_t pps = pages_per_seq(capacity), npages = pps * sequences;
    const size_t kv_esz = b->kv_bf16 ? 2 : 4;
    size_t layer_bytes, kvb;
    if (mul_ovf(npages, m->c.kv_heads * kPageTokens * m->c.head_dim * kv_esz, &layer_bytes) ||
        mul_ovf(round16(layer_bytes), 2 * m->c.layers, &kvb) || npages > 0x7fffffffu)
        return QB_DIMENSION_OVERFLOW;
    uint32_t st;
    QB_CUDA(cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking));
    {
        std::vector<int> tab(npages);
        for (size_t sq = 0; sq < sequences; ++sq)
            for (size_t j = 0; j < pps; ++j) tab[sq * pps + j] = (int)(j * sequences + sq);
        if ((st = b->ptab.alloc(npages * 4, false))) return st == QB_CUDA_ERROR ? QB_ALLOCATION : st;
        QB_CUDA(cudaMemcpy(b->ptab.p, tab.data(), npages * 4, cudaMemcpyHostToDevice));
    }
    if ((st = b->kv.alloc(kvb)) || (st = build_rope(m->c, capacity, b->rope)) ||
        (st = prefill_workspace(*m, chunk, b->ws, a)) ||
        (st = b->logits.alloc(sequences * m->nv * 4, false)) || (st = b->amax.alloc(sequences * 4)))
        return st == QB_CUDA_ERROR ? QB_ALLOCATION : st;
    b->hlayers.resize(m->c.layers);
    QB_CUDA(cudaMemcpy(b->hlayers.data(), m->dlayers.p, m->c.layers * sizeof(DecodeLayer), cudaMemcpyDeviceToHost));
    a.layers = b->hlayers.data();
    tc_prepare(*m, a, b->tcm);
    a.rope = b->rope.as<float2>();
    a.kv.pool = b->kv.as<uint8_t>();
    a.kv.layer_bytes = round16(layer_bytes);
    a.kv.ptab = b->ptab.as<int>();
    a.kv.pps = (int)pps;
    a.logits = b->logits.as<float>();
    a.amax = b->amax.as<uint32_t>();
    if (cm) {
        b->comm = cm;
        a.tp = &cm->view;
        a.tp_seq = &cm->seq;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    uint64_t id = g_next++;
    g_batches[id] = b;
    *out = id;
    return QB_OK;
}

uint32_t qb_batch_create(uint64_t model, size_t sequences, size_t capacity, uint32_t kv_dtype, uint64_t *out) {
    return batch_create(model, 0, sequences, capacity, kv_dtype, out);
}

uint32_t qb_batch_create_tp(uint64_t model, uint64_t comm, size_t sequences, size_t capacity, uint32_t kv_dtype,
                            uint64_t *out) {
    if (!comm) return QB_INVALID_HANDLE;
    return batch_create(model, comm, sequences, capacity, kv_dtype, out);
}

// ------------------------------------------------------------- tp ABI ----

uint32_t qb_tp_comm_create(int device, size_t rows, size_t hidden, uint64_t *out) {
    clear_detail();
    if (!out || rows == 0 || hidden == 0 || hidden % 4 || rows > (1u << 20) || hidden > 0xffffff)
        return QB_INVALID_PARAMETERS;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
        cudaGetLastError();
        return QB_CUDA_ERROR;
    }
    auto c = std::make_shared<Comm>();
    c->device = device;
    c->rows = (int)rows;
    c->h = (int)hidden;
    DeviceGuard dg(device);
    uint32_t st = c->buf.alloc(tp_buffer_bytes(c->rows, c->h));  // zeroed: no flag is up
    if (st) return st == QB_CUDA_ERROR ? QB_ALLOCATION : st;
    std::lock_guard<std::mutex> lk(g_mu);
    uint64_t id = g_next++;
    g_comms[id] = c;
    *out = id;
    return QB_OK;
}

uint32_t qb_tp_comm_handle(uint64_t comm, void *out, size_t len) {
    auto c = find_comm(comm);
    if (!c) return QB_INVALID_HANDLE;
    if (!out || len != sizeof(cudaIpcMemHandle_t)) return QB_INVALID_LENGTH;
    DeviceGuard dg(c->device);
    cudaIpcMemHandle_t hnd;
    QB_CUDA(cudaIpcGetMemHandle(&hnd, c->buf.p));
    memcpy(out, &hnd, sizeof(hnd));
    return QB_OK;
}

uint32_t qb_tp_comm_connect(uint64_t comm, int rank, int size, const void *handles, size_t len) {
    auto c = find_comm(comm);
    if (!c) return QB_INVALID_HANDLE;
    if (c->connected) return QB_INVALID_STATE;
    if (size < 1 || size > kMaxTp || rank < 0 || rank >= size || !handles ||
        len != (size_t)size * sizeof(cudaIpcMemHandle_t))
        return QB_INVALID_PARAMETERS;
    DeviceGuard dg(c->device);
    TpPeers &v = c->view;
    v.rank = rank;
    v.size = size;
    v.rows = c->rows;
    v.h = c->h;
    for (int r = 0; r < size; ++r) {
        void *base = c->buf.p;
        if (r != rank) {
            cudaIpcMemHandle_t hnd;
            memcpy(&hnd, (const uint8_t *)handles + (size_t)r * sizeof(hnd), sizeof(hnd));
            cudaError_t e = cudaIpcOpenMemHandle(&base, hnd, cudaIpcMemLazyEnablePeerAccess);
            if (e != cudaSuccess) {
                cudaGetLastError();
                return QB_CUDA_ERROR;
            }
            c->peer_base[r] = base;
        }
        tp_carve(base, c->rows, c->h, &v.flags[r], &v.part[r], &v.amx[r]);
    }
    c->rank = rank;
    c->size = size;
    c->connected = true;
    return QB_OK;
}

uint32_t qb_tp_comm_free(uint64_t comm) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_comms.find(comm);
    if (it == g_comms.end()) return QB_INVALID_HANDLE;
    g_comms.erase(it);
    return QB_OK;
}

uint32_t qb_batch_prefill(uint64_t batch, const uint32_t *prompts, size_t prompt_len, uint32_t *next_ids) {
    clear_detail();
    auto bp = find_batch(batch);
    if (!bp) return QB_INVALID_HANDLE;
    Batch &b = *bp;
    if (!b.valid) return QB_INVALID_STATE;
    if (b.processed != 0) return QB_NOT_EMPTY;
    if (prompt_len == 0 || !prompts) return QB_EMPTY_INPUT;
    if (prompt_len > b.capacity) return QB_FULL;
    const size_t V = b.m->c.vocab_size, B = b.nseq;
    for (size_t i = 0; i < B * prompt_len; ++i)
        if (prompts[i] >= V) { set_detail(0, V, prompts[i], i); return QB_INVALID_TOKEN; }
    DeviceGuard dg(b.device);
    PrefillArgs &a = b.a;
    cudaError_t e = cudaMemsetAsync(a.err, 0, sizeof(unsigned), b.stream);
    if (e != cudaSuccess) return batch_fail(b, cuda_status(e));
    // K/V of every prompt token but each sequence's last, in chunks that mix
    // sequences; then the last tokens together, with the LM head.
    const size_t fill = prompt_len - 1, total = B * fill;
    std::vector<uint32_t> hid(a.chunk);
    std::vector<int> hpos(a.chunk), hseq(a.chunk);
    for (size_t c0 = 0; c0 < total; c0 += a.chunk) {
        const int nc = (int)std::min<size_t>(a.chunk, total - c0);
        int maxp = 0;
        for (int t = 0; t < nc; ++t) {
            const size_t g = c0 + t, sq = g / fill, p = g % fill;
            hid[t] = prompts[sq * prompt_len + p];
            hpos[t] = (int)p;
            hseq[t] = (int)sq;
            maxp = std::max(maxp, (int)p);
        }
        if ((e = cudaMemcpyAsync(a.ids, hid.data(), nc * 4, cudaMemcpyHostToDevice, b.stream)) ||
            (e = cudaMemcpyAsync(a.pos, hpos.data(), nc * 4, cudaMemcpyHostToDevice, b.stream)) ||
            (e = cudaMemcpyAsync(a.seq, hseq.data(), nc * 4, cudaMemcpyHostToDevice, b.stream)))
            return batch_fail(b, cuda_status(e));
        uint32_t st = batch_forward(b, nc, maxp, false);
        if (st) return st;
        if ((e = cudaStreamSynchronize(b.stream)) != cudaSuccess) return batch_fail(b, cuda_status(e));
    }
    for (size_t sq = 0; sq < B; ++sq) {
        hid[sq] = prompts[sq * prompt_len + fill];
        hpos[sq] = (int)fill;
        hseq[sq] = (int)sq;
    }
    if ((e = cudaMemcpyAsync(a.ids, hid.data(), B * 4, cudaMemcpyHostToDevice, b.stream)) ||
        (e = cudaMemcpyAsync(a.pos, hpos.data(), B * 4, cudaMemcpyHostToDevice, b.stream)) ||
        (e = cudaMemcpyAsync(a.seq, hseq.data(), B * 4, cudaMemcpyHostToDevice, b.stream)))
        return batch_fail(b, cuda_status(e));
    uint32_t st = batch_forward(b, (int)B, (int)fill, true);
    if (st) return st;
    if (next_ids && (e = cudaMemcpyAsync(next_ids, a.amax, B * 4, cudaMemcpyDeviceToHost, b.stream)))
        return batch_fail(b, cuda_status(e));
    if ((st = batch_check(b))) return st;
    b.processed = prompt_len;
    b.logits_valid = true;
    return QB_OK;
}

uint32_t qb_batch_decode_greedy(uint64_t batch, const uint32_t *tokens, size_t steps, uint32_t *ids) {
    clear_detail();
    auto bp = find_batch(batch);
    if (!bp) return QB_INVALID_HANDLE;
    Batch &b = *bp;
    if (!b.valid) return QB_INVALID_STATE;
    if (!tokens || steps == 0) return QB_EMPTY_INPUT;
    if (b.processed + steps > b.capacity) return QB_FULL;
    const size_t V = b.m->c.vocab_size, B = b.nseq;
    for (size_t i = 0; i < B; ++i)
        if (tokens[i] >= V) { set_detail(0, V, tokens[i], i); return QB_INVALID_TOKEN; }
    DeviceGuard dg(b.device);
    PrefillArgs &a = b.a;
    size_t hb;
    if (mul_ovf(steps, B * 4, &hb)) return QB_DIMENSION_OVERFLOW;
    if (b.hist.bytes < hb) {
        uint32_t st = b.hist.alloc(hb, false);
        if (st) return st;
    }
    std::vector<int> hpos(B, (int)b.processed), hseq(B);
    for (size_t sq = 0; sq < B; ++sq) hseq[sq] = (int)sq;
    cudaError_t e;
    if ((e = cudaMemsetAsync(a.err, 0, sizeof(unsigned), b.stream)) ||
        (e = cudaMemcpyAsync(a.ids, tokens, B * 4, cudaMemcpyHostToDevice, b.stream)) ||
        (e = cudaMemcpyAsync(a.pos, hpos.data(), B * 4, cudaMemcpyHostToDevice, b.stream)) ||
        (e = cudaMemcpyAsync(a.seq, hseq.data(), B * 4, cudaMemcpyHostToDevice, b.stream)))
        return batch_fail(b, cuda_status(e));
    for (size_t k = 0; k < steps; ++k) {
        uint32_t st = batch_forward(b, (int)B, (int)(b.processed + k), true);
        if (st) return st;
        if ((e = cudaMemcpyAsync(b.hist.as<uint32_t>() + k * B, a.amax, B * 4, cudaMemcpyDeviceToDevice,
                                 b.stream)) ||
            (e = advance_tokens(a, (int)B, b.stream)))
            return batch_fail(b, cuda_status(e));
    }
    if (ids && (e = cudaMemcpyAsync(ids, b.hist.p, steps * B * 4, cudaMemcpyDeviceToHost, b.stream)))
        return batch_fail(b, cuda_status(e));
    uint32_t st = batch_check(b);
    if (st) return st;
    b.processed += steps;
    b.logits_valid = true;
    return QB_OK;
}

uint32_t qb_batch_logits(uint64_t batch, float *logits, size_t logits_len) {
    clear_detail();
    auto bp = find_batch(batch);
    if (!bp) return QB_INVALID_HANDLE;
    Batch &b = *bp;
    if (!b.valid || !b.logits_valid) return QB_NOT_STARTED;
    if (logits_len != b.nseq * b.m->nv) {  // a shard's own vocabulary rows
        set_detail(0, b.nseq * b.m->nv, logits_len);
        return QB_INVALID_OUTPUT_LENGTH;
    }
    DeviceGuard dg(b.device);
    QB_CUDA(cudaMemcpy(logits, b.logits.p, logits_len * 4, cudaMemcpyDeviceToHost));
    return QB_OK;
}

uint32_t qb_batch_info_get(uint64_t batch, qb_batch_info *out) {
    auto bp = find_batch(batch);
    if (!bp) return QB_INVALID_HANDLE;
    if (!out) return QB_INVALID_PARAMETERS;
    out->sequences = bp->nseq;
    out->capacity = bp->capacity;
    out->processed = bp->processed;
    out->valid = bp->valid ? 1 : 0;
    return QB_OK;
}

uint32_t qb_batch_reset(uint64_t batch) {
    auto bp = find_batch(batch);
    if (!bp) return QB_INVALID_HANDLE;
    bp->processed = 0;
    bp->valid = true;
    bp->logits_valid = false;
    return QB_OK;
}

uint32_t qb_batch_stream(uint64_t batch, void **stream) {
    auto bp = find_batch(batch);
    if (!bp) return QB_INVALID_HANDLE;
    if (!stream) return QB_INVALID_PARAMETERS;
    *stream = (void *)bp->stream;
    return QB_OK;
}

uint32_t qb_batch_free(uint64_t batch) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_batches.find(batch);
    if (it == g_batches.end()) return QB_INVALID_HANDLE;
    g_batches.erase(it);
    return QB_OK;
}

}  // extern "C"
