// Multi-token forward.  The reference evaluates every token with one
// CachedSession step (src/kv_cache.rs:249-475); here a run of tokens --
// the prompt of a session (CachedSession::prefill_into / append_into), or
// one token of each of many independent sequences (batched greedy decoding)
// -- goes through a few wide kernels per layer: row RMSNorm, register-tiled
// FP32 GEMMs over the decode weight layouts (split-K with a deterministic
// reduce when the token count is small), RoPE with the KV write, causal
// attention, and optionally the final norm, the LM head and the greedy
// argmax.  Values agree with the serial path to FP32 summation-order
// differences: the same formulas, FP32 accumulation, reference-order dot
// products in attention, the same RoPE table and the same BF16 rounding of
// stored keys and values.
#include <math.h>

#include <algorithm>
#include <vector>

#include "common.cuh"
#include "prefill.cuh"

namespace qb {
namespace {

__device__ __forceinline__ void flag_bad(unsigned *err, float v) {
    if (!isfinite(v)) atomicOr(err, ERR_NONFINITE);
}

__device__ __forceinline__ float silu_ref(float v) {
    if (v >= 0.0f) return v / (1.0f + expf(-v));
    const float e = expf(v);
    return v * e / (1.0f + e);
}

__device__ float block_max(float v, float *red) {
    for (int off = 16; off; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float m = red[0];
    for (int k = 1; k < nw; ++k) m = fmaxf(m, red[k]);
    return m;
}

__device__ float block_sum(float v, float *red) {
    for (int off = 16; off; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float s = red[0];
    for (int k = 1; k < nw; ++k) s += red[k];
    return s;
}

// ----------------------------------------------------------------- rows ----

template <int TF>
__global__ void embed_rows(const uint32_t *ids, int n, const uint8_t *emb, size_t semb, int h, float *x) {
    for (int t = blockIdx.x; t < n; t += gridDim.x) {
        const uint8_t *row = emb + (size_t)ids[t] * semb;
        for (int i = threadIdx.x; i < h; i += blockDim.x)
            x[(size_t)t * h + i] =
                TF == WF_BF16 ? bf16_to_f32(((const uint16_t *)row)[i]) : ((const float *)row)[i];
    }
}

// Scaled RMSNorm of each row (src/ops.rs:137-149), one CTA per row.
__global__ void rmsnorm_rows(const float *x, const float *g, float *y, int n, int w, float eps, unsigned *err) {
    __shared__ float red[32];
    for (int t = blockIdx.x; t < n; t += gridDim.x) {
        const float *xr = x + (size_t)t * w;
        const float se = sqrtf(eps);
        float m = se;
        for (int i = threadIdx.x; i < w; i += blockDim.x) m = rust_max(m, fabsf(xr[i]));
        m = block_max(m, red);
        float ss = 0.0f;
        for (int i = threadIdx.x; i < w; i += blockDim.x) {
            const float v = xr[i] / m;
            ss = ss + v * v;
        }
        ss = block_sum(ss, red);
        const float seps = se / m;
        const float den = sqrtf(ss / (float)w + seps * seps);
        for (int i = threadIdx.x; i < w; i += blockDim.x) {
            const float o = (xr[i] / m) / den * g[i];
            y[(size_t)t * w + i] = o;
            flag_bad(err, o);
        }
    }
}

// ----------------------------------------------------------------- gemm ----
//
// Y[t][r] = epilogue(sum_k X[t][k] W[r][k]) for t < n tokens and r < N rows,
// FP32 products and accumulation.  W is the decode layout: row r, segment
// s (of seg_len elements) starts at base + s * seg_stride + r * row_stride,
// so the head-blocked o_proj is one segmented matrix.  K, seg_len and every
// leading dimension are multiples of 4.

enum { EPI_QKV = 0, EPI_RESID = 1, EPI_GU = 2, EPI_PLAIN = 3 };

struct GemmW {
    const uint8_t *base;
    size_t row_stride, seg_stride;
    int seg_len;
    const float *scale;  // per row (INT8) or null
    const float *bias;   // per row (EPI_QKV) or null
};

// Four consecutive elements k .. k+3 of row r (k % 4 == 0).
template <int WF>
__device__ __forceinline__ float4 load4(const GemmW &w, int r, int k) {
    const int s = k / w.seg_len, kk = k - s * w.seg_len;
    const uint8_t *row = w.base + (size_t)s * w.seg_stride + (size_t)r * w.row_stride;
    if (WF == WF_F32) return *(const float4 *)(row + (size_t)kk * 4);
    if (WF == WF_BF16) {
        const uint2 v = *(const uint2 *)(row + (size_t)kk * 2);
        return make_float4(bf16_lo(v.x), bf16_hi(v.x), bf16_lo(v.y), bf16_hi(v.y));
    }
    const uint32_t v = *(const uint32_t *)(row + kk);
    return make_float4(u8b_to_f32(v, 0), u8b_to_f32(v, 1), u8b_to_f32(v, 2), u8b_to_f32(v, 3));
}

constexpr int BM = 64, BN = 64, BK = 32;

// The epilogue of one output (t, r) (all kinds but the SwiGLU pairs).
template <int EPI>
__device__ __forceinline__ void epilogue1(const GemmW &w, int t, int r, float v, const float *R, int ldr, float *Y,
                                          int ldy, unsigned *err) {
    if (w.scale) v = v * w.scale[r];
    if (EPI == EPI_QKV) {
        if (w.bias) v = v + w.bias[r];
    } else if (EPI == EPI_RESID) {
        v = R[(size_t)t * ldr + r] + v;
    }
    Y[(size_t)t * ldy + r] = v;
    flag_bad(err, v);
}

// The SwiGLU epilogue of a (gate, up) row pair r, r + 1.
__device__ __forceinline__ void epilogue_gu(const GemmW &w, int t, int r, float g, float u, float *Y, int ldy,
                                            unsigned *err) {
    if (w.scale) {
        g = g * w.scale[r];
        u = u * w.scale[r + 1];
    }
    const float a = silu_ref(g) * u;
    Y[(size_t)t * ldy + (r >> 1)] = a;
    flag_bad(err, g);
    flag_bad(err, a);
}

// grid.z = ksplit slices of K (each kper elements, a multiple of BK).  With
// ksplit > 1 the raw sums go to part[z][t][r] and reduce_epilogue finishes.
template <int WF, int EPI>
__global__ void __launch_bounds__(256) gemm_rows(const float *X, int ldx, int n, int N, int K, GemmW w,
                                                 const float *R, int ldr, float *Y, int ldy, unsigned *err,
                                                 int kper, float *part) {
    __shared__ __align__(16) float Xs[BK][BM + 4];
    __shared__ __align__(16) float Ws[BK][BN + 4];
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int kz0 = blockIdx.z * kper, kz1 = min(K, kz0 + kper);
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
    for (int k0 = kz0; k0 < kz1; k0 += BK) {
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const int f = tid + q * 256, tt = f >> 3, kk = (f & 7) * 4;
            float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (m0 + tt < n && k0 + kk < kz1) v = *(const float4 *)(X + (size_t)(m0 + tt) * ldx + k0 + kk);
            Xs[kk][tt] = v.x;
            Xs[kk + 1][tt] = v.y;
            Xs[kk + 2][tt] = v.z;
            Xs[kk + 3][tt] = v.w;
            const int rr = tt;
            float4 u = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (n0 + rr < N && k0 + kk < kz1) u = load4<WF>(w, n0 + rr, k0 + kk);
            Ws[kk][rr] = u.x;
            Ws[kk + 1][rr] = u.y;
            Ws[kk + 2][rr] = u.z;
            Ws[kk + 3][rr] = u.w;
        }
        __syncthreads();
#pragma unroll 8
        for (int k = 0; k < BK; ++k) {
            const float4 a = *(const float4 *)&Xs[k][ty * 4];
            const float4 b = *(const float4 *)&Ws[k][tx * 4];
            const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
    if (gridDim.z > 1) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int t = m0 + ty * 4 + i;
            if (t >= n) continue;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int r = n0 + tx * 4 + j;
                if (r < N) part[((size_t)blockIdx.z * n + t) * N + r] = acc[i][j];
            }
        }
        return;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int t = m0 + ty * 4 + i;
        if (t >= n) continue;
        if (EPI == EPI_GU) {
            // Rows come in (gate, up) pairs: the thread's four rows hold two.
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
                const int r = n0 + tx * 4 + 2 * jj;
                if (r + 1 < N) epilogue_gu(w, t, r, acc[i][2 * jj], acc[i][2 * jj + 1], Y, ldy, err);
            }
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int r = n0 + tx * 4 + j;
                if (r < N) epilogue1<EPI>(w, t, r, acc[i][j], R, ldr, Y, ldy, err);
            }
        }
    }
}

// Sums the ksplit partials of each output in slice order, then the
// epilogue (SwiGLU outputs one value per row pair).
template <int EPI>
__global__ void reduce_epilogue(const float *part, int ks, int n, int N, GemmW w, const float *R, int ldr, float *Y,
                                int ldy, unsigned *err) {
    const size_t per = (size_t)n * N;
    const size_t total = EPI == EPI_GU ? per / 2 : per;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        if (EPI == EPI_GU) {
            const size_t t = i / (N / 2);
            const int r = (int)(i - t * (N / 2)) * 2;
            float g = 0.0f, u = 0.0f;
            for (int z = 0; z < ks; ++z) {
                g += part[z * per + t * N + r];
                u += part[z * per + t * N + r + 1];
            }
            epilogue_gu(w, (int)t, r, g, u, Y, ldy, err);
        } else {
            const size_t t = i / N;
            const int r = (int)(i - t * N);
            float v = 0.0f;
            for (int z = 0; z < ks; ++z) v += part[z * per + i];
            epilogue1<EPI>(w, (int)t, r, v, R, ldr, Y, ldy, err);
        }
    }
}

// -------------------------------------------------------------- attention ----

// K (layer l) of sequence `seq`; V follows at + kv_layer_bytes.
__device__ __forceinline__ uint8_t *kv_k(uint8_t *kv, size_t seq_bytes, size_t layer_bytes, int seq, int l) {
    return kv + (size_t)seq * seq_bytes + (size_t)(2 * l) * layer_bytes;
}

// RoPE of every query and key head of each token (at its own position) with
// the host table, in place, and the K (rotated) and V write into its
// sequence's cache -- BF16 round-to-nearest-even when the cache is BF16.
__global__ void rope_kv(float *qkv, int n, const int *pos, const int *seqs, int l, int h, int qh, int kvh, int hd,
                        const float2 *rope, int cap, uint8_t *kv, size_t seq_bytes, size_t layer_bytes, int kv_bf16,
                        unsigned *err) {
    const int half = hd / 2, rq = h + 2 * kvh * hd;
    for (int t = blockIdx.x; t < n; t += gridDim.x) {
        const int p = pos[t];
        uint8_t *kc = kv_k(kv, seq_bytes, layer_bytes, seqs[t], l), *vc = kc + layer_bytes;
        float *row = qkv + (size_t)t * rq;
        const float2 *rp = rope + (size_t)p * half;
        for (int idx = threadIdx.x; idx < qh * half; idx += blockDim.x) {
            const int hh = idx / half, j = idx - hh * half;
            float *q = row + (size_t)hh * hd;
            const float2 cs = rp[j];
            const float a = q[j], b = q[j + half];
            const float q0 = a * cs.x - b * cs.y, q1 = b * cs.x + a * cs.y;
            q[j] = q0;
            q[j + half] = q1;
            flag_bad(err, q0);
            flag_bad(err, q1);
        }
        for (int idx = threadIdx.x; idx < kvh * half; idx += blockDim.x) {
            const int g = idx / half, j = idx - g * half;
            const float *k = row + h + (size_t)g * hd;
            const float2 cs = rp[j];
            const float a = k[j], b = k[j + half];
            const float k0 = a * cs.x - b * cs.y, k1 = b * cs.x + a * cs.y;
            flag_bad(err, k0);
            flag_bad(err, k1);
            const size_t base = ((size_t)g * cap + p) * hd;
            if (kv_bf16) {
                ((uint16_t *)kc)[base + j] = f32_to_bf16_rne(k0);
                ((uint16_t *)kc)[base + j + half] = f32_to_bf16_rne(k1);
            } else {
                ((float *)kc)[base + j] = k0;
                ((float *)kc)[base + j + half] = k1;
            }
        }
        for (int idx = threadIdx.x; idx < kvh * hd; idx += blockDim.x) {
            const int g = idx / hd, i = idx - g * hd;
            const float v = row[h + (size_t)kvh * hd + (size_t)g * hd + i];
            const size_t at = ((size_t)g * cap + p) * hd + i;
            if (kv_bf16) ((uint16_t *)vc)[at] = f32_to_bf16_rne(v);
            else ((float *)vc)[at] = v;
        }
    }
}

template <int KVBF16>
__device__ __forceinline__ float kv_at(const uint8_t *base, size_t idx) {
    if (KVBF16) return bf16_to_f32(((const uint16_t *)base)[idx]);
    return ((const float *)base)[idx];
}

// One CTA per (token, query head): scores q.k / sqrt(hd) over the token's
// sequence positions 0 .. pos (dot products by increasing index), softmax
// with the maximum subtracted and division by the sum, and the context by
// increasing position (src/kv_cache.rs:555-575).  Shared memory: q [hd],
// scores [max_pos + 1], 32 floats of reduction space.
template <int KVBF16>
__global__ void attention_rows(const float *qkv, int n, const int *pos, const int *seqs, int l, int max_pos, int h,
                               int qh, int kvh, int hd, int group, int cap, const uint8_t *kv, size_t seq_bytes,
                               size_t layer_bytes, float sqrt_hd, float *ctx, unsigned *err) {
    extern __shared__ float asm_[];
    const int t = blockIdx.x / qh, hh = blockIdx.x - t * qh, g = hh / group, p = pos[t];
    const int rq = h + 2 * kvh * hd;
    const uint8_t *kc = kv + (size_t)seqs[t] * seq_bytes + (size_t)(2 * l) * layer_bytes, *vc = kc + layer_bytes;
    float *qs = asm_, *sc = qs + hd, *red = sc + (max_pos + 1);
    for (int i = threadIdx.x; i < hd; i += blockDim.x) qs[i] = qkv[(size_t)t * rq + (size_t)hh * hd + i];
    __syncthreads();
    const size_t kv0 = (size_t)g * cap * hd;
    float m = -INFINITY;
    for (int q = threadIdx.x; q <= p; q += blockDim.x) {
        const size_t row = kv0 + (size_t)q * hd;
        float s = 0.0f;
        for (int i = 0; i < hd; ++i) s = s + qs[i] * kv_at<KVBF16>(kc, row + i);
        s = s / sqrt_hd;
        sc[q] = s;
        m = rust_max(m, s);
    }
    m = block_max(m, red);
    float se = 0.0f;
    for (int q = threadIdx.x; q <= p; q += blockDim.x) {
        const float e = expf(sc[q] - m);
        sc[q] = e;
        se += e;
    }
    se = block_sum(se, red);
    for (int i = threadIdx.x; i < hd; i += blockDim.x) {
        float acc = 0.0f;
#pragma unroll 4
        for (int q = 0; q <= p; ++q) acc = acc + (sc[q] / se) * kv_at<KVBF16>(vc, kv0 + (size_t)q * hd + i);
        ctx[(size_t)t * h + (size_t)hh * hd + i] = acc;
        flag_bad(err, acc);
    }
}

// Greedy id of each logits row: strict > over increasing ids keeps the
// lowest id among equal maxima (src/sampling.rs:65-70).
__global__ void argmax_rows(const float *logits, int n, int V, uint32_t *out, unsigned *err) {
    __shared__ float bvs[32];
    __shared__ int bis[32];
    for (int t = blockIdx.x; t < n; t += gridDim.x) {
        const float *row = logits + (size_t)t * V;
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int v = threadIdx.x; v < V; v += blockDim.x) {
            const float x = row[v];
            flag_bad(err, x);
            if (x > bv) { bv = x; bi = v; }
        }
        for (int off = 16; off; off >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
        __syncthreads();
        if (lane == 0) { bvs[warp] = bv; bis[warp] = bi; }
        __syncthreads();
        if (threadIdx.x == 0) {
            float gv = bvs[0];
            int gi = bis[0];
            for (int k = 1; k < nw; ++k)
                if (bvs[k] > gv || (bvs[k] == gv && bis[k] < gi)) { gv = bvs[k]; gi = bis[k]; }
            out[t] = gi >= 0 && gi < V ? (uint32_t)gi : 0u;
        }
    }
}

__global__ void advance_kernel(const uint32_t *amax, uint32_t *ids, int *pos, int n) {
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < n; t += gridDim.x * blockDim.x) {
        ids[t] = amax[t];
        pos[t] += 1;
    }
}

// ------------------------------------------------------------------ host ----

// Splits K into ks slices (each a multiple of BK) when the output tiles
// alone leave most SMs idle; the partials must fit the workspace.
int choose_split(int n, int N, int K, size_t part_floats) {
    const int tiles = ((N + BN - 1) / BN) * ((n + BM - 1) / BM);
    int ks = 1;
    while (ks < 8 && tiles * ks * 2 <= 296 && K / (ks * 2) >= 256 &&
           (size_t)(ks * 2) * n * N <= part_floats)
        ks *= 2;
    return ks;
}

template <int WF, int EPI>
cudaError_t gemm(const PrefillArgs &a, const float *X, int ldx, int n, int N, int K, const GemmW &w, const float *R,
                 int ldr, float *Y, int ldy, cudaStream_t st) {
    const int ks = choose_split(n, N, K, a.part_floats);
    const int kper = ((K + ks - 1) / ks + BK - 1) / BK * BK;
    const int ksn = (K + kper - 1) / kper;
    dim3 grid((N + BN - 1) / BN, (n + BM - 1) / BM, ksn);
    gemm_rows<WF, EPI><<<grid, 256, 0, st>>>(X, ldx, n, N, K, w, R, ldr, Y, ldy, a.err, kper, a.part);
    if (ksn > 1) {
        const size_t total = (size_t)n * N / (EPI == EPI_GU ? 2 : 1);
        const unsigned blocks = (unsigned)std::min<size_t>((total + 255) / 256, 4096);
        reduce_epilogue<EPI><<<blocks, 256, 0, st>>>(a.part, ksn, n, N, w, R, ldr, Y, ldy, a.err);
    }
    return cudaGetLastError();
}

template <int WF>
cudaError_t layer_gemm(int which, const PrefillArgs &a, const DecodeLayer &Ly, int n, cudaStream_t st) {
    const int kv = a.kvh * a.hd, rq = a.h + 2 * kv;
    switch (which) {
    case 0: {  // QKV (+ bias)
        GemmW w{Ly.wqkv, a.sh, 0, a.h, Ly.sqkv, Ly.bqkv};
        return gemm<WF, EPI_QKV>(a, a.xn, a.h, n, rq, a.h, w, nullptr, 0, a.qkv, rq, st);
    }
    case 1: {  // o_proj (head-blocked K) + residual
        GemmW w{Ly.wo, a.shd, (size_t)a.h * a.shd, a.hd, Ly.so, nullptr};
        return gemm<WF, EPI_RESID>(a, a.ctx, a.h, n, a.h, a.qh * a.hd, w, a.x, a.h, a.h2, a.h, st);
    }
    case 2: {  // (gate, up) pairs -> SwiGLU
        GemmW w{Ly.wgu, a.sh, 0, a.h, Ly.sgu, nullptr};
        return gemm<WF, EPI_GU>(a, a.xn, a.h, n, 2 * a.ff, a.h, w, nullptr, 0, a.act, a.ff, st);
    }
    default: {  // down + residual
        GemmW w{Ly.wd, a.sff, 0, a.ff, Ly.sd, nullptr};
        return gemm<WF, EPI_RESID>(a, a.act, a.ff, n, a.h, a.ff, w, a.h2, a.h, a.x, a.h, st);
    }
    }
}

cudaError_t run_gemm(int which, const PrefillArgs &a, const DecodeLayer &Ly, int n, cudaStream_t st) {
    if (a.wfmt == WF_I8) return layer_gemm<WF_I8>(which, a, Ly, n, st);
    if (a.wfmt == WF_BF16) return layer_gemm<WF_BF16>(which, a, Ly, n, st);
    return layer_gemm<WF_F32>(which, a, Ly, n, st);
}

size_t attention_smem(const PrefillArgs &a, int max_pos) { return ((size_t)a.hd + max_pos + 1 + 32) * sizeof(float); }

}  // namespace

bool prefill_supported(const PrefillArgs &a) {
    if (a.chunk < 1 || a.h % 4 || a.ff % 4 || a.hd % 4 || a.hd < 2) return false;
    return attention_smem(a, a.cap - 1) <= 48 * 1024;
}

cudaError_t forward_tokens(const PrefillArgs &a, int n, int max_pos, bool lm_head, cudaStream_t st) {
    if (n < 1 || n > a.chunk || max_pos >= a.cap) return cudaErrorInvalidValue;
    const int rows_grid = std::min(n, 4096);
    if (a.tfmt == WF_BF16) embed_rows<WF_BF16><<<rows_grid, 256, 0, st>>>(a.ids, n, a.emb, a.semb, a.h, a.x);
    else embed_rows<WF_F32><<<rows_grid, 256, 0, st>>>(a.ids, n, a.emb, a.semb, a.h, a.x);
    cudaError_t e = cudaGetLastError();
    for (int l = 0; l < a.L && e == cudaSuccess; ++l) {
        const DecodeLayer &Ly = a.layers[l];
        rmsnorm_rows<<<rows_grid, 256, 0, st>>>(a.x, Ly.attn_norm, a.xn, n, a.h, a.eps, a.err);
        if ((e = run_gemm(0, a, Ly, n, st)) != cudaSuccess) break;
        rope_kv<<<rows_grid, 128, 0, st>>>(a.qkv, n, a.pos, a.seq, l, a.h, a.qh, a.kvh, a.hd, a.rope, a.cap, a.kv,
                                           a.kv_seq_bytes, a.kv_layer_bytes, a.kv_bf16, a.err);
        const size_t sm = attention_smem(a, max_pos);
        if (a.kv_bf16)
            attention_rows<1><<<n * a.qh, 128, sm, st>>>(a.qkv, n, a.pos, a.seq, l, max_pos, a.h, a.qh, a.kvh, a.hd,
                                                         a.group, a.cap, a.kv, a.kv_seq_bytes, a.kv_layer_bytes,
                                                         a.sqrt_hd, a.ctx, a.err);
        else
            attention_rows<0><<<n * a.qh, 128, sm, st>>>(a.qkv, n, a.pos, a.seq, l, max_pos, a.h, a.qh, a.kvh, a.hd,
                                                         a.group, a.cap, a.kv, a.kv_seq_bytes, a.kv_layer_bytes,
                                                         a.sqrt_hd, a.ctx, a.err);
        if ((e = cudaGetLastError()) != cudaSuccess) break;
        if (l + 1 == a.L && !lm_head) break;  // the last layer's MLP feeds only the logits
        if ((e = run_gemm(1, a, Ly, n, st)) != cudaSuccess) break;
        rmsnorm_rows<<<rows_grid, 256, 0, st>>>(a.h2, Ly.ffn_norm, a.xn, n, a.h, a.eps, a.err);
        if ((e = run_gemm(2, a, Ly, n, st)) != cudaSuccess) break;
        if ((e = run_gemm(3, a, Ly, n, st)) != cudaSuccess) break;
    }
    if (e != cudaSuccess || !lm_head) return e;
    // Final norm, the LM head (tied table or untied head) and the argmax.
    rmsnorm_rows<<<rows_grid, 256, 0, st>>>(a.x, a.final_norm, a.xn, n, a.h, a.eps, a.err);
    GemmW w{a.head, a.semb, 0, a.h, nullptr, nullptr};
    if (a.tfmt == WF_BF16) e = gemm<WF_BF16, EPI_PLAIN>(a, a.xn, a.h, n, a.V, a.h, w, nullptr, 0, a.logits, a.V, st);
    else e = gemm<WF_F32, EPI_PLAIN>(a, a.xn, a.h, n, a.V, a.h, w, nullptr, 0, a.logits, a.V, st);
    if (e != cudaSuccess) return e;
    argmax_rows<<<rows_grid, 256, 0, st>>>(a.logits, n, a.V, a.amax, a.err);
    return cudaGetLastError();
}

cudaError_t advance_tokens(const PrefillArgs &a, int n, cudaStream_t st) {
    advance_kernel<<<(n + 255) / 256, 256, 0, st>>>(a.amax, a.ids, a.pos, n);
    return cudaGetLastError();
}

cudaError_t prefill_kv(const PrefillArgs &a, const uint32_t *tokens, int n, int p0, cudaStream_t st,
                       bool *nonfinite) {
    *nonfinite = false;
    cudaError_t e = cudaMemsetAsync(a.err, 0, sizeof(unsigned), st);
    std::vector<int> hpos(a.chunk), hseq(a.chunk, 0);
    for (int c0 = 0; c0 < n && e == cudaSuccess; c0 += a.chunk) {
        const int nc = std::min(a.chunk, n - c0);
        for (int t = 0; t < nc; ++t) hpos[t] = p0 + c0 + t;
        if ((e = cudaMemcpyAsync(a.ids, tokens + c0, (size_t)nc * sizeof(uint32_t), cudaMemcpyHostToDevice, st)) ||
            (e = cudaMemcpyAsync(a.pos, hpos.data(), (size_t)nc * sizeof(int), cudaMemcpyHostToDevice, st)) ||
            (e = cudaMemcpyAsync(a.seq, hseq.data(), (size_t)nc * sizeof(int), cudaMemcpyHostToDevice, st)))
            break;
        e = forward_tokens(a, nc, p0 + c0 + nc - 1, false, st);
        // The host position array is rewritten by the next chunk: wait for
        // this chunk's copies (and kernels) first.
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    }
    unsigned herr = 0;
    if (e == cudaSuccess) e = cudaMemcpyAsync(&herr, a.err, sizeof(unsigned), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e == cudaSuccess) *nonfinite = herr != 0;
    return e;
}

}  // namespace qb
