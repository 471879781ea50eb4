// Persistent decode-step kernel for batch-1 greedy decoding on sm_100a.
//
// One cooperative launch evaluates one token through every layer and the LM
// head (src/kv_cache.rs:347-475 with attend_one :479-590) and leaves the
// greedy argmax (src/sampling.rs:65-70) in the control block.  The grid is
// one 512-thread CTA per SM.  Phases are separated by a grid barrier whose
// wait is bounded by a timeout (the kernel then reports ERR_TIMEOUT and
// returns; it never spins forever):
//
//   per layer:  QKV      RMSNorm (each CTA, redundantly) -> rows of [Wq;Wk;Wv]
//                        + bias
//               ATTN     per (query head, o_proj row split): RoPE from the host
//                        cos/sin table, K/V write, softmax(q.K/sqrt d).V, then
//                        that head's o_proj partial for a slice of rows
//               GATE/UP  residual + sum of head partials, RMSNorm, rows of
//                        gate and up, SiLU(gate)*up
//               DOWN     rows of down + residual
//   final:      LM HEAD  RMSNorm, rows of the (tied) table, logits, argmax;
//                        the last CTA reduces the per-CTA argmaxes.
//
// Weights stream with 16-byte non-allocating loads; each CTA prefetches a
// slice of the weights two phases ahead into L2 with cp.async.bulk.prefetch,
// so HBM keeps streaming while the grid waits at a barrier.
#include <math.h>

#include "common.cuh"
#include "decode.cuh"

namespace qb {

constexpr int NT = kDecodeThreads;
constexpr int NW = NT / 32;
constexpr int ITEMS = 8;

template <int WF> struct Fmt;
template <> struct Fmt<WF_F32> { static constexpr int EPC = 4; static constexpr int ESZ = 4; };
template <> struct Fmt<WF_BF16> { static constexpr int EPC = 8; static constexpr int ESZ = 2; };
template <> struct Fmt<WF_I8> { static constexpr int EPC = 16; static constexpr int ESZ = 1; };

__device__ __forceinline__ float ldcg(const float *p) { return __ldcg(p); }

// Dot product of one 16-byte weight chunk with EPC activations (FMA chain).
template <int WF>
__device__ __forceinline__ float chunk_dot(const uint4 &w, const float *x) {
    float a = 0.0f;
    if (WF == WF_F32) {
        a = fmaf(x[0], __uint_as_float(w.x), a);
        a = fmaf(x[1], __uint_as_float(w.y), a);
        a = fmaf(x[2], __uint_as_float(w.z), a);
        a = fmaf(x[3], __uint_as_float(w.w), a);
    } else if (WF == WF_BF16) {
        a = fmaf(x[0], bf16_lo(w.x), a);
        a = fmaf(x[1], bf16_hi(w.x), a);
        a = fmaf(x[2], bf16_lo(w.y), a);
        a = fmaf(x[3], bf16_hi(w.y), a);
        a = fmaf(x[4], bf16_lo(w.z), a);
        a = fmaf(x[5], bf16_hi(w.z), a);
        a = fmaf(x[6], bf16_lo(w.w), a);
        a = fmaf(x[7], bf16_hi(w.w), a);
    } else {
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
#pragma unroll
            for (int b = 0; b < 4; ++b) a = fmaf(x[4 * k + b], u8b_to_f32(ws[k], b), a);
        }
    }
    return a;
}

// Block-wide reductions in a fixed order (warp xor tree, then warp partials
// summed in warp order by thread 0), broadcast to every thread.
__device__ __forceinline__ float block_sum(float v, float *red) {
    int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int off = 16; off; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = red[0];
        for (int i = 1; i < NW; ++i) s += red[i];
        red[NW] = s;
    }
    __syncthreads();
    return red[NW];
}

__device__ __forceinline__ float block_max(float v, float *red) {
    int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int off = 16; off; off >>= 1) v = rust_max(v, __shfl_xor_sync(0xffffffffu, v, off));
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = red[0];
        for (int i = 1; i < NW; ++i) s = rust_max(s, red[i]);
        red[NW] = s;
    }
    __syncthreads();
    return red[NW];
}

// Scaled RMSNorm of `in` (shared, width w) into `out` (shared, zero-padded
// to `padded`), src/ops.rs:137-149.  The row scale is an exact maximum.
__device__ void block_rmsnorm(const float *in, const float *__restrict__ gain, float *out, int w,
                              int padded, float eps, float *red) {
    const float se = sqrtf(eps);
    float m = se;
    for (int i = threadIdx.x; i < w; i += NT) m = rust_max(m, fabsf(in[i]));
    m = block_max(m, red);
    float ss = 0.0f;
    for (int i = threadIdx.x; i < w; i += NT) {
        float v = in[i] / m;
        ss = ss + v * v;
    }
    ss = block_sum(ss, red);
    float seps = se / m;
    float den = sqrtf(ss / (float)w + seps * seps);
    for (int i = threadIdx.x; i < padded; i += NT) out[i] = i < w ? (in[i] / m) / den * gain[i] : 0.0f;
    __syncthreads();
}

// CTA matrix-vector product over R rows of C 16-byte chunks each.
// rowp(r) gives row r's base; emit(r, y) runs once per row on lane 0 of a
// warp.  When C <= NT every thread owns one chunk column (its activations in
// registers) and walks rows; otherwise threads stride the chunks of each row.
// Partial sums meet in shared memory and are reduced per row in a fixed order.
template <int WF, class RowPtr, class Emit>
__device__ void cta_gemv(RowPtr rowp, int R, int C, const float *xs, float *part, int part_cap,
                         Emit emit) {
    constexpr int EPC = Fmt<WF>::EPC;
    if (R <= 0 || C <= 0) return;
    const int t = threadIdx.x, lane = t & 31;
    if (C <= NT) {
        const int RS = NT / C;
        const int c = t % C, rs = t / C;
        const bool active = rs < RS;
        float xr[EPC];
#pragma unroll
        for (int k = 0; k < EPC; ++k) xr[k] = active ? xs[c * EPC + k] : 0.0f;
        int RR = part_cap / C;
        if (RR < 1) RR = 1;
        for (int row0 = 0; row0 < R; row0 += RR) {
            const int rr = min(RR, R - row0);
            if (active) {
                for (int r = rs; r < rr; r += RS * ITEMS) {
                    uint4 w[ITEMS];
#pragma unroll
                    for (int k = 0; k < ITEMS; ++k) {
                        int rk = r + k * RS;
                        if (rk < rr) w[k] = ld_stream_u4(rowp(row0 + rk) + (size_t)c * 16);
                    }
#pragma unroll
                    for (int k = 0; k < ITEMS; ++k) {
                        int rk = r + k * RS;
                        if (rk < rr) part[rk * C + c] = chunk_dot<WF>(w[k], xr);
                    }
                }
            }
            __syncthreads();
            for (int r = t >> 5; r < rr; r += NW) {
                float s = 0.0f;
                for (int cc = lane; cc < C; cc += 32) s += part[r * C + cc];
#pragma unroll
                for (int off = 16; off; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
                if (lane == 0) emit(row0 + r, s);
            }
            __syncthreads();
        }
    } else {
        int RR = part_cap / NT;
        if (RR < 1) RR = 1;
        for (int row0 = 0; row0 < R; row0 += RR) {
            const int rr = min(RR, R - row0);
            for (int r = 0; r < rr; ++r) {
                const uint8_t *row = rowp(row0 + r);
                float acc = 0.0f;
                for (int c0 = t; c0 < C; c0 += NT * ITEMS) {
                    uint4 w[ITEMS];
#pragma unroll
                    for (int k = 0; k < ITEMS; ++k) {
                        int c = c0 + k * NT;
                        if (c < C) w[k] = ld_stream_u4(row + (size_t)c * 16);
                    }
#pragma unroll
                    for (int k = 0; k < ITEMS; ++k) {
                        int c = c0 + k * NT;
                        if (c < C) acc += chunk_dot<WF>(w[k], xs + c * EPC);
                    }
                }
                part[r * NT + t] = acc;
            }
            __syncthreads();
            for (int r = t >> 5; r < rr; r += NW) {
                float s = 0.0f;
                for (int cc = lane; cc < NT; cc += 32) s += part[r * NT + cc];
#pragma unroll
                for (int off = 16; off; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
                if (lane == 0) emit(row0 + r, s);
            }
            __syncthreads();
        }
    }
}

// Grid barrier with a bounded wait.  Returns false (after recording
// ERR_TIMEOUT) when the arrivals do not complete within the timeout or when
// another CTA has already timed out.
__device__ bool grid_barrier(DecodeCtrl *ctrl, unsigned target, unsigned long long timeout_ns,
                             int *s_flag) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        red_release_add_u32(&ctrl->bar, 1u);
        int ok = 1;
        if (ld_acquire_u32(&ctrl->bar) < target) {
            const uint64_t t0 = globaltimer_ns();
            unsigned spins = 0;
            while (ld_acquire_u32(&ctrl->bar) < target) {
                if ((++spins & 255u) == 0) {
                    if (*(volatile unsigned *)&ctrl->error & ERR_TIMEOUT) { ok = 0; break; }
                    if (globaltimer_ns() - t0 > timeout_ns) {
                        atomicOr(&ctrl->error, ERR_TIMEOUT);
                        ok = 0;
                        break;
                    }
                }
            }
        }
        *s_flag = ok;
    }
    __syncthreads();
    return *s_flag != 0;
}

__device__ __forceinline__ void flag_nonfinite(DecodeCtrl *ctrl, float v) {
    if (!isfinite(v)) atomicOr(&ctrl->error, ERR_NONFINITE);
}

// Prefetches this CTA's 1/G slice of [base, base+bytes) into L2.
__device__ __forceinline__ void prefetch_slice(const void *base, size_t bytes, int b, int G) {
    if (!base || bytes == 0) return;
    size_t lo = (bytes * (size_t)b / (size_t)G) & ~(size_t)15;
    size_t hi = (bytes * (size_t)(b + 1) / (size_t)G) & ~(size_t)15;
    if (b == G - 1) hi = bytes & ~(size_t)15;
    const int lane = threadIdx.x & 31;
    const size_t piece = 16384;
    for (size_t off = lo + (size_t)lane * piece; off < hi; off += 32 * piece) {
        size_t n = hi - off < piece ? hi - off : piece;
        prefetch_l2_bulk((const char *)base + off, (uint32_t)n);
    }
}

// Phase k in the step's sequence: 4 per layer (QKV, ATTN, GATE/UP, DOWN),
// then the LM head.  Prefetch the weights phase k will stream.
__device__ void prefetch_phase(const DecodeParams &p, int k, int pos, int b, int G) {
    if (!p.prefetch || threadIdx.x >= 32) return;
    if (k >= 4 * p.L) {
        // LM head: the first rows of this CTA's own range (later rounds
        // prefetch further ahead inside the phase).
        int v0 = (int)((long long)p.V * b / G), v1 = (int)((long long)p.V * (b + 1) / G);
        int n = min(v1 - v0, 64);
        if (n > 0 && threadIdx.x == 0)
            prefetch_l2_bulk(p.head + (size_t)v0 * p.semb, (uint32_t)((size_t)n * p.semb));
        return;
    }
    const DecodeLayer &Ly = p.layers[k >> 2];
    const size_t kv = (size_t)p.kvh * p.hd;
    switch (k & 3) {
    case 0: prefetch_slice(Ly.wqkv, (size_t)p.rqkv * p.sh, b, G); break;
    case 1: {
        prefetch_slice(Ly.wo, (size_t)p.qh * p.h * p.shd, b, G);
        // Cached keys/values of earlier positions do not depend on this step.
        const size_t esz = p.kv_bf16 ? 2 : 4;
        for (int g = 0; g < p.kvh; ++g) {
            prefetch_slice(Ly.kc + (size_t)g * p.cap * p.hd * esz, (size_t)pos * p.hd * esz, b, G);
            prefetch_slice(Ly.vc + (size_t)g * p.cap * p.hd * esz, (size_t)pos * p.hd * esz, b, G);
        }
        (void)kv;
        break;
    }
    case 2:
        prefetch_slice(Ly.wg, (size_t)p.ff * p.sh, b, G);
        prefetch_slice(Ly.wu, (size_t)p.ff * p.sh, b, G);
        break;
    case 3: prefetch_slice(Ly.wd, (size_t)p.h * p.sff, b, G); break;
    }
}

__device__ __forceinline__ float round_bf16(float x) {
    return __uint_as_float((uint32_t)f32_to_bf16_rne(x) << 16);
}

// Residual-stream input of layer l at element i: the embedding row for
// layer 0, the previous layer's output otherwise.
__device__ __forceinline__ float resid_in(const DecodeParams &p, int l, int token, int i) {
    if (l > 0) return ldcg(p.hidden + i);
    const uint8_t *row = p.emb + (size_t)token * p.semb;
    return p.tfmt == WF_BF16 ? bf16_to_f32(((const uint16_t *)row)[i]) : ((const float *)row)[i];
}

// h' = x + o_proj(ctx): the head partials summed in head order, then the
// residual added (src/kv_cache.rs:405-406).  Identical in every phase that
// needs it.
__device__ __forceinline__ float after_attention(const DecodeParams &p, int l, int token, int i) {
    float o = ldcg(p.part + i);
    for (int hh = 1; hh < p.qh; ++hh) o += ldcg(p.part + (size_t)hh * p.h + i);
    return resid_in(p, l, token, i) + o;
}

__device__ __forceinline__ float silu1(float v) {
    if (v >= 0.0f) return v / (1.0f + expf(-v));
    float e = expf(v);
    return v * e / (1.0f + e);
}

template <int KVBF16>
__device__ __forceinline__ float kv_load(const uint8_t *base, size_t idx) {
    if (KVBF16) return bf16_to_f32(__ldcg((const unsigned short *)base + idx));
    return __ldcg((const float *)base + idx);
}

// Attention for query head hh at position pos, then its o_proj partial over
// rows [r0, r1) (src/kv_cache.rs:550-585).
template <int WF, int KVBF16>
__device__ void attention_head(const DecodeParams &p, const DecodeLayer &Ly, int hh, int sp,
                               int pos, float *sm) {
    const int hd = p.hd, half = hd / 2, g = hh / p.group;
    const size_t kvw = (size_t)p.kvh * hd;
    float *qs = sm + p.sm_q, *ks = qs + hd, *vs = ks + hd, *ctx = vs + hd;
    float *sc = sm + p.sm_sc, *red = sm + p.sm_red, *part = sm + p.sm_part;
    const float2 *rp = p.rope + (size_t)pos * half;
    for (int j = threadIdx.x; j < half; j += NT) {
        float2 cs = rp[j];
        float a = ldcg(p.qkv + (size_t)hh * hd + j), b = ldcg(p.qkv + (size_t)hh * hd + j + half);
        qs[j] = a * cs.x - b * cs.y;
        qs[j + half] = b * cs.x + a * cs.y;
        float ka = ldcg(p.qkv + p.h + (size_t)g * hd + j), kb = ldcg(p.qkv + p.h + (size_t)g * hd + j + half);
        float k0 = ka * cs.x - kb * cs.y, k1 = kb * cs.x + ka * cs.y;
        if (KVBF16) { k0 = round_bf16(k0); k1 = round_bf16(k1); }
        ks[j] = k0;
        ks[j + half] = k1;
    }
    for (int i = threadIdx.x; i < hd; i += NT) {
        float v = ldcg(p.qkv + p.h + kvw + (size_t)g * hd + i);
        vs[i] = KVBF16 ? round_bf16(v) : v;
    }
    const int ctx_pad = p.chd * Fmt<WF>::EPC;
    for (int i = hd + threadIdx.x; i < ctx_pad; i += NT) ctx[i] = 0.0f;
    __syncthreads();
    if (!isfinite(qs[threadIdx.x % hd]) || !isfinite(ks[threadIdx.x % hd])) atomicOr(&p.ctrl->error, ERR_NONFINITE);
    const size_t esz = KVBF16 ? 2 : 4;
    const uint8_t *K = Ly.kc + (size_t)g * p.cap * hd * esz;
    const uint8_t *Vc = Ly.vc + (size_t)g * p.cap * hd * esz;
    if (sp == 0 && hh % p.group == 0) {
        for (int i = threadIdx.x; i < hd; i += NT) {
            size_t idx = (size_t)pos * hd + i;
            if (KVBF16) {
                ((uint16_t *)Ly.kc)[(size_t)g * p.cap * hd + idx] = f32_to_bf16_rne(ks[i]);
                ((uint16_t *)Ly.vc)[(size_t)g * p.cap * hd + idx] = f32_to_bf16_rne(vs[i]);
            } else {
                ((float *)Ly.kc)[(size_t)g * p.cap * hd + idx] = ks[i];
                ((float *)Ly.vc)[(size_t)g * p.cap * hd + idx] = vs[i];
            }
        }
    }
    // scores: q.k / sqrt(d), one position per thread, increasing i.
    for (int q = threadIdx.x; q <= pos; q += NT) {
        float s = 0.0f;
        if (q == pos) {
            for (int i = 0; i < hd; ++i) s = s + qs[i] * ks[i];
        } else {
            for (int i = 0; i < hd; ++i) s = s + qs[i] * kv_load<KVBF16>(K, (size_t)q * hd + i);
        }
        sc[q] = s / p.sqrt_hd;
    }
    __syncthreads();
    float m = -INFINITY;
    for (int q = threadIdx.x; q <= pos; q += NT) m = rust_max(m, sc[q]);
    m = block_max(m, red);
    float se = 0.0f;
    for (int q = threadIdx.x; q <= pos; q += NT) {
        float e = expf(sc[q] - m);
        sc[q] = e;
        se += e;
    }
    se = block_sum(se, red);
    for (int q = threadIdx.x; q <= pos; q += NT) sc[q] = sc[q] / se;
    __syncthreads();
    // context: thread (i, pg) sums positions pg, pg+PG, ... in order.
    const int PG = NT / hd > 0 ? NT / hd : 1;
    {
        const int i = threadIdx.x % hd, pg = threadIdx.x / hd;
        float acc = 0.0f;
        if (pg < PG && threadIdx.x < PG * hd) {
            for (int q = pg; q <= pos; q += PG) {
                float v = q == pos ? vs[i] : kv_load<KVBF16>(Vc, (size_t)q * hd + i);
                acc = acc + sc[q] * v;
            }
            part[pg * hd + i] = acc;
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < hd; i += NT) {
        float s = part[i];
        for (int k = 1; k < PG; ++k) s += part[k * hd + i];
        ctx[i] = s;
        flag_nonfinite(p.ctrl, s);
    }
    __syncthreads();
    // o_proj partial of this head for rows [r0, r1).
    const int r0 = (int)((long long)p.h * sp / p.s_o), r1 = (int)((long long)p.h * (sp + 1) / p.s_o);
    const uint8_t *wo = Ly.wo + (size_t)hh * p.h * p.shd;
    const float *so = Ly.so;
    float *outp = p.part + (size_t)hh * p.h;
    DecodeCtrl *ctrl = p.ctrl;
    const size_t shd = p.shd;
    cta_gemv<WF>([=](int r) { return wo + (size_t)(r0 + r) * shd; }, r1 - r0, p.chd, ctx, part,
                 p.part_cap, [=](int r, float v) {
                     if (WF == WF_I8) v = v * so[r0 + r];
                     outp[r0 + r] = v;
                     flag_nonfinite(ctrl, v);
                 });
}

template <int WF, int KVBF16>
__global__ void __launch_bounds__(NT, 1) decode_kernel(const __grid_constant__ DecodeParams p) {
    extern __shared__ __align__(16) float sm[];
    __shared__ int s_flag;
    float *xs = sm + p.sm_xs, *part = sm + p.sm_part, *h2 = sm + p.sm_h2, *gu = sm + p.sm_gu;
    float *red = sm + p.sm_red;
    const int G = gridDim.x, b = blockIdx.x;
    DecodeCtrl *ctrl = p.ctrl;
    const int token = *(volatile int *)&ctrl->token;
    const int pos = *(volatile int *)&ctrl->pos;
    constexpr int EPC = Fmt<WF>::EPC;
    unsigned target = 0;
    int phase = 0;
    prefetch_phase(p, 0, pos, b, G);
    prefetch_phase(p, 1, pos, b, G);

    for (int l = 0; l < p.L; ++l) {
        const DecodeLayer &Ly = p.layers[l];
        // ---------------- QKV ----------------
        prefetch_phase(p, phase + 2, pos, b, G);
        for (int i = threadIdx.x; i < p.h; i += NT) h2[i] = resid_in(p, l, token, i);
        __syncthreads();
        block_rmsnorm(h2, Ly.attn_norm, xs, p.h, p.ch * EPC, p.eps, red);
        {
            const int r0 = (int)((long long)p.rqkv * b / G), r1 = (int)((long long)p.rqkv * (b + 1) / G);
            const uint8_t *w = Ly.wqkv;
            const float *s = Ly.sqkv, *bias = Ly.bqkv;
            float *out = p.qkv;
            const size_t sh = p.sh;
            cta_gemv<WF>([=](int r) { return w + (size_t)(r0 + r) * sh; }, r1 - r0, p.ch, xs, part,
                         p.part_cap, [=](int r, float v) {
                             if (WF == WF_I8) v = v * s[r0 + r];
                             v = v + bias[r0 + r];
                             out[r0 + r] = v;
                             flag_nonfinite(ctrl, v);
                         });
        }
        target += G;
        ++phase;
        if (!grid_barrier(ctrl, target, p.timeout_ns, &s_flag)) return;
        // ---------------- ATTENTION + o_proj partials ----------------
        prefetch_phase(p, phase + 2, pos, b, G);
        for (int wi = b; wi < p.qh * p.s_o; wi += G) {
            attention_head<WF, KVBF16>(p, Ly, wi / p.s_o, wi % p.s_o, pos, sm);
            __syncthreads();
        }
        target += G;
        ++phase;
        if (!grid_barrier(ctrl, target, p.timeout_ns, &s_flag)) return;
        // ---------------- GATE / UP ----------------
        prefetch_phase(p, phase + 2, pos, b, G);
        for (int i = threadIdx.x; i < p.h; i += NT) {
            float v = after_attention(p, l, token, i);
            h2[i] = v;
            if (b == 0) flag_nonfinite(ctrl, v);
        }
        __syncthreads();
        block_rmsnorm(h2, Ly.ffn_norm, xs, p.h, p.ch * EPC, p.eps, red);
        {
            const int f0 = (int)((long long)p.ff * b / G), f1 = (int)((long long)p.ff * (b + 1) / G);
            const int R = f1 - f0;
            const uint8_t *wg = Ly.wg, *wu = Ly.wu;
            const size_t sh = p.sh;
            float *g = gu;
            cta_gemv<WF>(
                [=](int r) { return r < R ? wg + (size_t)(f0 + r) * sh : wu + (size_t)(f0 + r - R) * sh; },
                2 * R, p.ch, xs, part, p.part_cap, [=](int r, float v) { g[r] = v; });
            __syncthreads();
            for (int r = threadIdx.x; r < R; r += NT) {
                float gv = gu[r], uv = gu[R + r];
                if (WF == WF_I8) {
                    gv = gv * Ly.sg[f0 + r];
                    uv = uv * Ly.su[f0 + r];
                }
                float a = silu1(gv) * uv;
                p.act[f0 + r] = a;
                flag_nonfinite(ctrl, gv);
                flag_nonfinite(ctrl, a);
            }
        }
        target += G;
        ++phase;
        if (!grid_barrier(ctrl, target, p.timeout_ns, &s_flag)) return;
        // ---------------- DOWN ----------------
        prefetch_phase(p, phase + 2, pos, b, G);
        for (int i = threadIdx.x; i < p.cff * EPC; i += NT) xs[i] = i < p.ff ? ldcg(p.act + i) : 0.0f;
        __syncthreads();
        {
            const int r0 = (int)((long long)p.h * b / G), r1 = (int)((long long)p.h * (b + 1) / G);
            const uint8_t *w = Ly.wd;
            const float *s = Ly.sd;
            const size_t sff = p.sff;
            const int lay = l, tok = token;
            const DecodeParams *pp = &p;
            cta_gemv<WF>([=](int r) { return w + (size_t)(r0 + r) * sff; }, r1 - r0, p.cff, xs, part,
                         p.part_cap, [=](int r, float v) {
                             if (WF == WF_I8) v = v * s[r0 + r];
                             float o = after_attention(*pp, lay, tok, r0 + r) + v;
                             pp->hidden[r0 + r] = o;
                             flag_nonfinite(ctrl, o);
                         });
        }
        target += G;
        ++phase;
        if (!grid_barrier(ctrl, target, p.timeout_ns, &s_flag)) return;
    }

    // ---------------- LM HEAD + argmax ----------------
    for (int i = threadIdx.x; i < p.h; i += NT) h2[i] = ldcg(p.hidden + i);
    __syncthreads();
    const int tEPC = p.tfmt == WF_BF16 ? 8 : 4;
    block_rmsnorm(h2, p.final_norm, xs, p.h, p.cemb * tEPC, p.eps, red);
    const int v0 = (int)((long long)p.V * b / G), v1 = (int)((long long)p.V * (b + 1) / G);
    float best_v = -INFINITY;
    int best_i = 0x7fffffff;
    {
        const uint8_t *tab = p.head;
        const size_t semb = p.semb;
        float *logits = ctrl->write_logits ? p.logits : nullptr;
        float *bv = &best_v;
        int *bi = &best_i;
        auto emit = [=](int r, float v) {
            const int id = v0 + r;
            if (logits) logits[id] = v;
            flag_nonfinite(ctrl, v);
            if (v > *bv || (v == *bv && id < *bi)) { *bv = v; *bi = id; }
        };
        // Rows are streamed in blocks; each block prefetches the next into L2.
        const int R = v1 - v0, BLK = 256;
        for (int r0 = 0; r0 < R; r0 += BLK) {
            if (p.prefetch && threadIdx.x == 0 && r0 + BLK < R) {
                int n = min(BLK, R - r0 - BLK);
                prefetch_l2_bulk(tab + (size_t)(v0 + r0 + BLK) * semb, (uint32_t)((size_t)n * semb));
            }
            const int n = min(BLK, R - r0);
            const int base = v0 + r0;
            auto rowp = [=](int r) { return tab + (size_t)(base + r) * semb; };
            auto em = [=](int r, float v) { emit(r0 + r, v); };
            if (p.tfmt == WF_BF16) cta_gemv<WF_BF16>(rowp, n, p.cemb, xs, part, p.part_cap, em);
            else cta_gemv<WF_F32>(rowp, n, p.cemb, xs, part, p.part_cap, em);
        }
    }
    // CTA argmax over the warps' lane-0 bests (lowest id on ties).
    {
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
        int *redi = (int *)(red + 2 * NW + 4);
        __syncthreads();
        if (lane == 0) {
            red[warp] = best_v;
            redi[warp] = best_i;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            float bv = red[0];
            int bi = redi[0];
            for (int k = 1; k < NW; ++k)
                if (red[k] > bv || (red[k] == bv && redi[k] < bi)) { bv = red[k]; bi = redi[k]; }
            p.amax_v[b] = bv;
            p.amax_i[b] = bi;
            __threadfence();
            unsigned tk = atomicAdd(&ctrl->ticket, 1u);
            if (tk == (unsigned)G - 1) {
                __threadfence();
                float gv = __ldcg(p.amax_v);
                int gi = __ldcg(p.amax_i);
                for (int k = 1; k < G; ++k) {
                    float v = __ldcg(p.amax_v + k);
                    int i = __ldcg(p.amax_i + k);
                    if (v > gv || (v == gv && i < gi)) { gv = v; gi = i; }
                }
                if (gi < 0 || gi >= p.V) gi = 0;
                ctrl->next_token = gi;
                if (p.emitted) p.emitted[pos] = gi;
                ctrl->token = gi;
                ctrl->pos = pos + 1;
                ctrl->bar = 0;
                ctrl->ticket = 0;
                __threadfence();
            }
        }
    }
}

size_t decode_smem_bytes(const DecodeParams &p) { return (size_t)p.sm_total * sizeof(float); }

template <int WF, int KV>
static cudaError_t launch_t(const DecodeParams &p, int grid, cudaStream_t stream) {
    auto kern = decode_kernel<WF, KV>;
    size_t smem = decode_smem_bytes(p);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(NT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

cudaError_t decode_launch(const DecodeParams &p, int grid, cudaStream_t stream) {
    if (p.wfmt == WF_I8) return p.kv_bf16 ? launch_t<WF_I8, 1>(p, grid, stream) : launch_t<WF_I8, 0>(p, grid, stream);
    if (p.wfmt == WF_BF16) return p.kv_bf16 ? launch_t<WF_BF16, 1>(p, grid, stream) : launch_t<WF_BF16, 0>(p, grid, stream);
    return p.kv_bf16 ? launch_t<WF_F32, 1>(p, grid, stream) : launch_t<WF_F32, 0>(p, grid, stream);
}

// Largest number of co-resident CTAs of the decode kernel on this device.
int decode_max_ctas(int wfmt, int kv_bf16, size_t smem) {
    int dev = 0, sms = 0, per = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const void *f;
    if (wfmt == WF_I8) f = kv_bf16 ? (const void *)decode_kernel<WF_I8, 1> : (const void *)decode_kernel<WF_I8, 0>;
    else if (wfmt == WF_BF16) f = kv_bf16 ? (const void *)decode_kernel<WF_BF16, 1> : (const void *)decode_kernel<WF_BF16, 0>;
    else f = kv_bf16 ? (const void *)decode_kernel<WF_F32, 1> : (const void *)decode_kernel<WF_F32, 0>;
    if (cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, f, NT, smem) != cudaSuccess) return 0;
    return per * sms;
}

}  // namespace qb
