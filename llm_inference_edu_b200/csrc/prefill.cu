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
#include <atomic>
#include <vector>

#include "common.cuh"
#include "multitoken.cuh"
#include "prefill.cuh"
#include "tc_gemm.cuh"

namespace qb {
namespace {

using namespace mt;

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
    pdl_trigger();
    pdl_wait();
    for (int t = blockIdx.x; t < n; t += gridDim.x) {
        const uint8_t *row = emb + (size_t)ids[t] * semb;
        for (int i = threadIdx.x; i < h; i += blockDim.x)
            x[(size_t)t * h + i] =
                TF == WF_BF16 ? bf16_to_f32(((const uint16_t *)row)[i]) : ((const float *)row)[i];
    }
}

// Scaled RMSNorm of each row (src/ops.rs:137-149), one CTA per row; rows of
// up to 16 x blockDim elements stay in registers between the passes.
__global__ void rmsnorm_rows(const float *x, const float *g, float *y, Planes P, int n, int w, float eps,
                             unsigned *err) {
    pdl_trigger();
    pdl_wait();
    __shared__ float red[32];
    constexpr int VPT = 16;
    const float se = sqrtf(eps);
    for (int t = blockIdx.x; t < n; t += gridDim.x) {
        const float *xr = x + (size_t)t * w;
        float *yr = y + (size_t)t * w;
        if (w <= (int)blockDim.x * VPT) {
            float v[VPT];
            float m = se;
#pragma unroll
            for (int k = 0; k < VPT; ++k) {
                const int i = threadIdx.x + k * blockDim.x;
                v[k] = i < w ? xr[i] : 0.0f;
                if (i < w) m = rust_max(m, fabsf(v[k]));
            }
            m = block_max(m, red);
            float ss = 0.0f;
#pragma unroll
            for (int k = 0; k < VPT; ++k) {
                const float q = v[k] / m;
                if (threadIdx.x + k * blockDim.x < w) ss = ss + q * q;
            }
            ss = block_sum(ss, red);
            const float seps = se / m;
            const float den = sqrtf(ss / (float)w + seps * seps);
#pragma unroll
            for (int k = 0; k < VPT; ++k) {
                const int i = threadIdx.x + k * blockDim.x;
                if (i < w) {
                    const float o = (v[k] / m) / den * g[i];
                    yr[i] = o;
                    if (P.p) store_planes(P, (size_t)t * w + i, o);
                    flag_bad(err, o);
                }
            }
            continue;
        }
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
            yr[i] = o;
            if (P.p) store_planes(P, (size_t)t * w + i, o);
            flag_bad(err, o);
        }
    }
}

// The same RMSNorm with one warp per row (rows of w <= 1024 elements, w a
// multiple of 4): the row stays in registers and both reductions are warp
// shuffles, with no CTA barrier.  Eight rows per 256-thread CTA.  The two
// divisions per element become multiplications by the reciprocals of the
// row maximum and of the denominator (as in the decode kernel's RMSNorm:
// within a few ulps of the divisions).  A row maximum of 2^125 or more
// would make its reciprocal subnormal (lost precision), so such rows keep
// the division by the maximum; the denominator lies in [w^-1/2, 2^1/2],
// whose reciprocal is always normal.
__global__ void rmsnorm_rows_warp(const float *x, const float *g, float *y, Planes P, int n, int w, float eps,
                                  unsigned *err) {
    pdl_trigger();
    pdl_wait();
    constexpr int V4 = 8;  // float4 per lane: w <= 32 * 4 * 8
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= n) return;
    const float4 *xr = reinterpret_cast<const float4 *>(x + (size_t)t * w);
    const int w4 = w >> 2;
    const float se = sqrtf(eps);
    float4 v[V4];
    float m = se;
#pragma unroll
    for (int k = 0; k < V4; ++k) {
        const int i = lane + 32 * k;
        v[k] = i < w4 ? xr[i] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (i < w4)
            m = rust_max(rust_max(rust_max(rust_max(m, fabsf(v[k].x)), fabsf(v[k].y)), fabsf(v[k].z)), fabsf(v[k].w));
    }
    for (int off = 16; off; off >>= 1) m = rust_max(m, __shfl_xor_sync(0xffffffffu, m, off));
    const bool big = m >= 0x1p125f;  // warp-uniform
    const float r = 1.0f / m;
    if (big) {
#pragma unroll
        for (int k = 0; k < V4; ++k) {
            v[k].x = v[k].x / m; v[k].y = v[k].y / m; v[k].z = v[k].z / m; v[k].w = v[k].w / m;
        }
    } else {
#pragma unroll
        for (int k = 0; k < V4; ++k) {
            v[k].x = v[k].x * r; v[k].y = v[k].y * r; v[k].z = v[k].z * r; v[k].w = v[k].w * r;
        }
    }
    // v now holds x / m.
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < V4; ++k) {
        if (lane + 32 * k < w4) {
            const float a = v[k].x, b = v[k].y, c = v[k].z, d = v[k].w;
            ss = ss + a * a;
            ss = ss + b * b;
            ss = ss + c * c;
            ss = ss + d * d;
        }
    }
    for (int off = 16; off; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float seps = big ? se / m : se * r;
    const float rd = 1.0f / sqrtf(ss / (float)w + seps * seps);
    float4 *yr = reinterpret_cast<float4 *>(y + (size_t)t * w);
    const float4 *g4 = reinterpret_cast<const float4 *>(g);
#pragma unroll
    for (int k = 0; k < V4; ++k) {
        const int i = lane + 32 * k;
        if (i < w4) {
            const float4 gg = g4[i];
            float4 o;
            o.x = v[k].x * rd * gg.x;
            o.y = v[k].y * rd * gg.y;
            o.z = v[k].z * rd * gg.z;
            o.w = v[k].w * rd * gg.w;
            yr[i] = o;
            if (P.p) {
                const size_t at = (size_t)t * w + 4 * (size_t)i;
                store_planes(P, at, o.x);
                store_planes(P, at + 1, o.y);
                store_planes(P, at + 2, o.z);
                store_planes(P, at + 3, o.w);
            }
            flag_bad(err, o.x);
            flag_bad(err, o.y);
            flag_bad(err, o.z);
            flag_bad(err, o.w);
        }
    }
}

// Row RMSNorm launch: the warp-per-row kernel when the row fits it.
cudaError_t rmsnorm(const float *x, const float *g, float *y, Planes P, int n, int w, float eps, unsigned *err,
                    cudaStream_t st) {
    if (w % 4 == 0 && w <= 32 * 4 * 8 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)y & 15) == 0 &&
        ((uintptr_t)g & 15) == 0)
        return launch_pdl(rmsnorm_rows_warp, dim3((n + 7) / 8), dim3(256), 0, st, x, g, y, P, n, w, eps, err);
    return launch_pdl(rmsnorm_rows, dim3(std::min(n, 4096)), dim3(256), 0, st, x, g, y, P, n, w, eps, err);
}

// ----------------------------------------------------------------- gemm ----
//
// Y[t][r] = epilogue(sum_k X[t][k] W[r][k]) for t < n tokens and r < N rows,
// FP32 products and accumulation.  W is the decode layout: row r, segment
// s (of seg_len elements) starts at base + s * seg_stride + r * row_stride,
// so the head-blocked o_proj is one segmented matrix.  K, seg_len and every
// leading dimension are multiples of 4.

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

// grid.z = ksplit slices of K (each kper elements, a multiple of BK).  With
// ksplit > 1 the raw sums go to part[z][t][r] and reduce_epilogue finishes.
template <int WF, int EPI>
__global__ void __launch_bounds__(256) gemm_rows(const float *X, int ldx, int n, int N, int K, GemmW w,
                                                 const float *R, int ldr, float *Y, int ldy, Planes P,
                                                 unsigned *err, int kper, float *part) {
    pdl_trigger();
    pdl_wait();
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
                if (r + 1 < N) epilogue_gu(w, t, r, acc[i][2 * jj], acc[i][2 * jj + 1], Y, ldy, P, err);
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

// ----------------------------------------------------------- skinny GEMM ----
//
// Y[t][r] = epilogue(sum_k X[t][k] W[r][k]) for n <= GV_MAXT tokens (batched
// decode of a few sequences, a tensor-parallel rank's batch-1 step): an
// HBM-bound streaming kernel with no tensor-core setup.  Each warp owns two
// adjacent rows (the gate/up pairs, or two rows sharing the activation
// reads); its lanes stride the rows' 16-byte chunks and multiply each with
// the same K elements of all n tokens, staged in shared memory one K tile at
// a time.  Every weight byte is read
// once per call with streaming loads; the first tile's weights are loaded
// before the dependent-launch wait (they do not depend on earlier kernels).
constexpr int GV_WARPS = 8, GV_MAXT = 1, GV_TILE_BYTES = 2048;  // measured: two tokens already favour the tensor cores

template <int WF>
__device__ __forceinline__ const uint8_t *gv_chunk(const GemmW &w, int r, int k) {
    constexpr int ESZ = WF == WF_I8 ? 1 : (WF == WF_BF16 ? 2 : 4);
    const int s = k / w.seg_len, kk = k - s * w.seg_len;
    return w.base + (size_t)s * w.seg_stride + (size_t)r * w.row_stride + (size_t)kk * ESZ;
}

// acc[t] += sum_e x_t[e] * w[e] over one 16-byte chunk of weights.  The
// tile's inputs are quad-major: quad q of chunk c of token t is float4
// (t * Q + q) * CT + c, so lanes reading consecutive chunks read
// consecutive 16-byte words (no bank conflicts).
template <int WF, int NT>
__device__ __forceinline__ void gv_dot(const uint4 &c, const float4 *xs4, int ch, int CT, int n, float *acc) {
    constexpr int EPC = WF == WF_I8 ? 16 : (WF == WF_BF16 ? 8 : 4);
    float wv[EPC];
    const uint32_t u[4] = {c.x, c.y, c.z, c.w};
    if (WF == WF_I8) {
#pragma unroll
        for (int e = 0; e < 16; ++e) wv[e] = u8b_to_f32(u[e >> 2], e & 3);
    } else if (WF == WF_BF16) {
#pragma unroll
        for (int e = 0; e < 8; ++e) wv[e] = (e & 1) ? bf16_hi(u[e >> 1]) : bf16_lo(u[e >> 1]);
    } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) wv[e] = __uint_as_float(u[e]);
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        if (t >= n) break;
#pragma unroll
        for (int q = 0; q < EPC / 4; ++q) {
            const float4 x = xs4[((size_t)t * (EPC / 4) + q) * CT + ch];
            acc[t] = fmaf(x.x, wv[4 * q], acc[t]);
            acc[t] = fmaf(x.y, wv[4 * q + 1], acc[t]);
            acc[t] = fmaf(x.z, wv[4 * q + 2], acc[t]);
            acc[t] = fmaf(x.w, wv[4 * q + 3], acc[t]);
        }
    }
}

template <int WF, int EPI, int NT>
__global__ void __launch_bounds__(GV_WARPS * 32) gemv_tokens(const float *X, int ldx, int n, int N, int K, GemmW w,
                                                             const float *R, int ldr, float *Y, int ldy, Planes P,
                                                             unsigned *err) {
    constexpr int EPC = WF == WF_I8 ? 16 : (WF == WF_BF16 ? 8 : 4);
    constexpr int KT = GV_TILE_BYTES / 16 * EPC;   // elements per tile
    constexpr int CT = GV_TILE_BYTES / 16;         // chunks per row and tile
    constexpr int CPL = CT / 32;                     // chunks per lane per row and tile
    constexpr int Q = EPC / 4;                       // quads per chunk
    constexpr int RW = 2;                            // rows per warp
    extern __shared__ __align__(16) float xs[];    // [NT][KT]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r0 = (blockIdx.x * GV_WARPS + warp) * RW;
    const bool live = r0 < N;
    float acc[RW][NT];
#pragma unroll
    for (int i = 0; i < RW; ++i)
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[i][t] = 0.0f;
    uint4 wc[RW][CPL];
    auto load_tile = [&](int k0) {
#pragma unroll
        for (int i = 0; i < RW; ++i)
#pragma unroll
            for (int j = 0; j < CPL; ++j) {
                const int k = k0 + (lane + 32 * j) * EPC;
                wc[i][j] = live && r0 + i < N && k < K ? ld_stream_u4(gv_chunk<WF>(w, r0 + i, k))
                                                       : make_uint4(0u, 0u, 0u, 0u);
            }
    };
    load_tile(0);
    pdl_wait();
    for (int k0 = 0; k0 < K; k0 += KT) {
        // Stage the tokens' K elements [k0, k0 + KT) quad-major (zero past K).
        float4 *xs4 = reinterpret_cast<float4 *>(xs);
        for (int f = threadIdx.x; f < NT * (KT / 4); f += GV_WARPS * 32) {
            const int t = f / (KT / 4), g = f - t * (KT / 4), c = g / Q, q = g - c * Q;
            float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (t < n && k0 + 4 * g < K) v = *reinterpret_cast<const float4 *>(X + (size_t)t * ldx + k0 + 4 * g);
            xs4[((size_t)t * Q + q) * CT + c] = v;
        }
        __syncthreads();
        uint4 cur[RW][CPL];
#pragma unroll
        for (int i = 0; i < RW; ++i)
#pragma unroll
            for (int j = 0; j < CPL; ++j) cur[i][j] = wc[i][j];
        if (k0 + KT < K) load_tile(k0 + KT);  // the next tile's weights in flight
#pragma unroll
        for (int i = 0; i < RW; ++i)
#pragma unroll
            for (int j = 0; j < CPL; ++j) {
                const int ch = lane + 32 * j;
                if (k0 + ch * EPC < K) gv_dot<WF, NT>(cur[i][j], xs4, ch, CT, n, acc[i]);
            }
        __syncthreads();
    }
    // The next kernel may launch now: a dependent grid scheduled earlier would
    // hold SM slots that this grid's later waves still need.
    pdl_trigger();
    // Butterfly sums; lane t runs token t's epilogue.
#pragma unroll
    for (int i = 0; i < RW; ++i)
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
            for (int off = 16; off; off >>= 1) acc[i][t] += __shfl_xor_sync(0xffffffffu, acc[i][t], off);
    if (!live) return;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        if (lane != t || t >= n) continue;
        if (EPI == EPI_GU) {
            if (r0 + 1 < N) epilogue_gu(w, t, r0, acc[0][t], acc[1][t], Y, ldy, P, err);
        } else {
            epilogue1<EPI>(w, t, r0, acc[0][t], R, ldr, Y, ldy, err);
            if (r0 + 1 < N) epilogue1<EPI>(w, t, r0 + 1, acc[1][t], R, ldr, Y, ldy, err);
        }
    }
}

template <int WF, int EPI>
cudaError_t gemv(const float *X, int ldx, int n, int N, int K, const GemmW &w, const float *R, int ldr, float *Y,
                 int ldy, const Planes &P, unsigned *err, cudaStream_t st) {
    constexpr int EPC = WF == WF_I8 ? 16 : (WF == WF_BF16 ? 8 : 4);
    constexpr int KT = GV_TILE_BYTES / 16 * EPC, RW = 2;
    const int rows = GV_WARPS * RW;
    const dim3 grid((N + rows - 1) / rows);
    auto go = [&](auto kern, int nt) -> cudaError_t {
        const size_t sm = (size_t)nt * KT * sizeof(float);
        if (sm > 48 * 1024) {
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
            if (e != cudaSuccess) return e;
        }
        return launch_pdl(kern, grid, dim3(GV_WARPS * 32), sm, st, X, ldx, n, N, K, w, R, ldr, Y, ldy, P, err);
    };
    if (n <= 1) return go(gemv_tokens<WF, EPI, 1>, 1);
    if (n <= 2) return go(gemv_tokens<WF, EPI, 2>, 2);
    return go(gemv_tokens<WF, EPI, 4>, 4);
}

// -------------------------------------------------------------- attention ----

// RoPE of every query and key head of each token (at its own position) with
// the host table, in place, and the K (rotated) and V write into its
// sequence's cache -- BF16 round-to-nearest-even when the cache is BF16.
__global__ void rope_kv(float *qkv, int n, const int *pos, const int *seqs, int l, int h, int qh, int kvh, int hd,
                        const float2 *rope, KvPages kv, int kv_bf16, unsigned *err) {
    pdl_trigger();
    pdl_wait();
    const int half = hd / 2, rq = h + 2 * kvh * hd;
    for (int t = blockIdx.x; t < n; t += gridDim.x) {
        const int p = pos[t];
        uint8_t *kc = kv.k(l), *vc = kv.v(l);
        float *row = qkv + (size_t)t * rq;
        const float2 *rp = rope + (size_t)p * half;
        const int i0 = blockIdx.y * blockDim.x + threadIdx.x, istep = gridDim.y * blockDim.x;
        for (int idx = i0; idx < qh * half; idx += istep) {
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
        for (int idx = i0; idx < kvh * half; idx += istep) {
            const int g = idx / half, j = idx - g * half;
            const float *k = row + h + (size_t)g * hd;
            const float2 cs = rp[j];
            const float a = k[j], b = k[j + half];
            const float k0 = a * cs.x - b * cs.y, k1 = b * cs.x + a * cs.y;
            flag_bad(err, k0);
            flag_bad(err, k1);
            const size_t base = kv.row(seqs[t], g, p);
            if (kv_bf16) {
                ((uint16_t *)kc)[base + j] = f32_to_bf16_rne(k0);
                ((uint16_t *)kc)[base + j + half] = f32_to_bf16_rne(k1);
            } else {
                ((float *)kc)[base + j] = k0;
                ((float *)kc)[base + j + half] = k1;
            }
        }
        for (int idx = i0; idx < kvh * hd; idx += istep) {
            const int g = idx / hd, i = idx - g * hd;
            const float v = row[h + (size_t)kvh * hd + (size_t)g * hd + i];
            const size_t at = kv.row(seqs[t], g, p) + i;
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
                               int qh, int kvh, int hd, int group, KvPages kv, float sqrt_hd, float *ctx, Planes P,
                               unsigned *err) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ float asm_[];
    const int t = blockIdx.x / qh, hh = blockIdx.x - t * qh, g = hh / group, p = pos[t];
    const int rq = h + 2 * kvh * hd;
    const uint8_t *kc = kv.k(l), *vc = kv.v(l);
    const int sq = seqs[t];
    float *qs = asm_, *sc = qs + hd, *red = sc + (max_pos + 1);
    for (int i = threadIdx.x; i < hd; i += blockDim.x) qs[i] = qkv[(size_t)t * rq + (size_t)hh * hd + i];
    __syncthreads();
    float m = -INFINITY;
    for (int q = threadIdx.x; q <= p; q += blockDim.x) {
        const size_t row = kv.row(sq, g, q);
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
        for (int q = 0; q <= p; ++q) acc = acc + (sc[q] / se) * kv_at<KVBF16>(vc, kv.row(sq, g, q) + i);
        ctx[(size_t)t * h + (size_t)hh * hd + i] = acc;
        if (P.p) store_planes(P, (size_t)t * h + (size_t)hh * hd + i, acc);
        flag_bad(err, acc);
    }
}

// Grouped-query attention, one CTA per (token, KV head, position split):
// the G <= 8 query heads sharing a KV head are served by one pass over its
// K and V rows.  Per query head, as the reference (src/kv_cache.rs:555-575):
// scores q.k / sqrt(hd) with the dot by increasing index, softmax with the
// maximum subtracted and each weight divided by the sum, and the context as
// the weighted sum of V rows.  Scores: one lane per position (the K row in
// registers, q broadcast from shared memory).  Context: each warp sums a
// contiguous run of positions in order (one lane per hd/32 dimensions);
// the warps' sums are added in warp order.  A split covers at most AT_SPAN
// positions; with several splits each writes its maximum, sum and
// unnormalized context and attn_combine merges them (rescaled by
// exp(m_z - m)).
constexpr int AT_THREADS = 256, AT_WARPS = AT_THREADS / 32, AT_SPAN = 1024, AT_GMAX = 8;

size_t attn_gqa_smem(int G, int hd, int span) {
    return ((size_t)G * hd + (size_t)G * span + (size_t)AT_WARPS * G * hd + 2 * AT_GMAX) * sizeof(float);
}

// Eight consecutive cache elements as FP32.
template <int KVBF16>
__device__ __forceinline__ void kv_load8(const uint8_t *base, size_t idx, float (&f)[8]) {
    if (KVBF16) {
        const uint4 v = *(const uint4 *)(base + idx * 2);
        f[0] = bf16_lo(v.x); f[1] = bf16_hi(v.x); f[2] = bf16_lo(v.y); f[3] = bf16_hi(v.y);
        f[4] = bf16_lo(v.z); f[5] = bf16_hi(v.z); f[6] = bf16_lo(v.w); f[7] = bf16_hi(v.w);
    } else {
        const float4 a = *(const float4 *)(base + idx * 4), b = *(const float4 *)(base + idx * 4 + 16);
        f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
    }
}

template <int KVBF16, int HD>
__global__ void __launch_bounds__(AT_THREADS)
    attn_gqa(const float *qkv, const int *pos, const int *seqs, int l, int h, int kvh, int G, KvPages kv,
             float sqrt_hd, int span, float *ctx, Planes P, float *apart, unsigned *err) {
    pdl_trigger();
    pdl_wait();
    constexpr int DPL = HD / 32;  // context dimensions per lane
    extern __shared__ float asm_[];
    const int t = blockIdx.x, g = blockIdx.y, z = blockIdx.z, nz = gridDim.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int lo = z * span, cnt = max(0, min(pos[t] + 1, lo + span) - lo);
    const int rq = h + 2 * kvh * HD;
    float *qs = asm_, *sc = qs + G * HD, *wsum = sc + (size_t)G * span, *red = wsum + AT_WARPS * G * HD;
    const uint8_t *kc = kv.k(l), *vc = kv.v(l);
    const int sq = seqs[t];
    for (int i = tid; i < G * HD; i += AT_THREADS) qs[i] = qkv[(size_t)t * rq + (size_t)g * G * HD + i];
    __syncthreads();
    // Scores: lane per position.
    for (int q = tid; q < cnt; q += AT_THREADS) {
        float s[AT_GMAX];
#pragma unroll
        for (int gi = 0; gi < AT_GMAX; ++gi) s[gi] = 0.0f;
        const size_t krow = kv.row(sq, g, lo + q);
#pragma unroll 2
        for (int i0 = 0; i0 < HD; i0 += 8) {
            float k8[8];
            kv_load8<KVBF16>(kc, krow + i0, k8);
#pragma unroll
            for (int gi = 0; gi < AT_GMAX; ++gi) {
                if (gi < G) {
                    const float4 qa = *(const float4 *)(qs + gi * HD + i0);
                    const float4 qb = *(const float4 *)(qs + gi * HD + i0 + 4);
                    float a = s[gi];
                    a = a + qa.x * k8[0]; a = a + qa.y * k8[1]; a = a + qa.z * k8[2]; a = a + qa.w * k8[3];
                    a = a + qb.x * k8[4]; a = a + qb.y * k8[5]; a = a + qb.z * k8[6]; a = a + qb.w * k8[7];
                    s[gi] = a;
                }
            }
        }
#pragma unroll
        for (int gi = 0; gi < AT_GMAX; ++gi)
            if (gi < G) sc[(size_t)gi * span + q] = s[gi] / sqrt_hd;
    }
    __syncthreads();
    // Softmax of each head (one warp per head).
    for (int gi = warp; gi < G; gi += AT_WARPS) {
        float *row = sc + (size_t)gi * span;
        float mx = -INFINITY;
        for (int q = lane; q < cnt; q += 32) mx = rust_max(mx, row[q]);
        for (int off = 16; off; off >>= 1) mx = rust_max(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        float se = 0.0f;
        for (int q = lane; q < cnt; q += 32) {
            const float e = expf(row[q] - mx);
            row[q] = e;
            se += e;
        }
        for (int off = 16; off; off >>= 1) se += __shfl_xor_sync(0xffffffffu, se, off);
        if (nz == 1)
            for (int q = lane; q < cnt; q += 32) row[q] = row[q] / se;
        if (lane == 0) {
            red[gi] = mx;
            red[AT_GMAX + gi] = se;
        }
    }
    __syncthreads();
    // Context: warp w sums positions [w * per, (w + 1) * per) in order.
    float acc[AT_GMAX][DPL];
#pragma unroll
    for (int gi = 0; gi < AT_GMAX; ++gi)
#pragma unroll
        for (int d = 0; d < DPL; ++d) acc[gi][d] = 0.0f;
    const int per = (cnt + AT_WARPS - 1) / AT_WARPS, q0 = warp * per, q1 = min(cnt, q0 + per);
#pragma unroll 4
    for (int q = q0; q < q1; ++q) {
        float v[DPL];
        const size_t at = kv.row(sq, g, lo + q) + lane * DPL;
#pragma unroll
        for (int d = 0; d < DPL; ++d) v[d] = kv_at<KVBF16>(vc, at + d);
#pragma unroll
        for (int gi = 0; gi < AT_GMAX; ++gi) {
            if (gi < G) {
                const float w = sc[(size_t)gi * span + q];
#pragma unroll
                for (int d = 0; d < DPL; ++d) acc[gi][d] = acc[gi][d] + w * v[d];
            }
        }
    }
#pragma unroll
    for (int gi = 0; gi < AT_GMAX; ++gi)
        if (gi < G)
#pragma unroll
            for (int d = 0; d < DPL; ++d) wsum[((size_t)warp * G + gi) * HD + lane * DPL + d] = acc[gi][d];
    __syncthreads();
    for (int task = tid; task < G * HD; task += AT_THREADS) {
        float o = wsum[task];
        for (int w = 1; w < AT_WARPS; ++w) o = o + wsum[(size_t)w * G * HD + task];
        const int gi = task / HD, i = task - gi * HD;
        if (nz == 1) {
            const size_t at = (size_t)t * h + ((size_t)g * G + gi) * HD + i;
            ctx[at] = o;
            if (P.p) store_planes(P, at, o);
            flag_bad(err, o);
        } else {
            float *pp = apart + (((size_t)t * kvh + g) * nz + z) * G * (HD + 2) + (size_t)gi * (HD + 2);
            pp[i] = o;
            if (i == 0) {
                pp[HD] = red[gi];
                pp[HD + 1] = red[AT_GMAX + gi];
            }
        }
    }
}

// Merges the position splits of attn_gqa: m = max m_z, L = sum l_z e^(m_z - m),
// context = sum o_z e^(m_z - m) / L.  One CTA per (token, KV head).
__global__ void attn_combine(const float *apart, int nz, int h, int kvh, int hd, int G, float *ctx, Planes P,
                             unsigned *err) {
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.x, g = blockIdx.y;
    const float *base = apart + ((size_t)t * kvh + g) * nz * G * (hd + 2);
    for (int task = threadIdx.x; task < G * hd; task += blockDim.x) {
        const int gi = task / hd, i = task - gi * hd;
        float m = -INFINITY;
        for (int z = 0; z < nz; ++z) m = rust_max(m, base[((size_t)z * G + gi) * (hd + 2) + hd]);
        float L = 0.0f, o = 0.0f;
        for (int z = 0; z < nz; ++z) {
            const float *pp = base + ((size_t)z * G + gi) * (hd + 2);
            const float f = pp[hd + 1] > 0.0f ? expf(pp[hd] - m) : 0.0f;
            L += pp[hd + 1] * f;
            o += pp[i] * f;
        }
        const float v = o / L;
        const size_t at = (size_t)t * h + ((size_t)g * G + gi) * hd + i;
        ctx[at] = v;
        if (P.p) store_planes(P, at, v);
        flag_bad(err, v);
    }
}

// Greedy id of each logits row: strict > over increasing ids keeps the
// lowest id among equal maxima (src/sampling.rs:65-70).
__global__ void argmax_rows(const float *logits, int n, int V, uint32_t *out, unsigned *err) {
    pdl_trigger();
    pdl_wait();
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

// Greedy id of each token from the LM head's per-tile partials (tiles are
// disjoint id ranges; ties keep the lowest id).  One warp per token.
__global__ void argmax_tiles(const float *amv, const int *ami, int tiles, int n, int V, uint32_t *out) {
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.x, lane = threadIdx.x;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int k = lane; k < tiles; k += 32) {
        const float v = amv[(size_t)k * n + t];
        const int i = ami[(size_t)k * n + t];
        if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
    }
    for (int off = 16; off; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) out[t] = bi >= 0 && bi < V ? (uint32_t)bi : 0u;
}

__global__ void advance_kernel(const uint32_t *amax, uint32_t *ids, int *pos, int n) {
    pdl_trigger();
    pdl_wait();
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
                 int ldr, float *Y, int ldy, const Planes &P, cudaStream_t st) {
    const int ks = choose_split(n, N, K, a.part_floats);
    const int kper = ((K + ks - 1) / ks + BK - 1) / BK * BK;
    const int ksn = (K + kper - 1) / kper;
    dim3 grid((N + BN - 1) / BN, (n + BM - 1) / BM, ksn);
    cudaError_t e = launch_pdl(gemm_rows<WF, EPI>, grid, dim3(256), 0, st, X, ldx, n, N, K, w, R, ldr, Y, ldy, P, a.err,
                               kper, a.part);
    if (e != cudaSuccess) return e;
    if (ksn > 1) {
        const size_t total = (size_t)n * N / (EPI == EPI_GU ? 2 : 1);
        const unsigned blocks = (unsigned)std::min<size_t>((total + 255) / 256, 4096);
        return launch_pdl(reduce_epilogue<EPI>, dim3(blocks), dim3(256), 0, st, a.part, ksn, n, N, w, R, ldr, Y, ldy, P,
                          a.err);
    }
    return cudaGetLastError();
}

Planes xn_planes(const PrefillArgs &a) { return Planes{a.xnp, (size_t)a.chunk * a.h, TC_NP}; }
Planes ctx_planes(const PrefillArgs &a) { return Planes{a.ctxp, (size_t)a.chunk * a.qd, TC_NP}; }
Planes act_planes(const PrefillArgs &a) { return Planes{a.actp, (size_t)a.chunk * a.ff, TC_NP}; }

// The four GEMMs of a layer: 0 QKV (+ bias), 1 o_proj (head-blocked K) +
// residual, 2 (gate, up) pairs -> SwiGLU, 3 down + residual.  With `part`
// set, 1 and 3 write this rank's scaled partial sums there instead (no
// residual; the tensor-parallel sum adds it).
template <int WF>
cudaError_t layer_gemm(int which, const PrefillArgs &a, const DecodeLayer &Ly, int n, float *part, cudaStream_t st) {
    const int kv = a.kvh * a.hd, rq = a.qd + 2 * kv;
    const Planes none{nullptr, 0, TC_NP};
    switch (which) {
    case 0: {
        GemmW w{Ly.wqkv, a.sh, 0, a.h, Ly.sqkv, Ly.bqkv};
        return gemm<WF, EPI_QKV>(a, a.xn, a.h, n, rq, a.h, w, nullptr, 0, a.qkv, rq, none, st);
    }
    case 1: {
        GemmW w{Ly.wo, a.shd, (size_t)a.h * a.shd, a.hd, Ly.so, nullptr};
        if (part) return gemm<WF, EPI_QKV>(a, a.ctx, a.qd, n, a.h, a.qd, w, nullptr, 0, part, a.h, none, st);
        return gemm<WF, EPI_RESID>(a, a.ctx, a.qd, n, a.h, a.qd, w, a.x, a.h, a.h2, a.h, none, st);
    }
    case 2: {
        GemmW w{Ly.wgu, a.sh, 0, a.h, Ly.sgu, nullptr};
        return gemm<WF, EPI_GU>(a, a.xn, a.h, n, 2 * a.ff, a.h, w, nullptr, 0, a.act, a.ff, act_planes(a), st);
    }
    default: {
        GemmW w{Ly.wd, a.sff, 0, a.ff, Ly.sd, nullptr};
        if (part) return gemm<WF, EPI_QKV>(a, a.act, a.ff, n, a.h, a.ff, w, nullptr, 0, part, a.h, none, st);
        return gemm<WF, EPI_RESID>(a, a.act, a.ff, n, a.h, a.ff, w, a.h2, a.h, a.x, a.h, none, st);
    }
    }
}

// A few tokens (INT8 or BF16 linears) take the streaming skinny GEMM
// instead of the tensor-core or register-tiled GEMM.
bool use_gemv(const PrefillArgs &a, int n) { return n <= GV_MAXT && (a.wfmt == WF_I8 || a.wfmt == WF_BF16); }

// The four GEMMs of a layer on the skinny path (the same epilogues as
// layer_gemm).
template <int WF>
cudaError_t layer_gemv(int which, const PrefillArgs &a, const DecodeLayer &Ly, int n, float *part, cudaStream_t st) {
    const int kv = a.kvh * a.hd, rq = a.qd + 2 * kv;
    const Planes none{nullptr, 0, TC_NP};
    switch (which) {
    case 0:
        return gemv<WF, EPI_QKV>(a.xn, a.h, n, rq, a.h, GemmW{Ly.wqkv, a.sh, 0, a.h, Ly.sqkv, Ly.bqkv}, nullptr, 0,
                                 a.qkv, rq, none, a.err, st);
    case 1: {
        const GemmW w{Ly.wo, a.shd, (size_t)a.h * a.shd, a.hd, Ly.so, nullptr};
        if (part) return gemv<WF, EPI_QKV>(a.ctx, a.qd, n, a.h, a.qd, w, nullptr, 0, part, a.h, none, a.err, st);
        return gemv<WF, EPI_RESID>(a.ctx, a.qd, n, a.h, a.qd, w, a.x, a.h, a.h2, a.h, none, a.err, st);
    }
    case 2:
        return gemv<WF, EPI_GU>(a.xn, a.h, n, 2 * a.ff, a.h, GemmW{Ly.wgu, a.sh, 0, a.h, Ly.sgu, nullptr}, nullptr, 0,
                                a.act, a.ff, none, a.err, st);
    default: {
        const GemmW w{Ly.wd, a.sff, 0, a.ff, Ly.sd, nullptr};
        if (part) return gemv<WF, EPI_QKV>(a.act, a.ff, n, a.h, a.ff, w, nullptr, 0, part, a.h, none, a.err, st);
        return gemv<WF, EPI_RESID>(a.act, a.ff, n, a.h, a.ff, w, a.h2, a.h, a.x, a.h, none, a.err, st);
    }
    }
}

// RoPE and the KV write run in the QKV GEMM's epilogue when that GEMM is on
// the tensor cores and the RoPE partner rows (r ^ hd/2) share a 128-row tile.
bool rope_fused(const PrefillArgs &a, int n) {
    return a.tc && !a.tc->layers.empty() && (a.hd == 64 || a.hd == 128) && !use_gemv(a, n);
}

// The same GEMMs on the tensor cores (weights in the layer's tensor maps,
// inputs as BF16 planes).
cudaError_t layer_gemm_tc(int which, const PrefillArgs &a, int l, int n, float *part, cudaStream_t st) {
    const DecodeLayer &Ly = a.layers[l];
    const TcLayerMaps &M = a.tc->layers[l];
    const int kv = a.kvh * a.hd, rq = a.qd + 2 * kv;
    const Planes none{nullptr, 0, TC_NP};
    TcJob j;
    RopeKv rk;
    switch (which) {
    case 0:
        j = TcJob{EPI_QKV, n, rq, a.h, &M.qkv, &a.tc->xn, GemmW{nullptr, 0, 0, 0, Ly.sqkv, Ly.bqkv},
                  nullptr, 0, a.qkv, rq, none};
        if (rope_fused(a, n)) {
            rk = RopeKv{a.pos, a.seq, a.rope, a.kv, l, a.qd, a.kvh, a.hd, a.kv_bf16};
            j.rk = &rk;
        }
        break;
    case 1:
        j = part ? TcJob{EPI_QKV, n, a.h, a.qd, &M.o, &a.tc->ctx, GemmW{nullptr, 0, 0, 0, Ly.so, nullptr},
                         nullptr, 0, part, a.h, none}
                 : TcJob{EPI_RESID, n, a.h, a.qd, &M.o, &a.tc->ctx, GemmW{nullptr, 0, 0, 0, Ly.so, nullptr},
                         a.x, a.h, a.h2, a.h, none};
        break;
    case 2:
        j = TcJob{EPI_GU, n, 2 * a.ff, a.h, &M.gu, &a.tc->xn, GemmW{nullptr, 0, 0, 0, Ly.sgu, nullptr},
                  nullptr, 0, a.act, a.ff, act_planes(a)};
        break;
    default:
        j = part ? TcJob{EPI_QKV, n, a.h, a.ff, &M.down, &a.tc->act, GemmW{nullptr, 0, 0, 0, Ly.sd, nullptr},
                         nullptr, 0, part, a.h, none}
                 : TcJob{EPI_RESID, n, a.h, a.ff, &M.down, &a.tc->act, GemmW{nullptr, 0, 0, 0, Ly.sd, nullptr},
                         a.h2, a.h, a.x, a.h, none};
    }
    return tc_gemm(j, a.err, st);
}

cudaError_t run_gemm(int which, const PrefillArgs &a, int l, int n, cudaStream_t st, float *part = nullptr) {
    if (use_gemv(a, n)) {
        if (a.wfmt == WF_I8) return layer_gemv<WF_I8>(which, a, a.layers[l], n, part, st);
        return layer_gemv<WF_BF16>(which, a, a.layers[l], n, part, st);
    }
    if (a.tc && !a.tc->layers.empty()) return layer_gemm_tc(which, a, l, n, part, st);
    const DecodeLayer &Ly = a.layers[l];
    if (a.wfmt == WF_I8) return layer_gemm<WF_I8>(which, a, Ly, n, part, st);
    if (a.wfmt == WF_BF16) return layer_gemm<WF_BF16>(which, a, Ly, n, part, st);
    return layer_gemm<WF_F32>(which, a, Ly, n, part, st);
}

// o_proj (which 1) or down (3) with the tensor-parallel sum: this rank's
// partial sums into its exchange slot for the next call, then the sum over
// the ranks plus the residual (R + sum of partials in rank order -> Y).
cudaError_t run_gemm_tp(int which, const PrefillArgs &a, int l, int n, const float *R, float *Y, cudaStream_t st) {
    const unsigned q = ++*a.tp_seq;
    float *part = a.tp->part[a.tp->rank] + (size_t)(q & 1u) * a.tp->rows * a.h;
    cudaError_t e = run_gemm(which, a, l, n, st, part);
    if (e != cudaSuccess) return e;
    return tp_allreduce(*a.tp, q, n, R, Y, a.err, a.tp_timeout_ns, st);
}

size_t attention_smem(const PrefillArgs &a, int max_pos) { return ((size_t)a.hd + max_pos + 1 + 32) * sizeof(float); }

bool gqa_supported(const PrefillArgs &a) { return a.group <= AT_GMAX && (a.hd == 64 || a.hd == 128); }

// Position splits for the grouped-query kernel: enough that one split
// covers at most AT_SPAN positions, more (each at least 256 positions) while
// the (token, KV head) pairs leave SMs idle, bounded by the partial buffer.
int attention_splits(const PrefillArgs &a, int n, int max_pos, int *span) {
    const int len = max_pos + 1;
    int nz = (len + AT_SPAN - 1) / AT_SPAN;
    const int want = (2 * 148 + n * a.kvh - 1) / (n * a.kvh);
    nz = std::max(nz, std::min(want, n <= GV_MAXT ? (len + 63) / 64 : (len + 255) / 256));
    const size_t per = (size_t)a.group * (a.hd + 2);
    while (nz > 1 && (size_t)n * a.kvh * nz * per > a.apart_floats) --nz;
    int sp = (len + nz - 1) / nz;
    sp = (sp + 63) / 64 * 64;
    *span = sp;
    return (len + sp - 1) / sp;
}

cudaError_t attention(const PrefillArgs &a, int n, int l, int max_pos, cudaStream_t st) {
    if (gqa_supported(a) && a.apart) {
        int span = 0;
        const int nz = attention_splits(a, n, max_pos, &span);
        if (span <= AT_SPAN) {
            const size_t sm = attn_gqa_smem(a.group, a.hd, span);
            // Attribute set once per (instantiation, device): bit `which` of
            // the device's mask.
            static std::atomic<unsigned> configured[64];
            int dev = 0;
            if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
            const int which = a.kv_bf16 * 2 + (a.hd == 128);
            auto kern = which == 3 ? attn_gqa<1, 128> : which == 2 ? attn_gqa<1, 64>
                      : which == 1 ? attn_gqa<0, 128> : attn_gqa<0, 64>;
            if (!(configured[dev].load() & (1u << which))) {
                cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     (int)attn_gqa_smem(AT_GMAX, 128, AT_SPAN));
                if (e != cudaSuccess) return e;
                configured[dev].fetch_or(1u << which);
            }
            cudaError_t e = launch_pdl(kern, dim3(n, a.kvh, nz), dim3(AT_THREADS), sm, st, a.qkv, a.pos, a.seq, l, a.qd,
                                       a.kvh, a.group, a.kv, a.sqrt_hd, span, a.ctx, ctx_planes(a), a.apart, a.err);
            if (e != cudaSuccess) return e;
            if (nz > 1)
                return launch_pdl(attn_combine, dim3(n, a.kvh), dim3(128), 0, st, a.apart, nz, a.qd, a.kvh, a.hd,
                                  a.group, a.ctx, ctx_planes(a), a.err);
            return cudaSuccess;
        }
    }
    const size_t sm = attention_smem(a, max_pos);
    if (a.kv_bf16)
        return launch_pdl(attention_rows<1>, dim3(n * a.qh), dim3(128), sm, st, a.qkv, n, a.pos, a.seq, l, max_pos,
                          a.qd, a.qh, a.kvh, a.hd, a.group, a.kv, a.sqrt_hd, a.ctx, ctx_planes(a), a.err);
    return launch_pdl(attention_rows<0>, dim3(n * a.qh), dim3(128), sm, st, a.qkv, n, a.pos, a.seq, l, max_pos, a.qd,
                      a.qh, a.kvh, a.hd, a.group, a.kv, a.sqrt_hd, a.ctx, ctx_planes(a), a.err);
}

}  // namespace

bool prefill_supported(const PrefillArgs &a) {
    if (a.chunk < 1 || a.h % 4 || a.ff % 4 || a.hd % 4 || a.hd < 2) return false;
    return gqa_supported(a) || attention_smem(a, a.cap - 1) <= 48 * 1024;
}

cudaError_t forward_tokens(const PrefillArgs &a, int n, int max_pos, bool lm_head, cudaStream_t st) {
    if (n < 1 || n > a.chunk || max_pos >= a.cap) return cudaErrorInvalidValue;
    const int rows_grid = std::min(n, 4096);
    if (a.tfmt == WF_BF16) embed_rows<WF_BF16><<<rows_grid, 256, 0, st>>>(a.ids, n, a.emb, a.semb, a.h, a.x);
    else embed_rows<WF_F32><<<rows_grid, 256, 0, st>>>(a.ids, n, a.emb, a.semb, a.h, a.x);
    cudaError_t e = cudaGetLastError();
    for (int l = 0; l < a.L && e == cudaSuccess; ++l) {
        const DecodeLayer &Ly = a.layers[l];
        if ((e = rmsnorm(a.x, Ly.attn_norm, a.xn, xn_planes(a), n, a.h, a.eps, a.err, st)) != cudaSuccess)
            break;
        if ((e = run_gemm(0, a, l, n, st)) != cudaSuccess) break;
        if (!rope_fused(a, n) &&
            (e = launch_pdl(rope_kv, dim3(rows_grid, n < 16 ? 8 : 1), dim3(128), 0, st, a.qkv, n, a.pos, a.seq, l, a.qd,
                            a.qh, a.kvh,
                            a.hd, a.rope, a.kv, a.kv_bf16, a.err)) !=
                cudaSuccess)
            break;
        if ((e = attention(a, n, l, max_pos, st)) != cudaSuccess) break;
        if ((e = cudaGetLastError()) != cudaSuccess) break;
        if (l + 1 == a.L && !lm_head) break;  // the last layer's MLP feeds only the logits
        if ((e = a.tp ? run_gemm_tp(1, a, l, n, a.x, a.h2, st) : run_gemm(1, a, l, n, st)) != cudaSuccess) break;
        if ((e = rmsnorm(a.h2, Ly.ffn_norm, a.xn, xn_planes(a), n, a.h, a.eps, a.err, st)) != cudaSuccess)
            break;
        if ((e = run_gemm(2, a, l, n, st)) != cudaSuccess) break;
        if ((e = a.tp ? run_gemm_tp(3, a, l, n, a.h2, a.x, st) : run_gemm(3, a, l, n, st)) != cudaSuccess) break;
    }
    if (e != cudaSuccess || !lm_head) return e;
    // Final norm, the LM head (tied table or untied head) and the argmax.
    e = rmsnorm(a.x, a.final_norm, a.xn, xn_planes(a), n, a.h, a.eps, a.err, st);
    if (e != cudaSuccess) return e;
    const Planes none{nullptr, 0, TC_NP};
    GemmW w{a.head, a.semb, 0, a.h, nullptr, nullptr};
    int am_tiles = 0;
    if (n <= GV_MAXT) {
        e = a.tfmt == WF_BF16 ? gemv<WF_BF16, EPI_PLAIN>(a.xn, a.h, n, a.V, a.h, w, nullptr, 0, a.logits, a.V, none,
                                                         a.err, st)
                              : gemv<WF_F32, EPI_PLAIN>(a.xn, a.h, n, a.V, a.h, w, nullptr, 0, a.logits, a.V, none,
                                                        a.err, st);
    } else if (a.tc && a.tc->head.wf >= 0) {
        const TcJob j{EPI_PLAIN, n, a.V, a.h, &a.tc->head, &a.tc->xn, w, nullptr, 0, a.logits, a.V, none,
                      a.amv, a.ami};
        e = tc_gemm(j, a.err, st, &am_tiles);
    } else if (a.tfmt == WF_BF16) {
        e = gemm<WF_BF16, EPI_PLAIN>(a, a.xn, a.h, n, a.V, a.h, w, nullptr, 0, a.logits, a.V, none, st);
    } else {
        e = gemm<WF_F32, EPI_PLAIN>(a, a.xn, a.h, n, a.V, a.h, w, nullptr, 0, a.logits, a.V, none, st);
    }
    if (e != cudaSuccess) return e;
    if (a.tp)  // the per-tile greedy partials' space holds the slice partials
        return tp_argmax(*a.tp, ++*a.tp_seq, a.logits, n, a.V, a.v0, a.amax, a.amv, a.ami, a.err, a.tp_timeout_ns,
                         st);
    if (am_tiles > 0) return launch_pdl(argmax_tiles, dim3(n), dim3(32), 0, st, a.amv, a.ami, am_tiles, n, a.V, a.amax);
    return launch_pdl(argmax_rows, dim3(rows_grid), dim3(256), 0, st, a.logits, n, a.V, a.amax, a.err);
}

cudaError_t advance_tokens(const PrefillArgs &a, int n, cudaStream_t st) {
    return launch_pdl(advance_kernel, dim3((n + 255) / 256), dim3(256), 0, st, a.amax, a.ids, a.pos, n);
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
