// Device helpers shared by the multi-token kernels: the GEMM epilogues (per
// row INT8 scale, QKV bias, residual add, SwiGLU of (gate, up) row pairs),
// the deterministic split-K reduction, and the BF16 plane split of GEMM
// inputs read by the tensor-core path.
#pragma once
#include <math.h>

#include <utility>

#include "common.cuh"
#include "decode.cuh"
#include "prefill.cuh"

namespace qb {
namespace mt {

// Programmatic dependent launch: a kernel launched with launch_pdl may start
// while its predecessor in the stream is still running; pdl_wait blocks
// until every earlier kernel has completed and its writes are visible, so
// each such kernel calls it before it reads or writes activations.
// pdl_trigger lets the next kernel be scheduled early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

__device__ __forceinline__ void flag_bad(unsigned *err, float v) {
    if (!isfinite(v)) atomicOr(err, ERR_NONFINITE);
}

// SiLU with the reference's sign branch (src/ops.rs:158-172).
__device__ __forceinline__ float silu_ref(float v) {
    if (v >= 0.0f) return v / (1.0f + expf(-v));
    const float e = expf(v);
    return v * e / (1.0f + e);
}

enum { EPI_QKV = 0, EPI_RESID = 1, EPI_GU = 2, EPI_PLAIN = 3 };

// A weight matrix in the decode layout: row r, segment s (of seg_len
// elements) starts at base + s * seg_stride + r * row_stride, so the
// head-blocked o_proj is one segmented matrix.
struct GemmW {
    const uint8_t *base;
    size_t row_stride, seg_stride;
    int seg_len;
    const float *scale;  // per row (INT8) or null
    const float *bias;   // per row (EPI_QKV) or null
};

// BF16 planes of a GEMM input: v = p0 + p1 + p2 with p0 = bf16(v),
// p1 = bf16(v - p0), p2 = bf16(v - p0 - p1) (each difference is exact in
// FP32), so products with BF16-exact weights summed in FP32 reproduce FP32
// products to about 2^-24 relative.  Plane k of element i is at
// p[k * plane + i]; np is 2 or 3.
struct Planes {
    uint16_t *p;
    size_t plane;
    int np;
};

// FP32 -> BF16, round to nearest even (the hardware conversion).
__device__ __forceinline__ uint16_t bf16_rn(float x) {
    uint16_t r;
    asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(r) : "f"(x));
    return r;
}

__device__ __forceinline__ void store_planes(const Planes &P, size_t i, float v) {
    const uint16_t b0 = bf16_rn(v);
    const float r0 = v - bf16_to_f32(b0);
    const uint16_t b1 = bf16_rn(r0);
    P.p[i] = b0;
    P.p[P.plane + i] = b1;
    if (P.np > 2) P.p[2 * P.plane + i] = bf16_rn(r0 - bf16_to_f32(b1));
}

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

// The SwiGLU epilogue of a (gate, up) row pair r, r + 1 (output r / 2),
// also written as planes when P.p is set.
__device__ __forceinline__ void epilogue_gu(const GemmW &w, int t, int r, float g, float u, float *Y, int ldy,
                                            const Planes &P, unsigned *err) {
    if (w.scale) {
        g = g * w.scale[r];
        u = u * w.scale[r + 1];
    }
    const float a = silu_ref(g) * u;
    const size_t i = (size_t)t * ldy + (r >> 1);
    Y[i] = a;
    if (P.p) store_planes(P, i, a);
    flag_bad(err, g);
    flag_bad(err, a);
}

// RoPE and the KV write fused into the QKV epilogue: everything rope_kv
// needs (per-token positions and sequences, the host cos/sin table and the
// cache geometry).  hd is a power of two >= 64.
struct RopeKv {
    const int *pos, *seq;
    const float2 *rope;  // [cap][hd / 2]
    KvPages kv;          // the paged cache
    int l, h, kvh, hd, kv_bf16;
};

// Output row r of token t of the QKV projection, y (after scale and bias),
// with yp the same token's row r ^ (hd / 2) (the RoPE partner): q rows are
// rotated in place, k rows rotated into the cache, v rows copied into the
// cache (BF16 round-to-nearest-even when the cache is BF16) -- rope_kv's
// arithmetic (src/rope.rs:83-105 with the host table).
__device__ __forceinline__ void qkv_rope_store(const RopeKv &k, float *qkv, int ldq, int t, int r, float y, float yp,
                                               unsigned *err) {
    const int half = k.hd >> 1, kvw = k.kvh * k.hd;
    const int p = k.pos[t];
    flag_bad(err, y);
    if (r < k.h + kvw) {
        const int rr = r < k.h ? r : r - k.h, d = rr & (k.hd - 1);
        const float2 cs = k.rope[(size_t)p * half + (d & (half - 1))];
        const float o = d < half ? y * cs.x - yp * cs.y : y * cs.x + yp * cs.y;
        flag_bad(err, o);
        if (r < k.h) {
            qkv[(size_t)t * ldq + r] = o;
            return;
        }
        uint8_t *kc = k.kv.k(k.l);
        const size_t at = k.kv.row(k.seq[t], rr / k.hd, p) + d;
        if (k.kv_bf16) ((uint16_t *)kc)[at] = bf16_rn(o);
        else ((float *)kc)[at] = o;
    } else {
        const int rr = r - k.h - kvw, d = rr & (k.hd - 1);
        uint8_t *vc = k.kv.v(k.l);
        const size_t at = k.kv.row(k.seq[t], rr / k.hd, p) + d;
        if (k.kv_bf16) ((uint16_t *)vc)[at] = bf16_rn(y);
        else ((float *)vc)[at] = y;
    }
}

// Sums the ks split-K partials part[z][t][r] of each output in slice order,
// then the epilogue (SwiGLU outputs one value per row pair).
template <int EPI>
__global__ void reduce_epilogue(const float *part, int ks, int n, int N, GemmW w, const float *R, int ldr, float *Y,
                                int ldy, Planes P, unsigned *err) {
    pdl_trigger();
    pdl_wait();
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
            epilogue_gu(w, (int)t, r, g, u, Y, ldy, P, err);
        } else {
            const size_t t = i / N;
            const int r = (int)(i - t * N);
            float v = 0.0f;
            for (int z = 0; z < ks; ++z) v += part[z * per + i];
            epilogue1<EPI>(w, (int)t, r, v, R, ldr, Y, ldy, err);
        }
    }
}

}  // namespace mt
}  // namespace qb
