// Tensor-parallel exchanges over NVLink peer memory (CUDA IPC): the sums
// after o_proj and down, and the cross-rank greedy argmax.  One-shot
// scheme: every rank leaves its data in its own buffer, raises its flag in
// every rank's buffer (system-scope release), waits until every rank's flag
// for this call is up (bounded), then reads all ranks' data with plain peer
// loads and combines it in rank order, so every rank computes the same
// value with the same rounding.  No multicast, no library collective on
// the data path.
#include <algorithm>

#include "common.cuh"
#include "decode.cuh"
#include "tp.cuh"

namespace qb {

namespace {

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Peer data is read uncached: the same addresses are read again two calls
// later with new contents.
__device__ __forceinline__ float4 ld_peer4(const float4 *p) { return __ldcv(p); }
__device__ __forceinline__ float2 ld_peer2(const float2 *p) { return __ldcv(p); }

// This rank's flag for call `seq` in every rank's buffer (block 0), then
// every block waits until all ranks' flags for the call are up.  Returns
// false (ERR_TIMEOUT recorded) when a flag did not come within the limit.
__device__ bool tp_sync(const TpPeers &P, unsigned seq, unsigned *err, unsigned long long timeout_ns) {
    __shared__ int s_ok;
    const int slot = (int)(seq & 1u);
    if (blockIdx.x == 0 && threadIdx.x < (unsigned)P.size) {
        __threadfence_system();  // this rank's data (earlier kernels) before the flag
        st_release_sys(P.flags[threadIdx.x] + slot * kMaxTp + P.rank, seq);
    }
    if (threadIdx.x == 0) {
        int ok = 1;
        const unsigned *mine = P.flags[P.rank] + slot * kMaxTp;
        const uint64_t t0 = globaltimer_ns();
        for (int j = 0; j < P.size && ok; ++j) {
            unsigned spins = 0;
            while (ld_acquire_sys(mine + j) != seq) {
                if ((++spins & 255u) == 0 && globaltimer_ns() - t0 > timeout_ns) {
                    atomicOr(err, ERR_TIMEOUT);
                    ok = 0;
                    break;
                }
            }
        }
        s_ok = ok;
    }
    __syncthreads();
    return s_ok != 0;
}

__global__ void tp_allreduce_kernel(TpPeers P, unsigned seq, size_t n4, const float4 *R, float4 *Y, unsigned *err,
                                    unsigned long long timeout_ns) {
    if (!tp_sync(P, seq, err, timeout_ns)) return;
    const size_t off = (size_t)(seq & 1u) * P.rows * P.h / 4;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        float4 s = ld_peer4(reinterpret_cast<const float4 *>(P.part[0]) + off + i);
        for (int r = 1; r < P.size; ++r) {
            const float4 v = ld_peer4(reinterpret_cast<const float4 *>(P.part[r]) + off + i);
            s.x = s.x + v.x;
            s.y = s.y + v.y;
            s.z = s.z + v.z;
            s.w = s.w + v.w;
        }
        const float4 rr = R[i];
        float4 o;
        o.x = rr.x + s.x;
        o.y = rr.y + s.y;
        o.z = rr.z + s.z;
        o.w = rr.w + s.w;
        Y[i] = o;
        if (!isfinite(o.x) || !isfinite(o.y) || !isfinite(o.z) || !isfinite(o.w)) atomicOr(err, ERR_NONFINITE);
    }
}

// Local part of the argmax: block (t, z) scans slice z of token t's logits
// row (strict >, so the lowest index wins ties) and leaves (value, v0 +
// index) in pv / pi [t][z].
constexpr int AM_SLICES = 64;

__global__ void tp_argmax_local(const float *logits, int nv, int v0, float *pv, int *pi, unsigned *err) {
    const int t = blockIdx.x, z = blockIdx.y;
    const int per = (nv + AM_SLICES - 1) / AM_SLICES, lo = z * per, hi = min(nv, lo + per);
    const float *row = logits + (size_t)t * nv;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const float v = row[i];
        if (!isfinite(v)) atomicOr(err, ERR_NONFINITE);
        if (v > bv) { bv = v; bi = i; }
    }
    __shared__ float sv[32];
    __shared__ int si[32];
    for (int off = 16; off; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) { sv[warp] = bv; si[warp] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
            if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) { bv = sv[w]; bi = si[w]; }
        pv[(size_t)t * AM_SLICES + z] = bv;
        pi[(size_t)t * AM_SLICES + z] = bi == 0x7fffffff ? 0x7fffffff : v0 + bi;
    }
}

// One block: token t's slice partials in slice order (this rank's best),
// published in its amx slot; then the exchange and the best over ranks.
__global__ void tp_argmax_combine(TpPeers P, unsigned seq, int n, const float *pv, const int *pi, uint32_t *out,
                                  unsigned *err, unsigned long long timeout_ns) {
    const size_t off = (size_t)(seq & 1u) * P.rows;
    for (int t = threadIdx.x; t < n; t += blockDim.x) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int z = 0; z < AM_SLICES; ++z) {
            const float v = pv[(size_t)t * AM_SLICES + z];
            const int i = pi[(size_t)t * AM_SLICES + z];
            if (i != 0x7fffffff && (v > bv || bi == 0x7fffffff)) { bv = v; bi = i; }
        }
        P.amx[P.rank][off + t] = make_float2(bv, __int_as_float(bi == 0x7fffffff ? 0 : bi));
    }
    __syncthreads();
    if (!tp_sync(P, seq, err, timeout_ns)) return;
    for (int t = threadIdx.x; t < n; t += blockDim.x) {
        float2 best = ld_peer2(P.amx[0] + off + t);
        for (int r = 1; r < P.size; ++r) {
            const float2 v = ld_peer2(P.amx[r] + off + t);
            if (v.x > best.x) best = v;  // equal values keep the lower rank (lower ids)
        }
        out[t] = (uint32_t)__float_as_int(best.y);
    }
}

}  // namespace

size_t tp_buffer_bytes(int rows, int h) {
    return 256 + (size_t)2 * rows * h * 4 + (size_t)2 * rows * 8;
}

void tp_carve(void *base, int rows, int h, unsigned **flags, float **part, float2 **amx) {
    uint8_t *b = (uint8_t *)base;
    *flags = (unsigned *)b;
    *part = (float *)(b + 256);
    *amx = (float2 *)(b + 256 + (size_t)2 * rows * h * 4);
}

cudaError_t tp_allreduce(const TpPeers &P, unsigned seq, int n, const float *R, float *Y, unsigned *err,
                         unsigned long long timeout_ns, cudaStream_t st) {
    const size_t n4 = (size_t)n * P.h / 4;
    const unsigned blocks = (unsigned)std::max<size_t>(1, std::min<size_t>((n4 + 255) / 256, 1184));
    tp_allreduce_kernel<<<blocks, 256, 0, st>>>(P, seq, n4, reinterpret_cast<const float4 *>(R),
                                                reinterpret_cast<float4 *>(Y), err, timeout_ns);
    return cudaGetLastError();
}

cudaError_t tp_argmax(const TpPeers &P, unsigned seq, const float *logits, int n, int nv, int v0, uint32_t *out,
                      float *pv, int *pi, unsigned *err, unsigned long long timeout_ns, cudaStream_t st) {
    tp_argmax_local<<<dim3(n, AM_SLICES), 256, 0, st>>>(logits, nv, v0, pv, pi, err);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    tp_argmax_combine<<<1, 256, 0, st>>>(P, seq, n, pv, pi, out, err, timeout_ns);
    return cudaGetLastError();
}

size_t tp_argmax_scratch(int rows) { return (size_t)rows * AM_SLICES; }

}  // namespace qb
