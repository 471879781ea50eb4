// Tensor-core GEMM of the multi-token path (sm_100a: TMA, tcgen05.mma with
// the accumulator in tensor memory).
//
// Weight-stationary tiling: a CTA owns 128 weight rows (the MMA's M) and a
// tile of up to 128 tokens (its N); D[row][token] accumulates in TMEM over
// the CTA's share of K in blocks of 64.  Roles (256 threads):
//   warp 0        TMA producer: per K block the weight box (INT8 into a
//                 staging buffer, BF16 straight into the 128-byte-swizzled
//                 operand tile) and the TC_NP input-plane boxes;
//   warp 1        MMA issuer: 4 K-steps x TC_NP planes of
//                 tcgen05.mma.kind::f16 (BF16 x BF16 -> FP32) per block, a
//                 tcgen05.commit to release the stage;
//   warp 2        TMEM allocation;
//   warps 4..7    INT8 -> BF16 conversion of the staged weights into the
//                 swizzled operand layout (exact: |q| <= 128), then the
//                 epilogue: tcgen05.ld of their 32 TMEM lanes (rows) and
//                 the row-wise epilogue (scale, bias, residual, SwiGLU).
// When K is split, the ks CTAs of an output tile form a thread-block
// cluster: each leaves its partial tile in shared memory and, after a
// cluster barrier, reduces a share of the tile's tokens over the cluster's
// partials (distributed shared memory, in split order) and runs the
// epilogue for them.
// INT8 weights are exact in BF16 and the inputs arrive as BF16 planes
// x = p0 + p1 + p2 (mt::Planes), so every product is exact and only the
// FP32 accumulation order differs from the reference's sequential dot.
// Every wait is bounded: on timeout the CTA records ERR_TIMEOUT, stops
// issuing, drains its copies and MMAs and frees its TMEM.
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <mutex>

#include "tc_gemm.cuh"

namespace qb {
namespace {

using namespace mt;

constexpr int TC_THREADS = 256, TC_BM = 128, TC_BK = 64;
constexpr uint32_t A_BYTES = TC_BM * TC_BK * 2;   // BF16 operand tile, 16 KB
constexpr uint32_t S_BYTES = TC_BM * TC_BK;       // INT8 staging, 8 KB
constexpr unsigned long long TC_TIMEOUT_NS = 2000000000ull;
constexpr int kMaxDevices = 64;

struct TcArgs {
    int n, N, nkb, kb_per, nt, stages, seg_kb;
    GemmW w;
    const float *R;
    int ldr;
    float *Y;
    int ldy;
    Planes P;
    unsigned *err;
    float *amv;
    int *ami;
    RopeKv rk;
    int rope;
};

// AND of v over the 128 epilogue threads (named barrier 1).
__device__ __forceinline__ bool bar_and_128(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\tbar.red.and.pred p, 1, 128, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v)
        : "memory");
    return r != 0;
}

// The QKV value of row r from its raw accumulator (epilogue1's arithmetic).
__device__ __forceinline__ float qkv_value(const GemmW &w, int r, float acc) {
    float v = acc;
    if (w.scale) v = v * w.scale[r];
    if (w.bias) v = v + w.bias[r];
    return v;
}

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *m, int c0, int c1, int c2,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_addr(dst)),
        "l"((uint64_t)m), "r"(c0), "r"(c1), "r"(c2), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)),
                 "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D (TMEM) [+]= A (smem, K-major) * B (smem, K-major)^T.
__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives on `bar` once every MMA this thread issued so far has completed.
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_addr(bar))
                 : "memory");
}

// 16 consecutive TMEM columns of this warp's 32 lanes (one lane per thread);
// the registers are valid after tmem_wait_ld.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Cluster-wide barrier of every thread (release / acquire).
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// The address of the same shared-memory location in cluster CTA `rank`.
__device__ __forceinline__ uint32_t mapa_rank(uint32_t saddr, int rank) {
    uint32_t out;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(saddr), "r"(rank));
    return out;
}

__device__ __forceinline__ float ld_dsmem_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}

// Shared-memory matrix descriptor of a K-major operand tile with 128-byte
// rows in the 128-byte swizzle (8-row groups 1024 bytes apart).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor: BF16 A and B, FP32 D, both K-major, M = 128.
__device__ __forceinline__ uint32_t idesc_bf16(int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(TC_BM >> 4) << 24);
}

// Bounded wait; a timeout (or an abort raised by another role) records
// ERR_TIMEOUT, raises the abort flag and returns false.
__device__ bool tc_wait(uint64_t *bar, uint32_t parity, volatile int *abort_, unsigned *err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
#pragma unroll 1
    for (unsigned it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63u) == 0 && (*abort_ || globaltimer_ns() - t0 > TC_TIMEOUT_NS)) {
            atomicOr(err, ERR_TIMEOUT);
            *abort_ = 1;
            return false;
        }
    }
}

// Wait bounded by time only (draining copies and MMAs already issued).
__device__ bool tc_wait_time(uint64_t *bar, uint32_t parity) {
    const uint64_t t0 = globaltimer_ns();
#pragma unroll 1
    while (!mbar_try_wait(bar, parity))
        if (globaltimer_ns() - t0 > TC_TIMEOUT_NS) return false;
    return true;
}

// Biased INT8 bytes (q + 128) of `w` -> two BF16x2 words (exact).
__device__ __forceinline__ void u8x4_to_bf16x4(uint32_t w, uint32_t &lo, uint32_t &hi) {
    const float f0 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7650u)) - 8388736.0f;
    const float f1 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7651u)) - 8388736.0f;
    const float f2 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7652u)) - 8388736.0f;
    const float f3 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7653u)) - 8388736.0f;
    lo = __byte_perm(__float_as_uint(f0), __float_as_uint(f1), 0x7632u);
    hi = __byte_perm(__float_as_uint(f2), __float_as_uint(f3), 0x7632u);
}

// Row-wise epilogue of outputs (t + k, r) = v[k], k < cnt (the lanes of a
// warp hold 32 consecutive rows r; SwiGLU pairs neighbouring lanes).  Four
// tokens at a time, their loads issued before any store, for ILP.  The
// arithmetic is epilogue1 / epilogue_gu's.
template <int EPI>
__device__ __forceinline__ void epi_rows4(const TcArgs &g, int t, int r, const float (&v)[4], int cnt, int lane) {
    const bool rv = r < g.N;
    if (EPI == EPI_GU) {
        float u[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) u[k] = __shfl_down_sync(0xffffffffu, v[k], 1);
        if (!(lane & 1) && r + 1 < g.N) {
            const float sg = g.w.scale ? g.w.scale[r] : 1.0f, su = g.w.scale ? g.w.scale[r + 1] : 1.0f;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                if (k >= cnt) break;
                float gg = v[k], uu = u[k];
                if (g.w.scale) {
                    gg = gg * sg;
                    uu = uu * su;
                }
                const float a = silu_ref(gg) * uu;
                const size_t i = (size_t)(t + k) * g.ldy + (r >> 1);
                g.Y[i] = a;
                if (g.P.p) store_planes(g.P, i, a);
                flag_bad(g.err, gg);
                flag_bad(g.err, a);
            }
        }
    } else if (rv) {
        float rr[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (EPI == EPI_RESID) {
#pragma unroll
            for (int k = 0; k < 4; ++k)
                if (k < cnt) rr[k] = g.R[(size_t)(t + k) * g.ldr + r];
        }
        const float sc = g.w.scale ? g.w.scale[r] : 1.0f;
        const float b = EPI == EPI_QKV && g.w.bias ? g.w.bias[r] : 0.0f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            if (k >= cnt) break;
            float x = v[k];
            if (g.w.scale) x = x * sc;
            if (EPI == EPI_QKV) {
                if (g.w.bias) x = x + b;
            } else if (EPI == EPI_RESID) {
                x = rr[k] + x;
            }
            g.Y[(size_t)(t + k) * g.ldy + r] = x;
            flag_bad(g.err, x);
        }
    }
}

template <int WF, int EPI>
__global__ void __launch_bounds__(TC_THREADS, 2)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx, const TcArgs g) {
    extern __shared__ uint8_t tc_raw[];
    uint8_t *base = (uint8_t *)(((uintptr_t)tc_raw + 1023) & ~(uintptr_t)1023);
    const int S = g.stages, NT = g.nt;
    const uint32_t b_bytes = (uint32_t)NT * 128u;  // one plane of a stage
    const uint32_t st_bytes = WF == WF_I8 ? S_BYTES : 0u;
    uint8_t *sA = base;
    uint8_t *sB = sA + (size_t)S * A_BYTES;
    uint8_t *sS = sB + (size_t)S * TC_NP * b_bytes;
    float *red = (float *)sA;  // split-K partial tile [NT][128], once the stages are idle
    float *s_epi = (float *)(sS + (size_t)S * st_bytes);  // [4 warps][16][33] transpose tiles
    float *s_amv = s_epi + 4 * 16 * 33;                    // [4][NT] per-warp greedy partials
    int *s_ami = (int *)(s_amv + 4 * NT);
    uint64_t *full = (uint64_t *)(s_ami + 4 * NT);
    uint64_t *ready = full + S, *empty = ready + S, *done = empty + S;
    uint32_t *tslot = (uint32_t *)(done + 1);
    volatile int *abort_ = (volatile int *)(tslot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = blockIdx.x * TC_BM, z = blockIdx.y, t0 = blockIdx.z * NT;
    const int kb0 = z * g.kb_per, nk = min(g.nkb, kb0 + g.kb_per) - kb0;
    // The TC_NP planes of a stage are consecutive NT-row tiles: one MMA with
    // N = TC_NP * NT covers them, the planes landing in column blocks.
    const int NW = TC_NP * NT;
    const uint32_t ncols = NW <= 32 ? 32u : NW <= 64 ? 64u : NW <= 128 ? 128u : 256u;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(full + s, 1);
            mbar_init(ready + s, 128);
            mbar_init(empty + s, 1);
        }
        mbar_init(done, 1);
        *abort_ = 0;
        fence_mbar_init();
    }
    if (warp == 2) tmem_alloc(tslot, ncols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    pdl_trigger();

    if (warp == 0) {
        if (lane == 0) {
            const uint32_t tx_bytes = (WF == WF_I8 ? S_BYTES : A_BYTES) + TC_NP * b_bytes;
            auto load_w = [&](int i) {
                const int s = i % S, kb = kb0 + i;
                mbar_arrive_expect_tx(full + s, tx_bytes);
                tma_load_3d(WF == WF_I8 ? (void *)(sS + (size_t)s * S_BYTES) : (void *)(sA + (size_t)s * A_BYTES), &tw,
                            (kb % g.seg_kb) * TC_BK, row0, kb / g.seg_kb, full + s);
            };
            auto load_x = [&](int i) {
                const int s = i % S, kb = kb0 + i;
#pragma unroll
                for (int p = 0; p < TC_NP; ++p)
                    tma_load_3d(sB + ((size_t)s * TC_NP + p) * b_bytes, &tx, kb * TC_BK, t0, p, full + s);
            };
            // The weights do not depend on earlier kernels: the first stages'
            // weight boxes are in flight before the wait for the inputs.
            const int pre = min(S, nk);
            for (int i = 0; i < pre; ++i) load_w(i);
            pdl_wait();
            for (int i = 0; i < pre; ++i) load_x(i);
            int issued = pre;
#pragma unroll 1
            for (int i = pre; i < nk; ++i) {
                const int s = i % S;
                if (!tc_wait(empty + s, (uint32_t)(((i / S) - 1) & 1), abort_, g.err)) break;
                load_w(i);
                load_x(i);
                ++issued;
            }
            // Every copy issued must land before the CTA can exit.
            for (int i = max(0, issued - S); i < issued; ++i) tc_wait_time(full + (i % S), (uint32_t)((i / S) & 1));
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            pdl_wait();
            const uint32_t idesc = idesc_bf16(NW);
#pragma unroll 1
            for (int i = 0; i < nk; ++i) {
                const int s = i % S;
                const uint32_t ph = (uint32_t)((i / S) & 1);
                if (!tc_wait(WF == WF_I8 ? ready + s : full + s, ph, abort_, g.err)) break;
                tc_fence_after();
                const uint64_t ad = sw128_desc(smem_addr(sA + (size_t)s * A_BYTES));
                const uint64_t bd = sw128_desc(smem_addr(sB + (size_t)s * TC_NP * b_bytes));
#pragma unroll
                for (int k = 0; k < TC_BK / 16; ++k) tc_mma(tmem, ad + 2 * k, bd + 2 * k, idesc, (i | k) != 0);
                tc_commit(empty + s);
            }
            tc_commit(done);
        }
        __syncwarp();
    } else if (warp >= 4) {
        const int ct = threadIdx.x - 128;
        pdl_wait();
        if (WF == WF_I8) {
#pragma unroll 1
            for (int i = 0; i < nk; ++i) {
                const int s = i % S;
                if (!tc_wait(full + s, (uint32_t)((i / S) & 1), abort_, g.err)) break;
                const uint8_t *src = sS + (size_t)s * S_BYTES;
                uint8_t *dst = sA + (size_t)s * A_BYTES;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int item = ct + 128 * j, row = item >> 2, q = item & 3, sw = row & 7;
                    const uint4 w = *(const uint4 *)(src + row * 64 + q * 16);
                    uint4 o0, o1;
                    u8x4_to_bf16x4(w.x, o0.x, o0.y);
                    u8x4_to_bf16x4(w.y, o0.z, o0.w);
                    u8x4_to_bf16x4(w.z, o1.x, o1.y);
                    u8x4_to_bf16x4(w.w, o1.z, o1.w);
                    *(uint4 *)(dst + row * 128 + (((2 * q) ^ sw) << 4)) = o0;
                    *(uint4 *)(dst + row * 128 + (((2 * q + 1) ^ sw) << 4)) = o1;
                }
                fence_proxy_async_smem();
                mbar_arrive(ready + s);
            }
        }
        // Epilogue: wait for the MMAs (also after an abort: TMEM must be
        // idle before it is freed).
        const bool ok = tc_wait_time(done, 0u);
        tc_fence_after();
        if (!ok) atomicOr(g.err, ERR_TIMEOUT);
        const int q = warp & 3, r = row0 + 32 * q + lane;
        const bool split = gridDim.y > 1;
        const bool am = EPI == EPI_PLAIN && g.amv && !split;
        // Uniform over the epilogue warps (the RoPE exchange below uses
        // named barriers).
        const bool run = bar_and_128(ok && !*abort_);
        float *tile = s_epi + q * (16 * 33);
        const bool rope = EPI == EPI_QKV && g.rope;
        if (run) {
            const uint32_t lanes = (uint32_t)(32 * q) << 16;
#pragma unroll 1
            for (int c = 0; c < NT && t0 + c < g.n; c += 16) {
                uint32_t v0[16], v1[16], v2[16];
                tmem_ld16(tmem + lanes + (uint32_t)c, v0);
                tmem_ld16(tmem + lanes + (uint32_t)(c + NT), v1);
                tmem_ld16(tmem + lanes + (uint32_t)(c + 2 * NT), v2);
                tmem_wait_ld();
                // Through shared memory, so that the per-token loop below is
                // not unrolled (one compact copy of the epilogue).
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    tile[j * 33 + lane] = __uint_as_float(v0[j]) + __uint_as_float(v1[j]) + __uint_as_float(v2[j]);
                __syncwarp();
                const int tn = min(16, g.n - t0 - c);
                if (split) {
#pragma unroll 1
                    for (int j = 0; j < tn; ++j) red[(c + j) * TC_BM + ct] = tile[j * 33 + lane];
                } else if (rope) {
                    // The RoPE partner row r ^ (hd / 2) sits in another
                    // warp's tile, same lane.
                    asm volatile("bar.sync 1, 128;" ::: "memory");
                    const int rp = r ^ (g.rk.hd >> 1);
                    const float *ptile = s_epi + (((32 * q + lane) ^ (g.rk.hd >> 1)) >> 5) * (16 * 33);
#pragma unroll 1
                    for (int j = 0; j < tn; ++j)
                        if (r < g.N)
                            qkv_rope_store(g.rk, g.Y, g.ldy, t0 + c + j, r, qkv_value(g.w, r, tile[j * 33 + lane]),
                                           qkv_value(g.w, rp, ptile[j * 33 + lane]), g.err);
                    asm volatile("bar.sync 1, 128;" ::: "memory");
                } else {
#pragma unroll 1
                    for (int j = 0; j < tn; j += 4) {
                        float v[4];
#pragma unroll
                        for (int k = 0; k < 4; ++k) v[k] = tile[min(j + k, 15) * 33 + lane];
                        const int cnt = min(4, tn - j);
                        epi_rows4<EPI>(g, t0 + c + j, r, v, cnt, lane);
                        if (am) {
                            // The warp's greedy row for each token: strict >,
                            // lowest id on ties (a NaN never wins; it is
                            // flagged by the epilogue).
                            float bv[4];
                            int bi[4];
#pragma unroll
                            for (int k = 0; k < 4; ++k) {
                                bv[k] = r < g.N && v[k] == v[k] ? v[k] : -INFINITY;
                                bi[k] = r < g.N && v[k] == v[k] ? r : 0x7fffffff;
                            }
#pragma unroll
                            for (int off = 16; off; off >>= 1)
#pragma unroll
                                for (int k = 0; k < 4; ++k) {
                                    const float ov = __shfl_xor_sync(0xffffffffu, bv[k], off);
                                    const int oi = __shfl_xor_sync(0xffffffffu, bi[k], off);
                                    if (ov > bv[k] || (ov == bv[k] && oi < bi[k])) {
                                        bv[k] = ov;
                                        bi[k] = oi;
                                    }
                                }
                            if (lane == 0)
#pragma unroll
                                for (int k = 0; k < 4; ++k)
                                    if (k < cnt) {
                                        s_amv[q * NT + c + j + k] = bv[k];
                                        s_ami[q * NT + c + j + k] = bi[k];
                                    }
                        }
                    }
                }
                __syncwarp();
            }
        }
        // The conditions below are uniform over the CTA, so every epilogue
        // warp reaches each named barrier whatever `run` was in the others.
        if (am) {
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (run && ct < NT && t0 + ct < g.n) {
                float bv = s_amv[ct];
                int bi = s_ami[ct];
                for (int w = 1; w < 4; ++w) {
                    const float ov = s_amv[w * NT + ct];
                    const int oi = s_ami[w * NT + ct];
                    if (ov > bv || (ov == bv && oi < bi)) {
                        bv = ov;
                        bi = oi;
                    }
                }
                g.amv[(size_t)blockIdx.x * g.n + t0 + ct] = bv;
                g.ami[(size_t)blockIdx.x * g.n + t0 + ct] = bi;
            }
        }
    }
    if (gridDim.y > 1) {
        // Split K: the partial tiles of the cluster are complete after this
        // barrier; CTA z reduces tokens [z * tper, (z + 1) * tper) of the
        // tile over every CTA's partial, in split order.
        cluster_sync();
        if (warp >= 4) {
            const int ct = threadIdx.x - 128, r = row0 + ct;
            const bool run = __all_sync(0xffffffffu, !*abort_);
            const int tn = min(NT, g.n - t0), ks = (int)gridDim.y, tper = (tn + ks - 1) / ks;
            const uint32_t mine = smem_addr(red);
            const int j1 = min(tn, (z + 1) * tper);
            if (EPI == EPI_QKV && g.rope) {
                const int hl = g.rk.hd >> 1, rp = r ^ hl;
#pragma unroll 1
                for (int j = z * tper; j < j1; ++j) {
                    float v = 0.0f, vp = 0.0f;
#pragma unroll 1
                    for (int zz = 0; zz < ks; ++zz) {
                        v += ld_dsmem_f32(mapa_rank(mine + (uint32_t)(j * TC_BM + ct) * 4u, zz));
                        vp += ld_dsmem_f32(mapa_rank(mine + (uint32_t)(j * TC_BM + (ct ^ hl)) * 4u, zz));
                    }
                    if (run && r < g.N)
                        qkv_rope_store(g.rk, g.Y, g.ldy, t0 + j, r, qkv_value(g.w, r, v), qkv_value(g.w, rp, vp), g.err);
                }
            } else
#pragma unroll 1
            for (int j = z * tper; j < j1; j += 4) {
                float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 1
                for (int zz = 0; zz < ks; ++zz)
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        if (j + k < j1) v[k] += ld_dsmem_f32(mapa_rank(mine + (uint32_t)((j + k) * TC_BM + ct) * 4u, zz));
                if (run) epi_rows4<EPI>(g, t0 + j, r, v, min(4, j1 - j), lane);
            }
        }
        // No CTA may exit while another still reads its shared memory.
        cluster_sync();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem, ncols);
    }
}

// ------------------------------------------------------------------ host ----

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
    });
    return fn;
}

// Shared memory outside the stages: the epilogue's transpose tiles and
// greedy partials, the barriers and the TMEM slot.
size_t tc_fixed_bytes(int nt, int stages) {
    return 1024 + (size_t)4 * 16 * 33 * 4 + (size_t)8 * 4 * nt + (size_t)(3 * stages + 1) * 8 + 16;
}

size_t tc_stage_bytes(int wf, int nt) { return A_BYTES + (size_t)TC_NP * nt * 128 + (wf == WF_I8 ? S_BYTES : 0); }

size_t tc_smem_bytes(int wf, int nt, int stages) { return tc_fixed_bytes(nt, stages) + stages * tc_stage_bytes(wf, nt); }

template <int WF, int EPI>
cudaError_t launch(const TcJob &j, const TcArgs &g, dim3 grid, cudaStream_t st) {
    const size_t smem = tc_smem_bytes(WF, g.nt, g.stages);
    // Largest size set for this instantiation, per device (function
    // attributes apply to the current device).
    static std::atomic<size_t> configured[kMaxDevices];
    int dev = 0;
    cudaError_t de = cudaGetDevice(&dev);
    if (de != cudaSuccess) return de;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    if (smem > configured[dev].load()) {
        cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel<WF, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)std::max<size_t>(smem, 200 * 1024));
        if (e != cudaSuccess) return e;
        // Clusters of up to 16 CTAs (K splits of one output tile).
        e = cudaFuncSetAttribute(tc_gemm_kernel<WF, EPI>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
        configured[dev].store(std::max<size_t>(smem, 200 * 1024));
    }
    // Dependent launch; the K splits of an output tile form one cluster.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(TC_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    at[1].id = cudaLaunchAttributeClusterDimension;
    at[1].val.clusterDim.x = 1;
    at[1].val.clusterDim.y = grid.y;
    at[1].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = grid.y > 1 ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, tc_gemm_kernel<WF, EPI>, j.w->map, j.x->m[g.nt / 16 - 1], g);
}

template <int WF>
cudaError_t launch_epi(const TcJob &j, const TcArgs &g, dim3 grid, cudaStream_t st) {
    switch (j.epi) {
    case EPI_QKV: return launch<WF, EPI_QKV>(j, g, grid, st);
    case EPI_RESID: return launch<WF, EPI_RESID>(j, g, grid, st);
    case EPI_GU: return launch<WF, EPI_GU>(j, g, grid, st);
    default: return launch<WF, EPI_PLAIN>(j, g, grid, st);
    }
}

}  // namespace

bool tc_encode_weight(TcWeightMap &m, const uint8_t *base, int wf, size_t rows, size_t seg_len, size_t row_stride,
                      size_t nseg, size_t seg_stride) {
    m.wf = -1;
    auto fn = encode_fn();
    if (!fn || (wf != WF_I8 && wf != WF_BF16) || rows == 0 || seg_len == 0 || nseg == 0) return false;
    if (((uintptr_t)base & 15) || (row_stride & 15) || (seg_stride & 15)) return false;
    if (nseg > 1 && seg_len % TC_BK) return false;  // a K block may not straddle two segments
    const size_t esz = wf == WF_I8 ? 1 : 2;
    if (row_stride < seg_len * esz || (nseg > 1 && seg_stride < rows * row_stride)) return false;
    cuuint64_t dims[3] = {seg_len, rows, nseg};
    cuuint64_t strides[2] = {row_stride, nseg > 1 ? seg_stride : rows * row_stride};
    cuuint32_t box[3] = {TC_BK, TC_BM, 1};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = fn(&m.map, wf == WF_I8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                    (void *)base, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    wf == WF_I8 ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return false;
    m.wf = wf;
    m.seg_kb = nseg > 1 ? (int)(seg_len / TC_BK) : (int)((seg_len + TC_BK - 1) / TC_BK);
    return true;
}

bool tc_encode_planes(TcMaps::X &x, const uint16_t *p, int K, int chunk) {
    auto fn = encode_fn();
    if (!fn || K <= 0 || chunk <= 0 || (K % 8) || ((uintptr_t)p & 15)) return false;
    cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)chunk, (cuuint64_t)TC_NP};
    cuuint64_t strides[2] = {(cuuint64_t)K * 2, (cuuint64_t)K * 2 * chunk};
    cuuint32_t es[3] = {1, 1, 1};
    for (int i = 0; i < TC_TILES; ++i) {
        cuuint32_t box[3] = {TC_BK, (cuuint32_t)(16 * (i + 1)), 1};
        CUresult r = fn(&x.m[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, (void *)p, dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return false;
    }
    return true;
}

cudaError_t tc_gemm(const TcJob &j, unsigned *err, cudaStream_t st, int *am_tiles) {
    if (am_tiles) *am_tiles = 0;
    if (!j.w || j.w->wf < 0 || j.n < 1 || j.N < 1 || j.K < 1) return cudaErrorInvalidValue;
    // Token tiles of at most 80 (the stacked planes' N = 3 nt <= 256).
    const int nt = j.n <= 80 ? (j.n + 15) / 16 * 16 : 64;
    const int ttiles = (j.n + nt - 1) / nt, rtiles = (j.N + TC_BM - 1) / TC_BM;
    const int nkb = (j.K + TC_BK - 1) / TC_BK;
    // Two CTAs per SM when two or more stages fit in half the shared memory
    // (one CTA's conversion and epilogue then overlap the other's copies),
    // else one CTA with up to eight stages.
    const size_t per = tc_stage_bytes(j.w->wf, nt);
    int stages = (int)std::min<size_t>(8, (112 * 1024 - tc_fixed_bytes(nt, 8)) / per), slots = 2 * 148;
    if (stages < 2) {
        stages = (int)std::min<size_t>(8, std::max<size_t>(2, (227 * 1024 - tc_fixed_bytes(nt, 8)) / per));
        slots = 148;
    }
    // Split K (clusters of up to 16 CTAs) while the output tiles leave CTA
    // slots idle, staying in one wave and keeping at least two K blocks a
    // split.
    int ks = 1;
    while (rtiles * ttiles * ks * 2 <= slots && nkb >= ks * 2 * 2 && ks * 2 <= 16) ks *= 2;
    const int kb_per = (nkb + ks - 1) / ks;
    ks = (nkb + kb_per - 1) / kb_per;
    const bool am = j.epi == EPI_PLAIN && j.amv && j.ami && ks == 1;
    TcArgs g{j.n, j.N, nkb, kb_per, nt, stages, j.w->seg_kb, j.gw, j.R, j.ldr, j.Y, j.ldy, j.P, err,
             am ? j.amv : nullptr, am ? j.ami : nullptr, RopeKv{}, 0};
    if (j.epi == EPI_QKV && j.rk) {
        g.rk = *j.rk;
        g.rope = 1;
    }
    if (am && am_tiles) *am_tiles = rtiles;
    const dim3 grid(rtiles, ks, ttiles);
    return j.w->wf == WF_I8 ? launch_epi<WF_I8>(j, g, grid, st) : launch_epi<WF_BF16>(j, g, grid, st);
}

}  // namespace qb
