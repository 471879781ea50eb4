// Persistent decode-step kernel for batch-1 greedy decoding on sm_100a.
//
// One cooperative launch evaluates one token through every layer and the LM
// head (src/kv_cache.rs:347-475 with attend_one :479-590) and leaves the
// greedy argmax (src/sampling.rs:65-70) in the control block.  The grid is
// one CTA per SM: 15 compute warps and one producer warp.  A phase's
// outputs reach the next phase through exchange vectors that consumers poll
// word by word (no grid barrier); every poll is bounded by a timeout (the
// kernel then reports ERR_TIMEOUT and returns; it never spins forever):
//
//   per layer:  QKV      RMSNorm (each CTA, redundantly) -> rows of [Wq;Wk;Wv]
//                        + bias
//               ATTN     per (query head, o_proj row range): RoPE from the host
//                        cos/sin table, K/V write, softmax(q.K/sqrt d).V, then
//                        that head's o_proj partial for the row range
//               GATE/UP  residual + sum of head partials, RMSNorm, (gate, up)
//                        row pairs, SiLU(gate)*up
//               DOWN     rows of down + residual
//   final:      LM HEAD  RMSNorm, rows of the (tied) table, logits, argmax;
//                        the last CTA reduces the per-CTA argmaxes.
//
// Weight streaming.  Weights never depend on activations, so the producer
// warp streams every row block the CTA will multiply -- all phases of the
// step, in order -- through a shared-memory ring of `nslot` slots with 1-D
// bulk copies (cp.async.bulk ... mbarrier::complete_tx), waiting only for
// the compute warps to free a slot ("empty" mbarrier, one arrival per compute
// warp).  It never waits for another CTA, so a phase's weights are in
// shared memory before the activations they meet exist.
//
// Latency discipline.  Batch-1 decode moves ~1 MB per CTA per step; what
// costs time is dependent latency, so the compute side is written to keep
// every chain short: every helper is inlined (no stack frame, no local
// memory), global loads are issued in batches before their first use, each
// GEMV row is reduced by a team of threads with shuffles (no shared-memory
// partials), reductions over a vector are done redundantly per warp instead
// of across warps, and activations sit in shared memory in a layout whose
// 16-byte reads never conflict.
#include <math.h>

#include <algorithm>

#include "common.cuh"
#include "decode.cuh"

namespace qb {

constexpr int NT = kDecodeThreads;  // compute threads
constexpr int NW = NT / 32;         // compute warps
constexpr int LOOKAHEAD = 3;        // L2 prefetch distance in phases
constexpr int LM_PREFETCH = 8;      // LM-head rows: L2 prefetch distance in ring chunks
constexpr unsigned FULL = 0xffffffffu;

template <int WF> struct Fmt;
template <> struct Fmt<WF_F32> { static constexpr int EPC = 4; };
template <> struct Fmt<WF_BF16> { static constexpr int EPC = 8; };
template <> struct Fmt<WF_I8> { static constexpr int EPC = 16; };

__device__ __forceinline__ float ldcg(const float *p) { return __ldcg(p); }

// Barrier among the compute warps only (the producer warp never joins).
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(NT) : "memory"); }
// Barrier of the warps of one GEMV team wider than a warp (ids 2..15).
__device__ __forceinline__ void team_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ------------------------------------------------------ activations ----
//
// An activation vector that meets rows of C 16-byte chunks (EPC elements
// each) is kept "quad-major": element e, in chunk c = e / EPC at position
// k = e % EPC, lives at float (k / 4 * C + c) * 4 + k % 4.  Chunk c's quads
// are then C float4 apart and threads that read consecutive chunks read
// consecutive 16-byte words.

template <int EPC>
__device__ __forceinline__ int xq(int e, int C) {
    const int c = e / EPC, k = e % EPC;
    return ((k >> 2) * C + c) * 4 + (k & 3);
}

// Packed FP32 pairs (Blackwell f32x2 pipe): two FMAs or adds per
// instruction, each lane rounded exactly like fmaf / __fadd_rn.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

// Dot product of one 16-byte weight chunk with its EPC activations (the
// chunk's quads x[0..EPC/4)), accumulated into two pairs of partial sums
// (four independent FMA chains; the caller adds them at the end).  INT8
// bytes become exact floats by a byte permute into 2^23 + u and one packed
// subtract of 2^23 + 128.
template <int WF>
__device__ __forceinline__ void chunk_dot2(const uint4 &w, const float4 *x, float2 &acc, float2 &acc2) {
    if (WF == WF_F32) {
        acc = ffma2(make_float2(x[0].x, x[0].y), make_float2(__uint_as_float(w.x), __uint_as_float(w.y)), acc);
        acc2 = ffma2(make_float2(x[0].z, x[0].w), make_float2(__uint_as_float(w.z), __uint_as_float(w.w)), acc2);
    } else if (WF == WF_BF16) {
        acc = ffma2(make_float2(x[0].x, x[0].y), make_float2(bf16_lo(w.x), bf16_hi(w.x)), acc);
        acc2 = ffma2(make_float2(x[0].z, x[0].w), make_float2(bf16_lo(w.y), bf16_hi(w.y)), acc2);
        acc = ffma2(make_float2(x[1].x, x[1].y), make_float2(bf16_lo(w.z), bf16_hi(w.z)), acc);
        acc2 = ffma2(make_float2(x[1].z, x[1].w), make_float2(bf16_lo(w.w), bf16_hi(w.w)), acc2);
    } else {
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
        const float2 bias = make_float2(-8388736.0f, -8388736.0f);  // -(2^23 + 128)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 q01 = fadd2(make_float2(__uint_as_float(__byte_perm(ws[k], 0x4B000000u, 0x7650)),
                                                 __uint_as_float(__byte_perm(ws[k], 0x4B000000u, 0x7651))),
                                     bias);
            const float2 q23 = fadd2(make_float2(__uint_as_float(__byte_perm(ws[k], 0x4B000000u, 0x7652)),
                                                 __uint_as_float(__byte_perm(ws[k], 0x4B000000u, 0x7653))),
                                     bias);
            acc = ffma2(make_float2(x[k].x, x[k].y), q01, acc);
            acc2 = ffma2(make_float2(x[k].z, x[k].w), q23, acc2);
        }
    }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int off = 16; off; off >>= 1) v += __shfl_xor_sync(FULL, v, off);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int off = 16; off; off >>= 1) v = rust_max(v, __shfl_xor_sync(FULL, v, off));
    return v;
}

// Scaled RMSNorm (src/ops.rs:137-149) of `in` (shared, width w) into the
// quad-major layout for EPC/C, zero-padded to C * EPC.  Each warp reduces
// its slice to a pair (m_w = max |x|, s_w = sum (x / m_w)^2) and leaves it in
// red[2w, 2w + 1]; after one CTA barrier every warp combines the pairs,
// lane k taking warp k's: s = max(sqrt(eps), max m_w), sum (x/s)^2 =
// sum s_w (m_w/s)^2 (shuffle trees; no serial chain of loads).
// Scaling by reciprocals keeps the result within a few ulps of the
// reference's divisions; a maximum of 2^125 or more (whose reciprocal would
// be subnormal) keeps the divisions.
template <int EPC>
__device__ __forceinline__ void block_rmsnorm(const float *in, const float *gain, float *xs, int w, int C,
                                              float eps, float *red) {
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const float se = sqrtf(eps);
    float mw = se;
#pragma unroll 2
    for (int i = t; i < w; i += NT) mw = rust_max(mw, fabsf(in[i]));
    mw = warp_max(mw);
    const bool bigw = mw >= 0x1p125f;  // warp-uniform
    const float rw = 1.0f / mw;
    float sw = 0.0f;
#pragma unroll 2
    for (int i = t; i < w; i += NT) {
        const float v = bigw ? in[i] / mw : in[i] * rw;
        sw = sw + v * v;
    }
    sw = warp_sum(sw);
    if (lane == 0) {
        red[2 * warp] = mw;
        red[2 * warp + 1] = sw;
    }
    csync();
    const float2 pr = lane < NW ? *reinterpret_cast<const float2 *>(red + 2 * lane) : make_float2(se, 0.0f);
    const float m = warp_max(pr.x);
    const bool big = m >= 0x1p125f;  // CTA-uniform
    const float r = 1.0f / m;
    float f, seps;
    if (big) {
        f = pr.x / m;
        seps = se / m;
    } else {
        f = pr.x * r;
        seps = se * r;
    }
    const float ss = warp_sum(pr.y * (f * f));
    const float rd = 1.0f / sqrtf(ss / (float)w + seps * seps);
#define QB_XS(v) ((big ? (v) / m : (v) * r) * rd)
    const int padded = C * EPC;
    if ((w & 3) == 0) {
        // Four consecutive elements are one quad of the layout.
        float4 *x4 = reinterpret_cast<float4 *>(xs);
        for (int e = 4 * t; e < padded; e += 4 * NT) {
            float4 o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (e < w) {
                o.x = QB_XS(in[e]) * gain[e];
                o.y = QB_XS(in[e + 1]) * gain[e + 1];
                o.z = QB_XS(in[e + 2]) * gain[e + 2];
                o.w = QB_XS(in[e + 3]) * gain[e + 3];
            }
            x4[((e % EPC) >> 2) * C + e / EPC] = o;
        }
    } else {
        for (int i = t; i < padded; i += NT) xs[xq<EPC>(i, C)] = i < w ? QB_XS(in[i]) * gain[i] : 0.0f;
    }
#undef QB_XS
    csync();
}

// Statistics of the elements one thread staged: sum of squares and max |x|.
struct NormAcc {
    float ss = 0.0f, mx = 0.0f;
    __device__ __forceinline__ void add(float v) {
        ss = fmaf(v, v, ss);
        mx = fmaxf(mx, fabsf(v));
    }
};

// RMSNorm of `in` (shared, width w, staged by this CTA's threads, whose
// NormAcc covers exactly the elements each staged) into xs, as
// block_rmsnorm, starting right after the staging (no CTA barrier needed
// before the call).  The statistics come from the staging pass: one
// butterfly of (sum of squares, max) per warp, one CTA barrier, then every
// thread adds the warps' pairs in warp order and takes
// rd = 1 / sqrt(sum / w + eps); y = x * rd * gain.  This is the scaled form
// of src/ops.rs:137-149 without the scaling, equal to it up to rounding
// while max |x| < 2^58 (no square overflows a float sum of 2^10 terms) and
// eps >= 2^-60; outside that range the scaled block_rmsnorm runs instead.
template <int EPC>
__device__ __forceinline__ void norm_staged(const float *in, const float *gain, float *xs, int w, int C, float eps,
                                            float *red, NormAcc a) {
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
#pragma unroll
    for (int off = 16; off; off >>= 1) {
        a.ss += __shfl_xor_sync(FULL, a.ss, off);
        a.mx = fmaxf(a.mx, __shfl_xor_sync(FULL, a.mx, off));
    }
    if (lane == 0) *reinterpret_cast<float2 *>(red + 2 * warp) = make_float2(a.ss, a.mx);
    csync();
    float S = 0.0f, M = 0.0f;
#pragma unroll
    for (int k = 0; k < NW; ++k) {
        const float2 v = *reinterpret_cast<const float2 *>(red + 2 * k);
        S += v.x;
        M = fmaxf(M, v.y);
    }
    if (!(M < 0x1p58f && eps >= 0x1p-60f)) {  // CTA-uniform
        csync();  // every thread has read red
        block_rmsnorm<EPC>(in, gain, xs, w, C, eps, red);
        return;
    }
    const float rd = 1.0f / sqrtf(S / (float)w + eps);
    const int padded = C * EPC;
    if ((w & 3) == 0) {
        float4 *x4 = reinterpret_cast<float4 *>(xs);
        for (int e = 4 * t; e < padded; e += 4 * NT) {
            float4 o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (e < w) {
                const float4 v = *reinterpret_cast<const float4 *>(in + e);
                const float4 gg = *reinterpret_cast<const float4 *>(gain + e);
                o.x = (v.x * rd) * gg.x;
                o.y = (v.y * rd) * gg.y;
                o.z = (v.z * rd) * gg.z;
                o.w = (v.w * rd) * gg.w;
            }
            x4[((e % EPC) >> 2) * C + e / EPC] = o;
        }
    } else {
        for (int i = t; i < padded; i += NT) xs[xq<EPC>(i, C)] = i < w ? (in[i] * rd) * gain[i] : 0.0f;
    }
    csync();
}

__device__ __forceinline__ void flag_nonfinite(DecodeCtrl *ctrl, float v) {
    if (!isfinite(v)) atomicOr(&ctrl->error, ERR_NONFINITE);
}

// dst[i] = src[i], i < n, for read-only model vectors (gains, scales,
// biases): asynchronous copies issued by every compute thread (16 bytes at a
// time when both sides are 16-byte aligned and n % 4 == 0), completed by
// the next cp_async_wait_all.  A phase's vectors are issued at the start of
// the phase before it, so their latency is off the critical path.
__device__ __forceinline__ void stage_async(float *dst, const float *src, int n) {
    if ((n & 3) == 0 && ((uintptr_t)src & 15) == 0 && ((uintptr_t)dst & 15) == 0) {
#pragma unroll 1
        for (int i = threadIdx.x; i < (n >> 2); i += NT) cp_async16(dst + 4 * i, src + 4 * i);
    } else {
#pragma unroll 1
        for (int i = threadIdx.x; i < n; i += NT) cp_async4(dst + i, src + i);
    }
}

// --------------------------------------------------------------- ring ----
//
// Chunk k of the CTA's stream lives in slot k % nslot during round
// u = k / nslot.  full[slot] completes phase u when the copy lands; every
// compute warp arrives on empty[slot] (phase u) once it has read it.

struct Ring {
    uint8_t *slots;
    uint64_t *full, *empty;
    int nslot, slot_bytes;
};

__device__ __forceinline__ Ring ring_of(const DecodeParams &p, float *sm) {
    Ring r;
    r.slots = (uint8_t *)(sm + p.sm_ring);
    r.full = (uint64_t *)(sm + p.sm_bar);
    r.empty = r.full + p.nslot;
    r.nslot = p.nslot;
    r.slot_bytes = p.slot_bytes;
    return r;
}

// Bounded wait for `parity` on `bar`.  On timeout (or when the CTA is
// already aborting) records ERR_TIMEOUT, raises the abort flag and returns
// false; callers carry on to their next CTA barrier, after which the abort
// flag is tested uniformly.
__device__ __forceinline__ bool mbar_wait(const DecodeParams &p, uint64_t *bar, uint32_t parity,
                                          volatile int *s_abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
#pragma unroll 1
    for (unsigned it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63u) == 0 && (*s_abort || globaltimer_ns() - t0 > p.timeout_ns)) {
            atomicOr(&p.ctrl->error, ERR_TIMEOUT);
            *s_abort = 1;
            return false;
        }
    }
}

// Consumer cursor (identical in every compute thread).
struct Cursor {
    int slot, round;
    __device__ __forceinline__ void advance(int nslot) {
        if (++slot == nslot) { slot = 0; ++round; }
    }
};

// --------------------------------------------------------------- producer ----

struct Producer {
    const DecodeParams &p;
    Ring rg;
    volatile int *s_abort;
    int slot = 0, round = 0;
    bool alive = true;

    __device__ Producer(const DecodeParams &pp, const Ring &r, volatile int *a) : p(pp), rg(r), s_abort(a) {}

    // Bounded wait for a free slot.  The producer is usually far ahead of
    // the compute warps, so it waits suspended in hardware (not spinning,
    // which would take issue slots from the compute warps of its SM
    // sub-partition).
    __device__ bool wait_free(int s, uint32_t parity) {
        const uint64_t t0 = globaltimer_ns();
#pragma unroll 1
        while (!mbar_try_wait_suspend(rg.empty + s, parity, 20000u)) {
            if (*s_abort || globaltimer_ns() - t0 > p.timeout_ns) {
                atomicOr(&p.ctrl->error, ERR_TIMEOUT);
                *s_abort = 1;
                return false;
            }
        }
        return true;
    }

    // Streams rows [0, n) of a block (stride bytes each) in ring chunks.
    // With pf > 0 the chunk pf chunks ahead is prefetched into L2 as each
    // chunk is issued (the LM head, a stream much longer than the ring), so
    // more DRAM reads are in flight than the ring's slots hold.
    __device__ void block(const uint8_t *base, int n, const KindGeom &g, int pf = 0) {
#pragma unroll 1
        for (int r = 0; r < n && alive; r += g.rpc) {
            if (pf > 0) {
                const int rp = r + pf * g.rpc;
                if (rp < n)
                    prefetch_l2_bulk(base + (size_t)rp * g.stride, (uint32_t)(min(g.rpc, n - rp) * g.stride) & ~15u);
            }
            if (round > 0 && !wait_free(slot, (uint32_t)((round - 1) & 1))) {
                alive = false;
                return;
            }
            const uint32_t bytes = (uint32_t)(min(g.rpc, n - r) * g.stride);
            mbar_arrive_expect_tx(rg.full + slot, bytes);
            bulk_copy_g2s(rg.slots + (size_t)slot * rg.slot_bytes, base + (size_t)r * g.stride, bytes,
                          rg.full + slot);
            if (++slot == rg.nslot) { slot = 0; ++round; }
        }
    }

    // Waits (bounded, each slot with its own limit) for every copy this
    // producer issued, before the CTA exits early, so no bulk copy still
    // writes this CTA's shared memory after it is gone.  A copy that has
    // not landed within the limit means the memory system itself has
    // stalled for seconds; the producer then records ERR_TIMEOUT (the host
    // fails the step and invalidates the session) and stops waiting rather
    // than hold the SM forever.
    __device__ void drain() {
        for (int s = 0; s < rg.nslot; ++s) {
            // Slot s was last filled in round (s < slot ? round : round - 1).
            const int u = s < slot ? round : round - 1;
            if (u < 0) continue;
            const uint64_t t0 = globaltimer_ns();
            while (!mbar_try_wait(rg.full + s, (uint32_t)(u & 1)))
                if (globaltimer_ns() - t0 > p.timeout_ns) {
                    atomicOr(&p.ctrl->error, ERR_TIMEOUT);
                    return;
                }
        }
    }
};

// L2 prefetch of `bytes` at `base` by the producer warp's lanes.
__device__ __forceinline__ void prefetch_rows(const uint8_t *base, size_t bytes) {
    const int lane = threadIdx.x & 31;
    const size_t piece = 16384;
#pragma unroll 1
    for (size_t off = (size_t)lane * piece; off < bytes; off += 32 * piece) {
        const size_t n = bytes - off < piece ? bytes - off : piece;
        if (n >= 16) prefetch_l2_bulk(base + off, (uint32_t)(n & ~(size_t)15));
    }
}

// Prefetches into L2 everything phase k of this CTA will stream: its weight
// rows and, for attention, the cached K/V rows of its heads.
__device__ void prefetch_phase(const DecodeParams &p, const DecodeLayer *lay, const CtaGeom &cg, int k,
                               int pos, const float *sm) {
    if (!p.prefetch || k > 4 * p.L) return;
    if (k == 4 * p.L) {
        prefetch_rows(p.head + (size_t)cg.lm_v0 * p.semb, (size_t)min(cg.lm_n, LM_PREFETCH * p.kind[K_LM].rpc) * p.semb);
        return;
    }
    const DecodeLayer &Ly = lay[k >> 2];
    const size_t cap = (size_t)p.pf_cap;
    switch (k & 3) {
    case 0: prefetch_rows(Ly.wqkv + (size_t)cg.qkv_r0 * p.sh, min((size_t)cg.qkv_n * p.sh, cap)); break;
    case 1: {
        const size_t esz = p.kv_bf16 ? 2 : 4;
        for (int a = 0; a < cg.natt; ++a) {
            prefetch_rows(Ly.wo + ((size_t)cg.att_hh[a] * p.h + cg.att_r0[a]) * p.shd,
                          min((size_t)cg.att_n[a] * p.shd, cap));
            const int g = cg.att_hh[a] / p.group;
            // The group's block of every page that holds cached positions.
            const int *ptab = (const int *)(sm + p.sm_ptab);
            const size_t blk = (size_t)kPageTokens * p.hd * esz;
            const int np = (pos + kPageTokens - 1) / kPageTokens;
#pragma unroll 1
            for (int j = threadIdx.x & 31; j < np; j += 32) {
                const size_t off = ((size_t)ptab[j] * p.kvh + g) * blk;
                prefetch_l2_bulk(Ly.kc + off, (uint32_t)blk);
                prefetch_l2_bulk(Ly.vc + off, (uint32_t)blk);
            }
        }
        break;
    }
    case 2: prefetch_rows(Ly.wgu + (size_t)2 * cg.gu_f0 * p.sh, min((size_t)2 * cg.gu_n * p.sh, cap)); break;
    default: prefetch_rows(Ly.wd + (size_t)cg.dn_r0 * p.sff, min((size_t)cg.dn_n * p.sff, cap)); break;
    }
}

// Query-head splits of this step's attention (1 below att_split_min cached
// positions or in the kernel without the split path).
template <int SPLIT>
__device__ __forceinline__ int att_nsp(const DecodeParams &p, int pos) {
    return SPLIT && p.att_splits > 1 && pos + 1 >= p.att_split_min ? p.att_splits : 1;
}

// The producer warp: the step's blocks in consumption order.
__device__ void produce(const DecodeParams &p, const DecodeLayer *lay, const CtaGeom &cg, float *sm, int pos,
                        volatile int *s_abort) {
    Producer pr(p, ring_of(p, sm), s_abort);
    const bool leader = (threadIdx.x & 31) == 0;
    for (int k = 0; k < LOOKAHEAD; ++k) prefetch_phase(p, lay, cg, k, pos, sm);
#pragma unroll 1
    for (int l = 0; l < p.L && pr.alive; ++l) {
        const DecodeLayer &Ly = lay[l];
        const int ph = 4 * l;
        prefetch_phase(p, lay, cg, ph + LOOKAHEAD, pos, sm);
        if (leader) pr.block(Ly.wqkv + (size_t)cg.qkv_r0 * p.sh, cg.qkv_n, p.kind[K_QKV]);
        prefetch_phase(p, lay, cg, ph + 1 + LOOKAHEAD, pos, sm);
        if (leader)
            for (int a = 0; a < cg.natt; ++a)
                pr.block(Ly.wo + ((size_t)cg.att_hh[a] * p.h + cg.att_r0[a]) * p.shd, cg.att_n[a], p.kind[K_O]);
        prefetch_phase(p, lay, cg, ph + 2 + LOOKAHEAD, pos, sm);
        if (leader) pr.block(Ly.wgu + (size_t)2 * cg.gu_f0 * p.sh, 2 * cg.gu_n, p.kind[K_GU]);
        prefetch_phase(p, lay, cg, ph + 3 + LOOKAHEAD, pos, sm);
        if (leader) pr.block(Ly.wd + (size_t)cg.dn_r0 * p.sff, cg.dn_n, p.kind[K_DN]);
        pr.alive = __shfl_sync(FULL, (int)pr.alive, 0) != 0;
    }
    if (leader && pr.alive) pr.block(p.head + (size_t)cg.lm_v0 * p.semb, cg.lm_n, p.kind[K_LM], LM_PREFETCH);
    if (leader && !pr.alive) pr.drain();
}

// ------------------------------------------------------------ gemv ----

// Publishes v in an exchange slot of this step.
__device__ __forceinline__ void publish(float *slot, float v) {
    uint32_t b = __float_as_uint(v);
    if (b == kNotReady) b = 0x7fffffffu;
    st_relaxed_b32(slot, b);
}

// SiLU with the reference's sign branch (src/ops.rs:158-173).
__device__ __forceinline__ float silu1(float v) {
    if (v >= 0.0f) return v / (1.0f + expf(-v));
    const float e = expf(v);
    return v * e / (1.0f + e);
}

// Epilogues of the per-layer GEMVs, chosen by a run-time kind (the
// kernel's hot code must stay small: instruction-cache misses were its
// largest stall when every phase carried three specialised GEMV copies).
enum { EPI_QKV = 0, EPI_O = 1, EPI_GU = 2, EPI_DN = 3 };
struct Epi {
    float *out;         // exchange slots, by row (EPI_GU: by row pair)
    const float *rv;    // row scales (INT8; any memory space) and, for EPI_QKV, biases at rv + n
    const float *res;   // EPI_DN: the residual rows (shared memory)
    int kind;
    int pub;            // 0: EPI_QKV withholds its outputs (the fault-path hook)
};

__device__ __forceinline__ void epi_row(const Epi &e, int WFi8, int n, int r, float v, DecodeCtrl *ctrl) {
    if (e.kind == EPI_QKV) {
        if (WFi8) v = v * e.rv[r];
        v = v + e.rv[n + r];
        if (e.pub) publish(e.out + r, v);
    } else if (e.kind == EPI_O) {
        if (WFi8) v = v * e.rv[r];
        publish(e.out + r, v);
    } else {  // EPI_DN
        if (WFi8) v = v * e.rv[r];
        v = e.res[r] + v;
        publish(e.out + r, v);
    }
    flag_nonfinite(ctrl, v);
}

// y_r = dot(W_r, x) for the n rows of one streamed block, rows taken in
// pairs (2u, 2u + 1) when g.U == 2 (gate/up pairs, or two independent rows
// that share the activation loads; the host pairs rows only where two fit
// a ring slot) or one at a time when g.U == 1.  The block is consumed in waves of up to g.wave ring
// slots: every warp waits for the wave's slots, then teams of G = 2^g.lgG
// threads (G chosen by the host, a run-time value) take row pairs
// round-robin; a team's threads stride the rows' 16-byte chunks with four
// FP32 chains per row, meet in a shuffle butterfly, and the team's first
// thread runs the epilogue.  Each warp frees the wave's slots as soon as it
// is done with them.  A failed wait (timeout) leaves the abort flag set;
// the caller tests it after its next CTA barrier.  An odd block's last pair
// reads a stale (in-bounds) row of its slot, whose result is discarded.
// Inlined (a call costs more than the code it saves: the kernel parameters
// become generic loads and live registers spill around it); the team size
// is a run-time value, so each phase holds one copy of the loop.  Returns
// the advanced cursor.
// The wait of gemv_pairs for the first wave of a block of n rows starting
// at `cur`: each warp observes those copies (lane j the j-th) before it
// needs them.  Issued at the start of a phase, before the phase's inputs
// are polled, so the weights' acquire overlaps the hand-over instead of
// following it; gemv_pairs is then called with prewaited = true.
__device__ __forceinline__ void ring_prewait(const DecodeParams &p, const Ring &rg, const Cursor &cur,
                                             const KindGeom &g, int n, volatile int *s_abort) {
    const int lane = threadIdx.x & 31;
    const int rows = min(g.wave * g.rpc, n);
    const int ns = g.rpc == 1 ? rows : (int)__umulhi((unsigned)(rows + g.rpc - 1), g.rpc_magic);
#pragma unroll 1
    for (int j = lane; j < ns; j += 32) {
        int s = cur.slot + j, rd = cur.round;
        while (s >= rg.nslot) { s -= rg.nslot; ++rd; }
        mbar_wait(p, rg.full + s, (uint32_t)(rd & 1), s_abort);
    }
    __syncwarp();
}

template <int WF>
__device__ __forceinline__ Cursor gemv_pairs(const DecodeParams &p, const Ring rg, Cursor cur, const KindGeom &g,
                                          int n, const float *xs, volatile int *s_abort, const Epi e,
                                          bool prewaited, float *tscr) {
    constexpr int Q = Fmt<WF>::EPC / 4;
    const int lg = g.lgG, G = 1 << lg, T = NT >> lg;
    const int t = threadIdx.x, lane = t & 31;
    const int lt = t & (G - 1), tm = t >> lg;
    const int warp_team0 = (t & ~31) >> lg;
    const int C = g.C;
    const float4 *x4 = reinterpret_cast<const float4 *>(xs);
    DecodeCtrl *ctrl = p.ctrl;
#pragma unroll 1
    for (int r0 = 0; r0 < n;) {
        const int rows = min(g.wave * g.rpc, n - r0);
        const int ns = g.rpc == 1 ? rows : (int)__umulhi((unsigned)(rows + g.rpc - 1), g.rpc_magic);
        // Lane j of each warp observes the completion of the wave's j-th
        // copy (acquire); __syncwarp orders the rest of the warp's reads
        // after all of them.  The first wave was observed already when the
        // caller pre-waited.
        if (!(prewaited && r0 == 0)) {
#pragma unroll 1
            for (int j = lane; j < ns; j += 32) {
                int s = cur.slot + j, rd = cur.round;
                while (s >= rg.nslot) { s -= rg.nslot; ++rd; }
                mbar_wait(p, rg.full + s, (uint32_t)(rd & 1), s_abort);
            }
            __syncwarp();
        }
        const bool two = g.U == 2;
        const int nu = two ? (rows + 1) >> 1 : rows;
#pragma unroll 1
        for (int ub = 0; ub < nu; ub += T) {
            if (warp_team0 >= T || ub + warp_team0 >= nu) break;  // warp-uniform
            const int u = ub + tm;
            const bool act = u < nu;
            // Four independent partial-sum chains per row: two per chunk,
            // and alternate chunks in alternate pairs.
            float2 a0 = make_float2(0.0f, 0.0f), b0 = a0, c0 = a0, d0 = a0;
            float2 a1 = a0, b1 = a0, c1 = a0, d1 = a0;
            if (act) {
                const int row = two ? 2 * u : u;
                const int j = g.rpc == 1 ? row : (int)__umulhi((unsigned)row, g.rpc_magic);
                int s = cur.slot + j;
                if (s >= rg.nslot) s -= rg.nslot;
                const uint8_t *w0 = rg.slots + (size_t)s * rg.slot_bytes + (size_t)(row - j * g.rpc) * g.stride;
                int c = lt;
#pragma unroll 1
                for (; c + G < C; c += 2 * G) {
                    float4 x[Q], y[Q];
#pragma unroll
                    for (int q = 0; q < Q; ++q) { x[q] = x4[q * C + c]; y[q] = x4[q * C + c + G]; }
                    const uint4 w = *reinterpret_cast<const uint4 *>(w0 + (size_t)c * 16);
                    const uint4 v = *reinterpret_cast<const uint4 *>(w0 + (size_t)(c + G) * 16);
                    chunk_dot2<WF>(w, x, a0, b0);
                    chunk_dot2<WF>(v, y, c0, d0);
                    if (two) {
                        const uint4 w1 = *reinterpret_cast<const uint4 *>(w0 + g.stride + (size_t)c * 16);
                        const uint4 v1 = *reinterpret_cast<const uint4 *>(w0 + g.stride + (size_t)(c + G) * 16);
                        chunk_dot2<WF>(w1, x, a1, b1);
                        chunk_dot2<WF>(v1, y, c1, d1);
                    }
                }
                if (c < C) {
                    float4 x[Q];
#pragma unroll
                    for (int q = 0; q < Q; ++q) x[q] = x4[q * C + c];
                    const uint4 w = *reinterpret_cast<const uint4 *>(w0 + (size_t)c * 16);
                    chunk_dot2<WF>(w, x, a0, b0);
                    if (two) {
                        const uint4 w1 = *reinterpret_cast<const uint4 *>(w0 + g.stride + (size_t)c * 16);
                        chunk_dot2<WF>(w1, x, a1, b1);
                    }
                }
            }
            float s0 = ((a0.x + a0.y) + (b0.x + b0.y)) + ((c0.x + c0.y) + (d0.x + d0.y));
            float s1 = ((a1.x + a1.y) + (b1.x + b1.y)) + ((c1.x + c1.y) + (d1.x + d1.y));
#pragma unroll 1
            for (int off = (G < 32 ? G : 32) >> 1; off; off >>= 1) {
                s0 += __shfl_xor_sync(FULL, s0, off);
                s1 += __shfl_xor_sync(FULL, s1, off);
            }
            if (G > 32) {
                // A team of W = G / 32 warps (a long row over more lanes):
                // each warp's lane 0 leaves its sums in the team's scratch,
                // the team meets at its own barrier, and its first thread
                // adds them in warp order.  The second barrier frees the
                // scratch for the next round.
                const int W = G >> 5, wi = (t >> 5) & (W - 1);
                float *ts = tscr + 2 * W * tm;
                if (lane == 0) {
                    ts[2 * wi] = s0;
                    ts[2 * wi + 1] = s1;
                }
                team_sync(2 + tm, G);
                if (lt == 0) {
                    s0 = ts[0];
                    s1 = ts[1];
#pragma unroll 1
                    for (int w = 1; w < W; ++w) {
                        s0 += ts[2 * w];
                        s1 += ts[2 * w + 1];
                    }
                }
                team_sync(2 + tm, G);
            }
            if (act && lt == 0) {
                const int r = r0 + (two ? 2 * u : u);
                if (e.kind == EPI_GU) {
                    float gv = s0, uv = s1;
                    if (WF == WF_I8) {
                        gv = gv * e.rv[r];
                        uv = uv * e.rv[r + 1];
                    }
                    const float a = silu1(gv) * uv;
                    publish(e.out + (r >> 1), a);
                    flag_nonfinite(ctrl, gv);
                    flag_nonfinite(ctrl, a);
                } else {
                    epi_row(e, WF == WF_I8, n, r, s0, ctrl);
                    if (two && r + 1 < n) epi_row(e, WF == WF_I8, n, r + 1, s1, ctrl);
                }
            }
        }
        __syncwarp();
        if (lane == 0) {
            fence_proxy_async_smem();
            Cursor c = cur;
#pragma unroll 1
            for (int j = 0; j < ns; ++j) {
                mbar_arrive(rg.empty + c.slot);
                c.advance(rg.nslot);
            }
        }
        cur.slot += ns;
        if (cur.slot >= rg.nslot) { cur.slot -= rg.nslot; ++cur.round; }
        r0 += rows;
    }
    return cur;
}

// The LM head's stream: the CTA's table rows arrive slot by slot, and each
// slot (whole row pairs) is taken by one warp alone -- warp w < W reads
// slots w, w + W, ... -- so the slots' latencies overlap instead of every
// warp meeting at each wave.  W = min(NW, nslot): a warp then reaches a
// ring slot only after its previous use was filled, so the parity wait
// cannot match a phase two rounds old.  The warp frees its slot with all NW
// arrivals at once.  Per row pair: lanes stride the 16-byte chunks with four FP32
// chains, a shuffle butterfly, then lane 0 runs epi(row, y0, y1) (y1 of an
// odd tail row is discarded by the epilogue).
template <int TF, class Epi>
__device__ __forceinline__ void lm_stream(const DecodeParams &p, const Ring &rg, Cursor &cur, const KindGeom &g,
                                          int n, const float *xs, volatile int *s_abort, Epi &&epi) {
    constexpr int Q = Fmt<TF>::EPC / 4;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int C = g.C, rpc = g.rpc;
    const int nslots = (n + rpc - 1) / rpc, W = min(NW, rg.nslot);
    const float4 *x4 = reinterpret_cast<const float4 *>(xs);
#pragma unroll 1
    for (int k = warp; k < nslots && warp < W; k += W) {
        int s = cur.slot + k, rd = cur.round;
        while (s >= rg.nslot) { s -= rg.nslot; ++rd; }
        int ok = 1;
        if (lane == 0) ok = mbar_wait(p, rg.full + s, (uint32_t)(rd & 1), s_abort) ? 1 : 0;
        ok = __shfl_sync(FULL, ok, 0);
        __syncwarp();  // the rest of the warp reads after lane 0's acquire
        if (ok) {
            const uint8_t *base = rg.slots + (size_t)s * rg.slot_bytes;
            const int r0 = k * rpc, rows = min(rpc, n - r0);
#pragma unroll 1
            for (int u = 0; u < rows; u += 2) {
                const uint8_t *w0 = base + (size_t)u * g.stride;
                float2 a0 = make_float2(0.0f, 0.0f), b0 = a0, a1 = a0, b1 = a0;
#pragma unroll 1
                for (int c = lane; c < C; c += 32) {
                    float4 x[Q];
#pragma unroll
                    for (int q = 0; q < Q; ++q) x[q] = x4[q * C + c];
                    const uint4 w = *reinterpret_cast<const uint4 *>(w0 + (size_t)c * 16);
                    const uint4 w1 = *reinterpret_cast<const uint4 *>(w0 + g.stride + (size_t)c * 16);
                    chunk_dot2<TF>(w, x, a0, b0);
                    chunk_dot2<TF>(w1, x, a1, b1);
                }
                float s0 = (a0.x + a0.y) + (b0.x + b0.y), s1 = (a1.x + a1.y) + (b1.x + b1.y);
#pragma unroll
                for (int off = 16; off; off >>= 1) {
                    s0 += __shfl_xor_sync(FULL, s0, off);
                    s1 += __shfl_xor_sync(FULL, s1, off);
                }
                if (lane == 0) epi(r0 + u, s0, s1);
            }
        }
        __syncwarp();
        if (lane == 0) {
            fence_proxy_async_smem();
            mbar_arrive_cnt(rg.empty + s, NW);
        }
    }
    cur.slot += nslots;
    while (cur.slot >= rg.nslot) { cur.slot -= rg.nslot; ++cur.round; }
}

// ----------------------------------------------------------- exchange ----
//
// Phases hand their outputs to the CTAs that need them through exchange
// vectors instead of a grid barrier: each output word is published once per
// step with a relaxed store, and a consumer polls exactly the words it reads
// until none is kNotReady.  A 32-bit word is single-copy atomic, so a word
// that is not kNotReady is the producer's value; no fence or counter sits on
// the path.  Every CTA is co-resident (cooperative launch) and every phase
// only waits for outputs of the phase before it, so the polls end; each is
// bounded by the timeout all the same.

// Vector `off` of layer l in this step's exchange (xcur: its parity).
__device__ __forceinline__ float *xv(const DecodeParams &p, float *xcur, int l, int off) {
    return xcur + (size_t)l * p.xl + off;
}


// Resets this CTA's share of the other parity (the next step's exchange)
// to kNotReady; nothing reads or writes that parity during this step.  Run
// by the producer warp, off the compute path.
__device__ __forceinline__ void reset_next(const DecodeParams &p, unsigned par) {
    const size_t words = (size_t)p.L * p.xl;  // a multiple of 4
    uint4 *nx = reinterpret_cast<uint4 *>(p.xch + (size_t)(par ^ 1u) * words);
    const size_t n4 = words >> 2, G = gridDim.x, b = blockIdx.x;
    const size_t lo = n4 * b / G, hi = n4 * (b + 1) / G;
    const uint4 nr = make_uint4(kNotReady, kNotReady, kNotReady, kNotReady);
#pragma unroll 4
    for (size_t i = lo + (threadIdx.x & 31); i < hi; i += 32) nx[i] = nr;
}

// Poll bookkeeping of one thread: again() is true while the thread may poll
// once more; false after the timeout (ERR_TIMEOUT recorded, abort raised) or
// once this CTA or another one is aborting.  The clock and the flags are
// read every 64 polls.
struct Poll {
    uint64_t t0 = 0;
    unsigned it = 0;
    __device__ __forceinline__ bool again(const DecodeParams &p, volatile int *s_abort) {
        if (it++ == 0) {
            t0 = globaltimer_ns();
            return true;
        }
        if ((it & 63u) != 0) return true;
        if (*s_abort || (*(volatile unsigned *)&p.ctrl->error & ERR_TIMEOUT) ||
            globaltimer_ns() - t0 > p.timeout_ns) {
            atomicOr(&p.ctrl->error, ERR_TIMEOUT);
            *s_abort = 1;
            return false;
        }
        return true;
    }
};

__device__ __forceinline__ bool ready2(const uint2 &v) { return v.x != kNotReady && v.y != kNotReady; }
__device__ __forceinline__ bool ready4(const uint4 &v) {
    return v.x != kNotReady && v.y != kNotReady && v.z != kNotReady && v.w != kNotReady;
}

// One exchange word, polled until ready.
__device__ __forceinline__ float await1(const DecodeParams &p, const float *a, volatile int *s_abort) {
    uint32_t v = ld_relaxed_b32(a);
    Poll pl;
#pragma unroll 1
    while (v == kNotReady && pl.again(p, s_abort)) v = ld_relaxed_b32(a);
    return __uint_as_float(v);
}

// Four exchange words, all loads in flight at once; a pass reloads only the
// words still missing.
__device__ __forceinline__ void await4(const DecodeParams &p, const float *a0, const float *a1, const float *a2,
                                       const float *a3, float &o0, float &o1, float &o2, float &o3,
                                       volatile int *s_abort) {
    uint32_t v0 = ld_relaxed_b32(a0), v1 = ld_relaxed_b32(a1), v2 = ld_relaxed_b32(a2), v3 = ld_relaxed_b32(a3);
    Poll pl;
#pragma unroll 1
    while ((v0 == kNotReady || v1 == kNotReady || v2 == kNotReady || v3 == kNotReady) && pl.again(p, s_abort)) {
        if (v0 == kNotReady) v0 = ld_relaxed_b32(a0);
        if (v1 == kNotReady) v1 = ld_relaxed_b32(a1);
        if (v2 == kNotReady) v2 = ld_relaxed_b32(a2);
        if (v3 == kNotReady) v3 = ld_relaxed_b32(a3);
    }
    o0 = __uint_as_float(v0);
    o1 = __uint_as_float(v1);
    o2 = __uint_as_float(v2);
    o3 = __uint_as_float(v3);
}

// dst[i] = src[i], i < n, from an exchange vector (16 bytes per load when
// n % 4 == 0 and src is 16-byte aligned); acc gathers the statistics of
// the elements this thread staged (for norm_staged).
__device__ __forceinline__ void await_stage(const DecodeParams &p, float *dst, const float *src, int n,
                                            volatile int *s_abort, NormAcc &acc) {
    if ((n & 3) == 0 && ((uintptr_t)src & 15) == 0) {
        const uint4 *s4 = reinterpret_cast<const uint4 *>(src);
        uint4 *d4 = reinterpret_cast<uint4 *>(dst);
#pragma unroll 1
        for (int i = threadIdx.x; i < (n >> 2); i += NT) {
            uint4 v = ld_relaxed_v4(s4 + i);
            Poll pl;
#pragma unroll 1
            while (!ready4(v) && pl.again(p, s_abort)) v = ld_relaxed_v4(s4 + i);
            d4[i] = v;
            acc.add(__uint_as_float(v.x));
            acc.add(__uint_as_float(v.y));
            acc.add(__uint_as_float(v.z));
            acc.add(__uint_as_float(v.w));
        }
    } else {
#pragma unroll 1
        for (int i = threadIdx.x; i < n; i += NT) {
            const float v = await1(p, src + i, s_abort);
            dst[i] = v;
            acc.add(v);
        }
    }
}

// End of a phase: every compute thread is done with the phase's shared
// vectors (the next phase's prep overwrites them), and the trace records
// the CTA's finish.  False when aborting (uniform after the CTA barrier).
__device__ __forceinline__ bool phase_end(const DecodeParams &p, int idx, volatile int *s_abort) {
    csync();
    if (p.trace && threadIdx.x == 0) p.trace[(size_t)idx * gridDim.x + blockIdx.x] = globaltimer_ns();
    return *s_abort == 0;
}

// Trace mark: this CTA holds the inputs of the phase after phase idx.
__device__ __forceinline__ void mark_ready(const DecodeParams &p, int idx) {
    if (p.trace && idx >= 0 && threadIdx.x == 0)
        p.trace[((size_t)4 * p.L + idx) * gridDim.x + blockIdx.x] = globaltimer_ns();
}

// --------------------------------------------------------- elementwise ----

__device__ __forceinline__ float round_bf16(float x) {
    return __uint_as_float((uint32_t)f32_to_bf16_rne(x) << 16);
}

// Element i of the token's embedding row (the residual input of layer 0).
__device__ __forceinline__ float emb_in(const DecodeParams &p, int token, int i) {
    const uint8_t *row = p.emb + (size_t)token * p.semb;
    return p.tfmt == WF_BF16 ? bf16_to_f32(((const uint16_t *)row)[i]) : ((const float *)row)[i];
}

// h2 = x + o_proj(ctx) (src/kv_cache.rs:405-406): h2 already holds the
// layer's input x (staged by the QKV phase); the per-head partials are
// polled from the exchange, summed in head order, then added.  All of a
// batch's partials are in flight at once; a pass reloads only the missing.
__device__ __forceinline__ void stage_after_attention(const DecodeParams &p, float *xcur, int l, float *h2,
                                                      volatile int *s_abort, NormAcc &acc) {
    const float *part = xv(p, xcur, l, p.x_part);
    const size_t stride = (size_t)p.h;
    if ((p.h & 1) == 0) {
        // 8-byte loads: two consecutive elements per thread and pass, up to
        // 14 heads per batch (more would spill registers).
        constexpr int HB = 14;
#pragma unroll 1
        for (int i = threadIdx.x; i < (p.h >> 1); i += NT) {
            const uint2 *part2 = reinterpret_cast<const uint2 *>(part) + i;
            const int s2 = p.h >> 1;
            float2 o = make_float2(0.0f, 0.0f);
#pragma unroll 1
            for (int h0 = 0; h0 < p.qh; h0 += HB) {
                uint2 v[HB];
#pragma unroll
                for (int k = 0; k < HB; ++k)
                    if (h0 + k < p.qh) v[k] = ld_relaxed_v2(part2 + (h0 + k) * s2);
                Poll pl;
#pragma unroll 1
                for (;;) {
                    bool all = true;
#pragma unroll
                    for (int k = 0; k < HB; ++k)
                        if (h0 + k < p.qh && !ready2(v[k])) {
                            all = false;
                            v[k] = ld_relaxed_v2(part2 + (h0 + k) * s2);
                        }
                    if (all || !pl.again(p, s_abort)) break;
                }
#pragma unroll
                for (int k = 0; k < HB; ++k) {
                    if (h0 + k < p.qh) {
                        const float2 f = make_float2(__uint_as_float(v[k].x), __uint_as_float(v[k].y));
                        if (h0 + k == 0) o = f;
                        else { o.x = o.x + f.x; o.y = o.y + f.y; }
                    }
                }
            }
            float2 *h2v = reinterpret_cast<float2 *>(h2) + i;
            const float2 r = *h2v;
            const float2 y = make_float2(r.x + o.x, r.y + o.y);
            *h2v = y;
            acc.add(y.x);
            acc.add(y.y);
        }
        return;
    }
#pragma unroll 1
    for (int i = threadIdx.x; i < p.h; i += NT) {
        float o = 0.0f;
#pragma unroll 1
        for (int hh = 0; hh < p.qh; ++hh) {
            const float v = await1(p, part + (size_t)hh * stride + i, s_abort);
            o = hh == 0 ? v : o + v;
        }
        const float y = h2[i] + o;
        h2[i] = y;
        acc.add(y);
    }
}


// Element offset of the row of (KV head g, position q) in a layer's page
// pool; `ptab` is the page table staged in shared memory.
__device__ __forceinline__ size_t kv_row(const DecodeParams &p, const int *ptab, int g, int q) {
    return (((size_t)ptab[q / kPageTokens] * p.kvh + g) * kPageTokens + (q % kPageTokens)) * (size_t)p.hd;
}

template <int KVBF16>
__device__ __forceinline__ float kv_load(const uint8_t *base, size_t idx) {
    if (KVBF16) return bf16_to_f32(__ldcg((const unsigned short *)base + idx));
    return __ldcg((const float *)base + idx);
}

// Attention for query head hh at position pos (src/kv_cache.rs:550-576).
// Leaves the context vector in xs (quad-major for the o_proj rows,
// zero-padded).  The first CTA of a KV group writes the new K (rotated) and
// V at `pos`.  Scores keep the reference's order (q.k summed by increasing
// index, then divided by sqrt(hd)); softmax subtracts the maximum and
// divides by the sum.
// Per-head barrier of the attention splits: every split has written its
// partial before any reads them (a release reduction on a per-head counter,
// acquire polling bounded by the timeout).  Returns false when aborting.
__device__ __forceinline__ bool head_barrier(const DecodeParams &p, int hh, unsigned target, volatile int *s_abort) {
    csync();
    if (threadIdx.x == 0) {
        red_release_add_u32(p.hbar + hh, 1u);
        if (ld_acquire_u32(p.hbar + hh) < target) {
            const uint64_t t0 = globaltimer_ns();
            unsigned spins = 0;
            while (ld_acquire_u32(p.hbar + hh) < target) {
                if ((++spins & 63u) == 0) {
                    if ((*(volatile unsigned *)&p.ctrl->error & ERR_TIMEOUT) || globaltimer_ns() - t0 > p.timeout_ns) {
                        atomicOr(&p.ctrl->error, ERR_TIMEOUT);
                        *s_abort = 1;
                        break;
                    }
                }
            }
        }
    }
    csync();
    return *s_abort == 0;
}

// Attention of query head hh over positions [lo, hi) of 0..pos.  Without a
// split (lo = 0, hi = pos + 1) the weights are divided by the sum and the
// context lands in xs.  With a split (vectorised layouts only) the warps'
// unnormalized context sums stay in red[2 NW + w hd + i], with the maximum
// at red[2 NW + NW hd] and the sum after it, for split_exchange.
// q, k and v come from the exchange (qkv: this layer's QKV outputs); `mark`
// is the trace index recorded once they are staged (-1: none).
template <int WF, int KVBF16>
__device__ __forceinline__ void attention_context(const DecodeParams &p, const DecodeLayer &Ly, const float *qkv,
                                                  int hh, bool writer, int pos, float *sm, int lo, int hi, int mark,
                                                  volatile int *s_abort) {
    const bool split = hi - lo < pos + 1;
    constexpr int EPC = Fmt<WF>::EPC;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int hd = p.hd, half = hd / 2, g = hh / p.group;
    const size_t kvw = (size_t)p.kvh * hd;
    float *qs = sm + p.sm_q, *ks = qs + hd, *vs = ks + hd;
    float *sc = sm + p.sm_sc, *red = sm + p.sm_red, *xs = sm + p.sm_xs;
    // q and k rotated with the host table (threads [0, NT/2)), v (threads
    // [NT/2, NT)); every load is issued before its first use.
    if (t < NT / 2) {
        const float2 *rp = p.rope + (size_t)pos * half;
#pragma unroll 1
        for (int j = t; j < half; j += NT / 2) {
            const float2 cs = rp[j];
            const float *qa = qkv + (size_t)hh * hd + j, *kq = qkv + p.h + (size_t)g * hd + j;
            float a, b, ka, kb;
            await4(p, qa, qa + half, kq, kq + half, a, b, ka, kb, s_abort);
            qs[j] = a * cs.x - b * cs.y;
            qs[j + half] = b * cs.x + a * cs.y;
            float k0 = ka * cs.x - kb * cs.y, k1 = kb * cs.x + ka * cs.y;
            if (KVBF16) { k0 = round_bf16(k0); k1 = round_bf16(k1); }
            ks[j] = k0;
            ks[j + half] = k1;
        }
    } else {
#pragma unroll 1
        for (int i = t - NT / 2; i < hd; i += NT / 2) {
            const float v = await1(p, qkv + p.h + kvw + (size_t)g * hd + i, s_abort);
            vs[i] = KVBF16 ? round_bf16(v) : v;
        }
    }
    csync();
    mark_ready(p, mark);
#pragma unroll 1
    for (int i = t; i < hd; i += NT)
        if (!isfinite(qs[i]) || !isfinite(ks[i])) atomicOr(&p.ctrl->error, ERR_NONFINITE);
    const size_t esz = KVBF16 ? 2 : 4;
    const int *ptab = (const int *)(sm + p.sm_ptab);
    const uint8_t *K = Ly.kc, *Vc = Ly.vc;  // page pools; rows at kv_row()
    if (writer) {
#pragma unroll 1
        for (int i = t; i < hd; i += NT) {
            const size_t idx = kv_row(p, ptab, g, pos) + i;
            if (KVBF16) {
                ((uint16_t *)Ly.kc)[idx] = f32_to_bf16_rne(ks[i]);
                ((uint16_t *)Ly.vc)[idx] = f32_to_bf16_rne(vs[i]);
            } else {
                ((float *)Ly.kc)[idx] = ks[i];
                ((float *)Ly.vc)[idx] = vs[i];
            }
        }
    }
    // Scores.  TP = max(1, chunks / 4) adjacent lanes share a position: each
    // loads up to four 16-byte chunks of the key row (all in flight at
    // once) and sums its part in index order; the parts meet by shuffles.
    const int row_bytes = hd * (int)esz;
    const int nc = row_bytes >> 4;
    const bool vec = (row_bytes & 15) == 0 && nc <= 128 && (nc & (nc - 1)) == 0;
    constexpr int KEPC = KVBF16 ? 8 : 4;  // cache elements per 16-byte chunk
    const int tpl = vec && nc > 4 ? 31 - __clz(nc >> 2) : 0;
    const int TP = 1 << tpl, sub = t & (TP - 1), PPP = NT >> tpl;
    float mt = -INFINITY;
#pragma unroll 1
    for (int qb = lo; qb < hi; qb += PPP) {
        const int q = qb + (t >> tpl);
        float s = 0.0f;
        if (q >= hi) {
        } else if (q == pos) {
            if (sub == 0) {
#pragma unroll 4
                for (int i = 0; i < hd; ++i) s = s + qs[i] * ks[i];
            }
        } else if (q < pos) {
            if (vec) {
                const uint8_t *row = K + kv_row(p, ptab, g, q) * esz;
                const int c0 = sub * 4;
                uint4 kc[4];
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    if (c0 + c < nc) kc[c] = __ldcg((const uint4 *)(row + (size_t)(c0 + c) * 16));
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    if (c0 + c < nc) {
                        const uint32_t w4[4] = {kc[c].x, kc[c].y, kc[c].z, kc[c].w};
                        const float *qq = qs + (c0 + c) * KEPC;
#pragma unroll
                        for (int e = 0; e < KEPC; ++e) {
                            const float kv = KVBF16 ? ((e & 1) ? bf16_hi(w4[e >> 1]) : bf16_lo(w4[e >> 1]))
                                                    : __uint_as_float(w4[e]);
                            s = s + qq[e] * kv;
                        }
                    }
                }
            } else {
#pragma unroll 1
                for (int i = 0; i < hd; ++i) s = s + qs[i] * kv_load<KVBF16>(K, kv_row(p, ptab, g, q) + i);
            }
        }
#pragma unroll 1
        for (int off = TP >> 1; off; off >>= 1) s += __shfl_xor_sync(FULL, s, off);
        if (sub == 0 && q < hi) {
            s = s / p.sqrt_hd;
            sc[q] = s;
            mt = rust_max(mt, s);
        }
    }
    // Softmax: maximum and sum each meet through one shared array of warp
    // partials, read in warp order by every thread.
    mt = warp_max(mt);
    if (lane == 0) red[warp] = mt;
    csync();
    float m = red[0];
#pragma unroll
    for (int w = 1; w < NW; ++w) m = rust_max(m, red[w]);
    float st = 0.0f;
#pragma unroll 1
    for (int q = lo + t; q < hi; q += NT) {
        const float e = expf(sc[q] - m);
        sc[q] = e;
        st += e;
    }
    st = warp_sum(st);
    if (lane == 0) red[NW + warp] = st;
    csync();
    float se = red[NW];
#pragma unroll
    for (int w = 1; w < NW; ++w) se += red[NW + w];
    // Context: thread t takes chunk c = t % nc of the value rows of the
    // positions q = pg, pg + PG, ... (pg = t / nc); the position groups meet
    // by shuffles inside the warp, then across warps in warp order.
    const int ctx_pad = p.chd * EPC;
    if (vec && nc <= 32 && (nc & (nc - 1)) == 0) {
        const int PG = NT / nc;
        const int c = t & (nc - 1), pg = t / nc;
        float acc[KEPC];
#pragma unroll
        for (int e = 0; e < KEPC; ++e) acc[e] = 0.0f;
#pragma unroll 1
        for (int q0 = lo + pg; q0 < hi; q0 += 4 * PG) {
            uint4 vc[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int q = q0 + u * PG;
                if (q < pos && q < hi) vc[u] = __ldcg((const uint4 *)(Vc + kv_row(p, ptab, g, q) * esz + (size_t)c * 16));
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int q = q0 + u * PG;
                if (q < hi) {
                    const float pr = split ? sc[q] : sc[q] / se;
                    const uint32_t w4[4] = {vc[u].x, vc[u].y, vc[u].z, vc[u].w};
#pragma unroll
                    for (int e = 0; e < KEPC; ++e) {
                        const float v = q == pos ? vs[c * KEPC + e]
                                                 : (KVBF16 ? ((e & 1) ? bf16_hi(w4[e >> 1]) : bf16_lo(w4[e >> 1]))
                                                           : __uint_as_float(w4[e]));
                        acc[e] = acc[e] + pr * v;
                    }
                }
            }
        }
#pragma unroll 1
        for (int off = nc; off < 32; off <<= 1) {
#pragma unroll
            for (int e = 0; e < KEPC; ++e) acc[e] += __shfl_xor_sync(FULL, acc[e], off);
        }
        if (lane < nc) {
#pragma unroll
            for (int e = 0; e < KEPC; ++e) red[2 * NW + warp * hd + c * KEPC + e] = acc[e];
        }
        csync();
        if (split) {
            if (t == 0) {
                red[2 * NW + NW * hd] = m;
                red[2 * NW + NW * hd + 1] = se;
            }
            csync();
            return;
        }
#pragma unroll 1
        for (int i = t; i < ctx_pad; i += NT) {
            float s = 0.0f;
            if (i < hd) {
                s = red[2 * NW + i];
#pragma unroll
                for (int w = 1; w < NW; ++w) s += red[2 * NW + w * hd + i];
                flag_nonfinite(p.ctrl, s);
            }
            xs[xq<EPC>(i, p.chd)] = s;
        }
    } else {
        // General layout: one thread per output element, positions in order.
#pragma unroll 1
        for (int i = t; i < ctx_pad; i += NT) {
            float s = 0.0f;
            if (i < hd) {
#pragma unroll 1
                for (int q = 0; q <= pos; ++q) {
                    const float v = q == pos ? vs[i] : kv_load<KVBF16>(Vc, kv_row(p, ptab, g, q) + i);
                    s = s + (sc[q] / se) * v;
                }
                flag_nonfinite(p.ctrl, s);
            }
            xs[xq<EPC>(i, p.chd)] = s;
        }
    }
    csync();
}

// ------------------------------------------------------------ phases ----
//
// Each phase has a `prep` that stages its small read-only vectors -- norm
// gains and row scales and biases -- into shared memory, and a `run` that
// polls the phase's inputs from the exchange, computes and publishes.  The
// weights arrive through the ring.  A phase's prep is issued (cp.async) at
// the start of the phase before it, into the other half of two double
// buffers: gains in gain buffer 0 (QKV, final norm) or 1 (gate/up); scales
// and biases in rv buffer 0 (QKV, gate/up) or 1 (attention, down).

__device__ __forceinline__ float *gain_buf(const DecodeParams &p, float *sm, int b) {
    return sm + p.sm_gain + b * p.sm_gain_n;
}
__device__ __forceinline__ float *rv_buf(const DecodeParams &p, float *sm, int b) {
    return sm + p.sm_rv + b * p.sm_rv_n;
}

template <int WF>
__device__ __forceinline__ void prep_qkv(const DecodeParams &p, const DecodeLayer &Ly, const CtaGeom &cg,
                                         float *sm) {
    float *rv = rv_buf(p, sm, 0);
    stage_async(gain_buf(p, sm, 0), Ly.attn_norm, p.h);
    if (WF == WF_I8) stage_async(rv, Ly.sqkv + cg.qkv_r0, cg.qkv_n);
    stage_async(rv + cg.qkv_n, Ly.bqkv + cg.qkv_r0, cg.qkv_n);
}

template <int WF>
__device__ __forceinline__ void run_qkv(const DecodeParams &p, const CtaGeom &cg, float *xcur, int l, int token,
                                        float *sm, const Ring &rg, Cursor &cur, volatile int *s_abort) {
    constexpr int EPC = Fmt<WF>::EPC;
    float *xs = sm + p.sm_xs, *h2 = sm + p.sm_h2;
    const float *gain = gain_buf(p, sm, 0), *rv = rv_buf(p, sm, 0);
    ring_prewait(p, rg, cur, p.kind[K_QKV], cg.qkv_n, s_abort);
    NormAcc acc;
    if (l > 0) {
        await_stage(p, h2, xv(p, xcur, l - 1, p.x_hid), p.h, s_abort, acc);
    } else {
#pragma unroll 2
        for (int i = threadIdx.x; i < p.h; i += NT) {
            const float v = emb_in(p, token, i);
            h2[i] = v;
            acc.add(v);
        }
    }
    mark_ready(p, 4 * l - 1);
    norm_staged<EPC>(h2, gain, xs, p.h, p.ch, p.eps, sm + p.sm_red, acc);
    if (*s_abort) return;
    const Epi e{xv(p, xcur, l, p.x_qkv) + cg.qkv_r0, rv, nullptr, EPI_QKV,
                !(p.withhold && l == 0 && blockIdx.x == 0)};
    cur = gemv_pairs<WF>(p, rg, cur, p.kind[K_QKV], cg.qkv_n, xs, s_abort, e, true, sm + p.sm_red);
}

// The position-split exchange of head hh (split sp of nsp, layer l): this
// split's partial (context sums, maximum, sum) to its slot, the head
// barrier, then every split combines all slots in slot order, rescaled by
// exp(m_j - m), into xs.  Returns false when aborting.
template <int WF>
__device__ __forceinline__ bool split_exchange(const DecodeParams &p, int hh, int sp, int nsp, int l, float *sm,
                                            volatile int *s_abort) {
    constexpr int EPC = Fmt<WF>::EPC;
    const int t = threadIdx.x, hd = p.hd;
    const float *red = sm + p.sm_red;
    float *xs = sm + p.sm_xs;
    float *mine = p.apart + ((size_t)hh * nsp + sp) * (hd + 2);
#pragma unroll 1
    for (int i = t; i < hd + 2; i += NT) {
        float v;
        if (i < hd) {
            v = red[2 * NW + i];
#pragma unroll
            for (int w = 1; w < NW; ++w) v += red[2 * NW + w * hd + i];
        } else {
            v = red[2 * NW + NW * hd + (i - hd)];
        }
        mine[i] = v;
    }
    if (!head_barrier(p, hh, (unsigned)((l + 1) * nsp), s_abort)) return false;
    const float *all = p.apart + (size_t)hh * nsp * (hd + 2);
    // Lane j of every warp loads split j's (maximum, sum) (nsp <=
    // kMaxSplits <= 32); the rescale factors exp(m_j - M) and the combined
    // sum follow in split order.
    const int lane = t & 31;
    float mj = -INFINITY, lj = 0.0f;
    if (lane < nsp) {
        mj = __ldcg(all + (size_t)lane * (hd + 2) + hd);
        lj = __ldcg(all + (size_t)lane * (hd + 2) + hd + 1);
    }
    const float M = warp_max(mj);
    const float f = lane < nsp && lj > 0.0f ? expf(mj - M) : 0.0f;
    float fj[kMaxSplits];
    float Lsum = 0.0f;
#pragma unroll
    for (int j = 0; j < kMaxSplits; ++j) {
        fj[j] = __shfl_sync(FULL, f, j);
        const float l = __shfl_sync(FULL, lj, j);
        if (j < nsp) Lsum += l * fj[j];
    }
    const int ctx_pad = p.chd * EPC;
#pragma unroll 1
    for (int i = t; i < ctx_pad; i += NT) {
        float s = 0.0f;
        if (i < hd) {
            float oj[kMaxSplits];
#pragma unroll
            for (int j = 0; j < kMaxSplits; ++j)
                if (j < nsp) oj[j] = __ldcg(all + (size_t)j * (hd + 2) + i);
            float o = 0.0f;
#pragma unroll
            for (int j = 0; j < kMaxSplits; ++j)
                if (j < nsp) o += oj[j] * fj[j];
            s = o / Lsum;
            flag_nonfinite(p.ctrl, s);
        }
        xs[xq<EPC>(i, p.chd)] = s;
    }
    csync();
    return true;
}

template <int WF>
__device__ __forceinline__ void prep_attention(const DecodeParams &p, const DecodeLayer &Ly, const CtaGeom &cg,
                                               float *sm) {
    if (WF == WF_I8 && cg.natt > 0) stage_async(rv_buf(p, sm, 1), Ly.so + cg.att_r0[0], cg.att_n[0]);
}

template <int WF, int KVBF16, int SPLIT>
__device__ __forceinline__ void run_attention(const DecodeParams &p, const DecodeLayer &Ly, const CtaGeom &cg,
                                              float *xcur, int l, int pos, float *sm, const Ring &rg, Cursor &cur,
                                              volatile int *s_abort) {
    const float *rv = rv_buf(p, sm, 1), *xs = sm + p.sm_xs;
    if (cg.natt > 0) ring_prewait(p, rg, cur, p.kind[K_O], cg.att_n[0], s_abort);
#pragma unroll 1
    for (int a = 0; a < cg.natt; ++a) {
        const int hh = cg.att_hh[a], r0 = cg.att_r0[a], n = cg.att_n[a];
        const int nsp = att_nsp<SPLIT>(p, pos);
        const int sp = cg.att_sp[a];
        const int lo = nsp > 1 ? (int)((long long)(pos + 1) * sp / nsp) : 0;
        const int hi = nsp > 1 ? (int)((long long)(pos + 1) * (sp + 1) / nsp) : pos + 1;
        attention_context<WF, KVBF16>(p, Ly, xv(p, xcur, l, p.x_qkv), hh, r0 == 0 && hh % p.group == 0, pos, sm,
                                      lo, hi, a == 0 ? 4 * l : -1, s_abort);
        if (SPLIT && nsp > 1 && !split_exchange<WF>(p, hh, sp, nsp, l, sm, s_abort)) return;
        // Row scales: staged in shared memory for the first item, read from
        // global memory for the others.
        const Epi e{xv(p, xcur, l, p.x_part) + (size_t)hh * p.h + r0, a == 0 ? rv : Ly.so + r0, nullptr, EPI_O, 1};
        cur = gemv_pairs<WF>(p, rg, cur, p.kind[K_O], n, xs, s_abort, e, a == 0, sm + p.sm_red);
        if (a + 1 < cg.natt) csync();  // xs is rewritten by the next item
    }
}

template <int WF>
__device__ __forceinline__ void prep_gate_up(const DecodeParams &p, const DecodeLayer &Ly, const CtaGeom &cg,
                                             float *sm) {
    stage_async(gain_buf(p, sm, 1), Ly.ffn_norm, p.h);
    if (WF == WF_I8) stage_async(rv_buf(p, sm, 0), Ly.sgu + 2 * cg.gu_f0, 2 * cg.gu_n);
}

template <int WF>
__device__ __forceinline__ void run_gate_up(const DecodeParams &p, const CtaGeom &cg, float *xcur, int l, float *sm,
                                            const Ring &rg, Cursor &cur, volatile int *s_abort) {
    constexpr int EPC = Fmt<WF>::EPC;
    float *xs = sm + p.sm_xs, *h2 = sm + p.sm_h2;
    const float *gain = gain_buf(p, sm, 1), *rv = rv_buf(p, sm, 0);
    ring_prewait(p, rg, cur, p.kind[K_GU], 2 * cg.gu_n, s_abort);
    NormAcc acc;
    stage_after_attention(p, xcur, l, h2, s_abort, acc);
    mark_ready(p, 4 * l + 1);
    norm_staged<EPC>(h2, gain, xs, p.h, p.ch, p.eps, sm + p.sm_red, acc);
    if (*s_abort) return;
    if (blockIdx.x == 0)
        for (int i = threadIdx.x; i < p.h; i += NT) flag_nonfinite(p.ctrl, h2[i]);
    const Epi e{xv(p, xcur, l, p.x_act) + cg.gu_f0, rv, nullptr, EPI_GU, 1};
    cur = gemv_pairs<WF>(p, rg, cur, p.kind[K_GU], 2 * cg.gu_n, xs, s_abort, e, true, sm + p.sm_red);
}

template <int WF>
__device__ __forceinline__ void prep_down(const DecodeParams &p, const DecodeLayer &Ly, const CtaGeom &cg,
                                          float *sm) {
    if (WF == WF_I8) stage_async(rv_buf(p, sm, 1), Ly.sd + cg.dn_r0, cg.dn_n);
}

template <int WF>
__device__ __forceinline__ void run_down(const DecodeParams &p, const CtaGeom &cg, float *xcur, int l, float *sm,
                                         const Ring &rg, Cursor &cur, volatile int *s_abort) {
    constexpr int EPC = Fmt<WF>::EPC;
    float *xs = sm + p.sm_xs;
    const int padded = p.cff * EPC;
    const float *actv = xv(p, xcur, l, p.x_act);
    ring_prewait(p, rg, cur, p.kind[K_DN], cg.dn_n, s_abort);
    if ((p.ff & 3) == 0) {
        // act -> xs: four consecutive elements are one quad of the layout.
        const uint4 *a4 = reinterpret_cast<const uint4 *>(actv);
        uint4 *x4 = reinterpret_cast<uint4 *>(xs);
        constexpr int B4 = 4;
#pragma unroll 1
        for (int base = threadIdx.x; base < padded / 4; base += B4 * NT) {
            uint4 v[B4];
#pragma unroll
            for (int k = 0; k < B4; ++k) {
                const int e = 4 * (base + k * NT);
                v[k] = e < p.ff ? ld_relaxed_v4(a4 + (e >> 2)) : make_uint4(0u, 0u, 0u, 0u);
            }
            Poll pl;
#pragma unroll 1
            for (;;) {
                bool all = true;
#pragma unroll
                for (int k = 0; k < B4; ++k) {
                    const int e = 4 * (base + k * NT);
                    if (e < p.ff && !ready4(v[k])) {
                        all = false;
                        v[k] = ld_relaxed_v4(a4 + (e >> 2));
                    }
                }
                if (all || !pl.again(p, s_abort)) break;
            }
#pragma unroll
            for (int k = 0; k < B4; ++k) {
                const int e = 4 * (base + k * NT);
                if (e < padded) x4[((e % EPC) >> 2) * p.cff + e / EPC] = v[k];
            }
        }
    } else {
#pragma unroll 1
        for (int i = threadIdx.x; i < padded; i += NT) xs[xq<EPC>(i, p.cff)] = i < p.ff ? await1(p, actv + i, s_abort) : 0.0f;
    }
    csync();
    mark_ready(p, 4 * l + 2);
    if (*s_abort) return;
    // h' of this layer is still in shared memory from the gate/up phase of
    // this same CTA (src/kv_cache.rs:437-443: x_next = h' + down(a)).
    const float *h2 = sm + p.sm_h2 + cg.dn_r0, *rv = rv_buf(p, sm, 1);
    const Epi e{xv(p, xcur, l, p.x_hid) + cg.dn_r0, rv, h2, EPI_DN, 1};
    cur = gemv_pairs<WF>(p, rg, cur, p.kind[K_DN], cg.dn_n, xs, s_abort, e, true, sm + p.sm_red);
}

// Final RMSNorm, this CTA's rows of the (tied) table, logits and the CTA's
// argmax (lowest id on ties); the last CTA to finish reduces the grid.  The
// logits of all the CTA's rows land in `rowv`; warp 0 scans them in row
// order, so ties keep the lowest id.
template <int TF>
__device__ __forceinline__ void run_lm_head(const DecodeParams &p, const CtaGeom &cg, float *xcur, int pos,
                                            float *sm, const Ring &rg, Cursor &cur, volatile int *s_abort) {
    constexpr int TEPC = Fmt<TF>::EPC;
    const int G = gridDim.x, b = blockIdx.x;
    float *xs = sm + p.sm_xs, *h2 = sm + p.sm_h2;
    const float *gain = gain_buf(p, sm, 0);
    float *rowv = sm + p.sm_sc;
    DecodeCtrl *ctrl = p.ctrl;
    NormAcc acc;
    await_stage(p, h2, xv(p, xcur, p.L - 1, p.x_hid), p.h, s_abort, acc);
    mark_ready(p, 4 * p.L - 1);
    norm_staged<TEPC>(h2, gain, xs, p.h, p.cemb, p.eps, sm + p.sm_red, acc);
    if (*s_abort) return;
    const int nlm = cg.lm_n;
    lm_stream<TF>(p, rg, cur, p.kind[K_LM], nlm, xs, s_abort, [&](int r, float a0, float a1) {
        rowv[r] = a0;
        if (r + 1 < nlm) rowv[r + 1] = a1;
    });
    csync();
    if (*s_abort) return;
    if (ctrl->write_logits) {
        float *lg = p.logits + cg.lm_v0;
#pragma unroll 4
        for (int r = threadIdx.x; r < cg.lm_n; r += NT) lg[r] = rowv[r];
    }
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        float bv = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll 4
        for (int r = lane; r < cg.lm_n; r += 32) {
            const float v = rowv[r];
            if (!isfinite(v)) atomicOr(&ctrl->error, ERR_NONFINITE);
            if (v > bv) { bv = v; bi = r; }
        }
#pragma unroll
        for (int off = 16; off; off >>= 1) {
            const float ov = __shfl_xor_sync(FULL, bv, off);
            const int oi = __shfl_xor_sync(FULL, bi, off);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        unsigned tk = 0;
        if (lane == 0) {
            p.amax_v[b] = bv;
            p.amax_i[b] = bi == 0x7fffffff ? bi : cg.lm_v0 + bi;
            __threadfence();
            tk = atomicAdd(&ctrl->ticket, 1u);
        }
        tk = __shfl_sync(FULL, tk, 0);
        if (tk == (unsigned)G - 1) {
            // The last CTA: its warp 0 reduces the per-CTA partials, every
            // lane's loads in flight at once, then a butterfly (the maximum,
            // the lowest id among equal values).
            __syncwarp();
            __threadfence();
            float gv = -INFINITY;
            int gi = 0x7fffffff;
#pragma unroll 4
            for (int k = lane; k < G; k += 32) {
                const float v = __ldcg(p.amax_v + k);
                const int i = __ldcg(p.amax_i + k);
                if (v > gv || (v == gv && i < gi)) { gv = v; gi = i; }
            }
#pragma unroll
            for (int off = 16; off; off >>= 1) {
                const float ov = __shfl_xor_sync(FULL, gv, off);
                const int oi = __shfl_xor_sync(FULL, gi, off);
                if (ov > gv || (ov == gv && oi < gi)) { gv = ov; gi = oi; }
            }
            if (lane == 0) {
                if (gi < 0 || gi >= p.V) gi = 0;
                ctrl->next_token = gi;
                if (p.emitted) p.emitted[pos] = gi;
                ctrl->token = gi;
                ctrl->pos = pos + 1;
                ctrl->epoch = ctrl->epoch + 1u;
                ctrl->ticket = 0;
                if (p.hbar)
                    for (int k = 0; k < p.qh; ++k) p.hbar[k] = 0u;
                if (p.trace) p.trace[(size_t)8 * p.L * G + 1] = globaltimer_ns();
                __threadfence();
            }
        }
    }
}

// ------------------------------------------------------------ kernel ----

template <int WF, int TF, int KVBF16, int SPLIT>
// Four warps per sub-partition x 32 threads x 128 registers = its 16K registers.
__global__ void __maxnreg__(128) decode_kernel(const __grid_constant__ DecodeParams p) {
    extern __shared__ __align__(128) float sm[];
    __shared__ int s_abort_storage;
    volatile int *s_abort = &s_abort_storage;
    const int G = gridDim.x, b = blockIdx.x;
    DecodeCtrl *ctrl = p.ctrl;
    const int token = *(volatile int *)&ctrl->token;
    const int pos = *(volatile int *)&ctrl->pos;
    const unsigned par = *(volatile unsigned *)&ctrl->epoch & 1u;
    float *const xcur = p.xch + (size_t)par * p.L * p.xl;
    const int NB = 4 * p.L;
    // This CTA's row ranges live in shared memory for the whole step (a
    // global copy would be re-read from L2 on the critical path).
    __shared__ CtaGeom s_cg;
    const CtaGeom &cg = s_cg;
    if (threadIdx.x < (int)(sizeof(CtaGeom) / 4))
        ((int *)&s_cg)[threadIdx.x] = ((const int *)(p.geom + b))[threadIdx.x];
    if (p.trace && b == 0 && threadIdx.x == 0) p.trace[(size_t)2 * NB * G] = globaltimer_ns();
    // The layer table lives in shared memory for the whole step.
    DecodeLayer *lay = (DecodeLayer *)(sm + p.sm_lay);
    {
        const uint32_t *src = (const uint32_t *)p.layers;
        uint32_t *dst = (uint32_t *)lay;
        const int words = p.L * (int)(sizeof(DecodeLayer) / 4);
#pragma unroll 1
        for (int i = threadIdx.x; i < words; i += kDecodeBlock) dst[i] = src[i];
    }
    // The page table entries of the pages that hold positions 0 .. pos.
    {
        int *sp = (int *)(sm + p.sm_ptab);
        const int np = pos / kPageTokens + 1;
#pragma unroll 1
        for (int i = threadIdx.x; i < np; i += kDecodeBlock) sp[i] = __ldg(p.ptab + i);
    }
    const Ring rg = ring_of(p, sm);
    if (threadIdx.x == 0) {
        for (int i = 0; i < p.nslot; ++i) {
            mbar_init(rg.full + i, 1);
            mbar_init(rg.empty + i, NW);
        }
        fence_mbar_init();
        *s_abort = 0;
    }
    __syncthreads();  // the only all-thread barrier: roles split here

    if (threadIdx.x >= NT) {  // producer warp
        reset_next(p, par);
        produce(p, lay, cg, sm, pos, s_abort);
        return;
    }

    Cursor cur{0, 0};
    prep_qkv<WF>(p, lay[0], cg, sm);
    cp_async_commit();
    bool ok = true;
    // Each phase: wait for its own small read-only vectors (issued one
    // phase earlier), issue the next phase's, poll its inputs from the
    // exchange, run, publish.  Every exit decision is taken right after a
    // CTA barrier, so all compute threads agree on it.
#pragma unroll 1
    for (int l = 0; l < p.L && ok; ++l) {
        const DecodeLayer &Ly = lay[l];
        cp_async_wait_all();
        prep_attention<WF>(p, Ly, cg, sm);
        cp_async_commit();
        run_qkv<WF>(p, cg, xcur, l, token, sm, rg, cur, s_abort);
        if (!(ok = phase_end(p, 4 * l, s_abort))) break;
        cp_async_wait_all();
        prep_gate_up<WF>(p, Ly, cg, sm);
        cp_async_commit();
        run_attention<WF, KVBF16, SPLIT>(p, Ly, cg, xcur, l, pos, sm, rg, cur, s_abort);
        if (!(ok = phase_end(p, 4 * l + 1, s_abort))) break;
        cp_async_wait_all();
        prep_down<WF>(p, Ly, cg, sm);
        cp_async_commit();
        run_gate_up<WF>(p, cg, xcur, l, sm, rg, cur, s_abort);
        if (!(ok = phase_end(p, 4 * l + 2, s_abort))) break;
        cp_async_wait_all();
        if (l + 1 < p.L) prep_qkv<WF>(p, lay[l + 1], cg, sm);
        else stage_async(gain_buf(p, sm, 0), p.final_norm, p.h);
        cp_async_commit();
        run_down<WF>(p, cg, xcur, l, sm, rg, cur, s_abort);
        if (!(ok = phase_end(p, 4 * l + 3, s_abort))) break;
    }
    cp_async_wait_all();  // nothing lands in shared memory after an early exit
    if (ok) run_lm_head<TF>(p, cg, xcur, pos, sm, rg, cur, s_abort);
}

size_t decode_smem_bytes(const DecodeParams &p) { return (size_t)p.sm_total * sizeof(float); }

template <int WF, int TF, int KV>
static cudaError_t launch_t(const DecodeParams &p, int grid, cudaStream_t stream, bool split) {
    auto kern = split ? decode_kernel<WF, TF, KV, 1> : decode_kernel<WF, TF, KV, 0>;
    size_t smem = decode_smem_bytes(p);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kDecodeBlock);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int WF, int TF, int KV>
static const void *kernel_ptr(bool split) {
    return split ? (const void *)decode_kernel<WF, TF, KV, 1> : (const void *)decode_kernel<WF, TF, KV, 0>;
}

// Dispatch over (linear format, table format, KV type).
template <class F>
static auto dispatch(int wf, int tf, int kv, F f) {
#define QB_CASE(W, T, K) \
    if (wf == W && tf == T && kv == K) return f.template operator()<W, T, K>();
    QB_CASE(WF_F32, WF_F32, 0) QB_CASE(WF_F32, WF_F32, 1) QB_CASE(WF_F32, WF_BF16, 0) QB_CASE(WF_F32, WF_BF16, 1)
    QB_CASE(WF_BF16, WF_F32, 0) QB_CASE(WF_BF16, WF_F32, 1) QB_CASE(WF_BF16, WF_BF16, 0) QB_CASE(WF_BF16, WF_BF16, 1)
    QB_CASE(WF_I8, WF_F32, 0) QB_CASE(WF_I8, WF_F32, 1) QB_CASE(WF_I8, WF_BF16, 0)
#undef QB_CASE
    return f.template operator()<WF_I8, WF_BF16, 1>();
}

struct LaunchOp {
    const DecodeParams &p;
    int grid;
    cudaStream_t stream;
    bool split;
    template <int W, int T, int K> cudaError_t operator()() const { return launch_t<W, T, K>(p, grid, stream, split); }
};
struct PtrOp {
    bool split;
    template <int W, int T, int K> const void *operator()() const { return kernel_ptr<W, T, K>(split); }
};

cudaError_t decode_launch(const DecodeParams &p, int grid, cudaStream_t stream, bool split) {
    return dispatch(p.wfmt, p.tfmt, p.kv_bf16, LaunchOp{p, grid, stream, split});
}

// Largest number of co-resident CTAs of the decode kernel on this device.
int decode_max_ctas(int wfmt, int tfmt, int kv_bf16, size_t smem) {
    int dev = 0, sms = 0, per = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int lowest = 1 << 30;
    for (int split = 0; split < 2; ++split) {
        const void *f = dispatch(wfmt, tfmt, kv_bf16, PtrOp{split != 0});
        if (cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, f, kDecodeBlock, smem) != cudaSuccess) return 0;
        lowest = std::min(lowest, per * sms);
    }
    return lowest;
}

}  // namespace qb
