// Persistent decode-step kernel for batch-1 greedy decoding on sm_100a.
//
// One cooperative launch evaluates one token through every layer and the LM
// head (src/kv_cache.rs:347-475 with attend_one :479-590) and leaves the
// greedy argmax (src/sampling.rs:65-70) in the control block.  The grid is
// one CTA per SM: 16 compute warps and one producer warp.  Compute phases
// are separated by a grid barrier whose wait is bounded by a timeout (the
// kernel then reports ERR_TIMEOUT, drains its own bulk copies and returns;
// it never spins forever):
//
//   per layer:  QKV      RMSNorm (each CTA, redundantly) -> rows of [Wq;Wk;Wv]
//                        + bias
//               ATTN     per (query head, o_proj row range): RoPE from the host
//                        cos/sin table, K/V write, softmax(q.K/sqrt d).V, then
//                        that head's o_proj partial for the row range
//               GATE/UP  residual + sum of head partials, RMSNorm, rows of
//                        gate and up, SiLU(gate)*up
//               DOWN     rows of down + residual
//   final:      LM HEAD  RMSNorm, rows of the (tied) table, logits, argmax;
//                        the last CTA reduces the per-CTA argmaxes.
//
// Weight streaming.  Weights never depend on activations, so the producer
// warp streams every row block the CTA will multiply -- all phases of the
// step, in order -- through a shared-memory ring of `nslot` slots with 1-D
// bulk copies (cp.async.bulk ... mbarrier::complete_tx), waiting only for
// the compute warps to free a slot ("empty" mbarrier).  It never waits for
// a grid barrier, so the next phases' weights are in shared memory before
// the activations they meet exist, and no weight occupies a register.  The
// producer also prefetches the rows a few phases ahead into L2.  The per-CTA
// row ranges come precomputed from the host: the critical path has no
// integer division and no long serial chain.
#include <math.h>

#include "common.cuh"
#include "decode.cuh"

namespace qb {

constexpr int NT = kDecodeThreads;  // compute threads
constexpr int NW = NT / 32;         // compute warps
constexpr int LOOKAHEAD = 3;        // L2 prefetch distance in phases

template <int WF> struct Fmt;
template <> struct Fmt<WF_F32> { static constexpr int EPC = 4; };
template <> struct Fmt<WF_BF16> { static constexpr int EPC = 8; };
template <> struct Fmt<WF_I8> { static constexpr int EPC = 16; };

__device__ __forceinline__ float ldcg(const float *p) { return __ldcg(p); }

// Barrier among the compute warps only (the producer warp never joins).
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(NT) : "memory"); }

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

// Block reductions over the compute warps: warp xor trees, then warp 0 runs
// one more tree over the warp partials -- a fixed order, broadcast to all.
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int off = 16; off; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int off = 16; off; off >>= 1) v = rust_max(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}
__device__ __forceinline__ float block_sum(float v, float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    if (lane == 0) red[warp] = v;
    csync();
    if (warp == 0) {
        v = warp_sum(lane < NW ? red[lane] : 0.0f);
        if (lane == 0) red[NW] = v;
    }
    csync();
    return red[NW];
}
__device__ __forceinline__ float block_max(float v, float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_max(v);
    if (lane == 0) red[warp] = v;
    csync();
    if (warp == 0) {
        v = warp_max(lane < NW ? red[lane] : -INFINITY);
        if (lane == 0) red[NW] = v;
    }
    csync();
    return red[NW];
}

// Scaled RMSNorm of `in` (shared, width w) into `out` (shared, zero-padded
// to `padded`), src/ops.rs:137-149.  The row scale is an exact maximum.
__device__ __forceinline__ void block_rmsnorm(const float *in, const float *gain, float *out, int w,
                                              int padded, float eps, float *red) {
    const float se = sqrtf(eps);
    float m = se;
#pragma unroll 1
    for (int i = threadIdx.x; i < w; i += NT) m = rust_max(m, fabsf(in[i]));
    m = block_max(m, red);
    float ss = 0.0f;
#pragma unroll 1
    for (int i = threadIdx.x; i < w; i += NT) {
        float v = in[i] / m;
        ss = ss + v * v;
    }
    ss = block_sum(ss, red);
    const float seps = se / m;
    const float den = sqrtf(ss / (float)w + seps * seps);
#pragma unroll 1
    for (int i = threadIdx.x; i < padded; i += NT) out[i] = i < w ? (in[i] / m) / den * gain[i] : 0.0f;
    csync();
}

__device__ __forceinline__ void flag_nonfinite(DecodeCtrl *ctrl, float v) {
    if (!isfinite(v)) atomicOr(&ctrl->error, ERR_NONFINITE);
}

// --------------------------------------------------------------- ring ----
//
// Chunk k of the CTA's stream lives in slot k % nslot during round
// u = k / nslot.  full[slot] completes phase u when the copy lands; the
// compute warps arrive on empty[slot] (phase u) once they have read it.

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

// Bounded wait for `parity` on `bar`; on timeout (or when the CTA is already
// aborting) records ERR_TIMEOUT, raises the abort flag and returns false.
__device__ __noinline__ bool mbar_wait_slow(const DecodeParams &p, uint64_t *bar, uint32_t parity,
                                            volatile int *s_abort) {
    const uint64_t t0 = globaltimer_ns();
    for (unsigned it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63u) == 0 && (*s_abort || globaltimer_ns() - t0 > p.timeout_ns)) {
            atomicOr(&p.ctrl->error, ERR_TIMEOUT);
            *s_abort = 1;
            return false;
        }
    }
}
__device__ __forceinline__ bool mbar_wait(const DecodeParams &p, uint64_t *bar, uint32_t parity,
                                          volatile int *s_abort) {
    return mbar_try_wait(bar, parity) || mbar_wait_slow(p, bar, parity, s_abort);
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

    // Streams rows [0, n) of a block (stride bytes each) in ring chunks.
    __device__ void block(const uint8_t *base, int n, const KindGeom &g) {
#pragma unroll 1
        for (int r = 0; r < n && alive; r += g.rpc) {
            if (round > 0 && !mbar_wait(p, rg.empty + slot, (uint32_t)((round - 1) & 1), s_abort)) {
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

    // Waits (bounded) for every copy this producer issued, before exiting
    // early.
    __device__ void drain() {
        const uint64_t t0 = globaltimer_ns();
        for (int s = 0; s < rg.nslot; ++s) {
            // Slot s was last filled in round (s < slot ? round : round - 1).
            const int u = s < slot ? round : round - 1;
            if (u < 0) continue;
            while (!mbar_try_wait(rg.full + s, (uint32_t)(u & 1)))
                if (globaltimer_ns() - t0 > p.timeout_ns) return;
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
                               int pos) {
    if (!p.prefetch || k > 4 * p.L) return;
    if (k == 4 * p.L) {
        prefetch_rows(p.head + (size_t)cg.lm_v0 * p.semb, (size_t)min(cg.lm_n, 64) * p.semb);
        return;
    }
    const DecodeLayer &Ly = lay[k >> 2];
    switch (k & 3) {
    case 0: prefetch_rows(Ly.wqkv + (size_t)cg.qkv_r0 * p.sh, (size_t)cg.qkv_n * p.sh); break;
    case 1: {
        const size_t esz = p.kv_bf16 ? 2 : 4;
        for (int a = 0; a < cg.natt; ++a) {
            prefetch_rows(Ly.wo + ((size_t)cg.att_hh[a] * p.h + cg.att_r0[a]) * p.shd, (size_t)cg.att_n[a] * p.shd);
            const int g = cg.att_hh[a] / p.group;
            prefetch_rows(Ly.kc + (size_t)g * p.cap * p.hd * esz, (size_t)pos * p.hd * esz);
            prefetch_rows(Ly.vc + (size_t)g * p.cap * p.hd * esz, (size_t)pos * p.hd * esz);
        }
        break;
    }
    case 2:
        prefetch_rows(Ly.wg + (size_t)cg.gu_f0 * p.sh, (size_t)cg.gu_n * p.sh);
        prefetch_rows(Ly.wu + (size_t)cg.gu_f0 * p.sh, (size_t)cg.gu_n * p.sh);
        break;
    default: prefetch_rows(Ly.wd + (size_t)cg.dn_r0 * p.sff, (size_t)cg.dn_n * p.sff); break;
    }
}

// The producer warp: the step's blocks in consumption order.
__device__ void produce(const DecodeParams &p, const DecodeLayer *lay, const CtaGeom &cg, float *sm, int pos,
                        volatile int *s_abort) {
    Producer pr(p, ring_of(p, sm), s_abort);
    const bool leader = (threadIdx.x & 31) == 0;
    for (int k = 0; k < LOOKAHEAD; ++k) prefetch_phase(p, lay, cg, k, pos);
#pragma unroll 1
    for (int l = 0; l < p.L && pr.alive; ++l) {
        const DecodeLayer &Ly = lay[l];
        const int ph = 4 * l;
        prefetch_phase(p, lay, cg, ph + LOOKAHEAD, pos);
        if (leader) pr.block(Ly.wqkv + (size_t)cg.qkv_r0 * p.sh, cg.qkv_n, p.kind[K_QKV]);
        prefetch_phase(p, lay, cg, ph + 1 + LOOKAHEAD, pos);
        if (leader)
            for (int a = 0; a < cg.natt; ++a)
                pr.block(Ly.wo + ((size_t)cg.att_hh[a] * p.h + cg.att_r0[a]) * p.shd, cg.att_n[a], p.kind[K_O]);
        prefetch_phase(p, lay, cg, ph + 2 + LOOKAHEAD, pos);
        if (leader) {
            pr.block(Ly.wg + (size_t)cg.gu_f0 * p.sh, cg.gu_n, p.kind[K_GU]);
            pr.block(Ly.wu + (size_t)cg.gu_f0 * p.sh, cg.gu_n, p.kind[K_GU]);
        }
        prefetch_phase(p, lay, cg, ph + 3 + LOOKAHEAD, pos);
        if (leader) pr.block(Ly.wd + (size_t)cg.dn_r0 * p.sff, cg.dn_n, p.kind[K_DN]);
        pr.alive = __shfl_sync(0xffffffffu, (int)pr.alive, 0) != 0;
    }
    if (leader && pr.alive) pr.block(p.head + (size_t)cg.lm_v0 * p.semb, cg.lm_n, p.kind[K_LM]);
    if (leader && !pr.alive) pr.drain();
}

// ------------------------------------------------------------ gemv ----
//
// y_r = dot(W_r, x) for the n rows of one block, weights from the ring.
// When C <= NT thread t owns chunk column c = t % C (its activations stay in
// registers) and walks rows rs, rs + RS, ... of each chunk; otherwise threads
// stride the columns of each row.  Partials meet in shared memory and are
// reduced per row in a fixed order into rowout[r].

template <int WF>
__device__ __noinline__ bool ring_gemv(const DecodeParams &p, const Ring &rg, Cursor &cur, const KindGeom &g, int n,
                          const float *xs, float *part, volatile int *s_abort, float *rowout) {
    constexpr int EPC = Fmt<WF>::EPC;
    if (n <= 0) return true;
    const int t = threadIdx.x, lane = t & 31;
    const bool cols = g.RS > 0;
    const int pcols = cols ? g.C : NT;
    const int rs = cols ? (int)__umulhi((unsigned)t, g.magic) : 0;
    const int c = cols ? t - rs * g.C : t;
    const bool active = !cols || rs < g.RS;
    float xr[EPC];
    if (cols) {
#pragma unroll
        for (int k = 0; k < EPC; ++k) xr[k] = active ? xs[c * EPC + k] : 0.0f;
    }
    const int grows = g.rpc * g.group;  // rows per reduction group
#pragma unroll 1
    for (int r0 = 0; r0 < n; r0 += grows) {
        const int rows_g = min(grows, n - r0);
        const Cursor c0 = cur;
#pragma unroll 1
        for (int j = 0; j * g.rpc < rows_g; ++j) {
            if (!mbar_wait(p, rg.full + cur.slot, (uint32_t)(cur.round & 1), s_abort)) break;
            const uint8_t *slot = rg.slots + (size_t)cur.slot * rg.slot_bytes;
            const int nr = min(g.rpc, rows_g - j * g.rpc);
            const int pr0 = j * g.rpc;
            if (cols) {
                if (active)
#pragma unroll 1
                    for (int r = rs; r < nr; r += g.RS) {
                        const uint4 w = *(const uint4 *)(slot + (size_t)r * g.stride + (size_t)c * 16);
                        part[(pr0 + r) * g.C + c] = chunk_dot<WF>(w, xr);
                    }
            } else {
#pragma unroll 1
                for (int r = 0; r < nr; ++r) {
                    float acc = 0.0f;
#pragma unroll 1
                    for (int cc = t; cc < g.C; cc += NT) {
                        const uint4 w = *(const uint4 *)(slot + (size_t)r * g.stride + (size_t)cc * 16);
                        acc += chunk_dot<WF>(w, xs + cc * EPC);
                    }
                    part[(pr0 + r) * NT + t] = acc;
                }
            }
            cur.advance(rg.nslot);
        }
        csync();
        if (*s_abort) return false;
        // Every compute thread has read the group's slots: hand them back.
        if (t == 0) {
            fence_proxy_async_smem();
            Cursor e = c0;
            for (int j = 0; j * g.rpc < rows_g; ++j) {
                mbar_arrive(rg.empty + e.slot);
                e.advance(rg.nslot);
            }
        }
#pragma unroll 1
        for (int r = t >> 5; r < rows_g; r += NW) {
            float s = 0.0f;
#pragma unroll 1
            for (int cc = lane; cc < pcols; cc += 32) s += part[r * pcols + cc];
            s = warp_sum(s);
            if (lane == 0) rowout[r0 + r] = s;
        }
        csync();
    }
    return true;
}

// ------------------------------------------------------------ barrier ----

// Grid barrier in two halves (compute warps only).  barrier_arrive makes
// the CTA's writes visible (csync, then thread 0's release reduction);
// independent work can run before barrier_wait, which polls with relaxed
// loads (bounded by the timeout) and ends with an acquire fence and csync.
// barrier_wait returns false (after recording ERR_TIMEOUT and raising the
// abort flag) when the arrivals do not complete in time or another CTA has
// timed out.
__device__ __forceinline__ void barrier_arrive(const DecodeParams &p, unsigned target) {
    csync();
    if (threadIdx.x == 0) {
        if (p.trace) {
            const int G = gridDim.x, idx = (int)(target / (unsigned)G) - 1;
            p.trace[(size_t)idx * G + blockIdx.x] = globaltimer_ns();
        }
        red_release_add_u32(&p.ctrl->bar, 1u);
    }
}

__device__ __noinline__ bool barrier_wait(const DecodeParams &p, unsigned target, volatile int *s_abort) {
    DecodeCtrl *ctrl = p.ctrl;
    if (threadIdx.x == 0) {
        volatile unsigned *bar = &ctrl->bar;
        if (*bar < target) {
            const uint64_t t0 = globaltimer_ns();
            unsigned spins = 0;
            while (*bar < target) {
                if ((++spins & 63u) == 0) {
                    if ((*(volatile unsigned *)&ctrl->error & ERR_TIMEOUT) || globaltimer_ns() - t0 > p.timeout_ns) {
                        atomicOr(&ctrl->error, ERR_TIMEOUT);
                        *s_abort = 1;
                        break;
                    }
                }
            }
        }
        asm volatile("fence.acq_rel.gpu;" ::: "memory");
        if (p.trace && blockIdx.x == 0) {
            const int G = gridDim.x, idx = (int)(target / (unsigned)G) - 1;
            p.trace[(size_t)4 * p.L * G + idx] = globaltimer_ns();
        }
    }
    csync();
    return *s_abort == 0;
}

// --------------------------------------------------------- elementwise ----

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
// residual added (src/kv_cache.rs:405-406).
__device__ __forceinline__ float after_attention(const DecodeParams &p, int l, int token, int i) {
    // Eight heads' loads are in flight at a time; the sum runs in head order.
    const float *base = p.part + i;
    const size_t stride = (size_t)p.h;
    float o = 0.0f;
#pragma unroll 1
    for (int h0 = 0; h0 < p.qh; h0 += 8) {
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = h0 + k < p.qh ? ldcg(base + (size_t)(h0 + k) * stride) : 0.0f;
#pragma unroll
        for (int k = 0; k < 8; ++k)
            if (h0 + k < p.qh) o = (h0 + k == 0) ? v[k] : o + v[k];
    }
    return resid_in(p, l, token, i) + o;
}

__device__ __forceinline__ float silu1(float v) {
    if (v >= 0.0f) return v / (1.0f + expf(-v));
    const float e = expf(v);
    return v * e / (1.0f + e);
}

template <int KVBF16>
__device__ __forceinline__ float kv_load(const uint8_t *base, size_t idx) {
    if (KVBF16) return bf16_to_f32(__ldcg((const unsigned short *)base + idx));
    return __ldcg((const float *)base + idx);
}

// Attention for query head hh at position pos (src/kv_cache.rs:550-576),
// leaving the context vector in shared memory (ctx, zero-padded).  The
// first CTA of a KV group writes the new K (rotated) and V at `pos`.
template <int WF, int KVBF16>
__device__ __noinline__ void attention_context(const DecodeParams &p, const DecodeLayer &Ly, int hh, bool writer, int pos,
                                  float *sm) {
    const int hd = p.hd, half = hd / 2, g = hh / p.group;
    const size_t kvw = (size_t)p.kvh * hd;
    float *qs = sm + p.sm_q, *ks = qs + hd, *vs = ks + hd, *ctx = vs + hd;
    float *sc = sm + p.sm_sc, *red = sm + p.sm_red, *part = sm + p.sm_part;
    const float2 *rp = p.rope + (size_t)pos * half;
#pragma unroll 1
    for (int j = threadIdx.x; j < half; j += NT) {
        const float2 cs = rp[j];
        const float a = ldcg(p.qkv + (size_t)hh * hd + j), b = ldcg(p.qkv + (size_t)hh * hd + j + half);
        qs[j] = a * cs.x - b * cs.y;
        qs[j + half] = b * cs.x + a * cs.y;
        const float ka = ldcg(p.qkv + p.h + (size_t)g * hd + j), kb = ldcg(p.qkv + p.h + (size_t)g * hd + j + half);
        float k0 = ka * cs.x - kb * cs.y, k1 = kb * cs.x + ka * cs.y;
        if (KVBF16) { k0 = round_bf16(k0); k1 = round_bf16(k1); }
        ks[j] = k0;
        ks[j + half] = k1;
    }
#pragma unroll 1
    for (int i = threadIdx.x; i < hd; i += NT) {
        const float v = ldcg(p.qkv + p.h + kvw + (size_t)g * hd + i);
        vs[i] = KVBF16 ? round_bf16(v) : v;
    }
    const int ctx_pad = p.chd * Fmt<WF>::EPC;
#pragma unroll 1
    for (int i = hd + threadIdx.x; i < ctx_pad; i += NT) ctx[i] = 0.0f;
    csync();
    if (threadIdx.x < hd && (!isfinite(qs[threadIdx.x]) || !isfinite(ks[threadIdx.x])))
        atomicOr(&p.ctrl->error, ERR_NONFINITE);
    const size_t esz = KVBF16 ? 2 : 4;
    const uint8_t *K = Ly.kc + (size_t)g * p.cap * hd * esz;
    const uint8_t *Vc = Ly.vc + (size_t)g * p.cap * hd * esz;
    if (writer) {
#pragma unroll 1
        for (int i = threadIdx.x; i < hd; i += NT) {
            const size_t idx = (size_t)g * p.cap * hd + (size_t)pos * hd + i;
            if (KVBF16) {
                ((uint16_t *)Ly.kc)[idx] = f32_to_bf16_rne(ks[i]);
                ((uint16_t *)Ly.vc)[idx] = f32_to_bf16_rne(vs[i]);
            } else {
                ((float *)Ly.kc)[idx] = ks[i];
                ((float *)Ly.vc)[idx] = vs[i];
            }
        }
    }
    // scores: q.k / sqrt(d), one position per thread, increasing i.
    const int row_bytes = hd * (int)esz;
    const bool vec = (row_bytes & 15) == 0;
    constexpr int KEPC = KVBF16 ? 8 : 4;  // cache elements per 16-byte chunk
#pragma unroll 1
    for (int q = threadIdx.x; q <= pos; q += NT) {
        float s = 0.0f;
        if (q == pos) {
#pragma unroll 1
            for (int i = 0; i < hd; ++i) s = s + qs[i] * ks[i];
        } else if (vec) {
            const uint8_t *row = K + (size_t)q * row_bytes;
            const int nc = row_bytes >> 4;
#pragma unroll 1
            for (int c0 = 0; c0 < nc; c0 += 8) {
                uint4 kc[8];
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    if (c0 + c < nc) kc[c] = __ldcg((const uint4 *)(row + (size_t)(c0 + c) * 16));
#pragma unroll
                for (int c = 0; c < 8; ++c) {
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
            }
        } else {
#pragma unroll 1
            for (int i = 0; i < hd; ++i) s = s + qs[i] * kv_load<KVBF16>(K, (size_t)q * hd + i);
        }
        sc[q] = s / p.sqrt_hd;
    }
    csync();
    float m = -INFINITY;
#pragma unroll 1
    for (int q = threadIdx.x; q <= pos; q += NT) m = rust_max(m, sc[q]);
    m = block_max(m, red);
    float se = 0.0f;
#pragma unroll 1
    for (int q = threadIdx.x; q <= pos; q += NT) {
        const float e = expf(sc[q] - m);
        sc[q] = e;
        se += e;
    }
    se = block_sum(se, red);
#pragma unroll 1
    for (int q = threadIdx.x; q <= pos; q += NT) sc[q] = sc[q] / se;
    csync();
    // context: position groups pg sum positions pg, pg+PG, ... in order;
    // the groups then meet in group order.
    int PG;
    if (vec) {
        const int nc = row_bytes >> 4;
        PG = NT / nc;
        const int c = threadIdx.x % nc, pg = threadIdx.x / nc;
        if (pg < PG) {
            float acc[KEPC];
#pragma unroll
            for (int e = 0; e < KEPC; ++e) acc[e] = 0.0f;
#pragma unroll 1
            for (int q0 = pg; q0 <= pos; q0 += 4 * PG) {
                uint4 vc[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int q = q0 + u * PG;
                    if (q < pos) vc[u] = __ldcg((const uint4 *)(Vc + (size_t)q * row_bytes + (size_t)c * 16));
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int q = q0 + u * PG;
                    if (q <= pos) {
                        const float pr = sc[q];
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
#pragma unroll
            for (int e = 0; e < KEPC; ++e) part[pg * hd + c * KEPC + e] = acc[e];
        }
    } else {
        PG = NT / hd > 0 ? NT / hd : 1;
        const int i = threadIdx.x % hd, pg = threadIdx.x / hd;
        float acc = 0.0f;
        if (pg < PG && threadIdx.x < PG * hd) {
#pragma unroll 1
            for (int q = pg; q <= pos; q += PG) {
                const float v = q == pos ? vs[i] : kv_load<KVBF16>(Vc, (size_t)q * hd + i);
                acc = acc + sc[q] * v;
            }
            part[pg * hd + i] = acc;
        }
    }
    csync();
#pragma unroll 1
    for (int i = threadIdx.x; i < hd; i += NT) {
        float s = part[i];
#pragma unroll 1
        for (int k = 1; k < PG; ++k) s += part[k * hd + i];
        ctx[i] = s;
        flag_nonfinite(p.ctrl, s);
    }
    csync();
}

// ------------------------------------------------------------ phases ----
//
// Each phase has a `prep` that stages its small vectors -- `gain` (norm
// gains) and `rv` (row scales rv[0..R), biases or second scales rv[R..2R))
// -- into shared memory before the grid barrier that precedes it, and a
// `run` after the barrier.  The weights arrive through the ring.

// Stages n floats of global memory into shared memory.
__device__ __forceinline__ void stage(float *dst, const float *src, int n) {
#pragma unroll 1
    for (int i = threadIdx.x; i < n; i += NT) dst[i] = src[i];
}

template <int WF>
__device__ __forceinline__ void prep_qkv(const DecodeParams &p, const DecodeLayer &Ly, const CtaGeom &cg,
                                         float *sm) {
    float *gain = sm + p.sm_gain, *rv = sm + p.sm_rv;
    stage(gain, Ly.attn_norm, p.h);
    if (WF == WF_I8) stage(rv, Ly.sqkv + cg.qkv_r0, cg.qkv_n);
    stage(rv + cg.qkv_n, Ly.bqkv + cg.qkv_r0, cg.qkv_n);
}

template <int WF>
__device__ __forceinline__ bool run_qkv(const DecodeParams &p, const CtaGeom &cg, int l, int token, float *sm,
                                        const Ring &rg, Cursor &cur, volatile int *s_abort) {
    constexpr int EPC = Fmt<WF>::EPC;
    float *xs = sm + p.sm_xs, *part = sm + p.sm_part, *h2 = sm + p.sm_h2, *red = sm + p.sm_red;
    const float *gain = sm + p.sm_gain, *rv = sm + p.sm_rv;
#pragma unroll 1
    for (int i = threadIdx.x; i < p.h; i += NT) h2[i] = resid_in(p, l, token, i);
    csync();
    block_rmsnorm(h2, gain, xs, p.h, p.ch * EPC, p.eps, red);
    float *rows = sm + p.sm_gu;
    if (!ring_gemv<WF>(p, rg, cur, p.kind[K_QKV], cg.qkv_n, xs, part, s_abort, rows)) return false;
    const int R = cg.qkv_n;
    float *out = p.qkv + cg.qkv_r0;
#pragma unroll 1
    for (int r = threadIdx.x; r < R; r += NT) {
        float v = rows[r];
        if (WF == WF_I8) v = v * rv[r];
        v = v + rv[R + r];
        out[r] = v;
        flag_nonfinite(p.ctrl, v);
    }
    return true;
}

template <int WF>
__device__ __forceinline__ void prep_attention(const DecodeParams &p, const DecodeLayer &Ly, const CtaGeom &cg,
                                               float *sm) {
    if (WF == WF_I8 && cg.natt > 0) stage(sm + p.sm_rv, Ly.so + cg.att_r0[0], cg.att_n[0]);
}

template <int WF, int KVBF16>
__device__ __forceinline__ bool run_attention(const DecodeParams &p, const DecodeLayer &Ly, const CtaGeom &cg,
                                              int pos, float *sm, const Ring &rg, Cursor &cur,
                                              volatile int *s_abort) {
    float *part = sm + p.sm_part, *ctx = sm + p.sm_q + 3 * p.hd;
    const float *rv = sm + p.sm_rv;
#pragma unroll 1
    for (int a = 0; a < cg.natt; ++a) {
        const int hh = cg.att_hh[a], r0 = cg.att_r0[a], n = cg.att_n[a];
        attention_context<WF, KVBF16>(p, Ly, hh, r0 == 0 && hh % p.group == 0, pos, sm);
        float *rows = sm + p.sm_gu;
        if (!ring_gemv<WF>(p, rg, cur, p.kind[K_O], n, ctx, part, s_abort, rows)) return false;
        float *outp = p.part + (size_t)hh * p.h + r0;
#pragma unroll 1
        for (int r = threadIdx.x; r < n; r += NT) {
            float v = rows[r];
            if (WF == WF_I8) v = v * (a == 0 ? rv[r] : Ly.so[r0 + r]);
            outp[r] = v;
            flag_nonfinite(p.ctrl, v);
        }
        csync();
    }
    return true;
}

template <int WF>
__device__ __forceinline__ void prep_gate_up(const DecodeParams &p, const DecodeLayer &Ly, const CtaGeom &cg,
                                             float *sm) {
    float *gain = sm + p.sm_gain, *rv = sm + p.sm_rv;
    stage(gain, Ly.ffn_norm, p.h);
    if (WF == WF_I8) {
        stage(rv, Ly.sg + cg.gu_f0, cg.gu_n);
        stage(rv + cg.gu_n, Ly.su + cg.gu_f0, cg.gu_n);
    }
}

template <int WF>
__device__ __forceinline__ bool run_gate_up(const DecodeParams &p, const CtaGeom &cg, int l, int token, float *sm,
                                            const Ring &rg, Cursor &cur, volatile int *s_abort) {
    constexpr int EPC = Fmt<WF>::EPC;
    float *xs = sm + p.sm_xs, *part = sm + p.sm_part, *h2 = sm + p.sm_h2, *red = sm + p.sm_red;
    float *gu = sm + p.sm_gu;
    const float *gain = sm + p.sm_gain, *rv = sm + p.sm_rv;
#pragma unroll 1
    for (int i = threadIdx.x; i < p.h; i += NT) {
        const float v = after_attention(p, l, token, i);
        h2[i] = v;
        if (blockIdx.x == 0) flag_nonfinite(p.ctrl, v);
    }
    csync();
    block_rmsnorm(h2, gain, xs, p.h, p.ch * EPC, p.eps, red);
    const int R = cg.gu_n;
    if (!ring_gemv<WF>(p, rg, cur, p.kind[K_GU], R, xs, part, s_abort, gu)) return false;
    if (!ring_gemv<WF>(p, rg, cur, p.kind[K_GU], R, xs, part, s_abort, gu + R)) return false;
#pragma unroll 1
    for (int r = threadIdx.x; r < R; r += NT) {
        float gv = gu[r], uv = gu[R + r];
        if (WF == WF_I8) {
            gv = gv * rv[r];
            uv = uv * rv[R + r];
        }
        const float a = silu1(gv) * uv;
        p.act[cg.gu_f0 + r] = a;
        flag_nonfinite(p.ctrl, gv);
        flag_nonfinite(p.ctrl, a);
    }
    csync();  // rv is restaged by the next prep
    return true;
}

template <int WF>
__device__ __forceinline__ void prep_down(const DecodeParams &p, const DecodeLayer &Ly, const CtaGeom &cg,
                                          float *sm) {
    if (WF == WF_I8) stage(sm + p.sm_rv, Ly.sd + cg.dn_r0, cg.dn_n);
}

template <int WF>
__device__ __forceinline__ bool run_down(const DecodeParams &p, const CtaGeom &cg, float *sm, const Ring &rg,
                                         Cursor &cur, volatile int *s_abort) {
    constexpr int EPC = Fmt<WF>::EPC;
    float *xs = sm + p.sm_xs, *part = sm + p.sm_part;
#pragma unroll 1
    for (int i = threadIdx.x; i < p.cff * EPC; i += NT) xs[i] = i < p.ff ? ldcg(p.act + i) : 0.0f;
    csync();
    float *rows = sm + p.sm_gu;
    if (!ring_gemv<WF>(p, rg, cur, p.kind[K_DN], cg.dn_n, xs, part, s_abort, rows)) return false;
    // h' of this layer is still in shared memory from the gate/up phase of
    // this same CTA (src/kv_cache.rs:437-443: x_next = h' + down(a)).
    const float *h2 = sm + p.sm_h2 + cg.dn_r0, *rv = sm + p.sm_rv;
    float *hidden = p.hidden + cg.dn_r0;
#pragma unroll 1
    for (int r = threadIdx.x; r < cg.dn_n; r += NT) {
        float v = rows[r];
        if (WF == WF_I8) v = v * rv[r];
        const float o = h2[r] + v;
        hidden[r] = o;
        flag_nonfinite(p.ctrl, o);
    }
    return true;
}

// Final RMSNorm, this CTA's rows of the (tied) table, logits and the CTA's
// argmax (lowest id on ties); the last CTA to finish reduces the grid.  The
// logits of all the CTA's rows land in `rowv`; warp 0 scans them in row
// order, so ties keep the lowest id.
template <int TF>
__device__ __forceinline__ bool run_lm_head(const DecodeParams &p, const CtaGeom &cg, int pos, float *sm,
                                            const Ring &rg, Cursor &cur, volatile int *s_abort) {
    constexpr int TEPC = Fmt<TF>::EPC;
    const int G = gridDim.x, b = blockIdx.x;
    float *xs = sm + p.sm_xs, *part = sm + p.sm_part, *h2 = sm + p.sm_h2, *red = sm + p.sm_red;
    const float *gain = sm + p.sm_gain;
    float *rowv = sm + p.sm_sc;
    DecodeCtrl *ctrl = p.ctrl;
#pragma unroll 1
    for (int i = threadIdx.x; i < p.h; i += NT) h2[i] = ldcg(p.hidden + i);
    csync();
    block_rmsnorm(h2, gain, xs, p.h, p.cemb * TEPC, p.eps, red);
    if (!ring_gemv<TF>(p, rg, cur, p.kind[K_LM], cg.lm_n, xs, part, s_abort, rowv)) return false;
    // ring_gemv ends with a barrier, so every row's logit is in rowv.
    if (ctrl->write_logits) {
        float *lg = p.logits + cg.lm_v0;
#pragma unroll 1
        for (int r = threadIdx.x; r < cg.lm_n; r += NT) lg[r] = rowv[r];
    }
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        float bv = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll 1
        for (int r = lane; r < cg.lm_n; r += 32) {
            const float v = rowv[r];
            if (!isfinite(v)) atomicOr(&ctrl->error, ERR_NONFINITE);
            if (v > bv) { bv = v; bi = r; }
        }
#pragma unroll
        for (int off = 16; off; off >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) {
            p.amax_v[b] = bv;
            p.amax_i[b] = bi == 0x7fffffff ? bi : cg.lm_v0 + bi;
            __threadfence();
            const unsigned tk = atomicAdd(&ctrl->ticket, 1u);
            if (tk == (unsigned)G - 1) {
                __threadfence();
                float gv = __ldcg(p.amax_v);
                int gi = __ldcg(p.amax_i);
#pragma unroll 1
                for (int k = 1; k < G; ++k) {
                    const float v = __ldcg(p.amax_v + k);
                    const int i = __ldcg(p.amax_i + k);
                    if (v > gv || (v == gv && i < gi)) { gv = v; gi = i; }
                }
                if (gi < 0 || gi >= p.V) gi = 0;
                ctrl->next_token = gi;
                if (p.emitted) p.emitted[pos] = gi;
                ctrl->token = gi;
                ctrl->pos = pos + 1;
                ctrl->bar = 0;
                ctrl->ticket = 0;
                if (p.trace) p.trace[(size_t)4 * p.L * G + 4 * p.L + 1] = globaltimer_ns();
                __threadfence();
            }
        }
    }
    return true;
}

// ------------------------------------------------------------ kernel ----

template <int WF, int TF, int KVBF16>
__global__ void __launch_bounds__(kDecodeBlock, 1) decode_kernel(const __grid_constant__ DecodeParams p) {
    extern __shared__ __align__(128) float sm[];
    __shared__ int s_abort_storage;
    volatile int *s_abort = &s_abort_storage;
    const int G = gridDim.x, b = blockIdx.x;
    DecodeCtrl *ctrl = p.ctrl;
    const int token = *(volatile int *)&ctrl->token;
    const int pos = *(volatile int *)&ctrl->pos;
    const int NB = 4 * p.L;
    const CtaGeom &cg = p.geom[b];
    if (p.trace && b == 0 && threadIdx.x == 0) p.trace[(size_t)NB * G + NB] = globaltimer_ns();
    // The layer table lives in shared memory for the whole step.
    DecodeLayer *lay = (DecodeLayer *)(sm + p.sm_lay);
    {
        const uint32_t *src = (const uint32_t *)p.layers;
        uint32_t *dst = (uint32_t *)lay;
        const int words = p.L * (int)(sizeof(DecodeLayer) / 4);
#pragma unroll 1
        for (int i = threadIdx.x; i < words; i += kDecodeBlock) dst[i] = src[i];
    }
    const Ring rg = ring_of(p, sm);
    if (threadIdx.x == 0) {
        for (int i = 0; i < p.nslot; ++i) {
            mbar_init(rg.full + i, 1);
            mbar_init(rg.empty + i, 1);
        }
        fence_mbar_init();
        *s_abort = 0;
    }
    __syncthreads();  // the only all-thread barrier: roles split here

    if (threadIdx.x >= NT) {  // producer warp
        produce(p, lay, cg, sm, pos, s_abort);
        return;
    }

    Cursor cur{0, 0};
    prep_qkv<WF>(p, lay[0], cg, sm);
    csync();
    unsigned target = 0;
    bool ok = true;
    // Each phase: run, arrive at the grid barrier, stage the next phase's
    // vectors while the other CTAs arrive, then wait.
#pragma unroll 1
    for (int l = 0; l < p.L && ok; ++l) {
        const DecodeLayer &Ly = lay[l];
        if (!(ok = run_qkv<WF>(p, cg, l, token, sm, rg, cur, s_abort))) break;
        barrier_arrive(p, target += G);
        prep_attention<WF>(p, Ly, cg, sm);
        if (!(ok = barrier_wait(p, target, s_abort))) break;

        if (!(ok = run_attention<WF, KVBF16>(p, Ly, cg, pos, sm, rg, cur, s_abort))) break;
        barrier_arrive(p, target += G);
        prep_gate_up<WF>(p, Ly, cg, sm);
        if (!(ok = barrier_wait(p, target, s_abort))) break;

        if (!(ok = run_gate_up<WF>(p, cg, l, token, sm, rg, cur, s_abort))) break;
        barrier_arrive(p, target += G);
        prep_down<WF>(p, Ly, cg, sm);
        if (!(ok = barrier_wait(p, target, s_abort))) break;

        if (!(ok = run_down<WF>(p, cg, sm, rg, cur, s_abort))) break;
        barrier_arrive(p, target += G);
        if (l + 1 < p.L) prep_qkv<WF>(p, lay[l + 1], cg, sm);
        else stage(sm + p.sm_gain, p.final_norm, p.h);
        if (!(ok = barrier_wait(p, target, s_abort))) break;
    }
    if (ok) ok = run_lm_head<TF>(p, cg, pos, sm, rg, cur, s_abort);
    if (!ok && threadIdx.x == 0) *s_abort = 1;  // releases a producer waiting for a slot
}

size_t decode_smem_bytes(const DecodeParams &p) { return (size_t)p.sm_total * sizeof(float); }

template <int WF, int TF, int KV>
static cudaError_t launch_t(const DecodeParams &p, int grid, cudaStream_t stream) {
    auto kern = decode_kernel<WF, TF, KV>;
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
static const void *kernel_ptr() {
    return (const void *)decode_kernel<WF, TF, KV>;
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
    template <int W, int T, int K> cudaError_t operator()() const { return launch_t<W, T, K>(p, grid, stream); }
};
struct PtrOp {
    template <int W, int T, int K> const void *operator()() const { return kernel_ptr<W, T, K>(); }
};

cudaError_t decode_launch(const DecodeParams &p, int grid, cudaStream_t stream) {
    return dispatch(p.wfmt, p.tfmt, p.kv_bf16, LaunchOp{p, grid, stream});
}

// Largest number of co-resident CTAs of the decode kernel on this device.
int decode_max_ctas(int wfmt, int tfmt, int kv_bf16, size_t smem) {
    int dev = 0, sms = 0, per = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const void *f = dispatch(wfmt, tfmt, kv_bf16, PtrOp{});
    if (cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, f, kDecodeBlock, smem) != cudaSuccess) return 0;
    return per * sms;
}

}  // namespace qb
