// Device layout and parameters of the persistent decode-step kernel.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

namespace qb {

// Word of an exchange slot that has not received its value (a NaN that no
// producer stores: a computed value with this bit pattern is stored as
// 0x7fffffff and reported as non-finite).
constexpr uint32_t kNotReady = 0xffffffffu;

// Storage of the seven per-layer linears (DecodeParams::wfmt).
enum { WF_F32 = 0, WF_BF16 = 1, WF_I8 = 2 };

// Error bits reported by the kernel in DecodeCtrl::error.
enum { ERR_NONFINITE = 1u, ERR_TIMEOUT = 2u };

// Positions per KV-cache page.  A layer's cache is a pool of pages, each
// [kv_heads][kPageTokens][head_dim] (K and V in separate pools); a page
// table maps a sequence's page j (positions 16 j .. 16 j + 15) to a page of
// the pool.
constexpr int kPageTokens = 16;

// One layer's device tensors.  Every weight matrix is row-major with a row
// stride padded to a multiple of 16 bytes (zero padding).  INT8 rows are
// stored biased (u = q + 128) with one FP32 scale per output row.
struct DecodeLayer {
    const uint8_t *wqkv;  // [h + 2 kv, stride_h]: q rows, then k rows, then v rows
    const float *sqkv;    // row scales (INT8) or null
    const float *bqkv;    // [h + 2 kv] biases (zeros when the model has none)
    const uint8_t *wo;    // head-blocked o_proj: [qh][h rows][stride_hd]
    const float *so;      // [h] row scales (INT8) or null
    const uint8_t *wgu;   // [2 ff, stride_h]: row 2f = gate row f, row 2f + 1 = up row f
    const float *sgu;     // [2 ff] row scales in the same order (INT8) or null
    const uint8_t *wd;    // [h, stride_ff]
    const float *sd;
    const float *attn_norm;  // [h]
    const float *ffn_norm;   // [h]
    uint8_t *kc;          // K page pool: [pages][kv_heads][16][head_dim] rotated keys (FP32 or BF16)
    uint8_t *vc;          // V page pool, same layout
};

// Device-resident control block shared by the host and every step.
struct DecodeCtrl {
    int token;         // in: token evaluated by the next step
    int pos;           // in: its absolute position (== processed)
    int write_logits;  // in: nonzero = store the full logits row
    int pad0;
    int next_token;    // out: greedy argmax of this step
    unsigned error;    // out: ERR_* bits, sticky until the host clears them
    unsigned epoch;    // steps completed; its parity selects the exchange buffers
    unsigned ticket;   // end-of-step ticket (reset by the last CTA)
};

// The weight kinds a CTA streams, and their host-computed geometry.  A
// "unit" is the U consecutive rows one team of G = 2^lgG threads multiplies
// together (U = 2 pairs each gate row with its up row).
enum { K_QKV = 0, K_O = 1, K_GU = 2, K_DN = 3, K_LM = 4, NKIND = 5 };
struct KindGeom {
    int stride;  // bytes per padded row
    int C;       // 16-byte chunks per row
    int rpc;     // rows per ring slot (a multiple of U)
    int lgG;     // log2 of the threads per unit (2..7; above 5 a unit spans warps)
    int U;       // rows per unit
    int wave;    // ring slots waited for and released together (<= nslot / 2 or the block)
    unsigned rpc_magic;  // ceil(2^32 / rpc) when rpc > 1: r / rpc == umulhi(r, rpc_magic) for r < 2^16
};

// The rows each CTA owns in every phase (host-computed, no division on the
// device).  Attention items are (query head, o_proj row range) pairs.
constexpr int kMaxAttItems = 4;
// At most this many CTAs per query head (and position splits of a head).
constexpr int kMaxSplits = 8;
struct CtaGeom {
    int qkv_r0, qkv_n;  // rows of [Wq;Wk;Wv]
    int gu_f0, gu_n;    // rows of gate and of up
    int dn_r0, dn_n;    // rows of down (== hidden elements written)
    int lm_v0, lm_n;    // rows of the LM-head table
    int natt;
    int att_hh[kMaxAttItems], att_r0[kMaxAttItems], att_n[kMaxAttItems];
    int att_sp[kMaxAttItems];  // index of the item among its head's att_splits items
};

struct DecodeParams {
    int V, L, h, qh, kvh, hd, ff, cap, group;
    int wfmt, tfmt, kv_bf16;
    float eps, sqrt_hd;
    int ch, chd, cff, cemb;   // 16-byte chunks per row for K = h, hd, ff and the table
    size_t sh, shd, sff, semb;  // row strides in bytes
    const int *ptab;          // page table of the session: [ceil(cap / 16)] pool pages
    int rqkv;                 // h + 2 * kv_heads * head_dim
    KindGeom kind[NKIND];
    const CtaGeom *geom;      // [grid]
    const uint8_t *emb;       // [V, semb] embedding table (FP32 or BF16)
    const uint8_t *head;      // LM head table (== emb when tied)
    const float *final_norm;
    const DecodeLayer *layers;  // device array [L]
    const float2 *rope;       // [cap][hd/2] (cos, sin)
    // Exchange vectors between the CTAs: [2 parities][L][xl] floats; per
    // layer the QKV outputs at x_qkv ([rqkv]), the per-head o_proj partial
    // sums at x_part ([qh][h]), the SwiGLU activations at x_act ([ff]) and
    // the layer's output at x_hid ([h]), each 16-byte aligned.  A step uses
    // the parity of ctrl->epoch: every slot of it starts as kNotReady and
    // receives exactly one value, while the step resets the other parity to
    // kNotReady for the next step.  Consumers poll their inputs until no
    // word is kNotReady (no grid barrier).
    float *xch;
    int xl, x_qkv, x_part, x_act, x_hid;
    float *logits;            // [V]
    float *amax_v;            // [grid] per-CTA argmax value
    int *amax_i;              // [grid] per-CTA argmax index
    int *emitted;             // [cap] greedy id emitted after each position (nullable)
    DecodeCtrl *ctrl;
    // Optional phase trace (globaltimer ns): [4L phases][grid] times at which
    // each CTA finished the phase, then [4L phases][grid] times at which each
    // CTA held the outputs of the phase it consumes next (0: the CTA had no
    // work in that phase), then the kernel start (CTA 0) and the end of the
    // final reduction.  Null = off.
    unsigned long long *trace;
    unsigned long long timeout_ns;
    int prefetch;             // L2 prefetch of upcoming weights by the producer warp
    unsigned long long pf_cap;  // bytes of one block a CTA prefetches (the grid's share of L2 per phase)
    // Fault-path test hook: nonzero = CTA 0 does not publish its layer-0 QKV
    // outputs, so the polls that read them run out (ERR_TIMEOUT).  0 in
    // every normal step.
    int withhold;
    // Long-context attention: with att_splits > 1 and at least att_split_min
    // cached positions, the att_splits CTAs of a query head each take one
    // position range, exchange (max, sum, context) partials through apart
    // [qh][att_splits][hd + 2] and meet at a per-head barrier (hbar[qh],
    // arrivals reset by the last CTA of the step).
    int att_splits, att_split_min;
    float *apart;
    unsigned *hbar;
    // Shared-memory carve-up, in floats from the base (host-computed).
    // xs: the current activation vector in the quad-major layout; h2: the
    // residual stream; gain: norm gains; rv: per-row scales/biases; sc:
    // attention scores or the CTA's logits; q: q, k, v of one head; red:
    // cross-warp partials; lay: the layer table.  gain and rv are double
    // buffers of sm_gain_n and sm_rv_n floats each.
    int sm_xs, sm_h2, sm_gain, sm_rv, sm_sc, sm_q, sm_red, sm_lay;
    int sm_gain_n, sm_rv_n;
    // The page table's first ceil(cap / 16) entries, staged by every step.
    int sm_ptab;
    // Weight ring: nslot slots of slot_bytes at sm_ring (128-byte aligned) and
    // their full/empty mbarriers at sm_bar (2 * nslot, 8-byte aligned).
    int sm_bar, sm_ring, nslot, slot_bytes, sm_total;
};

// Shared-memory bytes the kernel needs for these parameters.
size_t decode_smem_bytes(const DecodeParams &p);
// Launches one decode step (cooperative, one CTA per SM).
// split: the instantiation with the long-context position-split attention
// (used from att_split_min cached positions on; the other one never splits).
cudaError_t decode_launch(const DecodeParams &p, int grid, cudaStream_t stream, bool split);
// Compute threads per CTA; one more warp streams the weights.  16 warps in
// all put 4 on each SM sub-partition, whose 16K registers then allow 128
// registers per thread.
constexpr int kDecodeThreads = 480;
constexpr int kDecodeBlock = kDecodeThreads + 32;

}  // namespace qb
