// Multi-token forward: many tokens per launch sequence instead of one
// decode step per token.  Serves the chunked prompt path of a session
// (KV fill) and batched greedy decoding of independent sequences.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

#include "decode.cuh"
#include "tp.cuh"

namespace qb {

struct TcMaps;

// The paged KV cache of one or more sequences: per layer l a K pool at
// pool + 2 l layer_bytes and a V pool right after it, each a pool of pages
// [kv_heads][16][head_dim]; sequence s's page j is pool page ptab[s pps + j].
struct KvPages {
    uint8_t *pool;
    size_t layer_bytes;
    const int *ptab;
    int pps;  // pages per sequence (table row length)
    int kvh, hd;
    // Element offset of the row of (sequence s, KV head g, position p) in a pool.
    __device__ __forceinline__ size_t row(int s, int g, int p) const {
        const int page = ptab[(size_t)s * pps + p / kPageTokens];
        return (((size_t)page * kvh + g) * kPageTokens + (p % kPageTokens)) * (size_t)hd;
    }
    __device__ __forceinline__ uint8_t *k(int l) const { return pool + (size_t)(2 * l) * layer_bytes; }
    __device__ __forceinline__ uint8_t *v(int l) const { return pool + (size_t)(2 * l + 1) * layer_bytes; }
};

// Everything the multi-token kernels read or write (device pointers unless
// noted).  The layer table is a host copy of a DecodeLayer array whose
// weights are in the decode layout; its KV pointers are ignored: the cache
// is `kv`.
struct PrefillArgs {
    // With tensor parallelism (tp set) the model is one rank's shard: qh
    // query heads of head_dim (qd = qh * hd query rows, the context width),
    // kvh KV heads (group = qh / kvh query heads each), ff FFN columns and
    // V LM-head rows starting at global id v0; h is always the full width.
    int V, L, h, qh, kvh, hd, ff, cap, group;
    int qd, v0;
    int wfmt, tfmt, kv_bf16;
    float eps, sqrt_hd;
    size_t sh, shd, sff, semb;
    const uint8_t *emb;           // [V, semb] embedding table
    const uint8_t *head;          // LM-head table (== emb when tied)
    const float *final_norm;      // [h]
    const DecodeLayer *layers;    // HOST array [L]
    const float2 *rope;           // [cap][hd/2] (cos, sin)
    KvPages kv;                   // the paged cache
    int chunk;                    // workspace rows (tokens per launch sequence)
    // Workspace, `chunk` rows each.
    float *x;                     // [chunk][h] residual stream
    float *xn;                    // [chunk][h] normalized rows
    float *h2;                    // [chunk][h] after attention
    float *qkv;                   // [chunk][h + 2 kv]
    float *ctx;                   // [chunk][h] attention context
    float *act;                   // [chunk][ff] SwiGLU output
    float *part;                  // split-K partial sums, part_floats floats
    size_t part_floats;
    uint32_t *ids;                // [chunk] token ids
    int *pos;                     // [chunk] positions
    int *seq;                     // [chunk] sequence indices
    float *logits;                // [chunk][V] (null unless the LM head runs)
    uint32_t *amax;               // [chunk] greedy ids (null unless the LM head runs)
    unsigned *err;                // error flags (ERR_NONFINITE)
    // Tensor-core path: BF16 planes [TC_NP][chunk][K] of the GEMM inputs
    // (normalized rows, attention context, SwiGLU output) and the tensor
    // maps (HOST; null: every GEMM runs on the CUDA cores).
    uint16_t *xnp, *ctxp, *actp;
    const TcMaps *tc;
    // Attention position-split partials (apart_floats floats) and the LM
    // head's per-tile greedy partials ([ceil(V / 128)][chunk]).
    float *apart;
    size_t apart_floats;
    float *amv;
    int *ami;
    // Tensor parallelism (HOST pointers; tp null without it): the ranks'
    // exchange buffers and the communicator's call counter (every rank makes
    // the same calls in the same order).
    const TpPeers *tp;
    unsigned *tp_seq;
    unsigned long long tp_timeout_ns;
};

// True when the shapes suit the multi-token kernels (else callers evaluate
// the tokens one decode step at a time).
bool prefill_supported(const PrefillArgs &a);

// Runs n <= chunk tokens whose ids, positions and sequences are already in
// a.ids / a.pos / a.seq; max_pos is the largest position among them.  Each
// token attends to its own sequence's positions 0 .. pos (its own K/V
// included).  With lm_head the final layer runs in full and a.logits /
// a.amax receive each token's logits and greedy id (strict >, lowest id on
// ties, src/sampling.rs:65-70); without it the final layer's MLP is skipped
// (only the cache is produced).  Errors land in a.err (not cleared here).
cudaError_t forward_tokens(const PrefillArgs &a, int n, int max_pos, bool lm_head, cudaStream_t st);

// Chunked prompt path of one session (sequence 0): the K/V of tokens[0, n)
// (HOST) at positions p0 .. p0+n-1.  *nonfinite is set when any value was
// not finite.
cudaError_t prefill_kv(const PrefillArgs &a, const uint32_t *tokens, int n, int p0, cudaStream_t st,
                       bool *nonfinite);

// Advances every position in a.pos[0, n) by one and copies a.amax into
// a.ids (the next step's tokens), on the device.
cudaError_t advance_tokens(const PrefillArgs &a, int n, cudaStream_t st);

}  // namespace qb
