// Chunked prompt evaluation: fills the KV cache for a run of prompt tokens
// with a few wide kernels per layer instead of one decode step per token.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

#include "decode.cuh"

namespace qb {

// Everything the chunked path reads or writes (device pointers unless
// noted).  The layer table is a host copy of the session's DecodeLayer
// array (weights in the decode layout, KV pointers of this session).
struct PrefillArgs {
    int V, L, h, qh, kvh, hd, ff, cap, group;
    int wfmt, tfmt, kv_bf16;
    float eps, sqrt_hd;
    size_t sh, shd, sff, semb;
    const uint8_t *emb;           // [V, semb] embedding table
    const DecodeLayer *layers;    // HOST array [L]
    const float2 *rope;           // [cap][hd/2] (cos, sin)
    int chunk;                    // workspace rows (tokens per chunk)
    // Workspace, `chunk` rows each.
    float *x;                     // [chunk][h] residual stream
    float *xn;                    // [chunk][h] normalized rows
    float *h2;                    // [chunk][h] after attention
    float *qkv;                   // [chunk][h + 2 kv]
    float *ctx;                   // [chunk][h] attention context
    float *act;                   // [chunk][ff] SwiGLU output
    uint32_t *ids;                // [chunk] token ids
    unsigned *err;                // error flags (ERR_NONFINITE)
};

// True when the shapes suit the chunked kernels (else callers evaluate the
// tokens one decode step at a time).
bool prefill_supported(const PrefillArgs &a);

// Writes the K/V of every layer for tokens[0, n) at positions p0 .. p0+n-1
// (tokens on the HOST).  The chunk's own attention is causal over the cache
// plus the chunk.  The final layer's MLP is skipped: only the cache is
// produced.  Errors: the CUDA status; *nonfinite set when any value was not
// finite.
cudaError_t prefill_kv(const PrefillArgs &a, const uint32_t *tokens, int n, int p0, cudaStream_t st,
                       bool *nonfinite);

}  // namespace qb
