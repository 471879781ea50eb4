// Tensor parallelism across the GPUs of one box: the sums after o_proj and
// down (the reduction sites of src/kv_cache.rs:581-585 and 437-443) and the
// greedy argmax over a vocabulary split by rank.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

namespace qb {

constexpr int kMaxTp = 8;

// What the exchange kernels see of the ranks' communication buffers (device
// pointers; index r is rank r's buffer, opened through CUDA IPC for the
// peers).  Rank r's buffer holds:
//   flags [2 slots][kMaxTp] u32: flags[s][j] = sequence number of rank j's
//         latest call that used slot s (rank j stores it with a system-scope
//         release once its data for that call is complete);
//   part  [2 slots][rows][h] FP32: this rank's partial sums of one reduction;
//   amx   [2 slots][rows] float2: this rank's (best logit, global id as bits).
// A call with sequence number q uses slot q & 1: a rank can only be one call
// ahead of the slowest (each call waits for every rank's flag), so a slot is
// never rewritten while a peer still reads it.
struct TpPeers {
    int rank, size, rows, h;
    unsigned *flags[kMaxTp];
    float *part[kMaxTp];
    float2 *amx[kMaxTp];
};

// Bytes of one rank's buffer for `rows` rows of width h.
size_t tp_buffer_bytes(int rows, int h);
// Pointers into a buffer at `base`.
void tp_carve(void *base, int rows, int h, unsigned **flags, float **part, float2 **amx);

// Y[i] = R[i] + (part_0[i] + part_1[i] + ... + part_{size-1}[i]) for the n
// rows of width h of slot `seq & 1`, every rank's partials summed in rank
// order (the same value on every rank).  Signals this rank's partials (its
// slot was written by the kernels before on `st`), waits (bounded) for every
// rank's, then sums.  ERR_TIMEOUT in *err when a rank's flag did not come.
cudaError_t tp_allreduce(const TpPeers &P, unsigned seq, int n, const float *R, float *Y, unsigned *err,
                         unsigned long long timeout_ns, cudaStream_t st);

// Each token's greedy id over the whole vocabulary: this rank's logits
// [n][nv] cover global ids v0 .. v0 + nv - 1; the best (strict >, lowest
// id) of every rank's slice is combined in rank order (ties keep the lower
// rank, whose ids are lower).  Writes out[t] on every rank.  pv / pi: the
// per-slice partials, tp_argmax_scratch(rows) of each.
cudaError_t tp_argmax(const TpPeers &P, unsigned seq, const float *logits, int n, int nv, int v0, uint32_t *out,
                      float *pv, int *pi, unsigned *err, unsigned long long timeout_ns, cudaStream_t st);
size_t tp_argmax_scratch(int rows);

}  // namespace qb
