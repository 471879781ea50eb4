// Tensor-core (tcgen05) GEMM of the multi-token path: Y[t][r] =
// epilogue(sum_k X[t][k] W[r][k]) for INT8 (per-row scale) or BF16 weights
// in the decode layouts, with the FP32 input X given as BF16 planes
// (mt::Planes) so that the BF16 x BF16 -> FP32 tensor-core products
// reproduce the FP32 products of the reference's dot to about 2^-24.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <vector>

#include "multitoken.cuh"

namespace qb {

// A weight matrix as a TMA tensor map: dimensions {seg_len, rows, nseg},
// boxes of 64 reduction elements x 128 rows.
struct alignas(64) TcWeightMap {
    CUtensorMap map;
    int wf = -1;        // WF_I8 or WF_BF16; -1 when not built
    int seg_kb = 0;     // 64-element blocks per segment
};

struct TcLayerMaps {
    TcWeightMap qkv, o, gu, down;
};

constexpr int TC_NP = 3;       // BF16 planes per input element
constexpr int TC_TILES = 8;    // token tiles 16, 32, ..., 128

// Every tensor map of one multi-token workspace.
struct TcMaps {
    std::vector<TcLayerMaps> layers;   // empty when the linears run on CUDA cores
    TcWeightMap head;                  // wf -1 when the LM head runs on CUDA cores
    // Input planes [TC_NP][chunk][K] for token tiles of 16 (i + 1) rows.
    struct alignas(64) X { CUtensorMap m[TC_TILES]; } xn, ctx, act;
};

// One GEMM on the tensor cores.
struct TcJob {
    int epi;                 // mt::EPI_*
    int n, N, K;
    const TcWeightMap *w;
    const TcMaps::X *x;
    mt::GemmW gw;            // scale and bias (the layout is in the map)
    const float *R;
    int ldr;
    float *Y;
    int ldy;
    mt::Planes P;            // SwiGLU output planes (EPI_GU) or null
    // EPI_PLAIN: per 128-row tile and token, the tile's greedy (value, id)
    // ([ceil(N / 128)][n]; null: not wanted).
    float *amv;
    int *ami;
    // EPI_QKV: RoPE and the KV write fused into the epilogue (null: the
    // plain QKV epilogue).
    const mt::RopeKv *rk;
};

// Builds a weight map; false when the layout does not suit TMA.
bool tc_encode_weight(TcWeightMap &m, const uint8_t *base, int wf, size_t rows, size_t seg_len, size_t row_stride,
                      size_t nseg, size_t seg_stride);
// Builds the input-plane maps of a [TC_NP][chunk][K] BF16 buffer.
bool tc_encode_planes(TcMaps::X &x, const uint16_t *p, int K, int chunk);

// Launches the GEMM (K split across the CTAs of a cluster when the output
// tiles alone leave SMs idle).  With amv / ami set, *am_tiles receives the
// number of tiles whose greedy partials were written (0 when K was split:
// the caller scans the logits).
cudaError_t tc_gemm(const TcJob &j, unsigned *err, cudaStream_t st, int *am_tiles = nullptr);

}  // namespace qb
