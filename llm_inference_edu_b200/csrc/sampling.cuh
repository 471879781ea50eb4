// Seeded temperature / top-k sampling (src/sampling.rs:5-110): the
// generator on the host, the selection over the vocabulary on the device.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

namespace qb {

// rand_chacha 0.9's ChaCha8Rng: ChaCha with 8 rounds, 256-bit key, 64-bit
// block counter (state words 12-13), stream 0 (words 14-15), a buffer of
// four blocks; next_u64 = word i | word i+1 << 32.  Seeded like rand_core
// 0.9's SeedableRng::seed_from_u64 (PCG32 output words form the key).
struct ChaCha8Rng {
    uint32_t key[8];
    uint64_t counter;
    uint32_t buf[64];
    unsigned index;
    void seed_from_u64(uint64_t seed);
    uint64_t next_u64();
    // rand 0.9's random::<f64>(): the top 53 bits times 2^-53.
    double next_f64();
};

struct SamplePolicy {
    bool greedy = true;
    float temperature = 1.0f;
    size_t top_k = 1;
};

// Device scratch of one sampler for vocabularies up to n.
size_t sample_scratch_bytes(int n);

// One sample from the n logits at `logits` (device) on `st`: out[0] = the
// id, out[1] = 0 or QB_NONFINITE (device words).  `u` is the generator's
// draw in [0, 1); unused by the greedy policy.  Requires 1 <= top_k <= n.
cudaError_t sample_launch(const float *logits, int n, const SamplePolicy &p, double u, void *scratch,
                          uint32_t *out, cudaStream_t st);

}  // namespace qb
