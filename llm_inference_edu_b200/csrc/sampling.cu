// Seeded temperature / top-k sampling, Sampler::sample (src/sampling.rs:57-110).
//
// One CTA of 1024 threads over the vocabulary row (it follows a decode step
// whose logits are still in L2):
//   pass 1   every logit: finiteness, the greedy id (strict >, lowest id on
//            ties) and a 256-bin histogram of the top byte of its rank key;
//   pass 2-4 the remaining bytes of the k-th key (radix select), each over
//            the logits whose key matches the bytes found so far;
//   gather   every id whose key is at or before the k-th (the k best plus the
//            ties of the k-th), as 64-bit (key, id) words;
//   sort     those words ascending (bitonic; shared memory up to 4096 words,
//            the scratch buffer beyond): the order (logit desc, id asc) the
//            reference gives its candidates; the first k are the top-k;
//   walk     FP64 masses exp((logit - max) / T) in that order (parallel),
//            then one thread sums them in order, scales the draw and walks
//            the cumulative sum, exactly as the reference does.
// The rank key of a logit x is ~ord(x), ord the order-preserving map of the
// float bits (-0 mapped with +0: they compare equal), so ascending keys are
// descending logits.  FP64 exp is CUDA's (max 1 ulp); the reference's is the
// platform libm's, so a draw landing within rounding of a cumulative
// boundary could pick the neighbouring id.
#include <climits>

#include "common.cuh"
#include "sampling.cuh"

namespace qb {

namespace {

constexpr int SAMPLE_THREADS = 1024;
constexpr int SAMPLE_SMEM_WORDS = 4096;
constexpr unsigned kNoBin = 0xffffffffu;

__device__ __forceinline__ unsigned rank_key(float x) {
    const unsigned b = __float_as_uint(x == 0.0f ? 0.0f : x);
    const unsigned ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ~ord;
}

__device__ __forceinline__ unsigned pow2_ceil(unsigned v) {
    unsigned p = 1;
    while (p < v) p <<= 1;
    return p;
}

// Visits every element once: f(i, x, ok) for this thread's elements, in
// batches of four 16-byte loads all in flight before the first use (the
// passes are bound by load latency, not bandwidth).  Every thread of the
// block makes the same calls (ok = false past the end), so f may use
// warp-collective operations.  A base that is not 16-byte aligned takes
// the scalar path.
constexpr int kVisitBatch = 4;
template <class F>
__device__ __forceinline__ void visit(const float *__restrict__ logits, int n, F &&f) {
    const int tid = threadIdx.x;
    if (((uintptr_t)logits & 15) == 0) {
        const float4 *l4 = reinterpret_cast<const float4 *>(logits);
        const int n4 = n >> 2, iters = (n4 + SAMPLE_THREADS - 1) / SAMPLE_THREADS;
#pragma unroll 1
        for (int it = 0; it < iters; it += kVisitBatch) {
            float4 v[kVisitBatch];
#pragma unroll
            for (int b = 0; b < kVisitBatch; ++b) {
                const int f4 = (it + b) * SAMPLE_THREADS + tid;
                v[b] = f4 < n4 ? __ldcg(l4 + f4) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
#pragma unroll
            for (int b = 0; b < kVisitBatch; ++b) {
                const int f4 = (it + b) * SAMPLE_THREADS + tid;
                const bool ok = f4 < n4;
                f(4 * f4, v[b].x, ok);
                f(4 * f4 + 1, v[b].y, ok);
                f(4 * f4 + 2, v[b].z, ok);
                f(4 * f4 + 3, v[b].w, ok);
            }
        }
        const int i = 4 * n4 + tid;  // the last n % 4 elements
        const bool ok = i < n;
        f(i, ok ? __ldcg(logits + i) : 0.0f, ok);
    } else {
        const int iters = (n + SAMPLE_THREADS - 1) / SAMPLE_THREADS;
#pragma unroll 1
        for (int it = 0; it < iters; it += kVisitBatch) {
            float v[kVisitBatch];
#pragma unroll
            for (int b = 0; b < kVisitBatch; ++b) {
                const int i = (it + b) * SAMPLE_THREADS + tid;
                v[b] = i < n ? __ldcg(logits + i) : 0.0f;
            }
#pragma unroll
            for (int b = 0; b < kVisitBatch; ++b) {
                const int i = (it + b) * SAMPLE_THREADS + tid;
                f(i, v[b], i < n);
            }
        }
    }
}

// Adds 1 to hist[bin] for every lane whose bin != kNoBin, one shared atomic
// per distinct bin of the warp (nothing when no lane has a bin).
__device__ __forceinline__ void warp_hist_add(unsigned *hist, unsigned bin) {
    if (!__any_sync(0xffffffffu, bin != kNoBin)) return;
    const unsigned peers = __match_any_sync(0xffffffffu, bin);
    const int lane = threadIdx.x & 31;
    if (bin != kNoBin && lane == __ffs(peers) - 1) atomicAdd(&hist[bin], __popc(peers));
}

// Warp 0: the bin holding the rem-th element (1-based) of the histogram in
// bin order; writes the bin, the count before it and its own count.
__device__ __forceinline__ void find_bin(const unsigned *hist, unsigned rem, unsigned *s_bin, unsigned *s_before,
                                         unsigned *s_count) {
    const int lane = threadIdx.x & 31;
    unsigned c[8], sum = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) { c[j] = hist[lane * 8 + j]; sum += c[j]; }
    unsigned incl = sum;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const unsigned o = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += o;
    }
    const unsigned excl = incl - sum;
    if (excl < rem && rem <= incl) {
        unsigned before = excl;
        for (int j = 0; j < 8; ++j) {
            if (rem <= before + c[j]) {
                *s_bin = lane * 8 + j;
                *s_before = before;
                *s_count = c[j];
                break;
            }
            before += c[j];
        }
    }
}

// Ascending bitonic sort of the P words at c (P a power of two), all
// threads of the block.
__device__ void bitonic_sort(unsigned long long *c, unsigned P) {
    for (unsigned size = 2; size <= P; size <<= 1) {
        for (unsigned stride = size >> 1; stride > 0; stride >>= 1) {
            for (unsigned t = threadIdx.x; t < P / 2; t += blockDim.x) {
                const unsigned lo = 2 * stride * (t / stride) + (t % stride), hi = lo + stride;
                const bool up = (lo & size) == 0;
                const unsigned long long a = c[lo], b = c[hi];
                if ((a > b) == up) { c[lo] = b; c[hi] = a; }
            }
            __syncthreads();
        }
    }
}

__global__ void __launch_bounds__(SAMPLE_THREADS, 1)
sample_kernel(const float *__restrict__ logits, int n, int greedy, float temperature, int k, double u,
              unsigned long long *__restrict__ gcand, double *__restrict__ gmass, uint32_t *out) {
    extern __shared__ __align__(16) unsigned char sample_smem[];
    unsigned long long *scand = reinterpret_cast<unsigned long long *>(sample_smem);
    double *smass = reinterpret_cast<double *>(sample_smem + SAMPLE_SMEM_WORDS * 8);
    __shared__ unsigned hist[256];
    __shared__ float red_v[32];
    __shared__ int red_i[32];
    __shared__ unsigned s_bin, s_before, s_count, s_fill, s_bad;
    __shared__ int s_best;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    if (tid == 0) s_bad = 0;
    if (tid < 256) hist[tid] = 0;
    __syncthreads();

    // Pass 1: finiteness, greedy id, top-byte histogram.
    float bv = 0.0f;
    int bi = INT_MAX;
    bool bad = false;
    // Each thread meets its elements in increasing index order, so strict >
    // keeps the lowest index among equal values.
    visit(logits, n, [&](int i, float x, bool ok) {
        unsigned bin = kNoBin;
        if (ok) {
            if (!isfinite(x)) bad = true;
            if (bi == INT_MAX || x > bv) { bv = x; bi = i; }
            bin = rank_key(x) >> 24;
        }
        if (!greedy) warp_hist_add(hist, bin);
    });
    if (bad) s_bad = 1;
#pragma unroll
    for (int off = 16; off; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (oi != INT_MAX && (bi == INT_MAX || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
    }
    if (lane == 0) { red_v[warp] = bv; red_i[warp] = bi; }
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < SAMPLE_THREADS / 32; ++w)
            if (red_i[w] != INT_MAX && (bi == INT_MAX || red_v[w] > bv || (red_v[w] == bv && red_i[w] < bi))) {
                bv = red_v[w];
                bi = red_i[w];
            }
        s_best = bi;
    }
    __syncthreads();
    if (s_bad) {
        if (tid == 0) { out[0] = 0; out[1] = QB_NONFINITE; }
        return;
    }
    const int best = s_best;
    if (greedy) {
        if (tid == 0) { out[0] = (uint32_t)best; out[1] = 0; }
        return;
    }

    // Passes 1-4 of the radix select: the k-th smallest rank key.
    unsigned prefix = 0, pmask = 0, rem = (unsigned)k;
    for (int shift = 24;; shift -= 8) {
        if (warp == 0) find_bin(hist, rem, &s_bin, &s_before, &s_count);
        __syncthreads();
        prefix |= s_bin << shift;
        pmask |= 0xffu << shift;
        rem -= s_before;
        if (shift == 0) break;
        __syncthreads();  // everyone has read s_bin / s_before
        if (tid < 256) hist[tid] = 0;
        __syncthreads();
        visit(logits, n, [&](int, float x, bool ok) {
            unsigned bin = kNoBin;
            if (ok) {
                const unsigned key = rank_key(x);
                if ((key & pmask) == prefix) bin = (key >> (shift - 8)) & 0xffu;
            }
            warp_hist_add(hist, bin);
        });
        __syncthreads();
    }
    // prefix = the k-th key; the gather takes (k - rem) keys before it and
    // all s_count keys equal to it.
    const unsigned kth = prefix;
    const unsigned m = (unsigned)k - rem + s_count;
    const unsigned P = pow2_ceil(m);
    unsigned long long *cand = P <= (unsigned)SAMPLE_SMEM_WORDS ? scand : gcand;
    double *mass = k <= SAMPLE_SMEM_WORDS ? smass : gmass;
    if (tid == 0) s_fill = 0;
    __syncthreads();
    visit(logits, n, [&](int i, float x, bool ok) {
        const unsigned key = ok ? rank_key(x) : 0xffffffffu;
        const bool take = ok && key <= kth;
        const unsigned vote = __ballot_sync(0xffffffffu, take);
        if (!vote) return;
        unsigned base = 0;
        if (lane == 0) base = atomicAdd(&s_fill, __popc(vote));
        base = __shfl_sync(0xffffffffu, base, 0);
        if (take) cand[base + __popc(vote & ((1u << lane) - 1u))] = (unsigned long long)key << 32 | (unsigned)i;
    });
    for (unsigned j = m + tid; j < P; j += SAMPLE_THREADS) cand[j] = ~0ull;
    __syncthreads();
    bitonic_sort(cand, P);

    // Masses of the top-k in order, then the reference's sequential walk.
    const double maximum = (double)logits[best], t = (double)temperature;
    for (int j = tid; j < k; j += SAMPLE_THREADS) {
        const unsigned id = (unsigned)(cand[j] & 0xffffffffu);
        mass[j] = exp(((double)logits[id] - maximum) / t);
    }
    __syncthreads();
    if (tid == 0) {
        double total = 0.0;
        for (int j = 0; j < k; ++j) total += mass[j];
        const double target = u * total;
        double cumulative = 0.0;
        unsigned last_positive = (unsigned)best, pick = kNoBin;
        for (int j = 0; j < k; ++j) {
            const double w = mass[j];
            const unsigned id = (unsigned)(cand[j] & 0xffffffffu);
            if (w > 0.0) last_positive = id;
            cumulative += w;
            if (target < cumulative) { pick = id; break; }
        }
        out[0] = pick == kNoBin ? last_positive : pick;
        out[1] = 0;
    }
}

}  // namespace

void ChaCha8Rng::seed_from_u64(uint64_t seed) {
    uint64_t state = seed;
    for (int i = 0; i < 8; ++i) {
        state = state * 6364136223846793005ull + 11634580027462260723ull;
        const uint32_t xs = (uint32_t)(((state >> 18) ^ state) >> 27);
        const uint32_t rot = (uint32_t)(state >> 59);
        key[i] = (xs >> rot) | (xs << ((32 - rot) & 31));  // the little-endian seed word
    }
    counter = 0;
    index = 64;
}

static inline uint32_t rotl(uint32_t v, int c) { return (v << c) | (v >> (32 - c)); }

uint64_t ChaCha8Rng::next_u64() {
    if (index >= 64) {
        for (int b = 0; b < 4; ++b) {
            uint32_t in[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u};
            for (int i = 0; i < 8; ++i) in[4 + i] = key[i];
            const uint64_t c = counter + (uint64_t)b;
            in[12] = (uint32_t)c;
            in[13] = (uint32_t)(c >> 32);
            in[14] = 0;
            in[15] = 0;
            uint32_t x[16];
            for (int i = 0; i < 16; ++i) x[i] = in[i];
            auto qr = [&x](int a, int bb, int cc, int d) {
                x[a] += x[bb]; x[d] = rotl(x[d] ^ x[a], 16);
                x[cc] += x[d]; x[bb] = rotl(x[bb] ^ x[cc], 12);
                x[a] += x[bb]; x[d] = rotl(x[d] ^ x[a], 8);
                x[cc] += x[d]; x[bb] = rotl(x[bb] ^ x[cc], 7);
            };
            for (int r = 0; r < 8; r += 2) {
                qr(0, 4, 8, 12); qr(1, 5, 9, 13); qr(2, 6, 10, 14); qr(3, 7, 11, 15);
                qr(0, 5, 10, 15); qr(1, 6, 11, 12); qr(2, 7, 8, 13); qr(3, 4, 9, 14);
            }
            for (int i = 0; i < 16; ++i) buf[16 * b + i] = x[i] + in[i];
        }
        counter += 4;
        index = 0;
    }
    const uint64_t v = (uint64_t)buf[index] | (uint64_t)buf[index + 1] << 32;
    index += 2;
    return v;
}

double ChaCha8Rng::next_f64() { return (double)(next_u64() >> 11) * (1.0 / 9007199254740992.0); }

static unsigned host_pow2_ceil(unsigned v) {
    unsigned p = 1;
    while (p < v) p <<= 1;
    return p;
}

size_t sample_scratch_bytes(int n) {
    // candidate words (rounded to a power of two) then the masses
    return (size_t)host_pow2_ceil((unsigned)n) * 8 + (size_t)n * 8;
}

cudaError_t sample_launch(const float *logits, int n, const SamplePolicy &p, double u, void *scratch,
                          uint32_t *out, cudaStream_t st) {
    const size_t smem = (size_t)SAMPLE_SMEM_WORDS * 16;
    cudaError_t e = cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    unsigned long long *gcand = (unsigned long long *)scratch;
    double *gmass = (double *)((uint8_t *)scratch + (size_t)host_pow2_ceil((unsigned)n) * 8);
    sample_kernel<<<1, SAMPLE_THREADS, smem, st>>>(logits, n, p.greedy ? 1 : 0, p.temperature,
                                                   p.greedy ? 1 : (int)p.top_k, u, gcand, gmass, out);
    return cudaGetLastError();
}

}  // namespace qb
