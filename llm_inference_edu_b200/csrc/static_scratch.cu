// qb_rope_static: RoPE that allocates nothing.  Same admission, results and
// error behaviour as qb_rope, but its device scratch is a fixed static array
// in this library's module, and the host stages the angle table through a
// small stack buffer.  No heap, no cudaMalloc/cudaFree, no allocating
// library routine.
//
// Who needs it: a serving process that has already divided device memory
// between weights and KV pages (a late cudaMalloc there can fail, or
// fragment memory another allocator owns), and latency-bound code with work
// in flight on other streams (cudaFree waits for the whole device).
#include <math.h>
#include <atomic>

#include "common.cuh"

namespace qb {

// Defined with the other operator kernels (ops.cu).
__global__ void nonfinite_scan(const float *__restrict__ v, size_t n,
                               unsigned long long *__restrict__ first);
__global__ void rope_kernel(const float *__restrict__ x, float *__restrict__ y,
                            const float *__restrict__ cs, size_t tokens, size_t heads,
                            size_t hd);

// Layout: bytes [0, 256) hold the flag word (first non-finite index, reset to
// all-ones by every call); bytes [256, end) hold the (cos, sin) table, fully
// written by every call before the kernel reads it.
constexpr size_t kStaticFlagBytes = 256;
static_assert(QB_ROPE_STATIC_SCRATCH_BYTES - kStaticFlagBytes == 4 * (size_t)QB_ROPE_STATIC_MAX_TABLE,
              "table limit must match the array");
static __device__ __align__(256) unsigned char g_rope_static_scratch[QB_ROPE_STATIC_SCRATCH_BYTES];

// Address of the array on each device (the module is loaded per device, so
// each device has its own copy).  Looked up once per device; the lookup is
// idempotent, so concurrent first calls store the same value.
constexpr int kMaxCachedDevices = 64;
static std::atomic<void *> g_static_addr[kMaxCachedDevices];

static uint32_t static_scratch(void **out) {
    int dev = 0;
    QB_CUDA(cudaGetDevice(&dev));
    if (dev >= 0 && dev < kMaxCachedDevices) {
        void *p = g_static_addr[dev].load(std::memory_order_acquire);
        if (p) {
            *out = p;
            return QB_OK;
        }
    }
    void *p = nullptr;
    QB_CUDA(cudaGetSymbolAddress(&p, g_rope_static_scratch));
    if (dev >= 0 && dev < kMaxCachedDevices) g_static_addr[dev].store(p, std::memory_order_release);
    *out = p;
    return QB_OK;
}

static unsigned static_grid(size_t n, size_t cap) {
    size_t b = (n + 255) / 256;
    return (unsigned)(b > cap ? cap : (b == 0 ? 1 : b));
}

}  // namespace qb

using namespace qb;

extern "C" uint32_t qb_rope_static(const float *x, size_t xl, float *y, size_t yl, size_t tokens,
                                   size_t heads, size_t hd, size_t start, float base,
                                   void *stream) {
    clear_detail();
    // Admission identical to qb_rope (src/rope.rs:38-105 order).
    if (tokens == 0 || heads == 0 || hd == 0) return QB_ZERO_DIMENSION;
    if (hd % 2) return QB_ODD_HEAD_DIMENSION;
    size_t row, len;
    if (mul_ovf(heads, hd, &row) || mul_ovf(tokens, row, &len)) return QB_DIMENSION_OVERFLOW;
    if (start > SIZE_MAX - (tokens - 1)) return QB_POSITION_OVERFLOW;
    size_t last = start + tokens - 1;
    if (last > ((size_t)1 << 24)) return QB_POSITION_OUT_OF_RANGE;
    if (!isfinite(base) || base <= 0.0f) return QB_INVALID_BASE;
    if (xl != len) { set_detail(0, len, xl); return QB_INVALID_LENGTH; }
    if (yl != len) { set_detail(1, len, yl); return QB_INVALID_LENGTH; }
    const size_t half = hd / 2;
    for (size_t j = 0; j < half; ++j) {
        float f = powf(base, -((float)(2 * j)) / (float)hd);
        if (!isfinite(f) || !isfinite((float)last * f)) return QB_INVALID_ANGLE;
    }
    // The fixed scratch bounds the table: tokens * head_dim floats.
    const size_t table = tokens * hd;  // <= len, so no overflow
    if (table > QB_ROPE_STATIC_MAX_TABLE) {
        set_detail(0, QB_ROPE_STATIC_MAX_TABLE, table);
        return QB_RESOURCE_BUDGET;
    }

    void *base_ptr;
    uint32_t s = static_scratch(&base_ptr);
    if (s) return s;
    unsigned long long *flag = (unsigned long long *)base_ptr;
    float *dcs = (float *)((char *)base_ptr + kStaticFlagBytes);
    cudaStream_t st = (cudaStream_t)stream;

    // Non-finite input check before any output is written.
    QB_CUDA(cudaMemsetAsync(flag, 0xff, sizeof(unsigned long long), st));
    nonfinite_scan<<<static_grid(len, 4096), 256, 0, st>>>(x, len, flag);
    QB_CUDA(cudaGetLastError());
    unsigned long long first;
    QB_CUDA(cudaMemcpyAsync(&first, flag, sizeof first, cudaMemcpyDeviceToHost, st));
    QB_CUDA(cudaStreamSynchronize(st));
    if (first != ~0ull) { set_detail(0, 0, 0, (size_t)first); return QB_NONFINITE; }

    // (cos, sin) per (token, pair) with the host's powf/cosf/sinf, staged in
    // 16 KiB pieces; the stream is synchronized before the buffer is reused.
    constexpr size_t kPiece = 4096;  // floats
    float buf[kPiece];
    const size_t pairs = tokens * half;
    for (size_t k0 = 0; k0 < pairs; k0 += kPiece / 2) {
        const size_t n = pairs - k0 < kPiece / 2 ? pairs - k0 : kPiece / 2;
        for (size_t i = 0; i < n; ++i) {
            const size_t k = k0 + i, t = k / half, j = k % half;
            const float f = powf(base, -((float)(2 * j)) / (float)hd);
            const float a = (float)(start + t) * f;
            buf[2 * i] = cosf(a);
            buf[2 * i + 1] = sinf(a);
        }
        QB_CUDA(cudaMemcpyAsync(dcs + 2 * k0, buf, n * 2 * sizeof(float), cudaMemcpyHostToDevice, st));
        QB_CUDA(cudaStreamSynchronize(st));
    }
    rope_kernel<<<static_grid(pairs * heads, 8192), 256, 0, st>>>(x, y, dcs, tokens, heads, hd);
    QB_CUDA(cudaGetLastError());
    QB_CUDA(cudaStreamSynchronize(st));
    return QB_OK;
}
