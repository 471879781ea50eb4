// Standalone sm_100a kernels behind the reference's operator interface:
// linear (src/lib.rs:51), linear_lanes4 (src/kernels.rs:10), the INT8 scheme
// (src/quantization.rs:55-281), the elementwise ops (src/ops.rs:67-257) and
// RoPE (src/rope.rs:38-105).  The decode megakernel fuses all of these; these
// entry points keep each operator callable and testable on its own.
//
// Admission mirrors the reference exactly and finishes before the first
// write.  Checks that must read device values (finiteness, masks, scale
// underflow) run as a scan kernel into a small library-owned flag buffer,
// and the call synchronizes its stream before writing any output.
#include <math.h>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace qb {

static thread_local qb_detail g_detail;
static thread_local int g_last_cuda = 0;

void set_detail(size_t buffer, size_t expected, size_t actual, size_t index) {
    g_detail.buffer = buffer;
    g_detail.expected = expected;
    g_detail.actual = actual;
    g_detail.index = index;
}
void clear_detail() { g_detail = qb_detail{0, 0, 0, 0}; }
uint32_t cuda_status(cudaError_t e) {
    if (e == cudaSuccess) return QB_OK;
    g_last_cuda = (int)e;
    return QB_CUDA_ERROR;
}

static std::mutex g_scratch_mu;
static std::vector<DeviceScratch> g_scratch;

uint32_t scratch_get(size_t bytes, void **out) {
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    int dev = 0;
    QB_CUDA(cudaGetDevice(&dev));
    for (auto &s : g_scratch) {
        if (s.device == dev) {
            if (s.bytes < bytes) {
                QB_CUDA(cudaFree(s.ptr));
                s.ptr = nullptr;
                QB_CUDA(cudaMalloc(&s.ptr, bytes));
                s.bytes = bytes;
            }
            *out = s.ptr;
            return QB_OK;
        }
    }
    DeviceScratch s;
    s.device = dev;
    QB_CUDA(cudaMalloc(&s.ptr, bytes < 4096 ? 4096 : bytes));
    s.bytes = bytes < 4096 ? 4096 : bytes;
    g_scratch.push_back(s);
    *out = s.ptr;
    return QB_OK;
}

// ------------------------------------------------------------- linear ----

// One thread per (token, output row), each dot product in the reference's
// exact FP32 order, so the results are bit-identical to the crate's:
//   LANES = 0: sum += x[i] * w[i] for increasing i (linear, src/lib.rs:63-69;
//              linear_int8, src/quantization.rs:200-212, with w[i] =
//              f32(q[i]) * scale rounded first);
//   LANES = 1: four lanes sums[i % 4] += x[i] * w[i] over the first
//              in - in % 4 elements, then ((s0 + s1) + s2) + s3, then the
//              tail added in order (dot_lanes4, src/kernels.rs:31-46;
//              linear_int8_lanes4, src/quantization.rs:246-276).
// A CTA owns 128 consecutive rows of one token; 32-column tiles of those
// rows and of x are staged in shared memory by coalesced loads (row stride
// 33 floats: no bank conflicts when each thread walks its own row).
// Every operation is an explicitly rounded FP32 multiply or add.
constexpr int kLinRows = 128, kLinCols = 32;

template <int KIND>  // 0 f32, 1 bf16, 2 int8 (groupwise)
__device__ __forceinline__ float lin_weight(const void *w, const float *scales, size_t o, size_t i, size_t in,
                                            size_t group, size_t gpr) {
    if (KIND == 0) return ((const float *)w)[o * in + i];
    if (KIND == 1) return bf16_to_f32(((const uint16_t *)w)[o * in + i]);
    return __fmul_rn((float)((const int8_t *)w)[o * in + i], scales[o * gpr + i / group]);
}

template <int KIND, int LANES>
__global__ void __launch_bounds__(kLinRows) linear_kernel(const float *__restrict__ x, const void *__restrict__ w,
                                                          const float *__restrict__ scales, float *__restrict__ y,
                                                          size_t tokens, size_t in, size_t out, size_t group) {
    __shared__ float ws[kLinRows][kLinCols + 1];
    __shared__ float xs[kLinCols];
    const size_t o0 = (size_t)blockIdx.x * kLinRows;
    const int tid = threadIdx.x;
    const size_t o = o0 + tid;
    const size_t gpr = KIND == 2 ? (in + group - 1) / group : 1;
    const size_t bulk = LANES ? in - in % 4 : in;
  for (size_t t = blockIdx.y; t < tokens; t += gridDim.y) {
    const float *xr = x + t * in;
    float sum = 0.0f, s4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (size_t i0 = 0; i0 < bulk; i0 += kLinCols) {
        const int n = (int)(bulk - i0 < (size_t)kLinCols ? bulk - i0 : (size_t)kLinCols);
        __syncthreads();
        // Rows [o0, o0 + 128) x columns [i0, i0 + n): element e = r * 32 + c.
        for (int e = tid; e < kLinRows * kLinCols; e += kLinRows) {
            const int r = e / kLinCols, c = e % kLinCols;
            if (o0 + r < out && c < n) ws[r][c] = lin_weight<KIND>(w, scales, o0 + r, i0 + c, in, group, gpr);
        }
        if (tid < n) xs[tid] = xr[i0 + tid];
        __syncthreads();
        if (o < out) {
            if (LANES) {
                // i0 is a multiple of 4, so lane k of this tile is lane k of the row.
                for (int c = 0; c < n; ++c) s4[c & 3] = __fadd_rn(s4[c & 3], __fmul_rn(xs[c], ws[tid][c]));
            } else {
                for (int c = 0; c < n; ++c) sum = __fadd_rn(sum, __fmul_rn(xs[c], ws[tid][c]));
            }
        }
    }
    if (o < out) {
        if (LANES) {
            sum = __fadd_rn(__fadd_rn(__fadd_rn(s4[0], s4[1]), s4[2]), s4[3]);
            for (size_t i = bulk; i < in; ++i)
                sum = __fadd_rn(sum, __fmul_rn(xr[i], lin_weight<KIND>(w, scales, o, i, in, group, gpr)));
        }
        y[t * out + o] = sum;
    }
  }
}

static uint32_t validate_linear(size_t xl, size_t wl, size_t yl, size_t t, size_t in, size_t out) {
    clear_detail();
    if (t == 0 || in == 0 || out == 0) return QB_ZERO_DIMENSION;
    size_t xn, wn, yn;
    if (mul_ovf(t, in, &xn) || mul_ovf(out, in, &wn) || mul_ovf(t, out, &yn))
        return QB_DIMENSION_OVERFLOW;
    const size_t e[3] = {xn, wn, yn}, a[3] = {xl, wl, yl};
    for (int i = 0; i < 3; ++i)
        if (e[i] != a[i]) {
            set_detail(i, e[i], a[i]);
            return QB_INVALID_LENGTH;
        }
    return QB_OK;
}

template <int KIND, int LANES = 0>
static uint32_t launch_linear(const float *x, const void *w, const float *scales, float *y,
                              size_t t, size_t in, size_t out, size_t group, void *stream) {
    const size_t bx = (out + kLinRows - 1) / kLinRows;
    if (bx > 0x7fffffffu) return QB_DIMENSION_OVERFLOW;
    const dim3 grid((unsigned)bx, (unsigned)(t < 65535 ? t : 65535));
    linear_kernel<KIND, LANES><<<grid, kLinRows, 0, (cudaStream_t)stream>>>(x, w, scales, y, t, in, out, group);
    QB_CUDA(cudaGetLastError());
    return QB_OK;
}

// ------------------------------------------------------------ scans ----

// Lowest index of a non-finite element (all-ones when none).
__global__ void nonfinite_scan(const float *__restrict__ v, size_t n,
                               unsigned long long *__restrict__ first) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        if (!isfinite(v[i])) atomicMin(first, (unsigned long long)i);
}

static unsigned scan_blocks(size_t n) {
    size_t b = (n + 255) / 256;
    return (unsigned)(b > 4096 ? 4096 : (b == 0 ? 1 : b));
}

// Runs the scan on up to two buffers; *index = first offending index and
// *which = 0/1, or returns QB_OK with which = -1 when all are finite.
static uint32_t find_nonfinite(const float *a, size_t na, const float *b, size_t nb,
                               cudaStream_t s, int *which, size_t *index) {
    void *p;
    uint32_t st = scratch_get(64, &p);
    if (st) return st;
    unsigned long long *flags = (unsigned long long *)p;
    QB_CUDA(cudaMemsetAsync(flags, 0xff, 16, s));
    if (na) nonfinite_scan<<<scan_blocks(na), 256, 0, s>>>(a, na, flags);
    if (nb) nonfinite_scan<<<scan_blocks(nb), 256, 0, s>>>(b, nb, flags + 1);
    unsigned long long h[2];
    QB_CUDA(cudaMemcpyAsync(h, flags, 16, cudaMemcpyDeviceToHost, s));
    QB_CUDA(cudaStreamSynchronize(s));
    *which = -1;
    if (h[0] != ~0ull) { *which = 0; *index = (size_t)h[0]; }
    else if (h[1] != ~0ull) { *which = 1; *index = (size_t)h[1]; }
    return QB_OK;
}

// ----------------------------------------------------------- quantize ----

__device__ __forceinline__ float block_max_abs(const float *__restrict__ v, size_t n, float *red) {
    float m = 0.0f;
    for (size_t i = threadIdx.x; i < n; i += blockDim.x) m = rust_max(m, fabsf(v[i]));
#pragma unroll
    for (int off = 16; off; off >>= 1) m = rust_max(m, __shfl_xor_sync(0xffffffffu, m, off));
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[warp] = m;
    __syncthreads();
    if (warp == 0) {
        m = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0f;
#pragma unroll
        for (int off = 16; off; off >>= 1) m = rust_max(m, __shfl_xor_sync(0xffffffffu, m, off));
        if (lane == 0) red[0] = m;
    }
    __syncthreads();
    return red[0];
}

// Pass 1: per group, flag a scale that underflows to zero (weights are
// already known finite).  max is exact in any order, so the scale is the
// reference's bit for bit.
__global__ void quant_check_kernel(const float *__restrict__ w, size_t in, size_t group,
                                   unsigned long long *__restrict__ bad) {
    __shared__ float red[32];
    size_t o = blockIdx.x;
    size_t gpr = (in + group - 1) / group;
    for (size_t g = 0; g < gpr; ++g) {
        size_t start = g * group, n = (start + group < in ? group : in - start);
        float m = block_max_abs(w + o * in + start, n, red);
        float scale = m == 0.0f ? 1.0f : __fdiv_rn(m, 127.0f);
        if (threadIdx.x == 0 && !(isfinite(scale) && scale > 0.0f)) atomicMin(bad, (unsigned long long)o);
    }
}

// Pass 2: scale = max/127 (zero group -> 1); q = clamp(round(w/scale)),
// round half away from zero (src/quantization.rs:36-40,90-101).
__global__ void quant_kernel(const float *__restrict__ w, size_t in, size_t group,
                             int8_t *__restrict__ values, float *__restrict__ scales) {
    __shared__ float red[32];
    size_t o = blockIdx.x;
    size_t gpr = (in + group - 1) / group;
    for (size_t g = 0; g < gpr; ++g) {
        size_t start = g * group, n = (start + group < in ? group : in - start);
        const float *src = w + o * in + start;
        float m = block_max_abs(src, n, red);
        float scale = m == 0.0f ? 1.0f : __fdiv_rn(m, 127.0f);
        if (threadIdx.x == 0) scales[o * gpr + g] = scale;
        for (size_t i = threadIdx.x; i < n; i += blockDim.x) {
            float r = roundf(__fdiv_rn(src[i], scale));
            r = fminf(fmaxf(r, -127.0f), 127.0f);
            values[o * in + start + i] = (int8_t)r;
        }
    }
}

__global__ void dequant_kernel(const int8_t *__restrict__ q, const float *__restrict__ s,
                               size_t out, size_t in, size_t group, float *__restrict__ y) {
    size_t gpr = (in + group - 1) / group;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < out * in;
         i += (size_t)gridDim.x * blockDim.x) {
        size_t o = i / in, c = i % in;
        y[i] = __fmul_rn((float)q[i], s[o * gpr + c / group]);
    }
}

// ------------------------------------------------------- elementwise ----

__global__ void embedding_kernel(const uint32_t *__restrict__ ids, size_t count,
                                 const float *__restrict__ table, size_t width,
                                 float *__restrict__ y) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < count * width;
         i += (size_t)gridDim.x * blockDim.x) {
        size_t p = i / width, c = i % width;
        y[i] = table[(size_t)ids[p] * width + c];
    }
}

__global__ void residual_kernel(const float *__restrict__ x, const float *__restrict__ r,
                                float *__restrict__ y, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        y[i] = __fadd_rn(x[i], r[i]);
}

// Scaled RMSNorm of one row per block (src/ops.rs:137-149): the row scale is
// an exact max; the sum of squares is a fixed-order tree.
__global__ void rmsnorm_kernel(const float *__restrict__ x, const float *__restrict__ g,
                               float *__restrict__ y, size_t width, float eps) {
    __shared__ float red[32];
    const float *row = x + (size_t)blockIdx.x * width;
    float *out = y + (size_t)blockIdx.x * width;
    float se = sqrtf(eps);
    float m = se;
    for (size_t i = threadIdx.x; i < width; i += blockDim.x) m = rust_max(m, fabsf(row[i]));
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
#pragma unroll
    for (int off = 16; off; off >>= 1) m = rust_max(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = red[0];
    for (int i = 1; i < nw; ++i) m = rust_max(m, red[i]);
    __syncthreads();
    float ss = 0.0f;
    for (size_t i = threadIdx.x; i < width; i += blockDim.x) {
        float v = __fdiv_rn(row[i], m);
        ss = __fadd_rn(ss, __fmul_rn(v, v));
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    ss = 0.0f;
    for (int i = 0; i < nw; ++i) ss = __fadd_rn(ss, red[i]);
    float seps = __fdiv_rn(se, m);
    float den = sqrtf(__fadd_rn(__fdiv_rn(ss, (float)width), __fmul_rn(seps, seps)));
    for (size_t i = threadIdx.x; i < width; i += blockDim.x)
        out[i] = __fmul_rn(__fdiv_rn(__fdiv_rn(row[i], m), den), g[i]);
}

__device__ __forceinline__ float silu1(float v) {
    if (v >= 0.0f) return __fdiv_rn(v, __fadd_rn(1.0f, expf(-v)));
    float e = expf(v);
    return __fdiv_rn(__fmul_rn(v, e), __fadd_rn(1.0f, e));
}

__global__ void silu_kernel(const float *__restrict__ x, float *__restrict__ y, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        y[i] = silu1(x[i]);
}

// Admission scan for softmax: per row, first non-finite allowed entry and
// whether any entry is allowed.
__global__ void softmax_scan(const float *__restrict__ lg, const uint8_t *__restrict__ mask,
                             size_t rows, size_t width, unsigned long long *__restrict__ flags) {
    size_t r = blockIdx.x;
    if (r >= rows) return;
    __shared__ int any;
    if (threadIdx.x == 0) any = 0;
    __syncthreads();
    for (size_t i = threadIdx.x; i < width; i += blockDim.x) {
        size_t k = r * width + i;
        if (!mask || mask[k]) {
            any = 1;
            if (!isfinite(lg[k])) atomicMin(&flags[0], (unsigned long long)k);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0 && !any) atomicMin(&flags[1], (unsigned long long)r);
}

__global__ void softmax_kernel(const float *__restrict__ lg, const uint8_t *__restrict__ mask,
                               float *__restrict__ y, size_t width) {
    __shared__ float red[32];
    size_t r = blockIdx.x;
    const float *row = lg + r * width;
    const uint8_t *mr = mask ? mask + r * width : nullptr;
    float *out = y + r * width;
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    float m = -INFINITY;
    for (size_t i = threadIdx.x; i < width; i += blockDim.x)
        if (!mr || mr[i]) m = rust_max(m, row[i]);
#pragma unroll
    for (int off = 16; off; off >>= 1) m = rust_max(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = red[0];
    for (int i = 1; i < nw; ++i) m = rust_max(m, red[i]);
    __syncthreads();
    float s = 0.0f;
    for (size_t i = threadIdx.x; i < width; i += blockDim.x) {
        float e = (!mr || mr[i]) ? expf(__fsub_rn(row[i], m)) : 0.0f;
        out[i] = e;
        s = __fadd_rn(s, e);
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    s = 0.0f;
    for (int i = 0; i < nw; ++i) s = __fadd_rn(s, red[i]);
    for (size_t i = threadIdx.x; i < width; i += blockDim.x) out[i] = __fdiv_rn(out[i], s);
}

// (a, b) -> (a cos - b sin, b cos + a sin) with the host angle table;
// separate roundings, as the reference's f32 expressions.
__global__ void rope_kernel(const float *__restrict__ x, float *__restrict__ y,
                            const float *__restrict__ cs, size_t tokens, size_t heads,
                            size_t hd) {
    size_t half = hd / 2;
    size_t n = tokens * heads * half;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        size_t j = i % half, th = i / half, t = th / heads;
        float c = cs[(t * half + j) * 2], s = cs[(t * half + j) * 2 + 1];
        size_t off = th * hd;
        float a = x[off + j], b = x[off + j + half];
        y[off + j] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
        y[off + j + half] = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
    }
}

static unsigned grid_for(size_t n) {
    size_t b = (n + 255) / 256;
    return (unsigned)(b > 8192 ? 8192 : (b == 0 ? 1 : b));
}

}  // namespace qb

using namespace qb;

extern "C" {

uint32_t qb_abi_version(void) { return QB_ABI_VERSION; }

void qb_last_detail(qb_detail *out) {
    if (out) *out = g_detail;
}

int qb_last_cuda_error(void) { return g_last_cuda; }

const char *qb_status_name(uint32_t s) {
    static const char *names[] = {
        "Ok", "ZeroDimension", "DimensionOverflow", "InvalidLength", "InvalidGroupSize",
        "InvalidShape", "NonFiniteWeight", "UnrepresentableScale", "Allocation", "InvalidToken",
        "InvalidEpsilon", "NonFinite", "AllMasked", "OddHeadDimension", "PositionOverflow",
        "PositionOutOfRange", "InvalidBase", "InvalidAngle", "InvalidCapacity", "ResourceBudget",
        "InvalidOutputLength", "EmptyInput", "NotEmpty", "Full", "InvalidState", "InvalidConfig",
        "InvalidHandle", "InvalidParameters", "NotStarted", "AlreadyStarted", "Cancelled",
        "EmptyLogits", "CudaError", "DeviceTimeout", "ContextLimit", "TraceLimit", "EmptyPrompt",
        "OutputLimit", "InvalidLayerCount", "Unsupported", "Format", "UnsupportedConfig", "MissingTensor",
        "UnexpectedTensor", "InvalidDtype", "Json", "Encoding", "UnsupportedAssets", "EmptyMessages",
        "InvalidToken", "InvalidStream"};
    return s < sizeof(names) / sizeof(names[0]) ? names[s] : "Unknown";
}

uint32_t qb_linear_f32(const float *x, size_t xl, const float *w, size_t wl, float *y, size_t yl,
                       size_t t, size_t in, size_t out, void *stream) {
    uint32_t s = validate_linear(xl, wl, yl, t, in, out);
    if (s) return s;
    return launch_linear<0>(x, w, nullptr, y, t, in, out, 1, stream);
}

uint32_t qb_linear_lanes4_f32(const float *x, size_t xl, const float *w, size_t wl, float *y,
                              size_t yl, size_t t, size_t in, size_t out, void *stream) {
    uint32_t s = validate_linear(xl, wl, yl, t, in, out);
    if (s) return s;
    return launch_linear<0, 1>(x, w, nullptr, y, t, in, out, 1, stream);
}

uint32_t qb_linear_bf16(const float *x, size_t xl, const uint16_t *w, size_t wl, float *y,
                        size_t yl, size_t t, size_t in, size_t out, void *stream) {
    uint32_t s = validate_linear(xl, wl, yl, t, in, out);
    if (s) return s;
    return launch_linear<1>(x, w, nullptr, y, t, in, out, 1, stream);
}

uint32_t qb_quantize_int8(const float *w, size_t wl, size_t out, size_t in, size_t group,
                          int8_t *values, float *scales, void *stream) {
    clear_detail();
    if (!((group >= 1 && group <= 256) || (group == in && in > 0))) return QB_INVALID_GROUP_SIZE;
    if (out == 0 || in == 0) return QB_ZERO_DIMENSION;
    size_t len, sc, sb;
    if (mul_ovf(out, in, &len)) return QB_DIMENSION_OVERFLOW;
    size_t gpr = in / group + (in % group != 0);
    if (mul_ovf(out, gpr, &sc) || mul_ovf(sc, 4, &sb) || sb > SIZE_MAX - len)
        return QB_DIMENSION_OVERFLOW;
    if (wl != len) {
        set_detail(0, len, wl);
        return QB_INVALID_LENGTH;
    }
    if (out > 0x7fffffffu) return QB_DIMENSION_OVERFLOW;
    cudaStream_t st = (cudaStream_t)stream;
    int which;
    size_t idx;
    uint32_t s = find_nonfinite(w, len, nullptr, 0, st, &which, &idx);
    if (s) return s;
    if (which >= 0) {
        set_detail(0, 0, 0, idx);
        return QB_NONFINITE_WEIGHT;
    }
    void *p;
    if ((s = scratch_get(64, &p))) return s;
    unsigned long long *bad = (unsigned long long *)p;
    QB_CUDA(cudaMemsetAsync(bad, 0xff, 8, st));
    quant_check_kernel<<<(unsigned)out, 256, 0, st>>>(w, in, group, bad);
    unsigned long long hb;
    QB_CUDA(cudaMemcpyAsync(&hb, bad, 8, cudaMemcpyDeviceToHost, st));
    QB_CUDA(cudaStreamSynchronize(st));
    if (hb != ~0ull) return QB_UNREPRESENTABLE_SCALE;
    quant_kernel<<<(unsigned)out, 256, 0, st>>>(w, in, group, values, scales);
    QB_CUDA(cudaGetLastError());
    return QB_OK;
}

uint32_t qb_dequantize_int8(const int8_t *values, const float *scales, size_t out, size_t in,
                            size_t group, float *y, size_t yl, void *stream) {
    clear_detail();
    if (out == 0 || in == 0 || group == 0) return QB_ZERO_DIMENSION;
    size_t len;
    if (mul_ovf(out, in, &len)) return QB_DIMENSION_OVERFLOW;
    if (yl != len) {
        set_detail(0, len, yl);
        return QB_INVALID_LENGTH;
    }
    dequant_kernel<<<grid_for(len), 256, 0, (cudaStream_t)stream>>>(values, scales, out, in, group, y);
    QB_CUDA(cudaGetLastError());
    return QB_OK;
}

static uint32_t validate_linear_int8(size_t xl, size_t out, size_t in, size_t group, size_t yl, size_t t) {
    clear_detail();
    if (t == 0) return QB_ZERO_DIMENSION;
    if (out == 0 || in == 0 || group == 0) return QB_ZERO_DIMENSION;
    size_t xn, yn;
    if (mul_ovf(t, in, &xn) || mul_ovf(t, out, &yn)) return QB_DIMENSION_OVERFLOW;
    if (xl != xn) {
        set_detail(0, xn, xl);
        return QB_INVALID_LENGTH;
    }
    if (yl != yn) {
        set_detail(2, yn, yl);
        return QB_INVALID_LENGTH;
    }
    return QB_OK;
}

uint32_t qb_linear_int8(const float *x, size_t xl, const int8_t *values, const float *scales,
                        size_t out, size_t in, size_t group, float *y, size_t yl, size_t t,
                        void *stream) {
    uint32_t s = validate_linear_int8(xl, out, in, group, yl, t);
    if (s) return s;
    return launch_linear<2>(x, values, scales, y, t, in, out, group, stream);
}

uint32_t qb_linear_int8_lanes4(const float *x, size_t xl, const int8_t *values, const float *scales,
                               size_t out, size_t in, size_t group, float *y, size_t yl, size_t t,
                               void *stream) {
    uint32_t s = validate_linear_int8(xl, out, in, group, yl, t);
    if (s) return s;
    return launch_linear<2, 1>(x, values, scales, y, t, in, out, group, stream);
}

uint32_t qb_embedding(const uint32_t *ids, size_t count, const float *table, size_t tl, float *y,
                      size_t yl, size_t vocab, size_t width, void *stream) {
    clear_detail();
    size_t tn, yn;
    if (vocab == 0 || width == 0) return QB_ZERO_DIMENSION;
    if (mul_ovf(vocab, width, &tn)) return QB_DIMENSION_OVERFLOW;
    if (count == 0) return QB_ZERO_DIMENSION;
    if (mul_ovf(count, width, &yn)) return QB_DIMENSION_OVERFLOW;
    if (tl != tn) { set_detail(0, tn, tl); return QB_INVALID_LENGTH; }
    if (yl != yn) { set_detail(1, yn, yl); return QB_INVALID_LENGTH; }
    for (size_t p = 0; p < count; ++p)
        if (ids[p] >= vocab) { set_detail(0, vocab, ids[p], p); return QB_INVALID_TOKEN; }
    void *dev;
    uint32_t s = scratch_get(64 + count * 4, &dev);
    if (s) return s;
    cudaStream_t st = (cudaStream_t)stream;
    uint32_t *dids = (uint32_t *)((char *)dev + 64);
    QB_CUDA(cudaMemcpyAsync(dids, ids, count * 4, cudaMemcpyHostToDevice, st));
    embedding_kernel<<<grid_for(yn), 256, 0, st>>>(dids, count, table, width, y);
    QB_CUDA(cudaGetLastError());
    QB_CUDA(cudaStreamSynchronize(st));  // the host id copy must complete before return
    return QB_OK;
}

uint32_t qb_residual_add(const float *x, size_t xl, const float *r, size_t rl, float *y,
                         size_t yl, void *stream) {
    clear_detail();
    if (xl == 0) return QB_ZERO_DIMENSION;
    if (rl != xl) { set_detail(1, xl, rl); return QB_INVALID_LENGTH; }
    if (yl != xl) { set_detail(2, xl, yl); return QB_INVALID_LENGTH; }
    residual_kernel<<<grid_for(xl), 256, 0, (cudaStream_t)stream>>>(x, r, y, xl);
    QB_CUDA(cudaGetLastError());
    return QB_OK;
}

uint32_t qb_rmsnorm(const float *x, size_t xl, const float *g, size_t gl, float *y, size_t yl,
                    size_t rows, size_t width, float eps, void *stream) {
    clear_detail();
    if (rows == 0 || width == 0) return QB_ZERO_DIMENSION;
    size_t len;
    if (mul_ovf(rows, width, &len)) return QB_DIMENSION_OVERFLOW;
    if (xl != len) { set_detail(0, len, xl); return QB_INVALID_LENGTH; }
    if (gl != width) { set_detail(1, width, gl); return QB_INVALID_LENGTH; }
    if (yl != len) { set_detail(2, len, yl); return QB_INVALID_LENGTH; }
    if (!isfinite(eps) || eps <= 0.0f) return QB_INVALID_EPSILON;
    if (rows > 0x7fffffffu) return QB_DIMENSION_OVERFLOW;
    cudaStream_t st = (cudaStream_t)stream;
    int which;
    size_t idx;
    uint32_t s = find_nonfinite(x, xl, g, gl, st, &which, &idx);
    if (s) return s;
    if (which >= 0) { set_detail((size_t)which, 0, 0, idx); return QB_NONFINITE; }
    rmsnorm_kernel<<<(unsigned)rows, 256, 0, st>>>(x, g, y, width, eps);
    QB_CUDA(cudaGetLastError());
    return QB_OK;
}

uint32_t qb_silu(const float *x, size_t xl, float *y, size_t yl, void *stream) {
    clear_detail();
    if (xl == 0) return QB_ZERO_DIMENSION;
    if (yl != xl) { set_detail(1, xl, yl); return QB_INVALID_LENGTH; }
    cudaStream_t st = (cudaStream_t)stream;
    int which;
    size_t idx;
    uint32_t s = find_nonfinite(x, xl, nullptr, 0, st, &which, &idx);
    if (s) return s;
    if (which >= 0) { set_detail(0, 0, 0, idx); return QB_NONFINITE; }
    silu_kernel<<<grid_for(xl), 256, 0, st>>>(x, y, xl);
    QB_CUDA(cudaGetLastError());
    return QB_OK;
}

uint32_t qb_softmax(const float *lg, size_t ll, const uint8_t *mask, size_t ml, float *y,
                    size_t yl, size_t rows, size_t width, void *stream) {
    clear_detail();
    if (rows == 0 || width == 0) return QB_ZERO_DIMENSION;
    size_t len;
    if (mul_ovf(rows, width, &len)) return QB_DIMENSION_OVERFLOW;
    if (ll != len) { set_detail(0, len, ll); return QB_INVALID_LENGTH; }
    if (yl != len) { set_detail(1, len, yl); return QB_INVALID_LENGTH; }
    if (mask && ml != len) { set_detail(2, len, ml); return QB_INVALID_LENGTH; }
    if (rows > 0x7fffffffu) return QB_DIMENSION_OVERFLOW;
    cudaStream_t st = (cudaStream_t)stream;
    void *p;
    uint32_t s = scratch_get(64, &p);
    if (s) return s;
    unsigned long long *flags = (unsigned long long *)p;
    QB_CUDA(cudaMemsetAsync(flags, 0xff, 16, st));
    softmax_scan<<<(unsigned)rows, 256, 0, st>>>(lg, mask, rows, width, flags);
    unsigned long long h[2];
    QB_CUDA(cudaMemcpyAsync(h, flags, 16, cudaMemcpyDeviceToHost, st));
    QB_CUDA(cudaStreamSynchronize(st));
    // The reference checks row by row: the first offending row decides.
    size_t nf_row = h[0] == ~0ull ? SIZE_MAX : (size_t)(h[0] / width);
    size_t am_row = h[1] == ~0ull ? SIZE_MAX : (size_t)h[1];
    if (nf_row != SIZE_MAX && nf_row <= am_row) { set_detail(0, 0, 0, (size_t)h[0]); return QB_NONFINITE; }
    if (am_row != SIZE_MAX) { set_detail(0, 0, 0, am_row); return QB_ALL_MASKED; }
    softmax_kernel<<<(unsigned)rows, 256, 0, st>>>(lg, mask, y, width);
    QB_CUDA(cudaGetLastError());
    return QB_OK;
}

uint32_t qb_rope(const float *x, size_t xl, float *y, size_t yl, size_t tokens, size_t heads,
                 size_t hd, size_t start, float base, void *stream) {
    clear_detail();
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
    size_t half = hd / 2;
    std::vector<float> freq(half);
    for (size_t j = 0; j < half; ++j) {
        freq[j] = powf(base, -((float)(2 * j)) / (float)hd);
        if (!isfinite(freq[j]) || !isfinite((float)last * freq[j])) return QB_INVALID_ANGLE;
    }
    cudaStream_t st = (cudaStream_t)stream;
    int which;
    size_t idx;
    uint32_t s = find_nonfinite(x, xl, nullptr, 0, st, &which, &idx);
    if (s) return s;
    if (which >= 0) { set_detail(0, 0, 0, idx); return QB_NONFINITE; }
    std::vector<float> cs(tokens * half * 2);
    for (size_t t = 0; t < tokens; ++t) {
        float pos = (float)(start + t);
        for (size_t j = 0; j < half; ++j) {
            float a = pos * freq[j];
            cs[(t * half + j) * 2] = cosf(a);
            cs[(t * half + j) * 2 + 1] = sinf(a);
        }
    }
    void *p;
    if ((s = scratch_get(64 + cs.size() * 4, &p))) return s;
    float *dcs = (float *)((char *)p + 64);
    QB_CUDA(cudaMemcpyAsync(dcs, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice, st));
    rope_kernel<<<grid_for(tokens * heads * half), 256, 0, st>>>(x, y, dcs, tokens, heads, hd);
    QB_CUDA(cudaGetLastError());
    QB_CUDA(cudaStreamSynchronize(st));  // the host table must outlive the copy
    return QB_OK;
}

}  // extern "C"
