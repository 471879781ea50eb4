// Shared device/host helpers for the sm_100a Qwen2 token-loop library.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

#include "../../include/qwen_b200.h"

namespace qb {

// ---------------------------------------------------------------- host ----

// Thread-local error detail (qb_last_detail) and last CUDA error.
void set_detail(size_t buffer, size_t expected, size_t actual, size_t index = 0);
void clear_detail();
uint32_t cuda_status(cudaError_t e);  // records e, returns QB_OK or QB_CUDA_ERROR

#define QB_CUDA(expr)                                  \
    do {                                               \
        cudaError_t _e = (expr);                       \
        if (_e != cudaSuccess) return ::qb::cuda_status(_e); \
    } while (0)

inline bool mul_ovf(size_t a, size_t b, size_t *out) {
    if (a != 0 && b > SIZE_MAX / a) return true;
    *out = a * b;
    return false;
}

// Host-side scratch reused by the elementwise ops: a small device buffer per
// device for error flags and per-call tables (grown on demand).
struct DeviceScratch {
    int device = -1;
    void *ptr = nullptr;
    size_t bytes = 0;
};
uint32_t scratch_get(size_t bytes, void **out);

// ---------------------------------------------------------------- device ----

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
__device__ __forceinline__ float bf16_to_f32(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

// Round-to-nearest-even FP32 -> BF16 bits.
__device__ __forceinline__ uint16_t f32_to_bf16_rne(float x) {
    uint32_t u = __float_as_uint(x);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return (uint16_t)((u | 0x00400000u) >> 16);
    uint32_t lsb = (u >> 16) & 1u;
    return (uint16_t)((u + 0x7fffu + lsb) >> 16);
}

// Rust's f32::max: a NaN operand yields the other operand.
__device__ __forceinline__ float rust_max(float a, float b) { return fmaxf(a, b); }

__device__ __forceinline__ uint32_t ld_acquire_u32(const unsigned *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_add_u32(unsigned *p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Relaxed GPU-scope 64-bit load for polling a word another CTA writes (a
// volatile asm, so repeated polls are never merged or hoisted).
__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p));
    return v;
}

// Relaxed GPU-scope loads and store of words that other CTAs of the same
// grid write or read while this one runs (volatile asm: polls are never
// merged or hoisted).  Each 32-bit word is single-copy atomic.
__device__ __forceinline__ uint32_t ld_relaxed_b32(const void *p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ uint2 ld_relaxed_v2(const void *p) {
    uint2 v;
    asm volatile("ld.relaxed.gpu.global.v2.b32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}
__device__ __forceinline__ uint4 ld_relaxed_v4(const void *p) {
    uint4 v;
    asm volatile("ld.relaxed.gpu.global.v4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ void st_relaxed_b32(void *p, uint32_t v) {
    asm volatile("st.relaxed.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Streaming 16-byte load that bypasses L1 allocation (weights are read once).
__device__ __forceinline__ uint4 ld_stream_u4(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// Bulk prefetch of [p, p+bytes) into L2 (p and bytes multiples of 16).
__device__ __forceinline__ void prefetch_l2_bulk(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// ---- shared-memory mbarriers and 1-D bulk copies (TMA, no tensor map) ----

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Makes barrier initialization visible to the async (bulk-copy) proxy.
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's (and, after a CTA barrier, the CTA's) generic-proxy
// shared-memory accesses before later async-proxy writes.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// `count` arrivals at once.
__device__ __forceinline__ void mbar_arrive_cnt(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// One bounded probe of phase `parity`; true once that phase has completed.
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// As mbar_try_wait, but the thread may be suspended in hardware for up to
// `suspend_ns` while the phase is incomplete (no issue slots are spent
// polling).
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t *bar, uint32_t parity, uint32_t suspend_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(suspend_ns)
        : "memory");
    return ok != 0;
}

// Global -> shared bulk copy of `bytes` (16-byte aligned addresses, size a
// multiple of 16) completing on `bar` via complete_tx.
__device__ __forceinline__ void bulk_copy_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// Per-thread asynchronous global -> shared copies of 4 or 16 bytes
// (cp.async): issued, then committed as a group; cp_async_wait_all waits for
// every group this thread committed.  The data is visible to other threads
// after their own wait and a CTA barrier.
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Exact int8 -> FP32 for weights stored biased as u = q + 128 (1..255):
// the byte is placed in the mantissa of 2^23 and 2^23 + 128 subtracted.
__device__ __forceinline__ float u8b_to_f32(uint32_t word, int byte) {
    uint32_t sel = 0x7650u | (uint32_t)byte;  // [b, 0, 0, 0x4B] little-endian
    uint32_t f = __byte_perm(word, 0x4B000000u, sel);
    return __uint_as_float(f) - 8388736.0f;   // 2^23 + 128
}

}  // namespace qb
