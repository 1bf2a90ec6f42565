// common.cuh -- shared device helpers for the sm_100a kernels of libopure_cuda.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "opure_cuda.h"

namespace opure {

// ---------------------------------------------------------------------------
// Device status word. Kernels never trap: a kernel that finds an index out of
// range or gives up a bounded wait records the first failure here and returns.
// opure_last_error() reads and clears it.
struct DeviceStatus {
    uint32_t code;     // opure_status of the first failure, 0 = none
    uint32_t where;    // kernel-specific site id
    uint32_t detail;   // e.g. the offending index
    uint32_t pad;
};

__device__ __forceinline__ void report(DeviceStatus *st, uint32_t code, uint32_t where,
                                       uint32_t detail) {
    if (st && atomicCAS(&st->code, 0u, code) == 0u) {
        st->where = where;
        st->detail = detail;
    }
}

// ---------------------------------------------------------------------------
// Chained tensor-core operand: vector `vec` of a [2][npad][len] fp16 buffer holds
// hi = fp16(v) in row vec and lo = fp16((v - hi) * 2^11) in row npad + vec, so that
// W.v = W.hi + 2^-11 W.lo keeps ~22 significant bits with fp16 x fp16 products (the
// consumer accumulates the two halves separately). A value outside fp16's range is
// reported at `site` and stored as 0.
__device__ __forceinline__ void store_packed(__half *pk, uint32_t npad, uint32_t len, uint32_t vec, uint32_t i,
                                             float v, DeviceStatus *st, uint32_t site) {
    if (!(fabsf(v) < 65504.f)) {
        report(st, OPURE_ERR_DEVICE_BOUNDS, site, i);
        v = 0.f;
    }
    const __half hi = __float2half_rn(v);
    pk[size_t(vec) * len + i] = hi;
    pk[size_t(npad + vec) * len + i] = __float2half_rn((v - __half2float(hi)) * 2048.f);
}

// ---------------------------------------------------------------------------
// Memory access helpers.

// 16-byte load from L2 (coherent across SMs within one kernel): for data other CTAs of the
// same (persistent) kernel write, which the non-coherent path may serve stale.
__device__ __forceinline__ uint4 ldcg_v4(const void *p) {
    uint4 r;
    asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// L2 policy for weights: every byte is read once per step, so weights are marked
// evict-first and the KV cache and activations (reused every step) stay resident in L2.
__device__ __forceinline__ uint64_t l2_evict_first() {
    uint64_t pol;
    asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// 16-byte streaming load that bypasses L1 allocation: weights are read once per step.
__device__ __forceinline__ uint4 ldg_stream(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// Shared-memory loads by explicit shared-window address. Pointers that reach a loop
// through an array or a struct can lose their address space in the compiler's view, which
// then emits slower generic loads; these always compile to ld.shared.
__device__ __forceinline__ uint32_t shared_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint4 lds128(const void *p) {
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "r"(shared_addr(p)));
    return r;
}
__device__ __forceinline__ float4 lds_f4(const float *p) {
    float4 r;
    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
                 : "r"(shared_addr(p)));
    return r;
}
__device__ __forceinline__ float lds_f32(const float *p) {
    float r;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(r) : "r"(shared_addr(p)));
    return r;
}
__device__ __forceinline__ float lds_h(const __half *p) {
    unsigned short r;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(r) : "r"(shared_addr(p)));
    return __half2float(__ushort_as_half(r));
}

__device__ __forceinline__ float lds_s8(const void *p) {
    int r;
    asm volatile("ld.shared.s8 %0, [%1];" : "=r"(r) : "r"(shared_addr(p)));
    return float(r);
}

__device__ __forceinline__ float2 h2f2(uint32_t u) {
    __half2 h = *reinterpret_cast<__half2 *>(&u);
    return __half22float2(h);
}

// 8 fp16 -> 8 fp32.
__device__ __forceinline__ void unpack8(const uint4 &w, float *f) {
    float2 a = h2f2(w.x), b = h2f2(w.y), c = h2f2(w.z), d = h2f2(w.w);
    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
    f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}

// 16 int8 (one 16-byte load) -> 16 fp32, little-endian byte order (element 4w+k in
// byte k of word w, as the reference packs GEMV_Quant weights).
__device__ __forceinline__ void unpack16_i8(const uint4 &w, float *f) {
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int32_t v = int32_t(words[j]);
        f[4 * j + 0] = float((v << 24) >> 24);
        f[4 * j + 1] = float((v << 16) >> 24);
        f[4 * j + 2] = float((v << 8) >> 24);
        f[4 * j + 3] = float(v >> 24);
    }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch (PDL). A kernel launched with the programmatic
// stream-serialization attribute may start while its predecessor is still running;
// it must call grid_dependency_wait() before touching anything the predecessor
// writes. Work that only reads weights can run before the wait.
__device__ __forceinline__ void grid_dependency_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_dependents_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Argmax keys: (orderable value << 32) | (0xffffffff - index). An unsigned max over
// keys picks the largest value and, among equal values, the lowest index. NaN maps
// to key 0 so it never wins; 0 is also the "empty" key the caller zeroes to.
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
    if (v != v) return 0ull;
    uint32_t b = __float_as_uint(v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return (static_cast<unsigned long long>(b) << 32) | (0xffffffffu - idx);
}
__host__ __device__ __forceinline__ uint32_t argmax_key_index(unsigned long long k) {
    return 0xffffffffu - static_cast<uint32_t>(k & 0xffffffffull);
}
__device__ __forceinline__ float argmax_key_value(unsigned long long k) {
    if (k == 0ull) return -__int_as_float(0x7f800000);  // empty / all-NaN: -inf
    uint32_t b = static_cast<uint32_t>(k >> 32);
    b = (b & 0x80000000u) ? (b & 0x7fffffffu) : ~b;
    return __uint_as_float(b);
}

// ---------------------------------------------------------------------------
// Residual stream in fixed point. Partial sums produced by many CTAs (o_proj and
// down_proj split over their contracted dimension) are added with 64-bit integer
// atomics, which are associative, so the result does not depend on arrival order.
constexpr double kFixScale = 4294967296.0;        // 2^32
constexpr double kFixInv = 1.0 / 4294967296.0;
__device__ __forceinline__ long long to_fix(float v) {
    return __double2ll_rn(double(v) * kFixScale);
}

// Sliding-window KV cache (opure_kv_layout.ring): the table entry of logical page lp, and
// the first position a query at position p attends to.
__device__ __forceinline__ uint32_t ring_slot(uint32_t lp, uint32_t ring) { return ring ? lp % ring : lp; }
__device__ __forceinline__ uint32_t window_begin(int32_t p, uint32_t page_size, uint32_t ring) {
    if (!ring || p < 0) return 0u;
    const uint32_t lp = uint32_t(p) / page_size;
    return lp + 1 > ring ? (lp + 1 - ring) * page_size : 0u;
}

}  // namespace opure

// Host-side error propagation inside the ABI implementation.
#define OPURE_CUDA_TRY(expr)                                   \
    do {                                                       \
        cudaError_t _e = (expr);                               \
        if (_e != cudaSuccess) return opure::cuda_status(_e);  \
    } while (0)

namespace opure {
inline opure_status cuda_status(cudaError_t e) {
    if (e == cudaErrorMemoryAllocation) return OPURE_ERR_OUT_OF_MEMORY;
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) return OPURE_ERR_NO_DEVICE;
    return OPURE_ERR_CUDA;
}
}  // namespace opure
