// Shared device helpers for the sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace cheetah {

// ---- error plumbing (thread-local last error, int status) ----
void set_error(const std::string &message);
const char *last_error();

#define CH_CUDA_TRY(expr)                                                           \
    do {                                                                            \
        cudaError_t err__ = (expr);                                                 \
        if (err__ != cudaSuccess) {                                                 \
            ::cheetah::set_error(std::string(#expr " failed: ") +                   \
                                 cudaGetErrorString(err__));                        \
            return -1;                                                              \
        }                                                                           \
    } while (0)

#define CH_REQUIRE(cond, message)                                                   \
    do {                                                                            \
        if (!(cond)) {                                                              \
            ::cheetah::set_error(message);                                          \
            return -1;                                                              \
        }                                                                           \
    } while (0)

constexpr int kWarp = 32;

// ---- bf16 <-> f32 (exact widening as ops.rs:59-62; RNE narrowing) ----
__device__ __forceinline__ float bf16_lo(uint32_t word) { return __uint_as_float(word << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t word) { return __uint_as_float(word & 0xFFFF0000u); }
__device__ __forceinline__ float bf16_to_f32(uint16_t bits) {
    return __uint_as_float(static_cast<uint32_t>(bits) << 16);
}
__device__ __forceinline__ uint16_t f32_to_bf16_rne(float value) {
    uint32_t bits = __float_as_uint(value);
    if ((bits & 0x7F800000u) == 0x7F800000u && (bits & 0x007FFFFFu)) return 0x7FC0;  // NaN
    bits += 0x7FFFu + ((bits >> 16) & 1u);
    return static_cast<uint16_t>(bits >> 16);
}

// 2^x and 1/x with the hardware approximations (subnormal results flush to
// zero), for values that are rounded to bf16 right after.
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float fast_rcp(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// ---- streaming loads (weights are read exactly once per step) ----
__device__ __forceinline__ uint4 ldg_stream(const uint4 *ptr) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(ptr));
    return v;
}

// ---- programmatic dependent launch (PDL) ----
// Every kernel calls pdl_wait() before touching any buffer an earlier kernel
// writes, and exits only after it, so completion stays transitive along the
// stream. pdl_launch_dependents() lets the next kernel's CTAs start staging
// their (input-independent) weights while this one finishes.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- reductions ----
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    return v;
}

// Total-order key of an f32 (Rust `f32::total_cmp`): monotone as u32.
__device__ __forceinline__ uint32_t total_order_key(float value) {
    uint32_t bits = __float_as_uint(value);
    return (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
}

}  // namespace cheetah
