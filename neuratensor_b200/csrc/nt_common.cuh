// Shared device/host helpers for the NeuraTensor B200 kernels (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <cstdio>

#include "../../include/neuratensor_native.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "neuratensor_b200 kernels are written for sm_100a (B200) only"
#endif

namespace nt {

// ----------------------------------------------------------------------------
// Host-side error reporting (thread-local last error, C-ABI friendly)
// ----------------------------------------------------------------------------
void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);
int check_launch(const char* what);

// Device error word layout: bit flags written by kernels whose bounded waits
// expired.  The host reads it with nt_get_error_flag().
enum : unsigned { ERRF_TIMEOUT_PRODUCER = 1u, ERRF_TIMEOUT_MMA = 2u, ERRF_TIMEOUT_EPILOGUE = 4u,
                  ERRF_BAD_ARG = 8u };
unsigned* device_error_word(int device);

// ----------------------------------------------------------------------------
// Numeric helpers
// ----------------------------------------------------------------------------
__device__ __forceinline__ float bf16_round(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
}

template <int DT> struct Elem;
template <> struct Elem<NT_F32> {
    using T = float;
    static __device__ __forceinline__ float load(const T* p) { return __ldg(p); }
    static __device__ __forceinline__ float to_f(T v) { return v; }
    static __device__ __forceinline__ T from_f(float v) { return v; }
    // Round an op result to the working dtype (identity in fp32).
    static __device__ __forceinline__ float rnd(float v) { return v; }
};
template <> struct Elem<NT_BF16> {
    using T = __nv_bfloat16;
    static __device__ __forceinline__ float load(const T* p) { return __bfloat162float(__ldg(p)); }
    static __device__ __forceinline__ float to_f(T v) { return __bfloat162float(v); }
    static __device__ __forceinline__ T from_f(float v) { return __float2bfloat16_rn(v); }
    static __device__ __forceinline__ float rnd(float v) { return bf16_round(v); }
};

// 2^x on the MUFU pipe (PTX ex2.approx; max relative error ~2^-22).
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

constexpr float kLog2e = 1.4426950408889634f;

// Bounded waits.  Every mbarrier wait in these kernels gives up after this
// much wall time (read from %globaltimer), raises a flag in the device error
// word and lets the kernel finish; no launch here runs for more than a few ms.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// ----------------------------------------------------------------------------
// mbarrier helpers (shared memory, CTA scope).  mbar_wait is bounded: it
// returns false when kWaitLimitNs of wall time pass without the phase
// completing, and the caller raises a flag in the device error word.
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait: false when kWaitLimitNs of wall time passed without the phase completing.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        for (int i = 0; i < 64; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
    }
}
}  // namespace nt
