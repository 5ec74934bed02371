// Shared device/host helpers for the Sana denoiser CUDA library (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>

namespace sana {

// Status codes of the C ABI (include/sana_cuda.h).
enum Status : int {
    kOk = 0,
    kInvalid = 1,   // shape / argument error (std::invalid_argument in the C++ shim)
    kCuda = 2,      // CUDA runtime error
    kTimeout = 3,   // a bounded device-side wait gave up (kernel returned early)
    kState = 4,     // call order / missing weights
    kNoMem = 5,
};

struct InvalidArg : std::invalid_argument {
    using std::invalid_argument::invalid_argument;
};
struct CudaError : std::runtime_error {
    using std::runtime_error::runtime_error;
};
struct TimeoutError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

#define SANA_CUDA(expr)                                                                       \
    do {                                                                                      \
        cudaError_t e_ = (expr);                                                              \
        if (e_ != cudaSuccess) {                                                              \
            throw ::sana::CudaError(std::string(#expr) + ": " + cudaGetErrorString(e_));      \
        }                                                                                     \
    } while (0)

#define SANA_REQUIRE(cond, msg)                                                               \
    do {                                                                                      \
        if (!(cond)) throw ::sana::InvalidArg(msg);                                           \
    } while (0)

using bf16 = __nv_bfloat16;

// Activation element type of a precision mode: bf16 (fast path) or fp32 (check mode).
template <class T> struct Act;
template <> struct Act<float> {
    static __device__ __forceinline__ float load(const float* p) { return *p; }
    static __device__ __forceinline__ void store(float* p, float v) { *p = v; }
};
template <> struct Act<bf16> {
    static __device__ __forceinline__ float load(const bf16* p) { return __bfloat162float(*p); }
    static __device__ __forceinline__ void store(bf16* p, float v) { *p = __float2bfloat16_rn(v); }
};

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(bf16 v) { return __bfloat162float(v); }
template <class T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ bf16 from_f<bf16>(float v) { return __float2bfloat16_rn(v); }

// Elementwise activations. SiLU is x / (1 + e^-x) as tensor.cpp:551-555; GELU is the tanh
// form of transformer_ops.cpp:15-18. Both call CUDA's own expf / tanhf.
__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }

// Packed fp32 pairs (sm_100 f32x2): a 64-bit register holds two fp32 values and one
// instruction does the arithmetic of both.
__device__ __forceinline__ uint64_t f2_from_bf2(uint32_t u) {  // bf16 pair -> fp32 pair (exact)
    uint64_t d;
    asm("{\n\t.reg .b32 lo, hi;\n\tshl.b32 lo, %1, 16;\n\tand.b32 hi, %1, 0xffff0000;\n\tmov.b64 %0, {lo, hi};\n\t}"
        : "=l"(d)
        : "r"(u));
    return d;
}
__device__ __forceinline__ uint64_t f2_make(float lo, float hi) {
    uint64_t d;
    asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
    return d;
}
__device__ __forceinline__ float2 f2_split(uint64_t u) {
    float lo, hi;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(u));
    return make_float2(lo, hi);
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
// SiLU of a pair for the tensor-core epilogues: x / (1 + e^-x) with e^-x = 2^(-x log2 e) from
// the hardware base-2 exponential and the quotient from the hardware reciprocal (ex2.approx,
// rcp.approx: a few ulp each, within 1.5e-5 of the exact value over the inputs the epilogue
// sees), the scaling, sum and product pairwise. Two special-function operations per element
// measured faster in the FF-inverted projection's epilogue than one exponential plus a
// reciprocal refined by Newton steps on the FMA pipe (0.317 vs 0.343 ms per launch at config 2).
// The exponent is capped at 126, where 1 + 2^t stays finite and x / (1 + 2^t) is below
// 1e-36 either way.
__device__ __forceinline__ float ex2_approx(float t) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(t));
    return r;
}
__device__ __forceinline__ float rcp_approx(float y) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(y));
    return r;
}
__device__ __forceinline__ uint64_t silu2(uint64_t g) {
    constexpr float kLog2e = 1.4426950408889634f;  // log2(e)
    const float2 t = f2_split(mul2(g, f2_make(-kLog2e, -kLog2e)));
    const uint64_t d = add2(f2_make(ex2_approx(fminf(t.x, 126.0f)), ex2_approx(fminf(t.y, 126.0f))),
                            f2_make(1.0f, 1.0f));
    const float2 ds = f2_split(d);
    return mul2(g, f2_make(rcp_approx(ds.x), rcp_approx(ds.y)));
}

__device__ __forceinline__ float gelu_tanh(float x) {
    const float alpha = sqrtf(2.0f / 3.14159265358979323846f);  // as transformer_ops.cpp:16
    return 0.5f * x * (1.0f + tanhf(alpha * (x + 0.044715f * x * x * x)));
}

// ---------------------------------------------------------------------------------------
// Bounded waits. Every spin in this library has a time limit: on expiry the waiter
// records `code` in the context's device error word and returns false, and the kernel
// unwinds. Waiters also give up early once any thread has recorded an error.
//
// A handle's device error word is 16 bytes: int [0] is the error code (0 = none), and the
// 64-bit value at byte 8 is the handle's wait limit in nanoseconds (sana_cuda_set_wait_limit;
// kWaitLimitNs by default). Waiters read the limit once they have spun a while.
// ---------------------------------------------------------------------------------------
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s
constexpr int kErrWordBytes = 16;

__device__ __forceinline__ uint64_t wait_limit_ns(const int* err) {
    return *reinterpret_cast<const volatile unsigned long long*>(err + 2);
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* err, int code) {
    for (int i = 0; i < 64; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
    }
    const uint64_t t0 = global_ns();
    const uint64_t limit = wait_limit_ns(err);
    for (uint32_t n = 0;; ++n) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((n & 255u) == 0) {
            if (*(volatile int*)err != 0) return false;
            if (global_ns() - t0 > limit) {
                atomicCAS(err, 0, code);
                return false;
            }
        }
    }
}

// Bounded wait that records nothing: used while unwinding after an error has already
// been recorded (draining copies or MMAs this thread issued).
__device__ __forceinline__ bool mbar_wait_quiet(uint32_t bar, uint32_t parity) {
    const uint64_t t0 = global_ns();
    for (uint32_t n = 0;; ++n) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((n & 255u) == 0 && global_ns() - t0 > kWaitLimitNs) return false;
    }
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

inline int ceil_div(long long a, long long b) { return static_cast<int>((a + b - 1) / b); }

// Kernel attributes (cudaFuncSetAttribute) belong to a device's context, so a launch site sets
// them once per device: `static PerDeviceOnce attr; if (attr.pending()) { set...; attr.mark(); }`.
struct PerDeviceOnce {
    bool done[64] = {};
    static int current() {
        int d = 0;
        return cudaGetDevice(&d) == cudaSuccess && d >= 0 && d < 64 ? d : -1;
    }
    bool pending() const {
        const int d = current();
        return d < 0 || !done[d];
    }
    void mark() {
        const int d = current();
        if (d >= 0) done[d] = true;
    }
};

}  // namespace sana
