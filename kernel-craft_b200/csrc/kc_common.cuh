// kc_common.cuh -- shared helpers for the sm_100a quantized-linear library.
//
// Error model: every entry point validates its arguments on the host before
// launching anything.  A failed check or a CUDA/NCCL error is recorded in a
// thread-local slot (kc_get_last_error / kc_get_last_error_string) and, for
// the kc_* API, returned as the int status.  The reference-named launchers
// keep their void signatures and record the same status.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include <cstdio>

#include "../../include/kernel_craft.h"

namespace kc {

// Records a status (and a formatted detail message) for the calling thread.
int set_error(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));

// Records KC_ERR_CUDA if `e` is an error; returns KC_OK or KC_ERR_CUDA.
int check_cuda(cudaError_t e, const char* what);

// Checks the launch status of the last kernel (cudaGetLastError).
inline int check_launch(const char* what) { return check_cuda(cudaGetLastError(), what); }

// Multiprocessor count of the current device (cached per device).
int sm_count();

// Device status words of the translation units with bounded device-side waits
// (KC_DEFINE_STATUS_READER in sm100.cuh): 0 or the first status recorded.
int read_device_status_gemv(bool clear);
int read_device_status_selftest(bool clear);
int read_device_status_gemm_fp8(bool clear);
int read_device_status_gemm_w4a16(bool clear);
int read_device_status_peer(bool clear);

__host__ __device__ inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

inline int ceil_div(long a, long b) { return (int)((a + b - 1) / b); }

}  // namespace kc

// Argument checks used by every launcher.
#define KC_REQUIRE(cond, code, ...)                                      \
    do {                                                                 \
        if (!(cond)) return ::kc::set_error((code), __VA_ARGS__);        \
    } while (0)

#define KC_CUDA_TRY(expr, what)                                          \
    do {                                                                 \
        int _st = ::kc::check_cuda((expr), (what));                      \
        if (_st != KC_OK) return _st;                                    \
    } while (0)

// ---------------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------------

// 128-bit streaming load: read-only path, no L1 allocation, 256-byte L2
// prefetch hint (weights are read exactly once per pass).
__device__ __forceinline__ uint4 kc_ldg_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// 128-bit read-only load that may allocate in L1 (activations, reused).
__device__ __forceinline__ uint4 kc_ldg_keep(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// Predicated 128-bit read-only load: zeros when !pred, no branch.
__device__ __forceinline__ uint4 kc_ldg_keep_if(const void* p, bool pred) {
    uint4 v;
    asm volatile(
        "{\n\t.reg .pred q;\n\t"
        "setp.ne.b32 q, %5, 0;\n\t"
        "mov.b32 %0, 0; mov.b32 %1, 0; mov.b32 %2, 0; mov.b32 %3, 0;\n\t"
        "@q ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];\n\t}"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
        : "l"(p), "r"((int)pred));
    return v;
}

__device__ __forceinline__ float kc_warp_sum(float v) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float kc_warp_max(float v) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
