// kc_status.cpp -- thread-local status slot, device queries, out-of-scope stubs.
#include <cuda_runtime.h>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "kc_common.cuh"

namespace {
thread_local int  t_last_error = KC_OK;
thread_local char t_last_msg[512] = "";
}  // namespace

namespace kc {

int set_error(int code, const char* fmt, ...) {
    t_last_error = code;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_last_msg, sizeof(t_last_msg), fmt, ap);
    va_end(ap);
    return code;
}

int check_cuda(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return KC_OK;
    return set_error(KC_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int sm_count() {
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

}  // namespace kc

extern "C" {

int kc_get_last_error(void) {
    int e = t_last_error;
    t_last_error = KC_OK;
    return e;
}

const char* kc_get_last_error_string(void) { return t_last_msg; }

const char* kc_version(void) { return "kernel-craft-b200 0.1 (sm_100a)"; }

int kc_get_device_status(void) {
    // Synchronizes the device so every launched kernel has finished updating
    // its unit's status word, then reads and clears all of them.
    if (cudaDeviceSynchronize() != cudaSuccess)
        return kc::set_error(KC_ERR_CUDA, "kc_get_device_status: device synchronize failed");
    int st = KC_OK;
    for (int v : {kc::read_device_status_gemv(true), kc::read_device_status_selftest(true),
                  kc::read_device_status_gemm_fp8(true), kc::read_device_status_gemm_w4a16(true),
                  kc::read_device_status_peer(true)})
        if (st == KC_OK && v != KC_OK) st = v;
    if (st != KC_OK) kc::set_error(st, "a device-side wait gave up (status %d)", st);
    return st;
}

// --- launchers outside this library's scope --------------------------------
// src/python/kernel_craft_torch_ops.py:105-168 resolves the attention and
// speculative-decoding symbols when it loads libkernels.so, and the pybind11
// module src/python/pybind_transformer.cpp:36-122 links those plus the
// prefix-length, Mamba and RMSNorm launchers; exporting all of them lets the
// unmodified bridge and module load.  Each records KC_ERR_UNSUPPORTED and
// launches nothing.
static void kc_out_of_scope(const char* name) {
    static std::once_flag once;
    std::call_once(once, [] {
        fprintf(stderr, "[kernel-craft-b200] attention, speculative-decoding, Mamba and RMSNorm "
                        "launchers are not part of this library; the call launched nothing\n");
    });
    kc::set_error(KC_ERR_UNSUPPORTED, "%s is outside the quantized-linear library", name);
}

void launch_flash_attention(const float*, const float*, const float*, float*, int, int, int,
                            int, int, bool, cudaStream_t) {
    kc_out_of_scope("launch_flash_attention");
}

void launch_paged_attention(const float*, const int*, const float*, const float*, float*,
                            const int*, int, int, int, int, int, int, cudaStream_t) {
    kc_out_of_scope("launch_paged_attention");
}

void launch_verify_draft_tokens(const float*, const float*, const int*, const float*,
                                const float*, int*, int*, int, int, cudaStream_t) {
    kc_out_of_scope("launch_verify_draft_tokens");
}

void launch_compute_prefix_length(const int*, int*, int, cudaStream_t) {
    kc_out_of_scope("launch_compute_prefix_length");
}

void launch_selective_scan(const float*, const float*, const float*, const float*, const float*,
                           float*, int, int, int, int, cudaStream_t) {
    kc_out_of_scope("launch_selective_scan");
}

void launch_depthwise_conv1d(const float*, const float*, const float*, float*, int, int, int, int,
                             cudaStream_t) {
    kc_out_of_scope("launch_depthwise_conv1d");
}

void launch_rmsnorm(const float*, const float*, float*, int, int, float, cudaStream_t) {
    kc_out_of_scope("launch_rmsnorm");
}

}  // extern "C"
