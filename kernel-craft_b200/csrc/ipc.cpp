// ipc.cpp -- device buffers shared between the processes of one node (one
// process per GPU), for kernels that write their results straight into the
// peers' memory over NVLink (the fused column-parallel GEMM + all-gather).
//
// A buffer is allocated with kc_ipc_alloc in its owner process, its handle is
// shipped to the peers out of band (e.g. torch.distributed), and each peer maps
// it with kc_ipc_open.  Peers must close their mappings (kc_ipc_close) before
// the owner frees the buffer (kc_ipc_free).
#include <cuda_runtime.h>

#include <cstring>

#include "kc_common.cuh"

extern "C" {

int kc_ipc_handle_bytes(void) { return (int)sizeof(cudaIpcMemHandle_t); }

int kc_ipc_alloc(void** dev_ptr, size_t bytes) {
    KC_REQUIRE(dev_ptr != nullptr && bytes > 0, KC_ERR_INVALID_ARG, "kc_ipc_alloc: bad arguments");
    *dev_ptr = nullptr;
    KC_CUDA_TRY(cudaMalloc(dev_ptr, bytes), "cudaMalloc (shared buffer)");
    return KC_OK;
}

int kc_ipc_free(void* dev_ptr) {
    if (dev_ptr == nullptr) return KC_OK;
    KC_CUDA_TRY(cudaFree(dev_ptr), "cudaFree (shared buffer)");
    return KC_OK;
}

int kc_ipc_get_handle(const void* dev_ptr, void* handle_out) {
    KC_REQUIRE(dev_ptr && handle_out, KC_ERR_INVALID_ARG, "kc_ipc_get_handle: null argument");
    cudaIpcMemHandle_t h;
    KC_CUDA_TRY(cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr)), "cudaIpcGetMemHandle");
    memcpy(handle_out, &h, sizeof(h));
    return KC_OK;
}

int kc_ipc_open(const void* handle, void** dev_ptr) {
    KC_REQUIRE(handle && dev_ptr, KC_ERR_INVALID_ARG, "kc_ipc_open: null argument");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    *dev_ptr = nullptr;
    KC_CUDA_TRY(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess),
                "cudaIpcOpenMemHandle");
    return KC_OK;
}

int kc_ipc_close(void* dev_ptr) {
    if (dev_ptr == nullptr) return KC_OK;
    KC_CUDA_TRY(cudaIpcCloseMemHandle(dev_ptr), "cudaIpcCloseMemHandle");
    return KC_OK;
}

}  // extern "C"
