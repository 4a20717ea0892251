// Device buffers shared between the processes of a row-sharded job (CUDA IPC).
//
// mxb_fused_gemm_allgather writes this GPU's output rows into the other GPUs'
// copies of the full output; those copies are ordinary cudaMalloc buffers of
// the other processes, exported with cudaIpcGetMemHandle and mapped here with
// cudaIpcOpenMemHandle (peer access enabled on the way).  No multicast object
// is created: every peer store is a plain NVLink write to one GPU.
#include <cuda_runtime.h>

#include <cstring>

#include "internal.h"

static_assert(sizeof(cudaIpcMemHandle_t) == MXB_IPC_HANDLE_BYTES, "IPC handle size");

namespace {

// Runs `fn` with `device` current and restores the caller's device.
template <typename F>
int on_device(int device, const char* what, F fn) {
    int prev = 0;
    if (cudaGetDevice(&prev) != cudaSuccess) {
        cudaGetLastError();
        mxb::set_error("%s: no CUDA device", what);
        return MXB_E_CUDA;
    }
    if (cudaSetDevice(device) != cudaSuccess) {
        cudaGetLastError();
        mxb::set_error("%s: cannot select device %d", what, device);
        return MXB_E_ARG;
    }
    const cudaError_t e = fn();
    cudaSetDevice(prev);
    if (e != cudaSuccess) {
        cudaGetLastError();
        mxb::set_error("%s: %s", what, cudaGetErrorString(e));
        return e == cudaErrorMemoryAllocation ? MXB_E_NOMEM : MXB_E_CUDA;
    }
    return MXB_OK;
}

}  // namespace

extern "C" {

int mxb_ipc_alloc(int device, size_t bytes, void** dptr, unsigned char* handle) {
    if (!dptr || !handle || bytes == 0) {
        mxb::set_error("mxb_ipc_alloc: invalid arguments");
        return MXB_E_ARG;
    }
    *dptr = nullptr;
    return on_device(device, "mxb_ipc_alloc", [&]() {
        void* p = nullptr;
        cudaError_t e = cudaMalloc(&p, bytes);
        if (e != cudaSuccess) return e;
        cudaIpcMemHandle_t h;
        e = cudaIpcGetMemHandle(&h, p);
        if (e != cudaSuccess) {
            cudaFree(p);
            return e;
        }
        memcpy(handle, &h, sizeof(h));
        *dptr = p;
        return cudaSuccess;
    });
}

int mxb_ipc_open(int device, const unsigned char* handle, void** dptr) {
    if (!dptr || !handle) {
        mxb::set_error("mxb_ipc_open: invalid arguments");
        return MXB_E_ARG;
    }
    *dptr = nullptr;
    return on_device(device, "mxb_ipc_open", [&]() {
        cudaIpcMemHandle_t h;
        memcpy(&h, handle, sizeof(h));
        return cudaIpcOpenMemHandle(dptr, h, cudaIpcMemLazyEnablePeerAccess);
    });
}

int mxb_ipc_close(int device, void* dptr) {
    if (!dptr) return MXB_OK;
    return on_device(device, "mxb_ipc_close", [&]() { return cudaIpcCloseMemHandle(dptr); });
}

int mxb_ipc_free(int device, void* dptr) {
    if (!dptr) return MXB_OK;
    return on_device(device, "mxb_ipc_free", [&]() { return cudaFree(dptr); });
}

}  // extern "C"
