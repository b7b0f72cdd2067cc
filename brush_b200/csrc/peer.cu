// peer.cu - device memory shared between the ranks' processes (CUDA IPC).
//
// A rank exports a cudaMalloc'd buffer with bsx_peer_alloc and sends the
// opaque handle to the other ranks, which map it with bsx_peer_open; loads and
// stores through the mapping cross NVLink. Used for the data-parallel exchange
// buffers (parameters, gradients, refine weights and flag words).
#include <string.h>

#include "common.cuh"

using namespace bsx;

static_assert(sizeof(cudaIpcMemHandle_t) == BSX_PEER_HANDLE_BYTES, "IPC handle size");

extern "C" bsx_status bsx_peer_alloc(bsx_ctx* ctx, uint64_t bytes, void** d_ptr, uint8_t* handle_out) {
    if (!ctx || !d_ptr || !handle_out || bytes == 0) return BSX_ERR_INVALID_ARG;
    *d_ptr = nullptr;
    cudaSetDevice(ctx->device);
    void* p = nullptr;
    bsx_status s = check_cuda(ctx, cudaMalloc(&p, bytes), "cudaMalloc (peer buffer)");
    if (s != BSX_OK) return s;
    s = check_cuda(ctx, cudaMemset(p, 0, bytes), "cudaMemset (peer buffer)");
    cudaIpcMemHandle_t h;
    if (s == BSX_OK) s = check_cuda(ctx, cudaIpcGetMemHandle(&h, p), "cudaIpcGetMemHandle");
    if (s != BSX_OK) {
        cudaFree(p);
        return s;
    }
    memcpy(handle_out, &h, sizeof(h));
    *d_ptr = p;
    return BSX_OK;
}

extern "C" bsx_status bsx_peer_free(bsx_ctx* ctx, void* d_ptr) {
    if (!ctx || !d_ptr) return BSX_ERR_INVALID_ARG;
    cudaSetDevice(ctx->device);
    return check_cuda(ctx, cudaFree(d_ptr), "cudaFree (peer buffer)");
}

extern "C" bsx_status bsx_peer_open(bsx_ctx* ctx, const uint8_t* handle, void** d_ptr) {
    if (!ctx || !handle || !d_ptr) return BSX_ERR_INVALID_ARG;
    *d_ptr = nullptr;
    cudaSetDevice(ctx->device);
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    return check_cuda(ctx, cudaIpcOpenMemHandle(d_ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
}

extern "C" bsx_status bsx_peer_close(bsx_ctx* ctx, void* d_ptr) {
    if (!ctx || !d_ptr) return BSX_ERR_INVALID_ARG;
    cudaSetDevice(ctx->device);
    return check_cuda(ctx, cudaIpcCloseMemHandle(d_ptr), "cudaIpcCloseMemHandle");
}
