// Device buffers another process on the same node can map (CUDA IPC), for
// the row-partitioned path's peer stores: each rank allocates the buffers its
// peers write halo rows into, hands out their IPC handles, and maps the
// peers' buffers with cudaIpcOpenMemHandle.  Plain peer mappings only: no
// multicast objects are created.
#include <cstring>

#include "bgnn_internal.cuh"

namespace {
int peer_ctx_ok(bgnn_ctx* ctx) {
  if (!ctx) return BGNN_ERR_INVALID_ARG;
  cudaError_t e = cudaSetDevice(ctx->device);
  if (e != cudaSuccess)
    return bgnn_set_error(ctx, BGNN_ERR_CUDA, "cudaSetDevice(%d): %s", ctx->device,
                          cudaGetErrorString(e));
  return BGNN_OK;
}
}  // namespace

extern "C" int bgnn_shared_alloc(bgnn_ctx* ctx, uint64_t bytes, void** out) {
  BGNN_TRY(peer_ctx_ok(ctx));
  BGNN_REQUIRE(ctx, out != nullptr, "NULL out");
  *out = nullptr;
  if (bytes == 0) return BGNN_OK;
  BGNN_CUDA(ctx, cudaMalloc(out, bytes));  // whole allocation: its IPC handle maps from its base
  return BGNN_OK;
}

extern "C" int bgnn_shared_free(bgnn_ctx* ctx, void* p) {
  BGNN_TRY(peer_ctx_ok(ctx));
  if (p) BGNN_CUDA(ctx, cudaFree(p));
  return BGNN_OK;
}

extern "C" int bgnn_ipc_handle(bgnn_ctx* ctx, void* base, uint8_t* handle_out) {
  BGNN_TRY(peer_ctx_ok(ctx));
  BGNN_REQUIRE(ctx, base && handle_out, "NULL argument");
  cudaIpcMemHandle_t h;
  BGNN_CUDA(ctx, cudaIpcGetMemHandle(&h, base));
  static_assert(sizeof(h) == BGNN_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle_out, &h, sizeof(h));
  return BGNN_OK;
}

extern "C" int bgnn_ipc_open(bgnn_ctx* ctx, const uint8_t* handle, void** out) {
  BGNN_TRY(peer_ctx_ok(ctx));
  BGNN_REQUIRE(ctx, handle && out, "NULL argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  BGNN_CUDA(ctx, cudaIpcOpenMemHandle(out, h, cudaIpcMemLazyEnablePeerAccess));
  return BGNN_OK;
}

extern "C" int bgnn_ipc_close(bgnn_ctx* ctx, void* p) {
  BGNN_TRY(peer_ctx_ok(ctx));
  if (p) BGNN_CUDA(ctx, cudaIpcCloseMemHandle(p));
  return BGNN_OK;
}
