// Peer-memory buffers shared between the processes of one node (one process per GPU): a rank allocates a buffer,
// exports its CUDA IPC handle, the other ranks map it into their own contexts and copy from it over NVLink with
// the copy engines.  Used to hand a layer's eigendecomposition from the rank that computed it to the ranks that
// solve the other row shards of the same layer, with no collective on their streams.
#include <string.h>
#include "common.cuh"

static_assert(sizeof(cudaIpcMemHandle_t) == MPQ_IPC_HANDLE_BYTES, "IPC handle size");

// cudaMalloc `bytes` on the current device and export the allocation's IPC handle (MPQ_IPC_HANDLE_BYTES bytes).
MPQ_API int mpq_peer_alloc(size_t bytes, void** out_ptr, void* out_handle, cudaStream_t stream) {
  (void)stream;
  MPQ_CHECK_ARG(out_ptr != nullptr && out_handle != nullptr, "mpq_peer_alloc: null output");
  MPQ_CHECK_ARG(bytes > 0, "mpq_peer_alloc: empty buffer");
  *out_ptr = nullptr;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) {
    mpq::set_last_error("mpq_peer_alloc: cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
    return (int)e;
  }
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    mpq::set_last_error("mpq_peer_alloc: cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
    return (int)e;
  }
  memcpy(out_handle, &h, sizeof(h));
  *out_ptr = p;
  return MPQ_OK;
}

// Map another process's exported buffer into the current device's context (peer access enabled on demand).
MPQ_API int mpq_peer_open(const void* handle, void** out_ptr, cudaStream_t stream) {
  (void)stream;
  MPQ_CHECK_ARG(handle != nullptr && out_ptr != nullptr, "mpq_peer_open: null argument");
  *out_ptr = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    mpq::set_last_error("mpq_peer_open: cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
    return (int)e;
  }
  *out_ptr = p;
  return MPQ_OK;
}

// Unmap a buffer opened with mpq_peer_open.
MPQ_API int mpq_peer_close(void* ptr, cudaStream_t stream) {
  (void)stream;
  if (ptr == nullptr) return MPQ_OK;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) {
    mpq::set_last_error("mpq_peer_close: %s", cudaGetErrorString(e));
    return (int)e;
  }
  return MPQ_OK;
}

// Free a buffer from mpq_peer_alloc (after every peer has closed its mapping).
MPQ_API int mpq_peer_free(void* ptr, cudaStream_t stream) {
  (void)stream;
  if (ptr == nullptr) return MPQ_OK;
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) {
    mpq::set_last_error("mpq_peer_free: %s", cudaGetErrorString(e));
    return (int)e;
  }
  return MPQ_OK;
}

// dst[0:bytes] = src[0:bytes] on `stream`; either pointer may be a peer mapping (unified addressing).
MPQ_API int mpq_copy_bytes(void* dst, const void* src, size_t bytes, cudaStream_t stream) {
  if (bytes == 0) return MPQ_OK;
  MPQ_CHECK_ARG(dst != nullptr && src != nullptr, "mpq_copy_bytes: null pointer");
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, stream);
  if (e != cudaSuccess) {
    mpq::set_last_error("mpq_copy_bytes: %s", cudaGetErrorString(e));
    return (int)e;
  }
  return MPQ_OK;
}
