// Peer-memory plumbing for the batch-sharded output gather: export / map
// device allocations between the processes of one node (CUDA IPC over
// NVLink), and enqueue lists of device-to-device copies and zero fills.
//
// The gather itself is host-orchestrated (sharding.py): every rank pushes the
// valid rows of each finished sample straight into the output buffer of every
// rank with the copy engines, so the bytes cross NVLink once, no SM is spent
// on the transfer and it overlaps the next micro-batch's kernels.  Padded
// rows never cross the link; each receiver zero-fills them locally.
#include <cuda.h>
#include <cuda_runtime.h>
#include <string.h>

#include "internal.h"

namespace tj {

static_assert(sizeof(cudaIpcMemHandle_t) == TJ_IPC_HANDLE_BYTES, "IPC handle size");

typedef CUresult (*PfnMemGetAddressRange)(CUdeviceptr*, size_t*, CUdeviceptr);

static PfnMemGetAddressRange address_range_fn() {
  static PfnMemGetAddressRange fn = nullptr;
  static bool tried = false;
  if (!tried) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PfnMemGetAddressRange>(ptr);
    tried = true;
  }
  return fn;
}

}  // namespace tj

using namespace tj;

extern "C" {

int tj_ipc_export(const void* ptr, void* handle_out, int64_t* offset_out) {
  if (!ptr || !handle_out || !offset_out)
    return set_error(TJ_ERR_INVALID_ARGUMENT, "ipc_export: null pointer");
  PfnMemGetAddressRange range = address_range_fn();
  if (!range) return set_error(TJ_ERR_CUDA, "ipc_export: cuMemGetAddressRange is unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  CUresult r = range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS)
    return set_error(TJ_ERR_INVALID_ARGUMENT, "ipc_export: %p is not device memory (driver error %d)", ptr,
                     (int)r);
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess)
    return set_error(TJ_ERR_CUDA, "ipc_export: cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = (int64_t)(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return TJ_OK;
}

int tj_ipc_open(const void* handle, void** base_out) {
  if (!handle || !base_out) return set_error(TJ_ERR_INVALID_ARGUMENT, "ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess)
    return set_error(TJ_ERR_CUDA, "ipc_open: cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  *base_out = p;
  return TJ_OK;
}

int tj_ipc_close(void* base) {
  if (!base) return TJ_OK;
  cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess)
    return set_error(TJ_ERR_CUDA, "ipc_close: cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
  return TJ_OK;
}

int tj_copy_segments(const tj_copy_segment* segs, int n, void* stream) {
  if (n < 0 || (n > 0 && !segs)) return set_error(TJ_ERR_INVALID_ARGUMENT, "copy_segments: bad list");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int i = 0; i < n; ++i) {
    const tj_copy_segment& g = segs[i];
    if (g.bytes < 0 || (g.bytes > 0 && !g.dst))
      return set_error(TJ_ERR_INVALID_ARGUMENT, "copy_segments: segment %d has no destination", i);
    if (g.bytes == 0) continue;
    cudaError_t e = g.src ? cudaMemcpyAsync(g.dst, g.src, (size_t)g.bytes, cudaMemcpyDeviceToDevice, s)
                          : cudaMemsetAsync(g.dst, 0, (size_t)g.bytes, s);
    if (e != cudaSuccess)
      return set_error(TJ_ERR_CUDA, "copy_segments: segment %d (%lld bytes): %s", i, (long long)g.bytes,
                       cudaGetErrorString(e));
  }
  return TJ_OK;
}

}  // extern "C"
