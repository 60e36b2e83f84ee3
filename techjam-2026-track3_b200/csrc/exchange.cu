// Peer-memory plumbing for the batch-sharded output gather: export / map
// device allocations between the processes of one node (CUDA IPC over
// NVLink), and enqueue lists of device-to-device copies and zero fills.
//
// The gather itself is host-orchestrated (sharding.py): every rank pushes the
// valid rows of each finished sample straight into the output buffer of every
// rank, so the bytes cross NVLink once and the transfer overlaps the next
// micro-batch's kernels.  Two transports: tj_copy_segments (copy engines, one
// stream per destination; the default, measured faster) and tj_push_segments
// (one small kernel storing over NVLink).  Padded rows never cross the link;
// each receiver zero-fills them locally with tj_copy_segments.
#include <cuda.h>
#include <cuda_runtime.h>
#include <string.h>

#include "internal.h"

namespace tj {

static_assert(sizeof(cudaIpcMemHandle_t) == TJ_IPC_HANDLE_BYTES, "IPC handle size");

typedef CUresult (*PfnMemGetAddressRange)(CUdeviceptr*, size_t*, CUdeviceptr);

static int check_device_for_push() {
  int sms = 0;
  return ensure_device_props(&sms);
}

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

// One kernel pushes a list of segments to every destination: each 16-byte
// unit is read once (read-only path) and stored to each destination's mapped
// buffer (local or a peer's, over NVLink).  Grid (blocks per segment,
// segments); small CTAs, so they can share SMs with the persistent GEMMs of
// the next micro-batch.
struct PushParams {
  char* dst[TJ_PUSH_MAX_DST];
  int num_dst;
  int64_t dst_off[TJ_PUSH_MAX_SEGS];
  const char* src[TJ_PUSH_MAX_SEGS];
  int64_t units[TJ_PUSH_MAX_SEGS];  // 16-byte units per segment
};

constexpr int kPushUnroll = 8;  // 16-byte loads in flight per thread

__global__ void __launch_bounds__(256) push_segments_kernel(const __grid_constant__ PushParams p) {
  const int s = blockIdx.y;
  const int64_t n = p.units[s];
  const uint4* src = reinterpret_cast<const uint4*>(p.src[s]);
  const int64_t tile = (int64_t)blockDim.x * kPushUnroll;
  // Each thread loads kPushUnroll units (coalesced across the block for each
  // k) before storing them, so enough bytes are in flight to cover the load
  // latency and the remote stores stream.
  for (int64_t base = (int64_t)blockIdx.x * tile; base < n; base += (int64_t)gridDim.x * tile) {
    uint4 v[kPushUnroll];
#pragma unroll
    for (int k = 0; k < kPushUnroll; ++k) {
      const int64_t u = base + (int64_t)k * blockDim.x + threadIdx.x;
      if (u < n) v[k] = __ldg(src + u);
    }
#pragma unroll 1
    for (int d = 0; d < p.num_dst; ++d) {
      uint4* dst = reinterpret_cast<uint4*>(p.dst[d] + p.dst_off[s]);
#pragma unroll
      for (int k = 0; k < kPushUnroll; ++k) {
        const int64_t u = base + (int64_t)k * blockDim.x + threadIdx.x;
        if (u < n) dst[u] = v[k];
      }
    }
  }
  // Make the stores visible to the other GPUs before anything ordered after
  // this kernel (the barrier that tells the peers their buffers are complete).
  __threadfence_system();
}

}  // namespace tj

using namespace tj;

extern "C" {

int tj_push_segments(void* const* dst_bases, int num_dst, const tj_push_segment* segs, int num_segs,
                     int blocks, void* stream) {
  if (num_dst < 1 || num_dst > TJ_PUSH_MAX_DST || num_segs < 0 || num_segs > TJ_PUSH_MAX_SEGS ||
      !dst_bases || (num_segs > 0 && !segs))
    return set_error(TJ_ERR_INVALID_ARGUMENT, "push_segments: %d destinations (1..%d), %d segments (0..%d)",
                     num_dst, TJ_PUSH_MAX_DST, num_segs, TJ_PUSH_MAX_SEGS);
  PushParams p{};
  p.num_dst = num_dst;
  for (int d = 0; d < num_dst; ++d) {
    if (!dst_bases[d] || (reinterpret_cast<uintptr_t>(dst_bases[d]) & 15u))
      return set_error(TJ_ERR_INVALID_ARGUMENT, "push_segments: destination %d not 16-byte aligned", d);
    p.dst[d] = static_cast<char*>(dst_bases[d]);
  }
  int live = 0;
  for (int i = 0; i < num_segs; ++i) {
    const tj_push_segment& g = segs[i];
    if (g.bytes < 0 || (g.bytes & 15) || (g.dst_offset & 15) || g.dst_offset < 0 ||
        (g.bytes > 0 && (!g.src || (reinterpret_cast<uintptr_t>(g.src) & 15u))))
      return set_error(TJ_ERR_INVALID_ARGUMENT,
                       "push_segments: segment %d must have 16-byte aligned source, offset and size", i);
    if (g.bytes == 0) continue;
    p.dst_off[live] = g.dst_offset;
    p.src[live] = static_cast<const char*>(g.src);
    p.units[live] = g.bytes / 16;
    ++live;
  }
  if (live == 0) return TJ_OK;
  int rc = check_device_for_push();
  if (rc) return rc;
  const int per_seg = blocks > 0 ? (blocks + live - 1) / live : 4;
  push_segments_kernel<<<dim3(per_seg, live), 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(TJ_ERR_CUDA, "push_segments launch: %s", cudaGetErrorString(e));
  return TJ_OK;
}

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
