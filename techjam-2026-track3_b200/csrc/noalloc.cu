// tj_encoder_forward_noalloc: the encoder forward with its workspace in a
// fixed, library-owned device array instead of caller-provided memory.
//
// Who needs this: callers that must not allocate device memory at the point
// where they run the encoder.  Examples are a host embedding the library
// through a thin FFI (cgo, JNI, ctypes) that has no device allocator of its
// own and does not want to link one just for scratch space, and serving code
// whose device memory is fully planned up front.  cudaMalloc/cudaFree can also
// synchronise the whole device, which such latency-sensitive callers avoid.
//
// The array is a file-scope __device__ variable, so every GPU that loads this
// library holds TJ_NOALLOC_WORKSPACE_BYTES of it until the process exits.  In
// host code its name is only a host-side stand-in, never a device address: the
// real address comes from cudaGetSymbolAddress, looked up on the first call
// made with a device current and cached for that device and its current CUDA
// context (a device reset or another context on the device makes the next
// call look it up again).
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace tj {

static __device__ __align__(256) uint8_t g_noalloc_workspace[TJ_NOALLOC_WORKSPACE_BYTES];

typedef CUresult (*PfnCtxGetCurrent)(CUcontext*);

static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[64] = {nullptr};
static CUcontext g_noalloc_ctx[64] = {nullptr};

static PfnCtxGetCurrent ctx_get_current_fn() {
  static PfnCtxGetCurrent fn = nullptr;
  static bool tried = false;
  if (!tried) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PfnCtxGetCurrent>(ptr);
    tried = true;
  }
  return fn;
}

// Device address of g_noalloc_workspace on the current device.
static int noalloc_workspace(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(TJ_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return set_error(TJ_ERR_UNSUPPORTED, "device index %d", dev);
  // The context current on this thread (null before the runtime has made one
  // current here; the lookup below does that, and the next call then sees
  // the real context and looks the address up once more).
  CUcontext ctx = nullptr;
  PfnCtxGetCurrent get_ctx = ctx_get_current_fn();
  if (get_ctx) get_ctx(&ctx);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr || g_noalloc_ctx[dev] != ctx) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_workspace);
    if (e != cudaSuccess || p == nullptr)
      return set_error(TJ_ERR_CUDA, "encoder_forward_noalloc: cudaGetSymbolAddress failed: %s",
                       cudaGetErrorString(e));
    g_noalloc_ptr[dev] = p;
    g_noalloc_ctx[dev] = ctx;
  }
  *out = g_noalloc_ptr[dev];
  return TJ_OK;
}

}  // namespace tj

extern "C" int tj_encoder_forward_noalloc(const tj_encoder_desc* desc, const tj_layer_weights* layers,
                                          const float* final_gamma, const float* final_beta,
                                          const float* x, const uint8_t* mask, float* out,
                                          void* stream) {
  using namespace tj;
  const int64_t need = tj_encoder_workspace_bytes(desc);
  if (need <= 0) return set_error(TJ_ERR_INVALID_ARGUMENT, "encoder_forward_noalloc: invalid descriptor");
  if (need > (int64_t)TJ_NOALLOC_WORKSPACE_BYTES)
    return set_error(TJ_ERR_WORKSPACE,
                     "encoder_forward_noalloc: this shape needs %lld bytes of workspace but the "
                     "static workspace holds %lld bytes; use tj_encoder_forward with a "
                     "caller-provided workspace",
                     (long long)need, (long long)TJ_NOALLOC_WORKSPACE_BYTES);
  void* ws = nullptr;
  int rc = noalloc_workspace(&ws);
  if (rc) return rc;
  // Nothing in the workspace has to start at zero: every entry a kernel reads
  // is written earlier in the same call, so the previous call's contents are
  // harmless.  Calls that overlap on the GPU (other streams, other threads)
  // share this one array and race.
  return tj_encoder_forward(desc, layers, final_gamma, final_beta, x, mask, out, ws,
                            (int64_t)TJ_NOALLOC_WORKSPACE_BYTES, stream);
}
