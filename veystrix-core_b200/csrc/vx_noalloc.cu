// vx_moe_block_noalloc: the whole MoE block for callers that cannot allocate
// device memory.
//
// Some hosts embed this library where no device allocator is reachable: a
// plugin running inside another runtime's memory pool, a caller that must not
// grow its footprint after start-up, or code that runs between a framework's
// allocations and is not allowed to call cudaMalloc.  This entry point takes
// the block's scratch from a fixed array in the library's own device memory
// instead of a caller workspace.  Every GPU that loads the library holds the
// array (VX_NOALLOC_SCRATCH_BYTES) until the process exits.
#include <cuda.h>

#include <mutex>

#include "vx_common.cuh"

namespace {

constexpr size_t kScratchBytes = VX_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

// Scratch shared by every call on a device.  Host code must not pass this
// symbol to a kernel: on the host it is only a stand-in for the device
// array; the device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

typedef CUresult (*PfnCtxGetCurrent)(CUcontext*);

// cuCtxGetCurrent through the runtime's driver entry point (the library
// links only the runtime).
PfnCtxGetCurrent ctx_get_current() {
  static PfnCtxGetCurrent fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PfnCtxGetCurrent>(p);
  });
  return fn;
}

std::mutex g_mu;
struct Cached {
  CUcontext ctx;
  void* addr;
};
Cached g_cache[kMaxDevices] = {};

// Device address of the scratch array in the current device's current
// context.  Looked up once per device (the first call on a device does this
// set-up) and again whenever the device's context differs from the one the
// address was taken in: after a cudaDeviceReset, or when the caller drives
// the device through a context other than the one seen before, the module is
// loaded again at another address.
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return vx_cuda_fail(e);
  if (dev < 0 || dev >= kMaxDevices) return VX_EUNSUPPORTED;
  PfnCtxGetCurrent get = ctx_get_current();
  if (!get) return VX_EUNSUPPORTED;
  // null until the runtime has made the device's context current on this thread
  CUcontext ctx = nullptr;
  if (get(&ctx) != CUDA_SUCCESS) return VX_EUNSUPPORTED;
  std::lock_guard<std::mutex> lk(g_mu);
  if (ctx && g_cache[dev].addr && g_cache[dev].ctx == ctx) {
    *out = g_cache[dev].addr;
    return VX_OK;
  }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_noalloc_scratch);   // makes the context current if needed
  if (e != cudaSuccess) return vx_cuda_fail(e);
  if (get(&ctx) != CUDA_SUCCESS || !ctx) return VX_EUNSUPPORTED;
  g_cache[dev] = {ctx, p};
  *out = p;
  return VX_OK;
}

}  // namespace

extern "C" int vx_moe_block_noalloc(const uint16_t* x, int32_t T, const vx_moe_weights* W,
                                    uint16_t* y, int32_t* inds, uint16_t* weights, void* stream) {
  // the same argument checks, in the same order, as vx_moe_block, so both
  // entry points return the same status for the same bad input
  const int bad = vx::block_args_status(x, T, W, y);
  if (bad != VX_OK || T == 0) return bad;
  const size_t need = vx_moe_block_workspace(T, W);
  if (need > kScratchBytes) return VX_EWORKSPACE;   // batch too large for the static scratch
  void* scratch = nullptr;
  const int s = scratch_address(&scratch);
  if (s != VX_OK) return s;
  // The same launch sequence as vx_moe_block; its permutation clears the
  // error word it accumulates into, and every other scratch piece is fully
  // written before it is read, so stale contents of the array do no harm.
  return vx_moe_block(x, T, W, y, inds, weights, scratch, kScratchBytes, stream);
}
