// sf_b200_bin_order_static: the depth ordering of sf_b200_bin_order for callers that
// cannot allocate device memory.
//
// Some integrations cannot hand the library a workspace: the host application owns
// the whole device memory budget through its own pool and does not let plugins call
// cudaMalloc, or the call happens on a path where an allocation (and the device-wide
// synchronisation cudaMalloc/cudaFree may imply) is not acceptable.  For them this
// entry point works in a scratch area that is part of the library image itself: a
// file-scope __device__ array, so nothing is allocated per call.
//
// Limits and sharing:
//  * at most SF_B200_STATIC_MAX_GAUSSIANS (1,048,576) Gaussians per call; larger
//    counts are rejected with SF_ERR_CAPACITY;
//  * the array (about 21 MB) is reserved on every GPU that loads libsf_b200.so, until
//    the process exits;
//  * all calls on a device share the one array and it keeps whatever the previous call
//    left in it.  Every byte a call reads is written by that same call first, so
//    nothing has to be cleared between calls; but two calls whose kernels overlap on
//    the GPU (different streams, or different host threads) race on the array and
//    must be serialised by the caller;
//  * the first call in each CUDA context looks up the device address of the array
//    (cudaGetSymbolAddress, with that context's device current) and keeps it for that
//    context; make that first call before any stream capture begins.  A context that
//    replaces a destroyed one gets its own lookup, but cudaDeviceReset may hand back
//    the old primary context's handle, so the entry point must not be used across a
//    cudaDeviceReset in one process;
//  * `stream` must belong to the current device (the array's address is the current
//    device's); a stream of another device is rejected with SF_ERR_ARGUMENT.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "sf_kernels.h"

namespace {

constexpr int64_t kMaxGaussians = 1 << 20;
constexpr size_t kScratchBytes = SF_B200_STATIC_SCRATCH_BYTES;  // >= the ordering workspace for kMaxGaussians

static __device__ __align__(256) unsigned char g_bin_order_scratch[kScratchBytes];

static_assert(kMaxGaussians == SF_B200_STATIC_MAX_GAUSSIANS, "limit stated in the header");

constexpr int kMaxDevices = 64;
std::mutex g_lock;
// per device: the context the address was looked up in, and the address
void* g_scratch_ctx[kMaxDevices] = {};
void* g_scratch_addr[kMaxDevices] = {};

using CtxGetCurrent = CUresult (*)(CUcontext*);
CtxGetCurrent g_ctx_get_current = nullptr;

int set_error(int code, const char* msg) {
  sf::set_last_error(msg);
  return code;
}

// The current driver context (the runtime's is current after cudaGetDevice), through the
// driver entry point the runtime exposes, so the library needs no libcuda link.
bool current_context(void** ctx) {
  if (!g_ctx_get_current) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return false;
    g_ctx_get_current = reinterpret_cast<CtxGetCurrent>(fn);
  }
  CUcontext c = nullptr;
  if (g_ctx_get_current(&c) != CUDA_SUCCESS) return false;
  *ctx = c;  // NULL while the runtime has not yet made a context current in this thread
  return true;
}

}  // namespace

extern "C" {

int sf_b200_bin_order_static(const int32_t* tile_count, const uint32_t* depth_key, int64_t n,
                             int32_t* order, int64_t* offsets, void* stream) {
  if (n < 0 || !offsets || (n > 0 && (!tile_count || !depth_key || !order)))
    return set_error(SF_ERR_ARGUMENT, "bin_order_static: bad arguments");
  if (n > kMaxGaussians)
    return set_error(SF_ERR_CAPACITY,
                     "bin_order_static: more than 1048576 Gaussians; use sf_b200_bin_order with a workspace");
  const size_t need = sf::bin_workspace_bytes(n, 0, 0);
  if (need > kScratchBytes) return set_error(SF_ERR_CAPACITY, "bin_order_static: static scratch too small");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return set_error(SF_ERR_CUDA, "bin_order_static: no current CUDA device");
  int stream_dev = -1;
  if (cudaStreamGetDevice(reinterpret_cast<cudaStream_t>(stream), &stream_dev) != cudaSuccess)
    return set_error(SF_ERR_ARGUMENT, "bin_order_static: invalid stream");
  if (stream_dev != dev)
    return set_error(SF_ERR_ARGUMENT, "bin_order_static: the stream belongs to another device than the current one");
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> guard(g_lock);
    void* ctx = nullptr;
    if (!current_context(&ctx)) return set_error(SF_ERR_CUDA, "bin_order_static: cuCtxGetCurrent unavailable");
    if (!ctx || !g_scratch_addr[dev] || g_scratch_ctx[dev] != ctx) {
      void* p = nullptr;
      // the lookup makes the device's context current in this thread if it was not
      const cudaError_t e = cudaGetSymbolAddress(&p, g_bin_order_scratch);
      if (e != cudaSuccess || !p) return set_error(SF_ERR_CUDA, "bin_order_static: cudaGetSymbolAddress failed");
      if (!current_context(&ctx) || !ctx) return set_error(SF_ERR_CUDA, "bin_order_static: no current CUDA context");
      g_scratch_addr[dev] = p;
      g_scratch_ctx[dev] = ctx;
    }
    scratch = g_scratch_addr[dev];
  }
  const cudaError_t e = sf::bin_order(tile_count, depth_key, n, order, offsets, scratch, kScratchBytes,
                                      reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return set_error(SF_ERR_CUDA, cudaGetErrorString(e));
  return SF_OK;
}

}  // extern "C"
