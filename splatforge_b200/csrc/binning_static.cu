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
//  * the first call on each device looks up the device address of the array
//    (cudaGetSymbolAddress, with that device current); make that first call before
//    any stream capture begins.
#include <cuda_runtime.h>

#include <mutex>

#include "sf_kernels.h"

namespace {

constexpr int64_t kMaxGaussians = 1 << 20;
constexpr size_t kScratchBytes = 21u << 20;  // >= the ordering workspace for kMaxGaussians

static __device__ __align__(256) unsigned char g_bin_order_scratch[kScratchBytes];

static_assert(kMaxGaussians == SF_B200_STATIC_MAX_GAUSSIANS, "limit stated in the header");

constexpr int kMaxDevices = 64;
std::mutex g_lock;
void* g_scratch_addr[kMaxDevices] = {};

int set_error(int code, const char* msg) {
  sf::set_last_error(msg);
  return code;
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
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> guard(g_lock);
    if (!g_scratch_addr[dev]) {
      void* p = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&p, g_bin_order_scratch);
      if (e != cudaSuccess || !p) return set_error(SF_ERR_CUDA, "bin_order_static: cudaGetSymbolAddress failed");
      g_scratch_addr[dev] = p;
    }
    scratch = g_scratch_addr[dev];
  }
  const cudaError_t e = sf::bin_order(tile_count, depth_key, n, order, offsets, scratch, kScratchBytes,
                                      reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return set_error(SF_ERR_CUDA, cudaGetErrorString(e));
  return SF_OK;
}

}  // extern "C"
