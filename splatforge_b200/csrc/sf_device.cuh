// Device-side utilities shared by the kernels of libsf_b200.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "sf_math.cuh"

namespace sf {

constexpr unsigned FULL = 0xffffffffu;
constexpr int TILE = 16;
constexpr int TILE_PIXELS = TILE * TILE;  // one CTA per tile, one thread per pixel

// Launch context: the stream and the status of the entry point being executed.
struct Launch {
  cudaStream_t stream;
};

__device__ __forceinline__ int warp_max(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(FULL, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
  return v;
}

// Transposed butterfly reduction of 16 per-lane values: 16 shuffles instead of 80.
// After it, every even lane l holds the warp total of value (l >> 1); lane l+1 holds
// the same total.
__device__ __forceinline__ float reduce16_transposed(float (&v)[16], int lane) {
  {
    const bool up = lane & 16;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float send = up ? v[i] : v[i + 8];
      float keep = up ? v[i + 8] : v[i];
      v[i] = keep + __shfl_xor_sync(FULL, send, 16);
    }
  }
  {
    const bool up = lane & 8;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float send = up ? v[i] : v[i + 4];
      float keep = up ? v[i + 4] : v[i];
      v[i] = keep + __shfl_xor_sync(FULL, send, 8);
    }
  }
  {
    const bool up = lane & 4;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      float send = up ? v[i] : v[i + 2];
      float keep = up ? v[i + 2] : v[i];
      v[i] = keep + __shfl_xor_sync(FULL, send, 4);
    }
  }
  {
    const bool up = lane & 2;
    float send = up ? v[0] : v[1];
    float keep = up ? v[1] : v[0];
    v[0] = keep + __shfl_xor_sync(FULL, send, 2);
  }
  v[0] += __shfl_xor_sync(FULL, v[0], 1);
  return v[0];
}

}  // namespace sf
