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

// Stable LSD radix sort of n <= capacity (key, value) pairs held in shared memory by
// one warp: 8-bit digits, bytes that are equal in every key skipped, ranks from
// __match_any_sync.  The result lands in (*kout, *vout), one of the two buffers.
__device__ __forceinline__ void warp_radix_sort_u32(uint32_t* k0, uint32_t* v0, uint32_t* k1, uint32_t* v1,
                                                uint32_t* hist, int n, int lane, uint32_t** kout,
                                                uint32_t** vout) {
  uint32_t orv = 0u, andv = 0xffffffffu;
  for (int i = lane; i < n; i += 32) { orv |= k0[i]; andv &= k0[i]; }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    orv |= __shfl_xor_sync(FULL, orv, o);
    andv &= __shfl_xor_sync(FULL, andv, o);
  }
  const uint32_t vary = orv ^ andv;
  const unsigned lt = (1u << lane) - 1u;
  uint32_t *ki = k0, *vi = v0, *ko = k1, *vo = v1;
  for (int shift = 0; shift < 32; shift += 8) {
    if (((vary >> shift) & 0xffu) == 0u) continue;
#pragma unroll
    for (int b = 0; b < 8; ++b) hist[lane * 8 + b] = 0u;
    __syncwarp();
    for (int c = 0; c < n; c += 32) {
      const int i = c + lane;
      const bool valid = i < n;
      const uint32_t d = valid ? (ki[i] >> shift) & 0xffu : 0u;
      const unsigned peers = __match_any_sync(FULL, valid ? d : 0x100u + lane);
      if (valid && lane == __ffs(peers) - 1) hist[d] += __popc(peers);
      __syncwarp();
    }
    // exclusive scan of the 256 counts: 8 per lane
    uint32_t loc[8], sum = 0u;
#pragma unroll
    for (int b = 0; b < 8; ++b) { loc[b] = hist[lane * 8 + b]; sum += loc[b]; }
    uint32_t incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(FULL, incl, o);
      if (lane >= o) incl += y;
    }
    uint32_t run = incl - sum;
#pragma unroll
    for (int b = 0; b < 8; ++b) { hist[lane * 8 + b] = run; run += loc[b]; }
    __syncwarp();
    for (int c = 0; c < n; c += 32) {
      const int i = c + lane;
      const bool valid = i < n;
      const uint32_t key = valid ? ki[i] : 0u;
      const uint32_t d = (key >> shift) & 0xffu;
      const unsigned peers = __match_any_sync(FULL, valid ? d : 0x100u + lane);
      const uint32_t base = valid ? hist[d] : 0u;
      __syncwarp();
      if (valid) {
        const uint32_t pos = base + __popc(peers & lt);
        ko[pos] = key;
        vo[pos] = vi[i];
        if (lane == 31 - __clz(peers)) hist[d] = base + __popc(peers);
      }
      __syncwarp();
    }
    uint32_t* t = ki; ki = ko; ko = t;
    t = vi; vi = vo; vo = t;
  }
  *kout = ki;
  *vout = vi;
}

}  // namespace sf
