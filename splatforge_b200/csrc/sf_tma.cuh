// Tensor-memory-accelerator staging of Gaussian records into shared memory.
//
// The record buffer [N, 20] float32 (80-byte rows) is described by a 2D tensor map
// (inner extent 20 floats, N rows, row stride 80 bytes, box 20 x 1).  One
// `cp.async.bulk.tensor ... tile::gather4` copies four rows named by their row
// indices (the Gaussian ids of four list entries) into 320 contiguous bytes of shared
// memory; completion is counted in bytes on an mbarrier.  The column coordinate is
// always 0 (16-byte aligned), the box is one row high, and every destination starts on
// a 128-byte boundary: groups of four records sit 384 bytes apart (GROUP_F4 float4).
// No multicast: each CTA loads its own rows from this GPU's memory.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace sf {

constexpr int TMA_GROUP = 4;             // records per gather4
constexpr int TMA_GROUP_BYTES = 384;     // 4 x 80 bytes, padded to a 128-byte multiple
constexpr int TMA_GROUP_F4 = TMA_GROUP_BYTES / 16;
constexpr int TMA_ROW_BYTES = 80;

// float4 offset of record slot j in a gather-staged batch
__device__ __forceinline__ int tma_slot_f4(int j) { return (j >> 2) * TMA_GROUP_F4 + (j & 3) * (TMA_ROW_BYTES / 16); }

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait for the phase with `parity`: false after `limit` polls (each poll
// suspends the thread for a hardware-bounded time), so a wait that can never finish
// returns instead of spinning forever.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity, int limit = 1 << 22) {
  for (int i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

__device__ __forceinline__ void tma_gather4(void* dst, const CUtensorMap* map, int r0, int r1, int r2, int r3,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(r0), "r"(r1), "r"(r2), "r"(r3), "r"(smem_addr(bar))
      : "memory");
}

// Issue the gathers of one batch: list entries ids[base .. base + n) into `stage`.  The
// calling warp's lanes each issue whole groups; a short last group repeats its last
// row (every row stays in bounds).  Returns the transaction bytes to expect.
__device__ __forceinline__ unsigned tma_issue_batch(float4* stage, const CUtensorMap* map, const int32_t* ids,
                                                    int base, int n, uint64_t* bar, int lane) {
  const int groups = (n + TMA_GROUP - 1) / TMA_GROUP;
  for (int g = lane; g < groups; g += 32) {
    const int j = g * TMA_GROUP;
    const int last = n - 1;
    const int r0 = __ldg(ids + base + j);
    const int r1 = __ldg(ids + base + min(j + 1, last));
    const int r2 = __ldg(ids + base + min(j + 2, last));
    const int r3 = __ldg(ids + base + min(j + 3, last));
    tma_gather4(stage + g * TMA_GROUP_F4, map, r0, r1, r2, r3, bar);
  }
  return (unsigned)(groups * TMA_GROUP * TMA_ROW_BYTES);
}

}  // namespace sf
