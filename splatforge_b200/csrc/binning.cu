// Tile binning on the device: stable depth order of the Gaussians, exclusive scan of
// their tile counts, emission of (tile, Gaussian) intersections in depth order and a
// stable LSD radix sort by tile -- the per-tile lists of tile_binning.py:10-34 (global
// stable argsort by depth, inclusive tile rectangles) built without a host copy.
//
// Radix sort: 8-bit digits, one pass = upsweep (per-CTA digit histogram) + scan of the
// digit-major histogram + downsweep.  The downsweep ranks keys stably inside a CTA
// with warp-level match (__match_any_sync) and per-warp digit counters, so no
// inter-CTA waiting is needed (no spin loops anywhere).
#include <cuda_runtime.h>

#include "sf_device.cuh"
#include "sf_kernels.h"

namespace sf {

namespace {

// ------------------------------------------------------------------ scan
constexpr int SC_THREADS = 256;
constexpr int SC_ITEMS = 8;
constexpr int SC_CHUNK = SC_THREADS * SC_ITEMS;  // elements per CTA
constexpr int SC_TOP_THREADS = 1024;
constexpr int SC_TOP_ITEMS = 16;
constexpr int64_t SC_MAX = (int64_t)SC_CHUNK * SC_TOP_THREADS * SC_TOP_ITEMS;

template <typename T>
__device__ __forceinline__ T block_exclusive_scan(T v, T* s_warp, T& total) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
  T x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    T y = __shfl_up_sync(FULL, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[wid] = x;
  __syncthreads();
  if (wid == 0) {
    T w = lane < nw ? s_warp[lane] : T(0);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      T y = __shfl_up_sync(FULL, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nw) s_warp[lane] = w;
  }
  __syncthreads();
  total = s_warp[nw - 1];
  T before = wid > 0 ? s_warp[wid - 1] : T(0);
  __syncthreads();
  return before + x - v;
}

template <typename TI, typename TO>
__global__ void __launch_bounds__(SC_THREADS) scan_reduce_kernel(const TI* in, int64_t n, TO* partial) {
  __shared__ TO s_warp[32];
  const int64_t base = (int64_t)blockIdx.x * SC_CHUNK + (int64_t)threadIdx.x * SC_ITEMS;
  TO acc = 0;
#pragma unroll
  for (int k = 0; k < SC_ITEMS; ++k)
    if (base + k < n) acc += (TO)in[base + k];
  TO total;
  block_exclusive_scan<TO>(acc, s_warp, total);
  if (threadIdx.x == 0) partial[blockIdx.x] = total;
}

template <typename TO>
__global__ void __launch_bounds__(SC_TOP_THREADS) scan_top_kernel(TO* partial, int64_t nb, TO* grand) {
  __shared__ TO s_warp[32];
  const int64_t base = (int64_t)threadIdx.x * SC_TOP_ITEMS;
  TO vals[SC_TOP_ITEMS];
  TO acc = 0;
#pragma unroll
  for (int k = 0; k < SC_TOP_ITEMS; ++k) {
    vals[k] = base + k < nb ? partial[base + k] : TO(0);
    acc += vals[k];
  }
  TO total;
  TO run = block_exclusive_scan<TO>(acc, s_warp, total);
#pragma unroll
  for (int k = 0; k < SC_TOP_ITEMS; ++k) {
    if (base + k < nb) partial[base + k] = run;
    run += vals[k];
  }
  if (threadIdx.x == 0 && grand) *grand = total;
}

template <typename TI, typename TO>
__global__ void __launch_bounds__(SC_THREADS) scan_down_kernel(const TI* in, int64_t n, const TO* partial, TO* out) {
  __shared__ TO s_warp[32];
  const int64_t base = (int64_t)blockIdx.x * SC_CHUNK + (int64_t)threadIdx.x * SC_ITEMS;
  TO vals[SC_ITEMS];
  TO acc = 0;
#pragma unroll
  for (int k = 0; k < SC_ITEMS; ++k) {
    vals[k] = base + k < n ? (TO)in[base + k] : TO(0);
    acc += vals[k];
  }
  TO total;
  TO run = block_exclusive_scan<TO>(acc, s_warp, total) + partial[blockIdx.x];
#pragma unroll
  for (int k = 0; k < SC_ITEMS; ++k) {
    if (base + k < n) out[base + k] = run;
    run += vals[k];
  }
}

inline int64_t scan_blocks(int64_t n) { return (n + SC_CHUNK - 1) / SC_CHUNK; }

// exclusive scan; when `grand` is non-null it receives the total
template <typename TI, typename TO>
cudaError_t exclusive_scan(const TI* in, int64_t n, TO* out, TO* partial, TO* grand, cudaStream_t s) {
  if (n <= 0) {
    if (grand) return cudaMemsetAsync(grand, 0, sizeof(TO), s);
    return cudaSuccess;
  }
  if (n > SC_MAX) return cudaErrorInvalidValue;
  const int64_t nb = scan_blocks(n);
  count_launches(3);
  scan_reduce_kernel<TI, TO><<<(unsigned)nb, SC_THREADS, 0, s>>>(in, n, partial);
  scan_top_kernel<TO><<<1, SC_TOP_THREADS, 0, s>>>(partial, nb, grand);
  scan_down_kernel<TI, TO><<<(unsigned)nb, SC_THREADS, 0, s>>>(in, n, partial, out);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ radix sort
constexpr int RS_THREADS = 256;
constexpr int RS_WARPS = RS_THREADS / 32;
#ifndef SF_RS_ROUNDS
#define SF_RS_ROUNDS 8
#endif
constexpr int RS_ROUNDS = SF_RS_ROUNDS;               // 32-key rounds per warp
constexpr int RS_CHUNK = RS_THREADS * RS_ROUNDS;      // keys per CTA
constexpr int RADIX = 256;
static_assert(RS_THREADS == RADIX, "one thread per digit in the histogram stages");

// Per-block digit histograms.  Each thread reads its keys four at a time (128-bit
// loads) when the block's slab is 16-byte aligned.
// Element counts: n, or with n_dev the count on the device (bounded by n; a count
// above n means "nothing": the binning that produced it overflowed its capacity).
__device__ __forceinline__ int64_t live_count(int64_t n, const int64_t* n_dev) {
  if (!n_dev) return n;
  const int64_t t = *n_dev;
  return t > n ? 0 : t;
}

__global__ void __launch_bounds__(RS_THREADS) radix_upsweep_kernel(const uint32_t* keys, int64_t n,
                                                                   const int64_t* n_dev, int shift, int nb,
                                                                   uint32_t* hist) {
  n = live_count(n, n_dev);
  if ((int64_t)blockIdx.x * RS_CHUNK >= n) {  // a block past the live count: empty histogram
    hist[(int64_t)threadIdx.x * nb + blockIdx.x] = 0;  // RS_THREADS == RADIX
    return;
  }
  __shared__ uint32_t s_hist[RS_WARPS][RADIX];
  const int wid = threadIdx.x >> 5;
  for (int k = threadIdx.x; k < RS_WARPS * RADIX; k += RS_THREADS) (&s_hist[0][0])[k] = 0;
  __syncthreads();
  const int64_t block0 = (int64_t)blockIdx.x * RS_CHUNK;
  const int rows = (int)max((int64_t)0, min((int64_t)RS_CHUNK, n - block0));
  if (rows == RS_CHUNK && (reinterpret_cast<uintptr_t>(keys + block0) & 15) == 0) {
    const uint4* k4 = reinterpret_cast<const uint4*>(keys + block0);
#pragma unroll
    for (int r = 0; r < RS_CHUNK / 4 / RS_THREADS; ++r) {
      const uint4 v = k4[r * RS_THREADS + threadIdx.x];
      atomicAdd(&s_hist[wid][(v.x >> shift) & 0xff], 1u);
      atomicAdd(&s_hist[wid][(v.y >> shift) & 0xff], 1u);
      atomicAdd(&s_hist[wid][(v.z >> shift) & 0xff], 1u);
      atomicAdd(&s_hist[wid][(v.w >> shift) & 0xff], 1u);
    }
  } else {
    for (int i = threadIdx.x; i < rows; i += RS_THREADS)
      atomicAdd(&s_hist[wid][(keys[block0 + i] >> shift) & 0xff], 1u);
  }
  __syncthreads();
  const int d = threadIdx.x;  // RS_THREADS == RADIX
  uint32_t sum = 0;
#pragma unroll
  for (int w = 0; w < RS_WARPS; ++w) sum += s_hist[w][d];
  hist[(int64_t)d * nb + blockIdx.x] = sum;
}

// Scatter pass: ranks within each warp from __match_any_sync (stable: keys of one digit
// keep their input order), then the block's keys are regrouped by digit in shared
// memory and written out from there, so consecutive threads store consecutive
// addresses of one digit's run instead of 32 scattered runs per instruction.
__global__ void __launch_bounds__(RS_THREADS, RS_ROUNDS <= 8 ? 4 : 2) radix_downsweep_kernel(
    const uint32_t* keys_in, const int32_t* vals_in, int64_t n, const int64_t* n_dev, int shift, int nb,
    const uint32_t* offsets, uint32_t* keys_out, int32_t* vals_out) {
  n = live_count(n, n_dev);
  if ((int64_t)blockIdx.x * RS_CHUNK >= n) return;  // past the live count: nothing to move
  __shared__ uint32_t s_cnt[RS_WARPS][RADIX];
  __shared__ uint32_t s_off[RADIX];    // this block's first output slot per digit
  __shared__ uint32_t s_local[RADIX];  // first slot of each digit inside the block
  __shared__ uint32_t s_wsum[RS_WARPS];
  __shared__ uint32_t s_keys[RS_CHUNK];
  __shared__ int32_t s_vals[RS_CHUNK];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int k = threadIdx.x; k < RS_WARPS * RADIX; k += RS_THREADS) (&s_cnt[0][0])[k] = 0;
  s_off[threadIdx.x] = offsets[(int64_t)threadIdx.x * nb + blockIdx.x];
  __syncthreads();
  const int64_t block0 = (int64_t)blockIdx.x * RS_CHUNK;
  const int64_t base = block0 + (int64_t)wid * (RS_CHUNK / RS_WARPS);
  const int rows = (int)max((int64_t)0, min((int64_t)RS_CHUNK, n - block0));
  const unsigned lt = (1u << lane) - 1u;
  uint32_t key[RS_ROUNDS];
  int32_t val[RS_ROUNDS];
  uint32_t rank[RS_ROUNDS];
  // all loads first, so that the 32 per thread are in flight together
#pragma unroll
  for (int r = 0; r < RS_ROUNDS; ++r) {
    const int64_t idx = base + r * 32 + lane;
    const bool valid = idx < n;
    key[r] = valid ? __ldg(keys_in + idx) : 0u;
    val[r] = valid ? __ldg(vals_in + idx) : 0;
  }
#pragma unroll
  for (int r = 0; r < RS_ROUNDS; ++r) {
    const int64_t idx = base + r * 32 + lane;
    const bool valid = idx < n;
    const uint32_t d = (key[r] >> shift) & 0xff;
    const unsigned peers = __match_any_sync(FULL, valid ? d : 0x100u + lane);
    const uint32_t before = valid ? s_cnt[wid][d] : 0u;
    __syncwarp();
    rank[r] = before + __popc(peers & lt);
    if (valid && lane == 31 - __clz(peers)) s_cnt[wid][d] = before + __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  {
    // per digit: exclusive prefix over warps, and the digit's total in this block
    const int d = threadIdx.x;
    uint32_t run = 0;
#pragma unroll
    for (int w = 0; w < RS_WARPS; ++w) {
      const uint32_t c = s_cnt[w][d];
      s_cnt[w][d] = run;
      run += c;
    }
    // exclusive scan of the 256 digit totals across the block
    uint32_t incl = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(FULL, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) s_wsum[wid] = incl;
    __syncthreads();
    uint32_t before = 0;
    for (int w = 0; w < wid; ++w) before += s_wsum[w];
    s_local[d] = before + incl - run;
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < RS_ROUNDS; ++r) {
    const int64_t idx = base + r * 32 + lane;
    if (idx < n) {
      const uint32_t d = (key[r] >> shift) & 0xff;
      const uint32_t lpos = s_local[d] + s_cnt[wid][d] + rank[r];
      s_keys[lpos] = key[r];
      s_vals[lpos] = val[r];
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < rows; i += RS_THREADS) {
    const uint32_t k = s_keys[i];
    const uint32_t d = (k >> shift) & 0xff;
    const uint32_t pos = s_off[d] + (uint32_t)i - s_local[d];
    keys_out[pos] = k;
    vals_out[pos] = s_vals[i];
  }
}

inline int64_t radix_blocks(int64_t n) { return (n + RS_CHUNK - 1) / RS_CHUNK; }

struct RadixScratch {
  uint32_t* hist;      // RADIX * nb
  uint32_t* partial;   // scan partials
};

// Stable sort of (key, value) pairs by key bits [0, bits).  Ping-pongs between
// (k0, v0) and (k1, v1); the result lands in (k_final, v_final) which is one of the two
// buffers, or v_out when given (the last pass then writes values there).
// With n_dev, n is the buffers' capacity and the live count is read on the device.
cudaError_t radix_sort(uint32_t* k0, int32_t* v0, uint32_t* k1, int32_t* v1, int64_t n, int bits,
                       RadixScratch sc, uint32_t** k_final, int32_t** v_final, int32_t* v_out,
                       cudaStream_t s, const int64_t* n_dev = nullptr) {
  const int passes = (bits + 7) / 8;
  uint32_t* ki = k0; int32_t* vi = v0; uint32_t* ko = k1; int32_t* vo = v1;
  const int64_t nb = radix_blocks(n);
  if (n > 0 && nb * RADIX > SC_MAX) return cudaErrorInvalidValue;
  for (int p = 0; p < passes && n > 0; ++p) {
    const int shift = 8 * p;
    int32_t* vdst = (p == passes - 1 && v_out) ? v_out : vo;
    count_launches(2);
    radix_upsweep_kernel<<<(unsigned)nb, RS_THREADS, 0, s>>>(ki, n, n_dev, shift, (int)nb, sc.hist);
    cudaError_t e = exclusive_scan<uint32_t, uint32_t>(sc.hist, RADIX * nb, sc.hist, sc.partial, nullptr, s);
    if (e != cudaSuccess) return e;
    radix_downsweep_kernel<<<(unsigned)nb, RS_THREADS, 0, s>>>(ki, vi, n, n_dev, shift, (int)nb, sc.hist, ko,
                                                                vdst);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    ki = ko; vi = vdst;
    ko = (ko == k1) ? k0 : k1;
    vo = (vo == v1) ? v0 : v1;
  }
  *k_final = ki;
  *v_final = vi;
  return cudaGetLastError();
}

// ------------------------------------------------------------------ binning kernels
__global__ void iota_copy_kernel(const uint32_t* keys, int64_t n, uint32_t* k, int32_t* v) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) { k[i] = keys[i]; v[i] = (int32_t)i; }
}

__global__ void gather_counts_kernel(const int32_t* order, const int32_t* count, int64_t n,
                                     int32_t* out_order, int32_t* sorted_count) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    const int32_t g = order[i];
    out_order[i] = g;
    sorted_count[i] = count[g];
  }
}

// One warp per 32 depth-ordered Gaussians: the warp writes each Gaussian's run of
// intersections in turn, lanes covering consecutive entries (coalesced stores).
// A total (offsets[n]) above cap writes nothing and raises *overflow.
__global__ void emit_kernel(const int32_t* order, const int64_t* offsets, const int32_t* rect,
                            int64_t n, int tiles_x, int64_t cap, int32_t* overflow, uint32_t* tiles, int32_t* ids) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t first = warp * 32;
  if (offsets[n] > cap) {
    if (blockIdx.x == 0 && threadIdx.x == 0 && overflow) *overflow = 1;
    return;
  }
  if (first >= n) return;
  const int64_t i = first + lane;
  int g = 0, x0 = 0, y0 = 0, w = 1;
  long long o = 0, c = 0;
  if (i < n) {
    g = order[i];
    o = offsets[i];
    c = offsets[i + 1] - o;
    const int4 r = reinterpret_cast<const int4*>(rect)[g];
    x0 = r.x; y0 = r.y; w = r.z - r.x + 1;
  }
  for (int src = 0; src < 32; ++src) {
    const long long cs = __shfl_sync(FULL, c, src);
    if (cs == 0) continue;
    const long long os = __shfl_sync(FULL, o, src);
    const int gs = __shfl_sync(FULL, g, src);
    const int xs = __shfl_sync(FULL, x0, src), ys = __shfl_sync(FULL, y0, src), ws = __shfl_sync(FULL, w, src);
    // row/column of entry k in the rectangle without an integer division: lane starts at
    // (lane / ws, lane % ws) and every step of 32 entries advances by (32 / ws, 32 % ws)
    int row = lane / ws, col = lane - (lane / ws) * ws;
    const int drow = 32 / ws, dcol = 32 - drow * ws;
    for (long long k = lane; k < cs; k += 32) {
      tiles[os + k] = (uint32_t)((ys + row) * tiles_x + xs + col);
      ids[os + k] = gs;
      row += drow;
      col += dcol;
      if (col >= ws) { col -= ws; ++row; }
    }
  }
}

// Per-tile [begin, end) of the sorted tile indices: each thread checks four
// consecutive entries (one 128-bit load plus its two neighbours) for boundaries.
__global__ void ranges_kernel(const uint32_t* tiles, int64_t n, const int64_t* n_dev, int2* ranges) {
  n = live_count(n, n_dev);
  const int64_t i0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (i0 >= n) return;
  constexpr uint32_t NONE = 0xffffffffu;  // never a tile index
  uint32_t t[6];
  t[0] = i0 > 0 ? tiles[i0 - 1] : NONE;
  if (i0 + 4 <= n) {
    const uint4 v = *reinterpret_cast<const uint4*>(tiles + i0);
    t[1] = v.x; t[2] = v.y; t[3] = v.z; t[4] = v.w;
  } else {
#pragma unroll
    for (int k = 0; k < 4; ++k) t[1 + k] = i0 + k < n ? tiles[i0 + k] : NONE;
  }
  t[5] = i0 + 4 < n ? tiles[i0 + 4] : NONE;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t cur = t[1 + k];
    if (cur == NONE) break;
    if (t[k] != cur) ranges[cur].x = (int)(i0 + k);
    if (t[k + 2] != cur) ranges[cur].y = (int)(i0 + k + 1);
  }
}

__global__ void keys_kernel(const int32_t* ids, const int2* ranges, const uint32_t* depth_key,
                            int n_tiles, uint64_t* keys) {
  const int t = blockIdx.x;
  if (t >= n_tiles) return;
  const int2 r = ranges[t];
  for (int i = r.x + threadIdx.x; i < r.y; i += blockDim.x)
    keys[i] = ((uint64_t)t << 32) | (uint64_t)depth_key[ids[i]];
}

inline unsigned grid_for(int64_t n, int per) { return (unsigned)((n + per - 1) / per); }

size_t align_up(size_t v) { return (v + 255) & ~(size_t)255; }

// workspace carving shared by bin_order / bin_emit
struct Carve {
  char* p;
  size_t used = 0;
  template <typename T> T* take(int64_t count) {
    T* r = reinterpret_cast<T*>(p ? p + used : nullptr);
    used += align_up((size_t)count * sizeof(T));
    return r;
  }
};

size_t order_bytes(int64_t n) {
  Carve c{nullptr};
  c.take<uint32_t>(n); c.take<int32_t>(n); c.take<uint32_t>(n); c.take<int32_t>(n);
  c.take<int32_t>(n);
  c.take<uint32_t>(RADIX * radix_blocks(n));
  c.take<uint32_t>(scan_blocks(RADIX * radix_blocks(n)) + 1);
  c.take<int64_t>(scan_blocks(n) + 1);
  return c.used;
}

size_t emit_bytes(int64_t m) {
  Carve c{nullptr};
  c.take<uint32_t>(m); c.take<int32_t>(m); c.take<uint32_t>(m); c.take<int32_t>(m);
  c.take<uint32_t>(RADIX * radix_blocks(m));
  c.take<uint32_t>(scan_blocks(RADIX * radix_blocks(m)) + 1);
  return c.used;
}

}  // namespace

size_t scan_workspace_bytes(int64_t n) { return align_up((size_t)(scan_blocks(n) + 1) * sizeof(int64_t)) + align_up((size_t)n * sizeof(int32_t)); }

cudaError_t scan_counts(const int32_t* in, int64_t n, int64_t* out, void* ws, size_t ws_bytes,
                        cudaStream_t s) {
  if (ws_bytes < align_up((size_t)(scan_blocks(n) + 1) * sizeof(int64_t))) return cudaErrorInvalidValue;
  return exclusive_scan<int32_t, int64_t>(in, n, out, reinterpret_cast<int64_t*>(ws), out + n, s);
}

size_t bin_workspace_bytes(int64_t n, int64_t n_isect, int n_tiles) {
  (void)n_tiles;
  const size_t a = order_bytes(n), b = emit_bytes(n_isect);
  return a > b ? a : b;
}

cudaError_t bin_order(const int32_t* count, const uint32_t* depth_key, int64_t n, int32_t* order,
                      int64_t* offsets, void* ws, size_t ws_bytes, cudaStream_t s) {
  if (ws_bytes < order_bytes(n)) return cudaErrorInvalidValue;
  if (n == 0) return cudaMemsetAsync(offsets, 0, sizeof(int64_t), s);
  Carve c{reinterpret_cast<char*>(ws)};
  uint32_t* kA = c.take<uint32_t>(n);
  int32_t* vA = c.take<int32_t>(n);
  uint32_t* kB = c.take<uint32_t>(n);
  int32_t* vB = c.take<int32_t>(n);
  int32_t* cs = c.take<int32_t>(n);
  RadixScratch sc;
  sc.hist = c.take<uint32_t>(RADIX * radix_blocks(n));
  sc.partial = c.take<uint32_t>(scan_blocks(RADIX * radix_blocks(n)) + 1);
  int64_t* spart = c.take<int64_t>(scan_blocks(n) + 1);
  count_launches(1);
  iota_copy_kernel<<<grid_for(n, 256), 256, 0, s>>>(depth_key, n, kA, vA);
  uint32_t* kf; int32_t* vf;
  cudaError_t e = radix_sort(kA, vA, kB, vB, n, 32, sc, &kf, &vf, nullptr, s);
  if (e != cudaSuccess) return e;
  count_launches(1);
  gather_counts_kernel<<<grid_for(n, 256), 256, 0, s>>>(vf, count, n, order, cs);
  return exclusive_scan<int32_t, int64_t>(cs, n, offsets, spart, offsets + n, s);
}

// m is the intersection count, or with `overflow` the capacity of the buffers: the count
// offsets[n] is then read on the device, and one above m emits nothing, leaves every
// tile range empty and sets *overflow.
cudaError_t bin_emit(const int32_t* order, const int64_t* offsets, const int32_t* rect, int64_t n,
                     int64_t m, int tiles_x, int n_tiles, int32_t* ids, int32_t* ranges, void* ws,
                     size_t ws_bytes, cudaStream_t s, int32_t* overflow) {
  if (ws_bytes < emit_bytes(m)) return cudaErrorInvalidValue;
  cudaError_t e = cudaMemsetAsync(ranges, 0, sizeof(int2) * (size_t)n_tiles, s);
  if (e != cudaSuccess || m == 0) return e;
  Carve c{reinterpret_cast<char*>(ws)};
  uint32_t* tA = c.take<uint32_t>(m);
  int32_t* vA = c.take<int32_t>(m);
  uint32_t* tB = c.take<uint32_t>(m);
  int32_t* vB = c.take<int32_t>(m);
  RadixScratch sc;
  sc.hist = c.take<uint32_t>(RADIX * radix_blocks(m));
  sc.partial = c.take<uint32_t>(scan_blocks(RADIX * radix_blocks(m)) + 1);
  count_launches(1);
  const int64_t* live = overflow ? offsets + n : nullptr;
  emit_kernel<<<grid_for(n, 256), 256, 0, s>>>(order, offsets, rect, n, tiles_x, m, overflow, tA, vA);
  int bits = 1;
  while ((1 << bits) < n_tiles) ++bits;
  uint32_t* kf; int32_t* vf;
  e = radix_sort(tA, vA, tB, vB, m, bits, sc, &kf, &vf, ids, s, live);
  if (e != cudaSuccess) return e;
  count_launches(1);
  ranges_kernel<<<grid_for((m + 3) / 4, 256), 256, 0, s>>>(kf, m, live, reinterpret_cast<int2*>(ranges));
  return cudaGetLastError();
}

size_t sort_pairs_workspace_bytes(int64_t n) {
  Carve c{nullptr};
  c.take<uint32_t>(n); c.take<int32_t>(n);
  c.take<uint32_t>(RADIX * radix_blocks(n));
  c.take<uint32_t>(scan_blocks(RADIX * radix_blocks(n)) + 1);
  return c.used;
}

cudaError_t sort_pairs(uint32_t* keys, int32_t* vals, int64_t n, int bits, void* ws, size_t ws_bytes,
                       cudaStream_t s) {
  if (ws_bytes < sort_pairs_workspace_bytes(n)) return cudaErrorInvalidValue;
  if (n == 0 || bits <= 0) return cudaSuccess;
  Carve c{reinterpret_cast<char*>(ws)};
  uint32_t* k1 = c.take<uint32_t>(n);
  int32_t* v1 = c.take<int32_t>(n);
  RadixScratch sc;
  sc.hist = c.take<uint32_t>(RADIX * radix_blocks(n));
  sc.partial = c.take<uint32_t>(scan_blocks(RADIX * radix_blocks(n)) + 1);
  uint32_t* kf;
  int32_t* vf;
  cudaError_t e = radix_sort(keys, vals, k1, v1, n, bits, sc, &kf, &vf, nullptr, s);
  if (e != cudaSuccess) return e;
  if (kf != keys) {
    e = cudaMemcpyAsync(keys, kf, (size_t)n * sizeof(uint32_t), cudaMemcpyDeviceToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(vals, vf, (size_t)n * sizeof(int32_t), cudaMemcpyDeviceToDevice, s);
  }
  return e;
}

cudaError_t key_ranges(const uint32_t* keys, int64_t n, int64_t n_keys, int32_t* ranges, cudaStream_t s) {
  cudaError_t e = cudaMemsetAsync(ranges, 0, sizeof(int2) * (size_t)n_keys, s);
  if (e != cudaSuccess || n == 0) return e;
  count_launches(1);
  ranges_kernel<<<grid_for((n + 3) / 4, 256), 256, 0, s>>>(keys, n, nullptr, reinterpret_cast<int2*>(ranges));
  return cudaGetLastError();
}

cudaError_t bin_keys(const int32_t* ids, const int32_t* ranges, const uint32_t* depth_key,
                     int n_tiles, int64_t m, uint64_t* keys, cudaStream_t s) {
  (void)m;
  if (n_tiles == 0) return cudaSuccess;
  count_launches(1);
  keys_kernel<<<n_tiles, 128, 0, s>>>(ids, reinterpret_cast<const int2*>(ranges), depth_key, n_tiles, keys);
  return cudaGetLastError();
}

}  // namespace sf
