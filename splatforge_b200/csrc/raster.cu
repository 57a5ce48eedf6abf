// Tile rasterizer: forward compositing, L1 resolve, reverse-order backward.
//
// One CTA per 16x16 tile, one thread per pixel.  Gaussian records of the tile's
// depth-ordered list are gathered in batches of 256 into shared memory (five 128-bit
// loads per 80-byte record) and evaluated by every pixel of the tile against the
// Torch provider's per-tile equations (src/splatforge/studio/batched_renderer.py:
// 240-338) with front-to-back alpha compositing (splat.alpha_composite@3,
// src/splatforge/providers/torch/gaussian/reference.py:151-186).
//
// There is no alpha threshold: every sample whose Mahalanobis distance passes
// squared <= extent^2 and near < depth < far contributes, exactly as in the
// reference.  A pixel stops once its transmittance is below settings.t_stop; the
// remaining samples could add at most t_stop to any weight sum.
#include <cuda_runtime.h>

#include "sf_device.cuh"
#include "sf_grad.cuh"
#include "sf_kernels.h"

namespace sf {

namespace {

constexpr int REC4 = SF_RECORD_FLOATS / 4;  // float4 per record
// Records staged per shared-memory batch (forward, backward); build-time parameters.
#ifndef SF_FWD_BATCH
#define SF_FWD_BATCH 384
#endif
#ifndef SF_BWD_BATCH
#define SF_BWD_BATCH 256
#endif

// resident CTAs per SM the forward is compiled for (register budget 65536 / (256 x this))
#ifndef SF_FWD_MIN_CTAS
#define SF_FWD_MIN_CTAS 4
#endif
// forward record access: 1 = each warp walks the tile list on its own and stages its
// hits' records in its shared-memory slice, 0 = CTA batches of FWD_BATCH records
#ifndef SF_FWD_WARP_WALK
#define SF_FWD_WARP_WALK 1
#endif
// backward record access: 1 = each warp walks the tile list on its own (records read
// through L1, sums added straight to global memory), 0 = batches staged in shared memory
#ifndef SF_BWD_WARP_WALK
#define SF_BWD_WARP_WALK 1
#endif
// with the walk: 1 = each group's hit records staged in the warp's own shared-memory
// slice, 0 = read from global memory at every use
#ifndef SF_BWD_WARP_STAGE
#define SF_BWD_WARP_STAGE 1
#endif
// with the walk: 1 = each lane loads its entry's Gaussian id for the next 32-entry
// group while the current group is evaluated (one dependent load fewer per group).
// Measured at C3: forward 3.085 -> 3.037 ms (on); backward 5.76 -> 5.80 ms (off: the
// extra live register adds spills at its 80-register budget)
#ifndef SF_FWD_PREFETCH_IDS
#define SF_FWD_PREFETCH_IDS 1
#endif
#ifndef SF_BWD_PREFETCH_IDS
#define SF_BWD_PREFETCH_IDS 0
#endif
// resident CTAs per SM the backward is compiled for (2: 103 registers without spills,
// measured 5.76 -> 6.24 ms at C3)
#ifndef SF_BWD_MIN_CTAS
#define SF_BWD_MIN_CTAS 3
#endif

constexpr int FWD_BATCH = SF_FWD_BATCH;
constexpr int BWD_BATCH = SF_BWD_BATCH;
static_assert(FWD_BATCH % 32 == 0 && BWD_BATCH % 32 == 0, "batches are whole culling groups");
constexpr int ACC = 24;                      // accumulator floats per batch slot (20 + absgrad 2 + pad)
// The backward's per-batch accumulator covers record slots [BASE, 24) of each Gaussian:
// GOF never produces adjoints for slots 0-3 (xy and the 2D conic), so its accumulator
// starts at slot 4 and is 20 floats (5 float4) wide; the other modes use all 24.
template <int MODE> struct AccWindow {
  static constexpr int BASE = MODE == SF_MODE_GOF ? 4 : 0;
  static constexpr int N = ACC - BASE;
};

// first slot of a pixel's contiguous L1 sample run (fixed capacity or CSR); ptid is
// the row-major index of the pixel inside its tile
__device__ __forceinline__ int64_t l1_base(int tile, int ptid, int cap, const int64_t* off, int64_t pix) {
  return off ? off[pix] : ((int64_t)tile * TILE_PIXELS + ptid) * cap;
}

// Pixel of thread tid: each warp covers an 8x4 block of its 16x16 tile (warps 0,1 the
// top two blocks side by side, ...), a more compact footprint than 16x2 rows, so fewer
// Gaussians reach a warp's box without reaching one of its pixels.
__device__ __forceinline__ void tile_pixel(int tid, int tx, int ty, int& u, int& v, int& ptid) {
  const int w = tid >> 5, lane = tid & 31;
  const int lx = (w & 1) * 8 + (lane & 7), ly = (w >> 1) * 4 + (lane >> 3);
  u = tx * TILE + lx;
  v = ty * TILE + ly;
  ptid = ly * TILE + lx;  // row-major index of the pixel inside its tile
}

#if !(SF_FWD_WARP_WALK && SF_BWD_WARP_WALK)
// Warp-level culling of batch slots g*32 .. g*32+31: bit l is set when the Gaussian in
// slot g*32+l may pass squared <= extent^2 at a pixel of this warp (box_may_pass over
// the box spanned by the warp's pixel centres).
__device__ __forceinline__ unsigned warp_cull(const float4* s_rec, int n_in, int g, int lane, float x0, float x1,
                                              float y0, float y1, float ext2) {
  const int j = g * 32 + lane;
  bool hit = false;
  if (j < n_in) {
    const float* rec = reinterpret_cast<const float*>(&s_rec[j * REC4]);
    hit = box_may_pass(rec[R_QA], rec[R_QB], rec[R_QC], rec[R_X], rec[R_Y], x0, x1, y0, y1, ext2);
  }
  return __ballot_sync(FULL, hit);
}
#endif

__device__ __forceinline__ float warp_minf(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(FULL, v, o));
  return v;
}
__device__ __forceinline__ float warp_maxf(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL, v, o));
  return v;
}

// ------------------------------------------------------------------ forward
// L1 samples are staged per pixel in an 8-deep shared-memory ring and written out 8 at
// a time as two 16-byte stores per column: a full 32-byte sector of depths and one of
// weights, instead of sixteen 4-byte stores that each touch their own sector.  Runs
// start on 8-float boundaries (fixed capacities are multiples of 32; CSR runs are
// rounded up to multiples of 8); an unaligned caller layout takes scalar stores.
constexpr int L1_RING = 8;

__device__ __forceinline__ void l1_flush(float* l1s, int64_t slots, int64_t at, int first, int count, int room,
                                         bool vec_ok, const float (*ring)[L1_RING][TILE_PIXELS], int tid) {
  if (vec_ok && count == L1_RING && first + L1_RING <= room) {
    float4* d = reinterpret_cast<float4*>(l1s + at + first);
    float4* w = reinterpret_cast<float4*>(l1s + slots + at + first);
    d[0] = make_float4(ring[0][0][tid], ring[0][1][tid], ring[0][2][tid], ring[0][3][tid]);
    d[1] = make_float4(ring[0][4][tid], ring[0][5][tid], ring[0][6][tid], ring[0][7][tid]);
    w[0] = make_float4(ring[1][0][tid], ring[1][1][tid], ring[1][2][tid], ring[1][3][tid]);
    w[1] = make_float4(ring[1][4][tid], ring[1][5][tid], ring[1][6][tid], ring[1][7][tid]);
  } else {
    for (int i = 0; i < count; ++i) {
      if (first + i < room) {
        l1s[at + first + i] = ring[0][i][tid];
        l1s[slots + at + first + i] = ring[1][i][tid];
      }
    }
  }
}

template <int MODE, int DIST>
__global__ void __launch_bounds__(TILE_PIXELS, SF_FWD_MIN_CTAS) raster_forward_kernel(const RasterFwdArgs a) {
  extern __shared__ float4 s_dyn[];  // the batch's records: FWD_BATCH * REC4 float4
  float4* s_rec = s_dyn;
  __shared__ float s_ring[(DIST & SF_DIST_L1) ? 2 : 1][L1_RING][TILE_PIXELS];
  __shared__ int s_max;
  const int tile = blockIdx.x;
  const int tid = threadIdx.x;
  const int tx = tile % a.tiles_x, ty = tile / a.tiles_x;
  int u, v, ptid;
  tile_pixel(tid, tx, ty, u, v, ptid);
  const int W = a.cam.width, H = a.cam.height;
  const bool inside = u < W && v < H;
  PixelRay pr;
  pixel_ray(a.cam, u, v, pr);
  const float wx0 = warp_minf(pr.px), wx1 = warp_maxf(pr.px);
  const float wy0 = warp_minf(pr.py), wy1 = warp_maxf(pr.py);
  const int2 rg = a.ranges[tile];
  const float ext2 = a.st.extent_sq, nearp = a.st.near_plane, farp = a.st.far_plane;
  const double t_stop = (double)a.st.t_stop;
  double Td = 1.0, Wd = 0.0;
  float C0 = 0.f, C1 = 0.f, C2 = 0.f, D = 0.f, N0 = 0.f, N1 = 0.f, N2 = 0.f;
  // L2 = 2 (W sum w d^2 - (sum w d)^2) cancels when the depths are large and close
  // (AmbiSuR plane depths at grazing angles): its moments accumulate in double
  double L2d1 = 0.0, L2d2 = 0.0;
  float Dn = 0.f, A = 0.f, Scc = 0.f, med_depth = 0.f;
  int last = rg.x, med = -1, cnt = 0, evaluated = 0;
  bool done = !inside;
  const int64_t pix = (int64_t)v * W + u;
  int64_t l1_at = 0;
  int l1_room = 0;
  bool l1_vec = false;
  if ((DIST & SF_DIST_L1) && inside) {
    l1_at = l1_base(tile, ptid, a.l1_cap, a.l1_off, pix);
    l1_room = a.l1_off ? (int)(a.l1_off[pix + 1] - a.l1_off[pix]) : a.l1_cap;
    l1_vec = ((l1_at | a.l1_slots) & 3) == 0 && (reinterpret_cast<uintptr_t>(a.l1s) & 15) == 0;
  }
  if (tid == 0) s_max = 0;
  __syncthreads();

#if SF_FWD_WARP_WALK
  // Each warp walks the tile's list on its own, 32 entries at a time: lane l tests
  // entry l against the warp's box, each passing lane copies its record into the warp's
  // own slice of shared memory, and the hits are evaluated from there.  No CTA barrier:
  // a warp never waits for a slower one and stops when its own pixels are done.
  {
    const int lane = tid & 31;
    float4* const s_w = s_rec + (tid >> 5) * 32 * REC4;
#if SF_FWD_PREFETCH_IDS
    int gid_next = rg.x + lane < rg.y ? __ldg(a.ids + rg.x + lane) : 0;
#endif
    for (int base = rg.x; base < rg.y; base += 32) {
      if (__all_sync(FULL, done)) break;
#if SF_FWD_PREFETCH_IDS
      const int gid_cur = gid_next;
      if (base + 32 + lane < rg.y) gid_next = __ldg(a.ids + base + 32 + lane);
#endif
      bool hit = false;
      if (base + lane < rg.y) {
#if SF_FWD_PREFETCH_IDS
        const int gid = gid_cur;
#else
        const int gid = __ldg(a.ids + base + lane);
#endif
        const float4* src = reinterpret_cast<const float4*>(a.records) + (int64_t)gid * REC4;
        const float4 w0 = __ldg(src);
        const float qc = __ldg(a.records + (int64_t)gid * SF_RECORD_FLOATS + R_QC);
        hit = box_may_pass(w0.z, w0.w, qc, w0.x, w0.y, wx0, wx1, wy0, wy1, ext2);
        if (hit) {
          float4* dst = s_w + lane * REC4;
          dst[0] = w0;
#pragma unroll
          for (int c = 1; c < REC4; ++c) dst[c] = __ldg(src + c);
        }
      }
      unsigned m = __ballot_sync(FULL, hit);
      __syncwarp();
      while (m) {
        const int j = __ffs(m) - 1;
        m &= m - 1;
        if (done) continue;
        const float* rec = reinterpret_cast<const float*>(&s_w[j * REC4]);
#else
  for (int base = rg.x; base < rg.y; base += FWD_BATCH) {
    if (__syncthreads_count(done) == TILE_PIXELS) break;
    const int n_in = min(FWD_BATCH, rg.y - base);
    for (int k = tid; k < n_in * REC4; k += TILE_PIXELS) {
      const int slot = k / REC4, comp = k - slot * REC4;
      const int id = __ldg(a.ids + base + slot);
      s_rec[k] = __ldg(reinterpret_cast<const float4*>(a.records) + (int64_t)id * REC4 + comp);
    }
    __syncthreads();
    const int groups = (n_in + 31) >> 5;
    for (int g = 0; g < groups; ++g) {
      if (__all_sync(FULL, done)) break;
      unsigned m = warp_cull(s_rec, n_in, g, tid & 31, wx0, wx1, wy0, wy1, ext2);
      while (m) {
        const int j = g * 32 + __ffs(m) - 1;
        m &= m - 1;
        if (done) continue;
        const float* rec = reinterpret_cast<const float*>(&s_rec[j * REC4]);
#endif
        Sample s;
        ++evaluated;
        if (!eval_sample<MODE>(rec, pr, ext2, nearp, farp, s)) continue;
        const int pos = base + j;
        const float w = s.alpha * (float)Td;
        const float c0 = rec[R_RGB], c1 = rec[R_RGB + 1], c2 = rec[R_RGB + 2];
        C0 += w * c0; C1 += w * c1; C2 += w * c2;
        D += w * s.depth;
        if (DIST & SF_DIST_L2) {
          const double wd = (double)w * (double)s.depth;
          L2d1 += wd;
          L2d2 += wd * (double)s.depth;
        }
        N0 += w * s.n[0]; N1 += w * s.n[1]; N2 += w * s.n[2];
        A += w * rec[R_SEL];
        if (MODE == SF_MODE_AMBISUR) {
          Dn += w * rec[R_PLANE];
          Scc += w * (c0 * c0 + c1 * c1 + c2 * c2);
        }
        Wd += (double)w;
        if (med < 0 && (float)Wd >= 0.5f) { med = pos; med_depth = s.depth; }
        if (DIST & SF_DIST_L1) {
          const int slot = cnt & (L1_RING - 1);
          s_ring[0][slot][tid] = s.depth;
          s_ring[(DIST & SF_DIST_L1) ? 1 : 0][slot][tid] = w;
          if (slot == L1_RING - 1)
            l1_flush(a.l1s, a.l1_slots, l1_at, cnt - (L1_RING - 1), L1_RING, l1_room, l1_vec, s_ring, tid);
        }
        ++cnt;
        last = pos + 1;
        Td *= (double)(1.f - s.alpha);
        if (Td < t_stop) done = true;
      }
#if SF_FWD_WARP_WALK
      __syncwarp();  // the slice is read before the next group overwrites it
#endif
    }
  }

  if ((DIST & SF_DIST_L1) && inside && (cnt & (L1_RING - 1)))
    l1_flush(a.l1s, a.l1_slots, l1_at, cnt & ~(L1_RING - 1), cnt & (L1_RING - 1), l1_room, l1_vec, s_ring, tid);
  if (inside) {
    const float Wf = (float)Wd;
    const float* bg = a.st.background;
    const int64_t p3 = pix * 3;
    a.rgb[p3 + 0] = C0 + (1.f - Wf) * bg[0];
    a.rgb[p3 + 1] = C1 + (1.f - Wf) * bg[1];
    a.rgb[p3 + 2] = C2 + (1.f - Wf) * bg[2];
    a.alpha[pix] = Wf;
    float expected = D / fmaxr(Wf, 1e-8f);
    if (MODE == SF_MODE_AMBISUR) {
      const float den = N0 * pr.r[0] + N1 * pr.r[1] + N2 * pr.r[2];
      expected = fabsf(den) > 1e-8f ? Dn / den : 0.f;
    }
    a.depth[pix] = Wf > 1e-8f ? expected : 0.f;
    const float nn = fmaxr(sqrtf(N0 * N0 + N1 * N1 + N2 * N2), 1e-12f);
    a.normals[p3 + 0] = N0 / nn;
    a.normals[p3 + 1] = N1 / nn;
    a.normals[p3 + 2] = N2 / nn;
    const float raw_l2 = (DIST & SF_DIST_L2) ? (float)(2.0 * (Wd * L2d2 - L2d1 * L2d1)) : 0.f;
    a.l2[pix] = fmaxr(raw_l2, 0.f);
    if (!(DIST & SF_DIST_L1)) a.l1[pix] = 0.f;
    a.median[pix] = med >= 0 ? med_depth : 0.f;
    a.ray_color[pix] =
        MODE == SF_MODE_AMBISUR ? Scc - 2.f * (C0 * C0 + C1 * C1 + C2 * C2) + (C0 * C0 + C1 * C1 + C2 * C2) * Wf : 0.f;
    a.amb[pix] = A;
    float* st = a.state + pix * SF_PIXEL_STATE_FLOATS;
    st[PS_T] = (float)Td;
    st[PS_W] = Wf;
    st[PS_D] = D;
    st[PS_D2] = (float)L2d2;
    st[PS_C] = C0; st[PS_C + 1] = C1; st[PS_C + 2] = C2;
    st[PS_N] = N0; st[PS_N + 1] = N1; st[PS_N + 2] = N2;
    st[PS_DNUM] = Dn;
    st[PS_L1] = 0.f;
    st[PS_L2] = raw_l2;
    st[PS_LAST] = i2f(last);
    st[PS_MEDIAN] = i2f(med);
    st[PS_COUNT] = i2f(cnt);
  }
  if ((DIST & SF_DIST_L1) && a.l1_needed) {
    const int m = warp_max(cnt);
    if ((tid & 31) == 0) atomicMax(&s_max, m);
    __syncthreads();
    if (tid == 0) atomicMax(a.l1_needed, s_max);
  }
  if (a.counters) {
    unsigned long long e = (unsigned long long)evaluated, c = (unsigned long long)cnt;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      e += __shfl_xor_sync(FULL, e, o);
      c += __shfl_xor_sync(FULL, c, o);
    }
    if ((tid & 31) == 0) {
      atomicAdd(a.counters, e);
      atomicAdd(a.counters + 1, c);
    }
  }
}

// ------------------------------------------------------------------ L1 resolve
// One warp per pixel.  The pixel's samples (depth, weight; compositing order) are
// staged in shared memory and sorted by depth with a stable warp-level LSD radix sort
// on the float bits (positive depths order like their bit patterns; bytes that are
// equal for every sample are skipped), then prefix sums of w and w*d in depth order
// give
//   L1     = sum_i 2 w_i (d_i W_<i - D_<i)
//   auxw_i = 2 (2 d_i W_<i - d_i W + D - 2 D_<i)     (dL1/dw_i)
//   auxd_i = 2 w_i (2 W_<i + w_i - W)                 (dL1/dd_i)
// (composite_cuda.cu:54-65 computes the same factors from torch's sort order).  The
// two factors replace (d_i, w_i) in place, written back contiguously.
// Register bitonic sort of one pixel's n <= 32*I samples, I per lane in blocked layout
// (lane l holds sorted positions l*I .. l*I+I-1); strides below I are compare-exchanges
// inside a lane, larger strides exchange with lane ^ (stride / I) by shuffle.  Ties are
// ordered by compositing index.  Then the sorted prefix sums, the L1 value and the two
// factors per sample, written back in place (by compositing index) once every lane has
// read its originals.  Returns this lane's share of the raw L1.
template <int I>
__device__ __noinline__ float l1_sort_pixel(float* col_d, float* col_w, int64_t base, int n, int lane) {
  constexpr int NN = 32 * I;
  // key = depth bits (positive depths order like their bit patterns) : sample index;
  // padding sorts last
  unsigned long long key[I];
#pragma unroll
  for (int j = 0; j < I; ++j) {
    const int e = lane * I + j;
    key[j] = e < n ? ((unsigned long long)__float_as_uint(col_d[base + e]) << 32) | (unsigned)e : ~0ull;
  }
  // sizes up to I sort inside each lane (directions known at compile time) ...
#pragma unroll
  for (int size = 2; size <= I; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
#pragma unroll
      for (int j = 0; j < I; ++j) {
        if ((j & stride) == 0) {
          const bool up = ((lane * I + j) & size) == 0;
          const unsigned long long a = key[j], b = key[j + stride];
          const bool sw = up ? (b < a) : (a < b);
          key[j] = sw ? b : a;
          key[j + stride] = sw ? a : b;
        }
      }
    }
  }
  // ... then each larger merge: the cross-lane strides in a rolled loop (exchange with
  // lane ^ (stride / I)), the last log2(I) strides inside the lane.  The rolled loops
  // keep the code small enough for the instruction cache.
#pragma unroll 1
  for (int size = 2 * I; size <= NN; size <<= 1) {
    const bool up = ((lane * I) & size) == 0;
#pragma unroll 1
    for (int lm = size / (2 * I); lm > 0; lm >>= 1) {
      const bool take_min = ((lane & lm) == 0) == up;
#pragma unroll
      for (int j = 0; j < I; ++j) {
        const unsigned long long o = __shfl_xor_sync(FULL, key[j], lm);
        const bool mine_less = key[j] < o;
        key[j] = (take_min == mine_less) ? key[j] : o;
      }
    }
#pragma unroll
    for (int stride = I >> 1; stride > 0; stride >>= 1) {
#pragma unroll
      for (int j = 0; j < I; ++j) {
        if ((j & stride) == 0) {
          const unsigned long long a = key[j], b = key[j + stride];
          const bool sw = up ? (b < a) : (a < b);
          key[j] = sw ? b : a;
          key[j + stride] = sw ? a : b;
        }
      }
    }
  }
  float w[I];
  float lw = 0.f, lwd = 0.f;
#pragma unroll
  for (int j = 0; j < I; ++j) {
    const unsigned k = (unsigned)key[j];
    const bool live = key[j] != ~0ull;
    w[j] = live ? col_w[base + k] : 0.f;
    lw += w[j];
    lwd += w[j] * (live ? __uint_as_float((unsigned)(key[j] >> 32)) : 0.f);
  }
  // totals and exclusive lane offsets of w and w*d in depth order
  float iw = lw, iwd = lwd;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float a1 = __shfl_up_sync(FULL, iw, o), a2 = __shfl_up_sync(FULL, iwd, o);
    if (lane >= o) { iw += a1; iwd += a2; }
  }
  const float Wt = __shfl_sync(FULL, iw, 31), Dt = __shfl_sync(FULL, iwd, 31);
  float pw = iw - lw, pwd = iwd - lwd;
  float raw = 0.f;
  __syncwarp();  // every lane has read its originals
#pragma unroll
  for (int j = 0; j < I; ++j) {
    if (key[j] != ~0ull) {
      const unsigned k = (unsigned)key[j];
      const float d = __uint_as_float((unsigned)(key[j] >> 32));
      raw += 2.f * w[j] * (d * pw - pwd);
      col_d[base + k] = 2.f * (2.f * d * pw - d * Wt + Dt - 2.f * pwd);
      col_w[base + k] = 2.f * w[j] * (2.f * pw + w[j] - Wt);
      pw += w[j];
      pwd += w[j] * d;
    }
  }
  return raw;
}

// The same resolve with 32-bit keys: key = ((depth bits - smallest depth bits) << LOGN)
// | compositing index, LOGN = log2(32 I).  Depths of contributing samples are positive
// and finite, so their bit patterns order like their values; when the pixel's span of
// depth bit patterns fits in 32 - LOGN bits (for 256 samples: max/min depth ratio
// below about 4), the packed keys are exact, unique and order like (depth, index),
// and the network needs no payload: unsigned min/max only.  Returns false (nothing
// written) when the span does not fit; the caller then runs the 64-bit path.
//
// The pixel's depths and weights arrive in one round of 16-byte loads in blocked layout
// (lane l holds samples l*I .. l*I+I-1); the weights are parked in the warp's slice of
// shared memory (s_w) by compositing index, so that after the sort each lane reads the
// weights of its sorted samples there instead of from global memory; the two factors
// are assembled in s_w / s_o by compositing index and leave in blocked layout.  A float4
// is loaded or stored only when it starts below n: runs start on 8-sample boundaries and
// their room is a multiple of 8, so it never leaves the pixel's run.
template <int I>
__device__ __forceinline__ void l1_load_run(const float* col, int64_t base, int n, int lane, bool vec, float (&v)[I]) {
  if constexpr (I == 2) {  // one 8-byte load per lane
    const int e0 = lane * 2;
    float2 x = make_float2(0.f, 0.f);
    if (e0 < n) {
      if (vec) {
        x = *reinterpret_cast<const float2*>(col + base + e0);
      } else {
        x.x = col[base + e0];
        x.y = e0 + 1 < n ? col[base + e0 + 1] : 0.f;
      }
    }
    v[0] = x.x;
    v[1] = x.y;
  } else {
#pragma unroll
    for (int q = 0; q < I / 4; ++q) {
      const int e0 = lane * I + 4 * q;
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (e0 < n) {
        if (vec) {
          x = *reinterpret_cast<const float4*>(col + base + e0);
        } else {
          x.x = col[base + e0];
          x.y = e0 + 1 < n ? col[base + e0 + 1] : 0.f;
          x.z = e0 + 2 < n ? col[base + e0 + 2] : 0.f;
          x.w = e0 + 3 < n ? col[base + e0 + 3] : 0.f;
        }
      }
      v[4 * q] = x.x; v[4 * q + 1] = x.y; v[4 * q + 2] = x.z; v[4 * q + 3] = x.w;
    }
  }
}

template <int I>
__device__ __forceinline__ void l1_store_run(float* col, int64_t base, int n, int lane, bool vec, const float* s) {
  if constexpr (I == 2) {
    const int e0 = lane * 2;
    if (e0 < n) {
      const float2 x = *reinterpret_cast<const float2*>(s + e0);
      if (vec && e0 + 2 <= n) {
        *reinterpret_cast<float2*>(col + base + e0) = x;
      } else {
        col[base + e0] = x.x;
        if (e0 + 1 < n) col[base + e0 + 1] = x.y;
      }
    }
  } else {
#pragma unroll
    for (int q = 0; q < I / 4; ++q) {
      const int e0 = lane * I + 4 * q;
      if (e0 >= n) continue;
      const float4 x = *reinterpret_cast<const float4*>(s + e0);
      if (vec && e0 + 4 <= n) {
        *reinterpret_cast<float4*>(col + base + e0) = x;
      } else {
        col[base + e0] = x.x;
        if (e0 + 1 < n) col[base + e0 + 1] = x.y;
        if (e0 + 2 < n) col[base + e0 + 2] = x.z;
        if (e0 + 3 < n) col[base + e0 + 3] = x.w;
      }
    }
  }
}

template <int I>
__device__ __forceinline__ bool l1_sort_pixel_packed(float* col_d, float* col_w, int64_t base, int n, int lane,
                                                     bool vec, float* s_w, float* s_o, float& raw_out) {
  constexpr int NN = 32 * I;
  constexpr int LOGN = (NN == 64) ? 6 : (NN == 128) ? 7 : (NN == 256 ? 8 : 9);
  static_assert(NN == (1 << LOGN), "power of two");
  uint32_t key[I];
  uint32_t lo = 0xffffffffu, hi = 0u;
  {
    float dv[I], wv[I];
    l1_load_run<I>(col_d, base, n, lane, vec, dv);
    l1_load_run<I>(col_w, base, n, lane, vec, wv);
#pragma unroll
    for (int j = 0; j < I; ++j) {
      const int e = lane * I + j;
      key[j] = e < n ? __float_as_uint(dv[j]) : 0u;
      if (e < n) { lo = min(lo, key[j]); hi = max(hi, key[j]); }
    }
    if constexpr (I == 2) {
      *reinterpret_cast<float2*>(s_w + lane * 2) = make_float2(wv[0], wv[1]);
    } else {
#pragma unroll
      for (int q = 0; q < I / 4; ++q)
        *reinterpret_cast<float4*>(s_w + lane * I + 4 * q) =
            make_float4(wv[4 * q], wv[4 * q + 1], wv[4 * q + 2], wv[4 * q + 3]);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lo = min(lo, __shfl_xor_sync(FULL, lo, o));
    hi = max(hi, __shfl_xor_sync(FULL, hi, o));
  }
  if (hi - lo >= (1u << (32 - LOGN))) return false;  // warp-uniform
#pragma unroll
  for (int j = 0; j < I; ++j) {
    const int e = lane * I + j;
    // padding sorts last: a real key is at most (2^(32-LOGN) - 1) << LOGN | (n - 1),
    // and n - 1 < NN - 1 whenever there is padding
    key[j] = e < n ? ((key[j] - lo) << LOGN) | (uint32_t)e : 0xffffffffu;
  }
  // Bitonic sort in its all-ascending form: each merge of size s first compares
  // position p with its mirror p ^ (s - 1), then runs half-cleaners p vs p ^ t for
  // t = s/4 .. 1, the lower position always taking the minimum, so compare-exchanges
  // inside a lane need no direction select.  Position p = lane * I + j; the mirror of
  // (lane, j) is (lane ^ (s/I - 1), I - 1 - j) once s > I.
#pragma unroll
  for (int size = 2; size <= I; size <<= 1) {
#pragma unroll
    for (int j = 0; j < I; ++j) {
      const int m = j ^ (size - 1);
      if (j < m) {
        const uint32_t a = min(key[j], key[m]), b = max(key[j], key[m]);
        key[j] = a;
        key[m] = b;
      }
    }
#pragma unroll
    for (int stride = size >> 2; stride > 0; stride >>= 1) {
#pragma unroll
      for (int j = 0; j < I; ++j) {
        if ((j & stride) == 0) {
          const uint32_t a = min(key[j], key[j + stride]), b = max(key[j], key[j + stride]);
          key[j] = a;
          key[j + stride] = b;
        }
      }
    }
  }
#pragma unroll 1
  for (int size = 2 * I; size <= NN; size <<= 1) {
    {
      const int lm = size / I - 1;
      const bool take_min = (lane & (size / (2 * I))) == 0;
#pragma unroll
      for (int j = 0; j < I / 2; ++j) {
        const uint32_t o1 = __shfl_xor_sync(FULL, key[I - 1 - j], lm);
        const uint32_t o2 = __shfl_xor_sync(FULL, key[j], lm);
        key[j] = take_min ? min(key[j], o1) : max(key[j], o1);
        key[I - 1 - j] = take_min ? min(key[I - 1 - j], o2) : max(key[I - 1 - j], o2);
      }
    }
#pragma unroll 1
    for (int ls = size / (4 * I); ls > 0; ls >>= 1) {
      const bool take_min = (lane & ls) == 0;
#pragma unroll
      for (int j = 0; j < I; ++j) {
        const uint32_t o = __shfl_xor_sync(FULL, key[j], ls);
        key[j] = take_min ? min(key[j], o) : max(key[j], o);
      }
    }
#pragma unroll
    for (int stride = I >> 1; stride > 0; stride >>= 1) {
#pragma unroll
      for (int j = 0; j < I; ++j) {
        if ((j & stride) == 0) {
          const uint32_t a = min(key[j], key[j + stride]), b = max(key[j], key[j + stride]);
          key[j] = a;
          key[j + stride] = b;
        }
      }
    }
  }
  float w[I];
  float lw = 0.f, lwd = 0.f;
  __syncwarp();  // s_w holds every lane's weights
#pragma unroll
  for (int j = 0; j < I; ++j) {
    const bool live = key[j] != 0xffffffffu;
    w[j] = live ? s_w[key[j] & (NN - 1)] : 0.f;
    lw += w[j];
    lwd += w[j] * (live ? __uint_as_float((key[j] >> LOGN) + lo) : 0.f);
  }
  float iw = lw, iwd = lwd;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float a1 = __shfl_up_sync(FULL, iw, o), a2 = __shfl_up_sync(FULL, iwd, o);
    if (lane >= o) { iw += a1; iwd += a2; }
  }
  const float Wt = __shfl_sync(FULL, iw, 31), Dt = __shfl_sync(FULL, iwd, 31);
  float pw = iw - lw, pwd = iwd - lwd;
  float raw = 0.f;
  __syncwarp();  // every lane has read its weights from s_w
#pragma unroll
  for (int j = 0; j < I; ++j) {
    if (key[j] != 0xffffffffu) {
      const uint32_t k = key[j] & (NN - 1);
      const float d = __uint_as_float((key[j] >> LOGN) + lo);
      raw += 2.f * w[j] * (d * pw - pwd);
      s_o[k] = 2.f * (2.f * d * pw - d * Wt + Dt - 2.f * pwd);
      s_w[k] = 2.f * w[j] * (2.f * pw + w[j] - Wt);
      pw += w[j];
      pwd += w[j] * d;
    }
  }
  __syncwarp();  // both factors assembled by compositing index
  l1_store_run<I>(col_d, base, n, lane, vec, s_o);
  l1_store_run<I>(col_w, base, n, lane, vec, s_w);
  __syncwarp();  // s_w / s_o free for the warp's next pixel
  raw_out = raw;
  return true;
}

// CLASS 0 resolves pixels with at most 256 samples (register sorts), CLASS 1 those
// with 257..512 (16 per lane); each launch skips the pixels of the other classes, so the
// register budget of the rarer long runs does not limit the occupancy of the common case.
// Longer runs go to l1_resolve_long_kernel.
template <int CLASS>
#ifndef SF_RESOLVE0_MIN_CTAS
#define SF_RESOLVE0_MIN_CTAS 7  // 72 registers (7 CTAs of 4 warps per SM)
#endif
#ifndef SF_RESOLVE1_MIN_CTAS
#define SF_RESOLVE1_MIN_CTAS 4  // 128 registers
#endif
__global__ void __launch_bounds__(128, CLASS == 0 ? SF_RESOLVE0_MIN_CTAS : SF_RESOLVE1_MIN_CTAS) l1_resolve_kernel(
    sf_camera cam, float* state, float* l1s, int64_t slots, const int64_t* off, int cap, int smem_k,
    float* out_l1) {
  (void)smem_k;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int warps = blockDim.x >> 5;

  const int64_t npix = (int64_t)cam.width * cam.height;
  const int tiles_x = (cam.width + TILE - 1) / TILE;
  float* col_d = l1s;
  float* col_w = l1s + slots;
  // per warp: weights parked by compositing index, and the second output column
  constexpr int NMAX = CLASS == 0 ? 256 : 512;
  __shared__ __align__(16) float s_stage[CLASS == 2 ? 1 : 4][CLASS == 2 ? 1 : 2 * NMAX];
  float* s_w = s_stage[CLASS == 2 ? 0 : wid];
  float* s_o = s_w + (CLASS == 2 ? 0 : NMAX);
  // 16-byte loads and stores need aligned columns (runs start on 8-sample boundaries)
  const bool vec = ((reinterpret_cast<uintptr_t>(l1s) | (uintptr_t)(slots * sizeof(float))) & 15) == 0;
  // Pixels go to warps in groups of 32: lane l of group g reads the sample count and
  // run start of pixel g + l G (G groups, so a group's pixels lie spread over the frame
  // and a cluster of long runs spreads over many warps), a ballot picks the group's
  // pixels of this class, and the warp resolves them one after another with their
  // counts already in registers: one load latency per 32 pixels, where a launch that
  // skips most pixels (the longer classes) would otherwise wait once per pixel.
  const int64_t groups = (npix + 31) >> 5;
  for (int64_t g = (int64_t)blockIdx.x * warps + wid; g < groups; g += (int64_t)gridDim.x * warps) {
    const int64_t mine = g + lane * groups;
    int my_n = 0;
    int64_t my_base = 0;
    bool here = false;
    if (mine < npix) {
      my_n = f2i(state[mine * SF_PIXEL_STATE_FLOATS + PS_COUNT]);
      const int u = (int)(mine % cam.width), v = (int)(mine / cam.width);
      const int tile = (v / TILE) * tiles_x + (u / TILE);
      const int tid = (v % TILE) * TILE + (u % TILE);
      my_base = l1_base(tile, tid, cap, off, mine);
      // never read past the pixel's run (a capacity overflow is rerun by the caller)
      const int room = off ? (int)(off[mine + 1] - off[mine]) : cap;
      if (my_n > room) my_n = room;
      here = (my_n <= 256 ? 0 : (my_n <= 512 ? 1 : 2)) == CLASS;
      if (CLASS == 0 && here && my_n <= 1) {
        // nothing to sort: the lane writes its own pixel's outputs
        if (my_n == 1) { col_d[my_base] = 0.f; col_w[my_base] = 0.f; }
        state[mine * SF_PIXEL_STATE_FLOATS + PS_L1] = 0.f;
        out_l1[mine] = 0.f;
        here = false;
      }
    }
    unsigned todo = __ballot_sync(FULL, here);
    while (todo) {
      const int l = __ffs(todo) - 1;
      todo &= todo - 1;
      const int64_t pix = g + l * groups;
      const int n = __shfl_sync(FULL, my_n, l);
      const int64_t base = __shfl_sync(FULL, my_base, l);
      float raw = 0.f;
      if (CLASS == 0) {
        if (n <= 64) {
          if (!l1_sort_pixel_packed<2>(col_d, col_w, base, n, lane, vec, s_w, s_o, raw))
            raw = l1_sort_pixel<2>(col_d, col_w, base, n, lane);
        } else if (n <= 128) {
          if (!l1_sort_pixel_packed<4>(col_d, col_w, base, n, lane, vec, s_w, s_o, raw))
            raw = l1_sort_pixel<4>(col_d, col_w, base, n, lane);
        } else {
          if (!l1_sort_pixel_packed<8>(col_d, col_w, base, n, lane, vec, s_w, s_o, raw))
            raw = l1_sort_pixel<8>(col_d, col_w, base, n, lane);
        }
      } else if (CLASS == 1) {
        if (!l1_sort_pixel_packed<16>(col_d, col_w, base, n, lane, vec, s_w, s_o, raw))
          raw = l1_sort_pixel<16>(col_d, col_w, base, n, lane);
      }
      raw = warp_sum(raw);
      if (lane == 0) {
        state[pix * SF_PIXEL_STATE_FLOATS + PS_L1] = raw;
        out_l1[pix] = fmaxr(raw, 0.f);
      }
    }
  }
}

// Runs longer than 512 samples (a camera close to a dense surface): one CTA of 256
// threads per pixel.
constexpr int LONG_THREADS = 256;

__device__ __forceinline__ unsigned long long kmin(unsigned long long a, unsigned long long b) { return a < b ? a : b; }
__device__ __forceinline__ unsigned long long kmax(unsigned long long a, unsigned long long b) { return a < b ? b : a; }

// Runs of up to T I samples (T threads, I = 4, 8, 16 per thread): the CTA sorts the
// pixel's exact 64-bit (depth bits, compositing index) keys as one bitonic network of
// NN = T I positions held in registers, thread t owning positions t I .. t I + I - 1.  The network is the
// all-ascending form of l1_sort_pixel_packed (a merge of size s first compares p with
// its mirror p ^ (s - 1), then half-cleaners p vs p ^ h, the lower position taking the
// minimum).  A compare-exchange whose partner is in the same thread is a register
// min/max, one in the same warp a shuffle, and only the stages whose partner is in
// another warp (6 of the 78 stages at NN = 4096) exchange through shared memory, where
// the keys sit striped (position t I + j at j T + t: conflict-free for every partner
// distance).  The weights are parked by compositing index in s_w; after the
// sort each thread scans its I sorted samples, a block scan of the per-thread totals
// gives each its prefix, and both factors are assembled in shared memory by compositing
// index and leave in blocked layout.  Returns this thread's share of the L1 value.
template <int T, int I>
__device__ float l1_sort_pixel_cta(float* col_d, float* col_w, int64_t base, int n, bool vec,
                                   unsigned long long* s_key, float* s_w, float (*s_tot)[T / 32]) {
  constexpr int NN = T * I;
  constexpr int WI = 32 * I;  // positions per warp
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  unsigned long long key[I];
  {
    float dv[I], wv[I];
    l1_load_run<I>(col_d, base, n, tid, vec, dv);
    l1_load_run<I>(col_w, base, n, tid, vec, wv);
#pragma unroll
    for (int j = 0; j < I; ++j) {
      const int e = tid * I + j;
      key[j] = e < n ? ((unsigned long long)__float_as_uint(dv[j]) << 32) | (unsigned)e : ~0ull;
    }
#pragma unroll
    for (int q = 0; q < I / 4; ++q)
      *reinterpret_cast<float4*>(s_w + tid * I + 4 * q) =
          make_float4(wv[4 * q], wv[4 * q + 1], wv[4 * q + 2], wv[4 * q + 3]);
  }
  // in-thread merges of sizes 2 .. I
#pragma unroll
  for (int size = 2; size <= I; size <<= 1) {
#pragma unroll
    for (int j = 0; j < I; ++j) {
      const int m = j ^ (size - 1);
      if (j < m) {
        const unsigned long long a = kmin(key[j], key[m]), b = kmax(key[j], key[m]);
        key[j] = a;
        key[m] = b;
      }
    }
#pragma unroll
    for (int stride = size >> 2; stride > 0; stride >>= 1) {
#pragma unroll
      for (int j = 0; j < I; ++j) {
        if ((j & stride) == 0) {
          const unsigned long long a = kmin(key[j], key[j + stride]), b = kmax(key[j], key[j + stride]);
          key[j] = a;
          key[j + stride] = b;
        }
      }
    }
  }
#pragma unroll 1
  for (int size = 2 * I; size <= NN; size <<= 1) {
    if (size <= WI) {
      // mirror partner in this warp: lane ^ (size / I - 1), element I - 1 - j
      const int lm = size / I - 1;
      const bool take_min = (lane & (size / (2 * I))) == 0;
#pragma unroll
      for (int j = 0; j < I / 2; ++j) {
        const unsigned long long o1 = __shfl_xor_sync(FULL, key[I - 1 - j], lm);
        const unsigned long long o2 = __shfl_xor_sync(FULL, key[j], lm);
        key[j] = take_min ? kmin(key[j], o1) : kmax(key[j], o1);
        key[I - 1 - j] = take_min ? kmin(key[I - 1 - j], o2) : kmax(key[I - 1 - j], o2);
      }
    } else {
      // mirror partner in another warp: thread tid ^ (size / I - 1), element I - 1 - j
      const int tm = size / I - 1;
      const bool take_min = (tid & (size / (2 * I))) == 0;
      __syncthreads();  // the previous exchange has been read
#pragma unroll
      for (int j = 0; j < I; ++j) s_key[j * T + tid] = key[j];
      __syncthreads();
#pragma unroll
      for (int j = 0; j < I; ++j) {
        const unsigned long long o = s_key[(I - 1 - j) * T + (tid ^ tm)];
        key[j] = take_min ? kmin(key[j], o) : kmax(key[j], o);
      }
    }
#pragma unroll 1
    for (int h = size >> 2; h >= I; h >>= 1) {
      const int ts = h / I;  // partner thread distance
      const bool take_min = (tid & ts) == 0;
      if (h >= WI) {
        __syncthreads();
#pragma unroll
        for (int j = 0; j < I; ++j) s_key[j * T + tid] = key[j];
        __syncthreads();
#pragma unroll
        for (int j = 0; j < I; ++j) {
          const unsigned long long o = s_key[j * T + (tid ^ ts)];
          key[j] = take_min ? kmin(key[j], o) : kmax(key[j], o);
        }
      } else {
#pragma unroll
        for (int j = 0; j < I; ++j) {
          const unsigned long long o = __shfl_xor_sync(FULL, key[j], ts);
          key[j] = take_min ? kmin(key[j], o) : kmax(key[j], o);
        }
      }
    }
#pragma unroll
    for (int stride = I >> 1; stride > 0; stride >>= 1) {
#pragma unroll
      for (int j = 0; j < I; ++j) {
        if ((j & stride) == 0) {
          const unsigned long long a = kmin(key[j], key[j + stride]), b = kmax(key[j], key[j + stride]);
          key[j] = a;
          key[j + stride] = b;
        }
      }
    }
  }
  __syncthreads();  // every thread's weights are in s_w; the last exchange has been read
  float w[I];
  float lw = 0.f, lwd = 0.f;
#pragma unroll
  for (int j = 0; j < I; ++j) {
    const bool live = key[j] != ~0ull;
    w[j] = live ? s_w[(uint32_t)key[j]] : 0.f;
    lw += w[j];
    lwd += w[j] * (live ? __uint_as_float((uint32_t)(key[j] >> 32)) : 0.f);
  }
  // block scan of the per-thread totals (threads hold consecutive sorted positions)
  float iw = lw, iwd = lwd;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float a1 = __shfl_up_sync(FULL, iw, o), a2 = __shfl_up_sync(FULL, iwd, o);
    if (lane >= o) { iw += a1; iwd += a2; }
  }
  if (lane == 31) { s_tot[0][wid] = iw; s_tot[1][wid] = iwd; }
  __syncthreads();  // also: every thread has read its weights from s_w
  float pw = iw - lw, pwd = iwd - lwd, Wt = 0.f, Dt = 0.f;
#pragma unroll
  for (int q = 0; q < T / 32; ++q) {
    if (q < wid) { pw += s_tot[0][q]; pwd += s_tot[1][q]; }
    Wt += s_tot[0][q];
    Dt += s_tot[1][q];
  }
  float* s_o = reinterpret_cast<float*>(s_key);  // the keys' space is free
  float raw = 0.f;
#pragma unroll
  for (int j = 0; j < I; ++j) {
    if (key[j] != ~0ull) {
      const uint32_t k = (uint32_t)key[j];
      const float d = __uint_as_float((uint32_t)(key[j] >> 32));
      raw += 2.f * w[j] * (d * pw - pwd);
      s_o[k] = 2.f * (2.f * d * pw - d * Wt + Dt - 2.f * pwd);
      s_w[k] = 2.f * w[j] * (2.f * pw + w[j] - Wt);
      pw += w[j];
      pwd += w[j] * d;
    }
  }
  __syncthreads();  // both factors assembled by compositing index
  l1_store_run<I>(col_d, base, n, tid, vec, s_o);
  l1_store_run<I>(col_w, base, n, tid, vec, s_w);
  return raw;
}

// The long-run kernel: runs of up to 4096 samples take l1_sort_pixel_cta; longer ones
// (up to the launcher's smem_k) sort their exact 64-bit keys by a bitonic network in
// shared memory padded to the next power of two of the pixel's count, each thread then
// scans a contiguous slice of the sorted samples, a block scan of the slices' totals
// gives every slice its prefix, and the two factors are written back by compositing
// index.

__global__ void __launch_bounds__(LONG_THREADS, 2) l1_resolve_long_kernel(
    sf_camera cam, float* state, float* l1s, int64_t slots, const int64_t* off, int cap, int smem_k,
    float* out_l1) {
  extern __shared__ unsigned long long s_long[];  // smem_k keys, then smem_k weights
  float* s_w = reinterpret_cast<float*>(s_long + smem_k);
  __shared__ float s_tot[2][LONG_THREADS / 32];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int64_t npix = (int64_t)cam.width * cam.height;
  const int tiles_x = (cam.width + TILE - 1) / TILE;
  float* col_d = l1s;
  float* col_w = l1s + slots;
  // 16-byte loads and stores need aligned columns (runs start on 8-sample boundaries)
  const bool vec = ((reinterpret_cast<uintptr_t>(l1s) | (uintptr_t)(slots * sizeof(float))) & 15) == 0;
  __shared__ int s_list[LONG_THREADS];
  __shared__ int s_nlist;
  // Pixels go to CTAs in groups of LONG_THREADS: thread t of group j reads the count of
  // pixel j + t J (J groups: a cluster of long runs spreads over many CTAs), the group's
  // long runs are listed in shared memory, and the CTA resolves the listed pixels one
  // after another (one load latency per group, not per pixel).
  const int64_t ngroups = (npix + LONG_THREADS - 1) / LONG_THREADS;
  for (int64_t j = blockIdx.x; j < ngroups; j += gridDim.x) {
    if (tid == 0) s_nlist = 0;
    __syncthreads();
    if (j + tid * ngroups < npix) {
      const int64_t q = j + tid * ngroups;
      int c = f2i(state[q * SF_PIXEL_STATE_FLOATS + PS_COUNT]);
      const int room = off ? (int)(off[q + 1] - off[q]) : cap;
      if (c > room) c = room;
      if (c > 512) s_list[atomicAdd(&s_nlist, 1)] = tid;
    }
    __syncthreads();
    const int nlist = s_nlist;
   for (int li = 0; li < nlist; ++li) {
    const int64_t pix = j + s_list[li] * ngroups;
    float* st = state + pix * SF_PIXEL_STATE_FLOATS;
    int n = f2i(st[PS_COUNT]);  // the same for every thread: the loop stays uniform
    const int u = (int)(pix % cam.width), v = (int)(pix / cam.width);
    const int tile = (v / TILE) * tiles_x + (u / TILE);
    const int ptid = (v % TILE) * TILE + (u % TILE);
    const int64_t base = l1_base(tile, ptid, cap, off, pix);
    const int room = off ? (int)(off[pix + 1] - off[pix]) : cap;
    if (n > room) n = room;
    if (n > smem_k) n = smem_k;  // the launcher sizes smem_k >= the largest count
    int nn = 1024;
    while (nn < n) nn <<= 1;
    float raw;
    if (nn <= 4096) {
      raw = nn == 1024 ? l1_sort_pixel_cta<LONG_THREADS, 4>(col_d, col_w, base, n, vec, s_long, s_w, s_tot)
          : nn == 2048 ? l1_sort_pixel_cta<LONG_THREADS, 8>(col_d, col_w, base, n, vec, s_long, s_w, s_tot)
                       : l1_sort_pixel_cta<LONG_THREADS, 16>(col_d, col_w, base, n, vec, s_long, s_w, s_tot);
    } else {
      float Wt = 0.f, Dt = 0.f;
      for (int k = tid; k < nn; k += LONG_THREADS) {
        if (k < n) {
          const float d = col_d[base + k], w = col_w[base + k];
          s_long[k] = ((unsigned long long)__float_as_uint(d) << 32) | (unsigned)k;
          s_w[k] = w;
          Wt += w; Dt += w * d;
        } else {
          s_long[k] = ~0ull;  // padding sorts last
        }
      }
      Wt = warp_sum(Wt); Dt = warp_sum(Dt);
      if (lane == 0) { s_tot[0][wid] = Wt; s_tot[1][wid] = Dt; }
      __syncthreads();
      Wt = 0.f; Dt = 0.f;
  #pragma unroll
      for (int q = 0; q < LONG_THREADS / 32; ++q) { Wt += s_tot[0][q]; Dt += s_tot[1][q]; }
      for (int size = 2; size <= nn; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
          for (int q = tid; q < nn / 2; q += LONG_THREADS) {
            const int i = ((q & ~(stride - 1)) << 1) | (q & (stride - 1));
            const int j = i + stride;
            const unsigned long long a = s_long[i], b = s_long[j];
            if ((a > b) == ((i & size) == 0)) { s_long[i] = b; s_long[j] = a; }
          }
          __syncthreads();
        }
      }
      // each thread's contiguous slice of E sorted samples
      const int E = nn / LONG_THREADS;
      const int r0 = tid * E;
      float tw = 0.f, twd = 0.f;
      for (int e = 0; e < E; ++e) {
        const int r = r0 + e;
        if (r < n) {
          const unsigned long long key = s_long[r];
          const float d = __uint_as_float((uint32_t)(key >> 32)), w = s_w[(uint32_t)key];
          tw += w; twd += w * d;
        }
      }
      // exclusive block scan of the slice totals
      float iw = tw, iwd = twd;
  #pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float a1 = __shfl_up_sync(FULL, iw, o), a2 = __shfl_up_sync(FULL, iwd, o);
        if (lane >= o) { iw += a1; iwd += a2; }
      }
      __syncthreads();  // every thread has read the block totals above
      if (lane == 31) { s_tot[0][wid] = iw; s_tot[1][wid] = iwd; }
      __syncthreads();
      float pw = iw - tw, pwd = iwd - twd;
      for (int q = 0; q < wid; ++q) { pw += s_tot[0][q]; pwd += s_tot[1][q]; }
      raw = 0.f;
      for (int e = 0; e < E; ++e) {
        const int r = r0 + e;
        if (r < n) {
          const unsigned long long key = s_long[r];
          const uint32_t k = (uint32_t)key;
          const float d = __uint_as_float((uint32_t)(key >> 32)), w = s_w[k];
          raw += 2.f * w * (d * pw - pwd);
          col_d[base + k] = 2.f * (2.f * d * pw - d * Wt + Dt - 2.f * pwd);
          col_w[base + k] = 2.f * w * (2.f * pw + w - Wt);
          pw += w;
          pwd += w * d;
        }
      }
    }
    raw = warp_sum(raw);
    __syncthreads();  // every thread has read the scan totals
    if (lane == 0) s_tot[0][wid] = raw;
    __syncthreads();
    if (tid == 0) {
      float total = 0.f;
#pragma unroll
      for (int q = 0; q < LONG_THREADS / 32; ++q) total += s_tot[0][q];
      st[PS_L1] = total;
      out_l1[pix] = fmaxr(total, 0.f);
    }
    __syncthreads();  // shared memory is free for the next pixel
   }
  }
}

// ------------------------------------------------------------------ backward
template <int MODE, int DIST>
__global__ void __launch_bounds__(TILE_PIXELS, SF_BWD_MIN_CTAS) raster_backward_kernel(const RasterBwdArgs a) {
#if SF_BWD_WARP_WALK && SF_BWD_WARP_STAGE
  // per warp: the records of its current group's hits (32 slots of REC4 float4)
  __shared__ float4 s_wrec[(TILE_PIXELS / 32) * 32 * REC4];
  const int wid = threadIdx.x >> 5;
#endif
#if !SF_BWD_WARP_WALK
  constexpr int AB = AccWindow<MODE>::BASE, AN = AccWindow<MODE>::N;
  // the batch's records (BWD_BATCH * REC4 float4), gradient accumulator (BWD_BATCH * AN
  // floats) and Gaussian ids (BWD_BATCH ints), in dynamic shared memory
  extern __shared__ float4 s_dyn[];
  float4* s_rec = s_dyn;
  float* s_acc = reinterpret_cast<float*>(s_dyn + BWD_BATCH * REC4);
  int* s_id = reinterpret_cast<int*>(s_dyn + BWD_BATCH * REC4 + BWD_BATCH * AN / 4);
  __shared__ int s_max;
#endif
  constexpr int NV = SampleLayout<MODE>::NV;
  const int tile = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31;
  const int tx = tile % a.tiles_x, ty = tile / a.tiles_x;
  int u, v, ptid;
  tile_pixel(tid, tx, ty, u, v, ptid);
  const int W = a.cam.width, H = a.cam.height;
  const bool inside = u < W && v < H;
  const int64_t pix = (int64_t)v * W + u;
  PixelRay pr;
  pixel_ray(a.cam, u, v, pr);
  const float wx0 = warp_minf(pr.px), wx1 = warp_maxf(pr.px);
  const float wy0 = warp_minf(pr.py), wy1 = warp_maxf(pr.py);
  const int2 rg = a.ranges[tile];
  const float ext2 = a.st.extent_sq, nearp = a.st.near_plane, farp = a.st.far_plane;
  const float inv_fx = 1.f / a.cam.K[0], inv_fy = 1.f / a.cam.K[4];

  PixelGrads pg;
  float T = 1.f;
  int last = rg.x, k = -1;
  int64_t l1_at = 0;
  float next_auxw = 0.f, next_auxd = 0.f;
  if (inside) {
    const float* st = a.state + pix * SF_PIXEL_STATE_FLOATS;
    PixelUpstream up;
    const int64_t p3 = pix * 3;
    for (int c = 0; c < 3; ++c) {
      up.rgb[c] = a.g_rgb ? a.g_rgb[p3 + c] : 0.f;
      up.normal[c] = a.g_normals ? a.g_normals[p3 + c] : 0.f;
    }
    up.alpha = a.g_alpha ? a.g_alpha[pix] : 0.f;
    up.depth = a.g_depth ? a.g_depth[pix] : 0.f;
    up.l1 = a.g_l1 ? a.g_l1[pix] : 0.f;
    up.l2 = a.g_l2 ? a.g_l2[pix] : 0.f;
    up.median = a.g_median ? a.g_median[pix] : 0.f;
    up.var = a.g_var ? a.g_var[pix] : 0.f;
    up.amb = a.g_amb ? a.g_amb[pix] : 0.f;
    pixel_grads(MODE, DIST, st, pr, a.st.background, up, pg);
    T = st[PS_T];
    last = f2i(st[PS_LAST]);
    k = f2i(st[PS_COUNT]) - 1;
    if (DIST & SF_DIST_L1) {
      l1_at = l1_base(tile, ptid, a.l1_cap, a.l1_off, pix);
      // never read past the pixel's run
      const int room = a.l1_off ? (int)(a.l1_off[pix + 1] - a.l1_off[pix]) : a.l1_cap;
      if (k >= room) k = room - 1;
      if (k >= 0) {
        next_auxw = a.l1s[l1_at + k];
        next_auxd = a.l1s[a.l1_slots + l1_at + k];
      }
    }
  } else {
    pg.gW = pg.gD = pg.gDnum = pg.gA = pg.gL1 = pg.gL2 = pg.gMed = pg.gVar = 0.f;
    for (int c = 0; c < 3; ++c) pg.gC[c] = pg.gN[c] = pg.C[c] = 0.f;
    pg.W = pg.D = 0.f;
    pg.med_pos = -1;
  }
#if !SF_BWD_WARP_WALK
  if (tid == 0) s_max = rg.x;
  __syncthreads();
  {
    const int m = warp_max(last);
    if (lane == 0) atomicMax(&s_max, m);
  }
  __syncthreads();
  const int maxlast = s_max;
#endif
  float S = 0.f;

#if SF_BWD_WARP_WALK
  // Each warp walks back from its own last contributing position, 32 entries at a
  // time, reading the records from global memory (L1-cached), and adds each (warp,
  // Gaussian) sum straight to the global gradient: no shared staging, no barrier.
  const int hi0 = warp_max(last);
#if SF_BWD_PREFETCH_IDS
  int gid_next = 0;
  if (lane < hi0 - max(rg.x, hi0 - 32)) gid_next = __ldg(a.ids + max(rg.x, hi0 - 32) + lane);
#endif
  for (int hi = hi0; hi > rg.x; hi -= 32) {
    const int lo = max(rg.x, hi - 32);
    {
#if SF_BWD_PREFETCH_IDS
     // this group's ids arrived during the previous group; request the next group's
     int gid = gid_next;
     {
       const int lo_n = max(rg.x, lo - 32);
       if (lane < lo - lo_n) gid_next = __ldg(a.ids + lo_n + lane);
     }
#else
     int gid = 0;
#endif
     bool hit = false;
     if (lane < hi - lo) {
#if !SF_BWD_PREFETCH_IDS
       gid = __ldg(a.ids + lo + lane);
#endif
       const float4 w0 = __ldg(reinterpret_cast<const float4*>(a.records) + (int64_t)gid * REC4);
       const float qc = __ldg(a.records + (int64_t)gid * SF_RECORD_FLOATS + R_QC);
       hit = box_may_pass(w0.z, w0.w, qc, w0.x, w0.y, wx0, wx1, wy0, wy1, ext2);
#if SF_BWD_WARP_STAGE
       // a hit's whole record into the warp's slice of shared memory, all lanes' loads
       // in flight together
       if (hit) {
         const float4* src = reinterpret_cast<const float4*>(a.records) + (int64_t)gid * REC4;
         float4* dst = s_wrec + (wid * 32 + lane) * REC4;
         dst[0] = w0;
#pragma unroll
         for (int c = 1; c < REC4; ++c) dst[c] = __ldg(src + c);
       }
#endif
     }
     unsigned m = __ballot_sync(FULL, hit);
#if SF_BWD_WARP_STAGE
     __syncwarp();
#endif
     while (m) {
      const int jb = 31 - __clz(m);
      m &= ~(1u << jb);
      const int j = jb;
      const int gj = __shfl_sync(FULL, gid, jb);
      const int pos = lo + j;
#else
  for (int hi = maxlast; hi > rg.x; hi -= BWD_BATCH) {
    const int lo = max(rg.x, hi - BWD_BATCH);
    const int n_in = hi - lo;
    __syncthreads();
    for (int q = tid; q < n_in * REC4; q += TILE_PIXELS) {
      const int slot = q / REC4, comp = q - slot * REC4;
      const int id = __ldg(a.ids + lo + slot);
      if (comp == 0) s_id[slot] = id;
      s_rec[q] = __ldg(reinterpret_cast<const float4*>(a.records) + (int64_t)id * REC4 + comp);
    }
    for (int q = tid; q < n_in * AN; q += TILE_PIXELS) s_acc[q] = 0.f;
    __syncthreads();
    for (int g = ((n_in + 31) >> 5) - 1; g >= 0; --g) {
     unsigned m = warp_cull(s_rec, n_in, g, lane, wx0, wx1, wy0, wy1, ext2);
     while (m) {
      const int jb = 31 - __clz(m);
      m &= ~(1u << jb);
      const int j = g * 32 + jb;
      const int pos = lo + j;
#endif
      float vals[NV];
#pragma unroll
      for (int q = 0; q < NV; ++q) vals[q] = 0.f;
      bool act = false;
      if (pos < last) {
#if SF_BWD_WARP_WALK && SF_BWD_WARP_STAGE
        const float* rec = reinterpret_cast<const float*>(s_wrec + (wid * 32 + j) * REC4);
#elif SF_BWD_WARP_WALK
        const float* rec = a.records + (int64_t)gj * SF_RECORD_FLOATS;
#else
        const float* rec = reinterpret_cast<const float*>(&s_rec[j * REC4]);
#endif
        Sample s;
        float auxw = 0.f, auxd = 0.f;
        // the sample evaluation is a fixed function of its inputs (explicit rounding
        // everywhere), so membership matches the forward pass exactly and this pixel's
        // k-th contributing sample (counted from the end) is its k-th stored sample
        const bool contrib = eval_sample<MODE>(rec, pr, ext2, nearp, farp, s);
        if ((DIST & SF_DIST_L1) && contrib) {
          // the factors of this sample were fetched one contributing sample ahead
          auxw = next_auxw;
          auxd = next_auxd;
          --k;
          if (k >= 0) {
            next_auxw = a.l1s[l1_at + k];
            next_auxd = a.l1s[a.l1_slots + l1_at + k];
          } else {
            next_auxw = next_auxd = 0.f;
          }
        }
        if (contrib) {
          act = true;
          const float al = s.alpha;
          const float om = 1.f - al;  // >= 0.001: alpha is clamped to 0.999
          const float inv_om = fast_rcp(om);
          const float Ti = T * inv_om;
          const float w = al * Ti;
          const float adj = sample_adj<MODE>(rec, s, pg, auxw);
          const float g_alpha = Ti * adj - S * inv_om;
          S += w * adj;
          T = Ti;
          float g_depth = w * pg.gD + (pos == pg.med_pos ? pg.gMed : 0.f) + pg.gL1 * auxd;
          if (DIST & SF_DIST_L2) g_depth += pg.gL2 * 4.f * w * (pg.W * s.depth - pg.D);
          sample_backward<MODE>(rec, pr, s, pg, w, g_alpha, g_depth, inv_fx, inv_fy, vals);
        }
      }
      if (__any_sync(FULL, act)) {
        float v16[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) v16[q] = q < NV ? vals[q] : 0.f;
        const float r = reduce16_transposed(v16, lane);
        const int qi = lane >> 1;
#if SF_BWD_WARP_WALK
        // record slots 0..19 to the gradient record, 20..21 to absgrad
        float* const grec = a.grad_records + (int64_t)gj * SF_RECORD_FLOATS;
        float* const gabs = a.absgrad + (int64_t)gj * 2;
        if ((lane & 1) == 0 && qi < NV && qi < 16 && r != 0.f) {
          const int sl = SampleLayout<MODE>::slot(qi);
          atomicAdd(sl < SF_RECORD_FLOATS ? grec + sl : gabs + (sl - SF_RECORD_FLOATS), r);
        }
#pragma unroll
        for (int q = 16; q < NV; ++q) {
          const float t = warp_sum(vals[q]);
          if (lane == 2 * (q - 16) + 1 && t != 0.f) {
            const int sl = SampleLayout<MODE>::slot(q);
            atomicAdd(sl < SF_RECORD_FLOATS ? grec + sl : gabs + (sl - SF_RECORD_FLOATS), t);
          }
        }
#else
        if ((lane & 1) == 0 && qi < NV && qi < 16 && r != 0.f)
          atomicAdd(&s_acc[j * AN + SampleLayout<MODE>::slot(qi) - AB], r);
#pragma unroll
        for (int q = 16; q < NV; ++q) {
          const float t = warp_sum(vals[q]);
          if (lane == 2 * (q - 16) + 1 && t != 0.f) atomicAdd(&s_acc[j * AN + SampleLayout<MODE>::slot(q) - AB], t);
        }
#endif
      }
     }
#if SF_BWD_WARP_STAGE
     __syncwarp();  // the slice is read before the next group overwrites it
#endif
    }
#if !SF_BWD_WARP_WALK
    __syncthreads();
    for (int q = tid; q < n_in * (AN / 4); q += TILE_PIXELS) {
      const int slot = q / (AN / 4), c4 = q - slot * (AN / 4) + AB / 4;
      const float4 val = reinterpret_cast<const float4*>(s_acc)[q];
      if (val.x == 0.f && val.y == 0.f && val.z == 0.f && val.w == 0.f) continue;
      const int id = s_id[slot];
      if (c4 < REC4) {
        atomicAdd(reinterpret_cast<float4*>(a.grad_records + (int64_t)id * SF_RECORD_FLOATS) + c4, val);
      } else {
        atomicAdd(reinterpret_cast<float2*>(a.absgrad + (int64_t)id * 2), make_float2(val.x, val.y));
      }
    }
#endif
  }
  if ((DIST & SF_DIST_L1) && inside && k != -1 && a.error_word) atomicOr(a.error_word, 1);
}

// GOF: proxy_xy = (xy - c) z / f  -> adjoint of the projected means and of camera z;
// RaDe-GS / AmbiSuR: the delta adjoint already is the projected-mean adjoint.
__global__ void raster_finalize_kernel(const float* records, int64_t n, sf_camera cam, int mode,
                                       float* grec, float* gxy) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float* g = grec + i * SF_RECORD_FLOATS;
  if (mode == SF_MODE_GOF) {
    const float* r = records + i * SF_RECORD_FLOATS;
    const float fx = cam.K[0], fy = cam.K[4], cx = cam.K[2], cy = cam.K[5];
    const float z = r[R_Z];
    const float gp0 = g[R_PROXY], gp1 = g[R_PROXY + 1], gp2 = g[R_PROXY + 2];
    gxy[i * 2 + 0] = gp0 * z / fx;
    gxy[i * 2 + 1] = gp1 * z / fy;
    g[R_Z] = gp0 * (r[R_X] - cx) / fx + gp1 * (r[R_Y] - cy) / fy + gp2;
  } else {
    gxy[i * 2 + 0] = g[R_X];
    gxy[i * 2 + 1] = g[R_Y];
  }
}

__global__ void pixel_counts_kernel(const float* state, int64_t npix, int32_t* counts) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  // runs rounded up to whole 8-sample groups (32-byte aligned starts for the forward's
  // sector-sized L1 stores)
  if (i < npix) counts[i] = (f2i(state[i * SF_PIXEL_STATE_FLOATS + PS_COUNT]) + 7) & ~7;
}

// Dynamic shared memory above the 48 KB default needs the per-kernel opt-in, set once
// per kernel instance; the carveout preference asks for the shared memory that `ctas`
// resident CTAs of `bytes` dynamic + `fixed` static bytes need (plus 1 KB reserved each).
template <typename K>
cudaError_t configure_smem(K kernel, size_t bytes, size_t fixed, int ctas, bool& done) {
  if (done) return cudaSuccess;
  cudaError_t e = cudaSuccess;
  // above 48 KB of static + dynamic shared memory a launch needs the opt-in
  if (bytes + fixed > 48 * 1024)
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  const size_t need = (size_t)ctas * (bytes + fixed + 1024);
  if (e == cudaSuccess && need > 132 * 1024) {
    const int pct = (int)((need * 100 + 228 * 1024 - 1) / (228 * 1024));
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, pct > 100 ? 100 : pct);
  }
  if (e == cudaSuccess) done = true;
  return e;
}

template <int MODE, int DIST>
cudaError_t fwd_launch(const RasterFwdArgs& a, int n_tiles, cudaStream_t s) {
  constexpr size_t bytes = sizeof(float4) * (SF_FWD_WARP_WALK ? TILE_PIXELS : FWD_BATCH) * REC4;
  constexpr size_t ring = sizeof(float) * ((DIST & SF_DIST_L1) ? 2 : 1) * L1_RING * TILE_PIXELS;
  static bool configured = false;
  cudaError_t e = configure_smem(raster_forward_kernel<MODE, DIST>, bytes, ring, SF_FWD_MIN_CTAS, configured);
  if (e != cudaSuccess) return e;
  raster_forward_kernel<MODE, DIST><<<n_tiles, TILE_PIXELS, bytes, s>>>(a);
  return cudaGetLastError();
}

template <int MODE>
cudaError_t fwd_dispatch(const RasterFwdArgs& a, int n_tiles, cudaStream_t s) {
  count_launches(1);
  switch (a.st.distortions & 3) {
    case 0: return fwd_launch<MODE, 0>(a, n_tiles, s);
    case 1: return fwd_launch<MODE, 1>(a, n_tiles, s);
    case 2: return fwd_launch<MODE, 2>(a, n_tiles, s);
    default: return fwd_launch<MODE, 3>(a, n_tiles, s);
  }
}

template <int MODE, int DIST>
cudaError_t bwd_launch(const RasterBwdArgs& a, int n_tiles, cudaStream_t s) {
  constexpr size_t bytes = SF_BWD_WARP_WALK ? 0 :
      sizeof(float4) * BWD_BATCH * REC4 + sizeof(float) * BWD_BATCH * AccWindow<MODE>::N + sizeof(int) * BWD_BATCH;
  static bool configured = false;
  cudaError_t e = configure_smem(raster_backward_kernel<MODE, DIST>, bytes, 16, SF_BWD_MIN_CTAS, configured);
  if (e != cudaSuccess) return e;
  raster_backward_kernel<MODE, DIST><<<n_tiles, TILE_PIXELS, bytes, s>>>(a);
  return cudaGetLastError();
}

template <int MODE>
cudaError_t bwd_dispatch(const RasterBwdArgs& a, int n_tiles, cudaStream_t s) {
  count_launches(1);
  switch (a.st.distortions & 3) {
    case 0: return bwd_launch<MODE, 0>(a, n_tiles, s);
    case 1: return bwd_launch<MODE, 1>(a, n_tiles, s);
    case 2: return bwd_launch<MODE, 2>(a, n_tiles, s);
    default: return bwd_launch<MODE, 3>(a, n_tiles, s);
  }
}

}  // namespace

cudaError_t launch_raster_forward(const RasterFwdArgs& a, int n_tiles, cudaStream_t s) {
  if (n_tiles <= 0) return cudaSuccess;
  switch (a.st.mode) {
    case SF_MODE_RADEGS: return fwd_dispatch<SF_MODE_RADEGS>(a, n_tiles, s);
    case SF_MODE_GOF: return fwd_dispatch<SF_MODE_GOF>(a, n_tiles, s);
    default: return fwd_dispatch<SF_MODE_AMBISUR>(a, n_tiles, s);
  }
}

cudaError_t launch_raster_backward(const RasterBwdArgs& a, int n_tiles, cudaStream_t s) {
  if (n_tiles <= 0) return cudaSuccess;
  switch (a.st.mode) {
    case SF_MODE_RADEGS: return bwd_dispatch<SF_MODE_RADEGS>(a, n_tiles, s);
    case SF_MODE_GOF: return bwd_dispatch<SF_MODE_GOF>(a, n_tiles, s);
    default: return bwd_dispatch<SF_MODE_AMBISUR>(a, n_tiles, s);
  }
}

size_t l1_resolve_smem_per_warp(int smem_k) { return (size_t)smem_k * (sizeof(unsigned long long) + sizeof(float)); }

cudaError_t launch_l1_resolve(const sf_camera& cam, const sf_settings& st, float* state,
                              float* l1s, int64_t slots, const int64_t* off, int cap, int max_samples,
                              float* out_l1, cudaStream_t s) {
  (void)st;
  const int64_t npix = (int64_t)cam.width * cam.height;
  if (npix == 0) return cudaSuccess;
  // one 32-pixel group per warp (4 warps per CTA) for the common class; the longer
  // classes stride over the groups with a grid of 8 CTAs per SM
  const int64_t blocks = (npix + 127) / 128;
  count_launches(1);
  l1_resolve_kernel<0><<<(unsigned)blocks, 128, 0, s>>>(cam, state, l1s, slots, off, cap, 0, out_l1);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || max_samples <= 256) return e;
  count_launches(1);
  l1_resolve_kernel<1><<<(unsigned)(blocks < 148 * 8 ? blocks : 148 * 8), 128, 0, s>>>(cam, state, l1s, slots, off,
                                                                                     cap, 0, out_l1);
  e = cudaGetLastError();
  if (e != cudaSuccess || max_samples <= 512) return e;
  int smem_k = 1024;  // a power of two >= the largest count (the largest bitonic network)
  while (smem_k < max_samples) smem_k <<= 1;
  const size_t smem = l1_resolve_smem_per_warp(smem_k);  // one pixel per CTA
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  e = cudaFuncSetAttribute(l1_resolve_long_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(l1_resolve_long_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  if (e != cudaSuccess) return e;
  // resident CTAs per SM: the register budget (launch bounds) allows 2
  const int per_sm = (int)min((size_t)2, (size_t)(220 * 1024) / (smem + 1024));
  const int64_t b2 = min(npix, (int64_t)148 * (per_sm > 0 ? per_sm : 1));
  count_launches(1);
  l1_resolve_long_kernel<<<(unsigned)b2, LONG_THREADS, smem, s>>>(cam, state, l1s, slots, off, cap, smem_k,
                                                                  out_l1);
  return cudaGetLastError();
}

cudaError_t launch_raster_finalize(const float* records, int64_t n, const sf_camera& cam,
                                   int mode, float* grad_records, float* grad_means2d,
                                   cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  count_launches(1);
  raster_finalize_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(records, n, cam, mode, grad_records, grad_means2d);
  return cudaGetLastError();
}

cudaError_t launch_pixel_counts(const float* state, int64_t npix, int32_t* counts, cudaStream_t s) {
  if (npix == 0) return cudaSuccess;
  count_launches(1);
  pixel_counts_kernel<<<(unsigned)((npix + 255) / 256), 256, 0, s>>>(state, npix, counts);
  return cudaGetLastError();
}

}  // namespace sf
