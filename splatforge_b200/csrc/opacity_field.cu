// gaussian.opacity_field@1 (src/splatforge/gaussian/semantics.json:25,
// reference.py:194-222): for every view origin o and query point p, walk the
// normalised ray o -> p, evaluate every Gaussian at min(peak t, |p - o|), drop peaks
// behind the origin, clamp to [0, 0.999], O_view = 1 - prod(1 - c); the field is the
// minimum over views (starting from 1).
//
// One thread per (point, view); a CTA stages 256 Gaussians at a time in shared memory
// (mean, symmetric inverse covariance, opacity: 10 floats) and every thread of the
// CTA sweeps the batch.  The per-view results meet in an atomicMin on the float bits
// (the field is non-negative, so its bit pattern orders like its value).  A thread
// stops early once its transmittance is below 1e-7 (the field is then within 1e-7
// of 1 for that view).
#include <cuda_runtime.h>

#include <vector>

#include "sf_device.cuh"
#include "sf_kernels.h"

namespace sf {

namespace {

constexpr int OF_THREADS = 256;
constexpr int OF_FLOATS = 10;

__global__ void field_init_kernel(uint32_t* out, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = __float_as_uint(1.f);
}

__global__ void __launch_bounds__(OF_THREADS) field_kernel(const float* __restrict__ pts, int64_t np,
                                                            const float* __restrict__ gauss, int64_t ng,
                                                            const float* __restrict__ origins,
                                                            uint32_t* out) {
  __shared__ float s_g[OF_THREADS * OF_FLOATS];
  const int64_t i = (int64_t)blockIdx.x * OF_THREADS + threadIdx.x;
  const int view = blockIdx.y;
  const float ox = origins[view * 3], oy = origins[view * 3 + 1], oz = origins[view * 3 + 2];
  const bool live = i < np;
  float dx = 0.f, dy = 0.f, dz = 0.f, dist = 0.f;
  if (live) {
    dx = pts[i * 3] - ox; dy = pts[i * 3 + 1] - oy; dz = pts[i * 3 + 2] - oz;
    dist = sqrtf(dx * dx + dy * dy + dz * dz);
    const float inv = 1.f / fmaxf(dist, 1e-12f);
    dx *= inv; dy *= inv; dz *= inv;
  }
  float T = 1.f;
  bool done = !live;
  for (int64_t base = 0; base < ng; base += OF_THREADS) {
    if (__syncthreads_and(done)) break;
    const int n_in = (int)min((int64_t)OF_THREADS, ng - base);
    for (int k = threadIdx.x; k < n_in * OF_FLOATS; k += OF_THREADS) s_g[k] = gauss[base * OF_FLOATS + k];
    __syncthreads();
    if (!done) {
      for (int j = 0; j < n_in; ++j) {
        const float* g = s_g + j * OF_FLOATS;
        // g: mean(3), q00 q01 q02 q11 q12 q22, opacity
        const float d0 = ox - g[0], d1 = oy - g[1], d2 = oz - g[2];
        const float qd0 = g[3] * dx + g[4] * dy + g[5] * dz;
        const float qd1 = g[4] * dx + g[6] * dy + g[7] * dz;
        const float qd2 = g[5] * dx + g[7] * dy + g[8] * dz;
        const float den = fmaxf(dx * qd0 + dy * qd1 + dz * qd2, 1e-12f);
        const float t = -(d0 * qd0 + d1 * qd1 + d2 * qd2) / den;
        if (!(t > 0.f)) continue;
        const float te = fminf(t, dist);
        const float f0 = d0 + te * dx, f1 = d1 + te * dy, f2 = d2 + te * dz;
        const float e = f0 * (g[3] * f0 + g[4] * f1 + g[5] * f2) + f1 * (g[4] * f0 + g[6] * f1 + g[7] * f2) +
                        f2 * (g[5] * f0 + g[7] * f1 + g[8] * f2);
        const float c = fminf(fmaxf(g[9] * expf(-0.5f * fmaxf(e, 0.f)), 0.f), 0.999f);
        T *= 1.f - c;
      }
      if (T < 1e-7f) done = true;
    }
  }
  if (live) atomicMin(out + i, __float_as_uint(fmaxf(1.f - T, 0.f)));
}

// pack means, the symmetric inverse covariance and opacities into 10-float records
__global__ void field_pack_kernel(const float* means, const float* invcov, const float* op, int64_t n, float* g) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float* r = g + i * OF_FLOATS;
  const float* q = invcov + i * 9;
  r[0] = means[i * 3]; r[1] = means[i * 3 + 1]; r[2] = means[i * 3 + 2];
  r[3] = q[0]; r[4] = 0.5f * (q[1] + q[3]); r[5] = 0.5f * (q[2] + q[6]);
  r[6] = q[4]; r[7] = 0.5f * (q[5] + q[7]); r[8] = q[8];
  r[9] = op[i];
}

// ------------------------------------------------------------------ culled field
// For large queries the field is evaluated against per-view candidate lists instead of
// every Gaussian.  A Gaussian whose opacity o exceeds the cutoff c0 contributes more
// than c0 only within the ball of radius R = sqrt(2 ln(o / c0) / lambda_min(Q)) around
// its mean (there (x-m)^T Q (x-m) >= |x-m|^2 lambda_min), and the field samples it on
// the ray from the view origin through the query point.  So per view the Gaussians are
// binned into the cells of a cube map around the origin that their ball's cone of
// directions can reach, and a query only visits the cells of its own direction (plus
// the Gaussians whose ball contains the origin).  Contributions below c0 are dropped;
// everything else is evaluated exactly as the brute-force kernel does.
constexpr int CF_REC = 12;  // mean 3, symmetric Q 6, opacity, bound radius, pad

__device__ __forceinline__ double sym3_min_eig(double a, double b, double c, double d, double e, double f) {
  // [[a b c] [b d e] [c e f]]: closed-form eigenvalues of a symmetric 3x3 matrix
  const double p1 = b * b + c * c + e * e;
  if (p1 == 0.0) return fmin(a, fmin(d, f));
  const double q = (a + d + f) / 3.0;
  const double p2 = (a - q) * (a - q) + (d - q) * (d - q) + (f - q) * (f - q) + 2.0 * p1;
  const double p = sqrt(p2 / 6.0);
  const double ia = (a - q) / p, id = (d - q) / p, iff = (f - q) / p, ib = b / p, ic = c / p, ie = e / p;
  double r = 0.5 * (ia * (id * iff - ie * ie) - ib * (ib * iff - ie * ic) + ic * (ib * ie - id * ic));
  r = fmin(1.0, fmax(-1.0, r));
  const double phi = acos(r) / 3.0;
  return q + 2.0 * p * cos(phi + 2.0943951023931957);  // + 2 pi / 3: the smallest
}

__global__ void cfield_prep_kernel(const float* means, const float* invcov, const float* op, int64_t n,
                                   float cutoff, float* rec) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float* q = invcov + i * 9;
  const float a = q[0], b = 0.5f * (q[1] + q[3]), c = 0.5f * (q[2] + q[6]);
  const float d = q[4], e = 0.5f * (q[5] + q[7]), f = q[8];
  const float o = op[i];
  float R;
  if (!(o > cutoff)) {
    R = -1.f;  // its contribution never exceeds the cutoff
  } else {
    const double lmax = fabs((double)a) + fabs((double)d) + fabs((double)f) + 2.0 * (fabs((double)b) + fabs((double)c) + fabs((double)e));
    const double lmin = sym3_min_eig(a, b, c, d, e, f) - 1e-9 * lmax;  // err on the small side
    if (!(lmin > 0.0)) {
      R = INFINITY;  // not positive definite: never culled
    } else {
      const double k2 = 2.0 * log((double)o / (double)cutoff);
      R = (float)(sqrt(k2 / lmin) * 1.001 + 1e-6);
    }
  }
  float* r = rec + i * CF_REC;
  r[0] = means[i * 3]; r[1] = means[i * 3 + 1]; r[2] = means[i * 3 + 2];
  r[3] = a; r[4] = b; r[5] = c; r[6] = d; r[7] = e; r[8] = f;
  r[9] = o; r[10] = R; r[11] = 0.f;
}

// Cube map around the origin: face 2*a + (negative), a the major axis of the direction;
// u = d[b] / |d[a]|, v = d[c] / |d[a]| with b = (a+1)%3, c = (a+2)%3; F x F cells per face.
__device__ __forceinline__ int cube_cell(float dx, float dy, float dz, int F) {
  const float ax = fabsf(dx), ay = fabsf(dy), az = fabsf(dz);
  int a;
  float m, ub, vc;
  if (ax >= ay && ax >= az) { a = 0; m = ax; ub = dy; vc = dz; }
  else if (ay >= az) { a = 1; m = ay; ub = dz; vc = dx; }
  else { a = 2; m = az; ub = dx; vc = dy; }
  const float major = a == 0 ? dx : (a == 1 ? dy : dz);
  const int face = 2 * a + (major < 0.f ? 1 : 0);
  const float inv = 1.f / m;
  int ix = (int)floorf((ub * inv + 1.f) * 0.5f * F);
  int iy = (int)floorf((vc * inv + 1.f) * 0.5f * F);
  ix = min(max(ix, 0), F - 1);
  iy = min(max(iy, 0), F - 1);
  return (face * F + iy) * F + ix;
}

// Cells [x0, x1] x [y0, y1] of face (axis a, sign s) that a cone of half-angle alpha
// around the unit direction c can reach: on the face u = tan(psi), psi the angle of
// the direction in the (a, b) plane, and a cap's psi stays within its centre's psi
// +- asin(sin(alpha) / cos(latitude about the c axis)) (every psi when the cap holds
// that axis); likewise v in the (a, c) plane.  Returns false when the cap misses the face.
__device__ __forceinline__ bool cap_face_box(const float* cv, float sin_a, int a, int s, int F, int& x0, int& x1,
                                             int& y0, int& y1) {
  const int b = (a + 1) % 3, c = (a + 2) % 3;
  const float ca = s > 0 ? cv[a] : -cv[a];
  const float margin = 1e-4f;
  float lo[2], hi[2];
  const int other[2] = {b, c};
  for (int k = 0; k < 2; ++k) {
    const int ax = other[k];
    const float r = sqrtf(ca * ca + cv[ax] * cv[ax]);
    const float psi = atan2f(cv[ax], ca);
    float half;
    if (sin_a >= r) half = 3.2f;  // the cap holds the pole: every angle
    else half = asinf(sin_a / r) + margin;
    float p0 = psi - half, p1 = psi + half;
    const float qpi = 0.78539816f;
    if (p1 < -qpi || p0 > qpi) return false;
    p0 = fmaxf(p0, -qpi);
    p1 = fminf(p1, qpi);
    lo[k] = tanf(p0);
    hi[k] = tanf(p1);
  }
  x0 = max(0, (int)floorf((lo[0] + 1.f) * 0.5f * F) - 1);
  x1 = min(F - 1, (int)floorf((hi[0] + 1.f) * 0.5f * F) + 1);
  y0 = max(0, (int)floorf((lo[1] + 1.f) * 0.5f * F) - 1);
  y1 = min(F - 1, (int)floorf((hi[1] + 1.f) * 0.5f * F) + 1);
  return x0 <= x1 && y0 <= y1;
}

// Per Gaussian and view: the number of cube-map cells its cone reaches (0 for skipped
// Gaussians and for those whose ball holds the origin, which go to the global list).
// key: float bits of the ball's nearest distance D - R (positive here), so that the
// stable depth order puts every cell list front to back; near[i] = D - R for the queries.
__global__ void cfield_count_kernel(const float* rec, int64_t n, float ox, float oy, float oz, int F,
                                    int32_t* count, int32_t* global_flag, uint32_t* key, float* near) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float* r = rec + i * CF_REC;
  const float R = r[10];
  int total = 0, glob = 0;
  uint32_t k = 0xffffffffu;
  float nd = 0.f;
  if (R >= 0.f) {
    const float cx = r[0] - ox, cy = r[1] - oy, cz = r[2] - oz;
    const float D = sqrtf(cx * cx + cy * cy + cz * cz);
    if (!(D > R * 1.0001f + 1e-6f)) {
      glob = 1;
    } else {
      nd = fmaxf((D - R) * 0.9999f - 1e-6f, 0.f);  // rounded towards the origin
      k = __float_as_uint(nd);
      const float cv[3] = {cx / D, cy / D, cz / D};
      const float sin_a = R / D;
      for (int face = 0; face < 6; ++face) {
        int x0, x1, y0, y1;
        if (cap_face_box(cv, sin_a, face >> 1, (face & 1) ? -1 : 1, F, x0, x1, y0, y1))
          total += (x1 - x0 + 1) * (y1 - y0 + 1);
      }
    }
  }
  count[i] = total;
  global_flag[i] = glob;
  key[i] = total > 0 ? k : 0xffffffffu;
  near[i] = nd;
}

// thread j emits the cells of the j-th Gaussian in depth order (order[j]) at offsets[j]
__global__ void cfield_emit_kernel(const float* rec, int64_t n, float ox, float oy, float oz, int F,
                                   const int32_t* order, const int64_t* offsets, const int64_t* goffsets,
                                   uint32_t* keys, int32_t* vals, int32_t* global_ids) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= n) return;
  if (goffsets[j + 1] != goffsets[j]) global_ids[goffsets[j]] = (int32_t)j;
  int64_t at = offsets[j];
  if (offsets[j + 1] == at) return;
  const int64_t i = order[j];
  const float* r = rec + i * CF_REC;
  const float cx = r[0] - ox, cy = r[1] - oy, cz = r[2] - oz;
  const float D = sqrtf(cx * cx + cy * cy + cz * cz);
  const float cv[3] = {cx / D, cy / D, cz / D};
  const float sin_a = r[10] / D;
  for (int face = 0; face < 6; ++face) {
    int x0, x1, y0, y1;
    if (!cap_face_box(cv, sin_a, face >> 1, (face & 1) ? -1 : 1, F, x0, x1, y0, y1)) continue;
    for (int y = y0; y <= y1; ++y)
      for (int x = x0; x <= x1; ++x) {
        keys[at] = (uint32_t)((face * F + y) * F + x);
        vals[at] = (int32_t)i;
        ++at;
      }
  }
}

__device__ __forceinline__ float field_contribution(const float* g, float ox, float oy, float oz, float dx, float dy,
                                                    float dz, float dist) {
  // same arithmetic as field_kernel: peak along the ray, evaluated at min(peak, dist)
  const float d0 = ox - g[0], d1 = oy - g[1], d2 = oz - g[2];
  const float qd0 = g[3] * dx + g[4] * dy + g[5] * dz;
  const float qd1 = g[4] * dx + g[6] * dy + g[7] * dz;
  const float qd2 = g[5] * dx + g[7] * dy + g[8] * dz;
  const float den = fmaxf(dx * qd0 + dy * qd1 + dz * qd2, 1e-12f);
  const float t = -(d0 * qd0 + d1 * qd1 + d2 * qd2) / den;
  if (!(t > 0.f)) return 0.f;
  const float te = fminf(t, dist);
  const float f0 = d0 + te * dx, f1 = d1 + te * dy, f2 = d2 + te * dz;
  const float e = f0 * (g[3] * f0 + g[4] * f1 + g[5] * f2) + f1 * (g[4] * f0 + g[6] * f1 + g[7] * f2) +
                  f2 * (g[5] * f0 + g[7] * f1 + g[8] * f2);
  return fminf(fmaxf(g[9] * expf(-0.5f * fmaxf(e, 0.f)), 0.f), 0.999f);
}

// Query order inside a cell: a query's sort key carries, below its cube-map cell, its
// position on a 2^SUB x 2^SUB grid inside the cell and its quantised log distance, so that
// the 32 queries of a warp look in nearly the same direction from nearly the same
// distance: they hit the same candidate balls and stop near the same list position,
// and fewer lanes idle beside the ones that evaluate a contribution.
#ifndef SF_FIELD_QUERY_ORDER
#define SF_FIELD_QUERY_ORDER 1
#endif
#ifndef SF_FIELD_SUB_BITS
#define SF_FIELD_SUB_BITS 1  // SUB: sub-cell bits per axis
#endif
// Low key bits (sub-cell bits per axis, distance bits) that fit below `cell_bits`.
inline void query_order_bits(int cell_bits, int& sub_bits, int& dist_bits) {
  sub_bits = dist_bits = 0;
  if (!SF_FIELD_QUERY_ORDER) return;
  if (cell_bits + 2 * SF_FIELD_SUB_BITS <= 32) sub_bits = SF_FIELD_SUB_BITS;
  const int room = 32 - cell_bits - 2 * sub_bits;
  dist_bits = room < 0 ? 0 : (room > 8 ? 8 : room);
}

// A query's cube-map cell (6 F^2 for a query at the origin) and its in-cell order bits.
__device__ __forceinline__ void query_key_parts(float dx, float dy, float dz, int F, int sub_bits, int dist_bits,
                                                uint32_t& cell_out, uint32_t& low_out) {
  const float d2 = dx * dx + dy * dy + dz * dz;
  if (!(d2 > 0.f)) { cell_out = (uint32_t)(6 * F * F); low_out = 0; return; }
  const int Ff = F << sub_bits;
  const int fine = cube_cell(dx, dy, dz, Ff);  // (face * Ff + iy) * Ff + ix at the finer grid
  const int ix = fine % Ff, rest = fine / Ff, iy = rest % Ff, face = rest / Ff;
  cell_out = (uint32_t)((face * F + (iy >> sub_bits)) * F + (ix >> sub_bits));
  const int mask = (1 << sub_bits) - 1;
  const uint32_t sub = (uint32_t)(((iy & mask) << sub_bits) | (ix & mask));
  uint32_t dq = 0;
  if (dist_bits > 0) {
    // 16 steps per octave of distance, centred so that distances 1/256 .. 256 stay apart
    const float l = 0.5f * __log2f(d2) * 16.f + (float)(1 << (dist_bits - 1));
    dq = (uint32_t)fminf(fmaxf(l, 0.f), (float)((1 << dist_bits) - 1));
  }
  low_out = (sub << dist_bits) | dq;
}

// The query's cell in the high bits, the in-cell order bits below.
__device__ __forceinline__ uint32_t query_key(float dx, float dy, float dz, int F, int sub_bits, int dist_bits) {
  uint32_t cell, low;
  query_key_parts(dx, dy, dz, F, sub_bits, dist_bits, cell, low);
  return (cell << (2 * sub_bits + dist_bits)) | low;
}

// Per view, every query's sort key (query_key) with the query's index; a query at the
// origin has no direction and gets field 0 for this view right here.
__global__ void cfield_qcell_kernel(const float* pts, int64_t np, float ox, float oy, float oz, int F,
                                    int sub_bits, int dist_bits, uint32_t* qkey, int32_t* qidx, uint32_t* out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= np) return;
  const float dx = pts[i * 3] - ox, dy = pts[i * 3 + 1] - oy, dz = pts[i * 3 + 2] - oz;
  const bool at_origin = !(dx * dx + dy * dy + dz * dz > 0.f);
  qkey[i] = query_key(dx, dy, dz, F, sub_bits, dist_bits);
  qidx[i] = (int32_t)i;
  if (at_origin) atomicMin(out + i, 0u);
}

// [begin, end) of every cell in keys sorted by query_key (the cell is key >> shift).
__global__ void cfield_cell_ranges_kernel(const uint32_t* keys, int64_t n, int shift, int2* ranges) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint32_t c = keys[i] >> shift;
  if (i == 0 || (keys[i - 1] >> shift) != c) ranges[c].x = (int)i;
  if (i == n - 1 || (keys[i + 1] >> shift) != c) ranges[c].y = (int)(i + 1);
}

#ifndef SF_FIELD_CHUNK
#define SF_FIELD_CHUNK 128
#endif
constexpr int CF_THREADS = SF_FIELD_CHUNK;  // queries per work item (one thread each)

// One CTA per cube-map cell: the cell's queries (in chunks of CF_THREADS, one per
// thread) walk the cell's front-to-back candidate list, staged CF_THREADS records at a
// time in shared memory.  A query stops at the first candidate whose ball starts
// beyond it or once its transmittance is below 1e-7; the CTA stops when all have.
// number of CF_THREADS-query chunks of every cell
__global__ void cfield_chunks_kernel(const int2* qranges, int ncells, int32_t* chunks) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= ncells) return;
  const int2 r = qranges[c];
  chunks[c] = (r.y - r.x + CF_THREADS - 1) / CF_THREADS;
}

// One (cell, chunk) work item: queries qidx[q0 .. min(q0 + CF_THREADS, q1)) walk the
// cell's front-to-back candidates cell_ids[cr.x .. cr.y) after the view's global list.
// Every barrier below is taken by the whole CTA (cr is uniform), so a CTA can run work
// items one after another.
//
// The field is the minimum over views and a view's 1 - T only grows along the walk, so
// a query stops as soon as 1 - T reaches the smallest value another view has already
// stored for it (M, re-read per staged batch): what it then stores cannot lower the
// minimum, and the view that attains the minimum is never stopped before reaching it.
// The stored minimum is the same, bit for bit, as without this stop.
__device__ __forceinline__ void field_chunk(const float* pts, const int32_t* qidx, int q0, int q1, float ox,
                                            float oy, float oz, const float* rec, const float* near,
                                            const int32_t* cell_ids, int2 cr, const int32_t* global_ids,
                                            int64_t n_global, uint32_t* out, float4* s_g, float4* s_c,
                                            float* s_near, unsigned long long* pair_counter) {
  const int tid = threadIdx.x;
  unsigned evaluated = 0;  // (query, candidate) pairs taken through field_contribution
  const int qi = q0 + tid < q1 ? qidx[q0 + tid] : -1;
  const volatile uint32_t* cur = reinterpret_cast<const volatile uint32_t*>(out);
  float dx = 0.f, dy = 0.f, dz = 0.f, dist = 0.f, T = 1.f, M = 0.f;
  bool stop = qi < 0;
  if (!stop) {
    M = __uint_as_float(cur[qi]);
    dx = pts[(int64_t)qi * 3] - ox; dy = pts[(int64_t)qi * 3 + 1] - oy; dz = pts[(int64_t)qi * 3 + 2] - oz;
    dist = sqrtf(dx * dx + dy * dy + dz * dz);
    const float inv = 1.f / fmaxf(dist, 1e-12f);
    dx *= inv; dy *= inv; dz *= inv;
    for (int64_t k = 0; k < n_global && T >= 1e-7f && 1.f - T < M; ++k) {
      const float4* g4 = reinterpret_cast<const float4*>(rec + (int64_t)global_ids[k] * CF_REC);
      const float4 a = g4[0], b = g4[1], c = g4[2];
      const float g[10] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w, c.x, c.y};
      T *= 1.f - field_contribution(g, ox, oy, oz, dx, dy, dz, dist);
      ++evaluated;
    }
    stop = T < 1e-7f || 1.f - T >= M;
  }
  for (int c0 = cr.x; c0 < cr.y; c0 += CF_THREADS) {
    if (!stop) {
      M = fminf(M, __uint_as_float(cur[qi]));
      stop = 1.f - T >= M;
    }
    if (__syncthreads_count(stop) == CF_THREADS) break;
    const int nc = min(CF_THREADS, cr.y - c0);
    if (tid < nc) {
      const int id = cell_ids[c0 + tid];
      const float4* g4 = reinterpret_cast<const float4*>(rec + (int64_t)id * CF_REC);
      const float4 a = g4[0];
      s_g[tid * 3] = a;
      s_g[tid * 3 + 1] = g4[1];
      s_g[tid * 3 + 2] = g4[2];
      s_near[tid] = near[id];
      const float cx = a.x - ox, cy = a.y - oy, cz = a.z - oz;
      s_c[tid] = make_float4(cx, cy, cz, cx * cx + cy * cy + cz * cz);
    }
    __syncthreads();
    if (!stop) {
      for (int k = 0; k < nc; ++k) {
        // sorted front to back: this and every later ball start beyond the query
        if (s_near[k] > dist) { stop = true; break; }
        const float* g = reinterpret_cast<const float*>(&s_g[k * 3]);
        // the ray misses the ball (squared distance of the mean from the ray's line
        // above R^2, with a margin for the rounding of the difference): skip
        const float4 c = s_c[k];
        const float cd = c.x * dx + c.y * dy + c.z * dz;
        const float R = g[10];
        if (c.w - cd * cd > R * R * 1.002f + 1e-6f * c.w) continue;
        T *= 1.f - field_contribution(g, ox, oy, oz, dx, dy, dz, dist);
        ++evaluated;
        if (T < 1e-7f || 1.f - T >= M) { stop = true; break; }
      }
    }
  }
  if (qi >= 0) atomicMin(out + qi, __float_as_uint(fmaxf(1.f - T, 0.f)));
  if (pair_counter) {  // uniform: one atomic per warp
    unsigned long long v = evaluated;
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((tid & 31) == 0 && v) atomicAdd(pair_counter, v);
  }
}

// One CTA per (cell, chunk of CF_THREADS queries): work item w belongs to the cell c
// with chunk_off[c] <= w < chunk_off[c + 1] (binary search), so a cell holding many
// queries (a plane seen edge-on) spreads over many SMs.
__global__ void __launch_bounds__(CF_THREADS) cfield_cell_kernel(
    const float* pts, const int32_t* qidx, const int2* qranges, const int64_t* chunk_off, int ncells, float ox,
    float oy, float oz, const float* rec, const float* near, const int32_t* cell_ids, const int2* cell_ranges,
    const int32_t* global_ids, int64_t n_global, uint32_t* out, unsigned long long* pair_counter) {
  __shared__ float4 s_g[CF_THREADS * 3];
  __shared__ float4 s_c[CF_THREADS];  // mean - origin, |mean - origin|^2
  __shared__ float s_near[CF_THREADS];
  const int64_t w = blockIdx.x;
  if (w >= chunk_off[ncells]) return;
  int lo = 0, hi = ncells - 1;  // largest c with chunk_off[c] <= w
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (chunk_off[mid] <= w) lo = mid; else hi = mid - 1;
  }
  const int2 qr = qranges[lo];
  field_chunk(pts, qidx, qr.x + (int)(w - chunk_off[lo]) * CF_THREADS, qr.y, ox, oy, oz, rec, near, cell_ids,
              cell_ranges[lo], global_ids, n_global, out, s_g, s_c, s_near, pair_counter);
}

// ------------------------------------------------------------------ field plan
// A plan holds every view's candidate lists (built once per Gaussian set and origin
// set); an evaluation sorts its queries by (view, cell) in one pass and hands out
// (view, cell, chunk) work items from a queue.

// query i of view v: key v * (ncells + 1) + cell, ncells for a query at the origin
// (whose field is 0 for that view, set here)
__global__ void cfield_plan_qcell_kernel(const float* pts, int64_t np, const float* origins, int nc, int F,
                                         int sub_bits, int dist_bits, uint32_t* qkey, int32_t* qidx, uint32_t* out) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= np * nc) return;
  const int v = (int)(j / np);
  const int64_t i = j - (int64_t)v * np;
  const float dx = pts[i * 3] - origins[v * 3], dy = pts[i * 3 + 1] - origins[v * 3 + 1],
              dz = pts[i * 3 + 2] - origins[v * 3 + 2];
  const bool at_origin = !(dx * dx + dy * dy + dz * dz > 0.f);
  const uint32_t cells = (uint32_t)(6 * F * F);
  uint32_t cell, low;
  query_key_parts(dx, dy, dz, F, sub_bits, dist_bits, cell, low);
  qkey[j] = (((uint32_t)v * (cells + 1) + cell) << (2 * sub_bits + dist_bits)) | low;
  qidx[j] = (int32_t)i;
  if (at_origin) atomicMin(out + i, 0u);
}

// chunks of every (view, cell) key; the at-origin key of each view has none
__global__ void cfield_plan_chunks_kernel(const int2* qranges, int64_t nkeys, int per_view, int32_t* chunks) {
  const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= nkeys) return;
  const int2 r = qranges[k];
  chunks[k] = (k % per_view == per_view - 1) ? 0 : (r.y - r.x + CF_THREADS - 1) / CF_THREADS;
}

// work item list: item chunk_off[k] + j is (key k, chunk j)
__global__ void cfield_plan_items_kernel(const int64_t* chunk_off, int64_t nkeys, int32_t* item_key) {
  const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= nkeys) return;
  for (int64_t w = chunk_off[k]; w < chunk_off[k + 1]; ++w) item_key[w] = (int32_t)k;
}

__global__ void __launch_bounds__(CF_THREADS) cfield_plan_kernel(
    const float* pts, const int32_t* qidx, const int2* qranges, const int64_t* chunk_off, const int32_t* item_key,
    int64_t nkeys, int per_view, const float* origins, const float* rec, const float* near, int64_t ng,
    const int32_t* vals, const int2* cell_ranges, const int64_t* view_info, const int32_t* gids,
    unsigned long long* queue, uint32_t* out) {
  __shared__ float4 s_g[CF_THREADS * 3];
  __shared__ float4 s_c[CF_THREADS];
  __shared__ float s_near[CF_THREADS];
  __shared__ long long s_w;
  const long long total = chunk_off[nkeys];
  const int ncells = per_view - 1;
  for (;;) {
    if (threadIdx.x == 0) s_w = (long long)atomicAdd(queue, 1ull);
    __syncthreads();
    const long long w = s_w;
    __syncthreads();
    if (w >= total) break;
    const int k = item_key[w];
    const int v = k / per_view, cell = k - v * per_view;
    const int2 qr = qranges[k];
    const int64_t base = view_info[v * 2], n_global = view_info[v * 2 + 1];
    field_chunk(pts, qidx, qr.x + (int)(w - chunk_off[k]) * CF_THREADS, qr.y, origins[v * 3], origins[v * 3 + 1],
                origins[v * 3 + 2], rec, near + (int64_t)v * ng, vals + base,
                cell_ranges[(int64_t)v * ncells + cell], gids + (int64_t)v * ng, n_global, out, s_g, s_c, s_near,
                nullptr);
  }
}

}  // namespace

size_t field_workspace_bytes(int64_t n) { return (size_t)n * OF_FLOATS * sizeof(float) + 256; }

cudaError_t launch_opacity_field(const float* pts, int64_t np, const float* means, const float* invcov,
                                 const float* op, int64_t ng, const float* origins, int nc, float* out, void* ws,
                                 cudaStream_t s) {
  if (np == 0) return cudaSuccess;
  uint32_t* o = reinterpret_cast<uint32_t*>(out);
  count_launches(1);
  field_init_kernel<<<(unsigned)((np + 255) / 256), 256, 0, s>>>(o, np);
  float* g = reinterpret_cast<float*>(ws);
  if (ng > 0) {
    count_launches(1);
    field_pack_kernel<<<(unsigned)((ng + 255) / 256), 256, 0, s>>>(means, invcov, op, ng, g);
  }
  const dim3 grid((unsigned)((np + OF_THREADS - 1) / OF_THREADS), (unsigned)nc);
  count_launches(1);
  field_kernel<<<grid, OF_THREADS, 0, s>>>(pts, np, g, ng, origins, o);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ culled launcher
namespace {
size_t aup(size_t v) { return (v + 255) & ~(size_t)255; }
int cube_bits(int F) {
  const int64_t cells = 6LL * F * F;
  int bits = 1;
  while ((1LL << bits) < cells) ++bits;
  return bits;
}
}  // namespace

size_t field_culled_workspace_bytes(int64_t ng, int64_t max_pairs, int F) {
  size_t b = 0;
  b += aup((size_t)ng * CF_REC * sizeof(float));
  b += 2 * aup((size_t)ng * sizeof(int32_t));          // count, global flag
  b += 2 * aup((size_t)(ng + 1) * sizeof(int64_t));    // offsets, global offsets
  b += aup(scan_workspace_bytes(ng));
  b += aup((size_t)ng * sizeof(int32_t));              // global ids
  b += aup((size_t)ng * sizeof(uint32_t));             // depth keys
  b += aup((size_t)ng * sizeof(float));                // near distances
  b += aup((size_t)ng * sizeof(int32_t));              // depth order
  b += aup(bin_workspace_bytes(ng, 0, 0));             // depth sort scratch
  b += 2 * aup((size_t)max_pairs * sizeof(uint32_t));  // keys, ids
  b += aup(sort_pairs_workspace_bytes(max_pairs));
  b += aup((size_t)6 * F * F * 2 * sizeof(int32_t));   // cell ranges
  return b;
}

// per-query buffers of the culled field (sorted by cell each view)
size_t field_culled_query_bytes(int64_t np, int F) {
  const int64_t cells = 6LL * F * F + 1;
  return 2 * aup((size_t)np * sizeof(uint32_t)) + aup(sort_pairs_workspace_bytes(np)) +
         aup((size_t)cells * 2 * sizeof(int32_t)) + aup((size_t)cells * sizeof(int32_t)) +
         aup((size_t)(cells + 1) * sizeof(int64_t)) + aup(scan_workspace_bytes(cells));
}

cudaError_t launch_opacity_field_culled(const float* pts, int64_t np, const float* means, const float* invcov,
                                        const float* op, int64_t ng, const float* origins, int nc, float cutoff,
                                        int F, float* out, void* ws, size_t ws_bytes, int64_t max_pairs,
                                        int64_t* pairs_needed, cudaStream_t s, unsigned long long* pair_counter,
                                        float* query_ms) {
  if (ws_bytes < field_culled_workspace_bytes(ng, max_pairs, F) + field_culled_query_bytes(np, F))
    return cudaErrorInvalidValue;
  uint32_t* o = reinterpret_cast<uint32_t*>(out);
  if (np == 0) return cudaSuccess;
  count_launches(1);
  field_init_kernel<<<(unsigned)((np + 255) / 256), 256, 0, s>>>(o, np);
  if (ng == 0 || nc == 0) return cudaGetLastError();
  char* p = reinterpret_cast<char*>(ws);
  auto take = [&](size_t bytes) { char* r = p; p += aup(bytes); return r; };
  float* rec = reinterpret_cast<float*>(take((size_t)ng * CF_REC * sizeof(float)));
  int32_t* count = reinterpret_cast<int32_t*>(take((size_t)ng * sizeof(int32_t)));
  int32_t* gflag = reinterpret_cast<int32_t*>(take((size_t)ng * sizeof(int32_t)));
  int64_t* offs = reinterpret_cast<int64_t*>(take((size_t)(ng + 1) * sizeof(int64_t)));
  int64_t* goffs = reinterpret_cast<int64_t*>(take((size_t)(ng + 1) * sizeof(int64_t)));
  const size_t scan_bytes = scan_workspace_bytes(ng);
  void* scan_ws = take(scan_bytes);
  int32_t* gids = reinterpret_cast<int32_t*>(take((size_t)ng * sizeof(int32_t)));
  uint32_t* dkey = reinterpret_cast<uint32_t*>(take((size_t)ng * sizeof(uint32_t)));
  float* near = reinterpret_cast<float*>(take((size_t)ng * sizeof(float)));
  int32_t* order = reinterpret_cast<int32_t*>(take((size_t)ng * sizeof(int32_t)));
  const size_t order_ws_bytes = bin_workspace_bytes(ng, 0, 0);
  void* order_ws = take(order_ws_bytes);
  uint32_t* keys = reinterpret_cast<uint32_t*>(take((size_t)max_pairs * sizeof(uint32_t)));
  int32_t* vals = reinterpret_cast<int32_t*>(take((size_t)max_pairs * sizeof(int32_t)));
  const size_t sort_bytes = sort_pairs_workspace_bytes(max_pairs);
  void* sort_ws = take(sort_bytes);
  int32_t* ranges = reinterpret_cast<int32_t*>(take((size_t)6 * F * F * 2 * sizeof(int32_t)));
  uint32_t* qkey = reinterpret_cast<uint32_t*>(take((size_t)np * sizeof(uint32_t)));
  int32_t* qidx = reinterpret_cast<int32_t*>(take((size_t)np * sizeof(int32_t)));
  const size_t qsort_bytes = sort_pairs_workspace_bytes(np);
  void* qsort_ws = take(qsort_bytes);
  int32_t* qranges = reinterpret_cast<int32_t*>(take((size_t)(6 * F * F + 1) * 2 * sizeof(int32_t)));
  const int ncells = 6 * F * F;
  int32_t* chunks = reinterpret_cast<int32_t*>(take((size_t)(ncells + 1) * sizeof(int32_t)));
  int64_t* chunk_off = reinterpret_cast<int64_t*>(take((size_t)(ncells + 2) * sizeof(int64_t)));
  const size_t cscan_bytes = scan_workspace_bytes(ncells + 1);
  void* cscan_ws = take(cscan_bytes);
  int qbits = 1;
  while ((1LL << qbits) < 6LL * F * F + 1) ++qbits;
  int sub_bits, dist_bits;
  query_order_bits(qbits, sub_bits, dist_bits);
  const int qlow = 2 * sub_bits + dist_bits;
  qbits += qlow;

  const unsigned gb = (unsigned)((ng + 255) / 256), qb = (unsigned)((np + 255) / 256);
  count_launches(1);
  cfield_prep_kernel<<<gb, 256, 0, s>>>(means, invcov, op, ng, cutoff, rec);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  float* host_origins = new float[(size_t)nc * 3];
  e = cudaMemcpyAsync(host_origins, origins, (size_t)nc * 3 * sizeof(float), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  int64_t most = 0;
  // first pass: the largest per-view candidate count, so that an undersized workspace
  // is reported before any view is evaluated
  for (int v = 0; v < nc && e == cudaSuccess; ++v) {
    const float ox = host_origins[v * 3], oy = host_origins[v * 3 + 1], oz = host_origins[v * 3 + 2];
    count_launches(1);
    cfield_count_kernel<<<gb, 256, 0, s>>>(rec, ng, ox, oy, oz, F, count, gflag, dkey, near);
    e = cudaGetLastError();
    if (e == cudaSuccess) e = scan_counts(count, ng, offs, scan_ws, scan_bytes, s);
    int64_t total = 0;
    if (e == cudaSuccess) e = cudaMemcpyAsync(&total, offs + ng, sizeof(int64_t), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (total > most) most = total;
  }
  if (e != cudaSuccess || most > max_pairs) {
    delete[] host_origins;
    if (pairs_needed) *pairs_needed = most;
    return e;
  }
  // optional timing of the query kernels (CUDA events on the launching stream)
  cudaEvent_t ev[2] = {nullptr, nullptr};
  if (query_ms) {
    if (e == cudaSuccess) e = cudaEventCreate(&ev[0]);
    if (e == cudaSuccess) e = cudaEventCreate(&ev[1]);
  }
  for (int v = 0; v < nc && e == cudaSuccess; ++v) {
    const float ox = host_origins[v * 3], oy = host_origins[v * 3 + 1], oz = host_origins[v * 3 + 2];
    count_launches(1);
    cfield_count_kernel<<<gb, 256, 0, s>>>(rec, ng, ox, oy, oz, F, count, gflag, dkey, near);
    e = cudaGetLastError();
    // stable order by nearest ball distance, and the counts' exclusive scan in that order
    if (e == cudaSuccess) e = bin_order(count, dkey, ng, order, offs, order_ws, order_ws_bytes, s);
    if (e == cudaSuccess) e = scan_counts(gflag, ng, goffs, scan_ws, scan_bytes, s);
    int64_t totals[2] = {0, 0};
    if (e == cudaSuccess) e = cudaMemcpyAsync(&totals[0], offs + ng, sizeof(int64_t), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(&totals[1], goffs + ng, sizeof(int64_t), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) break;
    const int64_t m = totals[0], n_global = totals[1];
    if (m > max_pairs) break;  // cannot happen after the first pass
    count_launches(1);
    cfield_emit_kernel<<<gb, 256, 0, s>>>(rec, ng, ox, oy, oz, F, order, offs, goffs, keys, vals, gids);
    e = cudaGetLastError();
    if (e == cudaSuccess) e = sort_pairs(keys, vals, m, cube_bits(F), sort_ws, sort_bytes, s);
    if (e == cudaSuccess) e = key_ranges(keys, m, 6LL * F * F, ranges, s);
    if (e != cudaSuccess) break;
    count_launches(1);
    cfield_qcell_kernel<<<qb, 256, 0, s>>>(pts, np, ox, oy, oz, F, sub_bits, dist_bits, qkey, qidx, o);
    e = cudaGetLastError();
    if (e == cudaSuccess) e = sort_pairs(qkey, qidx, np, qbits, qsort_ws, qsort_bytes, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(qranges, 0, sizeof(int2) * (size_t)(6LL * F * F + 1), s);
    if (e == cudaSuccess && np > 0) {
      count_launches(1);
      cfield_cell_ranges_kernel<<<qb, 256, 0, s>>>(qkey, np, qlow, reinterpret_cast<int2*>(qranges));
      e = cudaGetLastError();
    }
    if (e != cudaSuccess) break;
    count_launches(1);
    cfield_chunks_kernel<<<(unsigned)((ncells + 255) / 256), 256, 0, s>>>(reinterpret_cast<const int2*>(qranges),
                                                                           ncells, chunks);
    e = cudaGetLastError();
    if (e == cudaSuccess) e = scan_counts(chunks, ncells, chunk_off, cscan_ws, cscan_bytes, s);
    if (e != cudaSuccess) break;
    // at most one partial chunk per cell beyond the full ones
    const int64_t max_items = (np + CF_THREADS - 1) / CF_THREADS + ncells;
    if (query_ms && e == cudaSuccess) e = cudaEventRecord(ev[0], s);
    count_launches(1);
    cfield_cell_kernel<<<(unsigned)max_items, CF_THREADS, 0, s>>>(
        pts, qidx, reinterpret_cast<const int2*>(qranges), chunk_off, ncells, ox, oy, oz, rec, near, vals,
        reinterpret_cast<const int2*>(ranges), gids, n_global, o, pair_counter);
    e = cudaGetLastError();
    if (query_ms && e == cudaSuccess) {
      // the next view's count read synchronizes the stream anyway
      e = cudaEventRecord(ev[1], s);
      if (e == cudaSuccess) e = cudaEventSynchronize(ev[1]);
      float ms = 0.f;
      if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, ev[0], ev[1]);
      *query_ms += ms;
    }
  }
  if (query_ms) {
    cudaEventDestroy(ev[0]);
    cudaEventDestroy(ev[1]);
  }
  delete[] host_origins;
  if (pairs_needed) *pairs_needed = most;
  return e;
}

// ------------------------------------------------------------------ field plan
namespace {

struct PlanLayout {
  float* rec; float* near; int32_t* gids; int32_t* ranges; int64_t* view_info; int32_t* vals;
  // build scratch
  int32_t* count; int32_t* gflag; int64_t* offs; int64_t* goffs; void* scan_ws; size_t scan_bytes;
  uint32_t* dkey; int32_t* order; void* order_ws; size_t order_bytes; uint32_t* keys; void* sort_ws;
  size_t sort_bytes;
  size_t used;
};

PlanLayout plan_layout(void* base, int64_t ng, int nc, int F, int64_t total_pairs, int64_t max_view_pairs) {
  PlanLayout L{};
  char* p = reinterpret_cast<char*>(base);
  size_t used = 0;
  auto take = [&](size_t bytes) { char* r = p ? p + used : nullptr; used += aup(bytes); return r; };
  const int64_t ncells = 6LL * F * F;
  L.rec = reinterpret_cast<float*>(take((size_t)ng * CF_REC * sizeof(float)));
  L.near = reinterpret_cast<float*>(take((size_t)nc * ng * sizeof(float)));
  L.gids = reinterpret_cast<int32_t*>(take((size_t)nc * ng * sizeof(int32_t)));
  L.ranges = reinterpret_cast<int32_t*>(take((size_t)nc * ncells * 2 * sizeof(int32_t)));
  L.view_info = reinterpret_cast<int64_t*>(take((size_t)nc * 2 * sizeof(int64_t)));
  L.vals = reinterpret_cast<int32_t*>(take((size_t)total_pairs * sizeof(int32_t)));
  L.count = reinterpret_cast<int32_t*>(take((size_t)ng * sizeof(int32_t)));
  L.gflag = reinterpret_cast<int32_t*>(take((size_t)ng * sizeof(int32_t)));
  L.offs = reinterpret_cast<int64_t*>(take((size_t)(ng + 1) * sizeof(int64_t)));
  L.goffs = reinterpret_cast<int64_t*>(take((size_t)(ng + 1) * sizeof(int64_t)));
  L.scan_bytes = scan_workspace_bytes(ng);
  L.scan_ws = take(L.scan_bytes);
  L.dkey = reinterpret_cast<uint32_t*>(take((size_t)ng * sizeof(uint32_t)));
  L.order = reinterpret_cast<int32_t*>(take((size_t)ng * sizeof(int32_t)));
  L.order_bytes = bin_workspace_bytes(ng, 0, 0);
  L.order_ws = take(L.order_bytes);
  L.keys = reinterpret_cast<uint32_t*>(take((size_t)max_view_pairs * sizeof(uint32_t)));
  L.sort_bytes = sort_pairs_workspace_bytes(max_view_pairs);
  L.sort_ws = take(L.sort_bytes);
  L.used = used;
  return L;
}

struct PlanQueryLayout {
  uint32_t* qkey; int32_t* qidx; void* sort_ws; size_t sort_bytes; int32_t* qranges; int32_t* chunks;
  int64_t* chunk_off; void* scan_ws; size_t scan_bytes; int32_t* item_key; unsigned long long* queue;
  size_t used;
};

PlanQueryLayout plan_query_layout(void* base, int64_t np, int nc, int F) {
  PlanQueryLayout L{};
  char* p = reinterpret_cast<char*>(base);
  size_t used = 0;
  auto take = [&](size_t bytes) { char* r = p ? p + used : nullptr; used += aup(bytes); return r; };
  const int64_t n = np * nc, nkeys = (int64_t)nc * (6LL * F * F + 1);
  L.qkey = reinterpret_cast<uint32_t*>(take((size_t)n * sizeof(uint32_t)));
  L.qidx = reinterpret_cast<int32_t*>(take((size_t)n * sizeof(int32_t)));
  L.sort_bytes = sort_pairs_workspace_bytes(n);
  L.sort_ws = take(L.sort_bytes);
  L.qranges = reinterpret_cast<int32_t*>(take((size_t)nkeys * 2 * sizeof(int32_t)));
  L.chunks = reinterpret_cast<int32_t*>(take((size_t)nkeys * sizeof(int32_t)));
  L.chunk_off = reinterpret_cast<int64_t*>(take((size_t)(nkeys + 1) * sizeof(int64_t)));
  L.scan_bytes = scan_workspace_bytes(nkeys);
  L.scan_ws = take(L.scan_bytes);
  // at most one partial chunk per key beyond the full ones
  L.item_key = reinterpret_cast<int32_t*>(take((size_t)((n + CF_THREADS - 1) / CF_THREADS + nkeys) * sizeof(int32_t)));
  L.queue = reinterpret_cast<unsigned long long*>(take(sizeof(unsigned long long)));
  L.used = used;
  return L;
}

}  // namespace

size_t field_plan_bytes(int64_t ng, int nc, int F, int64_t total_pairs, int64_t max_view_pairs) {
  return plan_layout(nullptr, ng, nc, F, total_pairs, max_view_pairs).used;
}

size_t field_plan_query_bytes(int64_t np, int nc, int F) { return plan_query_layout(nullptr, np, nc, F).used; }

cudaError_t field_plan_build(const float* means, const float* invcov, const float* op, int64_t ng,
                             const float* origins, int nc, float cutoff, int F, void* plan, size_t plan_bytes,
                             int64_t total_pairs, int64_t max_view_pairs, int64_t* needed, cudaStream_t s) {
  const PlanLayout L = plan_layout(plan, ng, nc, F, total_pairs, max_view_pairs);
  if (plan_bytes < L.used) return cudaErrorInvalidValue;
  needed[0] = needed[1] = 0;
  const int64_t ncells = 6LL * F * F;
  std::vector<int64_t> info((size_t)nc * 2, 0);
  cudaError_t e = cudaSuccess;
  if (ng > 0) {
    const unsigned gb = (unsigned)((ng + 255) / 256);
    count_launches(1);
    cfield_prep_kernel<<<gb, 256, 0, s>>>(means, invcov, op, ng, cutoff, L.rec);
    e = cudaGetLastError();
    std::vector<float> o((size_t)nc * 3);
    if (e == cudaSuccess) e = cudaMemcpyAsync(o.data(), origins, o.size() * sizeof(float), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    // first pass: candidate pairs of every view, so that undersized lists are reported
    // before anything is written
    int64_t sum = 0, most = 0;
    for (int v = 0; v < nc && e == cudaSuccess; ++v) {
      count_launches(1);
      cfield_count_kernel<<<gb, 256, 0, s>>>(L.rec, ng, o[v * 3], o[v * 3 + 1], o[v * 3 + 2], F, L.count, L.gflag,
                                             L.dkey, L.near + (int64_t)v * ng);
      e = cudaGetLastError();
      if (e == cudaSuccess) e = scan_counts(L.count, ng, L.offs, L.scan_ws, L.scan_bytes, s);
      int64_t m = 0;
      if (e == cudaSuccess) e = cudaMemcpyAsync(&m, L.offs + ng, sizeof(int64_t), cudaMemcpyDeviceToHost, s);
      if (e == cudaSuccess) e = cudaStreamSynchronize(s);
      sum += m;
      most = m > most ? m : most;
    }
    needed[0] = sum;
    needed[1] = most;
    if (e != cudaSuccess || sum > total_pairs || most > max_view_pairs) return e;
    int64_t base = 0;
    for (int v = 0; v < nc && e == cudaSuccess; ++v) {
      float* near_v = L.near + (int64_t)v * ng;
      count_launches(1);
      cfield_count_kernel<<<gb, 256, 0, s>>>(L.rec, ng, o[v * 3], o[v * 3 + 1], o[v * 3 + 2], F, L.count, L.gflag,
                                             L.dkey, near_v);
      e = cudaGetLastError();
      if (e == cudaSuccess) e = bin_order(L.count, L.dkey, ng, L.order, L.offs, L.order_ws, L.order_bytes, s);
      if (e == cudaSuccess) e = scan_counts(L.gflag, ng, L.goffs, L.scan_ws, L.scan_bytes, s);
      int64_t totals[2] = {0, 0};
      if (e == cudaSuccess) e = cudaMemcpyAsync(&totals[0], L.offs + ng, sizeof(int64_t), cudaMemcpyDeviceToHost, s);
      if (e == cudaSuccess) e = cudaMemcpyAsync(&totals[1], L.goffs + ng, sizeof(int64_t), cudaMemcpyDeviceToHost, s);
      if (e == cudaSuccess) e = cudaStreamSynchronize(s);
      if (e != cudaSuccess) break;
      const int64_t m = totals[0];
      int32_t* vals_v = L.vals + base;
      count_launches(1);
      cfield_emit_kernel<<<gb, 256, 0, s>>>(L.rec, ng, o[v * 3], o[v * 3 + 1], o[v * 3 + 2], F, L.order, L.offs,
                                            L.goffs, L.keys, vals_v, L.gids + (int64_t)v * ng);
      e = cudaGetLastError();
      if (e == cudaSuccess) e = sort_pairs(L.keys, vals_v, m, cube_bits(F), L.sort_ws, L.sort_bytes, s);
      if (e == cudaSuccess) e = key_ranges(L.keys, m, ncells, L.ranges + (int64_t)v * ncells * 2, s);
      info[(size_t)v * 2] = base;
      info[(size_t)v * 2 + 1] = totals[1];
      base += m;
    }
  } else {
    e = cudaMemsetAsync(L.ranges, 0, (size_t)nc * ncells * 2 * sizeof(int32_t), s);
  }
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(L.view_info, info.data(), info.size() * sizeof(int64_t), cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);  // `info` is host stack memory
  return e;
}

cudaError_t field_plan_eval(const void* plan, int64_t ng, int nc, int F, int64_t total_pairs, int64_t max_view_pairs,
                            const float* origins, const float* pts, int64_t np, float* out, void* ws, size_t ws_bytes,
                            cudaStream_t s) {
  const PlanLayout P = plan_layout(const_cast<void*>(plan), ng, nc, F, total_pairs, max_view_pairs);
  const PlanQueryLayout Q = plan_query_layout(ws, np, nc, F);
  if (ws_bytes < Q.used) return cudaErrorInvalidValue;
  if (np == 0) return cudaSuccess;
  uint32_t* o = reinterpret_cast<uint32_t*>(out);
  count_launches(1);
  field_init_kernel<<<(unsigned)((np + 255) / 256), 256, 0, s>>>(o, np);
  const int64_t n = np * nc;
  const int per_view = 6 * F * F + 1;
  const int64_t nkeys = (int64_t)nc * per_view;
  int qbits = 1;
  while ((1LL << qbits) < nkeys) ++qbits;
  int sub_bits, dist_bits;
  query_order_bits(qbits, sub_bits, dist_bits);
  const int qlow = 2 * sub_bits + dist_bits;
  qbits += qlow;
  count_launches(1);
  cfield_plan_qcell_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(pts, np, origins, nc, F, sub_bits, dist_bits,
                                                                      Q.qkey, Q.qidx, o);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = sort_pairs(Q.qkey, Q.qidx, n, qbits, Q.sort_ws, Q.sort_bytes, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(Q.qranges, 0, sizeof(int2) * (size_t)nkeys, s);
  if (e == cudaSuccess) {
    count_launches(1);
    cfield_cell_ranges_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(Q.qkey, n, qlow,
                                                                         reinterpret_cast<int2*>(Q.qranges));
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) return e;
  const unsigned kb = (unsigned)((nkeys + 255) / 256);
  count_launches(1);
  cfield_plan_chunks_kernel<<<kb, 256, 0, s>>>(reinterpret_cast<const int2*>(Q.qranges), nkeys, per_view, Q.chunks);
  e = cudaGetLastError();
  if (e == cudaSuccess) e = scan_counts(Q.chunks, nkeys, Q.chunk_off, Q.scan_ws, Q.scan_bytes, s);
  if (e != cudaSuccess) return e;
  count_launches(1);
  cfield_plan_items_kernel<<<kb, 256, 0, s>>>(Q.chunk_off, nkeys, Q.item_key);
  e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaMemsetAsync(Q.queue, 0, sizeof(unsigned long long), s);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  count_launches(1);
  cfield_plan_kernel<<<(unsigned)(sms * 6), CF_THREADS, 0, s>>>(
      pts, Q.qidx, reinterpret_cast<const int2*>(Q.qranges), Q.chunk_off, Q.item_key, nkeys, per_view, origins, P.rec,
      P.near, ng, P.vals, reinterpret_cast<const int2*>(P.ranges), P.view_info, P.gids, Q.queue, o);
  return cudaGetLastError();
}

}  // namespace sf
