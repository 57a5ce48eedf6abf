// Device stages of the GOF mesh extraction.
//
// * grid points: every seed Gaussian's centre and the 8 corners of its extent-sigma box
//   along its own axes, in float64, with the per-Gaussian vertex radius
//   (src/splatforge/studio/exporters.py:20-38).  Deduplication and the Delaunay
//   triangulation of those points stay on the host, as in the reference.
// * marching tetrahedra with shared-edge bisection (src/splatforge/mesh/tetrahedra.py:34-109):
//   inside flags, active cells, the crossing edges of every active cell, their
//   deduplication in (low vertex, high vertex) order, the bisection updates between the
//   caller's field evaluations, and one or two oriented faces per active cell with the
//   degenerate-area filter.
//
// Every float64 expression is evaluated with explicitly rounded operations in the
// reference's order, so with the same field values the vertex positions, the face list,
// its order and every orientation decision are the reference's exactly.

#include "sf_kernels.h"
#include "sf_math.cuh"

namespace sf {
namespace {

constexpr int MT_THREADS = 256;

inline unsigned grid_of(int64_t n) { return (unsigned)((n + MT_THREADS - 1) / MT_THREADS); }

// the six edges of a tetrahedron, itertools.combinations(range(4), 2) order
__device__ __forceinline__ int edge_a(int e) { return e < 3 ? 0 : (e < 5 ? 1 : 2); }
__device__ __forceinline__ int edge_b(int e) { return e < 3 ? e + 1 : (e < 5 ? e - 1 : 3); }
// index of the edge (a, b), a < b
__device__ __forceinline__ int edge_index(int a, int b) { return a == 0 ? b - 1 : (a == 1 ? b + 1 : 5); }

__device__ __forceinline__ double dadd(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ double dsub(double a, double b) { return __dsub_rn(a, b); }
__device__ __forceinline__ double dmul(double a, double b) { return __dmul_rn(a, b); }

__device__ __forceinline__ bool is_inside(double v, double level, int greater) {
  return greater ? v >= level : v <= level;
}

// bit k of the mask = vertex k of the cell is inside
__device__ __forceinline__ int cell_mask(const int4 v, const uint8_t* inside) {
  return (int)inside[v.x] | ((int)inside[v.y] << 1) | ((int)inside[v.z] << 2) | ((int)inside[v.w] << 3);
}

__device__ __forceinline__ int cell_vertex(const int4 v, int k) {
  return k == 0 ? v.x : (k == 1 ? v.y : (k == 2 ? v.z : v.w));
}

// -------------------------------------------------------------------- grid points
__global__ void grid_points_kernel(const float* means, const float* quats, const float* scales,
                                   const int32_t* chosen, int64_t n, double extent, double* points,
                                   double* radius) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int64_t g = chosen[i];
  float qn[4], R[9];
  quat_normalize(quats + g * 4, qn);
  quat_rotation(qn, R);
  const float s[3] = {scales[g * 3], scales[g * 3 + 1], scales[g * 3 + 2]};
  // the radius is a float32 product (scale max times the extent rounded to float32)
  radius[i] = (double)__fmul_rn(fmaxf(fmaxf(s[0], s[1]), s[2]), (float)extent);
  double* out = points + i * 27;
  for (int k = 0; k < 9; ++k) {
    // k = 0: the centre; k >= 1: signs of itertools.product((-1, 1), repeat=3)
    double l[3];
    for (int j = 0; j < 3; ++j) {
      const double sign = k == 0 ? 0.0 : ((((k - 1) >> (2 - j)) & 1) ? 1.0 : -1.0);
      l[j] = dmul(dmul(sign, (double)s[j]), extent);
    }
    for (int r = 0; r < 3; ++r) {
      const double rot = dadd(dadd(dmul((double)R[r * 3], l[0]), dmul((double)R[r * 3 + 1], l[1])),
                              dmul((double)R[r * 3 + 2], l[2]));
      out[k * 3 + r] = dadd((double)means[g * 3 + r], rot);
    }
  }
}

// -------------------------------------------------------------------- classification
__global__ void mt_inside_kernel(const double* values, int64_t n, double level, int greater, uint8_t* inside) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) inside[i] = is_inside(values[i], level, greater) ? 1 : 0;
}

// crossing edges (3 for a 1/3 split, 4 for 2/2) and faces (1 or 2) of every cell
__global__ void mt_count_kernel(const int4* cells, int64_t n_cells, const uint8_t* inside, int32_t* slots,
                                int32_t* faces) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= n_cells) return;
  const int m = cell_mask(cells[c], inside);
  const bool active = m != 0 && m != 15;
  const bool split2 = __popc(m) == 2;
  slots[c] = active ? (split2 ? 4 : 3) : 0;
  faces[c] = active ? (split2 ? 2 : 1) : 0;
}

// the crossing edges of each active cell as (low, high) vertex pairs, in edge order
__global__ void mt_edges_kernel(const int4* cells, int64_t n_cells, const uint8_t* inside,
                                const int64_t* slot_off, uint32_t* key_lo, uint32_t* key_hi, int32_t* slot) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= n_cells) return;
  int64_t s = slot_off[c];
  if (slot_off[c + 1] == s) return;
  const int4 v = cells[c];
  const int m = cell_mask(v, inside);
  for (int e = 0; e < 6; ++e) {
    const int a = edge_a(e), b = edge_b(e);
    if (((m >> a) ^ (m >> b)) & 1) {
      const int va = cell_vertex(v, a), vb = cell_vertex(v, b);
      key_lo[s] = (uint32_t)min(va, vb);
      key_hi[s] = (uint32_t)max(va, vb);
      slot[s] = (int32_t)s;
      ++s;
    }
  }
}

__global__ void gather_u32_kernel(const uint32_t* src, const int32_t* idx, int64_t n, uint32_t* dst) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = src[idx[i]];
}

// 1 where a sorted pair differs from its predecessor
__global__ void mt_unique_flags_kernel(const int32_t* order, const uint32_t* key_lo, const uint32_t* key_hi,
                                       int64_t n, int32_t* flag) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int32_t o = order[i];
  if (i == 0) {
    flag[i] = 1;
    return;
  }
  const int32_t p = order[i - 1];
  flag[i] = (key_lo[o] != key_lo[p] || key_hi[o] != key_hi[p]) ? 1 : 0;
}

__global__ void mt_unique_emit_kernel(const int32_t* order, const uint32_t* key_lo, const uint32_t* key_hi,
                                      int64_t n, const int64_t* upos, const double* points,
                                      const uint8_t* inside, int32_t* edge_uid, int32_t* pairs, double* low,
                                      double* high, uint8_t* low_inside) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int32_t o = order[i];
  const int64_t u = upos[i + 1] - 1;
  edge_uid[o] = (int32_t)u;
  if (upos[i + 1] == upos[i]) return;
  const uint32_t a = key_lo[o], b = key_hi[o];
  pairs[u * 2] = (int32_t)a;
  pairs[u * 2 + 1] = (int32_t)b;
  for (int r = 0; r < 3; ++r) {
    low[u * 3 + r] = points[(int64_t)a * 3 + r];
    high[u * 3 + r] = points[(int64_t)b * 3 + r];
  }
  low_inside[u] = inside[a];
}

// -------------------------------------------------------------------- bisection
__global__ void mt_midpoints_kernel(const double* low, const double* high, int64_t n3, double* mid) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n3) mid[i] = dmul(dadd(low[i], high[i]), 0.5);
}

__global__ void mt_bisect_kernel(double* low, double* high, const uint8_t* low_inside, int64_t n,
                                 const double* values, double level, int greater) {
  const int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (u >= n) return;
  const bool same = is_inside(values[u], level, greater) == (low_inside[u] != 0);
  double* dst = same ? low : high;
  for (int r = 0; r < 3; ++r) dst[u * 3 + r] = dmul(dadd(low[u * 3 + r], high[u * 3 + r]), 0.5);
}

// -------------------------------------------------------------------- faces
__device__ __forceinline__ void edge_vertex(const double* low, const double* high, int32_t u, double* p) {
  for (int r = 0; r < 3; ++r) p[r] = dmul(dadd(low[(int64_t)u * 3 + r], high[(int64_t)u * 3 + r]), 0.5);
}

__device__ __forceinline__ void cross3d(const double* a, const double* b, double* c) {
  c[0] = dsub(dmul(a[1], b[2]), dmul(a[2], b[1]));
  c[1] = dsub(dmul(a[2], b[0]), dmul(a[0], b[2]));
  c[2] = dsub(dmul(a[0], b[1]), dmul(a[1], b[0]));
}

// orients one face against `outward` and reports whether its area passes the filter
__device__ __forceinline__ bool orient_face(const double* low, const double* high, int32_t* f, const double* outward) {
  double v0[3], v1[3], v2[3], e1[3], e2[3], c[3];
  edge_vertex(low, high, f[0], v0);
  edge_vertex(low, high, f[1], v1);
  edge_vertex(low, high, f[2], v2);
  for (int r = 0; r < 3; ++r) {
    e1[r] = dsub(v1[r], v0[r]);
    e2[r] = dsub(v2[r], v0[r]);
  }
  cross3d(e1, e2, c);
  const double d = dadd(dadd(dmul(c[0], outward[0]), dmul(c[1], outward[1])), dmul(c[2], outward[2]));
  if (d < 0.0) {
    const int32_t t = f[1];
    f[1] = f[2];
    f[2] = t;
  }
  // the swap only negates the cross product, so its norm is the same either way
  const double area = __dsqrt_rn(dadd(dadd(dmul(c[0], c[0]), dmul(c[1], c[1])), dmul(c[2], c[2])));
  return area > 1e-16;
}

__global__ void mt_faces_kernel(const double* points, const int4* cells, int64_t n_cells, const uint8_t* inside,
                                const int64_t* slot_off, const int32_t* edge_uid, const double* low,
                                const double* high, const int64_t* face_off, int64_t* faces, int32_t* keep) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= n_cells) return;
  int64_t f = face_off[c];
  if (face_off[c + 1] == f) return;
  const int4 v = cells[c];
  const int m = cell_mask(v, inside);
  int32_t row[6];
  int64_t s = slot_off[c];
  for (int e = 0; e < 6; ++e) row[e] = (((m >> edge_a(e)) ^ (m >> edge_b(e))) & 1) ? edge_uid[s++] : -1;
  int inn[4], out[4], n_in = 0, n_out = 0;
  for (int k = 0; k < 4; ++k) {
    if ((m >> k) & 1) inn[n_in++] = k;
    else out[n_out++] = k;
  }
  // outward = mean of the outside vertices - mean of the inside vertices
  double outward[3];
  for (int r = 0; r < 3; ++r) {
    double so = points[(int64_t)cell_vertex(v, out[0]) * 3 + r];
    for (int k = 1; k < n_out; ++k) so = dadd(so, points[(int64_t)cell_vertex(v, out[k]) * 3 + r]);
    double si = points[(int64_t)cell_vertex(v, inn[0]) * 3 + r];
    for (int k = 1; k < n_in; ++k) si = dadd(si, points[(int64_t)cell_vertex(v, inn[k]) * 3 + r]);
    outward[r] = dsub(__ddiv_rn(so, (double)n_out), __ddiv_rn(si, (double)n_in));
  }
  auto get = [&](int x, int y) { return row[edge_index(min(x, y), max(x, y))]; };
  int32_t tri[2][3];
  int nt = 1;
  if (n_in == 1 || n_in == 3) {
    const int pivot = n_in == 1 ? inn[0] : out[0];
    const int* rest = n_in == 1 ? out : inn;
    for (int k = 0; k < 3; ++k) tri[0][k] = get(pivot, rest[k]);
  } else {
    const int a = inn[0], b = inn[1], cc = out[0], d = out[1];
    const int32_t ac = get(a, cc), ad = get(a, d), bc = get(b, cc), bd = get(b, d);
    tri[0][0] = ac; tri[0][1] = ad; tri[0][2] = bc;
    tri[1][0] = ad; tri[1][1] = bd; tri[1][2] = bc;
    nt = 2;
  }
  for (int t = 0; t < nt; ++t, ++f) {
    keep[f] = orient_face(low, high, tri[t], outward) ? 1 : 0;
    for (int k = 0; k < 3; ++k) faces[f * 3 + k] = tri[t][k];
  }
}

__global__ void mt_compact_faces_kernel(const int64_t* faces, const int32_t* keep, const int64_t* kpos, int64_t n,
                                        int64_t* out) {
  const int64_t f = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (f >= n || !keep[f]) return;
  const int64_t d = kpos[f];
  for (int k = 0; k < 3; ++k) out[d * 3 + k] = faces[f * 3 + k];
}

__global__ void mt_vertices_kernel(const double* low, const double* high, int64_t n3, double* vertices) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n3) vertices[i] = dmul(dadd(low[i], high[i]), 0.5);
}

// Bump allocator over a caller's workspace (256-byte aligned slices).
struct Slices {
  char* base;
  size_t used = 0;
  template <class T>
  T* take(int64_t n) {
    T* p = reinterpret_cast<T*>(base ? base + used : nullptr);
    used += ((size_t)n * sizeof(T) + 255) & ~(size_t)255;
    return p;
  }
};

int bits_for(int64_t n) {
  int b = 1;
  while (b < 32 && (int64_t(1) << b) < n) ++b;
  return b;
}

}  // namespace

cudaError_t launch_grid_points(const float* means, const float* quats, const float* scales, const int32_t* chosen,
                               int64_t n, double extent, double* points, double* radius, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  count_launches(1);
  grid_points_kernel<<<grid_of(n), MT_THREADS, 0, s>>>(means, quats, scales, chosen, n, extent, points, radius);
  return cudaGetLastError();
}

size_t mesh_count_workspace_bytes(int64_t n_cells) {
  Slices c{nullptr};
  c.take<int32_t>(n_cells);
  c.take<int32_t>(n_cells);
  c.take<char>(scan_workspace_bytes(n_cells));
  return c.used;
}

cudaError_t mesh_count(const double* values, int64_t n_points, const int32_t* cells, int64_t n_cells, double level,
                       int greater, uint8_t* inside, int64_t* slot_off, int64_t* face_off, void* ws,
                       size_t ws_bytes, cudaStream_t s) {
  if (ws_bytes < mesh_count_workspace_bytes(n_cells)) return cudaErrorInvalidValue;
  Slices c{reinterpret_cast<char*>(ws)};
  int32_t* slots = c.take<int32_t>(n_cells);
  int32_t* faces = c.take<int32_t>(n_cells);
  const size_t scan_bytes = scan_workspace_bytes(n_cells);
  void* scan_ws = c.take<char>(scan_bytes);
  if (n_points > 0) {
    count_launches(1);
    mt_inside_kernel<<<grid_of(n_points), MT_THREADS, 0, s>>>(values, n_points, level, greater, inside);
  }
  if (n_cells == 0) {
    cudaError_t e = cudaMemsetAsync(slot_off, 0, sizeof(int64_t), s);
    return e == cudaSuccess ? cudaMemsetAsync(face_off, 0, sizeof(int64_t), s) : e;
  }
  count_launches(1);
  mt_count_kernel<<<grid_of(n_cells), MT_THREADS, 0, s>>>(reinterpret_cast<const int4*>(cells), n_cells, inside,
                                                            slots, faces);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = scan_counts(slots, n_cells, slot_off, scan_ws, scan_bytes, s);
  if (e == cudaSuccess) e = scan_counts(faces, n_cells, face_off, scan_ws, scan_bytes, s);
  return e;
}

size_t mesh_edges_workspace_bytes(int64_t n_slots) {
  Slices c{nullptr};
  for (int k = 0; k < 4; ++k) c.take<uint32_t>(n_slots);  // lo, hi, sort key, order
  c.take<int32_t>(n_slots);                                // flags
  c.take<int64_t>(n_slots + 1);                            // unique positions
  c.take<char>(scan_workspace_bytes(n_slots));
  c.take<char>(sort_pairs_workspace_bytes(n_slots));
  return c.used;
}

cudaError_t mesh_edges(const double* points, int64_t n_points, const int32_t* cells, int64_t n_cells,
                       const uint8_t* inside, const int64_t* slot_off, int64_t n_slots, int32_t* edge_uid,
                       int32_t* pairs, double* low, double* high, uint8_t* low_inside, int64_t* n_unique,
                       void* ws, size_t ws_bytes, cudaStream_t s) {
  if (ws_bytes < mesh_edges_workspace_bytes(n_slots)) return cudaErrorInvalidValue;
  if (n_slots == 0) return cudaMemsetAsync(n_unique, 0, sizeof(int64_t), s);
  Slices c{reinterpret_cast<char*>(ws)};
  uint32_t* lo = c.take<uint32_t>(n_slots);
  uint32_t* hi = c.take<uint32_t>(n_slots);
  uint32_t* key = c.take<uint32_t>(n_slots);
  int32_t* order = reinterpret_cast<int32_t*>(c.take<uint32_t>(n_slots));
  int32_t* flag = c.take<int32_t>(n_slots);
  int64_t* upos = c.take<int64_t>(n_slots + 1);
  const size_t scan_bytes = scan_workspace_bytes(n_slots);
  void* scan_ws = c.take<char>(scan_bytes);
  const size_t sort_bytes = sort_pairs_workspace_bytes(n_slots);
  void* sort_ws = c.take<char>(sort_bytes);
  const int bits = bits_for(n_points);
  const unsigned g = grid_of(n_slots);

  count_launches(1);
  mt_edges_kernel<<<grid_of(n_cells), MT_THREADS, 0, s>>>(reinterpret_cast<const int4*>(cells), n_cells, inside,
                                                            slot_off, lo, hi, order);
  cudaError_t e = cudaGetLastError();
  // stable LSD order by (lo, hi): by hi, then by lo carrying the permutation
  if (e == cudaSuccess) e = cudaMemcpyAsync(key, hi, (size_t)n_slots * sizeof(uint32_t), cudaMemcpyDeviceToDevice, s);
  if (e == cudaSuccess) e = sort_pairs(key, order, n_slots, bits, sort_ws, sort_bytes, s);
  if (e == cudaSuccess) {
    count_launches(1);
    gather_u32_kernel<<<g, MT_THREADS, 0, s>>>(lo, order, n_slots, key);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = sort_pairs(key, order, n_slots, bits, sort_ws, sort_bytes, s);
  if (e == cudaSuccess) {
    count_launches(1);
    mt_unique_flags_kernel<<<g, MT_THREADS, 0, s>>>(order, lo, hi, n_slots, flag);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = scan_counts(flag, n_slots, upos, scan_ws, scan_bytes, s);
  if (e == cudaSuccess) {
    count_launches(1);
    mt_unique_emit_kernel<<<g, MT_THREADS, 0, s>>>(order, lo, hi, n_slots, upos, points, inside, edge_uid, pairs,
                                                   low, high, low_inside);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(n_unique, upos + n_slots, sizeof(int64_t), cudaMemcpyDeviceToDevice, s);
  return e;
}

cudaError_t mesh_midpoints(const double* low, const double* high, int64_t n_edges, double* mid, cudaStream_t s) {
  if (n_edges == 0) return cudaSuccess;
  count_launches(1);
  mt_midpoints_kernel<<<grid_of(n_edges * 3), MT_THREADS, 0, s>>>(low, high, n_edges * 3, mid);
  return cudaGetLastError();
}

cudaError_t mesh_bisect(double* low, double* high, const uint8_t* low_inside, int64_t n_edges, const double* values,
                        double level, int greater, cudaStream_t s) {
  if (n_edges == 0) return cudaSuccess;
  count_launches(1);
  mt_bisect_kernel<<<grid_of(n_edges), MT_THREADS, 0, s>>>(low, high, low_inside, n_edges, values, level, greater);
  return cudaGetLastError();
}

size_t mesh_faces_workspace_bytes(int64_t n_faces) {
  Slices c{nullptr};
  c.take<int64_t>(n_faces * 3);
  c.take<int32_t>(n_faces);
  c.take<int64_t>(n_faces + 1);
  c.take<char>(scan_workspace_bytes(n_faces));
  return c.used;
}

cudaError_t mesh_faces(const double* points, const int32_t* cells, int64_t n_cells, const uint8_t* inside,
                       const int64_t* slot_off, const int32_t* edge_uid, const double* low, const double* high,
                       int64_t n_edges, const int64_t* face_off, int64_t n_faces, double* vertices, int64_t* faces,
                       int64_t* n_kept, void* ws, size_t ws_bytes, cudaStream_t s) {
  if (ws_bytes < mesh_faces_workspace_bytes(n_faces)) return cudaErrorInvalidValue;
  if (n_edges > 0) {
    count_launches(1);
    mt_vertices_kernel<<<grid_of(n_edges * 3), MT_THREADS, 0, s>>>(low, high, n_edges * 3, vertices);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  if (n_faces == 0) return cudaMemsetAsync(n_kept, 0, sizeof(int64_t), s);
  Slices c{reinterpret_cast<char*>(ws)};
  int64_t* raw = c.take<int64_t>(n_faces * 3);
  int32_t* keep = c.take<int32_t>(n_faces);
  int64_t* kpos = c.take<int64_t>(n_faces + 1);
  const size_t scan_bytes = scan_workspace_bytes(n_faces);
  void* scan_ws = c.take<char>(scan_bytes);
  count_launches(1);
  mt_faces_kernel<<<grid_of(n_cells), MT_THREADS, 0, s>>>(points, reinterpret_cast<const int4*>(cells), n_cells,
                                                            inside, slot_off, edge_uid, low, high, face_off, raw,
                                                            keep);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = scan_counts(keep, n_faces, kpos, scan_ws, scan_bytes, s);
  if (e == cudaSuccess) {
    count_launches(1);
    mt_compact_faces_kernel<<<grid_of(n_faces), MT_THREADS, 0, s>>>(raw, keep, kpos, n_faces, faces);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaMemcpyAsync(n_kept, kpos + n_faces, sizeof(int64_t), cudaMemcpyDeviceToDevice, s);
  return e;
}

}  // namespace sf
