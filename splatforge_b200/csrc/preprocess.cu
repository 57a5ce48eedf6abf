// Per-Gaussian kernels: projection forward/backward (renderers.py:76-107,
// batched_renderer.py:51-115), gaussian.covariance@1 and gaussian.sh_color@1
// (reference.py:33-35, 85-113), and the tile rectangles of tile_binning.py:27-40.
//
// One thread per Gaussian.  The SH block (up to 16x3 floats) dominates the bytes
// read; a CTA stages its Gaussians' coefficients into shared memory with coalesced
// 128-bit loads before the per-thread math.
#include <cuda_runtime.h>

#include "sf_device.cuh"
#include "sf_grad.cuh"
#include "sf_kernels.h"

namespace sf {

namespace {

constexpr int PB = 128;  // Gaussians per CTA

// Copy rows [first, first+rows) of a [N, width] float array into shared memory rows of
// `stride` floats (stride = width + 1: an odd row stride, so that the threads of a warp,
// each reading its own row, hit distinct banks).  128-bit global loads when the slab
// is 16-byte aligned, scalar loads otherwise.
__device__ __forceinline__ int row_stride(int width) { return width + ((width & 1) ^ 1); }

// (row, column) of flat index k of a [rows, width] slab, advanced by a fixed step without
// a division per element: one division at the start, then carries.
struct RowCursor {
  int r, c, dr, dc, width;
  __device__ __forceinline__ RowCursor(int k, int step, int w)
      : r(k / w), c(k - (k / w) * w), dr(step / w), dc(step - (step / w) * w), width(w) {}
  __device__ __forceinline__ void advance() {
    r += dr;
    c += dc;
    if (c >= width) { c -= width; ++r; }
  }
};

__device__ __forceinline__ void stage_rows(float* dst, const float* src, int64_t first, int rows, int width,
                                           int stride) {
  const int count = rows * width;
  const float* base = src + first * width;
  if ((((uintptr_t)base) & 15) == 0 && (count & 3) == 0) {
    const float4* s4 = reinterpret_cast<const float4*>(base);
    RowCursor at(4 * (int)threadIdx.x, 4 * (int)blockDim.x, width);
    for (int k = threadIdx.x; k < count / 4; k += blockDim.x, at.advance()) {
      const float4 v = __ldg(s4 + k);
      const float e[4] = {v.x, v.y, v.z, v.w};
      // the four elements may cross into the next row
      int r = at.r, c = at.c;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        dst[r * stride + c] = e[q];
        if (++c == width) { c = 0; ++r; }
      }
    }
  } else {
    RowCursor at(threadIdx.x, blockDim.x, width);
    for (int k = threadIdx.x; k < count; k += blockDim.x, at.advance()) dst[at.r * stride + at.c] = __ldg(base + k);
  }
}

__device__ __forceinline__ void write_bounds(int64_t i, float x, float y, float r, float z,
                                             int width, int height, float nearp, float farp,
                                             int32_t* rect, int32_t* count, uint32_t* depth_key,
                                             int32_t* nonfinite) {
  int rc[4];
  int c = 0;
  if (!(isfinite(x) && isfinite(y) && isfinite(r) && isfinite(z))) {
    if (nonfinite) atomicAdd(nonfinite, 1);
    rc[0] = rc[1] = rc[2] = rc[3] = 0;
  } else {
    c = tile_rect(x, y, r, z, width, height, TILE, nearp, farp, rc);
  }
  reinterpret_cast<int4*>(rect)[i] = make_int4(rc[0], rc[1], rc[2], rc[3]);
  count[i] = c;
  depth_key[i] = c > 0 ? __float_as_uint(z) : 0xffffffffu;
}

template <int MODE>
__global__ void __launch_bounds__(PB) project_forward_kernel(
    const float* __restrict__ means, const float* __restrict__ quats,
    const float* __restrict__ scales, const float* __restrict__ opacities,
    const float* __restrict__ sh, const uint8_t* __restrict__ selected, int64_t n,
    const sf_camera cam, const sf_settings st, float* __restrict__ means2d,
    float* __restrict__ radii, float* __restrict__ records, int32_t* __restrict__ rect,
    int32_t* __restrict__ count, uint32_t* __restrict__ depth_key, int32_t* nonfinite) {
  extern __shared__ float s_sh[];  // [PB, row_stride(K*3)]
  const int K = st.sh_coeffs;
  const int64_t first = (int64_t)blockIdx.x * PB;
  const int rows = (int)min((int64_t)PB, n - first);
  const int stride = row_stride(K * 3);
  stage_rows(s_sh, sh, first, rows, K * 3, stride);
  __syncthreads();
  if ((int)threadIdx.x >= rows) return;
  const int64_t i = first + threadIdx.x;
  const float m[3] = {means[i * 3], means[i * 3 + 1], means[i * 3 + 2]};
  const float4 q4 = __ldg(reinterpret_cast<const float4*>(quats) + i);
  const float q[4] = {q4.x, q4.y, q4.z, q4.w};
  const float sc[3] = {scales[i * 3], scales[i * 3 + 1], scales[i * 3 + 2]};
  Projection p;
  project(m, q, sc, cam, st.eps2d, st.near_plane, st.extent, p);
  float opa = opacities[i];
  if (st.antialiased) {
    const float detS = p.s00 * p.s11 - p.s01 * p.s01;
    const float detF = p.fa * p.fc - p.fb * p.fb;
    opa = opa * sqrtf(fmaxr(detS, 0.f) / fmaxr(detF, 1e-12f));
  }
  float rec[SF_RECORD_FLOATS];
#pragma unroll
  for (int k = 0; k < SF_RECORD_FLOATS; ++k) rec[k] = 0.f;
  rec[R_X] = p.X; rec[R_Y] = p.Y;
  rec[R_QA] = p.qa; rec[R_QB] = p.qb; rec[R_QC] = p.qc;
  rec[R_OPA] = opa;
  const float dir[3] = {m[0] - cam.origin[0], m[1] - cam.origin[1], m[2] - cam.origin[2]};
  sh_color(s_sh + threadIdx.x * stride, st.sh_degree, dir, rec + R_RGB);
  rec[R_SEL] = selected && selected[i] ? 1.f : 0.f;
  rec[R_Z] = p.mc[2];
  if (MODE == SF_MODE_RADEGS) {
    RadeExtras e;
    rade_extras(p, e);
    rec[R_RADIAL] = e.radial;
    rec[R_GAIN] = e.gain[0]; rec[R_GAIN + 1] = e.gain[1];
    rec[R_NRM] = e.normal[0]; rec[R_NRM + 1] = e.normal[1]; rec[R_NRM + 2] = e.normal[2];
  } else if (MODE == SF_MODE_GOF) {
    const float fx = cam.K[0], fy = cam.K[4], cx = cam.K[2], cy = cam.K[5];
    rec[R_PROXY] = (p.X - cx) * p.mc[2] / fx;
    rec[R_PROXY + 1] = (p.Y - cy) * p.mc[2] / fy;
    rec[R_PROXY + 2] = p.mc[2];
    inv3_sym(p.Cc, rec + R_Q3);
  } else {
    AmbiExtras e;
    ambi_extras(sc, p, cam, e);
    rec[R_ANRM] = e.normal[0]; rec[R_ANRM + 1] = e.normal[1]; rec[R_ANRM + 2] = e.normal[2];
    rec[R_PLANE] = e.plane;
  }
  float4* r4 = reinterpret_cast<float4*>(records + i * SF_RECORD_FLOATS);
#pragma unroll
  for (int k = 0; k < SF_RECORD_FLOATS / 4; ++k)
    r4[k] = make_float4(rec[4 * k], rec[4 * k + 1], rec[4 * k + 2], rec[4 * k + 3]);
  reinterpret_cast<float2*>(means2d)[i] = make_float2(p.X, p.Y);
  radii[i] = p.radius;
  write_bounds(i, p.X, p.Y, p.radius, p.mc[2], cam.width, cam.height, st.near_plane,
               st.far_plane, rect, count, depth_key, nonfinite);
}

template <int MODE>
__global__ void __launch_bounds__(PB) project_backward_kernel(
    const float* __restrict__ means, const float* __restrict__ quats,
    const float* __restrict__ scales, const float* __restrict__ opacities,
    const float* __restrict__ sh, int64_t n, const sf_camera cam, const sf_settings st,
    const float* __restrict__ gxy, const float* __restrict__ grec, float* g_means,
    float* g_quats, float* g_scales, float* g_opacities, float* g_sh) {
  extern __shared__ float s_sh[];  // [PB, row_stride(K*3)] coefficients, then their adjoints
  const int K = st.sh_coeffs;
  const int64_t first = (int64_t)blockIdx.x * PB;
  const int rows = (int)min((int64_t)PB, n - first);
  const int stride = row_stride(K * 3);
  stage_rows(s_sh, sh, first, rows, K * 3, stride);
  __syncthreads();
  if ((int)threadIdx.x < rows) {
    const int64_t i = first + threadIdx.x;
    const float m[3] = {means[i * 3], means[i * 3 + 1], means[i * 3 + 2]};
    const float q[4] = {quats[i * 4], quats[i * 4 + 1], quats[i * 4 + 2], quats[i * 4 + 3]};
    const float sc[3] = {scales[i * 3], scales[i * 3 + 1], scales[i * 3 + 2]};
    float g[SF_RECORD_FLOATS];
    const float4* g4 = reinterpret_cast<const float4*>(grec + i * SF_RECORD_FLOATS);
#pragma unroll
    for (int k = 0; k < SF_RECORD_FLOATS / 4; ++k) {
      const float4 t = g4[k];
      g[4 * k] = t.x; g[4 * k + 1] = t.y; g[4 * k + 2] = t.z; g[4 * k + 3] = t.w;
    }
    const float gx[2] = {gxy[i * 2], gxy[i * 2 + 1]};
    float gm[3], gq[4], gs[3], go;
    float* coeffs = s_sh + threadIdx.x * stride;
    // the SH adjoint replaces the staged coefficients in place (read before written)
    project_backward_mode<MODE>(m, q, sc, opacities[i], coeffs, st.sh_degree, cam, st, gx, g, gm, gq, gs,
                                &go, coeffs);
    if (g_means) { g_means[i * 3] = gm[0]; g_means[i * 3 + 1] = gm[1]; g_means[i * 3 + 2] = gm[2]; }
    if (g_quats)
      reinterpret_cast<float4*>(g_quats)[i] = make_float4(gq[0], gq[1], gq[2], gq[3]);
    if (g_scales) { g_scales[i * 3] = gs[0]; g_scales[i * 3 + 1] = gs[1]; g_scales[i * 3 + 2] = gs[2]; }
    if (g_opacities) g_opacities[i] = go;
    for (int k = sh_count(st.sh_degree) * 3; k < K * 3; ++k) coeffs[k] = 0.f;
  }
  __syncthreads();
  if (g_sh) {
    // coalesced write-back of the staged coefficient adjoints
    const int count = rows * K * 3;
    float* base = g_sh + first * K * 3;
    RowCursor at(threadIdx.x, blockDim.x, K * 3);
    for (int k = threadIdx.x; k < count; k += blockDim.x, at.advance()) base[k] = s_sh[at.r * stride + at.c];
  }
}

__global__ void covariance_forward_kernel(const float* q, const float* s, int64_t n, float* cov) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float qn[4], R[9];
  quat_normalize(q + i * 4, qn);
  quat_rotation(qn, R);
  covariance3(R, s + i * 3, cov + i * 9);
}

__global__ void covariance_backward_kernel(const float* q, const float* s, int64_t n,
                                           const float* gcov, float* gq, float* gs) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float qn[4], R[9], gR[9], gqn[4], gsl[3], gql[4];
  const float nrm = quat_normalize(q + i * 4, qn);
  quat_rotation(qn, R);
  covariance3_backward(R, s + i * 3, gcov + i * 9, gR, gsl);
  quat_rotation_backward(qn, gR, gqn);
  quat_normalize_backward(q + i * 4, nrm, gqn, gql);
  if (gq) for (int k = 0; k < 4; ++k) gq[i * 4 + k] = gql[k];
  if (gs) for (int k = 0; k < 3; ++k) gs[i * 3 + k] = gsl[k];
}

__global__ void sh_forward_kernel(const float* coeffs, int K, const float* dirs, int64_t n,
                                  int degree, float* rgb) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  sh_color(coeffs + i * K * 3, degree, dirs + i * 3, rgb + i * 3);
}

__global__ void sh_backward_kernel(const float* coeffs, int K, const float* dirs, int64_t n,
                                   int degree, const float* grgb, float* gcoeffs, float* gdirs) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float gc[48], gd[3];
  sh_color_backward(coeffs + i * K * 3, degree, dirs + i * 3, grgb + i * 3, nullptr, gc, gd);
  const int used = sh_count(degree) * 3;
  if (gcoeffs)
    for (int k = 0; k < K * 3; ++k) gcoeffs[i * K * 3 + k] = k < used ? gc[k] : 0.f;
  if (gdirs) for (int k = 0; k < 3; ++k) gdirs[i * 3 + k] = gd[k];
}

__global__ void bin_rects_kernel(const float* bounds, int64_t n, int width, int height,
                                 float nearp, float farp, int32_t* rect, int32_t* count,
                                 uint32_t* depth_key, int32_t* nonfinite) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float4 b = __ldg(reinterpret_cast<const float4*>(bounds) + i);
  write_bounds(i, b.x, b.y, b.z, b.w, width, height, nearp, farp, rect, count, depth_key, nonfinite);
}

inline unsigned blocks_for(int64_t n, int per) { return (unsigned)((n + per - 1) / per); }

}  // namespace

cudaError_t launch_project_forward(const float* means, const float* quats, const float* scales,
                                   const float* opacities, const float* sh,
                                   const uint8_t* selected, int64_t n, const sf_camera& cam,
                                   const sf_settings& st, float* means2d, float* radii,
                                   float* records, int32_t* rect, int32_t* count,
                                   uint32_t* depth_key, int32_t* nonfinite, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  const size_t smem = (size_t)PB * (st.sh_coeffs * 3 + 1) * sizeof(float);
  count_launches(1);
#define SF_PROJECT_FORWARD(M)                                                                              \
  project_forward_kernel<M><<<blocks_for(n, PB), PB, smem, s>>>(means, quats, scales, opacities, sh, selected, n, \
                                                                 cam, st, means2d, radii, records, rect, count,   \
                                                                 depth_key, nonfinite)
  if (st.mode == SF_MODE_RADEGS) SF_PROJECT_FORWARD(SF_MODE_RADEGS);
  else if (st.mode == SF_MODE_GOF) SF_PROJECT_FORWARD(SF_MODE_GOF);
  else SF_PROJECT_FORWARD(SF_MODE_AMBISUR);
#undef SF_PROJECT_FORWARD
  return cudaGetLastError();
}

cudaError_t launch_project_backward(const float* means, const float* quats, const float* scales,
                                    const float* opacities, const float* sh, int64_t n,
                                    const sf_camera& cam, const sf_settings& st,
                                    const float* gxy, const float* grec, float* g_means,
                                    float* g_quats, float* g_scales, float* g_opacities,
                                    float* g_sh, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  const size_t smem = (size_t)PB * (st.sh_coeffs * 3 + 1) * sizeof(float);
  count_launches(1);
#define SF_PROJECT_BACKWARD(M)                                                                            \
  project_backward_kernel<M><<<blocks_for(n, PB), PB, smem, s>>>(means, quats, scales, opacities, sh, n, cam, st, \
                                                                  gxy, grec, g_means, g_quats, g_scales,          \
                                                                  g_opacities, g_sh)
  if (st.mode == SF_MODE_RADEGS) SF_PROJECT_BACKWARD(SF_MODE_RADEGS);
  else if (st.mode == SF_MODE_GOF) SF_PROJECT_BACKWARD(SF_MODE_GOF);
  else SF_PROJECT_BACKWARD(SF_MODE_AMBISUR);
#undef SF_PROJECT_BACKWARD
  return cudaGetLastError();
}

cudaError_t launch_covariance_forward(const float* q, const float* s_, int64_t n, float* cov,
                                      cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  count_launches(1);
  covariance_forward_kernel<<<blocks_for(n, 256), 256, 0, s>>>(q, s_, n, cov);
  return cudaGetLastError();
}

cudaError_t launch_covariance_backward(const float* q, const float* s_, int64_t n,
                                       const float* gcov, float* gq, float* gs, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  count_launches(1);
  covariance_backward_kernel<<<blocks_for(n, 256), 256, 0, s>>>(q, s_, n, gcov, gq, gs);
  return cudaGetLastError();
}

cudaError_t launch_sh_forward(const float* coeffs, int K, const float* dirs, int64_t n,
                              int degree, float* rgb, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  count_launches(1);
  sh_forward_kernel<<<blocks_for(n, 256), 256, 0, s>>>(coeffs, K, dirs, n, degree, rgb);
  return cudaGetLastError();
}

cudaError_t launch_sh_backward(const float* coeffs, int K, const float* dirs, int64_t n,
                               int degree, const float* grgb, float* gcoeffs, float* gdirs,
                               cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  count_launches(1);
  sh_backward_kernel<<<blocks_for(n, 256), 256, 0, s>>>(coeffs, K, dirs, n, degree, grgb, gcoeffs, gdirs);
  return cudaGetLastError();
}

cudaError_t launch_bin_rects(const float* bounds, int64_t n, int width, int height, int tile,
                             float near_plane, float far_plane, int32_t* rect, int32_t* count,
                             uint32_t* depth_key, int32_t* nonfinite, cudaStream_t s) {
  (void)tile;
  if (n == 0) return cudaSuccess;
  count_launches(1);
  bin_rects_kernel<<<blocks_for(n, 256), 256, 0, s>>>(bounds, n, width, height, near_plane,
                                                      far_plane, rect, count, depth_key, nonfinite);
  return cudaGetLastError();
}

}  // namespace sf
