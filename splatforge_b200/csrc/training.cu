// The training-step operations on either side of the rasterizer:
//
// * matching.patch_zncc@1 (src/splatforge/providers/torch/gaussian/reference.py:225-236):
//   masked zero-mean normalised cross-correlation of patch pairs, with its adjoint for a
//   and b.  One warp per patch; the sums are warp reductions in a fixed order.
// * the densifier's statistics (src/splatforge/studio/densification.py:18-43): per
//   Gaussian, the norm of its (optionally NDC-scaled) projected-mean gradient added to the
//   accumulator where its radius is positive, and the visibility count.
// * gaussian.sh_ambiguity@1 (reference.py:116-117), the AmbiSuR method's per-Gaussian
//   score (src/splatforge/studio/methods/ambisur.py:25).
// * the normal-consistency loss (src/splatforge/studio/losses.py:9-12, 45-53): depth normals
//   (geometry.depth_normals@1, geometry.cu), masked by validity, alpha > 0.1 and the caller's
//   mask, against the rendered normal numerator (alpha - n_num . n_depth) or unit normal
//   (1 - n . n_depth); the masked mean and its adjoint for depth, alpha and the normals.
#include <cuda_runtime.h>

#include "sf_device.cuh"
#include "sf_kernels.h"

namespace sf {
namespace {

constexpr int TR_THREADS = 256;
constexpr int TR_WARPS = TR_THREADS / 32;

inline unsigned blocks_of(int64_t n) { return (unsigned)((n + TR_THREADS - 1) / TR_THREADS); }

// --------------------------------------------------------------------------- ZNCC
struct ZnccStats {
  float count, av, bv, cov, ma, mb;
  bool valid;
};

__device__ __forceinline__ ZnccStats zncc_stats(const float* a, const float* b, const float* m, int S, int lane,
                                                float eps) {
  float sm = 0.f, sa = 0.f, sb = 0.f;
  for (int k = lane; k < S; k += 32) {
    sm += m[k];
    sa += a[k] * m[k];
    sb += b[k] * m[k];
  }
  sm = warp_sum(sm);
  sa = warp_sum(sa);
  sb = warp_sum(sb);
  ZnccStats z;
  z.count = fmaxf(sm, 1.f);
  z.ma = sa / z.count;
  z.mb = sb / z.count;
  float av = 0.f, bv = 0.f, cv = 0.f;
  for (int k = lane; k < S; k += 32) {
    const float ac = a[k] - z.ma, bc = b[k] - z.mb;
    av += m[k] * ac * ac;
    bv += m[k] * bc * bc;
    cv += m[k] * ac * bc;
  }
  z.av = warp_sum(av);
  z.bv = warp_sum(bv);
  z.cov = warp_sum(cv);
  z.valid = sm >= 2.f && z.av > eps && z.bv > eps;
  return z;
}

__global__ void zncc_forward_kernel(const float* a, const float* b, const float* m, int64_t rows, int S, float eps,
                                    float* corr, uint8_t* valid) {
  const int64_t r = (int64_t)blockIdx.x * TR_WARPS + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const int64_t o = r * S;
  const ZnccStats z = zncc_stats(a + o, b + o, m + o, S, lane, eps);
  if (lane == 0) {
    const float c = z.cov / sqrtf(fmaxf(z.av * z.bv, eps * eps));
    corr[r] = z.valid ? fminf(fmaxf(c, -1.f), 1.f) : 0.f;
    valid[r] = z.valid ? 1 : 0;
  }
}

// corr = C / D, D = sqrt(av bv): dcorr/dac_k = m_k bc_k / D - corr m_k ac_k / av (and
// symmetrically for b); ac_k = a_k - sum_j a_j m_j / count gives
// ga_k = g_k - m_k / count * sum_j g_j.  Clamped-out or invalid patches pass nothing.
__global__ void zncc_backward_kernel(const float* a, const float* b, const float* m, int64_t rows, int S, float eps,
                                     const float* g_corr, float* ga, float* gb) {
  const int64_t r = (int64_t)blockIdx.x * TR_WARPS + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const int64_t o = r * S;
  const ZnccStats z = zncc_stats(a + o, b + o, m + o, S, lane, eps);
  const float D = sqrtf(fmaxf(z.av * z.bv, eps * eps));
  const float c = z.cov / D;
  const float G = (z.valid && c >= -1.f && c <= 1.f) ? g_corr[r] : 0.f;
  float sa = 0.f, sb = 0.f;
  // G != 0 only for valid patches, where av, bv > eps (no division by zero)
  if (G != 0.f) {
    for (int k = lane; k < S; k += 32) {
      const float mk = m[o + k], ac = a[o + k] - z.ma, bc = b[o + k] - z.mb;
      sa += G * (mk * bc / D - c * mk * ac / z.av);
      sb += G * (mk * ac / D - c * mk * bc / z.bv);
    }
  }
  sa = warp_sum(sa);
  sb = warp_sum(sb);
  for (int k = lane; k < S; k += 32) {
    const float mk = m[o + k], ac = a[o + k] - z.ma, bc = b[o + k] - z.mb;
    const float gak = G == 0.f ? 0.f : G * (mk * bc / D - c * mk * ac / z.av);
    const float gbk = G == 0.f ? 0.f : G * (mk * ac / D - c * mk * bc / z.bv);
    ga[o + k] = gak - mk / z.count * sa;
    gb[o + k] = gbk - mk / z.count * sb;
  }
}

// --------------------------------------------------------------------------- densifier
__global__ void densify_observe_kernel(const float* grad2d, const float* radii, int64_t n, float sx, float sy,
                                       float* gradient, float* observations) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n || !(radii[i] > 0.f)) return;
  const float gx = grad2d[i * 2] * sx, gy = grad2d[i * 2 + 1] * sy;
  gradient[i] += sqrtf(gx * gx + gy * gy);
  observations[i] += 1.f;
}

// --------------------------------------------------------------------------- normal consistency
__device__ __forceinline__ bool nc_term(int64_t i, const float* normals, const uint8_t* valid, const float* alpha,
                                        const float* numer, const float* unit, const float* mask, float& term) {
  if (!(valid[i] && alpha[i] > 0.1f && mask[i] > 0.f)) return false;
  const float* n = normals + i * 3;
  const float* v = numer ? numer + i * 3 : unit + i * 3;
  const float d = v[0] * n[0] + v[1] * n[1] + v[2] * n[2];
  term = numer ? alpha[i] - d : 1.f - d;
  return true;
}

// per-block partial sums (double) and counts of the masked terms
__global__ void nc_partial_kernel(const float* normals, const uint8_t* valid, const float* alpha, const float* numer,
                                  const float* unit, const float* mask, int64_t n, double* psum, int64_t* pcount) {
  __shared__ double s_sum[TR_WARPS];
  __shared__ int s_cnt[TR_WARPS];
  const int64_t i = (int64_t)blockIdx.x * TR_THREADS + threadIdx.x;
  float t = 0.f;
  const bool on = i < n && nc_term(i, normals, valid, alpha, numer, unit, mask, t);
  double v = on ? (double)t : 0.0;
  int c = on ? 1 : 0;
  for (int o = 16; o > 0; o >>= 1) {
    v += __shfl_xor_sync(FULL, v, o);
    c += __shfl_xor_sync(FULL, c, o);
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) { s_sum[w] = v; s_cnt[w] = c; }
  __syncthreads();
  if (threadIdx.x == 0) {
    double sv = 0.0;
    int64_t sc = 0;
    for (int k = 0; k < TR_WARPS; ++k) { sv += s_sum[k]; sc += s_cnt[k]; }
    psum[blockIdx.x] = sv;
    pcount[blockIdx.x] = sc;
  }
}

// loss = sum / max(count, 1); the partials are added in block order by one CTA
__global__ void nc_finish_kernel(const double* psum, const int64_t* pcount, int64_t nb, float* loss, int64_t* count) {
  __shared__ double s_sum[TR_THREADS];
  __shared__ int64_t s_cnt[TR_THREADS];
  double v = 0.0;
  int64_t c = 0;
  for (int64_t k = threadIdx.x; k < nb; k += TR_THREADS) { v += psum[k]; c += pcount[k]; }
  s_sum[threadIdx.x] = v;
  s_cnt[threadIdx.x] = c;
  __syncthreads();
  for (int st = TR_THREADS / 2; st > 0; st >>= 1) {
    if (threadIdx.x < st) {
      s_sum[threadIdx.x] += s_sum[threadIdx.x + st];
      s_cnt[threadIdx.x] += s_cnt[threadIdx.x + st];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const int64_t total = s_cnt[0];
    loss[0] = (float)(s_sum[0] / (double)(total > 0 ? total : 1));
    count[0] = total;
  }
}

// adjoints of the masked mean: g = G / max(count, 1) on every counted pixel
__global__ void nc_backward_kernel(const float* normals, const uint8_t* valid, const float* alpha, const float* numer,
                                   const float* unit, const float* mask, int64_t n, const float* g_loss,
                                   const int64_t* count, float* g_alpha, float* g_vec, float* g_normals) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float t;
  const bool on = nc_term(i, normals, valid, alpha, numer, unit, mask, t);
  const float g = on ? g_loss[0] / (float)(count[0] > 0 ? count[0] : 1) : 0.f;
  const float* nd = normals + i * 3;
  const float* v = numer ? numer + i * 3 : unit + i * 3;
  if (g_alpha) g_alpha[i] = numer ? g : 0.f;
  for (int k = 0; k < 3; ++k) {
    if (g_vec) g_vec[i * 3 + k] = -g * nd[k];
    g_normals[i * 3 + k] = -g * v[k];
  }
}

// --------------------------------------------------------------------------- SH ambiguity
// gaussian.sh_ambiguity@1 (reference.py:116-117): sum of squares of every band but the DC
// one, per Gaussian; the adjoint is 2 c g outside the DC band.  One warp per Gaussian.
__global__ void sh_ambiguity_kernel(const float* coeffs, int64_t n, int K, float* out) {
  const int64_t i = (int64_t)blockIdx.x * TR_WARPS + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (i >= n) return;
  const float* c = coeffs + i * K * 3;
  float acc = 0.f;
  for (int k = 3 + lane; k < K * 3; k += 32) acc += c[k] * c[k];
  acc = warp_sum(acc);
  if (lane == 0) out[i] = acc;
}

__global__ void sh_ambiguity_backward_kernel(const float* coeffs, int64_t total, int K, const float* g,
                                             float* g_coeffs) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= total) return;
  const int64_t i = j / (K * 3);
  g_coeffs[j] = (j - i * K * 3) < 3 ? 0.f : 2.f * coeffs[j] * g[i];
}

}  // namespace

cudaError_t launch_sh_ambiguity(const float* coeffs, int64_t n, int K, float* out, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  count_launches(1);
  sh_ambiguity_kernel<<<(unsigned)((n + TR_WARPS - 1) / TR_WARPS), TR_THREADS, 0, s>>>(coeffs, n, K, out);
  return cudaGetLastError();
}

cudaError_t launch_sh_ambiguity_backward(const float* coeffs, int64_t n, int K, const float* g, float* g_coeffs,
                                         cudaStream_t s) {
  const int64_t total = n * K * 3;
  if (total == 0) return cudaSuccess;
  count_launches(1);
  sh_ambiguity_backward_kernel<<<blocks_of(total), TR_THREADS, 0, s>>>(coeffs, total, K, g, g_coeffs);
  return cudaGetLastError();
}

cudaError_t launch_patch_zncc(const float* a, const float* b, const float* m, int64_t rows, int S, float eps,
                              float* corr, uint8_t* valid, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  count_launches(1);
  zncc_forward_kernel<<<(unsigned)((rows + TR_WARPS - 1) / TR_WARPS), TR_THREADS, 0, s>>>(a, b, m, rows, S, eps,
                                                                                          corr, valid);
  return cudaGetLastError();
}

cudaError_t launch_patch_zncc_backward(const float* a, const float* b, const float* m, int64_t rows, int S, float eps,
                                       const float* g_corr, float* ga, float* gb, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  count_launches(1);
  zncc_backward_kernel<<<(unsigned)((rows + TR_WARPS - 1) / TR_WARPS), TR_THREADS, 0, s>>>(a, b, m, rows, S, eps,
                                                                                           g_corr, ga, gb);
  return cudaGetLastError();
}

cudaError_t launch_densify_observe(const float* grad2d, const float* radii, int64_t n, float sx, float sy,
                                   float* gradient, float* observations, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  count_launches(1);
  densify_observe_kernel<<<blocks_of(n), TR_THREADS, 0, s>>>(grad2d, radii, n, sx, sy, gradient, observations);
  return cudaGetLastError();
}

namespace {
// normals, validity, per-block partial sums and counts, the depth adjoint's scratch;
// every slice starts on a 256-byte boundary
struct NcLayout {
  float* normals; uint8_t* valid; double* psum; int64_t* pcount; float* scratch;
  size_t used;
};
NcLayout nc_layout(void* ws, int W, int H) {
  const int64_t n = (int64_t)W * H, nb = (n + TR_THREADS - 1) / TR_THREADS;
  char* p = reinterpret_cast<char*>(ws);
  size_t used = 0;
  auto take = [&](size_t bytes) { char* r = p ? p + used : nullptr; used += (bytes + 255) & ~(size_t)255; return r; };
  NcLayout L;
  L.normals = reinterpret_cast<float*>(take((size_t)n * 3 * sizeof(float)));
  L.valid = reinterpret_cast<uint8_t*>(take((size_t)n));
  L.psum = reinterpret_cast<double*>(take((size_t)nb * sizeof(double)));
  L.pcount = reinterpret_cast<int64_t*>(take((size_t)nb * sizeof(int64_t)));
  L.scratch = reinterpret_cast<float*>(take((size_t)n * 6 * sizeof(float)));
  L.used = used;
  return L;
}
}  // namespace

size_t normal_consistency_workspace_bytes(int W, int H) { return nc_layout(nullptr, W, H).used; }

cudaError_t normal_consistency(const float* depth, const float* K, int W, int H, const float* alpha,
                               const float* numer, const float* unit, const float* mask, float* loss, int64_t* count,
                               void* ws, cudaStream_t s) {
  const int64_t n = (int64_t)W * H;
  const NcLayout L = nc_layout(ws, W, H);
  cudaError_t e = launch_depth_normals(depth, K, W, H, L.normals, L.valid, s);
  if (e != cudaSuccess) return e;
  const int64_t nb = (n + TR_THREADS - 1) / TR_THREADS;
  if (nb > 0) {
    count_launches(1);
    nc_partial_kernel<<<(unsigned)nb, TR_THREADS, 0, s>>>(L.normals, L.valid, alpha, numer, unit, mask, n, L.psum,
                                                          L.pcount);
  }
  count_launches(1);
  nc_finish_kernel<<<1, TR_THREADS, 0, s>>>(L.psum, L.pcount, nb, loss, count);
  return cudaGetLastError();
}

cudaError_t normal_consistency_backward(const float* depth, const float* K, int W, int H, const float* alpha,
                                        const float* numer, const float* unit, const float* mask, const float* g_loss,
                                        const int64_t* count, float* g_depth, float* g_alpha, float* g_vec,
                                        float* g_normals, void* ws, cudaStream_t s) {
  const int64_t n = (int64_t)W * H;
  if (n == 0) return cudaSuccess;
  const NcLayout L = nc_layout(ws, W, H);
  count_launches(1);
  nc_backward_kernel<<<blocks_of(n), TR_THREADS, 0, s>>>(L.normals, L.valid, alpha, numer, unit, mask, n, g_loss,
                                                         count, g_alpha, g_vec, g_normals);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = launch_depth_normals_backward(depth, K, W, H, g_normals, g_depth, L.scratch, s);
  return e;
}

}  // namespace sf
