// Small geometry operators of the operator seam:
//   camera.pixel_rays@1       inv(K) (u + 0.5, v + 0.5, 1)            (reference.py:49-56)
//   gaussian.ray_peak@1       peak t, response and normal per (Gaussian, ray)  (:38-46)
//   geometry.depth_normals@1  back-projected z-depth -> face normals   (:59-83), with
//                             the depth adjoint for the normal-consistency losses
// All are bandwidth-bound elementwise kernels: one thread per output element.
#include <cuda_runtime.h>

#include "sf_device.cuh"
#include "sf_kernels.h"

namespace sf {

namespace {

// inverse of a 3x3 matrix by cofactors, in double (K is well conditioned)
__device__ __forceinline__ void inverse3(const float* K, float* Ki) {
  const double a = K[0], b = K[1], c = K[2], d = K[3], e = K[4], f = K[5], g = K[6], h = K[7], i = K[8];
  const double A = e * i - f * h, B = -(d * i - f * g), C = d * h - e * g;
  const double det = a * A + b * B + c * C;
  const double r = 1.0 / det;
  Ki[0] = (float)(A * r); Ki[1] = (float)(-(b * i - c * h) * r); Ki[2] = (float)((b * f - c * e) * r);
  Ki[3] = (float)(B * r); Ki[4] = (float)((a * i - c * g) * r); Ki[5] = (float)(-(a * f - c * d) * r);
  Ki[6] = (float)(C * r); Ki[7] = (float)(-(a * h - b * g) * r); Ki[8] = (float)((a * e - b * d) * r);
}

__device__ __forceinline__ void ray_of(const float* Ki, int x, int y, float* r) {
  const float u = x + 0.5f, v = y + 0.5f;
#pragma unroll
  for (int k = 0; k < 3; ++k) r[k] = u * Ki[k * 3] + v * Ki[k * 3 + 1] + Ki[k * 3 + 2];
}

__global__ void pixel_rays_kernel(const float* K, int W, int H, float* out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)W * H) return;
  float Ki[9], r[3];
  inverse3(K, Ki);
  ray_of(Ki, (int)(i % W), (int)(i / W), r);
  out[i * 3] = r[0]; out[i * 3 + 1] = r[1]; out[i * 3 + 2] = r[2];
}

__global__ void ray_peak_kernel(const float* means, const float* Q, int64_t N, const float* origins,
                                const float* dirs, int64_t P, float* t_out, float* r_out, float* n_out) {
  const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= N * P) return;
  const int64_t n = k / P, p = k - n * P;
  const float* q = Q + n * 9;
  const float d0 = dirs[p * 3], d1 = dirs[p * 3 + 1], d2 = dirs[p * 3 + 2];
  const float qd0 = q[0] * d0 + q[1] * d1 + q[2] * d2;
  const float qd1 = q[3] * d0 + q[4] * d1 + q[5] * d2;
  const float qd2 = q[6] * d0 + q[7] * d1 + q[8] * d2;
  const float den = fmaxf(d0 * qd0 + d1 * qd1 + d2 * qd2, 1e-12f);
  const float e0 = origins[p * 3] - means[n * 3], e1 = origins[p * 3 + 1] - means[n * 3 + 1];
  const float e2 = origins[p * 3 + 2] - means[n * 3 + 2];
  const float t = -(e0 * qd0 + e1 * qd1 + e2 * qd2) / den;
  const float o0 = e0 + t * d0, o1 = e1 + t * d1, o2 = e2 + t * d2;
  const float e = o0 * (q[0] * o0 + q[1] * o1 + q[2] * o2) + o1 * (q[3] * o0 + q[4] * o1 + q[5] * o2) +
                  o2 * (q[6] * o0 + q[7] * o1 + q[8] * o2);
  t_out[k] = t;
  r_out[k] = expf(-0.5f * fmaxf(e, 0.f));
  const float len = fmaxf(sqrtf(qd0 * qd0 + qd1 * qd1 + qd2 * qd2), 1e-12f);
  n_out[k * 3] = -qd0 / len;
  n_out[k * 3 + 1] = -qd1 / len;
  n_out[k * 3 + 2] = -qd2 / len;
}

// depth_normals at one interior pixel: the (unnormalised) cross product c = dy x dx,
// the unit normal turned towards the camera and whether the pixel is valid
struct DnPixel {
  float dx[3], dy[3], c[3], n[3], len, sign;
  bool good;
};

__device__ __forceinline__ void dn_pixel(const float* depth, const float* Ki, int W, int x, int y, DnPixel& px) {
  float rc[3], rl[3], rr[3], ru[3], rd[3];
  ray_of(Ki, x, y, rc);
  ray_of(Ki, x - 1, y, rl);
  ray_of(Ki, x + 1, y, rr);
  ray_of(Ki, x, y - 1, ru);
  ray_of(Ki, x, y + 1, rd);
  const float zc = depth[(int64_t)y * W + x], zl = depth[(int64_t)y * W + x - 1], zr = depth[(int64_t)y * W + x + 1];
  const float zu = depth[(int64_t)(y - 1) * W + x], zd = depth[(int64_t)(y + 1) * W + x];
  float pc[3];
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    pc[k] = rc[k] * zc;
    px.dx[k] = rr[k] * zr - rl[k] * zl;
    px.dy[k] = rd[k] * zd - ru[k] * zu;
  }
  px.c[0] = px.dy[1] * px.dx[2] - px.dy[2] * px.dx[1];
  px.c[1] = px.dy[2] * px.dx[0] - px.dy[0] * px.dx[2];
  px.c[2] = px.dy[0] * px.dx[1] - px.dy[1] * px.dx[0];
  px.len = fmaxf(sqrtf(px.c[0] * px.c[0] + px.c[1] * px.c[1] + px.c[2] * px.c[2]), 1e-12f);
  float u[3] = {px.c[0] / px.len, px.c[1] / px.len, px.c[2] / px.len};
  const float facing = u[0] * pc[0] + u[1] * pc[1] + u[2] * pc[2];
  px.sign = facing > 0.f ? -1.f : 1.f;
  for (int k = 0; k < 3; ++k) px.n[k] = px.sign * u[k];
  const bool finite = isfinite(px.n[0]) && isfinite(px.n[1]) && isfinite(px.n[2]);
  px.good = zc > 0.f && zr > 0.f && zl > 0.f && zd > 0.f && zu > 0.f && finite &&
            (px.n[0] * px.n[0] + px.n[1] * px.n[1] + px.n[2] * px.n[2]) > 0.f;
}

__global__ void depth_normals_kernel(const float* depth, const float* K, int W, int H, float* normals,
                                     uint8_t* valid) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)W * H) return;
  const int x = (int)(i % W), y = (int)(i / W);
  float n[3] = {0.f, 0.f, 0.f};
  bool good = false;
  if (x > 0 && y > 0 && x < W - 1 && y < H - 1) {
    float Ki[9];
    inverse3(K, Ki);
    DnPixel px;
    dn_pixel(depth, Ki, W, x, y, px);
    good = px.good;
    if (good) { n[0] = px.n[0]; n[1] = px.n[1]; n[2] = px.n[2]; }
  }
  normals[i * 3] = n[0]; normals[i * 3 + 1] = n[1]; normals[i * 3 + 2] = n[2];
  valid[i] = good ? 1 : 0;
}

// backward, pass 1: per valid interior pixel, the adjoints of its two differences,
// g_dx = g_c x dy and g_dy = dx x g_c, where g_c is the adjoint of the cross product
// through the orientation sign and the normalisation
__global__ void depth_normals_diff_grad_kernel(const float* depth, const float* K, int W, int H,
                                               const float* g_normals, float* g_dx, float* g_dy) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)W * H) return;
  const int x = (int)(i % W), y = (int)(i / W);
  float gx[3] = {0.f, 0.f, 0.f}, gy[3] = {0.f, 0.f, 0.f};
  if (x > 0 && y > 0 && x < W - 1 && y < H - 1) {
    float Ki[9];
    inverse3(K, Ki);
    DnPixel px;
    dn_pixel(depth, Ki, W, x, y, px);
    if (px.good) {
      const float g[3] = {px.sign * g_normals[i * 3], px.sign * g_normals[i * 3 + 1], px.sign * g_normals[i * 3 + 2]};
      float gc[3];
      if (sqrtf(px.c[0] * px.c[0] + px.c[1] * px.c[1] + px.c[2] * px.c[2]) >= 1e-12f) {
        const float u[3] = {px.c[0] / px.len, px.c[1] / px.len, px.c[2] / px.len};
        const float d = u[0] * g[0] + u[1] * g[1] + u[2] * g[2];
        for (int k = 0; k < 3; ++k) gc[k] = (g[k] - u[k] * d) / px.len;
      } else {
        for (int k = 0; k < 3; ++k) gc[k] = g[k] / px.len;
      }
      // c = dy x dx:  d(g.c)/d(dy) = dx x g_c,  d(g.c)/d(dx) = g_c x dy
      gy[0] = px.dx[1] * gc[2] - px.dx[2] * gc[1];
      gy[1] = px.dx[2] * gc[0] - px.dx[0] * gc[2];
      gy[2] = px.dx[0] * gc[1] - px.dx[1] * gc[0];
      gx[0] = gc[1] * px.dy[2] - gc[2] * px.dy[1];
      gx[1] = gc[2] * px.dy[0] - gc[0] * px.dy[2];
      gx[2] = gc[0] * px.dy[1] - gc[1] * px.dy[0];
    }
  }
  for (int k = 0; k < 3; ++k) { g_dx[i * 3 + k] = gx[k]; g_dy[i * 3 + k] = gy[k]; }
}

// backward, pass 2: point p(x, y) = ray * depth enters dx of its left and right
// neighbours and dy of the ones above and below; gather those adjoints
__global__ void depth_normals_depth_grad_kernel(const float* K, int W, int H, const float* g_dx, const float* g_dy,
                                                float* g_depth) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)W * H) return;
  const int x = (int)(i % W), y = (int)(i / W);
  float gp[3] = {0.f, 0.f, 0.f};
  if (x - 1 >= 0) for (int k = 0; k < 3; ++k) gp[k] += g_dx[(i - 1) * 3 + k];      // dx(x-1) = p(x) - p(x-2)
  if (x + 1 < W) for (int k = 0; k < 3; ++k) gp[k] -= g_dx[(i + 1) * 3 + k];       // dx(x+1) = p(x+2) - p(x)
  if (y - 1 >= 0) for (int k = 0; k < 3; ++k) gp[k] += g_dy[(i - W) * 3 + k];      // dy(y-1) = p(y) - p(y-2)
  if (y + 1 < H) for (int k = 0; k < 3; ++k) gp[k] -= g_dy[(i + W) * 3 + k];       // dy(y+1) = p(y+2) - p(y)
  float Ki[9], r[3];
  inverse3(K, Ki);
  ray_of(Ki, x, y, r);
  g_depth[i] = r[0] * gp[0] + r[1] * gp[1] + r[2] * gp[2];
}

inline unsigned blocks_for(int64_t n) { return (unsigned)((n + 255) / 256); }

}  // namespace

cudaError_t launch_pixel_rays(const float* K, int W, int H, float* out, cudaStream_t s) {
  if ((int64_t)W * H == 0) return cudaSuccess;
  count_launches(1);
  pixel_rays_kernel<<<blocks_for((int64_t)W * H), 256, 0, s>>>(K, W, H, out);
  return cudaGetLastError();
}

cudaError_t launch_ray_peak(const float* means, const float* Q, int64_t N, const float* origins, const float* dirs,
                            int64_t P, float* t, float* r, float* n, cudaStream_t s) {
  if (N * P == 0) return cudaSuccess;
  count_launches(1);
  ray_peak_kernel<<<blocks_for(N * P), 256, 0, s>>>(means, Q, N, origins, dirs, P, t, r, n);
  return cudaGetLastError();
}

cudaError_t launch_depth_normals(const float* depth, const float* K, int W, int H, float* normals, uint8_t* valid,
                                 cudaStream_t s) {
  if ((int64_t)W * H == 0) return cudaSuccess;
  count_launches(1);
  depth_normals_kernel<<<blocks_for((int64_t)W * H), 256, 0, s>>>(depth, K, W, H, normals, valid);
  return cudaGetLastError();
}

cudaError_t launch_depth_normals_backward(const float* depth, const float* K, int W, int H, const float* g_normals,
                                          float* g_depth, float* ws, cudaStream_t s) {
  const int64_t np = (int64_t)W * H;
  if (np == 0) return cudaSuccess;
  float* g_dx = ws;
  float* g_dy = ws + np * 3;
  count_launches(2);
  depth_normals_diff_grad_kernel<<<blocks_for(np), 256, 0, s>>>(depth, K, W, H, g_normals, g_dx, g_dy);
  depth_normals_depth_grad_kernel<<<blocks_for(np), 256, 0, s>>>(K, W, H, g_dx, g_dy, g_depth);
  return cudaGetLastError();
}

}  // namespace sf
