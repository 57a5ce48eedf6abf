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

}  // namespace sf
