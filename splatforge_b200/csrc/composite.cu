// splat.alpha_composite@3 over dense [B, N, P] tensors (the operator-level contract of
// src/splatforge/gaussian/semantics.json:23, reference.py:151-186), replacing the
// reference's one-thread-per-pixel composite_cuda.cu:26-98 with an sm_100a
// implementation:
//   forward  -- one thread per (b, p); P is the contiguous axis, so a warp reads 32
//               consecutive pixels of one sample (coalesced); transmittance and the
//               median crossing accumulate in double like torch's CPU cumprod/cumsum;
//   L1       -- one warp per (b, p): stable warp radix sort of the sample depths in
//               shared memory (no torch.sort), then sorted prefix sums;
//   backward -- one thread per (b, p), two forward sweeps: the first sums the total
//               suffix term sum_j w_j adj_j, the second emits d alpha, d depth and
//               d normal with the exact forward transmittance (no division);
//               d colour [b,n,:] = sum_p w g_rgb is a coalesced warp reduction over p.
#include <cuda_runtime.h>

#include "sf_device.cuh"
#include "sf_kernels.h"

namespace sf {

namespace {

struct CompositeArgs {
  const float* a; const float* c; const float* d; const float* nrm;
  int B, N, P, dist;
  float* rgb; float* alpha; float* znum; float* nnum; float* l1; float* l2; float* median; float* w;
  float* aux;  // [2, B, N, P] L1 factors (auxw, auxd), when L1 is requested
  float* raw;  // [2, B, P] raw L1 / L2 (sign decides whether the clamp passes the adjoint)
};

__global__ void composite_forward_kernel(const CompositeArgs a) {
  const int64_t bp = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (bp >= (int64_t)a.B * a.P) return;
  const int b = (int)(bp / a.P), p = (int)(bp % a.P);
  const int64_t P = a.P;
  double T = 1.0, Wd = 0.0;
  float C0 = 0.f, C1 = 0.f, C2 = 0.f, D = 0.f, D2 = 0.f, M0 = 0.f, M1 = 0.f, M2 = 0.f, med = 0.f;
  bool crossed = false;
  for (int i = 0; i < a.N; ++i) {
    const int64_t e = ((int64_t)b * a.N + i) * P + p;
    const float al = fminf(fmaxf(a.a[e], 0.f), 0.999f);
    const float w = al * (float)T;
    a.w[e] = w;
    const float depth = a.d[e];
    const float* col = a.c + ((int64_t)b * a.N + i) * 3;
    C0 += w * col[0]; C1 += w * col[1]; C2 += w * col[2];
    D += w * depth;
    D2 += w * depth * depth;
    M0 += w * a.nrm[e * 3]; M1 += w * a.nrm[e * 3 + 1]; M2 += w * a.nrm[e * 3 + 2];
    Wd += (double)w;
    if (!crossed && (float)Wd >= 0.5f) { crossed = true; med = depth; }
    T *= (double)(1.f - al);
  }
  const float W = (float)Wd;
  a.rgb[bp * 3] = C0; a.rgb[bp * 3 + 1] = C1; a.rgb[bp * 3 + 2] = C2;
  a.nnum[bp * 3] = M0; a.nnum[bp * 3 + 1] = M1; a.nnum[bp * 3 + 2] = M2;
  a.alpha[bp] = W;
  a.znum[bp] = D;
  a.median[bp] = crossed ? med : 0.f;
  const float raw2 = (a.dist & SF_DIST_L2) ? 2.f * (W * D2 - D * D) : 0.f;
  a.l2[bp] = fmaxf(raw2, 0.f);
  a.raw[(int64_t)a.B * a.P + bp] = raw2;
  if (!(a.dist & SF_DIST_L1)) { a.l1[bp] = 0.f; a.raw[bp] = 0.f; }
}

// L1 per (b, p): one warp each; samples staged in shared memory, stable radix sort by
// depth bits (ties keep sample order), sorted prefix sums.
__global__ void __launch_bounds__(128) composite_l1_kernel(const CompositeArgs a, int smem_k) {
  extern __shared__ uint32_t s_c[];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, warps = blockDim.x >> 5;
  uint32_t* k0 = s_c + (size_t)wid * (5 * smem_k + 256);
  uint32_t* v0 = k0 + smem_k;
  uint32_t* k1 = v0 + smem_k;
  uint32_t* v1 = k1 + smem_k;
  float* ws = reinterpret_cast<float*>(v1 + smem_k);
  uint32_t* hist = reinterpret_cast<uint32_t*>(ws + smem_k);
  const int64_t total = (int64_t)a.B * a.P;
  const int64_t P = a.P;
  const int n = a.N;
  const int64_t plane = (int64_t)a.B * a.N * a.P;
  for (int64_t bp = (int64_t)blockIdx.x * warps + wid; bp < total; bp += (int64_t)gridDim.x * warps) {
    const int b = (int)(bp / a.P), p = (int)(bp % a.P);
    const int64_t e0 = (int64_t)b * a.N * P + p;
    float Wt = 0.f, Dt = 0.f;
    for (int i = lane; i < n; i += 32) {
      const float d = a.d[e0 + i * P], w = a.w[e0 + i * P];
      // negative and positive depths: map float order onto unsigned order
      const uint32_t bits = __float_as_uint(d);
      k0[i] = (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
      v0[i] = (uint32_t)i;
      ws[i] = w;
      Wt += w; Dt += w * d;
    }
    Wt = warp_sum(Wt); Dt = warp_sum(Dt);
    __syncwarp();
    uint32_t *ks, *vs;
    warp_radix_sort_u32(k0, v0, k1, v1, hist, n, lane, &ks, &vs);
    float carry_w = 0.f, carry_wd = 0.f, raw = 0.f;
    for (int c = 0; c < n; c += 32) {
      const int r = c + lane;
      float d = 0.f, w = 0.f;
      uint32_t i = 0;
      if (r < n) { i = vs[r]; d = a.d[e0 + (int64_t)i * P]; w = ws[i]; }
      float sw = w, swd = w * d;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y1 = __shfl_up_sync(FULL, sw, o), y2 = __shfl_up_sync(FULL, swd, o);
        if (lane >= o) { sw += y1; swd += y2; }
      }
      const float pw = carry_w + sw - w, pwd = carry_wd + swd - w * d;
      carry_w += __shfl_sync(FULL, sw, 31);
      carry_wd += __shfl_sync(FULL, swd, 31);
      if (r < n) {
        raw += 2.f * w * (d * pw - pwd);
        const int64_t e = e0 + (int64_t)i * P;
        a.aux[e] = 2.f * (2.f * d * pw - d * Wt + Dt - 2.f * pwd);
        a.aux[plane + e] = 2.f * w * (2.f * pw + w - Wt);
      }
    }
    raw = warp_sum(raw);
    if (lane == 0) { a.raw[bp] = raw; a.l1[bp] = fmaxf(raw, 0.f); }
    __syncwarp();
  }
}

struct CompositeGrads {
  const float* g_rgb; const float* g_alpha; const float* g_znum; const float* g_nnum;
  const float* g_l1; const float* g_l2; const float* g_median; const float* g_w;
  float* da; float* dd; float* dn; float* dc;
};

__device__ __forceinline__ float gget(const float* g, int64_t i) { return g ? g[i] : 0.f; }

__global__ void composite_backward_kernel(const CompositeArgs a, const CompositeGrads g) {
  const int64_t bp = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (bp >= (int64_t)a.B * a.P) return;
  const int b = (int)(bp / a.P), p = (int)(bp % a.P);
  const int64_t P = a.P;
  const int64_t plane = (int64_t)a.B * a.N * a.P;
  const float gr0 = gget(g.g_rgb, bp * 3), gr1 = gget(g.g_rgb, bp * 3 + 1), gr2 = gget(g.g_rgb, bp * 3 + 2);
  const float gn0 = gget(g.g_nnum, bp * 3), gn1 = gget(g.g_nnum, bp * 3 + 1), gn2 = gget(g.g_nnum, bp * 3 + 2);
  const float ga = gget(g.g_alpha, bp), gz = gget(g.g_znum, bp), gm = gget(g.g_median, bp);
  const bool use1 = (a.dist & SF_DIST_L1) && a.raw[bp] >= 0.f;
  const bool use2 = (a.dist & SF_DIST_L2) && a.raw[(int64_t)a.B * a.P + bp] >= 0.f;
  const float g1 = use1 ? gget(g.g_l1, bp) : 0.f, g2 = use2 ? gget(g.g_l2, bp) : 0.f;
  // totals for L2 and the median position (recomputed exactly as in the forward)
  double Wd = 0.0;
  float W = 0.f, D = 0.f;
  int mid = -1;
  for (int i = 0; i < a.N; ++i) {
    const int64_t e = ((int64_t)b * a.N + i) * P + p;
    const float w = a.w[e];
    Wd += (double)w;
    if (mid < 0 && (float)Wd >= 0.5f) mid = i;
    D += w * a.d[e];
  }
  W = (float)Wd;
  auto adj_of = [&](int i, int64_t e, float w) {
    const float* col = a.c + ((int64_t)b * a.N + i) * 3;
    float adj = ga + gz * a.d[e] + gr0 * col[0] + gr1 * col[1] + gr2 * col[2] +
                gn0 * a.nrm[e * 3] + gn1 * a.nrm[e * 3 + 1] + gn2 * a.nrm[e * 3 + 2] + gget(g.g_w, e);
    if (use1) adj += g1 * a.aux[e];
    (void)w;
    return adj;
  };
  float S = 0.f;
  for (int i = 0; i < a.N; ++i) {
    const int64_t e = ((int64_t)b * a.N + i) * P + p;
    const float w = a.w[e];
    S += w * adj_of(i, e, w);
  }
  double T = 1.0;
  float pre = 0.f;
  for (int i = 0; i < a.N; ++i) {
    const int64_t e = ((int64_t)b * a.N + i) * P + p;
    const float raw = a.a[e];
    const float al = fminf(fmaxf(raw, 0.f), 0.999f);
    const float Tf = (float)T;
    const float w = a.w[e];
    const float adj = adj_of(i, e, w);
    pre += w * adj;
    const float suffix = S - pre;
    const bool pass = raw >= 0.f && raw <= 0.999f;
    g.da[e] = pass ? Tf * adj - suffix / (1.f - al) : 0.f;
    const float depth = a.d[e];
    float gd = w * gz + (i == mid ? gm : 0.f);
    if (use1) gd += g1 * a.aux[plane + e];
    if (use2) gd += g2 * 4.f * w * (W * depth - D);
    g.dd[e] = gd;
    g.dn[e * 3] = w * gn0; g.dn[e * 3 + 1] = w * gn1; g.dn[e * 3 + 2] = w * gn2;
    T *= (double)(1.f - al);
  }
}

// d colour [b, n, c] = sum_p w[b,n,p] g_rgb[b,p,c]: one warp per (b, n)
__global__ void composite_color_grad_kernel(const CompositeArgs a, const CompositeGrads g) {
  const int lane = threadIdx.x & 31;
  const int64_t bn = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (bn >= (int64_t)a.B * a.N) return;
  const int b = (int)(bn / a.N);
  float s0 = 0.f, s1 = 0.f, s2 = 0.f;
  if (g.g_rgb) {
    for (int p = lane; p < a.P; p += 32) {
      const float w = a.w[bn * a.P + p];
      const int64_t q = ((int64_t)b * a.P + p) * 3;
      s0 += w * g.g_rgb[q]; s1 += w * g.g_rgb[q + 1]; s2 += w * g.g_rgb[q + 2];
    }
  }
  s0 = warp_sum(s0); s1 = warp_sum(s1); s2 = warp_sum(s2);
  if (lane == 0) { g.dc[bn * 3] = s0; g.dc[bn * 3 + 1] = s1; g.dc[bn * 3 + 2] = s2; }
}

}  // namespace

size_t composite_l1_smem_per_warp(int n) {
  const int k = ((n > 0 ? n : 1) + 31) / 32 * 32;
  return ((size_t)5 * k + 256) * sizeof(uint32_t);
}

cudaError_t launch_composite_forward(const float* al, const float* col, const float* dep, const float* nrm, int B,
                                     int N, int P, int dist, float* rgb, float* alpha, float* znum, float* nnum,
                                     float* l1, float* l2, float* median, float* w, float* aux, float* raw,
                                     cudaStream_t s) {
  CompositeArgs a{al, col, dep, nrm, B, N, P, dist, rgb, alpha, znum, nnum, l1, l2, median, w, aux, raw};
  const int64_t total = (int64_t)B * P;
  if (total == 0) return cudaSuccess;
  count_launches(1);
  composite_forward_kernel<<<(unsigned)((total + 127) / 128), 128, 0, s>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || !(dist & SF_DIST_L1)) return e;
  const int k = (N + 31) / 32 * 32;
  const size_t per = composite_l1_smem_per_warp(N);
  if (per > 200 * 1024) return cudaErrorInvalidValue;
  const int warps = (int)((200 * 1024 / per) < 4 ? (200 * 1024 / per) : 4);
  const size_t smem = per * warps;
  e = cudaFuncSetAttribute(composite_l1_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  int64_t blocks = (total + warps - 1) / warps;
  if (blocks > 148 * 32) blocks = 148 * 32;
  count_launches(1);
  composite_l1_kernel<<<(unsigned)blocks, warps * 32, smem, s>>>(a, k);
  return cudaGetLastError();
}

cudaError_t launch_composite_backward(const float* al, const float* col, const float* dep, const float* nrm, int B,
                                      int N, int P, int dist, const float* w, const float* aux, const float* raw,
                                      const float* g_rgb, const float* g_alpha, const float* g_znum,
                                      const float* g_nnum, const float* g_l1, const float* g_l2,
                                      const float* g_median, const float* g_w, float* da, float* dc, float* dd,
                                      float* dn, cudaStream_t s) {
  CompositeArgs a{al, col, dep, nrm, B, N, P, dist, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                  nullptr, const_cast<float*>(w), const_cast<float*>(aux), const_cast<float*>(raw)};
  CompositeGrads g{g_rgb, g_alpha, g_znum, g_nnum, g_l1, g_l2, g_median, g_w, da, dd, dn, dc};
  const int64_t total = (int64_t)B * P;
  if (total > 0) {
    count_launches(1);
    composite_backward_kernel<<<(unsigned)((total + 127) / 128), 128, 0, s>>>(a, g);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  const int64_t bn = (int64_t)B * N;
  if (bn > 0) {
    count_launches(1);
    composite_color_grad_kernel<<<(unsigned)((bn * 32 + 255) / 256), 256, 0, s>>>(a, g);
  }
  return cudaGetLastError();
}

// ------------------------------------------------------------------ ray colour variance
// gaussian.ray_color_variance@1/@2 (reference.py:120-122, 189-191): per batch b and pixel
// p, sum_n w[b,n,p] |c[b,n] - composite[b,p]|^2 with the weights and the composite
// detached; the adjoint reaches the colours only: g_c[b,n] = 2 sum_p g[b,p] w[b,n,p]
// (c[b,n] - composite[b,p]).
namespace {
__global__ void ray_color_variance_kernel(const float* w, const float* c, const float* comp, int64_t B, int64_t N,
                                          int64_t P, float* out) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= B * P) return;
  const int64_t b = j / P, p = j - b * P;
  const float r0 = comp[j * 3], r1 = comp[j * 3 + 1], r2 = comp[j * 3 + 2];
  float acc = 0.f;
  for (int64_t n = 0; n < N; ++n) {
    const float* cn = c + (b * N + n) * 3;
    const float e0 = cn[0] - r0, e1 = cn[1] - r1, e2 = cn[2] - r2;
    acc += w[(b * N + n) * P + p] * (e0 * e0 + e1 * e1 + e2 * e2);
  }
  out[j] = acc;
}

// one warp per (b, n)
__global__ void ray_color_variance_backward_kernel(const float* w, const float* c, const float* comp, const float* g,
                                                   int64_t B, int64_t N, int64_t P, float* g_c) {
  const int64_t k = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (k >= B * N) return;
  const int64_t b = k / N;
  const float c0 = c[k * 3], c1 = c[k * 3 + 1], c2 = c[k * 3 + 2];
  float a0 = 0.f, a1 = 0.f, a2 = 0.f;
  for (int64_t p = lane; p < P; p += 32) {
    const float s = 2.f * g[b * P + p] * w[k * P + p];
    const float* r = comp + (b * P + p) * 3;
    a0 += s * (c0 - r[0]);
    a1 += s * (c1 - r[1]);
    a2 += s * (c2 - r[2]);
  }
  a0 = warp_sum(a0);
  a1 = warp_sum(a1);
  a2 = warp_sum(a2);
  if (lane == 0) {
    g_c[k * 3] = a0;
    g_c[k * 3 + 1] = a1;
    g_c[k * 3 + 2] = a2;
  }
}
}  // namespace

cudaError_t launch_ray_color_variance(const float* w, const float* c, const float* comp, int64_t B, int64_t N,
                                      int64_t P, float* out, cudaStream_t s) {
  if (B * P == 0) return cudaSuccess;
  count_launches(1);
  ray_color_variance_kernel<<<(unsigned)((B * P + 255) / 256), 256, 0, s>>>(w, c, comp, B, N, P, out);
  return cudaGetLastError();
}

cudaError_t launch_ray_color_variance_backward(const float* w, const float* c, const float* comp, const float* g,
                                               int64_t B, int64_t N, int64_t P, float* g_c, cudaStream_t s) {
  if (B * N == 0) return cudaSuccess;
  count_launches(1);
  ray_color_variance_backward_kernel<<<(unsigned)((B * N + 7) / 8), 256, 0, s>>>(w, c, comp, g, B, N, P, g_c);
  return cudaGetLastError();
}

}  // namespace sf
