// Per-Gaussian and per-(pixel, Gaussian) arithmetic of the rasterizer, shared by the
// CUDA kernels and by the host-compiled arithmetic check used in the CPU tests.
//
// Quantities that feed a discrete decision -- camera depth (compositing order), the
// projected bounds (tile rectangles) and the Mahalanobis distance tested against
// extent^2 -- are evaluated as fixed sequences of correctly rounded float32
// operations (rmul/radd/rsub/rdiv/rsqrt_rn below: never contracted into FMA).  The
// CPU oracle performs the same sequences with separate tensor operations, so both
// make the same decisions bit for bit.  Everything else is free-form float32.
#pragma once

#include <math.h>
#include <stdint.h>

#include "../../include/splatforge_b200.h"

#if defined(__CUDACC__)
#define SF_HD __host__ __device__ __forceinline__
#else
#define SF_HD inline
#endif

namespace sf {

// ---------------------------------------------------------------- exact operations
SF_HD float rmul(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fmul_rn(a, b);
#else
  return a * b;  // host build uses -ffp-contract=off
#endif
}
SF_HD float radd(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fadd_rn(a, b);
#else
  return a + b;
#endif
}
SF_HD float rsub(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fsub_rn(a, b);
#else
  return a - b;
#endif
}
SF_HD float rdiv(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fdiv_rn(a, b);
#else
  return a / b;
#endif
}
SF_HD float rsqrt_rn(float a) {
#if defined(__CUDA_ARCH__)
  return __fsqrt_rn(a);
#else
  return sqrtf(a);
#endif
}
// Explicitly fused multiply-add (never re-associated): together with rmul/radd it
// makes a sample's depth, response and alpha a fixed function of its inputs, so the
// forward and backward kernels reach bit-identical membership decisions.
SF_HD float ffma(float a, float b, float c) {
#if defined(__CUDA_ARCH__)
  return __fmaf_rn(a, b, c);
#else
  return fmaf(a, b, c);
#endif
}
SF_HD float dot3(float a0, float a1, float a2, float b0, float b1, float b2) {
  return ffma(a2, b2, ffma(a1, b1, rmul(a0, b0)));
}

SF_HD float fmaxr(float a, float b) { return a > b ? a : b; }

// reciprocal for values that feed no discrete decision (within 2 ulp on the device)
SF_HD float fast_rcp(float a) {
#if defined(__CUDA_ARCH__)
  return __fdividef(1.f, a);
#else
  return 1.f / a;
#endif
}
SF_HD int f2i(float f) {
#if defined(__CUDA_ARCH__)
  return __float_as_int(f);
#else
  union { float f; int i; } u; u.f = f; return u.i;
#endif
}
SF_HD float i2f(int i) {
#if defined(__CUDA_ARCH__)
  return __int_as_float(i);
#else
  union { float f; int i; } u; u.i = i; return u.f;
#endif
}
SF_HD float fminr(float a, float b) { return a < b ? a : b; }

// record layout (floats per Gaussian), see SF_RECORD_FLOATS
enum : int {
  R_X = 0, R_Y = 1, R_QA = 2, R_QB = 3, R_QC = 4, R_OPA = 5, R_RGB = 6, R_SEL = 9, R_Z = 10,
  // RaDe-GS
  R_RADIAL = 11, R_GAIN = 12, R_NRM = 14,
  // GOF
  R_PROXY = 11, R_Q3 = 14,
  // AmbiSuR
  R_ANRM = 11, R_PLANE = 14,
  // gradient-record extras (AmbiSuR ray colour adjoint)
  G_RAYC = 15
};

// pixel-state layout (floats per pixel), see SF_PIXEL_STATE_FLOATS
enum : int {
  PS_T = 0, PS_W = 1, PS_D = 2, PS_D2 = 3, PS_C = 4, PS_N = 7, PS_DNUM = 10, PS_L1 = 11,
  PS_L2 = 12, PS_LAST = 13, PS_MEDIAN = 14, PS_COUNT = 15
};

// Real SH constants of the gsplat/3DGS basis (reference.py:87-109)
constexpr float SH_C0 = 0.28209479177387814f;   // 1/sqrt(4 pi)
constexpr float SH_C1 = 0.4886025119029199f;    // sqrt(3/(4 pi))
constexpr float SH_C2 = 1.0925484305920792f;    // sqrt(15/(4 pi))
constexpr float SH_C2B = 0.31539156525252005f;  // sqrt(5/(16 pi))
constexpr float SH_C2C = 0.5462742152960396f;   // sqrt(15/(16 pi))
constexpr float SH_C30 = 0.5900435899266435f;   // sqrt(35/(32 pi))
constexpr float SH_C31 = 2.890611442640554f;    // sqrt(105/(4 pi))
constexpr float SH_C32 = 0.4570457994644658f;   // sqrt(21/(32 pi))
constexpr float SH_C33 = 0.3731763325901154f;   // sqrt(7/(16 pi))
constexpr float SH_C34 = 1.445305721320277f;    // sqrt(105/(16 pi))

SF_HD int sh_count(int degree) { return (degree + 1) * (degree + 1); }

SF_HD void sh_basis(float x, float y, float z, int degree, float* b) {
  b[0] = SH_C0;
  if (degree >= 1) { b[1] = -SH_C1 * y; b[2] = SH_C1 * z; b[3] = -SH_C1 * x; }
  if (degree >= 2) {
    b[4] = SH_C2 * x * y;
    b[5] = -SH_C2 * y * z;
    b[6] = SH_C2B * (3.f * z * z - 1.f);
    b[7] = -SH_C2 * x * z;
    b[8] = SH_C2C * (x * x - y * y);
  }
  if (degree >= 3) {
    b[9] = -SH_C30 * y * (3.f * x * x - y * y);
    b[10] = SH_C31 * x * y * z;
    b[11] = -SH_C32 * y * (5.f * z * z - 1.f);
    b[12] = SH_C33 * z * (5.f * z * z - 3.f);
    b[13] = -SH_C32 * x * (5.f * z * z - 1.f);
    b[14] = SH_C34 * z * (x * x - y * y);
    b[15] = -SH_C30 * x * (x * x - 3.f * y * y);
  }
}

// adjoint of the unit direction given the adjoint of every basis value
SF_HD void sh_basis_backward(float x, float y, float z, int degree, const float* gb, float* gd) {
  float gx = 0.f, gy = 0.f, gz = 0.f;
  if (degree >= 1) { gy -= SH_C1 * gb[1]; gz += SH_C1 * gb[2]; gx -= SH_C1 * gb[3]; }
  if (degree >= 2) {
    gx += SH_C2 * y * gb[4]; gy += SH_C2 * x * gb[4];
    gy -= SH_C2 * z * gb[5]; gz -= SH_C2 * y * gb[5];
    gz += 6.f * SH_C2B * z * gb[6];
    gx -= SH_C2 * z * gb[7]; gz -= SH_C2 * x * gb[7];
    gx += 2.f * SH_C2C * x * gb[8]; gy -= 2.f * SH_C2C * y * gb[8];
  }
  if (degree >= 3) {
    gx -= SH_C30 * 6.f * x * y * gb[9];
    gy -= SH_C30 * (3.f * x * x - 3.f * y * y) * gb[9];
    gx += SH_C31 * y * z * gb[10]; gy += SH_C31 * x * z * gb[10]; gz += SH_C31 * x * y * gb[10];
    gy -= SH_C32 * (5.f * z * z - 1.f) * gb[11]; gz -= SH_C32 * 10.f * y * z * gb[11];
    gz += SH_C33 * (15.f * z * z - 3.f) * gb[12];
    gx -= SH_C32 * (5.f * z * z - 1.f) * gb[13]; gz -= SH_C32 * 10.f * x * z * gb[13];
    gx += 2.f * SH_C34 * x * z * gb[14]; gy -= 2.f * SH_C34 * y * z * gb[14];
    gz += SH_C34 * (x * x - y * y) * gb[14];
    gx -= SH_C30 * (3.f * x * x - 3.f * y * y) * gb[15]; gy += 6.f * SH_C30 * x * y * gb[15];
  }
  gd[0] = gx; gd[1] = gy; gd[2] = gz;
}

// v / max(|v|, 1e-12) and its adjoint (torch.nn.functional.normalize)
SF_HD float norm3(const float* v) { return sqrtf(v[0] * v[0] + v[1] * v[1] + v[2] * v[2]); }
SF_HD void unit3(const float* v, float* out) {
  float n = fmaxr(norm3(v), 1e-12f);
  out[0] = v[0] / n; out[1] = v[1] / n; out[2] = v[2] / n;
}
SF_HD void unit3_backward(const float* v, const float* g, float* gv) {
  float n = norm3(v);
  if (n >= 1e-12f) {
    float inv = 1.f / n;
    float u0 = v[0] * inv, u1 = v[1] * inv, u2 = v[2] * inv;
    float d = u0 * g[0] + u1 * g[1] + u2 * g[2];
    gv[0] = (g[0] - u0 * d) * inv; gv[1] = (g[1] - u1 * d) * inv; gv[2] = (g[2] - u2 * d) * inv;
  } else {
    gv[0] = g[0] * 1e12f; gv[1] = g[1] * 1e12f; gv[2] = g[2] * 1e12f;
  }
}

// SH colour max(0, 0.5 + sum_k c_k Y_k(unit(dir))) for one Gaussian; coeffs [K,3]
SF_HD void sh_color(const float* coeffs, int degree, const float* dir, float* rgb) {
  float d[3];
  unit3(dir, d);
  float b[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) b[k] = 0.f;
  sh_basis(d[0], d[1], d[2], degree, b);
  const int K = sh_count(degree);
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k)
      if (k < K) acc += coeffs[k * 3 + c] * b[k];
    rgb[c] = fmaxr(0.5f + acc, 0.f);
  }
}

// Adjoint of sh_color.  g_live flows to coefficients and direction, g_detached
// (the AmbiSuR ray colour, whose direction is detached) to the coefficients only.
SF_HD void sh_color_backward(const float* coeffs, int degree, const float* dir,
                             const float* g_live, const float* g_detached, float* g_coeffs,
                             float* g_dir) {
  float d[3];
  unit3(dir, d);
  // fixed-size loops with a bound check (k < K), fully unrolled, so that b and gb stay
  // in registers for any degree
  float b[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) b[k] = 0.f;
  sh_basis(d[0], d[1], d[2], degree, b);
  const int K = sh_count(degree);
  float gl[3], gdt[3];
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k)
      if (k < K) acc += coeffs[k * 3 + c] * b[k];
    bool pass = (0.5f + acc) >= 0.f;  // clamp_min(0) passes at >= 0
    gl[c] = pass && g_live ? g_live[c] : 0.f;
    gdt[c] = pass && g_detached ? g_detached[c] : 0.f;
  }
  float gb[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    gb[k] = 0.f;
    if (k < K) {
      gb[k] = coeffs[k * 3 + 0] * gl[0] + coeffs[k * 3 + 1] * gl[1] + coeffs[k * 3 + 2] * gl[2];
      if (g_coeffs) {
        g_coeffs[k * 3 + 0] = b[k] * (gl[0] + gdt[0]);
        g_coeffs[k * 3 + 1] = b[k] * (gl[1] + gdt[1]);
        g_coeffs[k * 3 + 2] = b[k] * (gl[2] + gdt[2]);
      }
    }
  }
  if (g_dir) {
    float gu[3];
    sh_basis_backward(d[0], d[1], d[2], degree, gb, gu);
    unit3_backward(dir, gu, g_dir);
  }
}

// ---------------------------------------------------------------- rotation / covariance
// normalised wxyz quaternion -> R (reference.py:15-30), exact-sequence evaluation
SF_HD float quat_normalize(const float* q, float* qn) {
  float n = rsqrt_rn(radd(radd(radd(rmul(q[0], q[0]), rmul(q[1], q[1])), rmul(q[2], q[2])),
                          rmul(q[3], q[3])));
  float nc = fmaxr(n, 1e-12f);
  for (int k = 0; k < 4; ++k) qn[k] = rdiv(q[k], nc);
  return n;
}

SF_HD void quat_rotation(const float* qn, float* R) {
  float w = qn[0], x = qn[1], y = qn[2], z = qn[3];
  R[0] = rsub(1.f, rmul(2.f, radd(rmul(y, y), rmul(z, z))));
  R[1] = rmul(2.f, rsub(rmul(x, y), rmul(w, z)));
  R[2] = rmul(2.f, radd(rmul(x, z), rmul(w, y)));
  R[3] = rmul(2.f, radd(rmul(x, y), rmul(w, z)));
  R[4] = rsub(1.f, rmul(2.f, radd(rmul(x, x), rmul(z, z))));
  R[5] = rmul(2.f, rsub(rmul(y, z), rmul(w, x)));
  R[6] = rmul(2.f, rsub(rmul(x, z), rmul(w, y)));
  R[7] = rmul(2.f, radd(rmul(y, z), rmul(w, x)));
  R[8] = rsub(1.f, rmul(2.f, radd(rmul(x, x), rmul(y, y))));
}

// C = R diag(s*s) R^T as (M_i0 R_j0 + M_i1 R_j1) + M_i2 R_j2 with M = R diag(s*s)
SF_HD void covariance3(const float* R, const float* s, float* C) {
  float s2[3] = {rmul(s[0], s[0]), rmul(s[1], s[1]), rmul(s[2], s[2])};
  float M[9];
  for (int i = 0; i < 3; ++i)
    for (int k = 0; k < 3; ++k) M[i * 3 + k] = rmul(R[i * 3 + k], s2[k]);
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j)
      C[i * 3 + j] = radd(radd(rmul(M[i * 3 + 0], R[j * 3 + 0]), rmul(M[i * 3 + 1], R[j * 3 + 1])),
                          rmul(M[i * 3 + 2], R[j * 3 + 2]));
}

// adjoint of quat_rotation wrt the normalised quaternion
SF_HD void quat_rotation_backward(const float* qn, const float* gR, float* gq) {
  float w = qn[0], x = qn[1], y = qn[2], z = qn[3];
  gq[0] = 2.f * (-z * gR[1] + y * gR[2] + z * gR[3] - x * gR[5] - y * gR[6] + x * gR[7]);
  gq[1] = 2.f * (y * gR[1] + z * gR[2] + y * gR[3] - 2.f * x * gR[4] - w * gR[5] + z * gR[6] +
                 w * gR[7] - 2.f * x * gR[8]);
  gq[2] = 2.f * (-2.f * y * gR[0] + x * gR[1] + w * gR[2] + x * gR[3] + z * gR[5] - w * gR[6] +
                 z * gR[7] - 2.f * y * gR[8]);
  gq[3] = 2.f * (-2.f * z * gR[0] - w * gR[1] + x * gR[2] + w * gR[3] - 2.f * z * gR[4] +
                 y * gR[5] + x * gR[6] + y * gR[7]);
}

// adjoint of q -> q / max(|q|, 1e-12)
SF_HD void quat_normalize_backward(const float* q, float n, const float* gqn, float* gq) {
  if (n >= 1e-12f) {
    float inv = 1.f / n;
    float u[4] = {q[0] * inv, q[1] * inv, q[2] * inv, q[3] * inv};
    float d = u[0] * gqn[0] + u[1] * gqn[1] + u[2] * gqn[2] + u[3] * gqn[3];
    for (int k = 0; k < 4; ++k) gq[k] = (gqn[k] - u[k] * d) * inv;
  } else {
    for (int k = 0; k < 4; ++k) gq[k] = gqn[k] * 1e12f;
  }
}

// adjoint of C = R diag(s^2) R^T; gC is the full 3x3 adjoint
SF_HD void covariance3_backward(const float* R, const float* s, const float* gC, float* gR,
                                float* gs) {
  float s2[3] = {s[0] * s[0], s[1] * s[1], s[2] * s[2]};
  float Gs[9];
  for (int i = 0; i < 9; ++i) Gs[i] = gC[i] + gC[(i % 3) * 3 + i / 3];  // gC + gC^T
  for (int i = 0; i < 3; ++i)
    for (int k = 0; k < 3; ++k) {
      float acc = 0.f;
      for (int j = 0; j < 3; ++j) acc += Gs[i * 3 + j] * R[j * 3 + k];
      gR[i * 3 + k] = acc * s2[k];
    }
  for (int k = 0; k < 3; ++k) {
    float acc = 0.f;
    for (int i = 0; i < 3; ++i)
      for (int j = 0; j < 3; ++j) acc += R[i * 3 + k] * gC[i * 3 + j] * R[j * 3 + k];
    gs[k] = 2.f * s[k] * acc;
  }
}

// ---------------------------------------------------------------- projection
struct Projection {
  float qn[4], qnorm;
  float R[9];
  float C[9];      // world covariance
  float mc[3];     // camera-space mean
  float Cc[9];     // camera covariance
  bool active;     // z > near
  float zs, xg, yg;
  float j00, j02, j11, j12;
  float X, Y;      // projected mean
  float s00, s01, s11;  // screen covariance
  float fa, fb, fc;     // filtered (screen + eps2d I)
  float det;
  float qa, qb, qc;     // conic = inverse of filtered
  float radius;
};

// renderers.py:76-107 + batched_renderer.py:57-59, exact-sequence evaluation
SF_HD void project(const float* mean, const float* quat, const float* scale,
                   const sf_camera& cam, float eps2d, float near_plane, float extent,
                   Projection& p) {
  p.qnorm = quat_normalize(quat, p.qn);
  quat_rotation(p.qn, p.R);
  covariance3(p.R, scale, p.C);
  const float* W = cam.R;
  for (int i = 0; i < 3; ++i)
    p.mc[i] = radd(radd(radd(rmul(W[i * 3 + 0], mean[0]), rmul(W[i * 3 + 1], mean[1])),
                        rmul(W[i * 3 + 2], mean[2])),
                   cam.t[i]);
  float A[9];
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j)
      A[i * 3 + j] = radd(radd(rmul(W[i * 3 + 0], p.C[0 * 3 + j]), rmul(W[i * 3 + 1], p.C[1 * 3 + j])),
                          rmul(W[i * 3 + 2], p.C[2 * 3 + j]));
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j)
      p.Cc[i * 3 + j] = radd(radd(rmul(A[i * 3 + 0], W[j * 3 + 0]), rmul(A[i * 3 + 1], W[j * 3 + 1])),
                             rmul(A[i * 3 + 2], W[j * 3 + 2]));
  p.active = p.mc[2] > near_plane;
  p.zs = p.active ? p.mc[2] : 1.f;
  p.xg = p.active ? p.mc[0] : 0.f;
  p.yg = p.active ? p.mc[1] : 0.f;
  float fx = cam.K[0], fy = cam.K[4], cx = cam.K[2], cy = cam.K[5];
  float zz = rmul(p.zs, p.zs);
  p.j00 = rdiv(fx, p.zs);
  p.j02 = rdiv(rmul(-fx, p.xg), zz);
  p.j11 = rdiv(fy, p.zs);
  p.j12 = rdiv(rmul(-fy, p.yg), zz);
  p.X = radd(rdiv(rmul(fx, p.xg), p.zs), cx);
  p.Y = radd(rdiv(rmul(fy, p.yg), p.zs), cy);
  const float* c = p.Cc;
  float T00 = radd(rmul(p.j00, c[0]), rmul(p.j02, c[6]));
  float T01 = radd(rmul(p.j00, c[1]), rmul(p.j02, c[7]));
  float T02 = radd(rmul(p.j00, c[2]), rmul(p.j02, c[8]));
  float T11 = radd(rmul(p.j11, c[4]), rmul(p.j12, c[7]));
  float T12 = radd(rmul(p.j11, c[5]), rmul(p.j12, c[8]));
  p.s00 = radd(rmul(T00, p.j00), rmul(T02, p.j02));
  p.s01 = radd(rmul(T01, p.j11), rmul(T02, p.j12));
  p.s11 = radd(rmul(T11, p.j11), rmul(T12, p.j12));
  p.fa = radd(p.s00, eps2d);
  p.fb = p.s01;
  p.fc = radd(p.s11, eps2d);
  p.det = rsub(rmul(p.fa, p.fc), rmul(p.fb, p.fb));
  p.qa = rdiv(p.fc, p.det);
  p.qb = rdiv(-p.fb, p.det);
  p.qc = rdiv(p.fa, p.det);
  float mid = rmul(0.5f, radd(p.fa, p.fc));
  float half = rmul(0.5f, rsub(p.fa, p.fc));
  float lam = radd(mid, rsqrt_rn(radd(rmul(half, half), rmul(p.fb, p.fb))));
  p.radius = rmul(extent, rsqrt_rn(fmaxr(lam, 0.f)));
}

// tile rectangle of tile_binning.py:27-40 from the float32 bounds (x, y, r, z)
SF_HD int tile_rect(float x, float y, float r, float z, int width, int height, int tile,
                    float near_plane, float far_plane, int* rect) {
  int cols = (width + tile - 1) / tile, rows = (height + tile - 1) / tile;
  bool keep = (z > near_plane) && (z < far_plane) && !(radd(x, r) < 0.f) && !(radd(y, r) < 0.f) &&
              !(rsub(x, r) > (float)width) && !(rsub(y, r) > (float)height);
  if (!keep) { rect[0] = rect[1] = rect[2] = rect[3] = 0; return 0; }
  float ts = (float)tile;
  float lx = ceilf(rdiv(rsub(x, r), ts)) - 1.f, hx = floorf(rdiv(radd(x, r), ts));
  float ly = ceilf(rdiv(rsub(y, r), ts)) - 1.f, hy = floorf(rdiv(radd(y, r), ts));
  // clamp in float first: huge bounds must not overflow the int conversion
  lx = fmaxr(lx, 0.f); ly = fmaxr(ly, 0.f);
  hx = fminr(hx, (float)(cols - 1)); hy = fminr(hy, (float)(rows - 1));
  rect[0] = (int)lx; rect[1] = (int)ly; rect[2] = (int)hx; rect[3] = (int)hy;
  int w = rect[2] - rect[0] + 1, h = rect[3] - rect[1] + 1;
  if (w <= 0 || h <= 0) { rect[0] = rect[1] = rect[2] = rect[3] = 0; return 0; }
  return w * h;
}

// 2x2 inverse of a (not necessarily symmetric) matrix, row-major
SF_HD void inv2(const float* a, float* o) {
  float det = a[0] * a[3] - a[1] * a[2];
  float id = 1.f / det;
  o[0] = a[3] * id; o[1] = -a[1] * id; o[2] = -a[2] * id; o[3] = a[0] * id;
}

// inverse of a symmetric 3x3 (upper triangle of the symmetrised input) -> 6 values
SF_HD void inv3_sym(const float* c, float* q) {
  float a = c[0], b = 0.5f * (c[1] + c[3]), d = 0.5f * (c[2] + c[6]);
  float e = c[4], f = 0.5f * (c[5] + c[7]), i = c[8];
  float A = e * i - f * f, B = -(b * i - d * f), Cf = b * f - d * e;
  float det = a * A + b * B + d * Cf;
  float id = 1.f / det;
  q[0] = A * id;                  // 00
  q[1] = B * id;                  // 01
  q[2] = Cf * id;                 // 02
  q[3] = (a * i - d * d) * id;    // 11
  q[4] = -(a * f - b * d) * id;   // 12
  q[5] = (a * e - b * b) * id;    // 22
}

// RaDe-GS extras (batched_renderer.py:90-99): radial distance, gain, normal
struct RadeExtras {
  float mhat[3], radial;
  float F[9];      // [J; mhat]
  float Tm[9];     // F Cc F^T
  float Ainv[4];   // inverse of Tm[:2,:2]
  float gain[2];
  float v[3];      // F^T (gain, -1)
  float normal[3];
};

SF_HD void rade_extras(const Projection& p, RadeExtras& e) {
  e.radial = norm3(p.mc);
  unit3(p.mc, e.mhat);
  float* F = e.F;
  F[0] = p.j00; F[1] = 0.f; F[2] = p.j02;
  F[3] = 0.f; F[4] = p.j11; F[5] = p.j12;
  F[6] = e.mhat[0]; F[7] = e.mhat[1]; F[8] = e.mhat[2];
  float FC[9];
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j)
      FC[i * 3 + j] = F[i * 3 + 0] * p.Cc[0 * 3 + j] + F[i * 3 + 1] * p.Cc[1 * 3 + j] + F[i * 3 + 2] * p.Cc[2 * 3 + j];
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j)
      e.Tm[i * 3 + j] = FC[i * 3 + 0] * F[j * 3 + 0] + FC[i * 3 + 1] * F[j * 3 + 1] + FC[i * 3 + 2] * F[j * 3 + 2];
  float A[4] = {e.Tm[0], e.Tm[1], e.Tm[3], e.Tm[4]};
  inv2(A, e.Ainv);
  e.gain[0] = e.Tm[6] * e.Ainv[0] + e.Tm[7] * e.Ainv[2];
  e.gain[1] = e.Tm[6] * e.Ainv[1] + e.Tm[7] * e.Ainv[3];
  float rn[3] = {e.gain[0], e.gain[1], -1.f};
  for (int j = 0; j < 3; ++j) e.v[j] = F[0 * 3 + j] * rn[0] + F[1 * 3 + j] * rn[1] + F[2 * 3 + j] * rn[2];
  unit3(e.v, e.normal);
}

// AmbiSuR extras (batched_renderer.py:100-111): camera normal of the thinnest axis,
// flipped to face the camera, and the plane distance n . m
struct AmbiExtras {
  int axis;
  float sign;
  float normal[3];
  float plane;
};

// (a0 b0 + a1 b1) + a2 b2 with every product and sum rounded on its own (no FMA)
SF_HD float dot3_rn(float a0, float a1, float a2, float b0, float b1, float b2) {
  return radd(radd(rmul(a0, b0), rmul(a1, b1)), rmul(a2, b2));
}

// The AmbiSuR plane (batched_renderer.py:96-108): the rotation's column of the smallest
// scale, turned into the camera frame and flipped to face the camera, and its plane
// distance.  The per-pixel plane depth plane / (n . ray) is ill-conditioned at grazing
// angles, so every step here is an exact-rounding sequence on the projection's exact
// rotation (the oracle performs the same sequence).
SF_HD void ambi_extras(const float* scale, const Projection& p, const sf_camera& cam, AmbiExtras& e) {
  int a = 0;
  if (scale[1] < scale[a]) a = 1;
  if (scale[2] < scale[a]) a = 2;
  e.axis = a;
  // column a of R, selected with constant indices (keeps R in registers)
  const float w0 = a == 0 ? p.R[0] : (a == 1 ? p.R[1] : p.R[2]);
  const float w1 = a == 0 ? p.R[3] : (a == 1 ? p.R[4] : p.R[5]);
  const float w2 = a == 0 ? p.R[6] : (a == 1 ? p.R[7] : p.R[8]);
  float nc[3];
  for (int i = 0; i < 3; ++i) nc[i] = dot3_rn(w0, w1, w2, cam.R[i * 3 + 0], cam.R[i * 3 + 1], cam.R[i * 3 + 2]);
  const float facing = dot3_rn(nc[0], nc[1], nc[2], p.mc[0], p.mc[1], p.mc[2]);
  e.sign = facing > 0.f ? -1.f : 1.f;
  for (int i = 0; i < 3; ++i) e.normal[i] = e.sign * nc[i];
  e.plane = dot3_rn(e.normal[0], e.normal[1], e.normal[2], p.mc[0], p.mc[1], p.mc[2]);
}

// ---------------------------------------------------------------- per-pixel geometry
struct PixelRay {
  float r[3];   // inv(K) (u+.5, v+.5, 1)
  float px, py; // K r (pixel coordinates as the reference recomputes them)
  float rnorm;  // |r|
  float inv_rnorm;  // 1 / |r|
};

SF_HD void pixel_ray(const sf_camera& cam, int u, int v, PixelRay& pr) {
  float uf = (float)u + 0.5f, vf = (float)v + 0.5f;
  const float* Ki = cam.Kinv;
  const float* K = cam.K;
  for (int i = 0; i < 3; ++i)
    pr.r[i] = radd(radd(rmul(uf, Ki[i * 3 + 0]), rmul(vf, Ki[i * 3 + 1])), Ki[i * 3 + 2]);
  pr.px = radd(radd(rmul(pr.r[0], K[0]), rmul(pr.r[1], K[1])), rmul(pr.r[2], K[2]));
  pr.py = radd(radd(rmul(pr.r[0], K[3]), rmul(pr.r[1], K[4])), rmul(pr.r[2], K[5]));
  pr.rnorm = rsqrt_rn(dot3(pr.r[0], pr.r[1], pr.r[2], pr.r[0], pr.r[1], pr.r[2]));
  pr.inv_rnorm = rdiv(1.f, pr.rnorm);
}

// exp for the per-sample response: the hardware exp2 path on the device (within a few
// ulp), the C library on the host.  The response feeds no bit-exact comparison with
// the oracle; the forward and backward kernels evaluate it with the same instructions.
SF_HD float fast_exp(float x) {
#if defined(__CUDA_ARCH__)
  return __expf(x);
#else
  return expf(x);
#endif
}

// delta^T Q delta as dx (Q delta)_x + dy (Q delta)_y, exact sequence
SF_HD float mahalanobis2(float dx, float dy, float qa, float qb, float qc) {
  return radd(rmul(dx, radd(rmul(qa, dx), rmul(qb, dy))), rmul(dy, radd(rmul(qb, dx), rmul(qc, dy))));
}

// q(x, y) = qa x^2 + 2 qb x y + qc y^2 and the sum of the magnitudes of its terms
SF_HD float quad_form(float qa, float qb, float qc, float x, float y, float& mag) {
  const float t0 = qa * x * x, t1 = 2.f * qb * x * y, t2 = qc * y * y;
  mag = fabsf(t0) + fabsf(t1) + fabsf(t2);
  return t0 + t1 + t2;
}

// May a Gaussian centred at (X, Y) with conic (qa, qb; qb, qc) pass squared <= ext2 at
// some pixel centre inside the box [x0, x1] x [y0, y1]?  Takes the minimum of the
// quadratic form over the box: zero when the centre is inside, else the smallest of
// the four edge minima (the 1D minimiser of a convex quadratic, clamped to the edge).
// Conservative by a margin far above the float rounding of either evaluation; a
// degenerate conic or a NaN always answers yes.
SF_HD bool box_may_pass(float qa, float qb, float qc, float X, float Y, float x0, float x1, float y0, float y1,
                        float ext2) {
  const float ax = x0 - X, bx = x1 - X, ay = y0 - Y, by = y1 - Y;
  if (!(qa > 0.f && qc > 0.f && qa * qc - qb * qb > 0.f)) return true;
  if (ax <= 0.f && bx >= 0.f && ay <= 0.f && by >= 0.f) return true;
  const float sy = -qb / qc, sx = -qb / qa;
  float mag, val;
  bool hit = false;
  val = quad_form(qa, qb, qc, ax, fminf(fmaxf(sy * ax, ay), by), mag);
  hit |= !(val > ext2 + 1e-5f * mag + 1e-6f);
  val = quad_form(qa, qb, qc, bx, fminf(fmaxf(sy * bx, ay), by), mag);
  hit |= !(val > ext2 + 1e-5f * mag + 1e-6f);
  val = quad_form(qa, qb, qc, fminf(fmaxf(sx * ay, ax), bx), ay, mag);
  hit |= !(val > ext2 + 1e-5f * mag + 1e-6f);
  val = quad_form(qa, qb, qc, fminf(fmaxf(sx * by, ax), bx), by, mag);
  hit |= !(val > ext2 + 1e-5f * mag + 1e-6f);
  return hit;
}

// One (pixel, Gaussian) sample of the per-tile evaluation (batched_renderer.py:240-306)
struct Sample {
  float dx, dy, sq;
  float resp;      // response after the validity mask
  float a_raw;     // opacity * response (before the [0, 0.999] clamp)
  float alpha;     // clamped
  float depth;
  float n[3];      // sample normal (GOF: normalize(-Q d); else per-Gaussian)
  // GOF intermediates (qo = Q off; ninv = 1 / max(|Q r|, 1e-12); inv_den = 1 / den)
  float qd[3], den_raw, den, inv_den, t, off[3], e, qo[3], ninv;
  // AmbiSuR intermediates
  float aden;
  bool aok;
};

// CHECK = false evaluates the values of a sample already known to contribute
// without re-testing the masks.
template <int MODE, bool CHECK = true>
SF_HD bool eval_sample(const float* rec, const PixelRay& pr, float ext2, float near_plane,
                       float far_plane, Sample& s) {
  s.dx = rsub(pr.px, rec[R_X]);
  s.dy = rsub(pr.py, rec[R_Y]);
  s.sq = mahalanobis2(s.dx, s.dy, rec[R_QA], rec[R_QB], rec[R_QC]);
  if (CHECK && !(s.sq <= ext2)) return false;
  float resp;
  if (MODE == SF_MODE_GOF) {
    const float* q = rec + R_Q3;  // q00 q01 q02 q11 q12 q22
    const float* r = pr.r;
    s.qd[0] = dot3(q[0], q[1], q[2], r[0], r[1], r[2]);
    s.qd[1] = dot3(q[1], q[3], q[4], r[0], r[1], r[2]);
    s.qd[2] = dot3(q[2], q[4], q[5], r[0], r[1], r[2]);
    s.den_raw = dot3(s.qd[0], s.qd[1], s.qd[2], r[0], r[1], r[2]);
    s.den = fmaxr(s.den_raw, 1e-12f);
    const float* pm = rec + R_PROXY;
    s.inv_den = fast_rcp(s.den);
    s.t = dot3(pm[0], pm[1], pm[2], s.qd[0], s.qd[1], s.qd[2]) * s.inv_den;
    s.off[0] = ffma(s.t, r[0], -pm[0]);
    s.off[1] = ffma(s.t, r[1], -pm[1]);
    s.off[2] = ffma(s.t, r[2], -pm[2]);
    s.qo[0] = dot3(q[0], q[1], q[2], s.off[0], s.off[1], s.off[2]);
    s.qo[1] = dot3(q[1], q[3], q[4], s.off[0], s.off[1], s.off[2]);
    s.qo[2] = dot3(q[2], q[4], q[5], s.off[0], s.off[1], s.off[2]);
    s.e = dot3(s.off[0], s.off[1], s.off[2], s.qo[0], s.qo[1], s.qo[2]);
    resp = fast_exp(rmul(-0.5f, fmaxr(s.e, 0.f)));
    s.depth = s.t;
    // normal = normalize(-Q r), one reciprocal square root (F.normalize's 1e-12 guard)
    const float nn = s.qd[0] * s.qd[0] + s.qd[1] * s.qd[1] + s.qd[2] * s.qd[2];
#if defined(__CUDA_ARCH__)
    s.ninv = rsqrtf(fmaxf(nn, 1e-24f));
#else
    s.ninv = 1.f / sqrtf(nn > 1e-24f ? nn : 1e-24f);
#endif
    s.n[0] = -s.qd[0] * s.ninv; s.n[1] = -s.qd[1] * s.ninv; s.n[2] = -s.qd[2] * s.ninv;
  } else {
    resp = fast_exp(rmul(-0.5f, s.sq));
    if (MODE == SF_MODE_RADEGS) {
      s.depth = radd(rec[R_RADIAL], ffma(rec[R_GAIN + 1], s.dy, rmul(rec[R_GAIN], s.dx))) * pr.inv_rnorm;
      s.n[0] = rec[R_NRM]; s.n[1] = rec[R_NRM + 1]; s.n[2] = rec[R_NRM + 2];
    } else {
      s.n[0] = rec[R_ANRM]; s.n[1] = rec[R_ANRM + 1]; s.n[2] = rec[R_ANRM + 2];
      // exact rounding: n . ray is ill-conditioned at grazing angles, and the depth
      // decides near/far membership
      s.aden = dot3_rn(s.n[0], s.n[1], s.n[2], pr.r[0], pr.r[1], pr.r[2]);
      s.aok = fabsf(s.aden) > 1e-8f;
      s.depth = rdiv(rec[R_PLANE], s.aok ? s.aden : 1.f);
      if (!s.aok) resp = 0.f;
    }
  }
  if (CHECK && !(s.depth > near_plane && s.depth < far_plane)) return false;
  s.resp = resp;
  s.a_raw = rmul(rec[R_OPA], resp);
  s.alpha = fminr(fmaxr(s.a_raw, 0.f), 0.999f);
  return s.alpha > 0.f;
}

}  // namespace sf
