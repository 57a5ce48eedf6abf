// Reverse-mode arithmetic of the rasterizer (the autograd of the Torch provider's
// composition, written out): per-pixel epilogue adjoints, per-sample adjoints and
// the per-Gaussian projection adjoint.  Shared by the CUDA kernels and the
// host-compiled arithmetic check.
#pragma once

#include "sf_math.cuh"

namespace sf {

// ---------------------------------------------------------------- per-pixel epilogue
// Adjoints of the composited numerators, given the adjoints of the output images
// (batched_renderer.py:310-338): rgb + (1-alpha) bg, expected depth, normalised
// normal, clamped distortions, median, ray-colour variance, ambiguity.
struct PixelGrads {
  float gW, gD, gC[3], gN[3], gDnum, gA, gL1, gL2, gMed, gVar;
  float W, D, C[3];
  int med_pos;
};

struct PixelUpstream {
  float rgb[3], alpha, depth, normal[3], l1, l2, median, var, amb;
};

SF_HD void pixel_grads(int mode, int distortions, const float* state, const PixelRay& pr,
                       const float* bg, const PixelUpstream& up, PixelGrads& g) {
  float W = state[PS_W], D = state[PS_D];
  const float* C = state + PS_C;
  const float* N = state + PS_N;
  g.W = W; g.D = D;
  for (int c = 0; c < 3; ++c) { g.C[c] = C[c]; g.gC[c] = up.rgb[c]; }
  g.gW = up.alpha - (up.rgb[0] * bg[0] + up.rgb[1] * bg[1] + up.rgb[2] * bg[2]);
  g.gD = 0.f; g.gDnum = 0.f;
  float gNn[3] = {0.f, 0.f, 0.f};
  unit3_backward(N, up.normal, gNn);
  for (int c = 0; c < 3; ++c) g.gN[c] = gNn[c];
  if (W > 1e-8f) {
    if (mode == SF_MODE_AMBISUR) {
      float den = N[0] * pr.r[0] + N[1] * pr.r[1] + N[2] * pr.r[2];
      if (fabsf(den) > 1e-8f) {
        float dnum = state[PS_DNUM];
        g.gDnum = up.depth / den;
        float gden = -up.depth * dnum / (den * den);
        for (int c = 0; c < 3; ++c) g.gN[c] += gden * pr.r[c];
      }
    } else {
      g.gD = up.depth / W;
      g.gW += -up.depth * D / (W * W);
    }
  }
  g.gA = up.amb;
  g.gL1 = ((distortions & SF_DIST_L1) && state[PS_L1] >= 0.f) ? up.l1 : 0.f;
  g.gL2 = ((distortions & SF_DIST_L2) && state[PS_L2] >= 0.f) ? up.l2 : 0.f;
  g.gMed = up.median;
  g.gVar = mode == SF_MODE_AMBISUR ? up.var : 0.f;
  g.med_pos = f2i(state[PS_MEDIAN]);
}

// ---------------------------------------------------------------- per-sample adjoints
// Number of per-Gaussian values a sample contributes, per mode, and where each lands
// in the gradient accumulator (0..19 mirror the record, 20..21 are absgrad).
template <int MODE> struct SampleLayout;
template <> struct SampleLayout<SF_MODE_GOF> {
  static constexpr int NV = 15;
  SF_HD static int slot(int v) {
    // op, rgb3, proxy3, Q6, abs2
    return v == 0 ? R_OPA : v < 4 ? R_RGB + (v - 1) : v < 7 ? R_PROXY + (v - 4) : v < 13 ? R_Q3 + (v - 7) : 20 + (v - 13);
  }
};
template <> struct SampleLayout<SF_MODE_RADEGS> {
  static constexpr int NV = 17;
  SF_HD static int slot(int v) {
    // xy2, conic3, op, rgb3, radial, gain2, normal3, abs2
    return v < 2 ? R_X + v : v < 5 ? R_QA + (v - 2) : v == 5 ? R_OPA : v < 9 ? R_RGB + (v - 6)
         : v == 9 ? R_RADIAL : v < 12 ? R_GAIN + (v - 10) : v < 15 ? R_NRM + (v - 12) : 20 + (v - 15);
  }
};
template <> struct SampleLayout<SF_MODE_AMBISUR> {
  static constexpr int NV = 18;
  SF_HD static int slot(int v) {
    // xy2, conic3, op, rgb3, normal3, plane, raycolor3, abs2
    return v < 2 ? R_X + v : v < 5 ? R_QA + (v - 2) : v == 5 ? R_OPA : v < 9 ? R_RGB + (v - 6)
         : v < 12 ? R_ANRM + (v - 9) : v == 12 ? R_PLANE : v < 16 ? G_RAYC + (v - 13) : 20 + (v - 16);
  }
};

// Adjoints of one contributing sample.  w = alpha * T_i; g_alpha is the adjoint of
// the clamped alpha (already combining T_i * adj and the suffix term); depth
// adjoint g_depth already includes median / L1 / L2 terms.
template <int MODE>
SF_HD void sample_backward(const float* rec, const PixelRay& pr, const Sample& s,
                           const PixelGrads& pg, float w, float g_alpha, float g_depth,
                           float inv_fx, float inv_fy, float* v) {
  float g_a = (s.a_raw >= 0.f && s.a_raw <= 0.999f) ? g_alpha : 0.f;
  float opa = rec[R_OPA];
  float g_resp = opa * g_a;
  float d_op = s.resp * g_a;
  if (MODE == SF_MODE_GOF) {
    const float* r = pr.r;
    const float* pm = rec + R_PROXY;
    float g_e = (s.e >= 0.f) ? -0.5f * s.resp * g_resp : 0.f;
    float goff0 = 2.f * g_e * s.qo[0], goff1 = 2.f * g_e * s.qo[1], goff2 = 2.f * g_e * s.qo[2];
    float gQ[6];
    gQ[0] = g_e * s.off[0] * s.off[0];
    gQ[1] = 2.f * g_e * s.off[0] * s.off[1];
    gQ[2] = 2.f * g_e * s.off[0] * s.off[2];
    gQ[3] = g_e * s.off[1] * s.off[1];
    gQ[4] = 2.f * g_e * s.off[1] * s.off[2];
    gQ[5] = g_e * s.off[2] * s.off[2];
    float g_t = g_depth + (r[0] * goff0 + r[1] * goff1 + r[2] * goff2);
    float gp0 = -goff0, gp1 = -goff1, gp2 = -goff2;
    float g_num = g_t * s.inv_den;
    float g_den = -g_num * s.t;
    gp0 += g_num * s.qd[0]; gp1 += g_num * s.qd[1]; gp2 += g_num * s.qd[2];
    float gqd0 = g_num * pm[0], gqd1 = g_num * pm[1], gqd2 = g_num * pm[2];
    if (s.den_raw >= 1e-12f) { gqd0 += g_den * r[0]; gqd1 += g_den * r[1]; gqd2 += g_den * r[2]; }
    // adjoint of n = normalize(-qd) with the forward's unit vector and inverse norm
    {
      const float g0 = w * pg.gN[0], g1 = w * pg.gN[1], g2 = w * pg.gN[2];
      const float d = s.n[0] * g0 + s.n[1] * g1 + s.n[2] * g2;
      const float c = s.ninv < 1e12f ? 1.f : 0.f;  // below the guard: n = -qd * 1e12
      gqd0 -= (g0 - c * s.n[0] * d) * s.ninv;
      gqd1 -= (g1 - c * s.n[1] * d) * s.ninv;
      gqd2 -= (g2 - c * s.n[2] * d) * s.ninv;
    }
    gQ[0] += gqd0 * r[0];
    gQ[1] += gqd0 * r[1] + gqd1 * r[0];
    gQ[2] += gqd0 * r[2] + gqd2 * r[0];
    gQ[3] += gqd1 * r[1];
    gQ[4] += gqd1 * r[2] + gqd2 * r[1];
    gQ[5] += gqd2 * r[2];
    float z = rec[R_Z];
    v[0] = d_op;
    v[1] = w * pg.gC[0]; v[2] = w * pg.gC[1]; v[3] = w * pg.gC[2];
    v[4] = gp0; v[5] = gp1; v[6] = gp2;
    for (int k = 0; k < 6; ++k) v[7 + k] = gQ[k];
    v[13] = fabsf(gp0 * z * inv_fx);
    v[14] = fabsf(gp1 * z * inv_fy);
  } else {
    float g_sq = -0.5f * s.resp * g_resp;
    float qa = rec[R_QA], qb = rec[R_QB], qc = rec[R_QC];
    float gdx = g_sq * 2.f * (qa * s.dx + qb * s.dy);
    float gdy = g_sq * 2.f * (qb * s.dx + qc * s.dy);
    float gqa = g_sq * s.dx * s.dx, gqb = g_sq * 2.f * s.dx * s.dy, gqc = g_sq * s.dy * s.dy;
    if (MODE == SF_MODE_RADEGS) {
      float inv = pr.inv_rnorm;
      float g_rad = g_depth * inv;
      float gg0 = g_depth * s.dx * inv, gg1 = g_depth * s.dy * inv;
      gdx += g_depth * rec[R_GAIN] * inv;
      gdy += g_depth * rec[R_GAIN + 1] * inv;
      v[0] = -gdx; v[1] = -gdy;
      v[2] = gqa; v[3] = gqb; v[4] = gqc;
      v[5] = d_op;
      v[6] = w * pg.gC[0]; v[7] = w * pg.gC[1]; v[8] = w * pg.gC[2];
      v[9] = g_rad; v[10] = gg0; v[11] = gg1;
      v[12] = w * pg.gN[0]; v[13] = w * pg.gN[1]; v[14] = w * pg.gN[2];
      v[15] = fabsf(gdx); v[16] = fabsf(gdy);
    } else {
      const float inv_aden = 1.f / s.aden;
      float g_plane = g_depth * inv_aden + w * pg.gDnum;
      float g_aden = -g_depth * s.depth * inv_aden;
      v[0] = -gdx; v[1] = -gdy;
      v[2] = gqa; v[3] = gqb; v[4] = gqc;
      v[5] = d_op;
      v[6] = w * pg.gC[0]; v[7] = w * pg.gC[1]; v[8] = w * pg.gC[2];
      v[9] = w * pg.gN[0] + g_aden * pr.r[0];
      v[10] = w * pg.gN[1] + g_aden * pr.r[1];
      v[11] = w * pg.gN[2] + g_aden * pr.r[2];
      v[12] = g_plane;
      const float* c = rec + R_RGB;
      v[13] = 2.f * w * (c[0] - pg.C[0]) * pg.gVar;
      v[14] = 2.f * w * (c[1] - pg.C[1]) * pg.gVar;
      v[15] = 2.f * w * (c[2] - pg.C[2]) * pg.gVar;
      v[16] = fabsf(gdx); v[17] = fabsf(gdy);
    }
  }
}

// adjoint of w = alpha * T that reaches this sample's alpha, and the per-sample
// adjoint "adj" of w (used by the suffix accumulation)
template <int MODE>
SF_HD float sample_adj(const float* rec, const Sample& s, const PixelGrads& pg, float auxw) {
  const float* c = rec + R_RGB;
  float adj = pg.gW + pg.gD * s.depth + pg.gC[0] * c[0] + pg.gC[1] * c[1] + pg.gC[2] * c[2] +
              pg.gN[0] * s.n[0] + pg.gN[1] * s.n[1] + pg.gN[2] * s.n[2] + pg.gA * rec[R_SEL] +
              pg.gL1 * auxw;
  if (MODE == SF_MODE_AMBISUR) adj += pg.gDnum * rec[R_PLANE];
  return adj;
}

// ---------------------------------------------------------------- projection adjoint
// Reverse of project() + mode extras + SH colour, for one Gaussian.
// MODE fixed at compile time (the kernels instantiate one per rendering mode); the
// untemplated overload below dispatches on st.mode
template <int MODE>
SF_HD void project_backward_mode(const float* mean, const float* quat, const float* scale,
                            float opacity, const float* sh, int degree, const sf_camera& cam,
                            const sf_settings& st, const float* gxy, const float* grec,
                            float* g_mean, float* g_quat, float* g_scale, float* g_opacity,
                            float* g_sh) {
  Projection p;
  project(mean, quat, scale, cam, st.eps2d, st.near_plane, st.extent, p);
  float g_mc[3] = {0.f, 0.f, 0.f};
  float gCc[9];
  for (int k = 0; k < 9; ++k) gCc[k] = 0.f;
  float gR[9];
  for (int k = 0; k < 9; ++k) gR[k] = 0.f;
  // conic -> filtered covariance (inverse adjoint with symmetric G)
  float ga = grec[R_QA], h = 0.5f * grec[R_QB], gc = grec[R_QC];
  float QG00 = p.qa * ga + p.qb * h, QG01 = p.qa * h + p.qb * gc;
  float QG10 = p.qb * ga + p.qc * h, QG11 = p.qb * h + p.qc * gc;
  float g_s00 = -(QG00 * p.qa + QG01 * p.qb);
  float g_s01 = -(QG00 * p.qb + QG01 * p.qc) - (QG10 * p.qa + QG11 * p.qb);
  float g_s11 = -(QG10 * p.qb + QG11 * p.qc);
  // opacity (optionally antialiased)
  float gop = grec[R_OPA];
  if (st.antialiased) {
    float detS = p.s00 * p.s11 - p.s01 * p.s01;
    float detF = p.fa * p.fc - p.fb * p.fb;
    float a = fmaxr(detS, 0.f), b = fmaxr(detF, 1e-12f);
    float ratio = a / b, f = sqrtf(ratio);
    *g_opacity = gop * f;
    float gf = gop * opacity;
    if (ratio > 0.f) {
      float gr = gf * 0.5f / f;
      float gA = detS >= 0.f ? gr / b : 0.f;
      float gB = detF >= 1e-12f ? -gr * a / (b * b) : 0.f;
      g_s00 += gA * p.s11 + gB * p.fc;
      g_s11 += gA * p.s00 + gB * p.fa;
      g_s01 += -2.f * p.s01 * gA - 2.f * p.fb * gB;
    }
  } else {
    *g_opacity = gop;
  }
  // screen = J Cc J^T
  float Gs[4] = {g_s00, 0.5f * g_s01, 0.5f * g_s01, g_s11};
  float J[6] = {p.j00, 0.f, p.j02, 0.f, p.j11, p.j12};
  const float* Cc = p.Cc;
  float M[6];
  for (int r = 0; r < 2; ++r)
    for (int k = 0; k < 3; ++k)
      M[r * 3 + k] = J[r * 3 + 0] * Cc[0 * 3 + k] + J[r * 3 + 1] * Cc[1 * 3 + k] + J[r * 3 + 2] * Cc[2 * 3 + k];
  float gJ[6];
  for (int r = 0; r < 2; ++r)
    for (int k = 0; k < 3; ++k) gJ[r * 3 + k] = 2.f * (Gs[r * 2 + 0] * M[0 * 3 + k] + Gs[r * 2 + 1] * M[1 * 3 + k]);
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) {
      float acc = 0.f;
      for (int r = 0; r < 2; ++r)
        for (int s2 = 0; s2 < 2; ++s2) acc += J[r * 3 + i] * Gs[r * 2 + s2] * J[s2 * 3 + j];
      gCc[i * 3 + j] += acc;
    }
  // mode extras
  if (MODE == SF_MODE_RADEGS) {
    RadeExtras e;
    rade_extras(p, e);
    float g_rad = grec[R_RADIAL];
    if (e.radial > 0.f)
      for (int k = 0; k < 3; ++k) g_mc[k] += g_rad * p.mc[k] / e.radial;
    float gv[3];
    unit3_backward(e.v, grec + R_NRM, gv);
    float rn[3] = {e.gain[0], e.gain[1], -1.f};
    float gF[9];
    for (int i = 0; i < 3; ++i)
      for (int j = 0; j < 3; ++j) gF[i * 3 + j] = rn[i] * gv[j];
    float grn[3];
    for (int i = 0; i < 3; ++i) grn[i] = e.F[i * 3 + 0] * gv[0] + e.F[i * 3 + 1] * gv[1] + e.F[i * 3 + 2] * gv[2];
    float gg0 = grec[R_GAIN] + grn[0], gg1 = grec[R_GAIN + 1] + grn[1];
    float gb0 = gg0 * e.Ainv[0] + gg1 * e.Ainv[1];
    float gb1 = gg0 * e.Ainv[2] + gg1 * e.Ainv[3];
    float GT[9] = {-e.gain[0] * gb0, -e.gain[0] * gb1, 0.f,
                   -e.gain[1] * gb0, -e.gain[1] * gb1, 0.f,
                   gb0, gb1, 0.f};
    // Tm = F Cc F^T: gF += (GT + GT^T) F Cc ; gCc += F^T GT F
    float FC[9];
    for (int i = 0; i < 3; ++i)
      for (int j = 0; j < 3; ++j)
        FC[i * 3 + j] = e.F[i * 3 + 0] * Cc[0 * 3 + j] + e.F[i * 3 + 1] * Cc[1 * 3 + j] + e.F[i * 3 + 2] * Cc[2 * 3 + j];
    for (int i = 0; i < 3; ++i)
      for (int j = 0; j < 3; ++j) {
        float acc = 0.f;
        for (int k = 0; k < 3; ++k) acc += (GT[i * 3 + k] + GT[k * 3 + i]) * FC[k * 3 + j];
        gF[i * 3 + j] += acc;
      }
    for (int i = 0; i < 3; ++i)
      for (int j = 0; j < 3; ++j) {
        float acc = 0.f;
        for (int a = 0; a < 3; ++a)
          for (int b = 0; b < 3; ++b) acc += e.F[a * 3 + i] * GT[a * 3 + b] * e.F[b * 3 + j];
        gCc[i * 3 + j] += acc;
      }
    gJ[0] += gF[0]; gJ[2] += gF[2]; gJ[4] += gF[4]; gJ[5] += gF[5];
    float gmh[3] = {gF[6], gF[7], gF[8]}, gm[3];
    unit3_backward(p.mc, gmh, gm);
    for (int k = 0; k < 3; ++k) g_mc[k] += gm[k];
  } else if (MODE == SF_MODE_GOF) {
    float Q[6];
    inv3_sym(p.Cc, Q);
    float Qf[9] = {Q[0], Q[1], Q[2], Q[1], Q[3], Q[4], Q[2], Q[4], Q[5]};
    const float* gq = grec + R_Q3;
    float G[9] = {gq[0], 0.5f * gq[1], 0.5f * gq[2], 0.5f * gq[1], gq[3], 0.5f * gq[4],
                  0.5f * gq[2], 0.5f * gq[4], gq[5]};
    float QG[9];
    for (int i = 0; i < 3; ++i)
      for (int j = 0; j < 3; ++j) QG[i * 3 + j] = Qf[i * 3 + 0] * G[0 * 3 + j] + Qf[i * 3 + 1] * G[1 * 3 + j] + Qf[i * 3 + 2] * G[2 * 3 + j];
    for (int i = 0; i < 3; ++i)
      for (int j = 0; j < 3; ++j)
        gCc[i * 3 + j] -= QG[i * 3 + 0] * Qf[0 * 3 + j] + QG[i * 3 + 1] * Qf[1 * 3 + j] + QG[i * 3 + 2] * Qf[2 * 3 + j];
    g_mc[2] += grec[R_Z];
  } else {
    AmbiExtras e;
    ambi_extras(scale, p, cam, e);
    float gpl = grec[R_PLANE];
    float gn[3];
    for (int k = 0; k < 3; ++k) {
      gn[k] = grec[R_ANRM + k] + gpl * p.mc[k];
      g_mc[k] += gpl * e.normal[k];
    }
    const int a = e.axis;
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const float gw = e.sign * (cam.R[0 * 3 + j] * gn[0] + cam.R[1 * 3 + j] * gn[1] + cam.R[2 * 3 + j] * gn[2]);
#pragma unroll
      for (int c = 0; c < 3; ++c)
        if (c == a) gR[j * 3 + c] += gw;  // constant indices (keeps gR in registers)
    }
  }
  // J and the projected mean -> guarded (x, y, z)
  if (p.active) {
    float fx = cam.K[0], fy = cam.K[4];
    float zs = p.zs, z2 = zs * zs, z3 = z2 * zs;
    float gX = gxy[0], gY = gxy[1];
    float gzs = -gJ[0] * fx / z2 - gJ[4] * fy / z2 + gJ[2] * 2.f * fx * p.xg / z3 +
                gJ[5] * 2.f * fy * p.yg / z3 - gX * fx * p.xg / z2 - gY * fy * p.yg / z2;
    float gx = -gJ[2] * fx / z2 + gX * fx / zs;
    float gy = -gJ[5] * fy / z2 + gY * fy / zs;
    g_mc[0] += gx; g_mc[1] += gy; g_mc[2] += gzs;
  }
  // camera transform
  const float* W = cam.R;
  for (int j = 0; j < 3; ++j) g_mean[j] = W[0 * 3 + j] * g_mc[0] + W[1 * 3 + j] * g_mc[1] + W[2 * 3 + j] * g_mc[2];
  float gC[9], tmp[9];
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) tmp[i * 3 + j] = W[0 * 3 + i] * gCc[0 * 3 + j] + W[1 * 3 + i] * gCc[1 * 3 + j] + W[2 * 3 + i] * gCc[2 * 3 + j];
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) gC[i * 3 + j] = tmp[i * 3 + 0] * W[0 * 3 + j] + tmp[i * 3 + 1] * W[1 * 3 + j] + tmp[i * 3 + 2] * W[2 * 3 + j];
  // covariance -> rotation, scale -> quaternion
  float gRc[9], gs[3];
  covariance3_backward(p.R, scale, gC, gRc, gs);
  for (int k = 0; k < 9; ++k) gR[k] += gRc[k];
  float gqn[4];
  quat_rotation_backward(p.qn, gR, gqn);
  float qraw[4] = {quat[0], quat[1], quat[2], quat[3]};
  quat_normalize_backward(qraw, p.qnorm, gqn, g_quat);
  for (int k = 0; k < 3; ++k) g_scale[k] = gs[k];
  // SH colour (live) and AmbiSuR ray colour (detached direction)
  float dir[3] = {mean[0] - cam.origin[0], mean[1] - cam.origin[1], mean[2] - cam.origin[2]};
  float gdir[3];
  sh_color_backward(sh, degree, dir, grec + R_RGB, MODE == SF_MODE_AMBISUR ? grec + G_RAYC : nullptr,
                    g_sh, gdir);
  for (int k = 0; k < 3; ++k) g_mean[k] += gdir[k];
}

SF_HD void project_backward(const float* mean, const float* quat, const float* scale, float opacity,
                            const float* sh, int degree, const sf_camera& cam, const sf_settings& st,
                            const float* gxy, const float* grec, float* g_mean, float* g_quat, float* g_scale,
                            float* g_opacity, float* g_sh) {
  if (st.mode == SF_MODE_RADEGS)
    project_backward_mode<SF_MODE_RADEGS>(mean, quat, scale, opacity, sh, degree, cam, st, gxy, grec, g_mean,
                                          g_quat, g_scale, g_opacity, g_sh);
  else if (st.mode == SF_MODE_GOF)
    project_backward_mode<SF_MODE_GOF>(mean, quat, scale, opacity, sh, degree, cam, st, gxy, grec, g_mean, g_quat,
                                       g_scale, g_opacity, g_sh);
  else
    project_backward_mode<SF_MODE_AMBISUR>(mean, quat, scale, opacity, sh, degree, cam, st, gxy, grec, g_mean,
                                           g_quat, g_scale, g_opacity, g_sh);
}

}  // namespace sf
