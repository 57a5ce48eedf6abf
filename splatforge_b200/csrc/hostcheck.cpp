// Host build of the rasterizer arithmetic (sf_math.cuh / sf_grad.cuh) for the CPU
// test-suite: the same per-Gaussian and per-sample functions the CUDA kernels call,
// driven by plain sequential loops.  It checks the hand-written reverse-mode
// arithmetic against autograd of the CPU oracle without a GPU.  It is a test
// library (libsf_b200_hostcheck.so), never loaded by the product path.
//
// Compiled with -ffp-contract=off so that the exact-sequence operations round like
// the oracle's separate tensor operations.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "sf_grad.cuh"

using namespace sf;

namespace {

void rect_bounds(int64_t i, float x, float y, float r, float z, const sf_camera& cam, const sf_settings& st,
                 int32_t* rect, int32_t* count, uint32_t* depth_key) {
  int rc[4] = {0, 0, 0, 0};
  int c = 0;
  if (std::isfinite(x) && std::isfinite(y) && std::isfinite(r) && std::isfinite(z))
    c = tile_rect(x, y, r, z, cam.width, cam.height, 16, st.near_plane, st.far_plane, rc);
  for (int k = 0; k < 4; ++k) rect[i * 4 + k] = rc[k];
  count[i] = c;
  uint32_t bits;
  std::memcpy(&bits, &z, 4);
  depth_key[i] = c > 0 ? bits : 0xffffffffu;
}

int64_t l1_index(int tile, int k, int tid, int cap) { return ((int64_t)tile * 256 + tid) * cap + k; }

}  // namespace

extern "C" {

int hc_project_forward(const float* means, const float* quats, const float* scales, const float* opacities,
                       const float* sh, const uint8_t* selected, int64_t n, const sf_camera* cam,
                       const sf_settings* st, float* means2d, float* radii, float* records, int32_t* rect,
                       int32_t* count, uint32_t* depth_key) {
  const int K = st->sh_coeffs;
  for (int64_t i = 0; i < n; ++i) {
    const float* m = means + i * 3;
    const float* q = quats + i * 4;
    const float* sc = scales + i * 3;
    Projection p;
    project(m, q, sc, *cam, st->eps2d, st->near_plane, st->extent, p);
    float opa = opacities[i];
    if (st->antialiased) {
      const float detS = p.s00 * p.s11 - p.s01 * p.s01;
      const float detF = p.fa * p.fc - p.fb * p.fb;
      opa = opa * std::sqrt(fmaxr(detS, 0.f) / fmaxr(detF, 1e-12f));
    }
    float* rec = records + i * SF_RECORD_FLOATS;
    for (int k = 0; k < SF_RECORD_FLOATS; ++k) rec[k] = 0.f;
    rec[R_X] = p.X; rec[R_Y] = p.Y;
    rec[R_QA] = p.qa; rec[R_QB] = p.qb; rec[R_QC] = p.qc;
    rec[R_OPA] = opa;
    const float dir[3] = {m[0] - cam->origin[0], m[1] - cam->origin[1], m[2] - cam->origin[2]};
    sh_color(sh + i * K * 3, st->sh_degree, dir, rec + R_RGB);
    rec[R_SEL] = selected && selected[i] ? 1.f : 0.f;
    rec[R_Z] = p.mc[2];
    if (st->mode == SF_MODE_RADEGS) {
      RadeExtras e;
      rade_extras(p, e);
      rec[R_RADIAL] = e.radial;
      rec[R_GAIN] = e.gain[0]; rec[R_GAIN + 1] = e.gain[1];
      for (int k = 0; k < 3; ++k) rec[R_NRM + k] = e.normal[k];
    } else if (st->mode == SF_MODE_GOF) {
      const float fx = cam->K[0], fy = cam->K[4], cx = cam->K[2], cy = cam->K[5];
      rec[R_PROXY] = (p.X - cx) * p.mc[2] / fx;
      rec[R_PROXY + 1] = (p.Y - cy) * p.mc[2] / fy;
      rec[R_PROXY + 2] = p.mc[2];
      inv3_sym(p.Cc, rec + R_Q3);
    } else {
      AmbiExtras e;
      ambi_extras(sc, p, *cam, e);
      for (int k = 0; k < 3; ++k) rec[R_ANRM + k] = e.normal[k];
      rec[R_PLANE] = e.plane;
    }
    means2d[i * 2] = p.X;
    means2d[i * 2 + 1] = p.Y;
    radii[i] = p.radius;
    rect_bounds(i, p.X, p.Y, p.radius, p.mc[2], *cam, *st, rect, count, depth_key);
  }
  return 0;
}

int hc_project_backward(const float* means, const float* quats, const float* scales, const float* opacities,
                        const float* sh, int64_t n, const sf_camera* cam, const sf_settings* st,
                        const float* gxy, const float* grec, float* g_means, float* g_quats, float* g_scales,
                        float* g_opacities, float* g_sh) {
  const int K = st->sh_coeffs;
  const int used = sh_count(st->sh_degree) * 3;
  for (int64_t i = 0; i < n; ++i) {
    float gsh[48];
    project_backward(means + i * 3, quats + i * 4, scales + i * 3, opacities[i], sh + i * K * 3, st->sh_degree,
                     *cam, *st, gxy + i * 2, grec + i * SF_RECORD_FLOATS, g_means + i * 3, g_quats + i * 4,
                     g_scales + i * 3, g_opacities + i, gsh);
    for (int k = 0; k < K * 3; ++k) g_sh[i * K * 3 + k] = k < used ? gsh[k] : 0.f;
  }
  return 0;
}

// Sequential emulation of raster_forward_kernel (+ l1_resolve) with the fixed-capacity
// L1 layout.  ranges are [n_tiles, 2].
int hc_raster_forward(const float* records, const int32_t* ids, const int32_t* ranges, const sf_camera* cam,
                      const sf_settings* st, float* rgb, float* alpha, float* depth, float* normals, float* l1,
                      float* l2, float* median, float* ray_color, float* amb, float* state, float* l1s,
                      int64_t slots, int32_t cap) {
  const int W = cam->width, H = cam->height;
  const int tx = (W + 15) / 16, ty = (H + 15) / 16;
  const int mode = st->mode, dist = st->distortions;
  for (int tile = 0; tile < tx * ty; ++tile) {
    const int r0 = ranges[tile * 2], r1 = ranges[tile * 2 + 1];
    for (int tid = 0; tid < 256; ++tid) {
      const int u = (tile % tx) * 16 + (tid & 15), v = (tile / tx) * 16 + (tid >> 4);
      if (u >= W || v >= H) continue;
      const int64_t pix = (int64_t)v * W + u;
      PixelRay pr;
      pixel_ray(*cam, u, v, pr);
      double Td = 1.0, Wd = 0.0;
      float C[3] = {0, 0, 0}, D = 0, N[3] = {0, 0, 0}, Dn = 0, A = 0, Scc = 0, med_depth = 0;
      double L2d1 = 0.0, L2d2 = 0.0;
      int last = r0, med = -1, cnt = 0;
      for (int pos = r0; pos < r1; ++pos) {
        const float* rec = records + (int64_t)ids[pos] * SF_RECORD_FLOATS;
        Sample s;
        bool ok;
        if (mode == SF_MODE_GOF) ok = eval_sample<SF_MODE_GOF>(rec, pr, st->extent_sq, st->near_plane, st->far_plane, s);
        else if (mode == SF_MODE_RADEGS) ok = eval_sample<SF_MODE_RADEGS>(rec, pr, st->extent_sq, st->near_plane, st->far_plane, s);
        else ok = eval_sample<SF_MODE_AMBISUR>(rec, pr, st->extent_sq, st->near_plane, st->far_plane, s);
        if (!ok) continue;
        const float w = s.alpha * (float)Td;
        const float* c = rec + R_RGB;
        for (int k = 0; k < 3; ++k) { C[k] += w * c[k]; N[k] += w * s.n[k]; }
        D += w * s.depth;
        if (dist & SF_DIST_L2) {
          const double wd = (double)w * (double)s.depth;
          L2d1 += wd;
          L2d2 += wd * (double)s.depth;
        }
        A += w * rec[R_SEL];
        if (mode == SF_MODE_AMBISUR) { Dn += w * rec[R_PLANE]; Scc += w * (c[0] * c[0] + c[1] * c[1] + c[2] * c[2]); }
        Wd += (double)w;
        if (med < 0 && (float)Wd >= 0.5f) { med = pos; med_depth = s.depth; }
        if ((dist & SF_DIST_L1) && cnt < cap) {
          const int64_t idx = l1_index(tile, cnt, tid, cap);
          l1s[idx] = s.depth;
          l1s[slots + idx] = w;
        }
        ++cnt;
        last = pos + 1;
        Td *= (double)(1.f - s.alpha);
        if (Td < (double)st->t_stop) break;
      }
      const float Wf = (float)Wd;
      for (int k = 0; k < 3; ++k) rgb[pix * 3 + k] = C[k] + (1.f - Wf) * st->background[k];
      alpha[pix] = Wf;
      float expected = D / fmaxr(Wf, 1e-8f);
      if (mode == SF_MODE_AMBISUR) {
        const float den = N[0] * pr.r[0] + N[1] * pr.r[1] + N[2] * pr.r[2];
        expected = std::fabs(den) > 1e-8f ? Dn / den : 0.f;
      }
      depth[pix] = Wf > 1e-8f ? expected : 0.f;
      const float nn = fmaxr(std::sqrt(N[0] * N[0] + N[1] * N[1] + N[2] * N[2]), 1e-12f);
      for (int k = 0; k < 3; ++k) normals[pix * 3 + k] = N[k] / nn;
      const float raw_l2 = (dist & SF_DIST_L2) ? (float)(2.0 * (Wd * L2d2 - L2d1 * L2d1)) : 0.f;
      l2[pix] = fmaxr(raw_l2, 0.f);
      median[pix] = med >= 0 ? med_depth : 0.f;
      const float CC = C[0] * C[0] + C[1] * C[1] + C[2] * C[2];
      ray_color[pix] = mode == SF_MODE_AMBISUR ? Scc - 2.f * CC + CC * Wf : 0.f;
      amb[pix] = A;
      float* stt = state + pix * SF_PIXEL_STATE_FLOATS;
      stt[PS_T] = (float)Td; stt[PS_W] = Wf; stt[PS_D] = D; stt[PS_D2] = (float)L2d2;
      for (int k = 0; k < 3; ++k) { stt[PS_C + k] = C[k]; stt[PS_N + k] = N[k]; }
      stt[PS_DNUM] = Dn; stt[PS_L2] = raw_l2; stt[PS_LAST] = i2f(last); stt[PS_MEDIAN] = i2f(med);
      stt[PS_COUNT] = i2f(cnt);
      // L1 resolve (sorted by depth, then compositing index)
      float raw = 0.f;
      if (dist & SF_DIST_L1) {
        const int n = std::min(cnt, (int)cap);
        std::vector<int> order(n);
        for (int k = 0; k < n; ++k) order[k] = k;
        auto dk = [&](int k) { return l1s[l1_index(tile, k, tid, cap)]; };
        auto wk = [&](int k) { return l1s[slots + l1_index(tile, k, tid, cap)]; };
        std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return dk(a) < dk(b); });
        float Wt = 0, Dt = 0;
        for (int k = 0; k < n; ++k) { Wt += wk(k); Dt += wk(k) * dk(k); }
        float pw = 0, pwd = 0;
        std::vector<float> aw(n), ad(n);
        for (int r = 0; r < n; ++r) {
          const int k = order[r];
          const float d = dk(k), w = wk(k);
          raw += 2.f * w * (d * pw - pwd);
          aw[k] = 2.f * (2.f * d * pw - d * Wt + Dt - 2.f * pwd);
          ad[k] = 2.f * w * (2.f * pw + w - Wt);
          pw += w; pwd += w * d;
        }
        for (int k = 0; k < n; ++k) {
          const int64_t idx = l1_index(tile, k, tid, cap);
          l1s[idx] = aw[k];
          l1s[slots + idx] = ad[k];
        }
      }
      stt[PS_L1] = raw;
      l1[pix] = fmaxr(raw, 0.f);
    }
  }
  return 0;
}

// Sequential emulation of raster_backward_kernel + raster_finalize_kernel.
int hc_raster_backward(const float* records, int64_t n, const int32_t* ids, const int32_t* ranges,
                       const sf_camera* cam, const sf_settings* st, const float* state, const float* l1s,
                       int64_t slots, int32_t cap, const float* g_rgb, const float* g_alpha, const float* g_depth,
                       const float* g_normals, const float* g_l1, const float* g_l2, const float* g_median,
                       const float* g_var, const float* g_amb, float* grad_records, float* grad_means2d,
                       float* absgrad) {
  const int W = cam->width, H = cam->height;
  const int tx = (W + 15) / 16, ty = (H + 15) / 16;
  const int mode = st->mode, dist = st->distortions;
  const float fx = cam->K[0], fy = cam->K[4];
  for (int tile = 0; tile < tx * ty; ++tile) {
    const int r0 = ranges[tile * 2];
    for (int tid = 0; tid < 256; ++tid) {
      const int u = (tile % tx) * 16 + (tid & 15), v = (tile / tx) * 16 + (tid >> 4);
      if (u >= W || v >= H) continue;
      const int64_t pix = (int64_t)v * W + u;
      PixelRay pr;
      pixel_ray(*cam, u, v, pr);
      const float* stt = state + pix * SF_PIXEL_STATE_FLOATS;
      PixelUpstream up;
      for (int c = 0; c < 3; ++c) {
        up.rgb[c] = g_rgb ? g_rgb[pix * 3 + c] : 0.f;
        up.normal[c] = g_normals ? g_normals[pix * 3 + c] : 0.f;
      }
      up.alpha = g_alpha ? g_alpha[pix] : 0.f;
      up.depth = g_depth ? g_depth[pix] : 0.f;
      up.l1 = g_l1 ? g_l1[pix] : 0.f;
      up.l2 = g_l2 ? g_l2[pix] : 0.f;
      up.median = g_median ? g_median[pix] : 0.f;
      up.var = g_var ? g_var[pix] : 0.f;
      up.amb = g_amb ? g_amb[pix] : 0.f;
      PixelGrads pg;
      pixel_grads(mode, dist, stt, pr, st->background, up, pg);
      float T = stt[PS_T], S = 0.f;
      const int last = f2i(stt[PS_LAST]);
      int k = std::min(f2i(stt[PS_COUNT]), (int)cap) - 1;
      for (int pos = last - 1; pos >= r0; --pos) {
        const float* rec = records + (int64_t)ids[pos] * SF_RECORD_FLOATS;
        Sample s;
        bool contrib;
        float auxw = 0.f, auxd = 0.f;
        if (mode == SF_MODE_GOF) {
          contrib = eval_sample<SF_MODE_GOF>(rec, pr, st->extent_sq, st->near_plane, st->far_plane, s);
        } else if (mode == SF_MODE_RADEGS) {
          contrib = eval_sample<SF_MODE_RADEGS>(rec, pr, st->extent_sq, st->near_plane, st->far_plane, s);
        } else {
          contrib = eval_sample<SF_MODE_AMBISUR>(rec, pr, st->extent_sq, st->near_plane, st->far_plane, s);
        }
        if ((dist & SF_DIST_L1) && contrib) {
          if (k >= 0) {
            const int64_t idx = l1_index(tile, k, tid, cap);
            auxw = l1s[idx];
            auxd = l1s[slots + idx];
          }
          --k;
        }
        if (!contrib || !(s.alpha > 0.f)) continue;
        const float al = s.alpha, om = 1.f - al;
        const float Ti = T * (1.f / om), w = al * Ti;
        float adj;
        if (mode == SF_MODE_GOF) adj = sample_adj<SF_MODE_GOF>(rec, s, pg, auxw);
        else if (mode == SF_MODE_RADEGS) adj = sample_adj<SF_MODE_RADEGS>(rec, s, pg, auxw);
        else adj = sample_adj<SF_MODE_AMBISUR>(rec, s, pg, auxw);
        const float g_alpha_s = Ti * adj - S * (1.f / om);
        S += w * adj;
        T = Ti;
        float g_d = w * pg.gD + (pos == pg.med_pos ? pg.gMed : 0.f) + pg.gL1 * auxd;
        if (dist & SF_DIST_L2) g_d += pg.gL2 * 4.f * w * (pg.W * s.depth - pg.D);
        float vals[18];
        int nv;
        float* g = grad_records + (int64_t)ids[pos] * SF_RECORD_FLOATS;
        float* ab = absgrad + (int64_t)ids[pos] * 2;
        if (mode == SF_MODE_GOF) {
          sample_backward<SF_MODE_GOF>(rec, pr, s, pg, w, g_alpha_s, g_d, 1.f / fx, 1.f / fy, vals);
          nv = SampleLayout<SF_MODE_GOF>::NV;
          for (int q = 0; q < nv; ++q) { int sl = SampleLayout<SF_MODE_GOF>::slot(q); if (sl < 20) g[sl] += vals[q]; else ab[sl - 20] += vals[q]; }
        } else if (mode == SF_MODE_RADEGS) {
          sample_backward<SF_MODE_RADEGS>(rec, pr, s, pg, w, g_alpha_s, g_d, 1.f / fx, 1.f / fy, vals);
          nv = SampleLayout<SF_MODE_RADEGS>::NV;
          for (int q = 0; q < nv; ++q) { int sl = SampleLayout<SF_MODE_RADEGS>::slot(q); if (sl < 20) g[sl] += vals[q]; else ab[sl - 20] += vals[q]; }
        } else {
          sample_backward<SF_MODE_AMBISUR>(rec, pr, s, pg, w, g_alpha_s, g_d, 1.f / fx, 1.f / fy, vals);
          nv = SampleLayout<SF_MODE_AMBISUR>::NV;
          for (int q = 0; q < nv; ++q) { int sl = SampleLayout<SF_MODE_AMBISUR>::slot(q); if (sl < 20) g[sl] += vals[q]; else ab[sl - 20] += vals[q]; }
        }
      }
    }
  }
  // finalize
  for (int64_t i = 0; i < n; ++i) {
    float* g = grad_records + i * SF_RECORD_FLOATS;
    const float* r = records + i * SF_RECORD_FLOATS;
    if (mode == SF_MODE_GOF) {
      const float cx = cam->K[2], cy = cam->K[5];
      const float z = r[R_Z];
      const float gp0 = g[R_PROXY], gp1 = g[R_PROXY + 1], gp2 = g[R_PROXY + 2];
      grad_means2d[i * 2] = gp0 * z / fx;
      grad_means2d[i * 2 + 1] = gp1 * z / fy;
      g[R_Z] = gp0 * (r[R_X] - cx) / fx + gp1 * (r[R_Y] - cy) / fy + gp2;
    } else {
      grad_means2d[i * 2] = g[R_X];
      grad_means2d[i * 2 + 1] = g[R_Y];
    }
  }
  return 0;
}

// box_may_pass over n Gaussians (5 floats each: qa qb qc X Y) and one box
void hc_box_may_pass(const float* g, int64_t n, float x0, float x1, float y0, float y1, float ext2,
                     uint8_t* out) {
  for (int64_t i = 0; i < n; ++i)
    out[i] = sf::box_may_pass(g[i * 5], g[i * 5 + 1], g[i * 5 + 2], g[i * 5 + 3], g[i * 5 + 4], x0, x1, y0, y1,
                              ext2);
}

}  // extern "C"
