// Host-side launchers of the kernels (C++), called by the C ABI layer in capi.cu.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/splatforge_b200.h"

namespace sf {

// kernels launched by this library (sf_b200_kernel_launches)
void count_launches(int k);
int64_t launches_total();
// message returned by sf_b200_last_error() on this thread
void set_last_error(const char* msg);

struct RasterFwdArgs {
  const float* records;
  const int32_t* ids;
  const int2* ranges;
  sf_camera cam;
  sf_settings st;
  int tiles_x;
  float* rgb; float* alpha; float* depth; float* normals; float* l1; float* l2;
  float* median; float* ray_color; float* amb;
  float* state;
  float* l1s; int64_t l1_slots; const int64_t* l1_off; int l1_cap; int32_t* l1_needed;
  unsigned long long* counters;
};

struct RasterBwdArgs {
  const float* records;
  const int32_t* ids;
  const int2* ranges;
  sf_camera cam;
  sf_settings st;
  int tiles_x;
  const float* state;
  const float* l1s; int64_t l1_slots; const int64_t* l1_off; int l1_cap;
  const float* g_rgb; const float* g_alpha; const float* g_depth; const float* g_normals;
  const float* g_l1; const float* g_l2; const float* g_median; const float* g_var;
  const float* g_amb;
  float* grad_records;
  float* absgrad;
  int32_t* error_word;
};

cudaError_t launch_raster_forward(const RasterFwdArgs& a, int n_tiles, cudaStream_t s);
cudaError_t launch_l1_resolve(const sf_camera& cam, const sf_settings& st, float* state,
                              float* l1s, int64_t l1_slots, const int64_t* l1_off, int l1_cap,
                              int max_samples, float* out_l1, cudaStream_t s);
size_t l1_resolve_smem_per_warp(int smem_k);
cudaError_t launch_raster_backward(const RasterBwdArgs& a, int n_tiles, cudaStream_t s);
cudaError_t launch_raster_finalize(const float* records, int64_t n, const sf_camera& cam,
                                   int mode, float* grad_records, float* grad_means2d,
                                   cudaStream_t s);
cudaError_t launch_pixel_counts(const float* state, int64_t npix, int32_t* counts,
                                cudaStream_t s);

cudaError_t launch_project_forward(const float* means, const float* quats, const float* scales,
                                   const float* opacities, const float* sh,
                                   const uint8_t* selected, int64_t n, const sf_camera& cam,
                                   const sf_settings& st, float* means2d, float* radii,
                                   float* records, int32_t* rect, int32_t* count,
                                   uint32_t* depth_key, int32_t* nonfinite, cudaStream_t s);
cudaError_t launch_project_backward(const float* means, const float* quats, const float* scales,
                                    const float* opacities, const float* sh, int64_t n,
                                    const sf_camera& cam, const sf_settings& st,
                                    const float* gxy, const float* grec, float* g_means,
                                    float* g_quats, float* g_scales, float* g_opacities,
                                    float* g_sh, cudaStream_t s);
cudaError_t launch_covariance_forward(const float* q, const float* s_, int64_t n, float* cov,
                                      cudaStream_t s);
cudaError_t launch_covariance_backward(const float* q, const float* s_, int64_t n,
                                       const float* gcov, float* gq, float* gs, cudaStream_t s);
cudaError_t launch_sh_forward(const float* coeffs, int K, const float* dirs, int64_t n,
                              int degree, float* rgb, cudaStream_t s);
cudaError_t launch_sh_backward(const float* coeffs, int K, const float* dirs, int64_t n,
                               int degree, const float* grgb, float* gcoeffs, float* gdirs,
                               cudaStream_t s);

// splat.alpha_composite@3 over dense [B, N, P]
size_t composite_l1_smem_per_warp(int n);
cudaError_t launch_composite_forward(const float* al, const float* col, const float* dep, const float* nrm, int B,
                                     int N, int P, int dist, float* rgb, float* alpha, float* znum, float* nnum,
                                     float* l1, float* l2, float* median, float* w, float* aux, float* raw,
                                     cudaStream_t s);
cudaError_t launch_composite_backward(const float* al, const float* col, const float* dep, const float* nrm, int B,
                                      int N, int P, int dist, const float* w, const float* aux, const float* raw,
                                      const float* g_rgb, const float* g_alpha, const float* g_znum,
                                      const float* g_nnum, const float* g_l1, const float* g_l2,
                                      const float* g_median, const float* g_w, float* da, float* dc, float* dd,
                                      float* dn, cudaStream_t s);

// camera.pixel_rays@1, gaussian.ray_peak@1, geometry.depth_normals@1
cudaError_t launch_pixel_rays(const float* K, int W, int H, float* out, cudaStream_t s);
cudaError_t launch_ray_peak(const float* means, const float* Q, int64_t N, const float* origins, const float* dirs,
                            int64_t P, float* t, float* r, float* n, cudaStream_t s);
cudaError_t launch_depth_normals(const float* depth, const float* K, int W, int H, float* normals, uint8_t* valid,
                                 cudaStream_t s);
// ws: 6 * W * H floats
cudaError_t launch_depth_normals_backward(const float* depth, const float* K, int W, int H, const float* g_normals,
                                          float* g_depth, float* ws, cudaStream_t s);
// gaussian.opacity_field@1, culled per view (cube-map candidate lists; contributions
// below `cutoff` dropped).  Synchronises the stream once per view; pairs_needed (host)
// receives the largest per-view candidate-pair count (views above max_pairs are skipped)
size_t field_culled_workspace_bytes(int64_t ng, int64_t max_pairs, int F);
size_t field_culled_query_bytes(int64_t np, int F);
cudaError_t launch_opacity_field_culled(const float* pts, int64_t np, const float* means, const float* invcov,
                                        const float* op, int64_t ng, const float* origins, int nc, float cutoff,
                                        int F, float* out, void* ws, size_t ws_bytes, int64_t max_pairs,
                                        int64_t* pairs_needed, cudaStream_t s,
                                        unsigned long long* pair_counter = nullptr, float* query_ms = nullptr);
// gaussian.opacity_field@1
size_t field_workspace_bytes(int64_t n);
cudaError_t launch_opacity_field(const float* pts, int64_t np, const float* means, const float* invcov,
                                 const float* op, int64_t ng, const float* origins, int nc, float* out, void* ws,
                                 cudaStream_t s);

// opacity field plan: every view's candidate lists built once, queries of all views
// evaluated per call
size_t field_plan_bytes(int64_t ng, int nc, int F, int64_t total_pairs, int64_t max_view_pairs);
size_t field_plan_query_bytes(int64_t np, int nc, int F);
cudaError_t field_plan_build(const float* means, const float* invcov, const float* op, int64_t ng,
                             const float* origins, int nc, float cutoff, int F, void* plan, size_t plan_bytes,
                             int64_t total_pairs, int64_t max_view_pairs, int64_t* needed, cudaStream_t s);
cudaError_t field_plan_eval(const void* plan, int64_t ng, int nc, int F, int64_t total_pairs, int64_t max_view_pairs,
                            const float* origins, const float* pts, int64_t np, float* out, void* ws, size_t ws_bytes,
                            cudaStream_t s);

// binning / sorting
cudaError_t launch_bin_rects(const float* bounds, int64_t n, int width, int height, int tile,
                             float near_plane, float far_plane, int32_t* rect, int32_t* count,
                             uint32_t* depth_key, int32_t* nonfinite, cudaStream_t s);
size_t bin_workspace_bytes(int64_t n, int64_t n_isect, int n_tiles);
cudaError_t bin_order(const int32_t* count, const uint32_t* depth_key, int64_t n,
                      int32_t* order, int64_t* offsets, void* ws, size_t ws_bytes,
                      cudaStream_t s);
// overflow == nullptr: n_isect is the exact count; else it is the buffers' capacity and
// the count is read on the device (see binning.cu)
cudaError_t bin_emit(const int32_t* order, const int64_t* offsets, const int32_t* rect,
                     int64_t n, int64_t n_isect, int tiles_x, int n_tiles, int32_t* ids,
                     int32_t* ranges, void* ws, size_t ws_bytes, cudaStream_t s,
                     int32_t* overflow = nullptr);
cudaError_t bin_keys(const int32_t* ids, const int32_t* ranges, const uint32_t* depth_key,
                     int n_tiles, int64_t n_isect, uint64_t* keys, cudaStream_t s);
// stable sort of n (key, value) pairs by key bits [0, bits), in place (keys, vals)
size_t sort_pairs_workspace_bytes(int64_t n);
cudaError_t sort_pairs(uint32_t* keys, int32_t* vals, int64_t n, int bits, void* ws, size_t ws_bytes,
                       cudaStream_t s);
// [begin, end) of every key value in sorted keys; ranges is int2[n_keys], zero for absent keys
cudaError_t key_ranges(const uint32_t* keys, int64_t n, int64_t n_keys, int32_t* ranges, cudaStream_t s);
// exclusive scan int32 -> int64 of n values; out has n+1 entries (out[n] = total)
cudaError_t scan_counts(const int32_t* in, int64_t n, int64_t* out, void* ws, size_t ws_bytes,
                        cudaStream_t s);
size_t scan_workspace_bytes(int64_t n);

// GOF mesh extraction (meshing.cu)
cudaError_t launch_grid_points(const float* means, const float* quats, const float* scales, const int32_t* chosen,
                               int64_t n, double extent, double* points, double* radius, cudaStream_t s);
size_t mesh_count_workspace_bytes(int64_t n_cells);
cudaError_t mesh_count(const double* values, int64_t n_points, const int32_t* cells, int64_t n_cells, double level,
                       int greater, uint8_t* inside, int64_t* slot_off, int64_t* face_off, void* ws,
                       size_t ws_bytes, cudaStream_t s);
size_t mesh_edges_workspace_bytes(int64_t n_slots);
cudaError_t mesh_edges(const double* points, int64_t n_points, const int32_t* cells, int64_t n_cells,
                       const uint8_t* inside, const int64_t* slot_off, int64_t n_slots, int32_t* edge_uid,
                       int32_t* pairs, double* low, double* high, uint8_t* low_inside, int64_t* n_unique,
                       void* ws, size_t ws_bytes, cudaStream_t s);
cudaError_t mesh_midpoints(const double* low, const double* high, int64_t n_edges, double* mid, cudaStream_t s);
cudaError_t mesh_bisect(double* low, double* high, const uint8_t* low_inside, int64_t n_edges, const double* values,
                        double level, int greater, cudaStream_t s);
size_t mesh_faces_workspace_bytes(int64_t n_faces);
cudaError_t mesh_faces(const double* points, const int32_t* cells, int64_t n_cells, const uint8_t* inside,
                       const int64_t* slot_off, const int32_t* edge_uid, const double* low, const double* high,
                       int64_t n_edges, const int64_t* face_off, int64_t n_faces, double* vertices, int64_t* faces,
                       int64_t* n_kept, void* ws, size_t ws_bytes, cudaStream_t s);

// training-step operations (training.cu)
cudaError_t launch_patch_zncc(const float* a, const float* b, const float* m, int64_t rows, int S, float eps,
                              float* corr, uint8_t* valid, cudaStream_t s);
cudaError_t launch_patch_zncc_backward(const float* a, const float* b, const float* m, int64_t rows, int S, float eps,
                                       const float* g_corr, float* ga, float* gb, cudaStream_t s);
cudaError_t launch_densify_observe(const float* grad2d, const float* radii, int64_t n, float sx, float sy,
                                   float* gradient, float* observations, cudaStream_t s);
size_t normal_consistency_workspace_bytes(int W, int H);
cudaError_t normal_consistency(const float* depth, const float* K, int W, int H, const float* alpha,
                               const float* numer, const float* unit, const float* mask, float* loss, int64_t* count,
                               void* ws, cudaStream_t s);
cudaError_t normal_consistency_backward(const float* depth, const float* K, int W, int H, const float* alpha,
                                        const float* numer, const float* unit, const float* mask, const float* g_loss,
                                        const int64_t* count, float* g_depth, float* g_alpha, float* g_vec,
                                        float* g_normals, void* ws, cudaStream_t s);

// gaussian.sh_ambiguity@1 (training.cu), gaussian.ray_color_variance@1/@2 (composite.cu)
cudaError_t launch_sh_ambiguity(const float* coeffs, int64_t n, int K, float* out, cudaStream_t s);
cudaError_t launch_sh_ambiguity_backward(const float* coeffs, int64_t n, int K, const float* g, float* g_coeffs,
                                         cudaStream_t s);
cudaError_t launch_ray_color_variance(const float* w, const float* c, const float* comp, int64_t B, int64_t N,
                                      int64_t P, float* out, cudaStream_t s);
cudaError_t launch_ray_color_variance_backward(const float* w, const float* c, const float* comp, const float* g,
                                               int64_t B, int64_t N, int64_t P, float* g_c, cudaStream_t s);

}  // namespace sf
