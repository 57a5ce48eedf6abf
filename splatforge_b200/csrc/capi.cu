// The extern "C" boundary of libsf_b200.so: argument validation, error strings,
// launches on the caller's stream.  See include/splatforge_b200.h.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>

#include <atomic>

#include "sf_kernels.h"

namespace sf {
namespace {
std::atomic<int64_t> g_launches{0};
}
void count_launches(int k) { g_launches.fetch_add(k, std::memory_order_relaxed); }
int64_t launches_total() { return g_launches.load(std::memory_order_relaxed); }
}  // namespace sf

namespace {

thread_local char g_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_status(cudaError_t e, const char* where) {
  if (e == cudaSuccess) return SF_OK;
  if (e == cudaErrorInvalidValue)
    return fail(SF_ERR_ARGUMENT, "%s: invalid size or workspace (%s)", where, cudaGetErrorString(e));
  return fail(SF_ERR_CUDA, "%s: %s", where, cudaGetErrorString(e));
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

int check_settings(const sf_settings* st, const char* where) {
  if (!st) return fail(SF_ERR_ARGUMENT, "%s: settings is NULL", where);
  if (st->mode < SF_MODE_RADEGS || st->mode > SF_MODE_AMBISUR)
    return fail(SF_ERR_ARGUMENT, "%s: unsupported rendering mode %d", where, st->mode);
  if (st->distortions < 0 || st->distortions > 3)
    return fail(SF_ERR_ARGUMENT, "%s: distortions must be none/l1/l2/both", where);
  if (st->tile_size != 16) return fail(SF_ERR_ARGUMENT, "%s: tile_size must be 16", where);
  if (st->sh_degree < 0 || st->sh_degree > 3) return fail(SF_ERR_ARGUMENT, "%s: SH degree must be 0..3", where);
  if (st->sh_coeffs < (st->sh_degree + 1) * (st->sh_degree + 1) || st->sh_coeffs > 16)
    return fail(SF_ERR_ARGUMENT, "%s: sh coefficient count %d invalid for degree %d (at most 16)", where,
                st->sh_coeffs, st->sh_degree);
  if (!(st->extent > 0.f)) return fail(SF_ERR_ARGUMENT, "%s: extent must be positive", where);
  return SF_OK;
}

int check_camera(const sf_camera* c, const char* where) {
  if (!c) return fail(SF_ERR_ARGUMENT, "%s: camera is NULL", where);
  if (c->width <= 0 || c->height <= 0) return fail(SF_ERR_ARGUMENT, "%s: width/height must be positive", where);
  return SF_OK;
}

int tiles_of(const sf_camera* c, int* tx) {
  *tx = (c->width + 15) / 16;
  return *tx * ((c->height + 15) / 16);
}

}  // namespace

void sf::set_last_error(const char* msg) { snprintf(g_error, sizeof(g_error), "%s", msg); }

extern "C" {

const char* sf_b200_last_error(void) { return g_error; }
int sf_b200_abi_version(void) { return SF_B200_ABI_VERSION; }
int64_t sf_b200_kernel_launches(void) { return sf::launches_total(); }

int sf_b200_covariance_forward(const float* quats, const float* scales, int64_t n, float* cov, void* stream) {
  if (n < 0 || (n > 0 && (!quats || !scales || !cov))) return fail(SF_ERR_ARGUMENT, "covariance_forward: bad arguments");
  return cuda_status(sf::launch_covariance_forward(quats, scales, n, cov, as_stream(stream)), "covariance_forward");
}

int sf_b200_covariance_backward(const float* quats, const float* scales, int64_t n, const float* grad_cov,
                                float* grad_quats, float* grad_scales, void* stream) {
  if (n < 0 || (n > 0 && (!quats || !scales || !grad_cov))) return fail(SF_ERR_ARGUMENT, "covariance_backward: bad arguments");
  return cuda_status(sf::launch_covariance_backward(quats, scales, n, grad_cov, grad_quats, grad_scales, as_stream(stream)),
                     "covariance_backward");
}

int sf_b200_sh_color_forward(const float* coeffs, int32_t coeff_count, const float* dirs, int64_t n, int32_t degree,
                             float* rgb, void* stream) {
  if (degree < 0 || degree > 3) return fail(SF_ERR_ARGUMENT, "sh_color_forward: SH degree must be 0..3");
  if (coeff_count < (degree + 1) * (degree + 1) || coeff_count > 16)
    return fail(SF_ERR_ARGUMENT, "sh_color_forward: coefficient count %d invalid for degree %d", coeff_count, degree);
  if (n < 0 || (n > 0 && (!coeffs || !dirs || !rgb))) return fail(SF_ERR_ARGUMENT, "sh_color_forward: bad arguments");
  return cuda_status(sf::launch_sh_forward(coeffs, coeff_count, dirs, n, degree, rgb, as_stream(stream)), "sh_color_forward");
}

int sf_b200_sh_color_backward(const float* coeffs, int32_t coeff_count, const float* dirs, int64_t n, int32_t degree,
                              const float* grad_rgb, float* grad_coeffs, float* grad_dirs, void* stream) {
  if (degree < 0 || degree > 3) return fail(SF_ERR_ARGUMENT, "sh_color_backward: SH degree must be 0..3");
  if (coeff_count < (degree + 1) * (degree + 1) || coeff_count > 16)
    return fail(SF_ERR_ARGUMENT, "sh_color_backward: coefficient count %d invalid for degree %d", coeff_count, degree);
  if (n < 0 || (n > 0 && (!coeffs || !dirs || !grad_rgb))) return fail(SF_ERR_ARGUMENT, "sh_color_backward: bad arguments");
  return cuda_status(sf::launch_sh_backward(coeffs, coeff_count, dirs, n, degree, grad_rgb, grad_coeffs, grad_dirs,
                                            as_stream(stream)),
                     "sh_color_backward");
}

int sf_b200_project_forward(const float* means, const float* quats, const float* scales, const float* opacities,
                            const float* sh, const uint8_t* selected, int64_t n, const sf_camera* camera,
                            const sf_settings* settings, float* means2d, float* radii, float* records,
                            int32_t* tile_rect, int32_t* tile_count, uint32_t* depth_key, int32_t* nonfinite,
                            void* stream) {
  int rc;
  if ((rc = check_settings(settings, "project_forward")) || (rc = check_camera(camera, "project_forward"))) return rc;
  if (n < 0) return fail(SF_ERR_ARGUMENT, "project_forward: negative count");
  if (n > 0 && (!means || !quats || !scales || !opacities || !sh || !means2d || !radii || !records || !tile_rect ||
                !tile_count || !depth_key))
    return fail(SF_ERR_ARGUMENT, "project_forward: NULL buffer");
  if (!aligned(quats, 16) || !aligned(records, 16) || !aligned(tile_rect, 16) || !aligned(means2d, 8))
    return fail(SF_ERR_ARGUMENT, "project_forward: quats/records/tile_rect need 16-byte and means2d 8-byte alignment");
  return cuda_status(sf::launch_project_forward(means, quats, scales, opacities, sh, selected, n, *camera, *settings,
                                                means2d, radii, records, tile_rect, tile_count, depth_key, nonfinite,
                                                as_stream(stream)),
                     "project_forward");
}

int sf_b200_project_backward(const float* means, const float* quats, const float* scales, const float* opacities,
                             const float* sh, int64_t n, const sf_camera* camera, const sf_settings* settings,
                             const float* grad_means2d, const float* grad_records, float* grad_means, float* grad_quats,
                             float* grad_scales, float* grad_opacities, float* grad_sh, void* stream) {
  int rc;
  if ((rc = check_settings(settings, "project_backward")) || (rc = check_camera(camera, "project_backward"))) return rc;
  if (n < 0) return fail(SF_ERR_ARGUMENT, "project_backward: negative count");
  if (n > 0 && (!means || !quats || !scales || !opacities || !sh || !grad_means2d || !grad_records))
    return fail(SF_ERR_ARGUMENT, "project_backward: NULL buffer");
  if (!aligned(grad_records, 16) || !aligned(grad_quats, 16))
    return fail(SF_ERR_ARGUMENT, "project_backward: grad_records/grad_quats need 16-byte alignment");
  return cuda_status(sf::launch_project_backward(means, quats, scales, opacities, sh, n, *camera, *settings,
                                                 grad_means2d, grad_records, grad_means, grad_quats, grad_scales,
                                                 grad_opacities, grad_sh, as_stream(stream)),
                     "project_backward");
}

int sf_b200_bin_rects(const float* bounds, int64_t n, int32_t width, int32_t height, int32_t tile_size,
                      float near_plane, float far_plane, int32_t* tile_rect, int32_t* tile_count,
                      uint32_t* depth_key, int32_t* nonfinite, void* stream) {
  if (tile_size != 16) return fail(SF_ERR_ARGUMENT, "bin_rects: tile_size must be 16");
  if (width <= 0 || height <= 0 || n < 0) return fail(SF_ERR_ARGUMENT, "bin_rects: bad sizes");
  if (n > 0 && (!bounds || !tile_rect || !tile_count || !depth_key)) return fail(SF_ERR_ARGUMENT, "bin_rects: NULL buffer");
  if (!aligned(bounds, 16) || !aligned(tile_rect, 16)) return fail(SF_ERR_ARGUMENT, "bin_rects: 16-byte alignment needed");
  return cuda_status(sf::launch_bin_rects(bounds, n, width, height, tile_size, near_plane, far_plane, tile_rect,
                                          tile_count, depth_key, nonfinite, as_stream(stream)),
                     "bin_rects");
}

int sf_b200_bin_workspace_bytes(int64_t n, int64_t n_isect, int32_t n_tiles, size_t* bytes) {
  if (n < 0 || n_isect < 0 || n_tiles < 0 || !bytes) return fail(SF_ERR_ARGUMENT, "bin_workspace_bytes: bad arguments");
  if (n_isect > 0x7fffffffLL || n > 0x7fffffffLL)
    return fail(SF_ERR_CAPACITY, "bin_workspace_bytes: %lld intersections exceed the 32-bit list index",
                (long long)n_isect);
  *bytes = sf::bin_workspace_bytes(n, n_isect, n_tiles);
  return SF_OK;
}

int sf_b200_bin_order(const int32_t* tile_count, const uint32_t* depth_key, int64_t n, int32_t* order,
                      int64_t* offsets, void* workspace, size_t workspace_bytes, void* stream) {
  if (n < 0 || !offsets || (n > 0 && (!tile_count || !depth_key || !order || !workspace)))
    return fail(SF_ERR_ARGUMENT, "bin_order: bad arguments");
  if (workspace_bytes < sf::bin_workspace_bytes(n, 0, 0))
    return fail(SF_ERR_CAPACITY, "bin_order: workspace of %zu bytes, %zu needed", workspace_bytes,
                sf::bin_workspace_bytes(n, 0, 0));
  return cuda_status(sf::bin_order(tile_count, depth_key, n, order, offsets, workspace, workspace_bytes,
                                   as_stream(stream)),
                     "bin_order");
}

int sf_b200_bin_emit(const int32_t* order, const int64_t* offsets, const int32_t* tile_rect, int64_t n,
                     int64_t n_isect, int32_t tiles_x, int32_t n_tiles, int32_t* isect_ids, int32_t* tile_ranges,
                     void* workspace, size_t workspace_bytes, void* stream) {
  if (n < 0 || n_isect < 0 || n_tiles <= 0 || tiles_x <= 0 || !tile_ranges ||
      (n_isect > 0 && (!order || !offsets || !tile_rect || !isect_ids || !workspace)))
    return fail(SF_ERR_ARGUMENT, "bin_emit: bad arguments");
  if (n_isect > 0x7fffffffLL) return fail(SF_ERR_CAPACITY, "bin_emit: too many intersections for 32-bit lists");
  if (workspace_bytes < sf::bin_workspace_bytes(0, n_isect, n_tiles))
    return fail(SF_ERR_CAPACITY, "bin_emit: workspace of %zu bytes, %zu needed", workspace_bytes,
                sf::bin_workspace_bytes(0, n_isect, n_tiles));
  if (!aligned(tile_rect, 16) || !aligned(tile_ranges, 8)) return fail(SF_ERR_ARGUMENT, "bin_emit: alignment");
  return cuda_status(sf::bin_emit(order, offsets, tile_rect, n, n_isect, tiles_x, n_tiles, isect_ids, tile_ranges,
                                  workspace, workspace_bytes, as_stream(stream)),
                     "bin_emit");
}

int sf_b200_bin_emit_bounded(const int32_t* order, const int64_t* offsets, const int32_t* tile_rect, int64_t n,
                             int64_t capacity, int32_t tiles_x, int32_t n_tiles, int32_t* isect_ids,
                             int32_t* tile_ranges, void* workspace, size_t workspace_bytes, int32_t* overflow,
                             void* stream) {
  if (n < 0 || capacity <= 0 || n_tiles <= 0 || tiles_x <= 0 || !tile_ranges || !overflow || !order ||
      !offsets || !tile_rect || !isect_ids || !workspace)
    return fail(SF_ERR_ARGUMENT, "bin_emit_bounded: bad arguments");
  if (capacity > 0x7fffffffLL) return fail(SF_ERR_CAPACITY, "bin_emit_bounded: capacity above 32-bit lists");
  if (workspace_bytes < sf::bin_workspace_bytes(0, capacity, n_tiles))
    return fail(SF_ERR_CAPACITY, "bin_emit_bounded: workspace of %zu bytes, %zu needed", workspace_bytes,
                sf::bin_workspace_bytes(0, capacity, n_tiles));
  if (!aligned(tile_rect, 16) || !aligned(tile_ranges, 8)) return fail(SF_ERR_ARGUMENT, "bin_emit_bounded: alignment");
  return cuda_status(sf::bin_emit(order, offsets, tile_rect, n, capacity, tiles_x, n_tiles, isect_ids, tile_ranges,
                                  workspace, workspace_bytes, as_stream(stream), overflow),
                     "bin_emit_bounded");
}

int sf_b200_bin_keys(const int32_t* isect_ids, const int32_t* tile_ranges, const uint32_t* depth_key, int32_t n_tiles,
                     int64_t n_isect, uint64_t* keys, void* stream) {
  if (n_tiles < 0 || n_isect < 0 || (n_isect > 0 && (!isect_ids || !tile_ranges || !depth_key || !keys)))
    return fail(SF_ERR_ARGUMENT, "bin_keys: bad arguments");
  return cuda_status(sf::bin_keys(isect_ids, tile_ranges, depth_key, n_tiles, n_isect, keys, as_stream(stream)),
                     "bin_keys");
}

int sf_b200_raster_forward(const float* records, int64_t n, const int32_t* isect_ids, const int32_t* tile_ranges,
                           const sf_camera* camera, const sf_settings* settings, float* rgb, float* alpha,
                           float* depth, float* normals, float* distortion_l1, float* distortion_l2,
                           float* median_depth, float* ray_color, float* ambiguity, float* pixel_state,
                           float* l1_samples, int64_t l1_slots, const int64_t* l1_offsets, int32_t l1_cap,
                           int32_t* l1_needed, int64_t* counters, void* stream) {
  int rc;
  if ((rc = check_settings(settings, "raster_forward")) || (rc = check_camera(camera, "raster_forward"))) return rc;
  if (!tile_ranges || !rgb || !alpha || !depth || !normals || !distortion_l1 || !distortion_l2 || !median_depth ||
      !ray_color || !ambiguity || !pixel_state || n < 0 || (n > 0 && !records))
    return fail(SF_ERR_ARGUMENT, "raster_forward: NULL buffer");
  int tx;
  const int n_tiles = tiles_of(camera, &tx);
  if (settings->distortions & SF_DIST_L1) {
    if (!l1_samples) return fail(SF_ERR_ARGUMENT, "raster_forward: L1 requested without sample storage");
    if (!l1_offsets && (l1_cap <= 0 || l1_slots < (int64_t)n_tiles * 256 * l1_cap))
      return fail(SF_ERR_CAPACITY, "raster_forward: L1 storage of %lld slots is smaller than tiles*256*cap",
                  (long long)l1_slots);
  }
  if (!aligned(records, 16)) return fail(SF_ERR_ARGUMENT, "raster_forward: records need 16-byte alignment");
  sf::RasterFwdArgs a;
  a.records = records; a.ids = isect_ids; a.ranges = reinterpret_cast<const int2*>(tile_ranges);
  a.cam = *camera; a.st = *settings; a.tiles_x = tx;
  a.rgb = rgb; a.alpha = alpha; a.depth = depth; a.normals = normals; a.l1 = distortion_l1; a.l2 = distortion_l2;
  a.median = median_depth; a.ray_color = ray_color; a.amb = ambiguity; a.state = pixel_state;
  a.l1s = l1_samples; a.l1_slots = l1_slots; a.l1_off = l1_offsets; a.l1_cap = l1_cap; a.l1_needed = l1_needed;
  a.counters = reinterpret_cast<unsigned long long*>(counters);
  if (counters && !aligned(counters, 8)) return fail(SF_ERR_ARGUMENT, "raster_forward: counters alignment");
  return cuda_status(sf::launch_raster_forward(a, n_tiles, as_stream(stream)), "raster_forward");
}

int sf_b200_l1_offsets(const sf_camera* camera, const float* pixel_state, int64_t* offsets, void* workspace,
                       size_t workspace_bytes, void* stream) {
  int rc;
  if ((rc = check_camera(camera, "l1_offsets"))) return rc;
  if (!pixel_state || !offsets || !workspace) return fail(SF_ERR_ARGUMENT, "l1_offsets: NULL buffer");
  const int64_t npix = (int64_t)camera->width * camera->height;
  const size_t need = sf::scan_workspace_bytes(npix);
  if (workspace_bytes < need) return fail(SF_ERR_CAPACITY, "l1_offsets: workspace of %zu bytes, %zu needed",
                                          workspace_bytes, need);
  char* ws = reinterpret_cast<char*>(workspace);
  const size_t part = need - ((size_t)npix * sizeof(int32_t) + 255) / 256 * 256;
  int32_t* counts = reinterpret_cast<int32_t*>(ws + part);
  cudaStream_t s = as_stream(stream);
  cudaError_t e = sf::launch_pixel_counts(pixel_state, npix, counts, s);
  if (e == cudaSuccess) e = sf::scan_counts(counts, npix, offsets, ws, part, s);
  return cuda_status(e, "l1_offsets");
}

int sf_b200_l1_resolve(const sf_camera* camera, const sf_settings* settings, float* pixel_state, float* l1_samples,
                       int64_t l1_slots, const int64_t* l1_offsets, int32_t l1_cap, int32_t max_samples,
                       float* distortion_l1, void* stream) {
  int rc;
  if ((rc = check_settings(settings, "l1_resolve")) || (rc = check_camera(camera, "l1_resolve"))) return rc;
  if (!pixel_state || !l1_samples || !distortion_l1) return fail(SF_ERR_ARGUMENT, "l1_resolve: NULL buffer");
  if (max_samples < 0) return fail(SF_ERR_ARGUMENT, "l1_resolve: negative max_samples");
  const int smem_k = ((max_samples > 0 ? max_samples : 1) + 31) / 32 * 32;
  if (sf::l1_resolve_smem_per_warp(smem_k) > 200 * 1024)
    return fail(SF_ERR_CAPACITY,
                "l1_resolve: a pixel has %d contributing samples, more than the %d the shared-memory sort "
                "stages; raise transmittance_floor",
                max_samples, (int)((200 * 1024 / 4 - 256) / 5));
  return cuda_status(sf::launch_l1_resolve(*camera, *settings, pixel_state, l1_samples, l1_slots, l1_offsets, l1_cap,
                                           max_samples, distortion_l1, as_stream(stream)),
                     "l1_resolve");
}

int sf_b200_raster_backward(const float* records, int64_t n, const int32_t* isect_ids, const int32_t* tile_ranges,
                            const sf_camera* camera, const sf_settings* settings, const float* pixel_state,
                            const float* l1_samples, int64_t l1_slots, const int64_t* l1_offsets, int32_t l1_cap,
                            const float* grad_rgb, const float* grad_alpha, const float* grad_depth,
                            const float* grad_normals, const float* grad_l1, const float* grad_l2,
                            const float* grad_median, const float* grad_ray_color, const float* grad_ambiguity,
                            float* grad_records, float* grad_means2d, float* absgrad, int32_t* error_word,
                            void* stream) {
  int rc;
  if ((rc = check_settings(settings, "raster_backward")) || (rc = check_camera(camera, "raster_backward"))) return rc;
  if (!tile_ranges || !pixel_state || n < 0 || (n > 0 && (!records || !grad_records || !grad_means2d || !absgrad)))
    return fail(SF_ERR_ARGUMENT, "raster_backward: NULL buffer");
  if ((settings->distortions & SF_DIST_L1) && !l1_samples)
    return fail(SF_ERR_ARGUMENT, "raster_backward: L1 requested without sample storage");
  if (!aligned(records, 16) || !aligned(grad_records, 16) || !aligned(absgrad, 8) || !aligned(grad_means2d, 8))
    return fail(SF_ERR_ARGUMENT, "raster_backward: alignment");
  int tx;
  const int n_tiles = tiles_of(camera, &tx);
  sf::RasterBwdArgs a;
  a.records = records; a.ids = isect_ids; a.ranges = reinterpret_cast<const int2*>(tile_ranges);
  a.cam = *camera; a.st = *settings; a.tiles_x = tx; a.state = pixel_state;
  a.l1s = l1_samples; a.l1_slots = l1_slots; a.l1_off = l1_offsets; a.l1_cap = l1_cap;
  a.g_rgb = grad_rgb; a.g_alpha = grad_alpha; a.g_depth = grad_depth; a.g_normals = grad_normals;
  a.g_l1 = grad_l1; a.g_l2 = grad_l2; a.g_median = grad_median; a.g_var = grad_ray_color; a.g_amb = grad_ambiguity;
  a.grad_records = grad_records; a.absgrad = absgrad; a.error_word = error_word;
  cudaStream_t s = as_stream(stream);
  cudaError_t e = sf::launch_raster_backward(a, n_tiles, s);
  if (e == cudaSuccess) e = sf::launch_raster_finalize(records, n, *camera, settings->mode, grad_records, grad_means2d, s);
  return cuda_status(e, "raster_backward");
}

int sf_b200_opacity_field_workspace_bytes(int64_t n_gaussians, size_t* bytes) {
  if (n_gaussians < 0 || !bytes) return fail(SF_ERR_ARGUMENT, "opacity_field_workspace_bytes: bad arguments");
  *bytes = sf::field_workspace_bytes(n_gaussians);
  return SF_OK;
}

int sf_b200_opacity_field(const float* points, int64_t n_points, const float* means, const float* inverse_covariances,
                          const float* opacities, int64_t n_gaussians, const float* origins, int32_t n_origins,
                          float* field, void* workspace, size_t workspace_bytes, void* stream) {
  if (n_points < 0 || n_gaussians < 0) return fail(SF_ERR_ARGUMENT, "opacity_field: negative size");
  if (n_origins < 1 || n_origins > 65535) return fail(SF_ERR_ARGUMENT, "opacity_field: requires 1..65535 origins");
  if (n_points > 0 && (!points || !field || !origins)) return fail(SF_ERR_ARGUMENT, "opacity_field: NULL buffer");
  if (n_gaussians > 0 && (!means || !inverse_covariances || !opacities || !workspace))
    return fail(SF_ERR_ARGUMENT, "opacity_field: NULL buffer");
  if (workspace_bytes < sf::field_workspace_bytes(n_gaussians))
    return fail(SF_ERR_CAPACITY, "opacity_field: workspace too small");
  return cuda_status(sf::launch_opacity_field(points, n_points, means, inverse_covariances, opacities, n_gaussians,
                                              origins, n_origins, field, workspace, as_stream(stream)),
                     "opacity_field");
}

int sf_b200_opacity_field_culled_workspace_bytes(int64_t n_points, int64_t n_gaussians, int64_t max_pairs,
                                                 int32_t face_cells, size_t* bytes) {
  if (n_points < 0 || n_gaussians < 0 || max_pairs < 0 || face_cells < 1 || face_cells > 1024 || !bytes)
    return fail(SF_ERR_ARGUMENT, "opacity_field_culled_workspace_bytes: bad arguments");
  *bytes = sf::field_culled_workspace_bytes(n_gaussians, max_pairs, face_cells) +
           sf::field_culled_query_bytes(n_points, face_cells);
  return SF_OK;
}

static int field_culled(const float* points, int64_t n_points, const float* means,
                                 const float* inverse_covariances, const float* opacities, int64_t n_gaussians,
                                 const float* origins, int32_t n_origins, float cutoff, int32_t face_cells,
                                 float* field, void* workspace, size_t workspace_bytes, int64_t max_pairs,
                                 int64_t* pairs_needed, void* stream, int64_t* pairs_evaluated, float* query_ms) {
  if (n_points < 0 || n_gaussians < 0 || max_pairs < 0) return fail(SF_ERR_ARGUMENT, "opacity_field_culled: negative size");
  if (n_origins < 1) return fail(SF_ERR_ARGUMENT, "opacity_field_culled: requires at least one origin");
  if (!(cutoff > 0.f && cutoff < 1.f)) return fail(SF_ERR_ARGUMENT, "opacity_field_culled: cutoff must be in (0, 1)");
  if (face_cells < 1 || face_cells > 1024) return fail(SF_ERR_ARGUMENT, "opacity_field_culled: face_cells in 1..1024");
  if (n_points > 0 && (!points || !field || !origins)) return fail(SF_ERR_ARGUMENT, "opacity_field_culled: NULL buffer");
  if (n_gaussians > 0 && (!means || !inverse_covariances || !opacities || !workspace))
    return fail(SF_ERR_ARGUMENT, "opacity_field_culled: NULL buffer");
  if (n_gaussians > INT32_MAX || max_pairs > ((int64_t)1 << 31))
    return fail(SF_ERR_ARGUMENT, "opacity_field_culled: 32-bit index range exceeded");
  if (n_points > INT32_MAX) return fail(SF_ERR_ARGUMENT, "opacity_field_culled: 32-bit index range exceeded");
  const size_t need = sf::field_culled_workspace_bytes(n_gaussians, max_pairs, face_cells) +
                      sf::field_culled_query_bytes(n_points, face_cells);
  if (workspace_bytes < need) return fail(SF_ERR_CAPACITY, "opacity_field_culled: workspace of %zu bytes, %zu needed",
                                          workspace_bytes, need);
  int64_t most = 0;
  const int rc = cuda_status(sf::launch_opacity_field_culled(points, n_points, means, inverse_covariances, opacities,
                                                             n_gaussians, origins, n_origins, cutoff, face_cells,
                                                             field, workspace, workspace_bytes, max_pairs, &most,
                                                             as_stream(stream),
                                                             reinterpret_cast<unsigned long long*>(pairs_evaluated),
                                                             query_ms),
                             "opacity_field_culled");
  if (pairs_needed) *pairs_needed = most;
  if (rc != SF_OK) return rc;
  if (most > max_pairs)
    return fail(SF_ERR_CAPACITY, "opacity_field_culled: %lld candidate pairs in one view, max_pairs is %lld",
                (long long)most, (long long)max_pairs);
  return SF_OK;
}

int sf_b200_opacity_field_culled(const float* points, int64_t n_points, const float* means,
                                 const float* inverse_covariances, const float* opacities, int64_t n_gaussians,
                                 const float* origins, int32_t n_origins, float cutoff, int32_t face_cells,
                                 float* field, void* workspace, size_t workspace_bytes, int64_t max_pairs,
                                 int64_t* pairs_needed, void* stream) {
  return field_culled(points, n_points, means, inverse_covariances, opacities, n_gaussians, origins, n_origins,
                      cutoff, face_cells, field, workspace, workspace_bytes, max_pairs, pairs_needed, stream,
                      nullptr, nullptr);
}

int sf_b200_opacity_field_culled_stats(const float* points, int64_t n_points, const float* means,
                                       const float* inverse_covariances, const float* opacities,
                                       int64_t n_gaussians, const float* origins, int32_t n_origins, float cutoff,
                                       int32_t face_cells, float* field, void* workspace, size_t workspace_bytes,
                                       int64_t max_pairs, int64_t* pairs_needed, int64_t* pairs_evaluated,
                                       float* query_ms, void* stream) {
  if (!pairs_evaluated || !query_ms) return fail(SF_ERR_ARGUMENT, "opacity_field_culled_stats: NULL counter");
  return field_culled(points, n_points, means, inverse_covariances, opacities, n_gaussians, origins, n_origins,
                      cutoff, face_cells, field, workspace, workspace_bytes, max_pairs, pairs_needed, stream,
                      pairs_evaluated, query_ms);
}

int sf_b200_opacity_field_plan_bytes(int64_t n_gaussians, int32_t n_origins, int32_t face_cells, int64_t total_pairs,
                                     int64_t max_view_pairs, size_t* bytes) {
  if (n_gaussians < 0 || n_origins < 1 || face_cells < 1 || face_cells > 1024 || total_pairs < 0 ||
      max_view_pairs < 0 || !bytes)
    return fail(SF_ERR_ARGUMENT, "opacity_field_plan_bytes: bad arguments");
  *bytes = sf::field_plan_bytes(n_gaussians, n_origins, face_cells, total_pairs, max_view_pairs);
  return SF_OK;
}

int sf_b200_opacity_field_plan_build(const float* means, const float* inverse_covariances, const float* opacities,
                                     int64_t n_gaussians, const float* origins, int32_t n_origins, float cutoff,
                                     int32_t face_cells, void* plan, size_t plan_bytes, int64_t total_pairs,
                                     int64_t max_view_pairs, int64_t* needed, void* stream) {
  if (n_gaussians < 0 || total_pairs < 0 || max_view_pairs < 0 || !needed)
    return fail(SF_ERR_ARGUMENT, "opacity_field_plan_build: bad arguments");
  if (n_origins < 1) return fail(SF_ERR_ARGUMENT, "opacity_field_plan_build: requires at least one origin");
  if (!(cutoff > 0.f && cutoff < 1.f)) return fail(SF_ERR_ARGUMENT, "opacity_field_plan_build: cutoff must be in (0, 1)");
  if (face_cells < 1 || face_cells > 1024) return fail(SF_ERR_ARGUMENT, "opacity_field_plan_build: face_cells in 1..1024");
  if (!origins || !plan || (n_gaussians > 0 && (!means || !inverse_covariances || !opacities)))
    return fail(SF_ERR_ARGUMENT, "opacity_field_plan_build: NULL buffer");
  if (n_gaussians > INT32_MAX || total_pairs > INT64_C(1) << 40 || max_view_pairs > ((int64_t)1 << 31))
    return fail(SF_ERR_ARGUMENT, "opacity_field_plan_build: index range exceeded");
  const size_t need = sf::field_plan_bytes(n_gaussians, n_origins, face_cells, total_pairs, max_view_pairs);
  if (plan_bytes < need)
    return fail(SF_ERR_CAPACITY, "opacity_field_plan_build: plan of %zu bytes, %zu needed", plan_bytes, need);
  const int rc = cuda_status(sf::field_plan_build(means, inverse_covariances, opacities, n_gaussians, origins, n_origins,
                                                  cutoff, face_cells, plan, plan_bytes, total_pairs, max_view_pairs,
                                                  needed, as_stream(stream)),
                             "opacity_field_plan_build");
  if (rc != SF_OK) return rc;
  if (needed[0] > total_pairs || needed[1] > max_view_pairs)
    return fail(SF_ERR_CAPACITY, "opacity_field_plan_build: %lld candidate pairs (%lld in one view) exceed %lld (%lld)",
                (long long)needed[0], (long long)needed[1], (long long)total_pairs, (long long)max_view_pairs);
  return SF_OK;
}

int sf_b200_opacity_field_plan_query_bytes(int64_t n_points, int32_t n_origins, int32_t face_cells, size_t* bytes) {
  if (n_points < 0 || n_origins < 1 || face_cells < 1 || face_cells > 1024 || !bytes)
    return fail(SF_ERR_ARGUMENT, "opacity_field_plan_query_bytes: bad arguments");
  if (n_points * n_origins > INT32_MAX)
    return fail(SF_ERR_CAPACITY, "opacity_field_plan_query_bytes: %lld (query, origin) pairs exceed 2^31 - 1",
                (long long)(n_points * n_origins));
  *bytes = sf::field_plan_query_bytes(n_points, n_origins, face_cells);
  return SF_OK;
}

int sf_b200_opacity_field_plan_eval(const void* plan, int64_t n_gaussians, int32_t n_origins, int32_t face_cells,
                                    int64_t total_pairs, int64_t max_view_pairs, const float* origins,
                                    const float* points, int64_t n_points, float* field, void* workspace,
                                    size_t workspace_bytes, void* stream) {
  if (n_gaussians < 0 || n_points < 0 || n_origins < 1 || face_cells < 1 || face_cells > 1024 || total_pairs < 0 ||
      max_view_pairs < 0)
    return fail(SF_ERR_ARGUMENT, "opacity_field_plan_eval: bad arguments");
  if (n_points * n_origins > INT32_MAX)
    return fail(SF_ERR_CAPACITY, "opacity_field_plan_eval: %lld (query, origin) pairs exceed 2^31 - 1",
                (long long)(n_points * n_origins));
  if (n_points > 0 && (!plan || !origins || !points || !field || !workspace))
    return fail(SF_ERR_ARGUMENT, "opacity_field_plan_eval: NULL buffer");
  const size_t need = sf::field_plan_query_bytes(n_points, n_origins, face_cells);
  if (workspace_bytes < need)
    return fail(SF_ERR_CAPACITY, "opacity_field_plan_eval: workspace of %zu bytes, %zu needed", workspace_bytes, need);
  return cuda_status(sf::field_plan_eval(plan, n_gaussians, n_origins, face_cells, total_pairs, max_view_pairs, origins,
                                         points, n_points, field, workspace, workspace_bytes, as_stream(stream)),
                     "opacity_field_plan_eval");
}

int sf_b200_pixel_rays(const float* K, int32_t width, int32_t height, float* rays, void* stream) {
  if (width <= 0 || height <= 0) return fail(SF_ERR_ARGUMENT, "pixel_rays: width and height must be positive");
  if (!K || !rays) return fail(SF_ERR_ARGUMENT, "pixel_rays: NULL buffer");
  return cuda_status(sf::launch_pixel_rays(K, width, height, rays, as_stream(stream)), "pixel_rays");
}

int sf_b200_ray_peak(const float* means, const float* inverse_covariances, int64_t n_gaussians, const float* origins,
                     const float* directions, int64_t n_rays, float* t, float* response, float* normals,
                     void* stream) {
  if (n_gaussians < 0 || n_rays < 0) return fail(SF_ERR_ARGUMENT, "ray_peak: negative size");
  if (n_gaussians * n_rays > 0 && (!means || !inverse_covariances || !origins || !directions || !t || !response ||
                                   !normals))
    return fail(SF_ERR_ARGUMENT, "ray_peak: NULL buffer");
  return cuda_status(sf::launch_ray_peak(means, inverse_covariances, n_gaussians, origins, directions, n_rays, t,
                                         response, normals, as_stream(stream)),
                     "ray_peak");
}

int sf_b200_depth_normals(const float* depth, const float* K, int32_t width, int32_t height, float* normals,
                          uint8_t* valid, void* stream) {
  if (width < 0 || height < 0) return fail(SF_ERR_ARGUMENT, "depth_normals: negative size");
  if ((int64_t)width * height > 0 && (!depth || !K || !normals || !valid))
    return fail(SF_ERR_ARGUMENT, "depth_normals: NULL buffer");
  return cuda_status(sf::launch_depth_normals(depth, K, width, height, normals, valid, as_stream(stream)),
                     "depth_normals");
}

int sf_b200_depth_normals_backward(const float* depth, const float* K, int32_t width, int32_t height,
                                   const float* grad_normals, float* grad_depth, float* workspace, void* stream) {
  if (width < 0 || height < 0) return fail(SF_ERR_ARGUMENT, "depth_normals_backward: negative size");
  if ((int64_t)width * height > 0 && (!depth || !K || !grad_normals || !grad_depth || !workspace))
    return fail(SF_ERR_ARGUMENT, "depth_normals_backward: NULL buffer");
  return cuda_status(sf::launch_depth_normals_backward(depth, K, width, height, grad_normals, grad_depth, workspace,
                                                       as_stream(stream)),
                     "depth_normals_backward");
}

int sf_b200_composite_workspace_bytes(int64_t B, int64_t N, int64_t P, int32_t distortions, size_t* bytes) {
  if (B < 0 || N < 0 || P < 0 || !bytes) return fail(SF_ERR_ARGUMENT, "composite_workspace_bytes: bad arguments");
  const size_t aux = (distortions & SF_DIST_L1) ? (size_t)2 * B * N * P * sizeof(float) : 0;
  *bytes = aux + (size_t)2 * B * P * sizeof(float) + 256;
  return SF_OK;
}

namespace {
int composite_checks(int64_t B, int64_t N, int64_t P, int32_t dist, size_t ws_bytes, const char* where) {
  if (B < 0 || N < 0 || P < 0) return fail(SF_ERR_ARGUMENT, "%s: negative size", where);
  if (dist < 0 || dist > 3) return fail(SF_ERR_ARGUMENT, "%s: distortions must be none/l1/l2/both", where);
  if (B * N * P >= (int64_t)1 << 40 || B * P > 0x7fffffffLL * 128 || N > 0x7fffffffLL)
    return fail(SF_ERR_ARGUMENT, "%s: sizes too large", where);
  size_t need = 0;
  sf_b200_composite_workspace_bytes(B, N, P, dist, &need);
  if (ws_bytes < need) return fail(SF_ERR_CAPACITY, "%s: workspace of %zu bytes, %zu needed", where, ws_bytes, need);
  if ((dist & SF_DIST_L1) && sf::composite_l1_smem_per_warp((int)N) > 200 * 1024)
    return fail(SF_ERR_CAPACITY, "%s: L1 over %lld samples exceeds the shared-memory sort", where, (long long)N);
  return SF_OK;
}
}  // namespace

int sf_b200_alpha_composite_forward(const float* alphas, const float* colors, const float* depths, const float* normals,
                                    int64_t B, int64_t N, int64_t P, int32_t distortions, float* rgb, float* alpha,
                                    float* znum, float* nnum, float* l1, float* l2, float* median, float* weights,
                                    void* workspace, size_t workspace_bytes, void* stream) {
  int rc;
  if ((rc = composite_checks(B, N, P, distortions, workspace_bytes, "alpha_composite_forward"))) return rc;
  if (B * P > 0 && (!rgb || !alpha || !znum || !nnum || !l1 || !l2 || !median || !workspace))
    return fail(SF_ERR_ARGUMENT, "alpha_composite_forward: NULL output");
  if (B * N * P > 0 && (!alphas || !colors || !depths || !normals || !weights))
    return fail(SF_ERR_ARGUMENT, "alpha_composite_forward: NULL input");
  float* raw = reinterpret_cast<float*>(workspace);
  float* aux = (distortions & SF_DIST_L1) ? raw + 2 * B * P : nullptr;
  return cuda_status(sf::launch_composite_forward(alphas, colors, depths, normals, (int)B, (int)N, (int)P, distortions,
                                                  rgb, alpha, znum, nnum, l1, l2, median, weights, aux, raw,
                                                  as_stream(stream)),
                     "alpha_composite_forward");
}

int sf_b200_alpha_composite_backward(const float* alphas, const float* colors, const float* depths,
                                     const float* normals, int64_t B, int64_t N, int64_t P, int32_t distortions,
                                     const float* weights, const void* workspace, size_t workspace_bytes,
                                     const float* grad_rgb, const float* grad_alpha, const float* grad_znum,
                                     const float* grad_nnum, const float* grad_l1, const float* grad_l2,
                                     const float* grad_median, const float* grad_weights, float* d_alphas,
                                     float* d_colors, float* d_depths, float* d_normals, void* stream) {
  int rc;
  if ((rc = composite_checks(B, N, P, distortions, workspace_bytes, "alpha_composite_backward"))) return rc;
  if (B * N * P > 0 && (!alphas || !colors || !depths || !normals || !weights || !workspace || !d_alphas ||
                        !d_colors || !d_depths || !d_normals))
    return fail(SF_ERR_ARGUMENT, "alpha_composite_backward: NULL buffer");
  const float* raw = reinterpret_cast<const float*>(workspace);
  const float* aux = (distortions & SF_DIST_L1) ? raw + 2 * B * P : nullptr;
  return cuda_status(sf::launch_composite_backward(alphas, colors, depths, normals, (int)B, (int)N, (int)P,
                                                   distortions, weights, aux, raw, grad_rgb, grad_alpha, grad_znum,
                                                   grad_nnum, grad_l1, grad_l2, grad_median, grad_weights, d_alphas,
                                                   d_colors, d_depths, d_normals, as_stream(stream)),
                     "alpha_composite_backward");
}

// ------------------------------------------------------------------ training-step operations
int sf_b200_sh_ambiguity(const float* coefficients, int64_t n, int32_t k, float* out, void* stream) {
  if (n < 0 || k < 1) return fail(SF_ERR_ARGUMENT, "sh_ambiguity: bad sizes");
  if (n > 0 && (!coefficients || !out)) return fail(SF_ERR_ARGUMENT, "sh_ambiguity: NULL buffer");
  return cuda_status(sf::launch_sh_ambiguity(coefficients, n, k, out, as_stream(stream)), "sh_ambiguity");
}

int sf_b200_sh_ambiguity_backward(const float* coefficients, int64_t n, int32_t k, const float* grad,
                                  float* grad_coefficients, void* stream) {
  if (n < 0 || k < 1) return fail(SF_ERR_ARGUMENT, "sh_ambiguity_backward: bad sizes");
  if (n > 0 && (!coefficients || !grad || !grad_coefficients))
    return fail(SF_ERR_ARGUMENT, "sh_ambiguity_backward: NULL buffer");
  return cuda_status(sf::launch_sh_ambiguity_backward(coefficients, n, k, grad, grad_coefficients, as_stream(stream)),
                     "sh_ambiguity_backward");
}

int sf_b200_ray_color_variance(const float* weights, const float* colors, const float* composite, int64_t batches,
                               int64_t n, int64_t pixels, float* out, void* stream) {
  if (batches < 0 || n < 0 || pixels < 0) return fail(SF_ERR_ARGUMENT, "ray_color_variance: negative size");
  if (batches * pixels > 0 && (!composite || !out || (n > 0 && (!weights || !colors))))
    return fail(SF_ERR_ARGUMENT, "ray_color_variance: NULL buffer");
  return cuda_status(sf::launch_ray_color_variance(weights, colors, composite, batches, n, pixels, out,
                                                   as_stream(stream)),
                     "ray_color_variance");
}

int sf_b200_ray_color_variance_backward(const float* weights, const float* colors, const float* composite,
                                        const float* grad, int64_t batches, int64_t n, int64_t pixels,
                                        float* grad_colors, void* stream) {
  if (batches < 0 || n < 0 || pixels < 0) return fail(SF_ERR_ARGUMENT, "ray_color_variance_backward: negative size");
  if (batches * n > 0 && (!weights || !colors || !grad_colors || (pixels > 0 && (!composite || !grad))))
    return fail(SF_ERR_ARGUMENT, "ray_color_variance_backward: NULL buffer");
  return cuda_status(sf::launch_ray_color_variance_backward(weights, colors, composite, grad, batches, n, pixels,
                                                            grad_colors, as_stream(stream)),
                     "ray_color_variance_backward");
}

int sf_b200_patch_zncc(const float* a, const float* b, const float* mask, int64_t rows, int32_t samples, float epsilon,
                       float* correlation, uint8_t* valid, void* stream) {
  if (rows < 0 || samples < 0) return fail(SF_ERR_ARGUMENT, "patch_zncc: negative size");
  if (rows > 0 && (!a || !b || !mask || !correlation || !valid)) return fail(SF_ERR_ARGUMENT, "patch_zncc: NULL buffer");
  return cuda_status(sf::launch_patch_zncc(a, b, mask, rows, samples, epsilon, correlation, valid, as_stream(stream)),
                     "patch_zncc");
}

int sf_b200_patch_zncc_backward(const float* a, const float* b, const float* mask, int64_t rows, int32_t samples,
                                float epsilon, const float* grad_correlation, float* grad_a, float* grad_b,
                                void* stream) {
  if (rows < 0 || samples < 0) return fail(SF_ERR_ARGUMENT, "patch_zncc_backward: negative size");
  if (rows > 0 && (!a || !b || !mask || !grad_correlation || !grad_a || !grad_b))
    return fail(SF_ERR_ARGUMENT, "patch_zncc_backward: NULL buffer");
  return cuda_status(sf::launch_patch_zncc_backward(a, b, mask, rows, samples, epsilon, grad_correlation, grad_a,
                                                    grad_b, as_stream(stream)),
                     "patch_zncc_backward");
}

int sf_b200_densify_observe(const float* grad2d, const float* radii, int64_t n, float scale_x, float scale_y,
                            float* gradient, float* observations, void* stream) {
  if (n < 0) return fail(SF_ERR_ARGUMENT, "densify_observe: negative size");
  if (n > 0 && (!grad2d || !radii || !gradient || !observations))
    return fail(SF_ERR_ARGUMENT, "densify_observe: NULL buffer");
  return cuda_status(sf::launch_densify_observe(grad2d, radii, n, scale_x, scale_y, gradient, observations,
                                                as_stream(stream)),
                     "densify_observe");
}

int sf_b200_normal_consistency_workspace_bytes(int32_t width, int32_t height, size_t* bytes) {
  if (width < 0 || height < 0 || !bytes) return fail(SF_ERR_ARGUMENT, "normal_consistency_workspace_bytes: bad arguments");
  *bytes = sf::normal_consistency_workspace_bytes(width, height);
  return SF_OK;
}

static int nc_check(const char* what, const float* depth, const float* K, int32_t width, int32_t height,
                    const float* alpha, const float* numer, const float* normals, const float* mask, size_t ws_bytes,
                    const void* ws) {
  if (width < 0 || height < 0) return fail(SF_ERR_ARGUMENT, "%s: negative size", what);
  if ((numer == nullptr) == (normals == nullptr))
    return fail(SF_ERR_ARGUMENT, "%s: pass exactly one of normal_numerator and normals", what);
  if (!K || !ws || ((int64_t)width * height > 0 && (!depth || !alpha || !mask)))
    return fail(SF_ERR_ARGUMENT, "%s: NULL buffer", what);
  if (ws_bytes < sf::normal_consistency_workspace_bytes(width, height))
    return fail(SF_ERR_CAPACITY, "%s: workspace of %zu bytes, %zu needed", what, ws_bytes,
                sf::normal_consistency_workspace_bytes(width, height));
  return SF_OK;
}

int sf_b200_normal_consistency(const float* depth, const float* K, int32_t width, int32_t height, const float* alpha,
                               const float* normal_numerator, const float* normals, const float* mask, float* loss,
                               int64_t* count, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = nc_check("normal_consistency", depth, K, width, height, alpha, normal_numerator, normals, mask,
                    workspace_bytes, workspace);
  if (rc != SF_OK) return rc;
  if (!loss || !count) return fail(SF_ERR_ARGUMENT, "normal_consistency: NULL buffer");
  return cuda_status(sf::normal_consistency(depth, K, width, height, alpha, normal_numerator, normals, mask, loss,
                                            count, workspace, as_stream(stream)),
                     "normal_consistency");
}

int sf_b200_normal_consistency_backward(const float* depth, const float* K, int32_t width, int32_t height,
                                        const float* alpha, const float* normal_numerator, const float* normals,
                                        const float* mask, const float* grad_loss, const int64_t* count,
                                        float* grad_depth, float* grad_alpha, float* grad_vector, float* grad_normals,
                                        void* workspace, size_t workspace_bytes, void* stream) {
  int rc = nc_check("normal_consistency_backward", depth, K, width, height, alpha, normal_numerator, normals, mask,
                    workspace_bytes, workspace);
  if (rc != SF_OK) return rc;
  if ((int64_t)width * height > 0 && (!grad_loss || !count || !grad_depth || !grad_normals))
    return fail(SF_ERR_ARGUMENT, "normal_consistency_backward: NULL buffer");
  return cuda_status(sf::normal_consistency_backward(depth, K, width, height, alpha, normal_numerator, normals, mask,
                                                     grad_loss, count, grad_depth, grad_alpha, grad_vector,
                                                     grad_normals, workspace, as_stream(stream)),
                     "normal_consistency_backward");
}

// ------------------------------------------------------------------ GOF mesh extraction
int sf_b200_mesh_grid_points(const float* means, const float* quats, const float* scales, const int32_t* chosen,
                             int64_t n, double extent, double* points, double* radius, void* stream) {
  if (n < 0) return fail(SF_ERR_ARGUMENT, "mesh_grid_points: negative size");
  if (n > 0 && (!means || !quats || !scales || !chosen || !points || !radius))
    return fail(SF_ERR_ARGUMENT, "mesh_grid_points: NULL buffer");
  return cuda_status(sf::launch_grid_points(means, quats, scales, chosen, n, extent, points, radius,
                                            as_stream(stream)),
                     "mesh_grid_points");
}

int sf_b200_mesh_count_workspace_bytes(int64_t n_cells, size_t* bytes) {
  if (n_cells < 0 || !bytes) return fail(SF_ERR_ARGUMENT, "mesh_count_workspace_bytes: bad arguments");
  *bytes = sf::mesh_count_workspace_bytes(n_cells);
  return SF_OK;
}

int sf_b200_mesh_count(const double* values, int64_t n_points, const int32_t* cells, int64_t n_cells, double level,
                       int32_t inside_greater, uint8_t* inside, int64_t* slot_offsets, int64_t* face_offsets,
                       void* workspace, size_t workspace_bytes, void* stream) {
  if (n_points < 0 || n_cells < 0 || n_points > 0x7fffffffLL)
    return fail(SF_ERR_ARGUMENT, "mesh_count: sizes must be non-negative and points fit 32-bit indices");
  if (!slot_offsets || !face_offsets || (n_points > 0 && (!values || !inside)) ||
      (n_cells > 0 && (!cells || !inside || !workspace)))
    return fail(SF_ERR_ARGUMENT, "mesh_count: NULL buffer");
  if (reinterpret_cast<uintptr_t>(cells) % 16) return fail(SF_ERR_ARGUMENT, "mesh_count: cells must be 16-byte aligned");
  if (workspace_bytes < sf::mesh_count_workspace_bytes(n_cells))
    return fail(SF_ERR_CAPACITY, "mesh_count: workspace of %zu bytes, %zu needed", workspace_bytes,
                sf::mesh_count_workspace_bytes(n_cells));
  return cuda_status(sf::mesh_count(values, n_points, cells, n_cells, level, inside_greater != 0, inside, slot_offsets,
                                    face_offsets, workspace, workspace_bytes, as_stream(stream)),
                     "mesh_count");
}

int sf_b200_mesh_edges_workspace_bytes(int64_t n_slots, size_t* bytes) {
  if (n_slots < 0 || !bytes) return fail(SF_ERR_ARGUMENT, "mesh_edges_workspace_bytes: bad arguments");
  if (n_slots > 0x7fffffffLL) return fail(SF_ERR_CAPACITY, "mesh_edges: %lld crossing slots exceed 32-bit indices",
                                          (long long)n_slots);
  *bytes = sf::mesh_edges_workspace_bytes(n_slots);
  return SF_OK;
}

int sf_b200_mesh_edges(const double* points, int64_t n_points, const int32_t* cells, int64_t n_cells,
                       const uint8_t* inside, const int64_t* slot_offsets, int64_t n_slots, int32_t* edge_ids,
                       int32_t* pairs, double* low, double* high, uint8_t* low_inside, int64_t* n_edges,
                       void* workspace, size_t workspace_bytes, void* stream) {
  if (n_points < 0 || n_cells < 0 || n_slots < 0 || !n_edges) return fail(SF_ERR_ARGUMENT, "mesh_edges: bad arguments");
  if (n_slots > 0x7fffffffLL || n_points > 0x7fffffffLL)
    return fail(SF_ERR_CAPACITY, "mesh_edges: sizes exceed 32-bit indices");
  if (n_slots > 0 && (!points || !cells || !inside || !slot_offsets || !edge_ids || !pairs || !low || !high ||
                      !low_inside || !workspace))
    return fail(SF_ERR_ARGUMENT, "mesh_edges: NULL buffer");
  if (reinterpret_cast<uintptr_t>(cells) % 16) return fail(SF_ERR_ARGUMENT, "mesh_edges: cells must be 16-byte aligned");
  if (workspace_bytes < sf::mesh_edges_workspace_bytes(n_slots))
    return fail(SF_ERR_CAPACITY, "mesh_edges: workspace of %zu bytes, %zu needed", workspace_bytes,
                sf::mesh_edges_workspace_bytes(n_slots));
  return cuda_status(sf::mesh_edges(points, n_points, cells, n_cells, inside, slot_offsets, n_slots, edge_ids, pairs,
                                    low, high, low_inside, n_edges, workspace, workspace_bytes, as_stream(stream)),
                     "mesh_edges");
}

int sf_b200_mesh_midpoints(const double* low, const double* high, int64_t n_edges, double* midpoints, void* stream) {
  if (n_edges < 0) return fail(SF_ERR_ARGUMENT, "mesh_midpoints: negative size");
  if (n_edges > 0 && (!low || !high || !midpoints)) return fail(SF_ERR_ARGUMENT, "mesh_midpoints: NULL buffer");
  return cuda_status(sf::mesh_midpoints(low, high, n_edges, midpoints, as_stream(stream)), "mesh_midpoints");
}

int sf_b200_mesh_bisect(double* low, double* high, const uint8_t* low_inside, int64_t n_edges, const double* values,
                        double level, int32_t inside_greater, void* stream) {
  if (n_edges < 0) return fail(SF_ERR_ARGUMENT, "mesh_bisect: negative size");
  if (n_edges > 0 && (!low || !high || !low_inside || !values)) return fail(SF_ERR_ARGUMENT, "mesh_bisect: NULL buffer");
  return cuda_status(sf::mesh_bisect(low, high, low_inside, n_edges, values, level, inside_greater != 0,
                                     as_stream(stream)),
                     "mesh_bisect");
}

int sf_b200_mesh_faces_workspace_bytes(int64_t n_faces, size_t* bytes) {
  if (n_faces < 0 || !bytes) return fail(SF_ERR_ARGUMENT, "mesh_faces_workspace_bytes: bad arguments");
  *bytes = sf::mesh_faces_workspace_bytes(n_faces);
  return SF_OK;
}

int sf_b200_mesh_faces(const double* points, const int32_t* cells, int64_t n_cells, const uint8_t* inside,
                       const int64_t* slot_offsets, const int32_t* edge_ids, const double* low, const double* high,
                       int64_t n_edges, const int64_t* face_offsets, int64_t n_faces, double* vertices,
                       int64_t* faces, int64_t* n_kept, void* workspace, size_t workspace_bytes, void* stream) {
  if (n_cells < 0 || n_edges < 0 || n_faces < 0 || !n_kept) return fail(SF_ERR_ARGUMENT, "mesh_faces: bad arguments");
  if (n_edges > 0 && (!low || !high || !vertices)) return fail(SF_ERR_ARGUMENT, "mesh_faces: NULL buffer");
  if (n_faces > 0 && (!points || !cells || !inside || !slot_offsets || !edge_ids || !face_offsets || !faces ||
                      !workspace))
    return fail(SF_ERR_ARGUMENT, "mesh_faces: NULL buffer");
  if (reinterpret_cast<uintptr_t>(cells) % 16) return fail(SF_ERR_ARGUMENT, "mesh_faces: cells must be 16-byte aligned");
  if (workspace_bytes < sf::mesh_faces_workspace_bytes(n_faces))
    return fail(SF_ERR_CAPACITY, "mesh_faces: workspace of %zu bytes, %zu needed", workspace_bytes,
                sf::mesh_faces_workspace_bytes(n_faces));
  return cuda_status(sf::mesh_faces(points, cells, n_cells, inside, slot_offsets, edge_ids, low, high, n_edges,
                                    face_offsets, n_faces, vertices, faces, n_kept, workspace, workspace_bytes,
                                    as_stream(stream)),
                     "mesh_faces");
}

}  // extern "C"
