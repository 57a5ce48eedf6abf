/*
 * splatforge_b200 -- C ABI of the B200 (sm_100a) Gaussian-splatting rasterizer.
 *
 * Every entry point takes DEVICE pointers (float32, contiguous, row-major), plain
 * sizes, a cudaStream_t passed as void*, and returns an int status (SF_OK == 0).
 * On failure the message of the calling thread is available from
 * sf_b200_last_error().  Nothing here allocates device memory: scratch space is
 * sized by the *_workspace_bytes() queries and passed in by the caller.  Inputs are
 * never written.  Kernels run on the given stream; no entry point synchronises the
 * device except where its comment says so.
 *
 * Reference interfaces replaced (paths relative to the SplatForge project):
 *   gaussian.covariance@1      src/splatforge/providers/torch/gaussian/reference.py:33-35
 *   gaussian.sh_color@1        src/splatforge/providers/torch/gaussian/reference.py:85-113
 *   projection + conic/radius/ src/splatforge/studio/renderers.py:76-107,
 *     SH colour + mode extras  src/splatforge/studio/batched_renderer.py:51-115
 *   tile binning               src/splatforge/studio/tile_binning.py:10-34 and the
 *                              bounds host copy batched_renderer.py:121-150
 *   per-tile evaluation +      src/splatforge/studio/batched_renderer.py:169-338,
 *     splat.alpha_composite@3  src/splatforge/providers/torch/gaussian/composite_cuda.cu:26-98
 *   backward (autograd)        same functions, reverse mode
 *   gaussian.opacity_field@1   src/splatforge/providers/torch/gaussian/reference.py:194-222
 *   camera.pixel_rays@1, gaussian.ray_peak@1, geometry.depth_normals@1
 *                              src/splatforge/providers/torch/gaussian/reference.py:38-83
 */
#ifndef SPLATFORGE_B200_H
#define SPLATFORGE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SF_B200_ABI_VERSION 1

/* rendering modes: the Studio ``rendering_mode`` (src/splatforge/studio/methods/*.py) */
enum { SF_MODE_RADEGS = 0, SF_MODE_GOF = 1, SF_MODE_AMBISUR = 2 };
/* distortion selection bits: splat.alpha_composite@3 ``distortions`` none/l1/l2/both */
enum { SF_DIST_L1 = 1, SF_DIST_L2 = 2 };
/* status codes */
enum {
  SF_OK = 0,
  SF_ERR_ARGUMENT = 1,  /* invalid size, pointer or setting */
  SF_ERR_CUDA = 2,      /* a CUDA runtime call or launch failed */
  SF_ERR_CAPACITY = 3,  /* caller-provided buffer too small (see message) */
  SF_ERR_KERNEL = 4     /* a kernel reported an internal error word */
};

/* floats per Gaussian record written by sf_b200_project_forward and read by the
 * raster kernels, and per gradient record written by sf_b200_raster_backward */
#define SF_RECORD_FLOATS 20
/* floats per pixel of the forward state kept for the backward pass */
#define SF_PIXEL_STATE_FLOATS 16
/* floats per stored L1 sample: depth and weight, which sf_b200_l1_resolve replaces by
 * the two adjoint factors the backward pass reads (stored column-wise) */
#define SF_L1_SAMPLE_FLOATS 2

/* Pinhole camera, OpenCV convention (src/splatforge/studio/cameras.py:8-22). */
typedef struct sf_camera {
  float R[9];      /* world-to-camera rotation, row-major */
  float t[3];      /* world-to-camera translation */
  float K[9];      /* intrinsics, row-major */
  float Kinv[9];   /* inverse of K (the caller computes it once, on the host) */
  float origin[3]; /* camera centre in world coordinates: inv(world_to_camera)[:3,3] */
  int32_t width;
  int32_t height;
} sf_camera;

/* The hot-path fields of RenderConfig (src/splatforge/studio/config.py:29-40) plus
 * the mode / distortion selection of a render call. */
typedef struct sf_settings {
  int32_t mode;         /* SF_MODE_* */
  int32_t distortions;  /* SF_DIST_* bits */
  int32_t tile_size;    /* must be 16 */
  int32_t sh_degree;    /* 0..3 */
  int32_t sh_coeffs;    /* K of sh[N,K,3]; K >= (sh_degree+1)^2 */
  int32_t antialiased;  /* opacity * sqrt(det(screen)/det(filtered)) */
  float extent;         /* sigma_extent (3.0), or trunc_sigma for AmbiSuR */
  float extent_sq;      /* float32(extent**2) as the host computes it (mask squared <= extent^2) */
  float eps2d;          /* 0.3 */
  float near_plane;     /* 0.01 */
  float far_plane;      /* 1e4 */
  float background[3];
  float t_stop;         /* a pixel stops once its transmittance falls below this (0: never) */
} sf_settings;

const char* sf_b200_last_error(void);
int sf_b200_abi_version(void);
/* Running total of kernels this library has launched in the process (diagnostics). */
int64_t sf_b200_kernel_launches(void);

/* ---- gaussian.covariance@1 (reference.py:33-35): cov[N,3,3] = R diag(s^2) R^T ---- */
int sf_b200_covariance_forward(const float* quats, const float* scales, int64_t n,
                               float* cov, void* stream);
/* grad_quats / grad_scales are overwritten (not accumulated). */
int sf_b200_covariance_backward(const float* quats, const float* scales, int64_t n,
                                const float* grad_cov, float* grad_quats,
                                float* grad_scales, void* stream);

/* ---- gaussian.sh_color@1 (reference.py:85-113): rgb[N,3] = max(0, 0.5 + SH(dir)) ---- */
int sf_b200_sh_color_forward(const float* coeffs, int32_t coeff_count, const float* dirs,
                             int64_t n, int32_t degree, float* rgb, void* stream);
/* grad_coeffs [N,K,3] and grad_dirs [N,3] are overwritten; either may be NULL. */
int sf_b200_sh_color_backward(const float* coeffs, int32_t coeff_count, const float* dirs,
                              int64_t n, int32_t degree, const float* grad_rgb,
                              float* grad_coeffs, float* grad_dirs, void* stream);

/* ---- projection, conic, radius, SH colour and mode extras -------------------------
 * renderers.py:76-107 + batched_renderer.py:57-115.  Per Gaussian writes:
 *   means2d[N,2], radii[N], records[N,SF_RECORD_FLOATS],
 *   tile_rect[N,4] (inclusive tile rectangle, int32), tile_count[N] (0 when culled),
 *   depth_key[N] (float bits of camera z; 0xFFFFFFFF when culled).
 * selected may be NULL (no ambiguity selection).  nonfinite (device int, may be NULL)
 * is incremented for every Gaussian whose projected bounds are not finite; such a
 * Gaussian is culled and the caller raises, as tile_binning.py:17-18 does. */
int sf_b200_project_forward(const float* means, const float* quats, const float* scales,
                            const float* opacities, const float* sh, const uint8_t* selected,
                            int64_t n, const sf_camera* camera, const sf_settings* settings,
                            float* means2d, float* radii, float* records, int32_t* tile_rect,
                            int32_t* tile_count, uint32_t* depth_key, int32_t* nonfinite,
                            void* stream);

/* Reverse of sf_b200_project_forward.  grad_means2d [N,2] is the total adjoint of the
 * projected means; grad_records [N,SF_RECORD_FLOATS] comes from sf_b200_raster_backward.
 * Outputs are overwritten; any output may be NULL. */
int sf_b200_project_backward(const float* means, const float* quats, const float* scales,
                             const float* opacities, const float* sh, int64_t n,
                             const sf_camera* camera, const sf_settings* settings,
                             const float* grad_means2d, const float* grad_records,
                             float* grad_means, float* grad_quats, float* grad_scales,
                             float* grad_opacities, float* grad_sh, void* stream);

/* ---- tile binning (tile_binning.py:10-34) ----------------------------------------
 * Bounds form (x, y, radius, z) per Gaussian, as the reference's host array; used by
 * the standalone binning entry point and its bit-exact tests.  Writes tile_rect,
 * tile_count, depth_key exactly like sf_b200_project_forward does. */
int sf_b200_bin_rects(const float* bounds, int64_t n, int32_t width, int32_t height,
                      int32_t tile_size, float near_plane, float far_plane,
                      int32_t* tile_rect, int32_t* tile_count, uint32_t* depth_key,
                      int32_t* nonfinite, void* stream);

/* Scratch needed by sf_b200_bin_order / sf_b200_bin_emit for n Gaussians, n_isect
 * intersections and n_tiles tiles. */
int sf_b200_bin_workspace_bytes(int64_t n, int64_t n_isect, int32_t n_tiles, size_t* bytes);

/* Stable depth order of the Gaussians and the exclusive scan of their tile counts in
 * that order.  order[N] (Gaussian ids), offsets[N+1] (int64); offsets[N] is the
 * intersection total, which the caller reads back to size the emit buffers. */
int sf_b200_bin_order(const int32_t* tile_count, const uint32_t* depth_key, int64_t n,
                      int32_t* order, int64_t* offsets, void* workspace,
                      size_t workspace_bytes, void* stream);

/* Emits every (tile, Gaussian) intersection in depth order, sorts them stably by tile
 * and writes per-tile [start,end) ranges.  isect_ids[n_isect] (Gaussian ids, tile-major,
 * depth order within a tile), tile_ranges[n_tiles,2]. */
int sf_b200_bin_emit(const int32_t* order, const int64_t* offsets, const int32_t* tile_rect,
                     int64_t n, int64_t n_isect, int32_t tiles_x, int32_t n_tiles,
                     int32_t* isect_ids, int32_t* tile_ranges, void* workspace,
                     size_t workspace_bytes, void* stream);

/* sf_b200_bin_emit without the host read of the intersection count: the count is
 * offsets[n] on the device and `capacity` sizes isect_ids and the workspace
 * (sf_b200_bin_workspace_bytes(0, capacity, n_tiles)).  A count above capacity emits
 * nothing, leaves every tile range empty and sets *overflow to 1 (a device int32 the
 * caller zeroes and reads back with its next synchronisation, then re-bins with the
 * exact count).  No counterpart in the reference (it bins on the host,
 * src/splatforge/studio/tile_binning.py:10-34). */
int sf_b200_bin_emit_bounded(const int32_t* order, const int64_t* offsets, const int32_t* tile_rect,
                             int64_t n, int64_t capacity, int32_t tiles_x, int32_t n_tiles,
                             int32_t* isect_ids, int32_t* tile_ranges, void* workspace,
                             size_t workspace_bytes, int32_t* overflow, void* stream);

/* Same result as sf_b200_bin_order, for callers that cannot allocate device memory
 * (for instance a host application that owns the whole device budget through its own
 * pool and lets no plugin call cudaMalloc).  No counterpart in the reference: it has
 * no device path at all.  The scratch is a static array inside the library (about 21
 * MB, held on every GPU that loads the library until exit); n is limited to
 * SF_B200_STATIC_MAX_GAUSSIANS and larger counts return SF_ERR_CAPACITY.  Calls share
 * that array: calls whose kernels overlap on the GPU race and must be serialised by
 * the caller.  The first call in each CUDA context resolves the array's device address
 * in that context; make it before any stream capture, and do not use the entry point
 * across a cudaDeviceReset in one process.  `stream` must belong to the current device
 * (SF_ERR_ARGUMENT otherwise).  Nothing is allocated or freed. */
#define SF_B200_STATIC_MAX_GAUSSIANS 1048576
/* bytes of the static array (checked against the ordering workspace of
 * SF_B200_STATIC_MAX_GAUSSIANS Gaussians, sf_b200_bin_workspace_bytes) */
#define SF_B200_STATIC_SCRATCH_BYTES (21u << 20)
int sf_b200_bin_order_static(const int32_t* tile_count, const uint32_t* depth_key, int64_t n,
                             int32_t* order, int64_t* offsets, void* stream);

/* 64-bit keys tile<<32 | depth bits of the sorted intersections (diagnostics/tests). */
int sf_b200_bin_keys(const int32_t* isect_ids, const int32_t* tile_ranges,
                     const uint32_t* depth_key, int32_t n_tiles, int64_t n_isect,
                     uint64_t* keys, void* stream);

/* ---- splat.alpha_composite@3 over dense [B,N,P] (reference.py:151-186; replaces
 * composite_cuda.cu:26-98 at the operator seam) -------------------------------------
 * Inputs alphas/depths [B,N,P], colors [B,N,3], normals [B,N,P,3]; outputs rgb
 * [B,P,3], alpha/znum/l1/l2/median [B,P], nnum [B,P,3], weights [B,N,P].  The
 * workspace (size from sf_b200_composite_workspace_bytes) carries the L1 factors and
 * the raw distortions from the forward call to the backward call. */
int sf_b200_composite_workspace_bytes(int64_t B, int64_t N, int64_t P, int32_t distortions,
                                      size_t* bytes);
int sf_b200_alpha_composite_forward(const float* alphas, const float* colors, const float* depths,
                                    const float* normals, int64_t B, int64_t N, int64_t P,
                                    int32_t distortions, float* rgb, float* alpha, float* znum,
                                    float* nnum, float* l1, float* l2, float* median,
                                    float* weights, void* workspace, size_t workspace_bytes,
                                    void* stream);
/* Any upstream adjoint may be NULL.  d_* outputs are overwritten. */
int sf_b200_alpha_composite_backward(const float* alphas, const float* colors, const float* depths,
                                     const float* normals, int64_t B, int64_t N, int64_t P,
                                     int32_t distortions, const float* weights,
                                     const void* workspace, size_t workspace_bytes,
                                     const float* grad_rgb, const float* grad_alpha,
                                     const float* grad_znum, const float* grad_nnum,
                                     const float* grad_l1, const float* grad_l2,
                                     const float* grad_median, const float* grad_weights,
                                     float* d_alphas, float* d_colors, float* d_depths,
                                     float* d_normals, void* stream);

/* ---- gaussian.opacity_field@1 (reference.py:194-222) -------------------------------
 * points [P,3], means [N,3], inverse_covariances [N,3,3], opacities [N], origins
 * [C,3] (C >= 1) -> field [P] (forward only).  Workspace from
 * sf_b200_opacity_field_workspace_bytes(N). */
int sf_b200_opacity_field_workspace_bytes(int64_t n_gaussians, size_t* bytes);
int sf_b200_opacity_field(const float* points, int64_t n_points, const float* means,
                          const float* inverse_covariances, const float* opacities,
                          int64_t n_gaussians, const float* origins, int32_t n_origins,
                          float* field, void* workspace, size_t workspace_bytes, void* stream);

/* The same field for large query sets (the GOF exporter's grid, exporters.py:42-102):
 * per view, Gaussians are binned into a cube map of face_cells x face_cells cells per
 * face around the origin by the cone of directions in which each can contribute more
 * than `cutoff` (0 < cutoff < 1); a query visits only its own direction's cell.
 * Contributions at or below `cutoff` are dropped, so the field differs from
 * sf_b200_opacity_field by at most about cutoff times the number of dropped terms.
 * No counterpart in the reference (its field is the brute-force loop).  Synchronises
 * the stream once per origin (candidate counts are read back).  max_pairs sizes the
 * per-view candidate lists in the workspace; *pairs_needed (host, may be NULL)
 * receives the largest per-view count; if that exceeds max_pairs the call returns
 * SF_ERR_CAPACITY and the caller retries with a larger workspace. */
int sf_b200_opacity_field_culled_workspace_bytes(int64_t n_points, int64_t n_gaussians,
                                                 int64_t max_pairs, int32_t face_cells,
                                                 size_t* bytes);
int sf_b200_opacity_field_culled(const float* points, int64_t n_points, const float* means,
                                 const float* inverse_covariances, const float* opacities,
                                 int64_t n_gaussians, const float* origins, int32_t n_origins,
                                 float cutoff, int32_t face_cells, float* field, void* workspace,
                                 size_t workspace_bytes, int64_t max_pairs, int64_t* pairs_needed,
                                 void* stream);
/* The same call, measured: *pairs_evaluated (a device int64, accumulated) receives the
 * number of (query, candidate) pairs whose contribution was evaluated, and *query_ms
 * (host, accumulated) the CUDA-event time of the per-view query kernels.  Used for
 * the field's roofline; the values equal sf_b200_opacity_field_culled's. */
int sf_b200_opacity_field_culled_stats(const float* points, int64_t n_points, const float* means,
                                       const float* inverse_covariances, const float* opacities,
                                       int64_t n_gaussians, const float* origins, int32_t n_origins,
                                       float cutoff, int32_t face_cells, float* field, void* workspace,
                                       size_t workspace_bytes, int64_t max_pairs, int64_t* pairs_needed,
                                       int64_t* pairs_evaluated, float* query_ms, void* stream);

/* A field plan for repeated evaluations against one Gaussian set and one origin set
 * (the GOF exporter evaluates the grid and then every bisection step against the same
 * scene, exporters.py:56-88): plan_build bins every view's Gaussians as
 * sf_b200_opacity_field_culled does and keeps all views' candidate lists in `plan`
 * (synchronises once per origin); plan_eval then evaluates a query set for all views
 * with one sort of its (view, cell) keys and no host synchronisation.  The values equal
 * sf_b200_opacity_field_culled's.  total_pairs and max_view_pairs size the lists: if
 * the scene needs more (needed[0] = all views' pairs, needed[1] = the largest view's,
 * host int64[2]) plan_build returns SF_ERR_CAPACITY and the caller retries.  plan_eval
 * takes the plan's sizes and origins again, and n_points * n_origins < 2^31. */
int sf_b200_opacity_field_plan_bytes(int64_t n_gaussians, int32_t n_origins, int32_t face_cells,
                                     int64_t total_pairs, int64_t max_view_pairs, size_t* bytes);
int sf_b200_opacity_field_plan_build(const float* means, const float* inverse_covariances,
                                     const float* opacities, int64_t n_gaussians,
                                     const float* origins, int32_t n_origins, float cutoff,
                                     int32_t face_cells, void* plan, size_t plan_bytes,
                                     int64_t total_pairs, int64_t max_view_pairs,
                                     int64_t* needed, void* stream);
int sf_b200_opacity_field_plan_query_bytes(int64_t n_points, int32_t n_origins, int32_t face_cells,
                                           size_t* bytes);
int sf_b200_opacity_field_plan_eval(const void* plan, int64_t n_gaussians, int32_t n_origins,
                                    int32_t face_cells, int64_t total_pairs, int64_t max_view_pairs,
                                    const float* origins, const float* points, int64_t n_points,
                                    float* field, void* workspace, size_t workspace_bytes,
                                    void* stream);

/* ---- small geometry operators -------------------------------------------------
 * camera.pixel_rays@1 (reference.py:49-56): K [3,3] -> rays [height, width, 3].
 * gaussian.ray_peak@1 (reference.py:38-46): means [N,3], inverse_covariances [N,3,3],
 *   origins [P,3], directions [P,3] -> t [N,P], response [N,P], normals [N,P,3].
 * geometry.depth_normals@1 (reference.py:59-83): depth [H,W], K [3,3] -> normals
 *   [H,W,3], valid [H,W] (uint8 0/1); the backward maps grad_normals to grad_depth
 *   and needs a workspace of 6*H*W floats. */
int sf_b200_pixel_rays(const float* K, int32_t width, int32_t height, float* rays, void* stream);
int sf_b200_ray_peak(const float* means, const float* inverse_covariances, int64_t n_gaussians,
                     const float* origins, const float* directions, int64_t n_rays, float* t,
                     float* response, float* normals, void* stream);
int sf_b200_depth_normals(const float* depth, const float* K, int32_t width, int32_t height,
                          float* normals, uint8_t* valid, void* stream);
int sf_b200_depth_normals_backward(const float* depth, const float* K, int32_t width, int32_t height,
                                   const float* grad_normals, float* grad_depth, float* workspace,
                                   void* stream);

/* ---- training-step operations --------------------------------------------------
 * matching.patch_zncc@1 (reference.py:225-236): a, b, mask [rows, S] (mask 0/1) ->
 *   correlation [rows] and valid [rows] (uint8); the backward maps grad_correlation
 *   [rows] to grad_a, grad_b [rows, S] (the mask is not differentiated).
 * densify_observe (studio/densification.py:18-43): where radii[i] > 0,
 *   gradient[i] += |(grad2d[i,0] * scale_x, grad2d[i,1] * scale_y)| and
 *   observations[i] += 1 (both accumulators updated in place).
 * normal_consistency (studio/losses.py:9-12, 45-53): depth [H,W], K [3,3], alpha [H,W],
 *   mask [H,W], and either normal_numerator [H,W,3] (loss term alpha - n_num . n_depth) or
 *   normals [H,W,3] (1 - n . n_depth; pass NULL for the other) -> loss (device float) and
 *   count (device int64) of the pixels where the depth normal is valid, alpha > 0.1 and
 *   mask > 0.  The backward takes the device scalar grad_loss, the same inputs and the
 *   same workspace (which keeps the depth normals between the calls) and writes
 *   grad_depth [H,W], grad_alpha [H,W] (zero in the normals case), grad_vector [H,W,3]
 *   (for whichever of normal_numerator / normals was given), plus a grad_normals [H,W,3]
 *   scratch.  Each may be NULL except grad_depth and grad_normals. */
/* gaussian.sh_ambiguity@1 (reference.py:116-117): coefficients [N,K,3] -> [N], the sum of
 * squares outside the DC band; the backward maps grad [N] to grad_coefficients [N,K,3].
 * gaussian.ray_color_variance@2 (reference.py:189-191), and @1 with batches = 1
 * (reference.py:120-122): weights [B,N,P], colors [B,N,3], composite [B,P,3] -> [B,P],
 * sum_n w |c - composite|^2 with weights and composite detached; the backward maps
 * grad [B,P] to grad_colors [B,N,3]. */
int sf_b200_sh_ambiguity(const float* coefficients, int64_t n, int32_t k, float* out, void* stream);
int sf_b200_sh_ambiguity_backward(const float* coefficients, int64_t n, int32_t k, const float* grad,
                                  float* grad_coefficients, void* stream);
int sf_b200_ray_color_variance(const float* weights, const float* colors, const float* composite,
                               int64_t batches, int64_t n, int64_t pixels, float* out, void* stream);
int sf_b200_ray_color_variance_backward(const float* weights, const float* colors, const float* composite,
                                        const float* grad, int64_t batches, int64_t n, int64_t pixels,
                                        float* grad_colors, void* stream);
int sf_b200_patch_zncc(const float* a, const float* b, const float* mask, int64_t rows, int32_t samples,
                       float epsilon, float* correlation, uint8_t* valid, void* stream);
int sf_b200_patch_zncc_backward(const float* a, const float* b, const float* mask, int64_t rows,
                                int32_t samples, float epsilon, const float* grad_correlation,
                                float* grad_a, float* grad_b, void* stream);
int sf_b200_densify_observe(const float* grad2d, const float* radii, int64_t n, float scale_x,
                            float scale_y, float* gradient, float* observations, void* stream);
int sf_b200_normal_consistency_workspace_bytes(int32_t width, int32_t height, size_t* bytes);
int sf_b200_normal_consistency(const float* depth, const float* K, int32_t width, int32_t height,
                               const float* alpha, const float* normal_numerator, const float* normals,
                               const float* mask, float* loss, int64_t* count, void* workspace,
                               size_t workspace_bytes, void* stream);
int sf_b200_normal_consistency_backward(const float* depth, const float* K, int32_t width, int32_t height,
                                        const float* alpha, const float* normal_numerator,
                                        const float* normals, const float* mask, const float* grad_loss,
                                        const int64_t* count, float* grad_depth, float* grad_alpha,
                                        float* grad_vector, float* grad_normals, void* workspace,
                                        size_t workspace_bytes, void* stream);

/* ---- GOF mesh extraction ---------------------------------------------------------
 * The device stages of GOFExporter.export (src/splatforge/studio/exporters.py:20-102)
 * and of marching_tetrahedra (src/splatforge/mesh/tetrahedra.py:34-109).  The caller
 * deduplicates the grid points and triangulates them on the host (as the reference
 * does), then runs, on one stream:
 *   mesh_count  -> host reads slot_offsets[n_cells] (S) and face_offsets[n_cells] (F)
 *   mesh_edges  -> host reads *n_edges (U, the unique crossing edges)
 *   binary_steps x (mesh_midpoints, field(midpoints) -> values, mesh_bisect)
 *   mesh_faces  -> host reads *n_kept
 * Points and vertices are float64 [*,3]; cells int32 [n_cells,4] (16-byte aligned);
 * values float64; inside and low_inside uint8 0/1.  n_edges and n_kept are DEVICE
 * int64 scalars.  With equal field values the output equals the reference's:
 * vertices [U,3] in ascending (low vertex, high vertex) edge order and faces [n_kept,3]
 * in cell order, oriented away from the inside vertices, degenerate ones removed.
 *
 * mesh_grid_points: exporters.py:20-38 without the deduplication: seed Gaussian
 *   chosen[i] -> points [n,9,3] (its centre, then the 8 corners of the extent-sigma box
 *   in itertools.product((-1,1), repeat=3) order) and radius [n] = max scale * extent
 *   (a float32 product).  scales are the activated (exponentiated) scales. */
int sf_b200_mesh_grid_points(const float* means, const float* quats, const float* scales,
                             const int32_t* chosen, int64_t n, double extent, double* points,
                             double* radius, void* stream);
int sf_b200_mesh_count_workspace_bytes(int64_t n_cells, size_t* bytes);
int sf_b200_mesh_count(const double* values, int64_t n_points, const int32_t* cells, int64_t n_cells,
                       double level, int32_t inside_greater, uint8_t* inside, int64_t* slot_offsets,
                       int64_t* face_offsets, void* workspace, size_t workspace_bytes, void* stream);
int sf_b200_mesh_edges_workspace_bytes(int64_t n_slots, size_t* bytes);
/* edge_ids [S] (unique edge of each crossing slot), pairs [S,2], low/high [S,3] and
 * low_inside [S]: the first U rows are the unique edges. */
int sf_b200_mesh_edges(const double* points, int64_t n_points, const int32_t* cells, int64_t n_cells,
                       const uint8_t* inside, const int64_t* slot_offsets, int64_t n_slots,
                       int32_t* edge_ids, int32_t* pairs, double* low, double* high,
                       uint8_t* low_inside, int64_t* n_edges, void* workspace,
                       size_t workspace_bytes, void* stream);
int sf_b200_mesh_midpoints(const double* low, const double* high, int64_t n_edges, double* midpoints,
                           void* stream);
int sf_b200_mesh_bisect(double* low, double* high, const uint8_t* low_inside, int64_t n_edges,
                        const double* values, double level, int32_t inside_greater, void* stream);
int sf_b200_mesh_faces_workspace_bytes(int64_t n_faces, size_t* bytes);
int sf_b200_mesh_faces(const double* points, const int32_t* cells, int64_t n_cells,
                       const uint8_t* inside, const int64_t* slot_offsets, const int32_t* edge_ids,
                       const double* low, const double* high, int64_t n_edges,
                       const int64_t* face_offsets, int64_t n_faces, double* vertices,
                       int64_t* faces, int64_t* n_kept, void* workspace, size_t workspace_bytes,
                       void* stream);

/* ---- raster forward (batched_renderer.py:169-338 + alpha_composite@3) -----------
 * One CTA per 16x16 tile.  Images are HWC float32: rgb/normals [H,W,3], the rest
 * [H,W].  pixel_state [H*W, SF_PIXEL_STATE_FLOATS] is kept for the backward pass.
 * L1 (settings->distortions & SF_DIST_L1) stores each pixel's contributing samples in
 * l1_samples, laid out [SF_L1_SAMPLE_FLOATS, l1_slots], each pixel's samples
 * contiguous: with l1_offsets == NULL pixel t*256+i (tile t, pixel i of the tile) owns
 * slots [(t*256+i)*l1_cap, +l1_cap) and l1_slots = n_tiles*256*l1_cap; otherwise pixel
 * p (row-major) owns [l1_offsets[p], l1_offsets[p+1]) and l1_slots = l1_offsets[H*W].
 * l1_needed (device int, may be NULL) receives the largest per-pixel sample count;
 * when it exceeds the capacity the caller reruns the forward with CSR offsets (the L1
 * result of this call is then incomplete).  counters (device int64[2], may be NULL)
 * accumulate the (pixel, Gaussian) pairs evaluated and the pairs that contributed. */
int sf_b200_raster_forward(const float* records, int64_t n, const int32_t* isect_ids,
                           const int32_t* tile_ranges, const sf_camera* camera,
                           const sf_settings* settings, float* rgb, float* alpha,
                           float* depth, float* normals, float* distortion_l1,
                           float* distortion_l2, float* median_depth, float* ray_color,
                           float* ambiguity, float* pixel_state, float* l1_samples,
                           int64_t l1_slots, const int64_t* l1_offsets, int32_t l1_cap,
                           int32_t* l1_needed, int64_t* counters, void* stream);

/* Per-pixel sample counts (pixel_state column) -> CSR offsets[H*W+1] (int64) for the
 * rerun of an L1 forward whose capacity was exceeded.  Each pixel's run is its count
 * rounded up to a multiple of 8 samples, so runs start 32-byte aligned.  workspace as
 * for binning with n = H*W. */
int sf_b200_l1_offsets(const sf_camera* camera, const float* pixel_state, int64_t* offsets,
                       void* workspace, size_t workspace_bytes, void* stream);

/* Sorts every pixel's stored samples by depth (a warp-level LSD radix sort in shared
 * memory), writes distortion_l1 and replaces each sample by the two factors the
 * backward pass needs.  max_samples bounds the per-pixel count (the l1_needed value of
 * the forward call); it sizes the shared-memory staging. */
int sf_b200_l1_resolve(const sf_camera* camera, const sf_settings* settings,
                       float* pixel_state, float* l1_samples, int64_t l1_slots,
                       const int64_t* l1_offsets, int32_t l1_cap, int32_t max_samples,
                       float* distortion_l1, void* stream);

/* ---- raster backward ---------------------------------------------------------------
 * Upstream image adjoints may each be NULL (zero).  grad_records [N,SF_RECORD_FLOATS]
 * and absgrad [N,2] are ACCUMULATED into (the caller zeroes them); grad_means2d [N,2]
 * is overwritten with the adjoint of the projected means.  error_word (device int,
 * may be NULL) is OR-ed with 1 when a pixel's recomputed contributing samples do not
 * match the count the forward pass stored (an internal consistency check). */
int sf_b200_raster_backward(const float* records, int64_t n, const int32_t* isect_ids,
                            const int32_t* tile_ranges, const sf_camera* camera,
                            const sf_settings* settings, const float* pixel_state,
                            const float* l1_samples, int64_t l1_slots,
                            const int64_t* l1_offsets, int32_t l1_cap,
                            const float* grad_rgb, const float* grad_alpha,
                            const float* grad_depth, const float* grad_normals,
                            const float* grad_l1, const float* grad_l2,
                            const float* grad_median, const float* grad_ray_color,
                            const float* grad_ambiguity, float* grad_records,
                            float* grad_means2d, float* absgrad, int32_t* error_word,
                            void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SPLATFORGE_B200_H */
