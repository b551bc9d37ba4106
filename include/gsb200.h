/*
 * gsb200.h -- C ABI of libgsb200.so, the B200 (sm_100a) Gaussian-splat render + L1/SSIM loss.
 *
 * Plain C: device pointers, sizes and a cudaStream_t passed as void*.  No torch types.
 * Every entry point is stream-ordered, allocates nothing (the caller owns all device memory,
 * workspaces included) and returns a gsb_status.  Status codes never trap the device: kernels
 * that can fail record a code in the caller's workspace, read back by gsb_read_status().
 *
 * The stages replace the reference's Python render path (nbardy/dynaworld, src/train):
 *
 *   gsb_depth_order      <- the stable argsort by camera z of
 *                           renderers/common.py:190-195 (project_gaussians_2d_batch)
 *   gsb_preprocess_fwd   <- renderers/common.py:149-231 (projection, EWA covariance,
 *                           near-plane mask) and, per view, the lens models of
 *                           renderers/projection.py:164-330 (project_gaussians_2d_camera[_batch]),
 *                           plus raw-parameter activation / SH / time offset
 *                           (the model head of gs_models/blocks.py:172-186), and the per-Gaussian
 *                           tile bounds of renderers/tiled.py:7-28
 *   gsb_bin              <- renderers/tiled.py:31-71 (build_tile_assignments: tile lists in
 *                           (tile, depth) order)
 *   gsb_raster_fwd       <- renderers/dense.py:208-236 (render_pytorch_3dgs_batch blend) and
 *                           renderers/tiled.py:162-198 (tile-local variant)
 *   gsb_raster_bwd,
 *   gsb_preprocess_bwd   <- torch autograd through the two above (dense.py / common.py)
 *   gsb_loss_fwd_bwd     <- losses.py:13-85 (reconstruction_loss_per_image, standard_gs)
 *   gsb_scale_planes     <- the upstream-gradient product autograd applies to the loss
 *
 * The Metal scaffold of the reference exposes the same split as a torch op pair
 * (third_party/fast-mac-gsplat-scaffold/csrc/bindings.cpp:44-52).
 */
#ifndef GSB200_H
#define GSB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GSB_API __attribute__((visibility("default")))

typedef enum gsb_status {
  GSB_OK = 0,
  GSB_ERR_SHAPE = 1,        /* inconsistent or unsupported sizes */
  GSB_ERR_WORKSPACE = 2,    /* workspace too small: the needed size was written back */
  GSB_ERR_KEY_OVERFLOW = 3, /* more (tile, Gaussian) pairs than the 2^30 a call supports */
  GSB_ERR_NONFINITE = 4,    /* non-finite projected values were counted (see gsb_read_status) */
  GSB_ERR_TIMEOUT = 5,      /* a bounded device-side wait gave up */
  GSB_ERR_CUDA = 6,         /* a CUDA runtime call failed (launch error etc.) */
  GSB_ERR_ARG = 7,          /* NULL pointer or bad option value */
  GSB_ERR_CAPACITY = 8      /* gsb_bin: more pairs than the capacity given (outputs invalid) */
} gsb_status;

/* Scene flags (gsb_scene.flags). */
#define GSB_SCENE_RAW 0x1u      /* scales are log-scales, quats are normalised, opacities are
                                   logits, colors are SH coefficients (else: activated values as
                                   the reference's render call takes them) */
#define GSB_SCENE_VELOCITY 0x2u /* means_t = means + t_view * velocity */
#define GSB_SCENE_SH_CLAMP 0x4u /* rgb = max(SH(dir) + 0.5, 0) (raw mode only) */
#define GSB_SCENE_BANK 0x8u     /* dynamic Gaussian bank (activated mode only, no velocity): see
                                   gsb_scene.bank_mu */
#define GSB_BANK_MAX_BASIS 16   /* temporal basis functions a bank may have */
#define GSB_SCENE_HEAD 0x10u    /* the decoder head's raw outputs (GaussianParameterHeads.forward,
                                   gs_models/blocks.py:172-186), activated here:
                                     means  = (tanh(x) xy_extent, tanh(y) xy_extent,
                                               sigmoid(z) z_extent + z_min)
                                     scales = exp(raw) scale_init, quats = raw / max(|raw|, 1e-12),
                                     opacities = sigmoid(raw), colors = sigmoid(raw) [S,G,3]
                                   (gsb_scene.head_*; not with RAW or BANK; velocity allowed) */

/* Render flags (gsb_options.flags). */
#define GSB_RENDER_TILED_COMPAT 0x1u /* tiled.py bounds (bound_scale, 1/255 threshold) and
                                        tile-local (1+eps) products, no cutoff, no early stop */
#define GSB_RENDER_DEPTH 0x2u        /* write depth = sum_i w_i z_i */
#define GSB_RENDER_NO_ELLIPSE 0x4u   /* exact mode: keep every tile of the bounding box */
#define GSB_RENDER_NO_CLAMP 0x8u     /* image = sum w c + (1 - clamp(sum w, 0, 1)) bg, not clamped
                                        to [0, 1] (the 2-D kernels' output, gsplat_kernels.metal:
                                        199-201) */

/* Gaussians: n_sets sets of n_gaussians each; view b draws on set b / views_per_set. */
typedef struct gsb_scene {
  int32_t n_sets;
  int32_t n_gaussians;
  int32_t sh_degree;      /* raw mode: 0..3; activated mode: ignored (colors are rgb) */
  uint32_t flags;         /* GSB_SCENE_* */
  const float* means;     /* [S,G,3] */
  const float* scales;    /* [S,G,3] linear (activated) or log-scales (raw) */
  const float* quats;     /* [S,G,4] (r,i,j,k); raw mode normalises them */
  const float* opacities; /* [S,G]   opacity in [0,1] (activated) or logits (raw) */
  const float* colors;    /* [S,G,3] rgb (activated) or SH [S,G,(d+1)^2,3] (raw) */
  const float* velocity;  /* [S,G,3] with GSB_SCENE_VELOCITY, else NULL */
  /* Dynamic bank (GSB_SCENE_BANK), the evaluation of
     gs_models/dynamic_video_token_gs_implicit_camera.py:1206-1224 (_eval_dynamic_bank) fused into
     the projection.  Gaussians g < bank_first are static; for g >= bank_first, d = g - bank_first
     and phi = gsb_views.basis[view] (M values):
       mean_t    = means + sum_m phi_m bank_mu[d,m]
       quat_t    = normalize(quats (x) axis_angle_quat(sum_m phi_m bank_rot[d,m]))   (:828-852)
       opacity_t = sigmoid(logit(clamp(opacities, 1e-6, 1 - 1e-6)) + sum_m phi_m bank_alpha[d,m])
     scales and colors as given (per set: arrays of S * (G - bank_first) rows). */
  const float* bank_mu;    /* [S, G - bank_first, M, 3] */
  const float* bank_rot;   /* [S, G - bank_first, M, 3] axis-angle, radians */
  const float* bank_alpha; /* [S, G - bank_first, M]    opacity-logit offsets */
  int32_t bank_first;      /* 0 <= bank_first <= G */
  int32_t bank_basis;      /* M, 1 .. GSB_BANK_MAX_BASIS */
  /* Decoder-head constants (GSB_SCENE_HEAD), the GaussianParameterHeads attributes of the same
     names (blocks.py:120-123): z_extent = z_max - z_min. */
  float head_xy_extent;
  float head_z_min;
  float head_z_extent;
  float head_scale_init;
} gsb_scene;

/* Lens models (gsb_views.lens_models), the CameraSpec lens_model values of camera.py:7-31. */
#define GSB_LENS_PINHOLE 0            /* common.py:149-231 projection */
#define GSB_LENS_RADIAL_TANGENTIAL 1  /* distortion k1, k2, p1, p2, k3 (projection.py:93-116) */
#define GSB_LENS_OPENCV_FISHEYE 2     /* distortion k1, k2, k3, k4, 0 (projection.py:119-161) */

/* Views (cameras). */
typedef struct gsb_views {
  int32_t n_views;
  int32_t views_per_set;
  int32_t height;
  int32_t width;
  const float* intrinsics;      /* [B,4] fx, fy, cx, cy (device) */
  const float* camera_to_world; /* [B,4,4] row-major, camera +z is the optical axis (device) */
  const float* times;           /* [B] or NULL (device) */
  const int32_t* lens_models;   /* [B] GSB_LENS_* or NULL: every view pinhole (device) */
  const float* distortion;      /* [B,5] coefficients (zero-padded), read for non-pinhole views */
  const float* basis;           /* [B,M] temporal basis of each view's time (GSB_SCENE_BANK; the
                                   reference's _temporal_basis, :806-825), else NULL */
} gsb_views;

typedef struct gsb_options {
  int32_t tile_size;              /* 8 or 16 */
  uint32_t flags;                 /* GSB_RENDER_* */
  float near_plane;               /* reference default 1e-4 (common.py:3) */
  float alpha_clamp;              /* 0.99 (dense.py:220) */
  float alpha_cutoff;             /* exact mode: pairs with alpha below it count as alpha 0 */
  float transmittance_threshold;  /* exact mode: a pixel stops once T falls below it */
  float eps;                      /* 1e-6 (dense.py:225) */
  float pixel_center;             /* 0.0 (common.py:13-19) */
  float background[3];            /* (1,1,1) (dense.py:231) */
  float bound_scale;              /* tiled compat: 3.0 (tiled.py:7) */
  float tiled_alpha_threshold;    /* tiled compat: 1/255 (tiled.py:7) */
  int32_t backward_segments;      /* 1, 2 or 4: the reverse blend walks every tile list as that
                                     many independent pieces (needs gsb_raster_checkpoint_floats
                                     of checkpoints from the forward); 0: the library's choice for
                                     the grid size.  Results do not depend on it. */
} gsb_options;

/* Gradients of the scene parameters (device, shapes as gsb_scene; NULL entries are skipped). */
typedef struct gsb_scene_grads {
  float* means;
  float* scales;
  float* quats;
  float* opacities;
  float* colors;
  float* velocity;
  float* bank_mu;    /* GSB_SCENE_BANK: shapes as gsb_scene */
  float* bank_rot;
  float* bank_alpha;
} gsb_scene_grads;

/* Gradients of the cameras (device; NULL entries are skipped; outputs are overwritten). */
typedef struct gsb_camera_grads {
  float* intrinsics;       /* [B,4] d/d(fx, fy, cx, cy) */
  float* camera_to_world;  /* [B,4,4] rotation and centre entries (bottom row zero) */
  float* distortion;       /* [B,5] (zero for pinhole views and unused coefficients) */
} gsb_camera_grads;

typedef struct gsb_loss_options {
  int32_t type;          /* 0 standard_gs, 1 l1, 2 mse, 3 l1_mse */
  int32_t window_size;   /* odd, 3..31; reference 11 */
  int32_t window;        /* 0 box (reference), 1 gaussian */
  int32_t dssim_half;    /* 1: (1-SSIM)/2 as the reference, 0: (1-SSIM) */
  float l1_weight;       /* 0.8 */
  float dssim_weight;    /* 0.2 */
  float mse_weight;      /* 0.2 */
  float c1;              /* 1e-4 */
  float c2;              /* 9e-4 */
  float sigma;           /* gaussian window sigma, 1.5 */
} gsb_loss_options;

/* Size of one projected record (floats), of one 2-D gradient record (floats), and of the
   per-pixel state the backward reads.  A record is mx, my, A, B, C, opacity, z, tau, r, g, b, 0,
   then the ellipse's culling extents: half widths ex, ey of {q <= tau} (with margins; +inf for a
   degenerate conic) and the slopes -B/(2C), -B/(2A) of its extreme points. */
#define GSB_RECORD_FLOATS 16
#define GSB_GRAD2D_FLOATS 10

/* ---- library ------------------------------------------------------------------------------ */
GSB_API const char* gsb_version(void);
/* Number of kernels this library has launched in this process (all devices, all threads). */
GSB_API uint64_t gsb_kernel_launches(void);
GSB_API const char* gsb_status_string(int status);
/* Reads the device status word of a workspace (after the stream is synchronised by the caller).
   Returns GSB_OK or the first error recorded by a kernel using that workspace. */
GSB_API gsb_status gsb_read_status(const void* workspace, int* status_out, void* stream);

/* ---- stage 1: per-view stable depth order (common.py:190-195) ----------------------------- */
GSB_API size_t gsb_depth_order_workspace(const gsb_scene* scene, const gsb_views* views);
/* sorted_ids[b*G + r] = index of the r-th nearest Gaussian of view b (ties by index);
   rank_of[b*G + g] = its inverse. */
GSB_API gsb_status gsb_depth_order(const gsb_scene* scene, const gsb_views* views,
                                   int32_t* sorted_ids, int32_t* rank_of,
                                   void* workspace, size_t workspace_bytes, void* stream);

/* ---- stage 2: projection in depth order, tile bounds, pair count prefix ------------------- */
GSB_API size_t gsb_preprocess_workspace(const gsb_views* views, int32_t n_gaussians);
/* records[(b*G + r)*GSB_RECORD_FLOATS ..] = mx, my, A, B, C, opacity, z, tau, r, g, b, 0, then
   the culling extents, for the r-th nearest Gaussian of view b (A, B, C: inv_cov00,
   inv_cov01+inv_cov10, inv_cov11; tau: the q above which alpha < alpha_cutoff).  tile_rects[(b*G + r)*4 ..] = tx0, ty0, tx1, ty1 (inclusive;
   empty when tx0 > tx1).  pair_offsets[B*G + 1]: exclusive prefix of the per-Gaussian pair
   counts; pair_offsets[B*G] is the total (<= 2^30, else GSB_ERR_KEY_OVERFLOW at gsb_bin).
   cov2d_out ([B*G*3] c00, c01, c11 in depth order) may be NULL.  Non-finite projected values
   (NaN / inf parameters, overflowing scales) are counted on the device: the workspace's first
   three int32 words then hold GSB_ERR_NONFINITE, the first offending b*G + g, and the count (read
   them after the stream is synchronised; gsb_read_status gives the first).  Such a Gaussian is
   never blended. */
GSB_API gsb_status gsb_preprocess_fwd(const gsb_scene* scene, const gsb_views* views,
                                      const gsb_options* opts, const int32_t* rank_of,
                                      float* records, int32_t* tile_rects, uint32_t* pair_offsets,
                                      float* cov2d_out, void* workspace, size_t workspace_bytes,
                                      void* stream);

/* ---- stage 3: pair keys, radix sort by (view, tile), tile ranges (tiled.py:31-71) ---------- */
GSB_API size_t gsb_bin_workspace(const gsb_views* views, const gsb_options* opts,
                                 int32_t n_gaussians, uint32_t n_pairs);
/* n_pairs: capacity of sorted_keys, at least the pair count pair_offsets[B*G] (passing the count
   itself is the usual call).  The count is read on the device, so the stage (and the raster after
   it) can be queued before the count reaches the host, with a capacity guessed from earlier
   frames; a count above the capacity records GSB_ERR_CAPACITY (gsb_read_status), writes nothing
   past the capacity and leaves the outputs invalid: call again with the count.
   sorted_keys[count]: ((view*n_tiles + tile) << 32) | depth_rank, ascending.
   tile_ranges[B*n_tiles*2]: [start, end) of each tile's run in sorted_keys.
   tile_order[B*n_tiles] (may be NULL): view*n_tiles + tile, longest lists first -- the launch
   order the raster stages use so that the heaviest tiles do not finish last. */
GSB_API gsb_status gsb_bin(const gsb_views* views, const gsb_options* opts, int32_t n_gaussians,
                           const float* records, const int32_t* tile_rects,
                           const uint32_t* pair_offsets, uint32_t n_pairs,
                           uint64_t* sorted_keys, uint32_t* tile_ranges, uint32_t* tile_order,
                           void* workspace, size_t workspace_bytes, void* stream);

/* ---- stage 4: front-to-back blend (dense.py:208-236) -------------------------------------- */
/* Floats of per-pixel checkpoints the reverse blend needs for opts->backward_segments (0: none;
   then pixel_ckpt may be NULL). */
GSB_API size_t gsb_raster_checkpoint_floats(const gsb_views* views, const gsb_options* opts);
/* image [B,3,H,W] (clamped), alpha [B,H,W] = sum of weights, depth [B,H,W] or NULL,
   pixel_t [B,H,W], pixel_state [B,H,W] and pixel_ckpt: the per-pixel state gsb_raster_bwd needs.
   tile_order: gsb_bin's launch order, or NULL for (view, tile) order. */
GSB_API gsb_status gsb_raster_fwd(const gsb_views* views, const gsb_options* opts,
                                  int32_t n_gaussians, const float* records,
                                  const uint64_t* sorted_keys, const uint32_t* tile_ranges,
                                  const uint32_t* tile_order,
                                  float* image, float* alpha, float* depth,
                                  float* pixel_t, uint32_t* pixel_state, float* pixel_ckpt,
                                  void* stream);

/* ---- stage 5: fused L1 + SSIM loss and its gradient (losses.py:13-85) --------------------- */
GSB_API size_t gsb_loss_workspace(int32_t n_images);
/* loss[B]; dpred (may be NULL): d loss[b] / d pred for a unit upstream gradient. */
GSB_API gsb_status gsb_loss_fwd_bwd(const gsb_loss_options* lopts, int32_t n_images,
                                    int32_t channels, int32_t height, int32_t width,
                                    const float* pred, const float* target, float* loss,
                                    float* dpred, void* workspace, size_t workspace_bytes,
                                    void* stream);
/* Allocation-free variant of gsb_loss_fwd_bwd.  No counterpart in the reference: it exists for
   callers that cannot allocate device memory at all -- typically a plugin or language binding
   that is handed its input and output buffers by a host framework owning the device allocator.
   Same results as gsb_loss_fwd_bwd; its scratch (three double sums and one flag per image) is a
   fixed array inside the library, about 112 KiB, held by every GPU that loads the library until
   the process exits.  Limit: n_images <= GSB_LOSS_NOALLOC_MAX_IMAGES, larger batches return
   GSB_ERR_SHAPE before anything is launched.  The first call on each device looks up the array's
   device address with that device current and caches it: make that first call before any stream
   capture.  The cached address belongs to the device's primary context (the one the CUDA runtime
   and torch use): it stays valid while that context lives, so do not call this entry after
   cudaDeviceReset or from a context of your own made current with the driver API.  Every call
   uses the same array; each call clears the sums it needs, but calls that overlap on the GPU
   (several streams or host threads at once) race on it and give wrong results, so order them on
   one stream. */
#define GSB_LOSS_NOALLOC_MAX_IMAGES 4096
GSB_API gsb_status gsb_loss_fwd_bwd_noalloc(const gsb_loss_options* lopts, int32_t n_images,
                                            int32_t channels, int32_t height, int32_t width,
                                            const float* pred, const float* target, float* loss,
                                            float* dpred, void* stream);
/* out[b, ...] = scale[b] * in[b, ...] for n_images (<= 65535, else GSB_ERR_SHAPE) planes of
   plane_elems floats (in == out ok). */
GSB_API gsb_status gsb_scale_planes(const float* in, const float* scale, float* out,
                                    int32_t n_images, int64_t plane_elems, void* stream);

/* ---- stage 6: reverse blend, per-(view, Gaussian) 2-D gradients --------------------------- */
/* grad2d[(b*G + r)*10 ..] = dL/d(mx, my, A, B, C, opacity, r, g, b, z) of the r-th nearest
   Gaussian of view b; zeroed by the call; grad2d 8-byte aligned (GSB_ERR_ARG otherwise).
   d_alpha, d_depth, view_scale may be NULL (d_depth is read only with GSB_RENDER_DEPTH); opts
   and pixel_ckpt as given to gsb_raster_fwd. */
GSB_API gsb_status gsb_raster_bwd(const gsb_views* views, const gsb_options* opts,
                                  int32_t n_gaussians, const float* records,
                                  const uint64_t* sorted_keys, const uint32_t* tile_ranges,
                                  const uint32_t* tile_order,
                                  const float* pixel_t, const uint32_t* pixel_state,
                                  const float* pixel_ckpt,
                                  const float* d_image, const float* d_alpha,
                                  const float* d_depth, const float* view_scale,
                                  float* grad2d, void* stream);

/* ---- stage 7: chain rule to the scene parameters (common.py:149-231 backward) ------------- */
/* Gradients are summed over the views that share a set and overwrite the outputs. */
GSB_API gsb_status gsb_preprocess_bwd(const gsb_scene* scene, const gsb_views* views,
                                      const gsb_options* opts, const int32_t* rank_of,
                                      const float* grad2d, gsb_scene_grads* grads, void* stream);
/* gsb_preprocess_bwd for the Gaussians (set * G + index) [first, first + count) only: writes
   their rows of the outputs and nothing else, so the rows can be handed to a collective while the
   next range is computed (no counterpart in the reference: its autograd has no such split). */
GSB_API gsb_status gsb_preprocess_bwd_range(const gsb_scene* scene, const gsb_views* views,
                                            const gsb_options* opts, const int32_t* rank_of,
                                            const float* grad2d, gsb_scene_grads* grads,
                                            int64_t first, int64_t count, void* stream);

/* ---- stage 7b: camera gradients (torch autograd through common.py / projection.py into the
   camera tensors, which the implicit-camera models of gs_models/implicit_camera.py:146-262
   train through the render call) ---------------------------------------------------------- */
/* Per view, summed over its Gaussians: d/d intrinsics, d/d camera_to_world (rotation entries and
   the centre column), d/d lens distortion.  Launch only when a camera tensor needs gradients. */
GSB_API gsb_status gsb_camera_bwd(const gsb_scene* scene, const gsb_views* views,
                                  const gsb_options* opts, const int32_t* rank_of,
                                  const float* grad2d, gsb_camera_grads* grads, void* stream);

/* ---- already-projected 2-D Gaussians -------------------------------------------------------
 * The reference's 2-D rasterizer contracts, on the same bin and raster stages as the 3-D path:
 *   conic  <- third_party/fast-mac-gsplat-scaffold/torch_gsplat_bridge/rasterize.py:93-126
 *             (rasterize_projected_gaussians, called by src/train/renderers/fast_mac.py:253,301)
 *             and third_party/raw-metal-mlx-gsplat/mlx_projected_gaussian_rasterizer.py:787;
 *             kernels gsplat_kernels.metal:40-205
 *   packed <- the [mean, axis, sigma, opacity] rows of src/train/renderers/taichi.py:107-176 and
 *             src/benchmarks/splat_renderer_accuracy.py:262-305 (torch_reference_rasterize)
 * Order: gsb_splats2d_order -> gsb_splats2d_preprocess -> gsb_bin -> gsb_raster_fwd, and
 * gsb_raster_bwd -> gsb_splats2d_preprocess_bwd; the bin and raster stages take a gsb_views with
 * n_views = batch, views_per_set = 1 and the image size (intrinsics / camera_to_world unused, may
 * be NULL there).  Options that give the reference kernels' semantics: eps 0, pixel_center 0.5,
 * alpha_cutoff = alpha_threshold, transmittance_threshold as given (1 - saturate_threshold for
 * the packed contract), alpha_clamp 0.99, GSB_RENDER_NO_CLAMP. */
#define GSB_SPLATS2D_CONIC 0  /* means [B,G,2], conics [B,G,3] (a, b, c): q = a dx^2 + 2 b dx dy
                                 + c dy^2, opacities [B,G] */
#define GSB_SPLATS2D_PACKED 1 /* packed [B,G,7]: mean x, y, unit axis x, y, sigma along the axis,
                                 sigma across it, opacity */
typedef struct gsb_splats2d {
  int32_t n_views;        /* B: independent images */
  int32_t n_gaussians;    /* G per image */
  int32_t format;         /* GSB_SPLATS2D_* */
  int32_t reserved;
  const float* means;     /* conic format */
  const float* conics;    /* conic format */
  const float* opacities; /* conic format */
  const float* packed;    /* packed format */
  const float* colors;    /* [B,G,3] */
  const float* depths;    /* [B,G] blend order (ascending, ties by index), or NULL: index order */
} gsb_splats2d;

typedef struct gsb_splats2d_grads { /* NULL entries are skipped; outputs are overwritten */
  float* means;
  float* conics;    /* d/d(a, b, c) with b the half cross coefficient */
  float* opacities;
  float* packed;    /* [B,G,7] */
  float* colors;
} gsb_splats2d_grads;

GSB_API size_t gsb_splats2d_order_workspace(const gsb_splats2d* splats);
/* As gsb_depth_order, keyed by the given depths. */
GSB_API gsb_status gsb_splats2d_order(const gsb_splats2d* splats, int32_t* sorted_ids,
                                      int32_t* rank_of, void* workspace, size_t workspace_bytes,
                                      void* stream);
GSB_API size_t gsb_splats2d_preprocess_workspace(const gsb_splats2d* splats);
/* As gsb_preprocess_fwd: records (z = the given depth), tile_rects and pair_offsets in blend
   order.  Conic format also drops Gaussians with a c - b^2 <= 1e-8 (gsplat_kernels.metal:57-59). */
GSB_API gsb_status gsb_splats2d_preprocess(const gsb_splats2d* splats, int32_t height,
                                           int32_t width, const gsb_options* opts,
                                           const int32_t* rank_of, float* records,
                                           int32_t* tile_rects, uint32_t* pair_offsets,
                                           void* workspace, size_t workspace_bytes, void* stream);
/* grad2d (gsb_raster_bwd) -> gradients of the caller's parameters. */
GSB_API gsb_status gsb_splats2d_preprocess_bwd(const gsb_splats2d* splats, const int32_t* rank_of,
                                               const float* grad2d, gsb_splats2d_grads* grads,
                                               void* stream);

/* ---- utility: the library's radix sort on its own (tests, benchmarks) --------------------- */
GSB_API size_t gsb_radix_sort_workspace(uint32_t n, int key_bytes, int with_values);
/* Stable LSD sort of n keys by bits [bit_lo, bit_hi); keys are uint32 (key_bytes 4) or uint64
   (key_bytes 8); values (uint32) may be NULL. Input buffers are left unchanged. */
GSB_API gsb_status gsb_radix_sort(const void* keys_in, void* keys_out, const uint32_t* values_in,
                                  uint32_t* values_out, uint32_t n, int key_bytes, int bit_lo,
                                  int bit_hi, void* workspace, size_t workspace_bytes,
                                  void* stream);
/* Test hook for the bounded look-back waits of the radix sort (no counterpart in the reference):
   one 8-bit pass over n (> 2048) uint32 keys in which the first partition never runs, so the
   partition after it waits for a predecessor that never publishes.  The wait gives up after
   spin_limit polls (0 means 1) and records GSB_ERR_TIMEOUT (gsb_read_status on the workspace);
   every kernel returns and nothing is written outside keys_out[0, n).  keys_out is not sorted.
   Workspace: gsb_radix_sort_workspace(n, 4, 0) bytes. */
GSB_API gsb_status gsb_debug_sort_lookback_timeout(const uint32_t* keys_in, uint32_t* keys_out,
                                                   uint32_t n, uint32_t spin_limit,
                                                   void* workspace, size_t workspace_bytes,
                                                   void* stream);

#ifdef __cplusplus
}
#endif
#endif /* GSB200_H */
