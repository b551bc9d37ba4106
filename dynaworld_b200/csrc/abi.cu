// extern "C" entry points of libgsb200.so (declared in include/gsb200.h).
#include <atomic>
#include <cmath>
#include <cstring>

#include "gsb_common.cuh"
#include "gsb_internal.h"

namespace gsb {

static std::atomic<unsigned long long> g_launches{0};
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int bits_for(uint64_t count) {
  int b = 0;
  while ((uint64_t(1) << b) < count) ++b;
  return b;
}

// The float nearest 1 / f0 (searched within four ulp) whose float product with f0 is exactly 1;
// *found = 0 and plain 1 / f0 when there is none.  With it the blend multiplies S by f * inv_f0
// for a skipped pair (alpha 0, f = f0) and keeps S to the bit.
static float unit_inverse(float f0, int* found) {
  volatile float num = 1.0f;
  const float inv = num / f0;
  float cand[9] = {inv};
  float up = inv, down = inv;
  for (int d = 0; d < 4; ++d) {
    up = std::nextafter(up, 2.0f);
    down = std::nextafter(down, 0.0f);
    cand[1 + 2 * d] = up;
    cand[2 + 2 * d] = down;
  }
  for (float c : cand) {
    volatile float prod = f0 * c;
    if (prod == 1.0f) {
      *found = 1;
      return c;
    }
  }
  *found = 0;
  return inv;
}

RenderConsts make_consts(const gsb_views& v, const gsb_options& o) {
  RenderConsts rc{};
  rc.tile = o.tile_size;
  rc.tiles_x = (v.width + o.tile_size - 1) / o.tile_size;
  rc.tiles_y = (v.height + o.tile_size - 1) / o.tile_size;
  rc.n_tiles = rc.tiles_x * rc.tiles_y;
  rc.compat = (o.flags & GSB_RENDER_TILED_COMPAT) != 0;
  rc.depth = (o.flags & GSB_RENDER_DEPTH) != 0;
  rc.ellipse = (o.flags & GSB_RENDER_NO_ELLIPSE) == 0;
  rc.clamp_image = (o.flags & GSB_RENDER_NO_CLAMP) == 0;
  rc.near_plane = o.near_plane;
  rc.alpha_clamp = o.alpha_clamp;
  rc.alpha_cutoff = rc.compat ? 0.0f : o.alpha_cutoff;
  rc.t_threshold = rc.compat ? 0.0f : o.transmittance_threshold;
  rc.eps = o.eps;
  rc.pixel_center = o.pixel_center;
  for (int k = 0; k < 3; ++k) rc.bg[k] = o.background[k];
  rc.bound_scale = o.bound_scale;
  rc.tiled_threshold = o.tiled_alpha_threshold;
  volatile float one = 1.0f;
  rc.f0 = one + o.eps;  // fl32(1 + eps)
  // T_i = F0^pos_i * S_i in both modes; pos is the depth rank (exact) or the list index (compat)
  rc.log2_f0 = float(std::log2(double(rc.f0)));
  rc.inv_f0 = unit_inverse(rc.f0, &rc.unit_inv);
  return rc;
}

static cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

static gsb_status check_views(const gsb_views* v) {
  if (!v || !v->intrinsics || !v->camera_to_world) return GSB_ERR_ARG;
  if (v->lens_models && !v->distortion) return GSB_ERR_ARG;
  if (v->n_views <= 0 || v->height <= 0 || v->width <= 0 || v->views_per_set <= 0) return GSB_ERR_SHAPE;
  return GSB_OK;
}

// The bin and raster stages read only the batch and image sizes (no cameras).
static gsb_status check_frame(const gsb_views* v) {
  if (!v) return GSB_ERR_ARG;
  if (v->n_views <= 0 || v->height <= 0 || v->width <= 0) return GSB_ERR_SHAPE;
  return GSB_OK;
}

static gsb_status check_splats2d(const gsb_splats2d* s) {
  if (!s || !s->colors) return GSB_ERR_ARG;
  if (s->format == GSB_SPLATS2D_CONIC) {
    if (!s->means || !s->conics || !s->opacities) return GSB_ERR_ARG;
  } else if (s->format == GSB_SPLATS2D_PACKED) {
    if (!s->packed) return GSB_ERR_ARG;
  } else {
    return GSB_ERR_ARG;
  }
  if (s->n_views <= 0 || s->n_gaussians <= 0) return GSB_ERR_SHAPE;
  if (uint64_t(s->n_views) * uint64_t(s->n_gaussians) >= (uint64_t(1) << 30)) return GSB_ERR_SHAPE;
  return GSB_OK;
}

static gsb_status check_scene(const gsb_scene* s, const gsb_views* v) {
  if (!s || !s->means || !s->scales || !s->quats || !s->opacities || !s->colors) return GSB_ERR_ARG;
  if ((s->flags & GSB_SCENE_VELOCITY) && !s->velocity) return GSB_ERR_ARG;
  if (s->n_sets <= 0 || s->n_gaussians <= 0) return GSB_ERR_SHAPE;
  if ((v->n_views - 1) / v->views_per_set >= s->n_sets) return GSB_ERR_SHAPE;
  if ((s->flags & GSB_SCENE_RAW) && (s->sh_degree < 0 || s->sh_degree > 3)) return GSB_ERR_ARG;
  if (uint64_t(v->n_views) * uint64_t(s->n_gaussians) >= (uint64_t(1) << 30)) return GSB_ERR_SHAPE;
  if (s->flags & GSB_SCENE_HEAD) {  // the head's raw outputs: its own activation, rgb colours
    if (s->flags & (GSB_SCENE_RAW | GSB_SCENE_BANK)) return GSB_ERR_ARG;
    if (!(s->head_scale_init > 0.0f) || !(s->head_xy_extent >= 0.0f) || !(s->head_z_extent >= 0.0f))
      return GSB_ERR_ARG;
  }
  if (s->flags & GSB_SCENE_BANK) {  // activated values only, one motion model per scene
    if (s->flags & (GSB_SCENE_RAW | GSB_SCENE_VELOCITY)) return GSB_ERR_ARG;
    if (!s->bank_mu || !s->bank_rot || !s->bank_alpha || !v->basis) return GSB_ERR_ARG;
    if (s->bank_basis < 1 || s->bank_basis > GSB_BANK_MAX_BASIS) return GSB_ERR_ARG;
    if (s->bank_first < 0 || s->bank_first > s->n_gaussians) return GSB_ERR_SHAPE;
  }
  return GSB_OK;
}

static gsb_status check_opts(const gsb_options* o) {
  if (!o) return GSB_ERR_ARG;
  if (o->tile_size != 8 && o->tile_size != 16) return GSB_ERR_ARG;
  if (!(o->near_plane > 0.0f)) return GSB_ERR_ARG;
  if (!(o->alpha_cutoff >= 0.0f) || !(o->transmittance_threshold >= 0.0f) || !(o->eps >= 0.0f)) return GSB_ERR_ARG;
  const int seg = o->backward_segments;
  if (seg != 0 && seg != 1 && seg != 2 && seg != 4) return GSB_ERR_ARG;
  return GSB_OK;
}

// Clears the status words of a workspace header: code, detail and a count (used by the projection's
// non-finite check).
static int32_t* begin_status(void* ws, cudaStream_t st) {
  auto* h = static_cast<WorkspaceHeader*>(ws);
  cudaMemsetAsync(h, 0, 12, st);
  return &h->status;
}

}  // namespace gsb

using namespace gsb;

extern "C" {

GSB_API const char* gsb_version(void) { return "gsb200 1.0 sm_100a"; }

GSB_API uint64_t gsb_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }

GSB_API const char* gsb_status_string(int s) {
  switch (s) {
    case GSB_OK: return "ok";
    case GSB_ERR_SHAPE: return "inconsistent or unsupported sizes";
    case GSB_ERR_WORKSPACE: return "workspace too small";
    case GSB_ERR_KEY_OVERFLOW: return "too many (tile, Gaussian) pairs (limit 2^30 per call)";
    case GSB_ERR_NONFINITE: return "non-finite values";
    case GSB_ERR_TIMEOUT: return "a bounded device-side wait gave up";
    case GSB_ERR_CUDA: return "CUDA runtime error";
    case GSB_ERR_ARG: return "invalid argument";
    case GSB_ERR_CAPACITY: return "more (tile, Gaussian) pairs than the capacity given to gsb_bin";
    default: return "unknown status";
  }
}

GSB_API gsb_status gsb_read_status(const void* workspace, int* status_out, void* stream) {
  if (!workspace || !status_out) return GSB_ERR_ARG;
  int32_t v[2] = {0, 0};
  if (cudaMemcpyAsync(v, workspace, 8, cudaMemcpyDeviceToHost, as_stream(stream))) return GSB_ERR_CUDA;
  if (cudaStreamSynchronize(as_stream(stream))) return GSB_ERR_CUDA;
  *status_out = v[0];
  return GSB_OK;
}

// ---- stage 1 ---------------------------------------------------------------------------------

// Per-view segmented sort of 32-bit depth keys: the views are independent runs of G keys.
static size_t depth_ws(int32_t B, int32_t G) {
  const uint32_t n = uint32_t(size_t(B) * G);
  Carver c(nullptr, 0);
  c.take<WorkspaceHeader>(1);
  c.take<uint32_t>(n);  // keys
  c.take<uint32_t>(n);  // values
  c.take<uint32_t>(n);  // sorted keys
  c.take<uint32_t>(n);  // sorted values
  c.take<char>(segmented_sort_workspace(uint32_t(B), uint32_t(G)));
  return c.used;
}

GSB_API size_t gsb_depth_order_workspace(const gsb_scene* scene, const gsb_views* views) {
  if (!scene || !views) return 0;
  return depth_ws(views->n_views, scene->n_gaussians);
}

GSB_API gsb_status gsb_depth_order(const gsb_scene* scene, const gsb_views* views, int32_t* sorted_ids,
                                   int32_t* rank_of, void* workspace, size_t workspace_bytes, void* stream) {
  gsb_status s;
  if ((s = check_views(views)) != GSB_OK) return s;
  if ((s = check_scene(scene, views)) != GSB_OK) return s;
  if (!sorted_ids || !rank_of || !workspace) return GSB_ERR_ARG;
  const int32_t B = views->n_views, G = scene->n_gaussians;
  if (workspace_bytes < depth_ws(B, G)) return GSB_ERR_WORKSPACE;
  cudaStream_t st = as_stream(stream);
  const uint32_t n = uint32_t(size_t(B) * G);
  Carver c(workspace, workspace_bytes);
  c.take<WorkspaceHeader>(1);
  uint32_t* keys = c.take<uint32_t>(n);
  uint32_t* vals = c.take<uint32_t>(n);
  uint32_t* skeys = c.take<uint32_t>(n);
  uint32_t* svals = c.take<uint32_t>(n);
  const size_t sws = segmented_sort_workspace(uint32_t(B), uint32_t(G));
  void* sort_ws = c.take<char>(sws);
  int32_t* status = begin_status(workspace, st);
  uint32_t* hist = nullptr;
  if ((s = segmented_sort_prepare(sort_ws, sws, uint32_t(B), uint32_t(G), st, &hist)) != GSB_OK) return s;
  if ((s = launch_depth_keys(*scene, *views, keys, vals, hist, st)) != GSB_OK) return s;
  // the last pass writes sorted_ids and rank_of directly
  return segmented_sort_run(keys, skeys, vals, svals, uint32_t(B), uint32_t(G), sort_ws, sws, st, status, sorted_ids,
                            rank_of);
}

// ---- stage 2 ---------------------------------------------------------------------------------

static size_t preprocess_ws(int32_t B, int32_t G) {
  const uint32_t n = uint32_t(size_t(B) * G);
  Carver c(nullptr, 0);
  c.take<WorkspaceHeader>(1);
  c.take<uint32_t>(n);
  c.take<char>(exclusive_scan_workspace(n));
  return c.used;
}

GSB_API size_t gsb_preprocess_workspace(const gsb_views* views, int32_t n_gaussians) {
  if (!views) return 0;
  return preprocess_ws(views->n_views, n_gaussians);
}

GSB_API gsb_status gsb_preprocess_fwd(const gsb_scene* scene, const gsb_views* views, const gsb_options* opts,
                                      const int32_t* rank_of, float* records, int32_t* tile_rects,
                                      uint32_t* pair_offsets, float* cov2d_out, void* workspace,
                                      size_t workspace_bytes, void* stream) {
  gsb_status s;
  if ((s = check_views(views)) != GSB_OK) return s;
  if ((s = check_scene(scene, views)) != GSB_OK) return s;
  if ((s = check_opts(opts)) != GSB_OK) return s;
  if (!rank_of || !records || !tile_rects || !pair_offsets || !workspace) return GSB_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(records) % 16 || reinterpret_cast<uintptr_t>(tile_rects) % 16) return GSB_ERR_ARG;
  const int32_t B = views->n_views, G = scene->n_gaussians;
  if (workspace_bytes < preprocess_ws(B, G)) return GSB_ERR_WORKSPACE;
  cudaStream_t st = as_stream(stream);
  const uint32_t n = uint32_t(size_t(B) * G);
  Carver c(workspace, workspace_bytes);
  c.take<WorkspaceHeader>(1);
  uint32_t* counts = c.take<uint32_t>(n);
  const size_t scan_bytes = exclusive_scan_workspace(n);
  void* scan_ws = c.take<char>(scan_bytes);
  int32_t* status = begin_status(workspace, st);
  const RenderConsts rc = make_consts(*views, *opts);
  if ((s = launch_preprocess_fwd(*scene, *views, rc, rank_of, records, reinterpret_cast<int4*>(tile_rects), counts,
                                 cov2d_out, st, status)) != GSB_OK)
    return s;
  if (!rc.compat && rc.ellipse &&
      (s = launch_count_pairs(views->n_views, scene->n_gaussians, rc, views->height, views->width, records,
                              reinterpret_cast<const int4*>(tile_rects), counts, status, st)) != GSB_OK)
    return s;
  return exclusive_scan(counts, n, pair_offsets, scan_ws, scan_bytes, st, status);
}

// ---- stage 3 ---------------------------------------------------------------------------------

static size_t bin_ws(uint32_t n_pairs, uint32_t n_views, size_t n_tiles_total) {
  const uint32_t nt = uint32_t(n_tiles_total);
  Carver c(nullptr, 0);
  c.take<WorkspaceHeader>(1);
  c.take<uint64_t>(n_pairs);
  c.take<char>(pair_sort_workspace(n_pairs, n_views, n_views ? nt / n_views : 0u));
  c.take<uint32_t>(nt);  // order keys
  c.take<uint32_t>(nt);  // order values
  c.take<uint32_t>(nt);  // sorted order keys
  c.take<char>(radix_sort_workspace(nt, 4, 1));
  return c.used;
}

static size_t n_tiles_total(const gsb_views* views, const gsb_options* opts) {
  if (!views || !opts || opts->tile_size <= 0) return 0;
  const size_t tx = (size_t(views->width) + opts->tile_size - 1) / opts->tile_size;
  const size_t ty = (size_t(views->height) + opts->tile_size - 1) / opts->tile_size;
  return size_t(views->n_views) * tx * ty;
}

GSB_API size_t gsb_bin_workspace(const gsb_views* views, const gsb_options* opts, int32_t n_gaussians,
                                 uint32_t n_pairs) {
  (void)n_gaussians;
  return bin_ws(n_pairs, views ? uint32_t(views->n_views) : 0u, n_tiles_total(views, opts));
}

GSB_API gsb_status gsb_bin(const gsb_views* views, const gsb_options* opts, int32_t n_gaussians, const float* records,
                           const int32_t* tile_rects, const uint32_t* pair_offsets, uint32_t n_pairs,
                           uint64_t* sorted_keys, uint32_t* tile_ranges, uint32_t* tile_order, void* workspace,
                           size_t workspace_bytes, void* stream) {
  gsb_status s;
  if ((s = check_frame(views)) != GSB_OK) return s;
  if ((s = check_opts(opts)) != GSB_OK) return s;
  if (n_gaussians <= 0) return GSB_ERR_SHAPE;
  if (!records || !tile_rects || !pair_offsets || !tile_ranges || !workspace) return GSB_ERR_ARG;
  if (n_pairs > 0 && !sorted_keys) return GSB_ERR_ARG;
  if (n_pairs >= (1u << 30)) return GSB_ERR_KEY_OVERFLOW;
  const size_t NT = n_tiles_total(views, opts);
  if (NT >= (size_t(1) << 30)) return GSB_ERR_SHAPE;
  if (workspace_bytes < bin_ws(n_pairs, uint32_t(views->n_views), NT)) return GSB_ERR_WORKSPACE;
  cudaStream_t st = as_stream(stream);
  const RenderConsts rc = make_consts(*views, *opts);
  const int32_t B = views->n_views;
  Carver c(workspace, workspace_bytes);
  c.take<WorkspaceHeader>(1);
  uint64_t* keys = c.take<uint64_t>(n_pairs);
  const size_t sws = pair_sort_workspace(n_pairs, uint32_t(B), uint32_t(rc.n_tiles));
  void* sort_ws = c.take<char>(sws);
  uint32_t* okeys = c.take<uint32_t>(NT);
  uint32_t* ovals = c.take<uint32_t>(NT);
  uint32_t* okeys_sorted = c.take<uint32_t>(NT);
  const size_t ows = radix_sort_workspace(uint32_t(NT), 4, 1);
  void* order_ws = c.take<char>(ows);
  int32_t* status = begin_status(workspace, st);
  // n_pairs is the capacity of the key buffers; the count itself is read on the device, so the
  // stage can be queued before the count reaches the host.
  const uint32_t* n_dev = pair_offsets + size_t(B) * size_t(n_gaussians);
  bool ranges_done = false;
  if (n_pairs > 0) {  // keys in (view, rank) order, then each view's run sorted by tile
    uint32_t* hist = nullptr;
    if ((s = pair_sort_prepare(sort_ws, sws, n_pairs, uint32_t(B), uint32_t(rc.n_tiles), st, &hist)) != GSB_OK)
      return s;
    if ((s = launch_emit(B, n_gaussians, rc, views->height, views->width, records,
                         reinterpret_cast<const int4*>(tile_rects), pair_offsets, n_pairs, keys, hist,
                         pair_sort_passes(uint32_t(rc.n_tiles)), status, st)) != GSB_OK)
      return s;
    if ((s = pair_sort_run(keys, sorted_keys, n_pairs, uint32_t(B), uint32_t(rc.n_tiles), n_gaussians, pair_offsets,
                           sort_ws, sws, st, status, tile_ranges, tile_order ? okeys : nullptr, ovals,
                           &ranges_done)) != GSB_OK)
      return s;
  }
  if (!ranges_done &&
      (s = launch_tile_ranges(sorted_keys, n_pairs, n_dev, tile_ranges, size_t(B) * rc.n_tiles, status, st)) != GSB_OK)
    return s;
  if (!tile_order) return GSB_OK;
  // launch order: tiles by descending list length (8-bit log-scale key, one radix pass)
  if (!ranges_done && (s = launch_tile_order_keys(tile_ranges, uint32_t(NT), okeys, ovals, st)) != GSB_OK) return s;
  return radix_sort(okeys, okeys_sorted, ovals, tile_order, uint32_t(NT), 4, 0, 8, order_ws, ows, st, status);
}

// ---- stages 4 and 6 --------------------------------------------------------------------------

static size_t checkpoint_floats(const gsb_views& v, const gsb_options& o) {
  const int nseg = raster_segments(v, o);
  return nseg > 1 ? size_t(nseg - 1) * 6 * size_t(v.n_views) * size_t(v.height) * size_t(v.width) : 0;
}

GSB_API size_t gsb_raster_checkpoint_floats(const gsb_views* views, const gsb_options* opts) {
  if (check_frame(views) != GSB_OK || check_opts(opts) != GSB_OK) return 0;
  return checkpoint_floats(*views, *opts);
}

GSB_API gsb_status gsb_raster_fwd(const gsb_views* views, const gsb_options* opts, int32_t n_gaussians,
                                  const float* records, const uint64_t* sorted_keys, const uint32_t* tile_ranges,
                                  const uint32_t* tile_order, float* image, float* alpha, float* depth,
                                  float* pixel_t, uint32_t* pixel_state, float* pixel_ckpt, void* stream) {
  gsb_status s;
  if ((s = check_frame(views)) != GSB_OK) return s;
  if ((s = check_opts(opts)) != GSB_OK) return s;
  if (n_gaussians <= 0) return GSB_ERR_SHAPE;
  if (!records || !tile_ranges || !image || !pixel_t || !pixel_state) return GSB_ERR_ARG;
  RasterArgs a{};
  a.B = views->n_views, a.G = n_gaussians, a.H = views->height, a.W = views->width;
  a.rc = make_consts(*views, *opts);
  a.records = records, a.keys = sorted_keys, a.ranges = tile_ranges, a.order = tile_order;
  a.image = image, a.alpha = alpha, a.depth = (opts->flags & GSB_RENDER_DEPTH) ? depth : nullptr;
  a.pixel_t = pixel_t, a.pixel_state = pixel_state;
  a.nseg = raster_segments(*views, *opts), a.ckpt = pixel_ckpt;
  if (a.nseg > 1 && !pixel_ckpt) return GSB_ERR_ARG;
  if (views->n_views > 65535) return GSB_ERR_SHAPE;
  return launch_raster_fwd(a, as_stream(stream));
}

GSB_API gsb_status gsb_raster_bwd(const gsb_views* views, const gsb_options* opts, int32_t n_gaussians,
                                  const float* records, const uint64_t* sorted_keys, const uint32_t* tile_ranges,
                                  const uint32_t* tile_order, const float* pixel_t, const uint32_t* pixel_state,
                                  const float* pixel_ckpt, const float* d_image,
                                  const float* d_alpha, const float* d_depth, const float* view_scale, float* grad2d,
                                  void* stream) {
  gsb_status s;
  if ((s = check_frame(views)) != GSB_OK) return s;
  if ((s = check_opts(opts)) != GSB_OK) return s;
  if (n_gaussians <= 0) return GSB_ERR_SHAPE;
  if (!records || !tile_ranges || !pixel_t || !pixel_state || !d_image || !grad2d) return GSB_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(grad2d) % 8u) return GSB_ERR_ARG;  // added to as pairs of floats
  RasterArgs a{};
  a.B = views->n_views, a.G = n_gaussians, a.H = views->height, a.W = views->width;
  a.rc = make_consts(*views, *opts);
  a.records = records, a.keys = sorted_keys, a.ranges = tile_ranges, a.order = tile_order;
  a.pixel_t = const_cast<float*>(pixel_t), a.pixel_state = const_cast<uint32_t*>(pixel_state);
  a.nseg = raster_segments(*views, *opts), a.ckpt = const_cast<float*>(pixel_ckpt);
  if (a.nseg > 1 && !pixel_ckpt) return GSB_ERR_ARG;
  // the depth gradient needs the forward's depth sums (GSB_RENDER_DEPTH, the option the forward ran with)
  a.d_image = d_image, a.d_alpha = d_alpha, a.view_scale = view_scale, a.grad2d = grad2d;
  a.d_depth = (opts->flags & GSB_RENDER_DEPTH) ? d_depth : nullptr;
  if (views->n_views > 65535) return GSB_ERR_SHAPE;
  return launch_raster_bwd(a, as_stream(stream));
}

// ---- stage 5 ---------------------------------------------------------------------------------

GSB_API size_t gsb_loss_workspace(int32_t n_images) { return loss_workspace(n_images); }

GSB_API gsb_status gsb_loss_fwd_bwd(const gsb_loss_options* lopts, int32_t n_images, int32_t channels, int32_t height,
                                    int32_t width, const float* pred, const float* target, float* loss, float* dpred,
                                    void* workspace, size_t workspace_bytes, void* stream) {
  if (!lopts) return GSB_ERR_ARG;
  return loss_fwd_bwd(*lopts, n_images, channels, height, width, pred, target, loss, dpred, workspace,
                      workspace_bytes, as_stream(stream));
}

GSB_API gsb_status gsb_scale_planes(const float* in, const float* scale, float* out, int32_t n_images,
                                    int64_t plane_elems, void* stream) {
  return scale_planes(in, scale, out, n_images, plane_elems, as_stream(stream));
}

// ---- stage 7 ---------------------------------------------------------------------------------

GSB_API gsb_status gsb_preprocess_bwd(const gsb_scene* scene, const gsb_views* views, const gsb_options* opts,
                                      const int32_t* rank_of, const float* grad2d, gsb_scene_grads* grads,
                                      void* stream) {
  gsb_status s;
  if ((s = check_views(views)) != GSB_OK) return s;
  if ((s = check_scene(scene, views)) != GSB_OK) return s;
  if ((s = check_opts(opts)) != GSB_OK) return s;
  if (!rank_of || !grad2d || !grads) return GSB_ERR_ARG;
  const RenderConsts rc = make_consts(*views, *opts);
  return launch_preprocess_bwd(*scene, *views, rc, rank_of, grad2d, *grads, as_stream(stream));
}

GSB_API gsb_status gsb_preprocess_bwd_range(const gsb_scene* scene, const gsb_views* views, const gsb_options* opts,
                                            const int32_t* rank_of, const float* grad2d, gsb_scene_grads* grads,
                                            int64_t first, int64_t count, void* stream) {
  gsb_status s;
  if ((s = check_views(views)) != GSB_OK) return s;
  if ((s = check_scene(scene, views)) != GSB_OK) return s;
  if ((s = check_opts(opts)) != GSB_OK) return s;
  if (!rank_of || !grad2d || !grads) return GSB_ERR_ARG;
  const int64_t total = int64_t(scene->n_sets) * scene->n_gaussians;
  if (first < 0 || count < 0 || first > total || count > total - first) return GSB_ERR_SHAPE;
  if (count == 0) return GSB_OK;
  RenderConsts rc = make_consts(*views, *opts);
  rc.bwd_first = uint64_t(first);
  rc.bwd_count = uint64_t(count);
  return launch_preprocess_bwd(*scene, *views, rc, rank_of, grad2d, *grads, as_stream(stream));
}

GSB_API gsb_status gsb_camera_bwd(const gsb_scene* scene, const gsb_views* views, const gsb_options* opts,
                                  const int32_t* rank_of, const float* grad2d, gsb_camera_grads* grads, void* stream) {
  gsb_status s;
  if ((s = check_views(views)) != GSB_OK) return s;
  if ((s = check_scene(scene, views)) != GSB_OK) return s;
  if ((s = check_opts(opts)) != GSB_OK) return s;
  if (!rank_of || !grad2d || !grads) return GSB_ERR_ARG;
  if (views->n_views > 65535) return GSB_ERR_SHAPE;
  const RenderConsts rc = make_consts(*views, *opts);
  return launch_camera_bwd(*scene, *views, rc, rank_of, grad2d, *grads, as_stream(stream));
}

// ---- already-projected 2-D Gaussians ---------------------------------------------------------

GSB_API size_t gsb_splats2d_order_workspace(const gsb_splats2d* splats) {
  if (!splats) return 0;
  return depth_ws(splats->n_views, splats->n_gaussians);
}

GSB_API gsb_status gsb_splats2d_order(const gsb_splats2d* splats, int32_t* sorted_ids, int32_t* rank_of,
                                      void* workspace, size_t workspace_bytes, void* stream) {
  gsb_status s;
  if ((s = check_splats2d(splats)) != GSB_OK) return s;
  if (!sorted_ids || !rank_of || !workspace) return GSB_ERR_ARG;
  const int32_t B = splats->n_views, G = splats->n_gaussians;
  if (workspace_bytes < depth_ws(B, G)) return GSB_ERR_WORKSPACE;
  cudaStream_t st = as_stream(stream);
  const uint32_t n = uint32_t(size_t(B) * G);
  Carver c(workspace, workspace_bytes);  // the layout of depth_ws
  c.take<WorkspaceHeader>(1);
  uint32_t* keys = c.take<uint32_t>(n);
  uint32_t* vals = c.take<uint32_t>(n);
  uint32_t* skeys = c.take<uint32_t>(n);
  uint32_t* svals = c.take<uint32_t>(n);
  const size_t sws = segmented_sort_workspace(uint32_t(B), uint32_t(G));
  void* sort_ws = c.take<char>(sws);
  int32_t* status = begin_status(workspace, st);
  uint32_t* hist = nullptr;
  if ((s = segmented_sort_prepare(sort_ws, sws, uint32_t(B), uint32_t(G), st, &hist)) != GSB_OK) return s;
  if ((s = launch_order_keys_2d(*splats, keys, vals, hist, st)) != GSB_OK) return s;
  if (splats->depths) {
    if ((s = segmented_sort_run(keys, skeys, vals, svals, uint32_t(B), uint32_t(G), sort_ws, sws, st, status)) !=
        GSB_OK)
      return s;
  } else {
    svals = vals;  // no depths: index order, the keys are already sorted
  }
  return launch_invert_order(svals, B, G, sorted_ids, rank_of, st);
}

GSB_API size_t gsb_splats2d_preprocess_workspace(const gsb_splats2d* splats) {
  if (!splats) return 0;
  return preprocess_ws(splats->n_views, splats->n_gaussians);
}

GSB_API gsb_status gsb_splats2d_preprocess(const gsb_splats2d* splats, int32_t height, int32_t width,
                                           const gsb_options* opts, const int32_t* rank_of, float* records,
                                           int32_t* tile_rects, uint32_t* pair_offsets, void* workspace,
                                           size_t workspace_bytes, void* stream) {
  gsb_status s;
  if ((s = check_splats2d(splats)) != GSB_OK) return s;
  if ((s = check_opts(opts)) != GSB_OK) return s;
  if (height <= 0 || width <= 0) return GSB_ERR_SHAPE;
  if (opts->flags & GSB_RENDER_TILED_COMPAT) return GSB_ERR_ARG;  // tiled.py bounds need a 2-D covariance
  if (!rank_of || !records || !tile_rects || !pair_offsets || !workspace) return GSB_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(records) % 16 || reinterpret_cast<uintptr_t>(tile_rects) % 16) return GSB_ERR_ARG;
  const int32_t B = splats->n_views, G = splats->n_gaussians;
  if (workspace_bytes < preprocess_ws(B, G)) return GSB_ERR_WORKSPACE;
  cudaStream_t st = as_stream(stream);
  const uint32_t n = uint32_t(size_t(B) * G);
  Carver c(workspace, workspace_bytes);
  c.take<WorkspaceHeader>(1);
  uint32_t* counts = c.take<uint32_t>(n);
  const size_t scan_bytes = exclusive_scan_workspace(n);
  void* scan_ws = c.take<char>(scan_bytes);
  int32_t* status = begin_status(workspace, st);
  gsb_views frame{};
  frame.n_views = B, frame.views_per_set = 1, frame.height = height, frame.width = width;
  const RenderConsts rc = make_consts(frame, *opts);
  if ((s = launch_preprocess_2d(*splats, height, width, rc, rank_of, records, reinterpret_cast<int4*>(tile_rects),
                                counts, st)) != GSB_OK)
    return s;
  if (rc.ellipse && (s = launch_count_pairs(B, G, rc, height, width, records,
                                            reinterpret_cast<const int4*>(tile_rects), counts, status, st)) != GSB_OK)
    return s;
  return exclusive_scan(counts, n, pair_offsets, scan_ws, scan_bytes, st, status);
}

GSB_API gsb_status gsb_splats2d_preprocess_bwd(const gsb_splats2d* splats, const int32_t* rank_of,
                                               const float* grad2d, gsb_splats2d_grads* grads, void* stream) {
  gsb_status s;
  if ((s = check_splats2d(splats)) != GSB_OK) return s;
  if (!rank_of || !grad2d || !grads) return GSB_ERR_ARG;
  return launch_preprocess_2d_bwd(*splats, rank_of, grad2d, *grads, as_stream(stream));
}

// ---- utility ---------------------------------------------------------------------------------

GSB_API size_t gsb_radix_sort_workspace(uint32_t n, int key_bytes, int with_values) {
  return align_up(sizeof(WorkspaceHeader)) + radix_sort_workspace(n, key_bytes, with_values);
}

GSB_API gsb_status gsb_radix_sort(const void* keys_in, void* keys_out, const uint32_t* values_in, uint32_t* values_out,
                                  uint32_t n, int key_bytes, int bit_lo, int bit_hi, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  if (n > 0 && (!keys_in || !keys_out)) return GSB_ERR_ARG;
  if (!workspace) return GSB_ERR_ARG;
  const size_t need = gsb_radix_sort_workspace(n, key_bytes, values_in != nullptr);
  if (workspace_bytes < need) return GSB_ERR_WORKSPACE;
  cudaStream_t st = as_stream(stream);
  int32_t* status = begin_status(workspace, st);
  char* inner = static_cast<char*>(workspace) + align_up(sizeof(WorkspaceHeader));
  return radix_sort(keys_in, keys_out, values_in, values_out, n, key_bytes, bit_lo, bit_hi, inner,
                    workspace_bytes - align_up(sizeof(WorkspaceHeader)), st, status);
}

GSB_API gsb_status gsb_debug_sort_lookback_timeout(const uint32_t* keys_in, uint32_t* keys_out, uint32_t n,
                                                   uint32_t spin_limit, void* workspace, size_t workspace_bytes,
                                                   void* stream) {
  if (!keys_in || !keys_out || !workspace) return GSB_ERR_ARG;
  const size_t need = gsb_radix_sort_workspace(n, 4, 0);
  if (workspace_bytes < need) return GSB_ERR_WORKSPACE;
  cudaStream_t st = as_stream(stream);
  int32_t* status = begin_status(workspace, st);
  char* inner = static_cast<char*>(workspace) + align_up(sizeof(WorkspaceHeader));
  return sort_lookback_timeout_probe(keys_in, keys_out, n, spin_limit, inner,
                                     workspace_bytes - align_up(sizeof(WorkspaceHeader)), st, status);
}

}  // extern "C"
