// Internal (host-side) interfaces between the translation units of libgsb200.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "gsb200.h"

namespace gsb {

// Counts kernel launches made by this library (diagnostic; read by gsb_kernel_launches()).
void note_launch();

// Status of the launches just queued: GSB_ERR_CUDA when one failed.  A failed launch's error is
// cleared from the thread's last-error slot (cudaGetLastError), so it is reported once, by this
// library, and does not make later calls of this library or of the caller fail as well.
inline gsb_status launch_status() {
  if (cudaPeekAtLastError() == cudaSuccess) return GSB_OK;
  (void)cudaGetLastError();
  return GSB_ERR_CUDA;
}

// Radix sort (sort.cu).
size_t radix_sort_workspace(uint32_t n, int key_bytes, int with_values);
// n_dev (may be NULL): a device word holding the element count; the sort then uses
// min(n, *n_dev) elements and n is only the capacity its grid and workspace are sized for.
gsb_status radix_sort(const void* keys_in, void* keys_out, const uint32_t* vals_in, uint32_t* vals_out, uint32_t n,
                      int key_bytes, int bit_lo, int bit_hi, void* ws, size_t ws_bytes, cudaStream_t stream,
                      int32_t* status, const uint32_t* n_dev = nullptr);

// Test hook: one look-back pass whose first partition never runs, so the bounded wait after it
// runs out (GSB_ERR_TIMEOUT); see sort.cu.
gsb_status sort_lookback_timeout_probe(const uint32_t* keys_in, uint32_t* keys_out, uint32_t n, uint32_t spin_limit,
                                       void* ws, size_t ws_bytes, cudaStream_t stream, int32_t* status);

// Segmented sort of 32-bit keys with values (sort.cu): n_seg independent runs of seg_len keys.
// segmented_sort_prepare clears the workspace's counters and returns the digit histograms
// [n_seg][4][256] that the kernel writing the keys must fill before segmented_sort_run.
size_t segmented_sort_workspace(uint32_t n_seg, uint32_t seg_len);
gsb_status segmented_sort_prepare(void* ws, size_t ws_bytes, uint32_t n_seg, uint32_t seg_len, cudaStream_t stream,
                                  uint32_t** hist);
// ids_out / rank_out (both or neither): the last pass writes the sorted values as ids_out and
// their inverse permutation per segment (rank_out[seg * seg_len + value] = position in the segment)
// instead of keys_out / vals_out.
gsb_status segmented_sort_run(const uint32_t* keys_in, uint32_t* keys_out, const uint32_t* vals_in, uint32_t* vals_out,
                              uint32_t n_seg, uint32_t seg_len, void* ws, size_t ws_bytes, cudaStream_t stream,
                              int32_t* status, int32_t* ids_out = nullptr, int32_t* rank_out = nullptr);

// Pair keys sorted by tile within each view's run (sort.cu): pair_sort_prepare clears the
// workspace and returns the digit histograms [n_views][passes][256] of the tile index (passes =
// ceil(log2(n_tiles) / 8)) that the kernel writing the keys fills; pair_sort_run reads the run
// bounds from pair_offsets (view v starts at pair_offsets[v * G], clipped to cap).
size_t pair_sort_workspace(uint32_t cap, uint32_t n_views, uint32_t n_tiles);
int pair_sort_passes(uint32_t n_tiles);
gsb_status pair_sort_prepare(void* ws, size_t ws_bytes, uint32_t cap, uint32_t n_views, uint32_t n_tiles,
                             cudaStream_t stream, uint32_t** hist);
// tile_ranges (may be NULL) [n_views * n_tiles * 2] and, when order_keys is given, the launch-order
// keys and values: written from the pass's counts when one pass sorts the runs (*ranges_done).
gsb_status pair_sort_run(const uint64_t* keys_in, uint64_t* keys_out, uint32_t cap, uint32_t n_views, uint32_t n_tiles,
                         int32_t G, const uint32_t* pair_offsets, void* ws, size_t ws_bytes, cudaStream_t stream,
                         int32_t* status, uint32_t* tile_ranges, uint32_t* order_keys, uint32_t* order_vals,
                         bool* ranges_done);

// Exclusive scan: offsets[0..n) and offsets[n] = total (sort.cu).
size_t exclusive_scan_workspace(uint32_t n);
gsb_status exclusive_scan(const uint32_t* counts, uint32_t n, uint32_t* offsets, void* scratch, size_t scratch_bytes,
                          cudaStream_t stream, int32_t* status);

// Values derived from gsb_options once per call.
struct RenderConsts {
  int tile;
  int tiles_x, tiles_y, n_tiles;
  bool compat;
  bool depth;
  bool ellipse;
  bool clamp_image;  // clamp the composited image to [0, 1]
  float near_plane, alpha_clamp, alpha_cutoff, t_threshold, eps, pixel_center;
  float bg[3];
  float bound_scale, tiled_threshold;
  float f0;      // fl32(1 + eps): the transmittance factor of an alpha-0 pair
  float inv_f0;  // a float within a few ulp of 1 / f0 whose product with f0 rounds to exactly 1
  int unit_inv;  // such a float exists (every eps up to 0.5): S * (f0 * inv_f0) == S
  float log2_f0; // log2(f0): T_i = F0^pos_i * S_i (pos = depth rank, or list index in compat mode)
  // preprocess backward: the Gaussians (set * G + index) [bwd_first, bwd_first + bwd_count) it
  // writes (bwd_count 0: all of them)
  uint64_t bwd_first, bwd_count;
};

RenderConsts make_consts(const gsb_views& v, const gsb_options& o);
int bits_for(uint64_t count);  // smallest b with 2^b >= count (0 for count <= 1)

// Raster stage arguments (raster.cu).
struct RasterArgs {
  int B, G, H, W;
  RenderConsts rc;
  const float* records;
  const uint64_t* keys;
  const uint32_t* ranges;
  const uint32_t* order;  // launch order of view*n_tiles + tile, or NULL
  float* image;
  float* alpha;
  float* depth;
  float* pixel_t;
  uint32_t* pixel_state;
  float* ckpt;   // backward segment checkpoints [nseg - 1][6][B*H*W], NULL when nseg == 1
  int nseg;      // backward list segments per tile (1, 2 or 4)
  const float* d_image;
  const float* d_alpha;
  const float* d_depth;
  const float* view_scale;
  float* grad2d;
};
gsb_status launch_raster_fwd(const RasterArgs& a, cudaStream_t st);
gsb_status launch_raster_bwd(const RasterArgs& a, cudaStream_t st);
int raster_segments(const gsb_views& v, const gsb_options& o);  // backward list segments (1, 2, 4)

// Preprocess (preprocess.cu).
// Depth keys [B*G] and Gaussian indices per view, digit histograms [B][4][256] accumulated.
gsb_status launch_depth_keys(const gsb_scene& sc, const gsb_views& vw, uint32_t* keys, uint32_t* vals, uint32_t* hist,
                             cudaStream_t st);
gsb_status launch_invert_order(const uint32_t* sorted_vals, int32_t B, int32_t G, int32_t* sorted_ids,
                               int32_t* rank_of, cudaStream_t st);
gsb_status launch_preprocess_fwd(const gsb_scene& sc, const gsb_views& vw, const RenderConsts& rc,
                                 const int32_t* rank_of, float* records, int4* rects, uint32_t* counts, float* cov,
                                 cudaStream_t st, int32_t* status);
gsb_status launch_preprocess_bwd(const gsb_scene& sc, const gsb_views& vw, const RenderConsts& rc,
                                 const int32_t* rank_of, const float* grad2d, const gsb_scene_grads& gr,
                                 cudaStream_t st);
gsb_status launch_camera_bwd(const gsb_scene& sc, const gsb_views& vw, const RenderConsts& rc, const int32_t* rank_of,
                             const float* grad2d, const gsb_camera_grads& out, cudaStream_t st);

// Already-projected 2-D Gaussians (splat2d.cu).
gsb_status launch_order_keys_2d(const gsb_splats2d& sp, uint32_t* keys, uint32_t* vals, uint32_t* hist,
                                cudaStream_t st);
gsb_status launch_preprocess_2d(const gsb_splats2d& sp, int H, int W, const RenderConsts& rc, const int32_t* rank_of,
                                float* records, int4* rects, uint32_t* counts, cudaStream_t st);
gsb_status launch_preprocess_2d_bwd(const gsb_splats2d& sp, const int32_t* rank_of, const float* grad2d,
                                    const gsb_splats2d_grads& gr, cudaStream_t st);

// Binning (bin.cu).
// Pair keys in (view, rank) order; hist [B][passes][256] gets the counts of their tile digits.
// Exact-mode pair count of every (view, depth rank) from the records and tile rects (rank order).
gsb_status launch_count_pairs(int32_t B, int32_t G, const RenderConsts& rc, int H, int W, const float* records,
                              const int4* rects, uint32_t* counts, int32_t* status, cudaStream_t st);
gsb_status launch_emit(int32_t B, int32_t G, const RenderConsts& rc, int H, int W, const float* records,
                       const int4* rects, const uint32_t* offsets, uint32_t n_pairs, uint64_t* keys, uint32_t* hist,
                       int passes, int32_t* status, cudaStream_t st);
// n: capacity of keys; the pair count is min(n, *n_dev) (n_dev may be NULL: n pairs).  A count
// above the capacity records GSB_ERR_CAPACITY.
gsb_status launch_tile_ranges(const uint64_t* keys, uint32_t n, const uint32_t* n_dev, uint32_t* ranges,
                              size_t n_ranges, int32_t* status, cudaStream_t st);
gsb_status launch_tile_order_keys(const uint32_t* ranges, uint32_t n_tiles_total, uint32_t* keys, uint32_t* vals,
                                  cudaStream_t st);

// Loss (loss.cu).
size_t loss_workspace(int32_t n_images);
gsb_status loss_fwd_bwd(const gsb_loss_options& o, int32_t B, int32_t C, int32_t H, int32_t W, const float* pred,
                        const float* target, float* loss, float* dpred, void* ws, size_t ws_bytes, cudaStream_t st);
gsb_status scale_planes(const float* in, const float* scale, float* out, int32_t B, int64_t per, cudaStream_t st);

}  // namespace gsb
