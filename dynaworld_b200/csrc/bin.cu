// Binning: one 64-bit key per (view, tile, Gaussian) pair, a stable radix sort by tile within each
// view, and the [start, end) run of every tile.
//
// Restates build_tile_assignments (src/train/renderers/tiled.py:31-71): the reference lists
// (tile, Gaussian) pairs and stable-argsorts them by tile (:59), with Gaussians already in depth
// order (renderers/common.py:191), so each tile's list is in depth order.  Here the pairs are
// emitted in (view, depth rank) order with the rank in the key's low 32 bits, so every view's
// pairs are one contiguous run, and each run is sorted by its tile index alone -- the stability
// of the LSD sort keeps depth order within a tile.
#include "gsb_common.cuh"
#include "gsb_internal.h"
#include "tiles.cuh"

namespace gsb {

constexpr int kMaxTilePasses = 4;

// One thread per (view blockIdx.y, depth rank): the Gaussian's keys in its slot of the pair array,
// and the block's counts of the tile digits its written keys carry (the per-view histograms of
// the pair sort's passes).  (Emitting the keys of a Gaussian with more than 32 tiles by the whole
// warp -- a thread per tile row, a warp scan, coalesced stores -- was measured slower on
// 2 x 1920x1080: 0.53 -> 0.60 ms, the extra registers costing more than the balance gains.)
__global__ void __launch_bounds__(256) emit_keys_kernel(int32_t G, RenderConsts rc, int H, int W,
                                                        const float* __restrict__ records,
                                                        const int4* __restrict__ rects,
                                                        const uint32_t* __restrict__ offsets, uint32_t n_pairs,
                                                        uint64_t* __restrict__ keys, uint32_t* __restrict__ hist,
                                                        int passes, int32_t* __restrict__ status) {
  __shared__ uint32_t s_hist[kMaxTilePasses][256];
  __shared__ uint32_t s_done;
  for (int i = threadIdx.x; i < kMaxTilePasses * 256; i += blockDim.x) s_hist[i / 256][i % 256] = 0u;
  if (threadIdx.x == 0) s_done = 0u;
  __syncthreads();
  const uint32_t b = blockIdx.y;
  const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
  const size_t i = size_t(b) * G + r;
  const uint32_t start = r < uint32_t(G) ? offsets[i] : 0u;
  const uint32_t end = r < uint32_t(G) ? offsets[i + 1] : 0u;
  const uint64_t view_base = uint64_t(b) * rc.n_tiles;
  uint32_t k = start;
  auto put = [&](int tx, int ty) {
    if (k < end && k < n_pairs) {
      const uint32_t t = uint32_t(ty * rc.tiles_x + tx);
      keys[k] = ((view_base + t) << 32) | r;
      for (int p = 0; p < passes; ++p) atomicAdd(&s_hist[p][(t >> (8 * p)) & 0xffu], 1u);
    }
    ++k;
  };
  if (start != end) {
    const int4 rc4 = rects[i];
    if (!rc.compat && rc.ellipse) {
      const float4* rec = reinterpret_cast<const float4*>(records + i * GSB_RECORD_FLOATS);
      const float4 r0 = rec[0], r1 = rec[1];
      ExactShape es;
      if (exact_shape(r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, rc.alpha_cutoff, H, W, rc.pixel_center, &es)) {
        for (int ty = rc4.y; ty <= rc4.w; ++ty) {
          int tx0, tx1;
          if (!exact_row_pairs(es, ty, rc.tile, rc.pixel_center, &tx0, &tx1)) continue;
          for (int tx = tx0; tx <= tx1; ++tx) put(tx, ty);
        }
      }
    } else {
      for (int ty = rc4.y; ty <= rc4.w; ++ty)
        for (int tx = rc4.x; tx <= rc4.z; ++tx) put(tx, ty);
    }
    if (k != end) record_error(status, GSB_ERR_KEY_OVERFLOW, int(i));
  }
  // The last warp to finish adds the block's counts to the view's histograms: no block barrier, so
  // warps done with short Gaussians do not wait for the block's longest one.
  __syncwarp();
  __threadfence_block();
  const int lane = threadIdx.x & 31;
  uint32_t done = 0u;
  if (lane == 0) done = atomicAdd(&s_done, 1u);
  done = __shfl_sync(0xffffffffu, done, 0);
  if (done != blockDim.x / 32 - 1) return;
  __threadfence_block();
  uint32_t* h = hist + size_t(b) * passes * 256;
  for (int j = lane; j < passes * 256; j += 32) {
    const uint32_t c = atomicAdd(&s_hist[j / 256][j % 256], 0u);  // read after the other warps' counts
    if (c) atomicAdd(h + j, c);
  }
}

__global__ void tile_ranges_kernel(const uint64_t* __restrict__ keys, uint32_t cap,
                                   const uint32_t* __restrict__ n_dev, uint32_t* __restrict__ ranges,
                                   size_t n_ranges, int32_t* __restrict__ status) {
  uint32_t n = cap;
  if (n_dev) {
    const uint32_t count = *n_dev;
    if (count > cap && blockIdx.x == 0 && threadIdx.x == 0) record_error(status, GSB_ERR_CAPACITY, int(cap));
    n = min(cap, count);
  }
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const uint32_t t = uint32_t(keys[i] >> 32);
    if (t >= n_ranges) continue;
    if (i == 0 || uint32_t(keys[i - 1] >> 32) != t) ranges[size_t(t) * 2] = i;
    if (i + 1 == n || uint32_t(keys[i + 1] >> 32) != t) ranges[size_t(t) * 2 + 1] = i + 1;
  }
}

// Sort key of a tile's launch slot: longer lists first.
__global__ void tile_order_keys_kernel(const uint32_t* __restrict__ ranges, uint32_t n, uint32_t* __restrict__ keys,
                                       uint32_t* __restrict__ vals) {
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const uint32_t len = ranges[size_t(i) * 2 + 1] - ranges[size_t(i) * 2];
    keys[i] = 255u - length_class(len);
    vals[i] = i;
  }
}

gsb_status launch_tile_order_keys(const uint32_t* ranges, uint32_t n, uint32_t* keys, uint32_t* vals,
                                  cudaStream_t st) {
  if (n == 0) return GSB_OK;
  const int grid = int(std::min<uint32_t>((n + 255) / 256, 148u * 16u));
  note_launch();
  tile_order_keys_kernel<<<grid, 256, 0, st>>>(ranges, n, keys, vals);
  return launch_status();
}

gsb_status launch_emit(int32_t B, int32_t G, const RenderConsts& rc, int H, int W, const float* records,
                       const int4* rects, const uint32_t* offsets, uint32_t n_pairs, uint64_t* keys, uint32_t* hist,
                       int passes, int32_t* status, cudaStream_t st) {
  if (passes < 0 || passes > kMaxTilePasses) return GSB_ERR_SHAPE;
  const dim3 grid(unsigned((size_t(G) + 255) / 256), unsigned(B));
  note_launch();
  emit_keys_kernel<<<grid, 256, 0, st>>>(G, rc, H, W, records, rects, offsets, n_pairs, keys, hist, passes, status);
  return launch_status();
}

gsb_status launch_tile_ranges(const uint64_t* keys, uint32_t n, const uint32_t* n_dev, uint32_t* ranges,
                              size_t n_ranges, int32_t* status, cudaStream_t st) {
  if (cudaMemsetAsync(ranges, 0, n_ranges * 2 * sizeof(uint32_t), st)) return GSB_ERR_CUDA;
  if (n == 0 && !n_dev) return GSB_OK;
  const int grid = int(std::min<uint32_t>(std::max<uint32_t>((n + 255) / 256, 1u), 148u * 32u));
  note_launch();
  tile_ranges_kernel<<<grid, 256, 0, st>>>(keys, n, n_dev, ranges, n_ranges, status);
  return launch_status();
}

}  // namespace gsb
