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

constexpr int kEmitThreads = 256;

// Exclusive scan of one value per thread of the 256-thread block (two barriers); returns the total.
__device__ __forceinline__ uint32_t emit_block_scan(uint32_t v, uint32_t* s_warp, uint32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  uint32_t before = 0, all = 0;
#pragma unroll
  for (int w = 0; w < kEmitThreads / 32; ++w) {
    const uint32_t t = s_warp[w];
    before += w < warp ? t : 0u;
    all += t;
  }
  __syncthreads();
  *total = all;
  return before + x - v;
}

// Last index j in [0, n) with a[j] <= v (a ascending, a[0] <= v).
__device__ __forceinline__ int emit_find(const uint32_t* a, int n, uint32_t v) {
  int lo = 0, hi = n;  // a[lo] <= v < a[hi] (a[n] taken as +inf)
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (a[mid] <= v) lo = mid;
    else hi = mid;
  }
  return lo;
}

// One block per 256 consecutive depth ranks of view blockIdx.y.  The work is flattened so that
// every lane has an item whatever the Gaussians' sizes: the block's Gaussians with tiles are
// compacted (one lane each forms the exact shape), their tile rows are numbered across the block
// (one lane per row forms the row's tile-column interval, in chunks of 256 rows), and (kEmit) each
// chunk's pairs are written one per lane: the block's keys are one contiguous run of the pair
// array (the offsets are in rank order), so consecutive lanes write consecutive keys.
//   kEmit = false: the exact-mode pair count of every rank (the rows' interval lengths summed);
//   kEmit = true:  the keys, and the block's counts of their tile digits (the per-view histograms
//                  of the pair sort's passes).
// (The previous form, one thread per Gaussian walking its own rows and tiles, kept 7 of 32 lanes
// busy on 2 x 1920x1080.)
template <bool kEmit>
__global__ void __launch_bounds__(kEmitThreads) pairs_kernel(int32_t G, RenderConsts rc, int H, int W,
                                                             const float* __restrict__ records,
                                                             const int4* __restrict__ rects,
                                                             const uint32_t* __restrict__ offsets, uint32_t n_pairs,
                                                             uint64_t* __restrict__ keys, uint32_t* __restrict__ hist,
                                                             int passes, uint32_t* __restrict__ counts,
                                                             int32_t* __restrict__ status) {
  __shared__ uint32_t s_hist[kEmit ? kMaxTilePasses : 1][256];
  __shared__ ExactShape s_shape[kEmitThreads];  // compacted Gaussians
  __shared__ int4 s_rect[kEmitThreads];
  __shared__ uint32_t s_rank[kEmitThreads], s_count[kEmitThreads], s_done[kEmitThreads];
  __shared__ uint32_t s_rowbase[kEmitThreads + 1];  // first row item of each compacted Gaussian
  __shared__ uint32_t s_scan[kEmitThreads];         // a chunk's row items: first pair (chunk-relative)
  __shared__ int s_tx0[kEmitThreads], s_ty[kEmitThreads];
  __shared__ uint16_t s_ci[kEmitThreads];
  __shared__ uint32_t s_warp[kEmitThreads / 32];
  __shared__ uint32_t s_first_key;
  const int tid = threadIdx.x, lane = tid & 31;
  if (kEmit)
    for (int k = tid; k < kMaxTilePasses * 256; k += kEmitThreads) s_hist[k / 256][k % 256] = 0u;
  const uint32_t b = blockIdx.y;
  const uint32_t r = blockIdx.x * kEmitThreads + tid;
  const size_t i = size_t(b) * G + r;
  const bool ellipse = !rc.compat && rc.ellipse;
  bool active;
  uint32_t start = 0, end = 0;
  int4 rc4 = make_int4(1, 1, 0, 0);
  if (kEmit) {
    start = r < uint32_t(G) ? offsets[i] : 0u;
    end = r < uint32_t(G) ? offsets[i + 1] : 0u;
    active = end > start;
    if (tid == 0) s_first_key = start;  // the block's keys begin at its first rank's offset
  } else {
    if (r < uint32_t(G)) rc4 = rects[i];
    active = rc4.x <= rc4.z && rc4.y <= rc4.w;
  }

  // 1. compact the Gaussians with tiles (rank order kept)
  const uint32_t bal = __ballot_sync(0xffffffffu, active);
  uint32_t n_active;
  const uint32_t ci_base = emit_block_scan(lane == 0 ? uint32_t(__popc(bal)) : 0u, s_warp, &n_active);
  const uint32_t my_ci = __shfl_sync(0xffffffffu, ci_base, 0) + __popc(bal & ((1u << lane) - 1u));
  if (active) {
    s_rank[my_ci] = r;
    s_count[my_ci] = end - start;
  }
  __syncthreads();

  // 2. one lane per compacted Gaussian: its shape and tile rows
  uint32_t rows = 0;
  if (uint32_t(tid) < n_active) {
    const size_t gi = size_t(b) * G + s_rank[tid];
    const int4 q4 = rects[gi];
    s_rect[tid] = q4;
    s_done[tid] = 0u;
    bool ok = q4.x <= q4.z && q4.y <= q4.w;
    if (ok && ellipse) {
      const float4* rec = reinterpret_cast<const float4*>(records + gi * GSB_RECORD_FLOATS);
      const float4 r0 = rec[0], r1 = rec[1];
      ok = exact_shape(r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, rc.alpha_cutoff, H, W, rc.pixel_center, &s_shape[tid]);
    }
    rows = ok ? uint32_t(q4.w - q4.y + 1) : 0u;
  }
  uint32_t total_rows;
  const uint32_t rb = emit_block_scan(rows, s_warp, &total_rows);
  if (uint32_t(tid) < n_active) s_rowbase[tid] = rb;
  if (tid == 0) s_rowbase[n_active] = total_rows;
  __syncthreads();

  // 3. row items in chunks of one per lane, then (kEmit) the chunk's pairs one per lane
  const uint64_t view_base = uint64_t(b) * rc.n_tiles;
  for (uint32_t chunk = 0; chunk < total_rows; chunk += kEmitThreads) {
    const uint32_t item = chunk + uint32_t(tid);
    uint32_t cnt = 0;
    int ci = 0, tx0 = 0, ty = 0;
    if (item < total_rows) {
      ci = emit_find(s_rowbase, int(n_active), item);
      const int4 q4 = s_rect[ci];
      ty = q4.y + int(item - s_rowbase[ci]);
      int tx1 = q4.z;
      tx0 = q4.x;
      const bool has = ellipse ? exact_row_pairs(s_shape[ci], ty, rc.tile, rc.pixel_center, &tx0, &tx1) : true;
      cnt = has ? uint32_t(tx1 - tx0 + 1) : 0u;
      if (cnt) atomicAdd(&s_done[ci], cnt);
    }
    if constexpr (kEmit) {
      uint32_t chunk_pairs;
      const uint32_t excl = emit_block_scan(cnt, s_warp, &chunk_pairs);
      s_scan[tid] = excl;
      s_tx0[tid] = tx0;
      s_ty[tid] = ty;
      s_ci[tid] = uint16_t(ci);
      __syncthreads();
      const uint32_t n_items = min(uint32_t(kEmitThreads), total_rows - chunk);
      const uint32_t key0 = s_first_key;
      for (uint32_t p = tid; p < chunk_pairs; p += kEmitThreads) {
        const int j = emit_find(s_scan, int(n_items), p);
        const uint32_t t = uint32_t(s_ty[j] * rc.tiles_x + s_tx0[j] + int(p - s_scan[j]));
        const uint32_t k = key0 + p;
        if (k < n_pairs) {
          keys[k] = ((view_base + t) << 32) | s_rank[s_ci[j]];
          for (int q = 0; q < passes; ++q) atomicAdd(&s_hist[q][(t >> (8 * q)) & 0xffu], 1u);
        }
      }
      __syncthreads();
      if (tid == 0) s_first_key = key0 + chunk_pairs;
    }
  }
  __syncthreads();
  if constexpr (kEmit) {
    // every Gaussian wrote exactly the pairs it was counted for
    if (uint32_t(tid) < n_active && s_done[tid] != s_count[tid])
      record_error(status, GSB_ERR_KEY_OVERFLOW, int(size_t(b) * G + s_rank[tid]));
    uint32_t* h = hist + size_t(b) * passes * 256;
    for (int k = tid; k < passes * 256; k += kEmitThreads) {
      const uint32_t c = s_hist[k / 256][k % 256];
      if (c) atomicAdd(h + k, c);
    }
  } else {
    if (r < uint32_t(G)) counts[i] = active ? s_done[my_ci] : 0u;
  }
}

// Run boundaries of the sorted keys: thread j reads keys 2j and 2j + 1 (one 16-byte load when the
// array is 16-byte aligned) and
// takes its neighbours' tiles from the adjacent lanes (lanes 0 and 31 read the one key beyond the
// warp), so every key is read once.  The loop bound is uniform over a block: every lane reaches the
// shuffles.
__global__ void tile_ranges_kernel(const uint64_t* __restrict__ keys, uint32_t cap,
                                   const uint32_t* __restrict__ n_dev, uint32_t* __restrict__ ranges,
                                   size_t n_ranges, int32_t* __restrict__ status, int aligned16) {
  uint32_t n = cap;
  if (n_dev) {
    const uint32_t count = *n_dev;
    if (count > cap && blockIdx.x == 0 && threadIdx.x == 0) record_error(status, GSB_ERR_CAPACITY, int(cap));
    n = min(cap, count);
  }
  constexpr uint32_t kNone = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  const uint32_t n2 = (n + 1u) / 2u;
  for (uint32_t base = blockIdx.x * blockDim.x; base < n2; base += gridDim.x * blockDim.x) {
    const uint32_t i = 2u * (base + threadIdx.x);
    uint32_t t0 = kNone, t1 = kNone;
    if (i + 1u < n) {
      if (aligned16) {
        const ulonglong2 v = *reinterpret_cast<const ulonglong2*>(keys + i);
        t0 = uint32_t(v.x >> 32), t1 = uint32_t(v.y >> 32);
      } else {
        t0 = uint32_t(keys[i] >> 32), t1 = uint32_t(keys[i + 1u] >> 32);
      }
    } else if (i < n) {
      t0 = uint32_t(keys[i] >> 32);
    }
    uint32_t prev = __shfl_up_sync(0xffffffffu, t1, 1);    // tile of key i - 1
    uint32_t next = __shfl_down_sync(0xffffffffu, t0, 1);  // tile of key i + 2
    if (lane == 0 && i > 0u && i < n) prev = uint32_t(keys[i - 1u] >> 32);
    if (lane == 31 && i + 2u < n) next = uint32_t(keys[i + 2u] >> 32);
    if (i < n && t0 < n_ranges) {
      if (i == 0u || prev != t0) ranges[size_t(t0) * 2] = i;
      if (i + 1u == n || t1 != t0) ranges[size_t(t0) * 2 + 1] = i + 1u;
    }
    if (i + 1u < n && t1 < n_ranges) {
      if (t0 != t1) ranges[size_t(t1) * 2] = i + 1u;
      if (i + 2u == n || next != t1) ranges[size_t(t1) * 2 + 1] = i + 2u;
    }
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
  const dim3 grid(unsigned((size_t(G) + kEmitThreads - 1) / kEmitThreads), unsigned(B));
  note_launch();
  pairs_kernel<true><<<grid, kEmitThreads, 0, st>>>(G, rc, H, W, records, rects, offsets, n_pairs, keys, hist, passes,
                                                    nullptr, status);
  return launch_status();
}

gsb_status launch_count_pairs(int32_t B, int32_t G, const RenderConsts& rc, int H, int W, const float* records,
                              const int4* rects, uint32_t* counts, int32_t* status, cudaStream_t st) {
  if (B == 0 || G == 0) return GSB_OK;
  const dim3 grid(unsigned((size_t(G) + kEmitThreads - 1) / kEmitThreads), unsigned(B));
  note_launch();
  pairs_kernel<false><<<grid, kEmitThreads, 0, st>>>(G, rc, H, W, records, rects, nullptr, 0u, nullptr, nullptr, 0,
                                                     counts, status);
  return launch_status();
}

gsb_status launch_tile_ranges(const uint64_t* keys, uint32_t n, const uint32_t* n_dev, uint32_t* ranges,
                              size_t n_ranges, int32_t* status, cudaStream_t st) {
  if (cudaMemsetAsync(ranges, 0, n_ranges * 2 * sizeof(uint32_t), st)) return GSB_ERR_CUDA;
  if (n == 0 && !n_dev) return GSB_OK;
  const int grid = int(std::min<uint32_t>(std::max<uint32_t>((n + 255) / 256, 1u), 148u * 32u));
  note_launch();
  tile_ranges_kernel<<<grid, 256, 0, st>>>(keys, n, n_dev, ranges, n_ranges, status,
                                           int(reinterpret_cast<uintptr_t>(keys) % 16 == 0));
  return launch_status();
}

}  // namespace gsb
