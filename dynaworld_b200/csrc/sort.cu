// Hand-written LSD radix sort (one-sweep: one read and one write of the keys per 8-bit digit,
// partition prefixes by decoupled look-back) and a three-phase exclusive prefix scan.
//
// Look-back waits are bounded: a partition that waits more than kSpinLimit polls (or the limit a
// launch gives in Segments::spin_limit) records GSB_ERR_TIMEOUT in the workspace status word and
// carries on with the prefix it has, so a bug can corrupt the output but never hangs the GPU.  Partitions take their index from an atomic
// counter in start order, so a partition only ever waits on partitions that are already running.
#include <cstring>

#include "gsb_common.cuh"
#include "gsb_internal.h"

namespace gsb {

constexpr int kSortThreads = 256;
constexpr int kSortWarps = kSortThreads / 32;
constexpr uint32_t kFlagAgg = 1u << 30;
constexpr uint32_t kFlagIncl = 2u << 30;
constexpr uint32_t kCountMask = (1u << 30) - 1u;
constexpr int kSpinLimit = 1 << 22;

template <typename K>
struct SortTraits;
// Keys per thread of a partition.  32-bit keys (the depth order, the tile launch order): 8, measured
// on one B200 against 16 / 12 (depth order, 8 x 200k keys: 0.188 / 0.179 ms -> 0.180 ms; 16 x 32768
// keys: 0.084 / 0.090 -> 0.084): twice the partitions fill the GPU at these sizes.
template <>
struct SortTraits<uint32_t> {
  static constexpr int kItems = 8;
  static constexpr int kItemsVals = 8;
};
template <>
struct SortTraits<uint64_t> {
  // keys only: 14 (measured on 8 x 1920x1080 with four CTAs per SM, pair sort of the bin stage:
  // 12 keys 2.28 ms, 14 keys 2.24 ms, 16 keys slower with 108 bytes of register spills)
  static constexpr int kItems = 14;
  static constexpr int kItemsVals = 12;  // 12 B per item staged: the static shared-memory limit
};
template <typename K, bool kVals>
__host__ __device__ constexpr int items_of() {
  return kVals ? SortTraits<K>::kItemsVals : SortTraits<K>::kItems;
}
// Predecessor words a look-back reads at once (measured on 8 x 1920x1080 against 4, 8 and 32 at
// the register counts each gave; the window mostly matters through the registers it takes).
constexpr int kLookbackWindow = 16;

// Look-back words hold a partition's flag and digit count in one 32-bit word, so a reader needs
// no ordering with any other data: relaxed gpu-scope accesses suffice, and a thread can keep a
// whole window of predecessors' words in flight at once.
__device__ __forceinline__ uint32_t ld_relaxed_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ void st_relaxed_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// Histograms of every pass's digit, all passes in one read of the keys.
template <typename K>
__global__ void __launch_bounds__(kSortThreads) radix_hist_kernel(const K* __restrict__ keys, uint32_t n,
                                                                  int bit_lo, int bit_hi, int passes,
                                                                  uint32_t* __restrict__ hist,
                                                                  const uint32_t* __restrict__ n_dev) {
  __shared__ uint32_t s_hist[8][256];
  if (n_dev) n = min(n, *n_dev);
  for (int i = threadIdx.x; i < passes * 256; i += blockDim.x) s_hist[i / 256][i % 256] = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const uint32_t stride = gridDim.x * blockDim.x;
  for (uint32_t base = blockIdx.x * blockDim.x; base < n; base += stride) {
    const uint32_t i = base + threadIdx.x;
    const bool valid = i < n;
    const K k = valid ? keys[i] : K(0);
    for (int p = 0; p < passes; ++p) {
      const int shift = bit_lo + 8 * p;
      const int nbits = min(8, bit_hi - shift);
      const uint32_t d = valid ? uint32_t((k >> shift) & K((1u << nbits) - 1u)) : 0xffffffffu;
      const uint32_t peers = __match_any_sync(0xffffffffu, d);
      if (valid && lane == __ffs(peers) - 1) atomicAdd(&s_hist[p][d], __popc(peers));
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < passes * 256; i += blockDim.x) {
    const uint32_t c = s_hist[i / 256][i % 256];
    if (c) atomicAdd(&hist[i], c);
  }
}

// Exclusive scan of 256 values held one per thread (blockDim == 256); returns the total too.
__device__ __forceinline__ uint32_t block_excl_scan_256(uint32_t v, uint32_t* s_tmp, uint32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_tmp[warp] = x;
  __syncthreads();
  uint32_t warp_base = 0, all = 0;
  for (int w = 0; w < kSortWarps; ++w) {
    const uint32_t t = s_tmp[w];
    if (w < warp) warp_base += t;
    all += t;
  }
  __syncthreads();
  if (total) *total = all;
  return warp_base + x - v;
}

// How the keys split into independently sorted segments (kSegNone: one sequence).
enum SegMode { kSegNone = 0, kSegFixed = 1, kSegRuns = 2 };
struct Segments {
  uint32_t hist_stride;        // histogram words per segment (digit histograms per segment)
  uint32_t fixed_len;          // kSegFixed: segment length
  uint32_t parts_per_seg;      // kSegFixed: partitions per segment
  uint32_t n_seg;              // kSegRuns: segments
  const uint32_t* start;       // kSegRuns: [n_seg + 1] first key of each segment (device)
  const uint32_t* part_start;  // kSegRuns: [n_seg + 1] first partition of each segment (device)
  uint32_t key_stride;         // kSegRuns: the digits are those of (key >> 32) - segment * key_stride
  int32_t* ids_out;            // kSegFixed, last pass (may be NULL): write the values as ids_out[pos]
  int32_t* rank_out;           //   and the inverse rank_out[segment start + value] = pos - segment start
  uint32_t spin_limit;         // look-back polls before giving up (0: kSpinLimit)
};

// One LSD pass.  Partitions never straddle a segment and look back only within theirs; with
// segments the digit histograms are per segment.  kSegNone sorts n keys (or *n_dev, when given).
// Four CTAs per SM (64 registers): measured on 8 x 1920x1080, the pair sort (64-bit keys, 79
// registers uncapped, three CTAs per SM) bin stage 3.33 -> 2.40 ms; the depth order unchanged.
constexpr int kSortMinBlocks = 4;
template <typename K, bool kVals, int kSeg>
__global__ void __launch_bounds__(kSortThreads, kSortMinBlocks) onesweep_kernel(
    const K* __restrict__ keys_in, K* __restrict__ keys_out, const uint32_t* __restrict__ vals_in,
    uint32_t* __restrict__ vals_out, uint32_t n, int shift, int nbits, const uint32_t* __restrict__ hist,
    uint32_t* __restrict__ lookback, uint32_t* __restrict__ part_counter, int32_t* __restrict__ status,
    const uint32_t* __restrict__ n_dev, Segments sg) {
  constexpr int kItems = items_of<K, kVals>();
  if (kSeg == kSegNone && n_dev) n = min(n, *n_dev);  // partitions past the count find no key, write nothing
  constexpr uint32_t kPart = kSortThreads * kItems;
  __shared__ uint32_t s_part, s_seg;
  __shared__ uint32_t s_warp_hist[kSortWarps][256];
  __shared__ uint32_t s_base[256];
  __shared__ uint32_t s_local[256];
  __shared__ uint32_t s_tmp[kSortWarps];
  __shared__ K s_keys[kPart];
  __shared__ uint32_t s_vals[kVals ? kPart : 1];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    const uint32_t p = atomicAdd(part_counter, 1u);
    s_part = p;
    if (kSeg == kSegRuns) {  // the segment whose partitions hold p (empty segments have none)
      uint32_t a = 0, b = sg.n_seg;  // invariant: part_start[a] <= p < part_start[b] (or p is past all)
      if (p >= sg.part_start[sg.n_seg]) a = sg.n_seg;
      while (b - a > 1 && a < sg.n_seg) {
        const uint32_t m = (a + b) / 2;
        if (sg.part_start[m] <= p) a = m;
        else b = m;
      }
      s_seg = a;
    }
  }
  for (int w = 0; w < kSortWarps; ++w) s_warp_hist[w][tid] = 0;
  __syncthreads();
  const uint32_t part = s_part;
  if (kSeg == kSegRuns && s_seg >= sg.n_seg) return;  // a spare partition: the grid covers the worst case
  const uint32_t mask = (1u << nbits) - 1u;
  const uint32_t seg = kSeg == kSegRuns ? s_seg : 0u;
  const uint32_t key_base = kSeg == kSegRuns ? seg * sg.key_stride : 0u;
  auto digit_of = [&](K key) -> uint32_t {
    if (kSeg == kSegRuns) return ((uint32_t(uint64_t(key) >> 32) - key_base) >> shift) & mask;
    return uint32_t((key >> shift) & K(mask));
  };
  // this partition's keys [lo, hi) in the segment [seg_lo, seg_hi); first_part opens the segment
  uint32_t lo, hi, seg_lo, seg_hi, first_part;
  if (kSeg == kSegFixed) {
    const uint32_t sf = part / sg.parts_per_seg, lp = part - sf * sg.parts_per_seg;
    seg_lo = sf * sg.fixed_len;
    seg_hi = seg_lo + sg.fixed_len;
    lo = seg_lo + lp * kPart;
    hi = min(lo + kPart, seg_hi);
    first_part = part - lp;
    hist += size_t(sf) * sg.hist_stride;
  } else if (kSeg == kSegRuns) {
    seg_lo = sg.start[seg];
    seg_hi = max(sg.start[seg + 1], seg_lo);
    first_part = sg.part_start[seg];
    lo = seg_lo + (part - first_part) * kPart;
    hi = lo < seg_hi ? min(lo + kPart, seg_hi) : lo;
    hist += size_t(seg) * sg.hist_stride;
  } else {
    seg_lo = 0u, seg_hi = n, first_part = 0u;
    lo = part * kPart;
    hi = lo < n ? min(lo + kPart, n) : lo;
  }

  const uint32_t hist_word = hist[tid];  // this digit's count over the segment (read early)
  // Warp-striped load: warp w owns keys [lo + w*32*kItems, +32*kItems), item j of lane l is key
  // base + 32*j + l, so (j, lane) order is input order: the ranking below is stable.
  const uint32_t base = lo + warp * 32 * kItems + lane;
  K k[kItems];
  uint32_t v[kItems];
  uint32_t rank[kItems];
  uint32_t dig[kItems];
#pragma unroll
  for (int j = 0; j < kItems; ++j) {
    const uint32_t idx = base + 32 * j;
    const bool valid = idx < hi;
    k[j] = valid ? keys_in[idx] : K(0);
    if (kVals) v[j] = valid ? vals_in[idx] : 0u;
    dig[j] = valid ? digit_of(k[j]) : 0xffffffffu;
  }
#pragma unroll
  for (int j = 0; j < kItems; ++j) {
    const uint32_t d = dig[j];
    const uint32_t peers = __match_any_sync(0xffffffffu, d);
    uint32_t cnt = 0;
    if (d != 0xffffffffu) cnt = s_warp_hist[warp][d];
    __syncwarp();
    if (d != 0xffffffffu) {
      rank[j] = cnt + __popc(peers & lanemask_lt());
      if (lane == 31 - __clz(peers)) s_warp_hist[warp][d] = cnt + __popc(peers);
    }
    __syncwarp();
  }
  __syncthreads();

  // Per digit (one per thread): exclusive prefix over warps, partition total.
  uint32_t total = 0;
  for (int w = 0; w < kSortWarps; ++w) {
    const uint32_t c = s_warp_hist[w][tid];
    s_warp_hist[w][tid] = total;
    total += c;
  }
  // Publish this partition's digit count at once; its successors look back while it stages keys.
  uint32_t* my = lookback + size_t(part) * 256 + tid;
  st_relaxed_u32(my, (part == first_part ? kFlagIncl : kFlagAgg) | total);
  // Stage the partition in (digit, input) order (local positions need no global prefix).
  s_local[tid] = block_excl_scan_256(total, s_tmp, nullptr);
  __syncthreads();
#pragma unroll
  for (int j = 0; j < kItems; ++j) {
    const uint32_t d = dig[j];
    if (d == 0xffffffffu) continue;
    const uint32_t lpos = s_local[d] + s_warp_hist[warp][d] + rank[j];
    s_keys[lpos] = k[j];
    if (kVals) s_vals[lpos] = v[j];
  }
  const uint32_t digit_start = block_excl_scan_256(hist_word, s_tmp, nullptr);
  // Look back for the exclusive prefix: a window of predecessors' words per read (the wait for a
  // predecessor's inclusive count then ends after about one memory round trip, not one per
  // partition between this one and the last inclusive one), summing counts up to the nearest
  // inclusive word; a word not yet published is read again.
  uint32_t excl = 0;
  if (part > first_part) {  // partitions of this segment only: first_part's word is inclusive
    const uint32_t spin_limit = sg.spin_limit ? sg.spin_limit : uint32_t(kSpinLimit);
    uint32_t spins = 0;
    uint32_t p = part;  // the next window reads p - 1, p - 2, ...
    for (;;) {
      uint32_t w[kLookbackWindow];
#pragma unroll
      for (int i = 0; i < kLookbackWindow; ++i)
        w[i] = p >= first_part + 1u + uint32_t(i) ? ld_relaxed_u32(lookback + size_t(p - 1u - uint32_t(i)) * 256 + tid)
                                                   : kFlagIncl;
      uint32_t used = 0;
      bool found = false, waiting = false;
#pragma unroll
      for (int i = 0; i < kLookbackWindow; ++i) {
        if (found || waiting) continue;
        const uint32_t flag = w[i] & ~kCountMask;
        if (flag == 0u) {
          waiting = true;
          continue;
        }
        excl += w[i] & kCountMask;
        ++used;
        found = flag == kFlagIncl;
      }
      if (found) break;
      p -= used;
      if (waiting && ++spins > spin_limit) {
        record_error(status, GSB_ERR_TIMEOUT, int(part));
        break;
      }
    }
    st_relaxed_u32(my, kFlagIncl | ((excl + total) & kCountMask));
  }
  s_base[tid] = seg_lo + digit_start + excl;
  __syncthreads();
  const uint32_t n_valid = hi - lo;
  for (uint32_t i = tid; i < n_valid; i += kSortThreads) {
    const K key = s_keys[i];
    const uint32_t d = digit_of(key);
    const uint32_t pos = s_base[d] + (i - s_local[d]);
    if (pos >= seg_hi) {  // only after a timed-out look-back: never write outside the segment
      record_error(status, GSB_ERR_TIMEOUT, int(part));
      continue;
    }
    if (kSeg == kSegFixed && kVals && sg.ids_out) {  // the permutation and its inverse, not the keys
      const uint32_t val = s_vals[i];
      sg.ids_out[pos] = int32_t(val);
      if (val < seg_hi - seg_lo) sg.rank_out[seg_lo + val] = int32_t(pos - seg_lo);
      continue;
    }
    keys_out[pos] = key;
    if (kVals) vals_out[pos] = s_vals[i];
  }
}

// ---- host driver ---------------------------------------------------------------------------

static uint32_t parts_for(uint32_t n, int key_bytes, bool with_values) {
  const int items = key_bytes == 8 ? (with_values ? items_of<uint64_t, true>() : items_of<uint64_t, false>())
                                   : (with_values ? items_of<uint32_t, true>() : items_of<uint32_t, false>());
  const uint32_t part = kSortThreads * uint32_t(items);
  return (n + part - 1) / part;
}

size_t radix_sort_workspace(uint32_t n, int key_bytes, int with_values) {
  const int passes = 8;  // worst case (64-bit keys)
  const uint32_t parts = parts_for(n, key_bytes, with_values != 0);
  Carver c(nullptr, 0);
  c.take<WorkspaceHeader>(1);
  c.take<uint32_t>(size_t(passes) * 256);          // histograms
  c.take<uint32_t>(size_t(passes));                // partition counters
  c.take<uint32_t>(size_t(passes) * parts * 256);  // look-back
  c.take<char>(size_t(n) * key_bytes);             // ping-pong keys
  if (with_values) c.take<uint32_t>(n);            // ping-pong values
  return c.used;
}

template <typename K>
static gsb_status radix_sort_t(const K* keys_in, K* keys_out, const uint32_t* vals_in, uint32_t* vals_out,
                               uint32_t n, int bit_lo, int bit_hi, void* ws, size_t ws_bytes,
                               cudaStream_t stream, int32_t* status, const uint32_t* n_dev) {
  const int passes = (bit_hi - bit_lo + 7) / 8;
  const bool with_vals = vals_in != nullptr;
  if (n == 0) return GSB_OK;
  if (passes <= 0) {  // one bucket: the input order is the output (copies the capacity)
    if (cudaMemcpyAsync(keys_out, keys_in, size_t(n) * sizeof(K), cudaMemcpyDeviceToDevice, stream)) return GSB_ERR_CUDA;
    if (with_vals && cudaMemcpyAsync(vals_out, vals_in, size_t(n) * 4, cudaMemcpyDeviceToDevice, stream)) return GSB_ERR_CUDA;
    return GSB_OK;
  }
  const uint32_t parts = parts_for(n, sizeof(K), with_vals);
  Carver c(ws, ws_bytes);
  c.take<WorkspaceHeader>(1);
  uint32_t* hist = c.take<uint32_t>(size_t(8) * 256);
  uint32_t* counters = c.take<uint32_t>(8);
  uint32_t* lookback = c.take<uint32_t>(size_t(8) * parts * 256);
  K* alt_keys = reinterpret_cast<K*>(c.take<char>(size_t(n) * sizeof(K)));
  uint32_t* alt_vals = with_vals ? c.take<uint32_t>(n) : nullptr;
  if (!c.ok()) return GSB_ERR_WORKSPACE;
  // hist, counters and the look-back of the passes run are contiguous: one memset clears them.
  const size_t clear_bytes =
      reinterpret_cast<char*>(lookback + size_t(passes) * parts * 256) - reinterpret_cast<char*>(hist);
  if (cudaMemsetAsync(hist, 0, clear_bytes, stream)) return GSB_ERR_CUDA;

  const int hist_blocks = int(std::min<uint32_t>((n + kSortThreads - 1) / kSortThreads, 148u * 8u));
  note_launch();
  radix_hist_kernel<K><<<hist_blocks, kSortThreads, 0, stream>>>(keys_in, n, bit_lo, bit_hi, passes, hist, n_dev);
  const K* src_k = keys_in;
  const uint32_t* src_v = vals_in;
  for (int p = 0; p < passes; ++p) {
    const bool to_out = ((passes - 1 - p) % 2) == 0;
    K* dst_k = to_out ? keys_out : alt_keys;
    uint32_t* dst_v = with_vals ? (to_out ? vals_out : alt_vals) : nullptr;
    const int shift = bit_lo + 8 * p;
    const int nbits = std::min(8, bit_hi - shift);
    if (with_vals) {
      note_launch();
      onesweep_kernel<K, true, kSegNone><<<parts, kSortThreads, 0, stream>>>(
          src_k, dst_k, src_v, dst_v, n, shift, nbits, hist + 256 * p, lookback + size_t(p) * parts * 256, counters + p,
          status, n_dev, Segments{});
    } else {
      note_launch();
      onesweep_kernel<K, false, kSegNone><<<parts, kSortThreads, 0, stream>>>(
          src_k, dst_k, nullptr, nullptr, n, shift, nbits, hist + 256 * p, lookback + size_t(p) * parts * 256,
          counters + p, status, n_dev, Segments{});
    }
    src_k = dst_k;
    src_v = dst_v;
  }
  return launch_status();
}

gsb_status radix_sort(const void* keys_in, void* keys_out, const uint32_t* vals_in, uint32_t* vals_out, uint32_t n,
                      int key_bytes, int bit_lo, int bit_hi, void* ws, size_t ws_bytes, cudaStream_t stream,
                      int32_t* status, const uint32_t* n_dev) {
  if (n >= (1u << 30)) return GSB_ERR_KEY_OVERFLOW;
  if (bit_lo < 0 || bit_hi > key_bytes * 8 || bit_hi < bit_lo) return GSB_ERR_ARG;
  if ((vals_in == nullptr) != (vals_out == nullptr)) return GSB_ERR_ARG;
  if (key_bytes == 4)
    return radix_sort_t<uint32_t>(static_cast<const uint32_t*>(keys_in), static_cast<uint32_t*>(keys_out), vals_in,
                                  vals_out, n, bit_lo, bit_hi, ws, ws_bytes, stream, status, n_dev);
  if (key_bytes == 8)
    return radix_sort_t<uint64_t>(static_cast<const uint64_t*>(keys_in), static_cast<uint64_t*>(keys_out), vals_in,
                                  vals_out, n, bit_lo, bit_hi, ws, ws_bytes, stream, status, n_dev);
  return GSB_ERR_ARG;
}

__global__ void set_word_kernel(uint32_t* p, uint32_t v) { *p = v; }

// Test hook for the bounded look-back: one 8-bit pass over n 32-bit keys in which the first
// partition never runs (the partition counter starts at 1 and the grid has one CTA fewer), so the
// partition after it waits for a predecessor that never publishes.  Its wait gives up after
// spin_limit polls and records GSB_ERR_TIMEOUT; the partitions after it wait at most as long.  All
// writes stay inside keys_out[0, n) (positions are short by the missing partition's counts), and
// the keys of the first partition are not written.  Workspace: radix_sort_workspace(n, 4, 0).
gsb_status sort_lookback_timeout_probe(const uint32_t* keys_in, uint32_t* keys_out, uint32_t n, uint32_t spin_limit,
                                       void* ws, size_t ws_bytes, cudaStream_t stream, int32_t* status) {
  const uint32_t parts = parts_for(n, 4, false);
  if (parts < 2 || n >= (1u << 30)) return GSB_ERR_SHAPE;
  Carver c(ws, ws_bytes);
  c.take<WorkspaceHeader>(1);
  uint32_t* hist = c.take<uint32_t>(size_t(8) * 256);
  uint32_t* counters = c.take<uint32_t>(8);
  uint32_t* lookback = c.take<uint32_t>(size_t(8) * parts * 256);
  if (!c.ok() || !ws) return GSB_ERR_WORKSPACE;
  const size_t clear_bytes = reinterpret_cast<char*>(lookback + size_t(parts) * 256) - reinterpret_cast<char*>(hist);
  if (cudaMemsetAsync(hist, 0, clear_bytes, stream)) return launch_status();
  const int hist_blocks = int(std::min<uint32_t>((n + kSortThreads - 1) / kSortThreads, 148u * 8u));
  note_launch();
  radix_hist_kernel<uint32_t><<<hist_blocks, kSortThreads, 0, stream>>>(keys_in, n, 0, 8, 1, hist, nullptr);
  note_launch();
  set_word_kernel<<<1, 1, 0, stream>>>(counters, 1u);
  Segments sg{};
  sg.spin_limit = spin_limit ? spin_limit : 1u;
  note_launch();
  onesweep_kernel<uint32_t, false, kSegNone><<<parts - 1, kSortThreads, 0, stream>>>(
      keys_in, keys_out, nullptr, nullptr, n, 0, 8, hist, lookback, counters, status, nullptr, sg);
  return launch_status();
}

// ---- segmented sort: independent runs of 32-bit keys (the per-view depth order) --------------
//
// n_seg segments of seg_len keys, each sorted on its own (stable, ascending, all 32 bits: four
// passes).  Partitions never straddle a segment and look back only within theirs; the digit
// histograms are per segment and are accumulated by the kernel that writes the keys (it gets
// their address from segmented_sort_prepare), so no pass re-reads the keys to count them.

constexpr int kSegPasses = 4;

static uint32_t seg_parts(uint32_t seg_len) {
  const uint32_t part = kSortThreads * items_of<uint32_t, true>();
  return (seg_len + part - 1) / part;
}

size_t segmented_sort_workspace(uint32_t n_seg, uint32_t seg_len) {
  const size_t parts = size_t(n_seg) * seg_parts(seg_len);
  Carver c(nullptr, 0);
  c.take<WorkspaceHeader>(1);
  c.take<uint32_t>(size_t(n_seg) * kSegPasses * 256);   // histograms [seg][pass][digit]
  c.take<uint32_t>(kSegPasses);                          // partition counters
  c.take<uint32_t>(size_t(kSegPasses) * parts * 256);   // look-back
  c.take<uint32_t>(size_t(n_seg) * seg_len);            // ping-pong keys
  c.take<uint32_t>(size_t(n_seg) * seg_len);            // ping-pong values
  return c.used;
}

struct SegWorkspace {
  uint32_t *hist, *counters, *lookback, *alt_keys, *alt_vals;
  size_t clear_bytes;
};

static bool seg_carve(void* ws, size_t ws_bytes, uint32_t n_seg, uint32_t seg_len, SegWorkspace& w) {
  const size_t parts = size_t(n_seg) * seg_parts(seg_len);
  Carver c(ws, ws_bytes);
  c.take<WorkspaceHeader>(1);
  w.hist = c.take<uint32_t>(size_t(n_seg) * kSegPasses * 256);
  w.counters = c.take<uint32_t>(kSegPasses);
  w.lookback = c.take<uint32_t>(size_t(kSegPasses) * parts * 256);
  w.alt_keys = c.take<uint32_t>(size_t(n_seg) * seg_len);
  w.alt_vals = c.take<uint32_t>(size_t(n_seg) * seg_len);
  w.clear_bytes = reinterpret_cast<char*>(w.lookback + size_t(kSegPasses) * parts * 256) -
                  reinterpret_cast<char*>(w.hist);  // hist, counters, look-back are contiguous
  return c.ok() && ws != nullptr;
}

gsb_status segmented_sort_prepare(void* ws, size_t ws_bytes, uint32_t n_seg, uint32_t seg_len, cudaStream_t stream,
                                  uint32_t** hist) {
  SegWorkspace w;
  if (!seg_carve(ws, ws_bytes, n_seg, seg_len, w)) return GSB_ERR_WORKSPACE;
  if (cudaMemsetAsync(w.hist, 0, w.clear_bytes, stream)) return GSB_ERR_CUDA;
  *hist = w.hist;
  return GSB_OK;
}

gsb_status segmented_sort_run(const uint32_t* keys_in, uint32_t* keys_out, const uint32_t* vals_in, uint32_t* vals_out,
                              uint32_t n_seg, uint32_t seg_len, void* ws, size_t ws_bytes, cudaStream_t stream,
                              int32_t* status, int32_t* ids_out, int32_t* rank_out) {
  if ((ids_out == nullptr) != (rank_out == nullptr)) return GSB_ERR_ARG;
  if (size_t(n_seg) * seg_len >= (size_t(1) << 30)) return GSB_ERR_KEY_OVERFLOW;
  if (n_seg == 0 || seg_len == 0) return GSB_OK;
  SegWorkspace w;
  if (!seg_carve(ws, ws_bytes, n_seg, seg_len, w)) return GSB_ERR_WORKSPACE;
  const uint32_t pps = seg_parts(seg_len);
  const uint32_t parts = n_seg * pps;
  const uint32_t* src_k = keys_in;
  const uint32_t* src_v = vals_in;
  for (int p = 0; p < kSegPasses; ++p) {
    const bool to_out = ((kSegPasses - 1 - p) % 2) == 0;
    uint32_t* dst_k = to_out ? keys_out : w.alt_keys;
    uint32_t* dst_v = to_out ? vals_out : w.alt_vals;
    note_launch();
    Segments sg{};
    sg.hist_stride = uint32_t(kSegPasses * 256), sg.fixed_len = seg_len, sg.parts_per_seg = pps;
    if (p == kSegPasses - 1) sg.ids_out = ids_out, sg.rank_out = rank_out;
    onesweep_kernel<uint32_t, true, kSegFixed><<<parts, kSortThreads, 0, stream>>>(
        src_k, dst_k, src_v, dst_v, n_seg * seg_len, 8 * p, 8, w.hist + 256 * p, w.lookback + size_t(p) * parts * 256,
        w.counters + p, status, nullptr, sg);
    src_k = dst_k;
    src_v = dst_v;
  }
  return launch_status();
}

// ---- pair keys: runs of one view each, sorted by tile ------------------------------------------
//
// The pair keys ((view * n_tiles + tile) << 32 | depth rank) arrive in (view, rank) order, so each
// view's pairs are a contiguous run, starting at pair_offsets[view * G].  Sorting every run by its
// tile index alone (stable) gives the (view, tile, rank) order with ceil(log2(n_tiles) / 8) passes
// instead of the passes of log2(B * n_tiles) bits.  The run bounds come from the device offsets
// (clipped to the keys' capacity), so the grid is sized for the worst case and spare partitions
// return at once.

constexpr uint32_t kPairPart = kSortThreads * items_of<uint64_t, false>();

static int pair_passes(uint32_t n_tiles) { return (bits_for(n_tiles) + 7) / 8; }
int pair_sort_passes(uint32_t n_tiles) { return pair_passes(n_tiles); }

static uint32_t pair_parts_max(uint32_t cap, uint32_t n_views) {
  return (cap + kPairPart - 1) / kPairPart + n_views;  // each run adds at most one partial partition
}

size_t pair_sort_workspace(uint32_t cap, uint32_t n_views, uint32_t n_tiles) {
  const int passes = std::max(pair_passes(n_tiles), 1);
  Carver c(nullptr, 0);
  c.take<WorkspaceHeader>(1);
  c.take<uint32_t>(size_t(n_views) * passes * 256);                             // histograms [view][pass][digit]
  c.take<uint32_t>(passes);                                                      // partition counters
  c.take<uint32_t>(size_t(passes) * pair_parts_max(cap, n_views) * 256);         // look-back
  c.take<uint32_t>(size_t(n_views) + 1);                                         // run starts
  c.take<uint32_t>(size_t(n_views) + 1);                                         // first partition of each run
  c.take<uint64_t>(std::max<uint32_t>(cap, 1));                                  // ping-pong keys
  return c.used;
}

struct PairWorkspace {
  uint32_t *hist, *counters, *lookback, *start, *part_start;
  uint64_t* alt;
  size_t clear_bytes;
};

static bool pair_carve(void* ws, size_t ws_bytes, uint32_t cap, uint32_t n_views, uint32_t n_tiles, PairWorkspace& w) {
  const int passes = std::max(pair_passes(n_tiles), 1);
  Carver c(ws, ws_bytes);
  c.take<WorkspaceHeader>(1);
  w.hist = c.take<uint32_t>(size_t(n_views) * passes * 256);
  w.counters = c.take<uint32_t>(passes);
  w.lookback = c.take<uint32_t>(size_t(passes) * pair_parts_max(cap, n_views) * 256);
  w.start = c.take<uint32_t>(size_t(n_views) + 1);
  w.part_start = c.take<uint32_t>(size_t(n_views) + 1);
  w.alt = c.take<uint64_t>(std::max<uint32_t>(cap, 1));
  w.clear_bytes = reinterpret_cast<char*>(w.lookback + size_t(passes) * pair_parts_max(cap, n_views) * 256) -
                  reinterpret_cast<char*>(w.hist);
  return c.ok() && ws != nullptr;
}

// Run bounds start[v] = min(pair_offsets[v * G], cap) (v <= n_views) and the exclusive prefix of
// the runs' partition counts; one block, runs in chunks of one per thread.
__global__ void __launch_bounds__(kSortThreads) pair_runs_kernel(const uint32_t* __restrict__ offsets, uint32_t n_views,
                                                                uint32_t G, uint32_t cap, uint32_t* __restrict__ start,
                                                                uint32_t* __restrict__ part_start) {
  __shared__ uint32_t s_tmp[kSortWarps];
  uint32_t carry = 0;
  for (uint32_t v0 = 0; v0 <= n_views; v0 += kSortThreads) {
    const uint32_t v = v0 + threadIdx.x;
    uint32_t parts = 0;
    if (v <= n_views) {
      const uint32_t a = min(offsets[size_t(v) * G], cap);
      start[v] = a;
      if (v < n_views) {
        const uint32_t b = min(offsets[size_t(v + 1) * G], cap);
        parts = b > a ? (b - a + kPairPart - 1) / kPairPart : 0u;
      }
    }
    uint32_t total = 0;
    const uint32_t ex = block_excl_scan_256(parts, s_tmp, &total);
    if (v <= n_views) part_start[v] = carry + ex;
    carry += total;
  }
}

gsb_status pair_sort_prepare(void* ws, size_t ws_bytes, uint32_t cap, uint32_t n_views, uint32_t n_tiles,
                             cudaStream_t stream, uint32_t** hist) {
  PairWorkspace w;
  if (!pair_carve(ws, ws_bytes, cap, n_views, n_tiles, w)) return GSB_ERR_WORKSPACE;
  if (cudaMemsetAsync(w.hist, 0, w.clear_bytes, stream)) return GSB_ERR_CUDA;
  *hist = w.hist;
  return GSB_OK;
}

// With one pass (at most 256 tiles per view) the pass's digit counts are the tile list lengths:
// view blockIdx.x's tile ranges are its run start plus their exclusive prefix, and the launch-order
// keys (longest first) follow from the same counts, so no kernel re-reads the sorted keys.
__global__ void __launch_bounds__(kSortThreads) run_tile_ranges_kernel(
    const uint32_t* __restrict__ hist, const uint32_t* __restrict__ start, uint32_t n_tiles,
    uint32_t* __restrict__ ranges, uint32_t* __restrict__ order_keys, uint32_t* __restrict__ order_vals,
    const uint32_t* __restrict__ n_dev, uint32_t cap, int32_t* __restrict__ status) {
  __shared__ uint32_t s_tmp[kSortWarps];
  const uint32_t v = blockIdx.x, t = threadIdx.x;
  if (v == 0 && t == 0 && *n_dev > cap) record_error(status, GSB_ERR_CAPACITY, int(cap));
  const uint32_t c = t < n_tiles ? hist[size_t(v) * 256 + t] : 0u;
  const uint32_t before = block_excl_scan_256(c, s_tmp, nullptr);
  if (t < n_tiles) {
    const size_t slot = size_t(v) * n_tiles + t;
    ranges[slot * 2] = start[v] + before;
    ranges[slot * 2 + 1] = start[v] + before + c;
    if (order_keys) {
      order_keys[slot] = 255u - length_class(c);
      order_vals[slot] = uint32_t(slot);
    }
  }
}

gsb_status pair_sort_run(const uint64_t* keys_in, uint64_t* keys_out, uint32_t cap, uint32_t n_views, uint32_t n_tiles,
                         int32_t G, const uint32_t* pair_offsets, void* ws, size_t ws_bytes, cudaStream_t stream,
                         int32_t* status, uint32_t* tile_ranges, uint32_t* order_keys, uint32_t* order_vals,
                         bool* ranges_done) {
  *ranges_done = false;
  if (cap == 0) return GSB_OK;
  PairWorkspace w;
  if (!pair_carve(ws, ws_bytes, cap, n_views, n_tiles, w)) return GSB_ERR_WORKSPACE;
  const int passes = pair_passes(n_tiles);
  if (passes == 0) {  // one tile per view: the runs are in order already
    return cudaMemcpyAsync(keys_out, keys_in, size_t(cap) * 8, cudaMemcpyDeviceToDevice, stream) ? GSB_ERR_CUDA
                                                                                                    : GSB_OK;
  }
  note_launch();
  pair_runs_kernel<<<1, kSortThreads, 0, stream>>>(pair_offsets, n_views, uint32_t(G), cap, w.start, w.part_start);
  const uint32_t parts = pair_parts_max(cap, n_views);
  Segments sg{};
  sg.hist_stride = uint32_t(passes * 256), sg.n_seg = n_views, sg.start = w.start, sg.part_start = w.part_start;
  sg.key_stride = n_tiles;
  const uint64_t* src = keys_in;
  for (int p = 0; p < passes; ++p) {
    uint64_t* dst = ((passes - 1 - p) % 2) == 0 ? keys_out : w.alt;
    const int nbits = std::min(8, bits_for(n_tiles) - 8 * p);
    note_launch();
    onesweep_kernel<uint64_t, false, kSegRuns><<<parts, kSortThreads, 0, stream>>>(
        src, dst, nullptr, nullptr, cap, 8 * p, nbits, w.hist + 256 * p, w.lookback + size_t(p) * parts * 256,
        w.counters + p, status, nullptr, sg);
    src = dst;
  }
  if (passes == 1 && tile_ranges) {
    note_launch();
    run_tile_ranges_kernel<<<n_views, kSortThreads, 0, stream>>>(w.hist, w.start, n_tiles, tile_ranges, order_keys,
                                                                 order_vals, pair_offsets + size_t(n_views) * G, cap,
                                                                 status);
    *ranges_done = true;
  }
  return launch_status();
}

// ---- exclusive prefix scan of uint32 counts (three phases, no inter-block waits) -------------

constexpr int kScanThreads = 256;
constexpr int kScanItems = 16;
constexpr uint32_t kScanTile = kScanThreads * kScanItems;

__global__ void __launch_bounds__(kScanThreads) scan_reduce_kernel(const uint32_t* __restrict__ in, uint32_t n,
                                                                    unsigned long long* __restrict__ block_sums) {
  __shared__ unsigned long long s[kScanThreads / 32];
  const uint32_t base = blockIdx.x * kScanTile;
  unsigned long long acc = 0;
  for (int j = 0; j < kScanItems; ++j) {
    const uint32_t i = base + j * kScanThreads + threadIdx.x;
    if (i < n) acc += in[i];
  }
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) s[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long t = 0;
    for (int w = 0; w < kScanThreads / 32; ++w) t += s[w];
    block_sums[blockIdx.x] = t;
  }
}

// One block: exclusive scan of the block sums in place; writes the grand total.
__global__ void __launch_bounds__(1024) scan_blocksums_kernel(unsigned long long* __restrict__ sums, uint32_t nb,
                                                                uint32_t* __restrict__ total_out,
                                                                int32_t* __restrict__ status) {
  __shared__ unsigned long long s_w[32];
  __shared__ unsigned long long s_carry;
  if (threadIdx.x == 0) s_carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (uint32_t base = 0; base < nb; base += blockDim.x) {
    const uint32_t i = base + threadIdx.x;
    const unsigned long long v = i < nb ? sums[i] : 0ull;
    unsigned long long x = v;
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) s_w[warp] = x;
    __syncthreads();
    unsigned long long wb = 0, all = 0;
    for (int w = 0; w < int(blockDim.x / 32); ++w) {
      if (w < warp) wb += s_w[w];
      all += s_w[w];
    }
    const unsigned long long carry = s_carry;
    if (i < nb) sums[i] = carry + wb + x - v;
    __syncthreads();
    if (threadIdx.x == 0) s_carry = carry + all;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const unsigned long long t = s_carry;
    if (t >= (1ull << 30)) record_error(status, GSB_ERR_KEY_OVERFLOW, 0);
    *total_out = uint32_t(t >= 0xffffffffull ? 0xffffffffull : t);
  }
}

__global__ void __launch_bounds__(kScanThreads) scan_apply_kernel(const uint32_t* __restrict__ in, uint32_t n,
                                                                   const unsigned long long* __restrict__ block_off,
                                                                   uint32_t* __restrict__ out) {
  __shared__ uint32_t s_tmp[kScanThreads / 32];
  // Blocked per-thread ranges keep the scan order: thread t owns items [t*kItems, (t+1)*kItems).
  const uint32_t base = blockIdx.x * kScanTile + threadIdx.x * kScanItems;
  uint32_t x[kScanItems];
  uint32_t sum = 0;
#pragma unroll
  for (int j = 0; j < kScanItems; ++j) {
    const uint32_t i = base + j;
    x[j] = i < n ? in[i] : 0u;
    sum += x[j];
  }
  const uint32_t before = block_excl_scan_256(sum, s_tmp, nullptr);
  uint32_t run = uint32_t(block_off[blockIdx.x]) + before;
#pragma unroll
  for (int j = 0; j < kScanItems; ++j) {
    const uint32_t i = base + j;
    if (i < n) out[i] = run;
    run += x[j];
  }
}

size_t exclusive_scan_workspace(uint32_t n) {
  const uint32_t nb = (n + kScanTile - 1) / kScanTile;
  return align_up(size_t(nb + 1) * sizeof(unsigned long long));
}

gsb_status exclusive_scan(const uint32_t* counts, uint32_t n, uint32_t* offsets, void* scratch, size_t scratch_bytes,
                          cudaStream_t stream, int32_t* status) {
  const uint32_t nb = (n + kScanTile - 1) / kScanTile;
  if (scratch_bytes < exclusive_scan_workspace(n)) return GSB_ERR_WORKSPACE;
  auto* sums = static_cast<unsigned long long*>(scratch);
  if (n == 0) return cudaMemsetAsync(offsets, 0, 4, stream) ? GSB_ERR_CUDA : GSB_OK;
  note_launch();
  scan_reduce_kernel<<<nb, kScanThreads, 0, stream>>>(counts, n, sums);
  note_launch();
  scan_blocksums_kernel<<<1, 1024, 0, stream>>>(sums, nb, offsets + n, status);
  note_launch();
  scan_apply_kernel<<<nb, kScanThreads, 0, stream>>>(counts, n, sums, offsets);
  return launch_status();
}

}  // namespace gsb
