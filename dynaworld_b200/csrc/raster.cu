// Raster: per-tile front-to-back blend and its reverse-order backward.
//
// Tiles of 16x16 (or 8x8) pixels, PX (1 or 2) pixels per thread: each warp owns an 8 x 4PX pixel
// block (lane l: pixels (l % 8, l / 8 + 4k), k < PX) and works independently of the other warps (no
// CTA barrier), so a tile's warp blocks may sit in one CTA or be spread over adjacent CTAs: a warp
// streams the tile's sorted list in chunks of 32 entries (one gather per lane; the warps of a tile
// in one CTA read the same records, so all but the first read hit L1), keeps the entries whose
// ellipse reaches its block, and walks those.  With PX = 2 the
// shared-memory reads, the loop control and (backward) the warp reduction and atomics of a kept
// entry are paid once for both pixels; the launch picks PX from the grid size.
//
// Semantics of the reference's dense blend (src/train/renderers/dense.py:208-233):
//   alpha_i = clamp(o_i exp(min(power_i, 0)), 0, alpha_clamp)     (dense.py:217-220)
//   T_i     = prod_{j<i} fl32(fl32(1 - alpha_j) + eps)  over ALL Gaussians of the view in depth
//             order (dense.py:222-228); a Gaussian that does not touch the pixel contributes
//             F0 = fl32(1 + eps) (exactly so when its alpha <= 2^-25).
//   out     = clamp(sum w c + (1 - clamp(sum w, 0, 1)) bg, 0, 1), w = T alpha (dense.py:229-233);
//             the outer clamp is left out for the 2-D kernels' contract (GSB_RENDER_NO_CLAMP)
// With pos_i the depth rank of entry i (exact mode) or its index in the tile list (tiled-compat
// mode, tile-local products as tiled.py:176-185):
//   T_i = F0^pos_i * S_i,   S_i = prod_{blended j < i} f_j / F0,
// so entries a pixel skips leave S unchanged and cost nothing.  A pair is skipped when its alpha
// is below alpha_cutoff; a pixel stops once T falls below the transmittance threshold.  The
// Gaussian's threshold tau on q (alpha >= cutoff <=> q <= tau, with a margin) only culls entries
// whose ellipse misses a warp's whole pixel block, when a chunk is loaded: testing it per pixel as
// well costs more than the falloff it would save (measured on one B200, 16 x 128^2: forward 0.345
// -> 0.337 ms, backward 0.657 -> 0.633 ms without it).
#include <cstdlib>
#include <type_traits>

#include "gsb_common.cuh"
#include "gsb_internal.h"

namespace gsb {

constexpr uint32_t kCountBits = 28;
constexpr uint32_t kCountMask = (1u << kCountBits) - 1u;
constexpr uint32_t kFull = 0xffffffffu;

// exp(-q / 2) = 2^(q k), k = -log2(e) / 2, on the SFU's base-2 exponential (PTX ex2.approx; relative
// error about 2^-22).  The warp slots hold the conic already multiplied by k (one multiply per entry
// and lane when the chunk is loaded), so a pixel evaluates qk = q k directly and pays one SFU op.
// Forward and backward evaluate the same expression, so the backward's alpha is the forward's to
// the bit.
constexpr float kFalloffScale = -0.72134752044448170368f;  // k
__device__ __forceinline__ float gauss_falloff(float qk) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(fminf(qk, 0.0f)));
  return y;
}
// The same for an entry whose computed qk cannot be positive (a well-conditioned conic: see
// load_entry), where the clamp to 0 is the identity.
__device__ __forceinline__ float gauss_falloff_nonpos(float qk) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(qk));
  return y;
}
// The backward accumulates the per-pixel power gradient without the 1/k that relates the k-scaled
// conic to q (dpow = d loss / d power times k, where power = -q / 2 and the slots hold k A, k B,
// k C), so a conditioned chunk multiplies nothing per pixel for it; the factors come in once per
// entry when the sums are flushed: 1/k on the mean gradients, -1/2 (= 1/k times -k/2) on the conic
// gradients -1/2 sum dpow dx^2 (and so on).  (Applying the conic coefficients once per entry to
// per-lane sums as well was measured slower: 8 x 1920x1080 backward 26.9 -> 28.1 ms.)
constexpr float kInvFalloffScale = -1.38629436111989061883f;  // 1 / k = -2 ln 2
constexpr float kConicFlushScale = -0.5f;                     // (1 / k) (-k / 2)

// q = A dx^2 + B dx dy + C dy^2 with a fixed rounding sequence (forward and backward agree).
__device__ __forceinline__ float pair_q(float A, float B, float C, float dx, float dy) {
  const float t0 = __fmul_rn(__fmul_rn(A, dx), dx);
  const float t1 = __fmaf_rn(__fmul_rn(B, dx), dy, t0);
  return __fmaf_rn(__fmul_rn(C, dy), dy, t1);
}

__device__ __forceinline__ uint32_t lane_mask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// PX pixels per lane, 4 rows apart: the warp block is 8 wide and 4 * PX high.
template <int PX>
__host__ __device__ constexpr int block_h() { return 4 * PX; }

// Pixel block of warp w inside a TILE x TILE tile.
template <int TILE, int PX>
__device__ __forceinline__ void block_of(int warp, int& bx, int& by) {
  constexpr int BX = TILE / 8;
  bx = (warp % BX) * 8;
  by = (warp / BX) * block_h<PX>();
}

template <int PX>
__device__ __forceinline__ bool all_of(const bool (&v)[PX]) {
  bool r = true;
#pragma unroll
  for (int k = 0; k < PX; ++k) r = r && v[k];
  return r;
}

template <int PX>
__device__ __forceinline__ uint32_t min_of(const uint32_t (&v)[PX]) {
  uint32_t r = 0xffffffffu;
#pragma unroll
  for (int k = 0; k < PX; ++k) r = min(r, v[k]);
  return r;
}

template <int PX>
__device__ __forceinline__ uint32_t max_of(const uint32_t (&v)[PX]) {
  uint32_t r = 0;
#pragma unroll
  for (int k = 0; k < PX; ++k) r = max(r, v[k]);
  return r;
}

struct WarpSlots {
  float4* geo;     // mx, my, A k, B k
  float4* cot;     // C k, opacity, stop bound (forward), F0^pos
  float4* col;     // r, g, b, z
  uint32_t* rank;  // depth rank (gradient slot)
};

// Lane loads list entry idx (list index li) into its warp slot and returns whether the Gaussian's
// ellipse {q <= tau} reaches the warp's pixel block [bx0, bx0+7] x [by0, by0+BH-1] (pixel
// centres; conservative).  FWD: the forward's slot carries the bound on S below which the pixel
// stops, and max(o, 0) for the opacity: with alpha = clamp(o e, 0, alpha_clamp) and e > 0,
// max(o, 0) e equals max(o e, 0) exactly, so the forward skips the lower clamp.
//
// conditioned: the entry is kept with finite extents and a finite conic with A, C > 0 and
// B^2 <= 4 A C (1 - 2^-8) (and, in the forward, an opacity in [0, alpha_clamp]).  Then |B dx dy| <=
// 0.999 (A dx^2 + C dy^2), so q >= 0.001 (A dx^2 + C dy^2) while the rounding of pair_q stays below
// 8 ulp of that sum: the computed q is never negative (qk never positive), the falloff needs no clamp
// and d min(power, 0) / d power is 1 wherever dx or dy is nonzero; with e <= 1 the forward's alpha
// = o e needs no clamp either (the rounded product is at most o).  A chunk whose kept entries are
// all conditioned takes that path; both paths give the same bits for such an entry, so forward and
// backward agree whichever each takes.  (Skipping the alpha clamps in the backward too raised its
// registers at four pixels per lane from 80 to 100 and was slower: 8 x 1920x1080 26.9 -> 31.7 ms.)
// One list entry as the walk reads it: the slot contents.
struct Entry {
  float4 geo, cot, col;
  uint32_t rank;
};

template <int BH, bool FWD>
__device__ __forceinline__ bool entry_of(const RasterArgs& a, const float* recs, uint32_t idx, uint32_t li,
                                         float bx0, float by0, Entry& en, bool& conditioned) {
  conditioned = false;
  const uint32_t r = min(uint32_t(a.keys[idx]), uint32_t(a.G - 1));  // ranks are < G for valid keys
  const float4* rec = reinterpret_cast<const float4*>(recs + size_t(r) * GSB_RECORD_FLOATS);
  const float4 r0 = __ldg(rec + 0), r1 = __ldg(rec + 1), r2 = __ldg(rec + 2), r3 = __ldg(rec + 3);
  const float pos = a.rc.compat ? float(li) : float(r);
  const float pw = exp2f(pos * a.rc.log2_f0);
  const float A = r0.z, B = r0.w, C = r1.x, tau = r1.w;
  en.geo = make_float4(r0.x, r0.y, A * kFalloffScale, B * kFalloffScale);
  // T after an entry = S after it * F0 * F0^pos: the forward compares S with the bound
  en.cot = make_float4(C * kFalloffScale, FWD ? fmaxf(r1.y, 0.0f) : r1.y,
                       FWD ? __fdividef(a.rc.t_threshold, a.rc.f0 * pw) : 0.0f, pw);
  en.col = make_float4(r2.x, r2.y, r2.z, r1.z);
  en.rank = r;
  if (!(tau >= 0.0f)) return false;
  // half extents of the ellipse (cull_extents: sqrt(tau (A^-1)_ii), +inf for a degenerate conic)
  const float ex = r3.x, ey = r3.y;
  if (!(ex < __int_as_float(0x7f800000))) return true;
  constexpr float kH = float(BH - 1);
  if (!((r0.x + ex >= bx0) && (r0.x - ex <= bx0 + 7.0f) && (r0.y + ey >= by0) && (r0.y - ey <= by0 + kH)))
    return false;
  conditioned = A > 0.0f && C > 0.0f && A < 1e30f && C < 1e30f && fabsf(B) < 1e30f &&
                B * B <= 4.0f * A * C * (1.0f - 1.0f / 256.0f) && (!FWD || (r1.y >= 0.0f && r1.y <= a.rc.alpha_clamp));
  // exact: the minimum of q over the block's pixel-centre box (on an edge unless the mean is inside)
  const float X0 = bx0 - r0.x, X1 = bx0 + 7.0f - r0.x, Y0 = by0 - r0.y, Y1 = by0 + kH - r0.y;
  if (X0 <= 0.0f && X1 >= 0.0f && Y0 <= 0.0f && Y1 >= 0.0f) return true;
  const float hC = r3.z, hA = r3.w;
  float q = __int_as_float(0x7f800000);
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const float dx = e ? X1 : X0;
    const float dy = fminf(fmaxf(hC * dx, Y0), Y1);
    q = fminf(q, (A * dx + B * dy) * dx + C * dy * dy);
    const float ey2 = e ? Y1 : Y0;
    const float dx2 = fminf(fmaxf(hA * ey2, X0), X1);
    q = fminf(q, (A * dx2 + B * ey2) * dx2 + C * ey2 * ey2);
  }
  return q <= tau * 1.0001f + 0.01f;
}

__device__ __forceinline__ void store_entry(const WarpSlots& s, int slot, const Entry& en) {
  s.geo[slot] = en.geo;
  s.cot[slot] = en.cot;
  s.col[slot] = en.col;
  if (s.rank) s.rank[slot] = en.rank;
}

template <int BH, bool FWD>
__device__ __forceinline__ bool load_entry(const RasterArgs& a, const float* recs, uint32_t idx, uint32_t li,
                                           float bx0, float by0, const WarpSlots& s, int lane, bool& conditioned) {
  Entry en;
  const bool keep = entry_of<BH, FWD>(a, recs, idx, li, bx0, by0, en, conditioned);
  store_entry(s, lane, en);
  return keep;
}

// Floats a checkpoint slot holds per pixel: S, then the suffix sums of r, g, b, weight, depth.
constexpr int kCkptFloats = 6;

// NSEG: list segments of the backward (checkpoints between).  CW: warps per CTA; the tile's NW warp
// blocks are spread over NW / CW adjacent CTAs.  DEPTH: the depth output is written (and its sums
// kept for the backward).
template <int TILE, int PX, int NSEG, int CW, bool DEPTH>
__global__ void __launch_bounds__(32 * CW) raster_fwd_kernel(RasterArgs a) {
  constexpr int NW = TILE * TILE / (32 * PX);
  constexpr int SPLIT = NW / CW;
  static_assert(SPLIT * CW == NW, "CTAs must hold whole warp blocks of one tile");
  constexpr int NB = NSEG > 1 ? NSEG - 1 : 1;  // checkpoint slots (boundaries between segments)
  __shared__ float4 s_geo[CW][32], s_cot[CW][32], s_col[CW][32];
  __shared__ uint32_t s_li[CW][32];  // chunk position (lane) of each compacted slot (kCompact)
  const RenderConsts& rc = a.rc;
  const uint32_t cta = blockIdx.y * uint32_t(rc.n_tiles) * SPLIT + blockIdx.x;
  const uint32_t slot = cta / SPLIT;
  const uint32_t vt = a.order ? a.order[slot] : slot;  // heaviest tiles first
  const int view = int(vt / uint32_t(rc.n_tiles)), tile = int(vt % uint32_t(rc.n_tiles));
  const int tid = threadIdx.x, lane = tid & 31, lw = tid >> 5;
  const int warp = int(cta % SPLIT) * CW + lw;  // warp block within the tile
  int bx, by;
  block_of<TILE, PX>(warp, bx, by);
  const int ox = (tile % rc.tiles_x) * TILE + bx, oy = (tile / rc.tiles_x) * TILE + by;  // block origin
  const int px = ox + (lane & 7);
  const float bx0 = float(ox) + rc.pixel_center, by0 = float(oy) + rc.pixel_center;
  const float fx = float(px) + rc.pixel_center;
  const size_t rb = (size_t(view) * rc.n_tiles + tile) * 2;
  const uint32_t start = a.ranges[rb], end = a.ranges[rb + 1];
  const float* recs = a.records + size_t(view) * a.G * GSB_RECORD_FLOATS;
  const float inv_f0 = rc.inv_f0;
  const WarpSlots ws{s_geo[lw], s_cot[lw], s_col[lw], nullptr};

  int py[PX];
  float fy[PX], S[PX], C0[PX], C1[PX], C2[PX], Ws[PX], D[PX];
  uint32_t n_proc[PX];
  bool done[PX];
#pragma unroll
  for (int k = 0; k < PX; ++k) {
    py[k] = oy + (lane >> 3) + 4 * k;
    fy[k] = float(py[k]) + rc.pixel_center;
    S[k] = 1.0f, C0[k] = C1[k] = C2[k] = Ws[k] = D[k] = 0.0f;
    n_proc[k] = end - start;
    done[k] = !(px < a.W && py[k] < a.H);
  }
  // Segment boundaries of the list (the backward runs each segment as its own CTA): the state of
  // every pixel just before entry bnd[s] is kept, as a prefix, and written out as the suffix the
  // backward of segment s starts from.
  uint32_t bnd[NB];
  float kS[NB][PX], kC0[NB][PX], kC1[NB][PX], kC2[NB][PX], kW[NB][PX], kD[NB][PX];
  int next = 0;
#pragma unroll
  for (int s = 0; s < NB; ++s) bnd[s] = start + uint32_t((uint64_t(s + 1) * (end - start)) / NSEG);
  auto snapshot = [&](int s) {  // held in registers (global stores inside the walk cost more)
#pragma unroll
    for (int k = 0; k < PX; ++k)
      kS[s][k] = S[k], kC0[s][k] = C0[k], kC1[s][k] = C1[k], kC2[s][k] = C2[k], kW[s][k] = Ws[k], kD[s][k] = D[k];
  };
  // blend the entry in slot j of the current chunk (list index c - start + j) into every live pixel;
  // fast: std::true_type when every kept entry of the chunk is conditioned
  auto blend = [&](uint32_t c, int j, auto fast) {
    const float4 g = s_geo[lw][j];
    const float4 ct = s_cot[lw][j];
    const float dx = __fsub_rn(fx, g.x);
#pragma unroll
    for (int k = 0; k < PX; ++k) {
      if (done[k]) continue;
      const float dy = __fsub_rn(fy[k], g.y);
      const float qk = pair_q(g.z, g.w, ct.x, dx, dy);
      const float e = decltype(fast)::value ? gauss_falloff_nonpos(qk) : gauss_falloff(qk);
      const float alpha = decltype(fast)::value ? ct.y * e : fminf(ct.y * e, rc.alpha_clamp);  // ct.y >= 0
      if (!(alpha >= rc.alpha_cutoff)) continue;
      const float4 col = s_col[lw][j];
      const float T = S[k] * ct.w;
      const float w = T * alpha;
      C0[k] = fmaf(w, col.x, C0[k]);
      C1[k] = fmaf(w, col.y, C1[k]);
      C2[k] = fmaf(w, col.z, C2[k]);
      Ws[k] += w;
      if (DEPTH) D[k] = fmaf(w, col.w, D[k]);
      const float f = __fadd_rn(__fsub_rn(1.0f, alpha), rc.eps);
      S[k] = S[k] * (f * inv_f0);
      if (S[k] < ct.z) {  // T after this entry below the threshold
        done[k] = true;
        n_proc[k] = c - start + uint32_t(j) + 1u;
      }
    }
  };
  auto walk = [&](uint32_t c, uint32_t m, auto fast) {
    if (NSEG > 1) {
      // boundaries inside this chunk (warp-uniform): blend the entries before one, then keep the state
#pragma unroll
      for (int s = 0; s < NB; ++s) {
        if (next == s && bnd[s] < c + 32u) {
          const uint32_t cut = bnd[s] > c ? bnd[s] - c : 0u;  // slots j < cut lie before the boundary
          const uint32_t before = (1u << cut) - 1u;           // cut <= 31
          uint32_t mb = m & before;
          while (mb && !all_of(done)) {
            const int j = __ffs(mb) - 1;
            mb &= mb - 1;
            blend(c, j, fast);
          }
          m &= ~before;
          snapshot(s);
          next = s + 1;
        }
      }
    }
    while (m && !all_of(done)) {
      const int j = __ffs(m) - 1;
      m &= m - 1;
      blend(c, j, fast);
    }
  };
  // Two walks of a chunk's kept entries.  Compact (two or more pixels per lane): the kept entries
  // sit in consecutive slots and every lane runs every slot, a pixel that has stopped or whose
  // alpha is below the cutoff taking alpha 0, so the walk has no per-pixel branches.  With alpha 0
  // the factor is f = F0 and S * (f * inv_f0) is S to the bit (inv_f0 is chosen so that
  // F0 * inv_f0 rounds to 1), so a skipped entry changes nothing; a stopped pixel's cutoff is
  // +inf.  Measured on one B200, 8 x 1920x1080 forward 11.63 -> 11.09 ms against the set-bit walk.
  // With one pixel per lane the lane's own early exit pays more (16 x 128^2: 0.332 ms, 0.351
  // compact), so it walks the set bits of the keep mask.
  constexpr bool kCompact = PX >= 2;
  if constexpr (kCompact) {
  const float kInf = __int_as_float(0x7f800000);
  float cut[PX];
#pragma unroll
  for (int k = 0; k < PX; ++k) cut[k] = done[k] ? kInf : rc.alpha_cutoff;
  auto stopped = [&]() {
    bool r = true;
#pragma unroll
    for (int k = 0; k < PX; ++k) r = r && cut[k] == kInf;
    return r;
  };
  auto blend2 = [&](uint32_t c, int j, auto fast) {
    const float4 g = s_geo[lw][j];
    const float4 ct = s_cot[lw][j];
    const float4 col = s_col[lw][j];
    const float dx = __fsub_rn(fx, g.x);
#pragma unroll
    for (int k = 0; k < PX; ++k) {
      const float dy = __fsub_rn(fy[k], g.y);
      const float qk = pair_q(g.z, g.w, ct.x, dx, dy);
      const float e = decltype(fast)::value ? gauss_falloff_nonpos(qk) : gauss_falloff(qk);
      const float a0 = decltype(fast)::value ? ct.y * e : fminf(ct.y * e, rc.alpha_clamp);  // ct.y >= 0
      const bool take = a0 >= cut[k];
      const float alpha = take ? a0 : 0.0f;
      const float T = S[k] * ct.w;
      const float w = T * alpha;
      C0[k] = fmaf(w, col.x, C0[k]);
      C1[k] = fmaf(w, col.y, C1[k]);
      C2[k] = fmaf(w, col.z, C2[k]);
      Ws[k] += w;
      if (DEPTH) D[k] = fmaf(w, col.w, D[k]);
      const float f = __fadd_rn(__fsub_rn(1.0f, alpha), rc.eps);
      S[k] = S[k] * (f * inv_f0);
      if (take && S[k] < ct.z) {  // T after this entry below the threshold
        cut[k] = kInf;
        n_proc[k] = c - start + s_li[lw][j] + 1u;
      }
    }
  };
  auto walk2 = [&](uint32_t c, uint32_t m, auto fast) {
    const int nk = __popc(m);
    int j = 0;
    if (NSEG > 1) {
#pragma unroll
      for (int s = 0; s < NB; ++s) {
        if (next == s && bnd[s] < c + 32u) {
          const uint32_t cut_at = bnd[s] > c ? bnd[s] - c : 0u;  // chunk positions < cut_at lie before it
          const int jb = __popc(m & ((1u << cut_at) - 1u));
          for (; j < jb; ++j) blend2(c, j, fast);
          snapshot(s);
          next = s + 1;
        }
      }
    }
    for (; j < nk; ++j) {
      blend2(c, j, fast);
      if ((j & 7) == 7 && __all_sync(kFull, stopped())) break;
    }
  };
  for (uint32_t c = start; c < end; c += 32) {
    if (__all_sync(kFull, stopped())) break;
    const uint32_t idx = c + lane;
    bool cond = false;
    Entry en;
    const bool keep = idx < end && entry_of<block_h<PX>(), true>(a, recs, idx, idx - start, bx0, by0, en, cond);
    const uint32_t m = __ballot_sync(kFull, keep);
    const bool fast = __all_sync(kFull, cond || !keep);
    if (keep) {
      const int pos = __popc(m & lane_mask_lt());
      store_entry(ws, pos, en);
      s_li[lw][pos] = uint32_t(lane);
    }
    __syncwarp();
    if (fast) walk2(c, m, std::true_type{});
    else walk2(c, m, std::false_type{});
    __syncwarp();  // slots are rewritten by the next chunk
  }
  } else {
  for (uint32_t c = start; c < end; c += 32) {
    if (__all_sync(kFull, all_of(done))) break;
    const uint32_t idx = c + lane;
    bool cond = false;
    const bool keep =
        idx < end && load_entry<block_h<PX>(), true>(a, recs, idx, idx - start, bx0, by0, ws, lane, cond);
    const uint32_t m = __ballot_sync(kFull, keep);
    const bool fast = __all_sync(kFull, cond || !keep);
    __syncwarp();
    if (fast) walk(c, m, std::true_type{});
    else walk(c, m, std::false_type{});
    __syncwarp();  // slots are rewritten by the next chunk
  }
  }

  if (NSEG > 1) {
    // boundaries the pixel never reached (stopped early, or no later entry) hold the final state
#pragma unroll
    for (int s = 0; s < NB; ++s)
      if (next <= s) snapshot(s);
  }
  const size_t HW = size_t(a.H) * a.W;
  const size_t total_px = size_t(a.B) * HW;
#pragma unroll
  for (int k = 0; k < PX; ++k) {
    if (!(px < a.W && py[k] < a.H)) continue;
    const size_t poff = size_t(py[k]) * a.W + px;
    const size_t pix = size_t(view) * HW + poff;
    if (NSEG > 1) {  // slot s: S before bnd[s] and the colour / weight / depth of the entries after it
#pragma unroll
      for (int s = 0; s < NB; ++s) {
        float* ck = a.ckpt + size_t(s) * kCkptFloats * total_px + pix;
        ck[0] = kS[s][k];
        ck[total_px] = C0[k] - kC0[s][k];
        ck[2 * total_px] = C1[k] - kC1[s][k];
        ck[3 * total_px] = C2[k] - kC2[s][k];
        ck[4 * total_px] = Ws[k] - kW[s][k];
        if (DEPTH) ck[5 * total_px] = D[k] - kD[s][k];
      }
    }
    const float wc = fminf(fmaxf(Ws[k], 0.0f), 1.0f);
    const float one_m = __fsub_rn(1.0f, wc);
    const float cc[3] = {C0[k], C1[k], C2[k]};
    uint32_t mask = (Ws[k] >= 0.0f && Ws[k] <= 1.0f) ? 8u : 0u;
#pragma unroll
    for (int ch = 0; ch < 3; ++ch) {
      const float pre = __fadd_rn(cc[ch], __fmul_rn(one_m, rc.bg[ch]));
      const bool pass = !rc.clamp_image || (pre >= 0.0f && pre <= 1.0f);
      if (pass) mask |= 1u << ch;
      a.image[(size_t(view) * 3 + ch) * HW + poff] = rc.clamp_image ? fminf(fmaxf(pre, 0.0f), 1.0f) : pre;
    }
    if (a.alpha) a.alpha[pix] = Ws[k];
    if (DEPTH) a.depth[pix] = D[k];
    a.pixel_t[pix] = S[k];  // normalised transmittance after the last blended entry
    a.pixel_state[pix] = min(n_proc[k], kCountMask) | (mask << kCountBits);
  }
}

// Warp sum of 10 per-lane values (v[10], v[11] are padding).  Afterwards lane l holds the total of
// value 6*b4 + 3*b3 + (2*b2 + b1) (b = bits of l) when 2*b2 + b1 < 3; 13 shuffles.
__device__ __forceinline__ float warp_sum10(float v[12], int lane, int* index) {
#pragma unroll
  for (int k = 0; k < 6; ++k) {
    const bool up = lane & 16;
    const float send = up ? v[k] : v[k + 6];
    const float keep = up ? v[k + 6] : v[k];
    v[k] = keep + __shfl_xor_sync(kFull, send, 16);
  }
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const bool up = lane & 8;
    const float send = up ? v[k] : v[k + 3];
    const float keep = up ? v[k + 3] : v[k];
    v[k] = keep + __shfl_xor_sync(kFull, send, 8);
  }
  v[3] = 0.0f;
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const bool up = lane & 4;
    const float send = up ? v[k] : v[k + 2];
    const float keep = up ? v[k + 2] : v[k];
    v[k] = keep + __shfl_xor_sync(kFull, send, 4);
  }
  {
    const bool up = lane & 2;
    const float send = up ? v[0] : v[1];
    const float keep = up ? v[1] : v[0];
    v[0] = keep + __shfl_xor_sync(kFull, send, 2);
  }
  const int sub = ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
  *index = sub < 3 ? ((lane >> 4) & 1) * 6 + ((lane >> 3) & 1) * 3 + sub : 99;
  return v[0] + __shfl_xor_sync(kFull, v[0], 1);
}

// Lanes contributing to one entry at or below this count add their own values atomically, as five
// 8-byte vector reductions (red.global.add.v2.f32; a gradient slot is 40 bytes, so every pair of
// floats is 8-byte aligned); up to partial_contributors the warp first sums each pixel column's four
// rows (two transpose steps, three values per lane, two reductions per lane); above that it sums
// over the whole warp (warp_sum10).  Measured on one B200 (backward ms, 16 x 128^2 / 8 x 384^2):
// scalar atomics, one per nonzero value, up to 12: 0.730 / 1.433; vector pairs up to 12: 0.667 /
// 1.312, 16: 0.660 / 1.291, 20: 0.661 / 1.289, 24: 0.692 / 1.349; 16-byte vectors (three per slot,
// placed by the slot's alignment) up to 16: 0.664 / 1.336, 24: 0.649 / 1.296, 32 (never reduce in
// the warp): 0.893 / 1.714.  Then, with pairs up to 16, column sums up to 18: 0.625 / 1.135, 20:
// 0.627 / 1.139, 22: 0.629 / 1.143, 24: 0.631 / 1.147, 28: 0.635 / 1.152, 32: 0.646 / 1.262, none:
// 0.630 / 1.233; pairs up to 12 or 14 with column sums up to 20: 0.637 / 1.164, 0.632 / 1.152.
// At four pixels per lane (a lane's four pixels share a column, so fewer lanes carry more of an
// entry's gradient) the per-lane atomics pay up to 24 contributors, and the column sums no longer:
// measured on 8 x 1920x1080 (backward ms, atomics / column sums up to): 16 / 18 26.85, 12 / 18 27.10,
// 20 / 20 26.65, 24 / 24 26.56, 16 / 24 26.94, 16 / 16 26.80 (8 x 384^2 at two pixels per lane:
// 16 / 18 1.120, 20 / 20 1.112, 24 / 24 1.217).
template <int PX>
__host__ __device__ constexpr int sparse_contributors() { return PX == 4 ? 24 : 16; }
template <int PX>
__host__ __device__ constexpr int partial_contributors() { return PX == 4 ? 24 : 18; }

// DEPTH: a depth gradient is given.  NSEG: the tile's list is cut into NSEG segments
// [s n / NSEG, (s + 1) n / NSEG), each walked by its own CTA (adjacent in launch order), starting
// from the forward's checkpoint of its upper boundary (the last segment from the final state).
// CW: warps per CTA, as in the forward.
// (Register caps measured on 8 x 1920x1080, four pixels per lane, 80 registers uncapped: 26.9 ms;
// capped at 72: 29.8 ms, at 64: 30.7 ms.)
template <int TILE, int PX, bool DEPTH, int NSEG, int CW>
__global__ void __launch_bounds__(32 * CW) raster_bwd_kernel(RasterArgs a) {
  constexpr int NW = TILE * TILE / (32 * PX);
  constexpr int SPLIT = NW / CW;
  static_assert(SPLIT * CW == NW, "CTAs must hold whole warp blocks of one tile");
  __shared__ float4 s_geo[CW][32], s_cot[CW][32], s_col[CW][32];
  __shared__ uint32_t s_rank[CW][32];
  const RenderConsts& rc = a.rc;
  const uint32_t cta = blockIdx.y * uint32_t(rc.n_tiles) * (NSEG * SPLIT) + blockIdx.x;
  const uint32_t slot = cta / (NSEG * SPLIT);
  const int seg = int((cta / SPLIT) % NSEG);
  const uint32_t vt = a.order ? a.order[slot] : slot;  // heaviest tiles first
  const int view = int(vt / uint32_t(rc.n_tiles)), tile = int(vt % uint32_t(rc.n_tiles));
  const int tid = threadIdx.x, lane = tid & 31, lw = tid >> 5;
  const int warp = int(cta % SPLIT) * CW + lw;  // warp block within the tile
  int bx, by;
  block_of<TILE, PX>(warp, bx, by);
  const int ox = (tile % rc.tiles_x) * TILE + bx, oy = (tile / rc.tiles_x) * TILE + by;  // block origin
  const int px = ox + (lane & 7);
  const float bx0 = float(ox) + rc.pixel_center, by0 = float(oy) + rc.pixel_center;
  const float fx = float(px) + rc.pixel_center;
  const size_t rb = (size_t(view) * rc.n_tiles + tile) * 2;
  const uint32_t start = a.ranges[rb];
  const uint32_t n_list = a.ranges[rb + 1] - start;
  const uint32_t lo = uint32_t((uint64_t(seg) * n_list) / NSEG);       // this segment's entries
  const uint32_t hi = uint32_t((uint64_t(seg + 1) * n_list) / NSEG);
  const float* recs = a.records + size_t(view) * a.G * GSB_RECORD_FLOATS;
  float* g2 = a.grad2d + size_t(view) * a.G * GSB_GRAD2D_FLOATS;
  const WarpSlots ws{s_geo[lw], s_cot[lw], s_col[lw], s_rank[lw]};

  const size_t HW = size_t(a.H) * a.W;
  const size_t total_px = size_t(a.B) * HW;
  float fy[PX], S[PX], g0[PX], g1[PX], g2c[PX], gW[PX], gD[PX];
  // d loss / d (weights of the entries after the current one), folded with the pixel's upstream
  // gradients: rs = sum_c g_c R_c + gW RW + gD RD over the suffix sums R of colour, weight and depth.
  // One entry adds w * dldw to it, so the suffix sums themselves are never kept.
  float rs[PX];
  uint32_t n_proc[PX];  // entries of this segment the pixel blended: list index < n_proc
  const float sc = a.view_scale ? a.view_scale[view] : 1.0f;
#pragma unroll
  for (int k = 0; k < PX; ++k) {
    const int py = oy + (lane >> 3) + 4 * k;
    fy[k] = float(py) + rc.pixel_center;
    S[k] = g0[k] = g1[k] = g2c[k] = gW[k] = gD[k] = rs[k] = 0.0f;
    n_proc[k] = 0;
    if (px < a.W && py < a.H) {
      const size_t poff = size_t(py) * a.W + px;
      const size_t pix = size_t(view) * HW + poff;
      S[k] = a.pixel_t[pix];
      const uint32_t st = a.pixel_state[pix];
      n_proc[k] = min(st & kCountMask, hi);
      const uint32_t mask = st >> kCountBits;
      const float* di = a.d_image + size_t(view) * 3 * HW + poff;
      g0[k] = (mask & 1u) ? di[0] * sc : 0.0f;
      g1[k] = (mask & 2u) ? di[HW] * sc : 0.0f;
      g2c[k] = (mask & 4u) ? di[2 * HW] * sc : 0.0f;
      gW[k] = (mask & 8u) ? -(g0[k] * rc.bg[0] + g1[k] * rc.bg[1] + g2c[k] * rc.bg[2]) : 0.0f;
      if (a.d_alpha) gW[k] += a.d_alpha[pix];
      if (a.d_depth) gD[k] = a.d_depth[pix];
      if (NSEG > 1 && seg < NSEG - 1) {  // start from the checkpoint at hi
        const float* ck = a.ckpt + size_t(seg) * kCkptFloats * total_px + pix;
        S[k] = ck[0];
        rs[k] = g0[k] * ck[total_px] + g1[k] * ck[2 * total_px] + g2c[k] * ck[3 * total_px] + gW[k] * ck[4 * total_px];
        if (DEPTH) rs[k] = fmaf(gD[k], ck[5 * total_px], rs[k]);  // written by the forward only with depth on
      }
    }
  }
  // list range [lo, wmax) this warp has to revisit; below wmin every pixel of the warp blended
  const uint32_t wmax = __reduce_max_sync(kFull, max_of(n_proc));
  const uint32_t wmin = __reduce_min_sync(kFull, min_of(n_proc));
  const int64_t cb_lo = int64_t(lo / 32) * 32;

  // the kept entries m of the chunk at list index cb, last first; fast as in the forward; live:
  // every entry of the chunk lies below every pixel's count, so no pixel tests it
  auto walk = [&](int64_t cb, uint32_t m, auto fast, auto live) {
    while (m) {
      const int j = 31 - __clz(m);
      m &= ~(1u << j);
      const uint32_t lj = uint32_t(cb) + uint32_t(j);
      float v[12];
#pragma unroll
      for (int k = 0; k < 12; ++k) v[k] = 0.0f;
      bool contrib = false;
      if (decltype(live)::value || lj < max_of(n_proc)) {
        const float4 g = s_geo[lw][j];
        const float4 ct = s_cot[lw][j];
        const float dx = __fsub_rn(fx, g.x);
        const float hB = 0.5f * g.w;  // half the cross coefficient
#pragma unroll
        for (int k = 0; k < PX; ++k) {
          if (!decltype(live)::value && !(lj < n_proc[k])) continue;
          const float dy = __fsub_rn(fy[k], g.y);
          const float qk = pair_q(g.z, g.w, ct.x, dx, dy);
          const float e = decltype(fast)::value ? gauss_falloff_nonpos(qk) : gauss_falloff(qk);
          const float araw = ct.y * e;
          const float alpha = fminf(fmaxf(araw, 0.0f), rc.alpha_clamp);
          if (!(alpha >= rc.alpha_cutoff)) continue;
          const float f = __fadd_rn(__fsub_rn(1.0f, alpha), rc.eps);
          const float rf = __fdividef(1.0f, f);
          S[k] = S[k] * (rc.f0 * rf);  // S before this entry: S_after / (f / F0)
          const float T = S[k] * ct.w;
          const float4 col = s_col[lw][j];
          const float w = T * alpha;
          float dldw = g0[k] * col.x + g1[k] * col.y + g2c[k] * col.z + gW[k];
          if (DEPTH) dldw = fmaf(gD[k], col.w, dldw);
          const float dlda = T * dldw - rs[k] * rf;
          rs[k] = fmaf(w, dldw, rs[k]);
          const float dlr = alpha == araw ? dlda : 0.0f;  // the clamp to [0, alpha_clamp] is inactive
          // d min(power, 0) / d power, power = -q / 2 (torch splits a tie at 0 evenly), divided by k;
          // q > 0 where qk < 0.  A conditioned entry has q = 0 only at dx = dy = 0, where the mask
          // multiplies zeros.
          const float pmask = decltype(fast)::value ? 1.0f : (qk < 0.0f ? 1.0f : (qk == 0.0f ? 0.5f : 0.0f));
          const float dpow = dlr * araw * pmask;
          const float u = dpow * dx, t = dpow * dy;
          v[0] = fmaf(g.z, u, fmaf(hB, t, v[0]));
          v[1] = fmaf(ct.x, t, fmaf(hB, u, v[1]));
          v[2] = fmaf(u, dx, v[2]);  // conic gradients: times -1/2 once the pixels are summed
          v[3] = fmaf(u, dy, v[3]);
          v[4] = fmaf(t, dy, v[4]);
          v[5] = fmaf(dlr, e, v[5]);
          v[6] = fmaf(g0[k], w, v[6]);
          v[7] = fmaf(g1[k], w, v[7]);
          v[8] = fmaf(g2c[k], w, v[8]);
          if (DEPTH) v[9] = fmaf(gD[k], w, v[9]);
          contrib = true;
        }
      }
      const uint32_t cm = __ballot_sync(kFull, contrib);
      if (cm == 0u) continue;
      float* dst = g2 + size_t(s_rank[lw][j]) * GSB_GRAD2D_FLOATS;
      if (__popc(cm) <= sparse_contributors<PX>()) {
        if (contrib) {
          float2* d2 = reinterpret_cast<float2*>(dst);
          atomicAdd(d2 + 0, make_float2(kInvFalloffScale * v[0], kInvFalloffScale * v[1]));
          atomicAdd(d2 + 1, make_float2(kConicFlushScale * v[2], kConicFlushScale * v[3]));
          atomicAdd(d2 + 2, make_float2(kConicFlushScale * v[4], v[5]));
          atomicAdd(d2 + 3, make_float2(v[6], v[7]));
          if (DEPTH) atomicAdd(d2 + 4, make_float2(v[8], v[9]));
          else atomicAdd(dst + 8, v[8]);
        }
      } else if (__popc(cm) <= partial_contributors<PX>()) {
        // column sums: lane l keeps values 3 grp + (0, 1, 2), grp = 2 b4 + b3, summed over l ^ {8, 16, 24}
#pragma unroll
        for (int k = 0; k < 6; ++k) {
          const bool up = lane & 16;
          const float send = up ? v[k] : v[k + 6];
          const float keep = up ? v[k + 6] : v[k];
          v[k] = keep + __shfl_xor_sync(kFull, send, 16);
        }
#pragma unroll
        for (int k = 0; k < 3; ++k) {
          const bool up = lane & 8;
          const float send = up ? v[k] : v[k + 3];
          const float keep = up ? v[k + 3] : v[k];
          v[k] = keep + __shfl_xor_sync(kFull, send, 8);
        }
        const int grp = ((lane >> 4) & 1) * 2 + ((lane >> 3) & 1);
        // a float pair at dst + p2 (8-byte aligned: p2 is 0, 4 or 6) and one float at dst + p1
        float2 pv;
        float sv;
        int p2, p1;
        if (grp == 0)
          pv = make_float2(kInvFalloffScale * v[0], kInvFalloffScale * v[1]), p2 = 0, sv = kConicFlushScale * v[2], p1 = 2;
        else if (grp == 1)
          pv = make_float2(kConicFlushScale * v[1], v[2]), p2 = 4, sv = kConicFlushScale * v[0], p1 = 3;
        else if (grp == 2) pv = make_float2(v[0], v[1]), p2 = 6, sv = v[2], p1 = 8;
        else pv = make_float2(0.0f, 0.0f), p2 = 0, sv = DEPTH ? v[0] : 0.0f, p1 = 9;
        if (pv.x != 0.0f || pv.y != 0.0f) atomicAdd(reinterpret_cast<float2*>(dst + p2), pv);
        if (sv != 0.0f) atomicAdd(dst + p1, sv);
      } else {
        int k;
        float s = warp_sum10(v, lane, &k);
        s *= k <= 1 ? kInvFalloffScale : (k <= 4 ? kConicFlushScale : 1.0f);
        if ((lane & 1) == 0 && k < GSB_GRAD2D_FLOATS && s != 0.0f) atomicAdd(dst + k, s);
      }
    }
  };
  for (int64_t cb = wmax > lo ? int64_t((wmax - 1) / 32) * 32 : -32; cb >= cb_lo; cb -= 32) {
    const uint32_t li = uint32_t(cb) + lane;
    bool cond = false;
    const bool keep = li >= lo && li < wmax &&
                      load_entry<block_h<PX>(), false>(a, recs, start + li, li, bx0, by0, ws, lane, cond);
    const uint32_t m = __ballot_sync(kFull, keep);
    const bool fast = __all_sync(kFull, cond || !keep);
    // (at four pixels per lane the live walk took 95 registers instead of 80 and was slower)
    const bool live = PX <= 2 && cb + 32 <= int64_t(wmin);
    __syncwarp();
    if (fast) {
      if (live) walk(cb, m, std::true_type{}, std::true_type{});
      else walk(cb, m, std::true_type{}, std::false_type{});
    } else {
      if (live) walk(cb, m, std::false_type{}, std::true_type{});
      else walk(cb, m, std::false_type{}, std::false_type{});
    }
    __syncwarp();  // slots are rewritten by the next chunk
  }
}

// Two pixels per lane halve the per-pixel cost of list streaming, loop control and (backward)
// the reductions, but give each tile half the warps and a longer serial walk, which loses while
// the grid is too small to fill the GPU.  Measured on one B200 (16x16 tiles): the backward gains
// from 4608 tiles up (8 x 384^2: 1.65 -> 1.53 ms; 32 x 1080p: 208 -> 164 ms) and loses at 1024
// (16 x 128^2: 1.09 -> 1.14 ms); the forward, whose pixels also stop early, gains only on the
// largest grids (32 x 1080p: 66 -> 60 ms; 8 x 384^2: 0.60 -> 0.69 ms).
constexpr uint64_t kFwdPairedTiles = 32768;
constexpr uint64_t kBwdPairedTiles = 2048;
// Four pixels per lane (an 8 x 16 block per warp, two warps per 16x16 tile) halve the per-entry
// cost of the walk and the gradient reduction once more; the backward takes them on grids this
// large.  Measured on one B200, 8 x 1920x1080 (65k tiles): backward 31.9 -> 26.9 ms with four; the
// forward 11.70 -> 11.94 ms with the set-bit walk, and with the compact walk 10.60 -> 10.36 ms, so
// it takes four on these grids as well.
// At 4 x 1920x1080 (32,640 tiles, one GPU's share of the 32 views at 8 GPUs): four in both stages
// 22.48 ms a step, two in both 24.08 (backward 14.98 -> 13.49 ms, forward 5.33 -> 5.21); grids
// between the segmented ones (below 8192 tiles) and 16k tiles were not measured.
// (Eight per lane, one warp walking and reducing a whole tile, was measured slower: 26.9 -> 30.7 ms,
// 117 registers; 4% fewer instructions but fewer warps in flight and more idle lanes.)
constexpr uint64_t kQuadTiles = 16384;
// Below this many tiles the backward cuts every tile's list in four (gsb_options.backward_segments
// = 0): four times the CTAs and a quarter of the serial walk per tile, which lets it pair pixels
// per lane at any size, for 72 bytes of checkpoint per pixel.  Measured on one B200, 16 x 128^2
// (1024 tiles): backward 1.10 ms (1 segment) -> 0.92 (2) -> 0.82 (4) -> 0.81 (8, whose forward
// checkpoints cost more than that); with the later kernels 8 x 384^2 (4608 tiles): step 352.8 ->
// 356.4 Mpix/s with 4 segments (backward 1.49 -> 1.43 ms, forward 0.54 -> 0.57); 32 x 1080p
// (261k tiles): 281.6 -> 279.5 with 2, so grids that large keep one segment.
constexpr uint64_t kSegmentedTiles = 8192;
constexpr int kAutoSegments = 4;

// Warps per CTA of the 16x16 kernels: GSB200_RASTER_CW (1, 2, 4 or 8; tuning, results do not
// depend on it), else 2 for the forward and the whole tile for the backward.  Measured on one B200
// (16x16 tiles, warps per CTA 8 / 4 / 2 / 1): forward 16 x 128^2 0.417 / 0.407 / 0.400 / 0.437 ms,
// 8 x 384^2 0.601 / 0.594 / 0.583 / 0.604 ms (small CTAs spread a tile's blocks over SMs that would
// otherwise idle at the end); backward (two pixels per lane, 4 / 2 / 1 warps) 16 x 128^2
// 0.823 / 0.864 / 0.874 ms, where the warps of a tile share the records through L1.
static int cta_warps(int nw, bool backward) {
  const char* v = std::getenv("GSB200_RASTER_CW");
  if (v && (v[0] == '1' || v[0] == '2' || v[0] == '4' || v[0] == '8') && v[1] == '\0') return min(nw, v[0] - '0');
  return backward ? nw : min(nw, 2);
}

template <int TILE, int PX, int NSEG, int CW>
static void fwd_launch_cw(const RasterArgs& a, cudaStream_t st) {
  constexpr int SPLIT = TILE * TILE / (32 * PX) / CW;
  const dim3 grid(unsigned(a.rc.n_tiles) * SPLIT, a.B);  // the CTAs of a tile are adjacent
  if (a.depth) raster_fwd_kernel<TILE, PX, NSEG, CW, true><<<grid, 32 * CW, 0, st>>>(a);
  else raster_fwd_kernel<TILE, PX, NSEG, CW, false><<<grid, 32 * CW, 0, st>>>(a);
}

template <int TILE, int PX, int NSEG>
static void fwd_launch_seg(const RasterArgs& a, cudaStream_t st) {
  constexpr int NW = TILE * TILE / (32 * PX);
  if constexpr (TILE == 16) {
    const int cw = cta_warps(NW, false);
    if (cw == 1) return fwd_launch_cw<TILE, PX, NSEG, 1>(a, st);
    if (cw == 2) return fwd_launch_cw<TILE, PX, NSEG, 2>(a, st);
    if constexpr (NW == 8) {
      if (cw == 4) return fwd_launch_cw<TILE, PX, NSEG, 4>(a, st);
    }
  }
  fwd_launch_cw<TILE, PX, NSEG, NW>(a, st);
}

template <int TILE, int PX>
static void fwd_launch(const RasterArgs& a, cudaStream_t st) {
  note_launch();
  if (a.nseg == 4) fwd_launch_seg<TILE, PX, 4>(a, st);
  else if (a.nseg == 2) fwd_launch_seg<TILE, PX, 2>(a, st);
  else fwd_launch_seg<TILE, PX, 1>(a, st);
}

template <int TILE, int PX, int NSEG, int CW>
static void bwd_launch_cw(const RasterArgs& a, cudaStream_t st) {
  constexpr int SPLIT = TILE * TILE / (32 * PX) / CW;
  const dim3 grid(unsigned(a.rc.n_tiles) * NSEG * SPLIT, a.B);  // the CTAs of a tile are adjacent
  if (a.d_depth) raster_bwd_kernel<TILE, PX, true, NSEG, CW><<<grid, 32 * CW, 0, st>>>(a);
  else raster_bwd_kernel<TILE, PX, false, NSEG, CW><<<grid, 32 * CW, 0, st>>>(a);
}

template <int TILE, int PX, int NSEG>
static void bwd_launch_seg(const RasterArgs& a, cudaStream_t st) {
  constexpr int NW = TILE * TILE / (32 * PX);
  if constexpr (TILE == 16) {
    const int cw = cta_warps(NW, true);
    if (cw == 1) return bwd_launch_cw<TILE, PX, NSEG, 1>(a, st);
    if (cw == 2) return bwd_launch_cw<TILE, PX, NSEG, 2>(a, st);
    if constexpr (NW == 8) {
      if (cw == 4) return bwd_launch_cw<TILE, PX, NSEG, 4>(a, st);
    }
  }
  bwd_launch_cw<TILE, PX, NSEG, NW>(a, st);
}

template <int TILE, int PX>
static void bwd_launch(const RasterArgs& a, cudaStream_t st) {
  note_launch();
  if (a.nseg == 4) bwd_launch_seg<TILE, PX, 4>(a, st);
  else if (a.nseg == 2) bwd_launch_seg<TILE, PX, 2>(a, st);
  else bwd_launch_seg<TILE, PX, 1>(a, st);
}

// GSB200_RASTER_PX=1, 2 or 4 forces the pixels per lane of both stages, GSB200_RASTER_PX_BWD of
// the backward alone (tests and tuning; results do not depend on them; 4 applies to 16x16 tiles
// only); read at every launch so that a process can switch them between calls.
static int forced_px(const char* name) {
  const char* v = std::getenv(name);
  if (v && (v[0] == '1' || v[0] == '2' || v[0] == '4') && v[1] == '\0') return v[0] - '0';
  return 0;
}

static int lane_pixels(uint64_t tiles, uint64_t threshold, bool backward, int tile) {
  int force = backward ? forced_px("GSB200_RASTER_PX_BWD") : 0;
  if (!force) force = forced_px("GSB200_RASTER_PX");
  if (force == 4 && tile != 16) force = 2;
  if (force) return force;
  if (tile == 16 && tiles >= kQuadTiles) return 4;
  return tiles >= threshold ? 2 : 1;
}

gsb_status launch_raster_fwd(const RasterArgs& a, cudaStream_t st) {
  // the compact walk (two or more pixels per lane) needs an inverse of F0 with F0 * inv_f0 == 1
  const int px = a.rc.unit_inv ? lane_pixels(uint64_t(a.rc.n_tiles) * uint64_t(a.B), kFwdPairedTiles, false,
                                             a.rc.tile)
                               : 1;
  if (a.rc.tile == 16) px == 4 ? fwd_launch<16, 4>(a, st) : px == 2 ? fwd_launch<16, 2>(a, st) : fwd_launch<16, 1>(a, st);
  else if (a.rc.tile == 8) px == 2 ? fwd_launch<8, 2>(a, st) : fwd_launch<8, 1>(a, st);
  else return GSB_ERR_ARG;
  return launch_status();
}

gsb_status launch_raster_bwd(const RasterArgs& a, cudaStream_t st) {
  if (cudaMemsetAsync(a.grad2d, 0, size_t(a.B) * a.G * GSB_GRAD2D_FLOATS * sizeof(float), st)) return GSB_ERR_CUDA;
  // segmented lists restore the parallelism two pixels per lane gives up: pair them always then
  const int px =
      lane_pixels(uint64_t(a.rc.n_tiles) * uint64_t(a.B), a.nseg > 1 ? 0 : kBwdPairedTiles, true, a.rc.tile);
  if (a.rc.tile == 16) px == 4 ? bwd_launch<16, 4>(a, st) : px == 2 ? bwd_launch<16, 2>(a, st) : bwd_launch<16, 1>(a, st);
  else if (a.rc.tile == 8) px == 2 ? bwd_launch<8, 2>(a, st) : bwd_launch<8, 1>(a, st);
  else return GSB_ERR_ARG;
  return launch_status();
}

int raster_segments(const gsb_views& v, const gsb_options& o) {
  if (o.backward_segments == 1 || o.backward_segments == 2 || o.backward_segments == 4) return o.backward_segments;
  const uint64_t tiles = uint64_t(v.n_views) * uint64_t((v.width + o.tile_size - 1) / o.tile_size) *
                         uint64_t((v.height + o.tile_size - 1) / o.tile_size);
  return tiles < kSegmentedTiles ? kAutoSegments : 1;
}

}  // namespace gsb
