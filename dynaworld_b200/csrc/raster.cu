// Raster: per-tile front-to-back blend and its reverse-order backward.
//
// One CTA per (view, tile), one thread per pixel (16x16 tile: 8 warps, each an 8x4 pixel block).
// The tile's list (sorted pair keys, low 32 bits = depth rank) is consumed in batches of one entry
// per thread: each thread gathers one projected record into shared memory and marks which warp
// blocks the Gaussian's ellipse box reaches; each warp then compacts the batch to the entries that
// reach its block and walks only those.
//
// Semantics of the reference's dense blend (src/train/renderers/dense.py:208-233):
//   alpha_i = clamp(o_i exp(min(power_i, 0)), 0, alpha_clamp)     (dense.py:217-220)
//   T_i     = prod_{j<i} fl32(fl32(1 - alpha_j) + eps)  over ALL Gaussians of the view in depth
//             order (dense.py:222-228); a Gaussian that does not touch the pixel contributes
//             F0 = fl32(1 + eps) (exactly so when its alpha <= 2^-25).
//   out     = clamp(sum w c + (1 - clamp(sum w, 0, 1)) bg, 0, 1), w = T alpha (dense.py:229-233)
// With pos_i the depth rank of entry i (exact mode) or its index in the tile list (tiled-compat
// mode, tile-local products as tiled.py:176-185):
//   T_i = F0^pos_i * S_i,   S_i = prod_{blended j < i} f_j / F0,
// so entries a pixel skips leave S unchanged and cost nothing.  A pair is skipped when its alpha
// is below alpha_cutoff, or when q exceeds the Gaussian's threshold (alpha < max(cutoff, 2^-25));
// a pixel stops once T falls below the transmittance threshold.
#include "gsb_common.cuh"
#include "gsb_internal.h"

namespace gsb {

constexpr uint32_t kCountBits = 28;
constexpr uint32_t kCountMask = (1u << kCountBits) - 1u;

// q = A dx^2 + B dx dy + C dy^2 with a fixed rounding sequence (forward and backward agree).
__device__ __forceinline__ float pair_q(float A, float B, float C, float dx, float dy) {
  const float t0 = __fmul_rn(__fmul_rn(A, dx), dx);
  const float t1 = __fmaf_rn(__fmul_rn(B, dx), dy, t0);
  return __fmaf_rn(__fmul_rn(C, dy), dy, t1);
}

// Pixel of thread tid: warp w covers the 8x4 block (w % (TILE/8), w / (TILE/8)).
template <int TILE>
__device__ __forceinline__ void pixel_of(int tid, int& lx, int& ly) {
  const int lane = tid & 31, warp = tid >> 5;
  constexpr int BX = TILE / 8;
  lx = (warp % BX) * 8 + (lane & 7);
  ly = (warp / BX) * 4 + (lane >> 3);
}

struct Batch {
  float4* geo;    // mx, my, A, B
  float4* cot;    // C, opacity, tau, F0^pos
  float4* col;    // r, g, b, z
  uint32_t* rank; // depth rank (gradient slot)
  uint32_t* mask; // warp blocks the entry's box reaches
};

// Loads list entry idx of the tile (list index li) into slot `slot` and marks the warp blocks of
// the tile that the ellipse box {q <= tau} reaches (conservative).
template <int TILE>
__device__ __forceinline__ void load_entry(const RasterArgs& a, const float* recs, uint32_t idx, uint32_t li,
                                           int slot, int tile_x0, int tile_y0, const Batch& s) {
  constexpr int NW = TILE * TILE / 32, BX = TILE / 8;
  const uint32_t r = min(uint32_t(a.keys[idx]), uint32_t(a.G - 1));  // ranks are < G for valid keys
  const float4* rec = reinterpret_cast<const float4*>(recs + size_t(r) * GSB_RECORD_FLOATS);
  const float4 r0 = __ldg(rec + 0), r1 = __ldg(rec + 1), r2 = __ldg(rec + 2);
  const float pos = a.rc.compat ? float(li) : float(r);
  const float pw = a.rc.log2_f0 != 0.0f ? exp2f(pos * a.rc.log2_f0) : 1.0f;
  s.geo[slot] = r0;
  s.cot[slot] = make_float4(r1.x, r1.y, r1.w, pw);
  s.col[slot] = make_float4(r2.x, r2.y, r2.z, r1.z);
  s.rank[slot] = r;
  // box of the ellipse q <= tau: half extents sqrt(tau (A^-1)_ii), (A^-1)_00 = C/det
  const float A = r0.z, B = r0.w, C = r1.x, tau = r1.w;
  uint32_t m = 0;
  if (tau >= 0.0f) {
    const float det = A * C - 0.25f * B * B;
    float ex, ey;
    if (det > 0.0f && isfinite(tau)) {
      ex = sqrtf(tau * C / det) * 1.0001f + 0.01f;
      ey = sqrtf(tau * A / det) * 1.0001f + 0.01f;
    } else {
      ex = ey = __int_as_float(0x7f800000);
    }
    const float pc = a.rc.pixel_center;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float bx0 = float(tile_x0 + (w % BX) * 8) + pc, by0 = float(tile_y0 + (w / BX) * 4) + pc;
      const bool hit = (r0.x + ex >= bx0) && (r0.x - ex <= bx0 + 7.0f) && (r0.y + ey >= by0) &&
                       (r0.y - ey <= by0 + 3.0f);
      m |= hit ? (1u << w) : 0u;
    }
  }
  s.mask[slot] = m;
}

// Compacts the batch's entries that reach this warp's block into list[0..count), in list order.
__device__ __forceinline__ int compact_warp(const uint32_t* mask, int nb, int warp, int lane, uint16_t* list) {
  int count = 0;
  for (int c = 0; c < nb; c += 32) {
    const int slot = c + lane;
    const bool keep = slot < nb && ((mask[slot] >> warp) & 1u);
    const uint32_t bal = __ballot_sync(0xffffffffu, keep);
    if (keep) list[count + __popc(bal & ((1u << lane) - 1u))] = uint16_t(slot);
    count += __popc(bal);
  }
  __syncwarp();
  return count;
}

template <int TILE>
__global__ void __launch_bounds__(TILE* TILE) raster_fwd_kernel(RasterArgs a) {
  constexpr int NT = TILE * TILE, NW = NT / 32;
  __shared__ float4 s_geo[NT], s_cot[NT], s_col[NT];
  __shared__ uint32_t s_rank[NT], s_mask[NT];
  __shared__ uint16_t s_list[NW][NT];
  const Batch sb{s_geo, s_cot, s_col, s_rank, s_mask};
  const RenderConsts& rc = a.rc;
  const int tile = blockIdx.x, view = blockIdx.y;
  const int tile_x0 = (tile % rc.tiles_x) * TILE, tile_y0 = (tile / rc.tiles_x) * TILE;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int lx, ly;
  pixel_of<TILE>(tid, lx, ly);
  const int px = tile_x0 + lx, py = tile_y0 + ly;
  const bool inside = px < a.W && py < a.H;
  const float fx = float(px) + rc.pixel_center, fy = float(py) + rc.pixel_center;
  const size_t rb = (size_t(view) * rc.n_tiles + tile) * 2;
  const uint32_t start = a.ranges[rb], end = a.ranges[rb + 1];
  const float* recs = a.records + size_t(view) * a.G * GSB_RECORD_FLOATS;
  const float inv_f0 = 1.0f / rc.f0;

  float S = 1.0f, C0 = 0.0f, C1 = 0.0f, C2 = 0.0f, Ws = 0.0f, D = 0.0f;
  uint32_t n_proc = end - start;
  bool done = !inside;
  for (uint32_t b0 = start; b0 < end; b0 += NT) {
    if (__syncthreads_and(done)) break;
    const int nb = min(NT, int(end - b0));
    if (tid < nb) load_entry<TILE>(a, recs, b0 + tid, b0 + tid - start, tid, tile_x0, tile_y0, sb);
    __syncthreads();
    const int cnt = compact_warp(s_mask, nb, warp, lane, s_list[warp]);
    if (done) continue;
    for (int i = 0; i < cnt; ++i) {
      const int j = s_list[warp][i];
      const float4 g = s_geo[j];
      const float4 ct = s_cot[j];
      const float dx = __fsub_rn(fx, g.x), dy = __fsub_rn(fy, g.y);
      const float q = pair_q(g.z, g.w, ct.x, dx, dy);
      if (!(q <= ct.z)) continue;
      const float e = __expf(fminf(-0.5f * q, 0.0f));
      const float alpha = fminf(fmaxf(ct.y * e, 0.0f), rc.alpha_clamp);
      if (!(alpha >= rc.alpha_cutoff)) continue;
      const float4 c = s_col[j];
      const float T = S * ct.w;
      const float w = T * alpha;
      C0 = fmaf(w, c.x, C0);
      C1 = fmaf(w, c.y, C1);
      C2 = fmaf(w, c.z, C2);
      Ws += w;
      D = fmaf(w, c.w, D);
      const float f = __fadd_rn(__fsub_rn(1.0f, alpha), rc.eps);
      S = S * (f * inv_f0);
      if (T * f < rc.t_threshold) {  // T after this entry
        done = true;
        n_proc = b0 - start + uint32_t(j) + 1u;
        break;
      }
    }
  }
  if (!inside) return;
  const size_t HW = size_t(a.H) * a.W;
  const size_t poff = size_t(py) * a.W + px;
  const size_t pix = size_t(view) * HW + poff;
  const float wc = fminf(fmaxf(Ws, 0.0f), 1.0f);
  const float one_m = __fsub_rn(1.0f, wc);
  const float col[3] = {C0, C1, C2};
  uint32_t mask = (Ws >= 0.0f && Ws <= 1.0f) ? 8u : 0u;
#pragma unroll
  for (int ch = 0; ch < 3; ++ch) {
    const float pre = __fadd_rn(col[ch], __fmul_rn(one_m, rc.bg[ch]));
    if (pre >= 0.0f && pre <= 1.0f) mask |= 1u << ch;
    a.image[(size_t(view) * 3 + ch) * HW + poff] = fminf(fmaxf(pre, 0.0f), 1.0f);
  }
  if (a.alpha) a.alpha[pix] = Ws;
  if (a.depth) a.depth[pix] = D;
  a.pixel_t[pix] = S;  // normalised transmittance after the last blended entry
  a.pixel_state[pix] = min(n_proc, kCountMask) | (mask << kCountBits);
}

// Sum of each of 16 per-lane values over the warp; afterwards lane l holds the total of value
// l >> 1.  Recursive halving: 8 + 4 + 2 + 1 + 1 shuffles instead of 16 * 5.
__device__ __forceinline__ float warp_sum16(float v[16], int lane) {
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const bool up = lane & 16;
    const float send = up ? v[k] : v[k + 8];
    const float keep = up ? v[k + 8] : v[k];
    v[k] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const bool up = lane & 8;
    const float send = up ? v[k] : v[k + 4];
    const float keep = up ? v[k + 4] : v[k];
    v[k] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const bool up = lane & 4;
    const float send = up ? v[k] : v[k + 2];
    const float keep = up ? v[k + 2] : v[k];
    v[k] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  {
    const bool up = lane & 2;
    const float send = up ? v[0] : v[1];
    const float keep = up ? v[1] : v[0];
    v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  }
  return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
}

template <int TILE>
__global__ void __launch_bounds__(TILE* TILE) raster_bwd_kernel(RasterArgs a) {
  constexpr int NT = TILE * TILE, NW = NT / 32;
  __shared__ float4 s_geo[NT], s_cot[NT], s_col[NT];
  __shared__ uint32_t s_rank[NT], s_mask[NT];
  __shared__ uint16_t s_list[NW][NT];
  __shared__ uint32_t s_red[NW];
  const Batch sb{s_geo, s_cot, s_col, s_rank, s_mask};
  const RenderConsts& rc = a.rc;
  const int tile = blockIdx.x, view = blockIdx.y;
  const int tile_x0 = (tile % rc.tiles_x) * TILE, tile_y0 = (tile / rc.tiles_x) * TILE;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int lx, ly;
  pixel_of<TILE>(tid, lx, ly);
  const int px = tile_x0 + lx, py = tile_y0 + ly;
  const bool inside = px < a.W && py < a.H;
  const float fx = float(px) + rc.pixel_center, fy = float(py) + rc.pixel_center;
  const size_t rb = (size_t(view) * rc.n_tiles + tile) * 2;
  const uint32_t start = a.ranges[rb], end = a.ranges[rb + 1];
  const float* recs = a.records + size_t(view) * a.G * GSB_RECORD_FLOATS;
  float* g2 = a.grad2d + size_t(view) * a.G * GSB_GRAD2D_FLOATS;
  const float inv_f0 = 1.0f / rc.f0;

  const size_t HW = size_t(a.H) * a.W;
  const size_t poff = size_t(py) * a.W + px;
  const size_t pix = size_t(view) * HW + poff;
  float S = 0.0f, g0 = 0.0f, g1 = 0.0f, g2c = 0.0f, gW = 0.0f, gD = 0.0f;
  uint32_t n_proc = 0;
  if (inside) {
    S = a.pixel_t[pix];
    const uint32_t st = a.pixel_state[pix];
    n_proc = st & kCountMask;
    const uint32_t mask = st >> kCountBits;
    const float sc = a.view_scale ? a.view_scale[view] : 1.0f;
    const float* di = a.d_image + size_t(view) * 3 * HW + poff;
    g0 = (mask & 1u) ? di[0] * sc : 0.0f;
    g1 = (mask & 2u) ? di[HW] * sc : 0.0f;
    g2c = (mask & 4u) ? di[2 * HW] * sc : 0.0f;
    gW = (mask & 8u) ? -(g0 * rc.bg[0] + g1 * rc.bg[1] + g2c * rc.bg[2]) : 0.0f;
    if (a.d_alpha) gW += a.d_alpha[pix];
    if (a.d_depth) gD = a.d_depth[pix];
  }
  const uint32_t wmax = __reduce_max_sync(0xffffffffu, n_proc);
  if (lane == 0) s_red[warp] = wmax;
  __syncthreads();
  uint32_t max_n = 0;
#pragma unroll
  for (int w = 0; w < NW; ++w) max_n = max(max_n, s_red[w]);

  float R0 = 0.0f, R1 = 0.0f, R2 = 0.0f, RW = 0.0f, RD = 0.0f;
  for (int64_t be = max_n; be > 0; be -= NT) {
    const uint32_t bs = uint32_t(be > NT ? be - NT : 0);
    const int nb = int(be - bs);
    __syncthreads();
    if (tid < nb) load_entry<TILE>(a, recs, start + bs + tid, bs + tid, tid, tile_x0, tile_y0, sb);
    __syncthreads();
    const int cnt = compact_warp(s_mask, nb, warp, lane, s_list[warp]);
    for (int i = cnt - 1; i >= 0; --i) {
      const int j = s_list[warp][i];
      float v[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) v[k] = 0.0f;
      bool contrib = false;
      if (bs + uint32_t(j) < n_proc) {
        const float4 g = s_geo[j];
        const float4 ct = s_cot[j];
        const float dx = __fsub_rn(fx, g.x), dy = __fsub_rn(fy, g.y);
        const float q = pair_q(g.z, g.w, ct.x, dx, dy);
        if (q <= ct.z) {
          const float e = __expf(fminf(-0.5f * q, 0.0f));
          const float araw = ct.y * e;
          const float alpha = fminf(fmaxf(araw, 0.0f), rc.alpha_clamp);
          if (alpha >= rc.alpha_cutoff) {
            const float f = __fadd_rn(__fsub_rn(1.0f, alpha), rc.eps);
            S = __fdividef(S, f * inv_f0);  // S before this entry
            const float T = S * ct.w;
            const float4 c = s_col[j];
            const float w = T * alpha;
            const float dldw = g0 * c.x + g1 * c.y + g2c * c.z + gW + gD * c.w;
            const float dlda = T * dldw - __fdividef(g0 * R0 + g1 * R1 + g2c * R2 + gW * RW + gD * RD, f);
            R0 = fmaf(w, c.x, R0);
            R1 = fmaf(w, c.y, R1);
            R2 = fmaf(w, c.z, R2);
            RW += w;
            RD = fmaf(w, c.w, RD);
            const float dlr = (araw >= 0.0f && araw <= rc.alpha_clamp) ? dlda : 0.0f;
            const float power = -0.5f * q;
            const float pmask = power < 0.0f ? 1.0f : (power == 0.0f ? 0.5f : 0.0f);
            const float dpow = dlr * araw * pmask;
            v[0] = dpow * (g.z * dx + 0.5f * g.w * dy);
            v[1] = dpow * (ct.x * dy + 0.5f * g.w * dx);
            v[2] = -0.5f * dpow * dx * dx;
            v[3] = -0.5f * dpow * dx * dy;
            v[4] = -0.5f * dpow * dy * dy;
            v[5] = dlr * e;
            v[6] = g0 * w;
            v[7] = g1 * w;
            v[8] = g2c * w;
            v[9] = gD * w;
            contrib = true;
          }
        }
      }
      if (__any_sync(0xffffffffu, contrib)) {
        const float s = warp_sum16(v, lane);
        const int k = lane >> 1;
        if ((lane & 1) == 0 && k < GSB_GRAD2D_FLOATS && s != 0.0f)
          atomicAdd(g2 + size_t(s_rank[j]) * GSB_GRAD2D_FLOATS + k, s);
      }
    }
  }
}

gsb_status launch_raster_fwd(const RasterArgs& a, cudaStream_t st) {
  const dim3 grid(a.rc.n_tiles, a.B);
  if (a.rc.tile == 16) { note_launch(); raster_fwd_kernel<16><<<grid, 256, 0, st>>>(a); }
  else if (a.rc.tile == 8) { note_launch(); raster_fwd_kernel<8><<<grid, 64, 0, st>>>(a); }
  else return GSB_ERR_ARG;
  return cudaPeekAtLastError() == cudaSuccess ? GSB_OK : GSB_ERR_CUDA;
}

gsb_status launch_raster_bwd(const RasterArgs& a, cudaStream_t st) {
  if (cudaMemsetAsync(a.grad2d, 0, size_t(a.B) * a.G * GSB_GRAD2D_FLOATS * sizeof(float), st)) return GSB_ERR_CUDA;
  const dim3 grid(a.rc.n_tiles, a.B);
  if (a.rc.tile == 16) { note_launch(); raster_bwd_kernel<16><<<grid, 256, 0, st>>>(a); }
  else if (a.rc.tile == 8) { note_launch(); raster_bwd_kernel<8><<<grid, 64, 0, st>>>(a); }
  else return GSB_ERR_ARG;
  return cudaPeekAtLastError() == cudaSuccess ? GSB_OK : GSB_ERR_CUDA;
}

}  // namespace gsb
