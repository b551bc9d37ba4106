// Raster: per-tile front-to-back blend and its reverse-order backward.
//
// One CTA per (view, tile), one thread per pixel (16x16 tile: 8 warps, each an 8x4 pixel block).
// The tile's list (sorted pair keys, low 32 bits = depth rank) is consumed in batches of one entry
// per thread: each thread gathers one projected record into shared memory, then every thread
// walks the batch for its pixel.
//
// Semantics of the reference's dense blend (src/train/renderers/dense.py:208-233):
//   alpha_i = clamp(o_i exp(min(power_i, 0)), 0, alpha_clamp)     (dense.py:217-220)
//   T_i     = prod_{j<i} fl32(fl32(1 - alpha_j) + eps)  over ALL Gaussians of the view in depth
//             order (dense.py:222-228); a Gaussian absent from the tile list contributes
//             F0 = fl32(1 + eps), restored here from depth ranks:
//             T before entry 0 = F0^rank0, T after entry i *= f_i * F0^(rank_{i+1} - rank_i - 1)
//   out     = clamp(sum w c + (1 - clamp(sum w, 0, 1)) bg, 0, 1), w = T alpha (dense.py:229-233)
// Pairs with alpha < alpha_cutoff count as alpha = 0 (exact for alpha <= 2^-25, where
// fl32(1 - alpha) == 1); a pixel stops once T < transmittance_threshold.  In tiled-compat mode
// F0 = 1 between entries (tile-local products, tiled.py:176-185), nothing is skipped and nothing
// stops.
#include "gsb_common.cuh"
#include "gsb_internal.h"

namespace gsb {


constexpr uint32_t kCountBits = 28;
constexpr uint32_t kCountMask = (1u << kCountBits) - 1u;

// q = A dx^2 + B dx dy + C dy^2 with a fixed rounding sequence (forward and backward must agree).
__device__ __forceinline__ float pair_q(float A, float B, float C, float dx, float dy) {
  const float t0 = __fmul_rn(__fmul_rn(A, dx), dx);
  const float t1 = __fmaf_rn(__fmul_rn(B, dx), dy, t0);
  return __fmaf_rn(__fmul_rn(C, dy), dy, t1);
}

template <int TILE>
__device__ __forceinline__ void pixel_of(int tid, int& lx, int& ly) {
  const int lane = tid & 31, warp = tid >> 5;
  if (TILE == 16) {
    lx = (warp & 1) * 8 + (lane & 7);
    ly = (warp >> 1) * 4 + (lane >> 3);
  } else {
    lx = lane & 7;
    ly = warp * 4 + (lane >> 3);
  }
}

// Loads list entry idx of [start, end) into shared slot `slot`.
__device__ __forceinline__ void load_entry(const RasterArgs& a, const float* recs, uint32_t idx, uint32_t end,
                                           int slot, float4* s_geo, float4* s_cot, float4* s_col, float* s_skip,
                                           uint32_t* s_rank) {
  const uint32_t r = min(uint32_t(a.keys[idx]), uint32_t(a.G - 1));  // ranks are < G for valid keys
  const uint32_t rn = (idx + 1 < end) ? uint32_t(a.keys[idx + 1]) : r + 1u;
  const float4* rec = reinterpret_cast<const float4*>(recs + size_t(r) * GSB_RECORD_FLOATS);
  const float4 r0 = __ldg(rec + 0), r1 = __ldg(rec + 1), r2 = __ldg(rec + 2);
  float E = 1.0f, Es = a.rc.f0;
  if (a.rc.log2_f0 != 0.0f) {
    E = exp2f(float(rn - r - 1u) * a.rc.log2_f0);
    Es = exp2f(float(rn - r) * a.rc.log2_f0);
  }
  s_geo[slot] = r0;
  s_cot[slot] = make_float4(r1.x, r1.y, r1.w, E);
  s_col[slot] = make_float4(r2.x, r2.y, r2.z, r1.z);
  s_skip[slot] = Es;
  if (s_rank) s_rank[slot] = r;
}

template <int TILE>
__global__ void __launch_bounds__(TILE* TILE) raster_fwd_kernel(RasterArgs a) {
  constexpr int NT = TILE * TILE;
  __shared__ float4 s_geo[NT];  // mx, my, A, B
  __shared__ float4 s_cot[NT];  // C, opacity, tau, E
  __shared__ float4 s_col[NT];  // r, g, b, z
  __shared__ float s_skip[NT];  // F0 * E: the factor of a skipped pair
  __shared__ float s_t0;
  const RenderConsts& rc = a.rc;
  const int tile = blockIdx.x, view = blockIdx.y;
  const int tx = tile % rc.tiles_x, ty = tile / rc.tiles_x;
  const int tid = threadIdx.x;
  int lx, ly;
  pixel_of<TILE>(tid, lx, ly);
  const int px = tx * TILE + lx, py = ty * TILE + ly;
  const bool inside = px < a.W && py < a.H;
  const float fx = float(px) + rc.pixel_center, fy = float(py) + rc.pixel_center;
  const size_t rb = (size_t(view) * rc.n_tiles + tile) * 2;
  const uint32_t start = a.ranges[rb], end = a.ranges[rb + 1];
  const float* recs = a.records + size_t(view) * a.G * GSB_RECORD_FLOATS;

  float T = 1.0f, C0 = 0.0f, C1 = 0.0f, C2 = 0.0f, Ws = 0.0f, D = 0.0f;
  uint32_t n_proc = end - start;
  bool done = !inside;
  for (uint32_t b0 = start; b0 < end; b0 += NT) {
    if (__syncthreads_and(done)) break;
    const uint32_t idx = b0 + tid;
    if (idx < end) load_entry(a, recs, idx, end, tid, s_geo, s_cot, s_col, s_skip, nullptr);
    if (idx == start) s_t0 = rc.log2_f0 != 0.0f ? exp2f(float(uint32_t(a.keys[start])) * rc.log2_f0) : 1.0f;
    __syncthreads();
    if (b0 == start) T = s_t0;
    if (done) continue;
    const int nb = min(NT, int(end - b0));
    for (int j = 0; j < nb; ++j) {
      const float4 g = s_geo[j];
      const float4 ct = s_cot[j];
      const float dx = __fsub_rn(fx, g.x), dy = __fsub_rn(fy, g.y);
      const float q = pair_q(g.z, g.w, ct.x, dx, dy);
      float fac = s_skip[j];
      if (q <= ct.z) {
        const float e = __expf(fminf(-0.5f * q, 0.0f));
        const float alpha = fminf(fmaxf(ct.y * e, 0.0f), rc.alpha_clamp);
        if (alpha >= rc.alpha_cutoff) {
          const float4 c = s_col[j];
          const float w = T * alpha;
          C0 = fmaf(w, c.x, C0);
          C1 = fmaf(w, c.y, C1);
          C2 = fmaf(w, c.z, C2);
          Ws += w;
          D = fmaf(w, c.w, D);
          fac = __fmul_rn(__fadd_rn(__fsub_rn(1.0f, alpha), rc.eps), ct.w);
        }
      }
      T = __fmul_rn(T, fac);
      if (T < rc.t_threshold) {
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
  a.pixel_t[pix] = T;
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
  constexpr int NT = TILE * TILE;
  __shared__ float4 s_geo[NT];
  __shared__ float4 s_cot[NT];
  __shared__ float4 s_col[NT];
  __shared__ float s_skip[NT];
  __shared__ uint32_t s_rank[NT];
  __shared__ uint32_t s_red[NT / 32];
  const RenderConsts& rc = a.rc;
  const int tile = blockIdx.x, view = blockIdx.y;
  const int tx = tile % rc.tiles_x, ty = tile / rc.tiles_x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int lx, ly;
  pixel_of<TILE>(tid, lx, ly);
  const int px = tx * TILE + lx, py = ty * TILE + ly;
  const bool inside = px < a.W && py < a.H;
  const float fx = float(px) + rc.pixel_center, fy = float(py) + rc.pixel_center;
  const size_t rb = (size_t(view) * rc.n_tiles + tile) * 2;
  const uint32_t start = a.ranges[rb], end = a.ranges[rb + 1];
  const float* recs = a.records + size_t(view) * a.G * GSB_RECORD_FLOATS;
  float* g2 = a.grad2d + size_t(view) * a.G * GSB_GRAD2D_FLOATS;

  const size_t HW = size_t(a.H) * a.W;
  const size_t poff = size_t(py) * a.W + px;
  const size_t pix = size_t(view) * HW + poff;
  float T = 0.0f, g0 = 0.0f, g1 = 0.0f, g2c = 0.0f, gW = 0.0f, gD = 0.0f;
  uint32_t n_proc = 0;
  if (inside) {
    T = a.pixel_t[pix];
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
  for (int w = 0; w < NT / 32; ++w) max_n = max(max_n, s_red[w]);

  float R0 = 0.0f, R1 = 0.0f, R2 = 0.0f, RW = 0.0f, RD = 0.0f;
  for (int64_t be = max_n; be > 0; be -= NT) {
    const uint32_t bs = uint32_t(be > NT ? be - NT : 0);
    const int nb = int(be - bs);
    __syncthreads();
    if (tid < nb) load_entry(a, recs, start + bs + tid, end, tid, s_geo, s_cot, s_col, s_skip, s_rank);
    __syncthreads();
    for (int j = nb - 1; j >= 0; --j) {
      float v[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) v[k] = 0.0f;
      bool contrib = false;
      if (bs + uint32_t(j) < n_proc) {
        const float4 g = s_geo[j];
        const float4 ct = s_cot[j];
        const float dx = __fsub_rn(fx, g.x), dy = __fsub_rn(fy, g.y);
        const float q = pair_q(g.z, g.w, ct.x, dx, dy);
        float fac = s_skip[j];
        float alpha = 0.0f, e = 0.0f;
        bool hit = false;
        if (q <= ct.z) {
          e = __expf(fminf(-0.5f * q, 0.0f));
          alpha = fminf(fmaxf(ct.y * e, 0.0f), rc.alpha_clamp);
          if (alpha >= rc.alpha_cutoff) {
            hit = true;
            fac = __fmul_rn(__fadd_rn(__fsub_rn(1.0f, alpha), rc.eps), ct.w);
          }
        }
        T = __fdiv_rn(T, fac);  // T before this entry
        if (hit) {
          const float4 c = s_col[j];
          const float w = T * alpha;
          const float f = __fadd_rn(__fsub_rn(1.0f, alpha), rc.eps);
          const float dldw = g0 * c.x + g1 * c.y + g2c * c.z + gW + gD * c.w;
          const float dlda = T * dldw - (g0 * R0 + g1 * R1 + g2c * R2 + gW * RW + gD * RD) / f;
          R0 = fmaf(w, c.x, R0);
          R1 = fmaf(w, c.y, R1);
          R2 = fmaf(w, c.z, R2);
          RW += w;
          RD = fmaf(w, c.w, RD);
          const float araw = ct.y * e;
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
