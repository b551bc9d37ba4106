// Entry from already-projected 2-D Gaussians: the reference's 2-D rasterizer contracts.
//
//  * conic format -- rasterize_projected_gaussians of the fast-mac bridge
//    (third_party/fast-mac-gsplat-scaffold/torch_gsplat_bridge/rasterize.py:93-126, called by
//    src/train/renderers/fast_mac.py:253,301): mean2d, conic (a, b, c) with power
//    -0.5 (a dx^2 + 2 b dx dy + c dy^2) (gsplat_kernels.metal:188), opacity, colour, and a depth
//    that orders the blend.  Culling as snugbox_count (gsplat_kernels.metal:57-59): opacity above
//    the alpha threshold, a > 0, c > 0, a c - b^2 > 1e-8.
//  * packed format -- rows [mean x, y, axis x, y, sigma0, sigma1, opacity] of
//    src/train/renderers/taichi.py:107-176 and src/benchmarks/splat_renderer_accuracy.py:262-305:
//    q = (d.axis / sigma0)^2 + (d.perp / sigma1)^2 with perp = (-axis y, axis x), which is the
//    conic a = ax^2/s0^2 + ay^2/s1^2, b = ax ay (1/s0^2 - 1/s1^2), c = ay^2/s0^2 + ax^2/s1^2
//    (src/benchmarks/raw_metal_mlx_bridge.py:106-121).
//
// Both become the projected records the 3-D path writes (mx, my, A, B, C with B = 2 b the dx dy
// coefficient), in per-image blend order, so binning and both raster stages are shared.
#include "gsb_common.cuh"
#include "gsb_internal.h"
#include "tiles.cuh"

namespace gsb {

namespace {

constexpr int kPackedFloats = 7;

struct Conic2D {
  float mx, my, A, B, C, o;
};

__device__ inline Conic2D load_conic(const gsb_splats2d& sp, size_t i) {
  Conic2D g;
  if (sp.format == GSB_SPLATS2D_PACKED) {
    const float* p = sp.packed + i * kPackedFloats;
    const float ax = p[2], ay = p[3], s0 = p[4], s1 = p[5];
    const float u0 = 1.0f / (s0 * s0), u1 = 1.0f / (s1 * s1);
    g.mx = p[0], g.my = p[1], g.o = p[6];
    g.A = ax * ax * u0 + ay * ay * u1;
    g.B = 2.0f * (ax * ay * (u0 - u1));
    g.C = ay * ay * u0 + ax * ax * u1;
  } else {
    g.mx = sp.means[i * 2 + 0], g.my = sp.means[i * 2 + 1], g.o = sp.opacities[i];
    const float a = sp.conics[i * 3 + 0], b = sp.conics[i * 3 + 1], c = sp.conics[i * 3 + 2];
    g.A = a, g.B = 2.0f * b, g.C = c;
  }
  return g;
}

constexpr int kOrderThreads = 256;
constexpr int kOrderItems = 8;  // Gaussians per thread

// Depth keys of view blockIdx.y (NULL depths: index order, keys 0) with the index as value, and the
// view's digit histograms for the segmented sort.
__global__ void __launch_bounds__(kOrderThreads) order_keys_2d_kernel(const float* __restrict__ depths, int32_t G,
                                                                      uint32_t* __restrict__ keys,
                                                                      uint32_t* __restrict__ vals,
                                                                      uint32_t* __restrict__ hist) {
  __shared__ uint32_t s_hist[4][256];
  for (int i = threadIdx.x; i < 4 * 256; i += kOrderThreads) s_hist[i / 256][i % 256] = 0u;
  __syncthreads();
  const size_t b = blockIdx.y;
  const size_t g0 = size_t(blockIdx.x) * kOrderThreads * kOrderItems + threadIdx.x;
  for (int it = 0; it < kOrderItems; ++it) {
    const size_t g = g0 + size_t(it) * kOrderThreads;
    const bool valid = g < size_t(G);
    uint32_t key = 0u;
    if (valid) {
      const size_t i = b * size_t(G) + g;
      key = depths ? float_sort_key(depths[i]) : 0u;
      keys[i] = key;
      vals[i] = uint32_t(g);
    }
    count_digits4(s_hist, key, valid);
  }
  __syncthreads();
  flush_digits4(s_hist, hist + b * 4 * 256);
}

__global__ void __launch_bounds__(256) preprocess_2d_kernel(gsb_splats2d sp, int H, int W, RenderConsts rc,
                                                            const int32_t* __restrict__ rank_of,
                                                            float* __restrict__ records, int4* __restrict__ rects,
                                                            uint32_t* __restrict__ counts) {
  const size_t G = sp.n_gaussians;
  const size_t total = size_t(sp.n_views) * G;
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < total; i += size_t(gridDim.x) * blockDim.x) {
    const size_t b = i / G;
    const Conic2D g = load_conic(sp, i);
    bool visible = true;
    if (sp.format == GSB_SPLATS2D_CONIC) {
      const float hb = 0.5f * g.B;
      visible = g.A * g.C - hb * hb > 1e-8f;
    }
    ExactShape es;
    TileRect rect{1, 1, 0, 0};
    uint32_t count = 0;
    float tau_f = -1.0f;
    if (visible && exact_shape(g.mx, g.my, g.A, g.B, g.C, g.o, rc.alpha_cutoff, H, W, rc.pixel_center, &es)) {
      rect = exact_rect_of(es, rc.tile);
      if (!rc.ellipse) count = uint32_t(rect.count());  // else counted afterwards (pairs_kernel)
      tau_f = __double2float_ru(es.L);
    }
    const size_t slot = b * G + size_t(rank_of[i]);
    float4* rec = reinterpret_cast<float4*>(records + slot * GSB_RECORD_FLOATS);
    rec[0] = make_float4(g.mx, g.my, g.A, g.B);
    rec[1] = make_float4(g.C, g.o, sp.depths ? sp.depths[i] : 0.0f, tau_f);
    rec[2] = make_float4(sp.colors[i * 3 + 0], sp.colors[i * 3 + 1], sp.colors[i * 3 + 2], 0.0f);
    rec[3] = cull_extents(g.A, g.B, g.C, tau_f);
    rects[slot] = make_int4(rect.tx0, rect.ty0, rect.tx1, rect.ty1);
    counts[slot] = count;
  }
}

// grad2d (blend order; d/d(mx, my, A, B, C, opacity, r, g, b)) back to the caller's parameters.
__global__ void preprocess_2d_bwd_kernel(gsb_splats2d sp, const int32_t* __restrict__ rank_of,
                                         const float* __restrict__ grad2d, gsb_splats2d_grads gr) {
  const size_t G = sp.n_gaussians;
  const size_t total = size_t(sp.n_views) * G;
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < total; i += size_t(gridDim.x) * blockDim.x) {
    const size_t b = i / G;
    const float* g = grad2d + (b * G + size_t(rank_of[i])) * GSB_GRAD2D_FLOATS;
    const float dA = g[2], dB = g[3], dC = g[4];
    if (sp.format == GSB_SPLATS2D_PACKED) {
      if (gr.packed) {
        const float* p = sp.packed + i * kPackedFloats;
        const float ax = p[2], ay = p[3], s0 = p[4], s1 = p[5];
        const float u0 = 1.0f / (s0 * s0), u1 = 1.0f / (s1 * s1), du = u0 - u1;
        const float dB2 = 2.0f * dB;  // B = 2 ax ay (u0 - u1)
        const float gu0 = dA * ax * ax + dB2 * ax * ay + dC * ay * ay;
        const float gu1 = dA * ay * ay - dB2 * ax * ay + dC * ax * ax;
        float* o = gr.packed + i * kPackedFloats;
        o[0] = g[0];
        o[1] = g[1];
        o[2] = 2.0f * ax * (dA * u0 + dC * u1) + dB2 * ay * du;
        o[3] = 2.0f * ay * (dA * u1 + dC * u0) + dB2 * ax * du;
        o[4] = gu0 * (-2.0f * u0 / s0);  // d u0 / d s0 = -2 / s0^3
        o[5] = gu1 * (-2.0f * u1 / s1);
        o[6] = g[5];
      }
    } else {
      if (gr.means) {
        gr.means[i * 2 + 0] = g[0];
        gr.means[i * 2 + 1] = g[1];
      }
      if (gr.conics) {
        gr.conics[i * 3 + 0] = dA;
        gr.conics[i * 3 + 1] = 2.0f * dB;  // B = 2 b
        gr.conics[i * 3 + 2] = dC;
      }
      if (gr.opacities) gr.opacities[i] = g[5];
    }
    if (gr.colors) {
      gr.colors[i * 3 + 0] = g[6];
      gr.colors[i * 3 + 1] = g[7];
      gr.colors[i * 3 + 2] = g[8];
    }
  }
}

int grid_for(size_t n) { return int(std::min<size_t>((n + 255) / 256, size_t(148) * 64)); }

}  // namespace

gsb_status launch_order_keys_2d(const gsb_splats2d& sp, uint32_t* keys, uint32_t* vals, uint32_t* hist,
                                cudaStream_t st) {
  const dim3 grid(unsigned((size_t(sp.n_gaussians) + kOrderThreads * kOrderItems - 1) / (kOrderThreads * kOrderItems)),
                  unsigned(sp.n_views));
  note_launch();
  order_keys_2d_kernel<<<grid, kOrderThreads, 0, st>>>(sp.depths, sp.n_gaussians, keys, vals, hist);
  return launch_status();
}

gsb_status launch_preprocess_2d(const gsb_splats2d& sp, int H, int W, const RenderConsts& rc, const int32_t* rank_of,
                                float* records, int4* rects, uint32_t* counts, cudaStream_t st) {
  note_launch();
  preprocess_2d_kernel<<<grid_for(size_t(sp.n_views) * sp.n_gaussians), 256, 0, st>>>(sp, H, W, rc, rank_of, records,
                                                                                       rects, counts);
  return launch_status();
}

gsb_status launch_preprocess_2d_bwd(const gsb_splats2d& sp, const int32_t* rank_of, const float* grad2d,
                                    const gsb_splats2d_grads& gr, cudaStream_t st) {
  note_launch();
  preprocess_2d_bwd_kernel<<<grid_for(size_t(sp.n_views) * sp.n_gaussians), 256, 0, st>>>(sp, rank_of, grad2d, gr);
  return launch_status();
}

}  // namespace gsb
