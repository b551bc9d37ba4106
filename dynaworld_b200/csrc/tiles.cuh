// Tile bounds of one projected Gaussian.  Used by both the pair count (preprocess) and the pair
// emission (bin), so the two always agree on the tile set.
//
// exact mode: every tile whose pixel-centre rectangle contains a point with
//   opacity * exp(-q/2) >= alpha_cutoff,   q = A dx^2 + B dx dy + C dy^2,
// i.e. min over the rectangle of q <= tau = 2 ln(opacity / alpha_cutoff), with a small relative
// and absolute slack.  Double precision, each operation rounded separately (explicit __d*_rn), so
// the float64 numpy restatement reproduces the lists bit for bit.
//
// tiled_compat mode: compute_gaussian_bounds + build_tile_assignments of the reference
// (src/train/renderers/tiled.py:7-45), float32 with torch's operation order.
#pragma once

#include "gsb_common.cuh"

namespace gsb {

constexpr double kExactRelMargin = 1e-5;
constexpr double kExactAbsMargin = 1e-3;

struct TileRect {
  int tx0, ty0, tx1, ty1;  // inclusive; empty when tx0 > tx1
  __device__ int count() const { return (tx0 > tx1 || ty0 > ty1) ? 0 : (tx1 - tx0 + 1) * (ty1 - ty0 + 1); }
};

struct ExactShape {
  double mx, my, a, b, c;  // record values widened to double
  double tau;              // 2 ln(o / cutoff)
  double thresh;           // tau * (1 + rel) + abs
};

__device__ inline double dmul(double x, double y) { return __dmul_rn(x, y); }
__device__ inline double dadd(double x, double y) { return __dadd_rn(x, y); }
__device__ inline double dsub(double x, double y) { return __dsub_rn(x, y); }
__device__ inline double ddiv(double x, double y) { return __ddiv_rn(x, y); }

// Returns false when the Gaussian touches no pixel.
__device__ inline bool exact_rect(float mxf, float myf, float af, float bf, float cf, float of, float cutoff, int H,
                                  int W, float pc, int tile, TileRect* rect, ExactShape* sh) {
  rect->tx0 = 1;
  rect->tx1 = 0;
  rect->ty0 = 1;
  rect->ty1 = 0;
  const double o = of, cut = cutoff;
  if (!(o > cut)) return false;
  const double a = af, b = bf, c = cf, mx = mxf, my = myf;
  const double tau = dmul(2.0, log(ddiv(o, cut)));
  const double det = dsub(dmul(a, c), dmul(dmul(0.25, b), b));
  if (!(det > 0.0) || !(a > 0.0) || !(c > 0.0)) return false;
  const double ex = dadd(dmul(__dsqrt_rn(dmul(tau, ddiv(c, det))), 1.0 + kExactRelMargin), kExactAbsMargin);
  const double ey = dadd(dmul(__dsqrt_rn(dmul(tau, ddiv(a, det))), 1.0 + kExactRelMargin), kExactAbsMargin);
  const double dpc = pc;
  const double px0 = fmax(ceil(dsub(dsub(mx, ex), dpc)), 0.0);
  const double px1 = fmin(floor(dsub(dadd(mx, ex), dpc)), double(W - 1));
  const double py0 = fmax(ceil(dsub(dsub(my, ey), dpc)), 0.0);
  const double py1 = fmin(floor(dsub(dadd(my, ey), dpc)), double(H - 1));
  if (!(px0 <= px1) || !(py0 <= py1) || !isfinite(mx) || !isfinite(my)) return false;
  rect->tx0 = int(px0) / tile;
  rect->tx1 = int(px1) / tile;
  rect->ty0 = int(py0) / tile;
  rect->ty1 = int(py1) / tile;
  sh->mx = mx;
  sh->my = my;
  sh->a = a;
  sh->b = b;
  sh->c = c;
  sh->tau = tau;
  sh->thresh = dadd(dmul(tau, 1.0 + kExactRelMargin), kExactAbsMargin);
  return true;
}

__device__ inline double quad_at(const ExactShape& s, double dx, double dy) {
  return dadd(dmul(dmul(s.a, dx), dx), dadd(dmul(dmul(s.b, dx), dy), dmul(dmul(s.c, dy), dy)));
}

// Minimum of q over the pixel-centre box [X0,X1] x [Y0,Y1] compared with the threshold.
__device__ inline bool exact_tile_hit(const ExactShape& s, int tx, int ty, int tile, int H, int W, float pc) {
  const double dpc = pc;
  const double X0 = dadd(double(max(tx * tile, 0)), dpc);
  const double X1 = dadd(double(min(tx * tile + tile - 1, W - 1)), dpc);
  const double Y0 = dadd(double(max(ty * tile, 0)), dpc);
  const double Y1 = dadd(double(min(ty * tile + tile - 1, H - 1)), dpc);
  if (X0 <= s.mx && s.mx <= X1 && Y0 <= s.my && s.my <= Y1) return true;  // min is 0
  double q = 1.0 / 0.0;
  // edges x = X0, X1: minimise over dy
  for (int e = 0; e < 2; ++e) {
    const double dx = dsub(e ? X1 : X0, s.mx);
    const double t = ddiv(-dmul(s.b, dx), dmul(2.0, s.c));
    const double dy = fmin(fmax(t, dsub(Y0, s.my)), dsub(Y1, s.my));
    q = fmin(q, quad_at(s, dx, dy));
  }
  // edges y = Y0, Y1: minimise over dx
  for (int e = 0; e < 2; ++e) {
    const double dy = dsub(e ? Y1 : Y0, s.my);
    const double t = ddiv(-dmul(s.b, dy), dmul(2.0, s.a));
    const double dx = fmin(fmax(t, dsub(X0, s.mx)), dsub(X1, s.mx));
    q = fmin(q, quad_at(s, dx, dy));
  }
  return q <= s.thresh;
}

// tiled.py:7-28 then :31-41, float32.  logf is formed in double and rounded once.
__device__ inline TileRect compat_rect(float mx, float my, float c00, float c11, float o, float bound_scale,
                                       float thr, int H, int W, int tile) {
  const float sx = __fsqrt_rn(fmaxf(c00, 1e-6f));
  const float sy = __fsqrt_rn(fmaxf(c11, 1e-6f));
  float rf;
  if (thr > 0.0f) {
    const float ratio = __fdiv_rn(fmaxf(o, thr), thr);
    const float lg = float(log(double(ratio)));
    rf = fminf(bound_scale, __fsqrt_rn(fmaxf(__fmul_rn(2.0f, lg), 0.0f)));
  } else {
    rf = bound_scale;
  }
  const float rx = __fmul_rn(rf, sx), ry = __fmul_rn(rf, sy);
  const float fminx = fminf(fmaxf(floorf(__fsub_rn(mx, rx)), 0.0f), float(W - 1));
  const float fmaxx = fminf(fmaxf(ceilf(__fadd_rn(mx, rx)), 0.0f), float(W - 1));
  const float fminy = fminf(fmaxf(floorf(__fsub_rn(my, ry)), 0.0f), float(H - 1));
  const float fmaxy = fminf(fmaxf(ceilf(__fadd_rn(my, ry)), 0.0f), float(H - 1));
  TileRect r;
  const bool valid = (fmaxx >= fminx) && (fmaxy >= fminy) && (rf > 0.0f);
  if (!valid) {
    r.tx0 = 1;
    r.tx1 = 0;
    r.ty0 = 1;
    r.ty1 = 0;
    return r;
  }
  r.tx0 = int(fminx) / tile;
  r.tx1 = int(fmaxx) / tile;
  r.ty0 = int(fminy) / tile;
  r.ty1 = int(fmaxy) / tile;
  return r;
}

}  // namespace gsb
