// Tile bounds of one projected Gaussian.  Used by both the pair count (preprocess) and the pair
// emission (bin), so the two always agree on the tile set.
//
// exact mode: the tiles holding a pixel centre with q = A dx^2 + B dx dy + C dy^2 <= L, where
// L = tau (1 + rel) + abs and tau = 2 ln(opacity / alpha_cutoff) (alpha >= cutoff <=> q <= tau).
// Per tile row, the ellipse restricted to the row's band of pixel-centre rows projects onto an
// x-interval [xl, xr] (a convex set's projection); the row's tiles are those holding a pixel
// column centre inside it.  O(rows) per Gaussian.  Double precision, every operation rounded
// separately (explicit __d*_rn), so the float64 numpy restatement gives the same lists bit for bit.
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
  double det;              // a c - b^2 / 4
  double L;                // ellipse level: tau (1 + rel) + abs
  double ex, ey;           // half extents sqrt(L c / det), sqrt(L a / det)
  int px0, px1, py0, py1;  // pixel rectangle (inclusive), clipped to the image
  double ul;               // row offset b ex / (2c) of the leftmost point (exact_row's one division
                           // that does not depend on the row, formed once)
  double inv_two_a;        // 1 / (2a): the rows' boundary offsets take a product, not a quotient
};

__device__ inline double dmul(double x, double y) { return __dmul_rn(x, y); }
__device__ inline double dadd(double x, double y) { return __dadd_rn(x, y); }
__device__ inline double dsub(double x, double y) { return __dsub_rn(x, y); }
__device__ inline double ddiv(double x, double y) { return __ddiv_rn(x, y); }

// Returns false when the Gaussian reaches no pixel centre.
__device__ inline bool exact_shape(float mxf, float myf, float af, float bf, float cf, float of, float cutoff, int H,
                                   int W, float pc, ExactShape* s) {
  const double o = of, cut = cutoff;
  if (!(o > cut)) return false;
  const double a = af, b = bf, c = cf, mx = mxf, my = myf;
  const double tau = dmul(2.0, log(ddiv(o, cut)));
  const double det = dsub(dmul(a, c), dmul(dmul(0.25, b), b));
  if (!(det > 0.0) || !(a > 0.0) || !(c > 0.0)) return false;
  const double L = dadd(dmul(tau, 1.0 + kExactRelMargin), kExactAbsMargin);
  const double ex = __dsqrt_rn(dmul(L, ddiv(c, det)));
  const double ey = __dsqrt_rn(dmul(L, ddiv(a, det)));
  const double dpc = pc;
  const double px0 = fmax(ceil(dsub(dsub(mx, ex), dpc)), 0.0);
  const double px1 = fmin(floor(dsub(dadd(mx, ex), dpc)), double(W - 1));
  const double py0 = fmax(ceil(dsub(dsub(my, ey), dpc)), 0.0);
  const double py1 = fmin(floor(dsub(dadd(my, ey), dpc)), double(H - 1));
  if (!(px0 <= px1) || !(py0 <= py1) || !isfinite(mx) || !isfinite(my)) return false;
  s->mx = mx, s->my = my, s->a = a, s->b = b, s->c = c, s->det = det, s->L = L, s->ex = ex, s->ey = ey;
  s->px0 = int(px0), s->px1 = int(px1), s->py0 = int(py0), s->py1 = int(py1);
  s->ul = ddiv(dmul(b, ex), dmul(2.0, c));
  s->inv_two_a = ddiv(1.0, dmul(2.0, a));
  return true;
}

// x offset of the ellipse boundary at row offset u: (-(b u) -/+ sqrt(4 a L - 4 det u^2)) (1 / (2 a)).
__device__ inline double ellipse_x(const ExactShape& s, double u, bool right) {
  const double disc = fmax(dsub(dmul(dmul(4.0, s.a), s.L), dmul(dmul(4.0, s.det), dmul(u, u))), 0.0);
  const double r = __dsqrt_rn(disc);
  const double nb = -dmul(s.b, u);
  return dmul(right ? dadd(nb, r) : dsub(nb, r), s.inv_two_a);
}

// Tile-column range [tx0, tx1] of tile row ty (false if the row has no tile).
__device__ inline bool exact_row(const ExactShape& s, int ty, int tile, float pc, int* tx0, int* tx1) {
  const double dpc = pc;
  const double Y0 = dadd(double(max(ty * tile, s.py0)), dpc);
  const double Y1 = dadd(double(min(ty * tile + tile - 1, s.py1)), dpc);
  const double u0 = fmax(dsub(Y0, s.my), -s.ey);
  const double u1 = fmin(dsub(Y1, s.my), s.ey);
  if (!(u0 <= u1)) return false;
  // leftmost point of the ellipse at u = b ex / (2c), rightmost at -b ex / (2c)
  const double ul = s.ul;
  const double ur = -ul;
  const double xl = (u0 <= ul && ul <= u1) ? -s.ex : fmin(ellipse_x(s, u0, false), ellipse_x(s, u1, false));
  const double xr = (u0 <= ur && ur <= u1) ? s.ex : fmax(ellipse_x(s, u0, true), ellipse_x(s, u1, true));
  const double qx0 = fmax(ceil(dsub(dadd(s.mx, xl), dpc)), double(s.px0));
  const double qx1 = fmin(floor(dsub(dadd(s.mx, xr), dpc)), double(s.px1));
  if (!(qx0 <= qx1)) return false;
  *tx0 = int(qx0) / tile;
  *tx1 = int(qx1) / tile;
  return true;
}

// exact_row with the left and right boundaries at u0 and u1 taken from one square root each (the
// same values; more registers live at once, so the register-capped preprocess count keeps
// exact_row and the key emission uses this one).
__device__ inline bool exact_row_pairs(const ExactShape& s, int ty, int tile, float pc, int* tx0, int* tx1) {
  const double dpc = pc;
  const double Y0 = dadd(double(max(ty * tile, s.py0)), dpc);
  const double Y1 = dadd(double(min(ty * tile + tile - 1, s.py1)), dpc);
  const double u0 = fmax(dsub(Y0, s.my), -s.ey);
  const double u1 = fmin(dsub(Y1, s.my), s.ey);
  if (!(u0 <= u1)) return false;
  const double ul = s.ul, ur = -s.ul;
  const bool at_l = u0 <= ul && ul <= u1, at_r = u0 <= ur && ur <= u1;
  double xl = -s.ex, xr = s.ex;
  if (!at_l || !at_r) {
    const double four_aL = dmul(dmul(4.0, s.a), s.L), four_det = dmul(4.0, s.det);
    double l[2], r[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const double u = e ? u1 : u0;
      const double root = __dsqrt_rn(fmax(dsub(four_aL, dmul(four_det, dmul(u, u))), 0.0));
      const double nb = -dmul(s.b, u);
      l[e] = dmul(dsub(nb, root), s.inv_two_a);
      r[e] = dmul(dadd(nb, root), s.inv_two_a);
    }
    if (!at_l) xl = fmin(l[0], l[1]);
    if (!at_r) xr = fmax(r[0], r[1]);
  }
  const double qx0 = fmax(ceil(dsub(dadd(s.mx, xl), dpc)), double(s.px0));
  const double qx1 = fmin(floor(dsub(dadd(s.mx, xr), dpc)), double(s.px1));
  if (!(qx0 <= qx1)) return false;
  *tx0 = int(qx0) / tile;
  *tx1 = int(qx1) / tile;
  return true;
}

__device__ inline TileRect exact_rect_of(const ExactShape& s, int tile) {
  TileRect r;
  r.tx0 = s.px0 / tile, r.tx1 = s.px1 / tile, r.ty0 = s.py0 / tile, r.ty1 = s.py1 / tile;
  return r;
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
