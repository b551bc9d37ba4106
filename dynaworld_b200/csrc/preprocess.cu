// Preprocess: depth keys, projection (+ activation, SH, time offset), tile bounds and counts,
// and the chain rule back to the scene parameters.
//
// Forward restates the reference's project_gaussians_2d_batch (src/train/renderers/common.py:
// 149-231): quaternion -> rotation (:169-179), Sigma = (R S)(R S)^T (:181-187), world -> camera
// (:39-51), near-plane mask keeping the depth slot with opacity 0 (:197-203), EWA Jacobian
// (:210-214), +0.3 low-pass (:216-218), det clamp 1e-6 and inverse (:220-225), means2D (:227-229).
// Views with a radial-tangential or fisheye lens take the pixel position and 2 x 3 Jacobian of
// project_gaussians_2d_camera instead (src/train/renderers/projection.py:227-276; lens.cuh).
// One thread per (view, Gaussian); outputs go to the Gaussian's depth-rank slot so that the
// binning and raster stages read them in depth order.
#include "gsb_common.cuh"
#include "gsb_internal.h"
#include "lens.cuh"
#include "tiles.cuh"

namespace gsb {

// ---- real spherical harmonics (degree <= 3), standard 3DGS sign convention -------------------
// Constants: sqrt((2l+1)/(4 pi) (l-m)!/(l+m)!) with the sqrt(2) of the real basis folded in.
constexpr float kC0 = 0.28209479177387814f;   // 1 / (2 sqrt(pi))
constexpr float kC1 = 0.4886025119029199f;    // sqrt(3 / (4 pi))
constexpr float kC2a = 1.0925484305920792f;   // sqrt(15 / pi) / 2
constexpr float kC2b = 0.31539156525252005f;  // sqrt(5 / pi) / 4
constexpr float kC2c = 0.5462742152960396f;   // sqrt(15 / pi) / 4
constexpr float kC3a = 0.5900435899266435f;   // sqrt(35 / (2 pi)) / 4
constexpr float kC3b = 2.890611442640554f;    // sqrt(105 / pi) / 2
constexpr float kC3c = 0.4570457994644658f;   // sqrt(21 / (2 pi)) / 4
constexpr float kC3d = 0.3731763325901154f;   // sqrt(7 / pi) / 4
constexpr float kC3e = 1.445305721320277f;    // sqrt(105 / pi) / 4

template <int K>
__device__ inline void sh_basis(float x, float y, float z, float* Y) {
  Y[0] = kC0;
  if (K > 1) {
    Y[1] = -kC1 * y;
    Y[2] = kC1 * z;
    Y[3] = -kC1 * x;
  }
  if (K > 4) {
    const float xx = x * x, yy = y * y, zz = z * z;
    Y[4] = kC2a * x * y;
    Y[5] = -kC2a * y * z;
    Y[6] = kC2b * (2.0f * zz - xx - yy);
    Y[7] = -kC2a * x * z;
    Y[8] = kC2c * (xx - yy);
    if (K > 9) {
      Y[9] = -kC3a * y * (3.0f * xx - yy);
      Y[10] = kC3b * x * y * z;
      Y[11] = -kC3c * y * (4.0f * zz - xx - yy);
      Y[12] = kC3d * z * (2.0f * zz - 3.0f * xx - 3.0f * yy);
      Y[13] = -kC3c * x * (4.0f * zz - xx - yy);
      Y[14] = kC3e * z * (xx - yy);
      Y[15] = -kC3a * x * (xx - 3.0f * yy);
    }
  }
}

// d Y_k / d(x, y, z) for k < K.
template <int K>
__device__ inline void sh_basis_grad(float x, float y, float z, float (*dY)[3]) {
  dY[0][0] = dY[0][1] = dY[0][2] = 0.0f;
  if (K > 1) {
    dY[1][0] = 0.0f, dY[1][1] = -kC1, dY[1][2] = 0.0f;
    dY[2][0] = 0.0f, dY[2][1] = 0.0f, dY[2][2] = kC1;
    dY[3][0] = -kC1, dY[3][1] = 0.0f, dY[3][2] = 0.0f;
  }
  if (K > 4) {
    const float xx = x * x, yy = y * y, zz = z * z;
    dY[4][0] = kC2a * y, dY[4][1] = kC2a * x, dY[4][2] = 0.0f;
    dY[5][0] = 0.0f, dY[5][1] = -kC2a * z, dY[5][2] = -kC2a * y;
    dY[6][0] = -2.0f * kC2b * x, dY[6][1] = -2.0f * kC2b * y, dY[6][2] = 4.0f * kC2b * z;
    dY[7][0] = -kC2a * z, dY[7][1] = 0.0f, dY[7][2] = -kC2a * x;
    dY[8][0] = 2.0f * kC2c * x, dY[8][1] = -2.0f * kC2c * y, dY[8][2] = 0.0f;
    if (K > 9) {
      dY[9][0] = -kC3a * 6.0f * x * y, dY[9][1] = -kC3a * (3.0f * xx - 3.0f * yy), dY[9][2] = 0.0f;
      dY[10][0] = kC3b * y * z, dY[10][1] = kC3b * x * z, dY[10][2] = kC3b * x * y;
      dY[11][0] = kC3c * 2.0f * x * y, dY[11][1] = -kC3c * (4.0f * zz - xx - 3.0f * yy), dY[11][2] = -kC3c * 8.0f * y * z;
      dY[12][0] = -kC3d * 6.0f * x * z, dY[12][1] = -kC3d * 6.0f * y * z,
      dY[12][2] = kC3d * (6.0f * zz - 3.0f * xx - 3.0f * yy);
      dY[13][0] = -kC3c * (4.0f * zz - 3.0f * xx - yy), dY[13][1] = kC3c * 2.0f * x * y, dY[13][2] = -kC3c * 8.0f * x * z;
      dY[14][0] = kC3e * 2.0f * x * z, dY[14][1] = -kC3e * 2.0f * y * z, dY[14][2] = kC3e * (xx - yy);
      dY[15][0] = -kC3a * (3.0f * xx - 3.0f * yy), dY[15][1] = kC3a * 6.0f * x * y, dY[15][2] = 0.0f;
    }
  }
}

// ---- parameter loading -----------------------------------------------------------------------

struct GaussParams {
  float m[3];    // means at the view's time
  float s[3];    // linear scales
  float q[4];    // quaternion used by the rotation formula
  float qn_inv;  // raw mode: 1/|q_raw| (for the normalisation backward)
  float o;       // opacity
};

// ---- dynamic bank: gs_models/dynamic_video_token_gs_implicit_camera.py:1206-1224 ----------------

// Row of Gaussian pg in the bank arrays; false for a static Gaussian or a scene without a bank.
__device__ inline bool bank_row(const gsb_scene& sc, size_t pg, size_t& row) {
  if (!(sc.flags & GSB_SCENE_BANK)) return false;
  const size_t G = size_t(sc.n_gaussians), first = size_t(sc.bank_first);
  const size_t s = pg / G, g = pg - s * G;
  if (g < first) return false;
  row = s * (G - first) + (g - first);
  return true;
}

// The temporal basis of view b (NULL without a bank).
__device__ inline const float* view_basis(const gsb_scene& sc, const gsb_views& vw, int b) {
  return (sc.flags & GSB_SCENE_BANK) ? vw.basis + size_t(b) * size_t(sc.bank_basis) : nullptr;
}

// out[c] = sum_m phi_m A[row, m, c] (the einsum "bm,bgmc->bgc" of :1213-1215).
template <int C>
__device__ inline void bank_combine(const float* __restrict__ A, size_t row, int M, const float* phi, float out[C]) {
  const float* a = A + row * size_t(M) * C;
#pragma unroll
  for (int c = 0; c < C; ++c) out[c] = 0.0f;
  for (int m = 0; m < M; ++m)
#pragma unroll
    for (int c = 0; c < C; ++c) out[c] = fmaf(phi[m], a[m * C + c], out[c]);
}

// Hamilton product (r, i, j, k) of :841-852.
__device__ inline void quat_mul(const float l[4], const float r[4], float u[4]) {
  u[0] = l[0] * r[0] - l[1] * r[1] - l[2] * r[2] - l[3] * r[3];
  u[1] = l[0] * r[1] + l[1] * r[0] + l[2] * r[3] - l[3] * r[2];
  u[2] = l[0] * r[2] - l[1] * r[3] + l[2] * r[0] + l[3] * r[1];
  u[3] = l[0] * r[3] + l[1] * r[2] - l[2] * r[1] + l[3] * r[0];
}

// y = x / max(|x|, 1e-12) (F.normalize); returns |x|.
__device__ inline float normalize4(const float x[4], float y[4]) {
  const float n = sqrtf(x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3]);
  const float d = fmaxf(n, 1e-12f);
#pragma unroll
  for (int k = 0; k < 4; ++k) y[k] = x[k] / d;
  return n;
}

// quat_t = normalize(q0 (x) normalize(cos(a/2), r sin(a/2) / a)), a = |r| (:828-838), with the
// intermediates the backward needs.
struct BankRotation {
  float r[3];
  float angle, half, s;  // |r|, |r| / 2, sin(half) / angle (series 0.5 - a^2 / 48 below 1e-6)
  float v[4], vn;        // (cos(half), r s) and its norm
  float qa[4];           // v normalised
  float u[4], un;        // q0 (x) qa and its norm
  float q[4];            // u normalised
};

__device__ inline void bank_rotation(const float q0[4], const float r[3], BankRotation& R) {
#pragma unroll
  for (int k = 0; k < 3; ++k) R.r[k] = r[k];
  R.angle = sqrtf(r[0] * r[0] + r[1] * r[1] + r[2] * r[2]);
  R.half = 0.5f * R.angle;
  R.s = R.angle < 1e-6f ? 0.5f - R.angle * R.angle / 48.0f : sinf(R.half) / fmaxf(R.angle, 1e-12f);
  R.v[0] = cosf(R.half);
#pragma unroll
  for (int k = 0; k < 3; ++k) R.v[k + 1] = r[k] * R.s;
  R.vn = normalize4(R.v, R.qa);
  quat_mul(q0, R.qa, R.u);
  R.un = normalize4(R.u, R.q);
}

// opacity_t = sigmoid(logit(clamp(o0, 1e-6, 1 - 1e-6)) + da) (:1216, 1222)
__device__ inline float bank_clamped(float o0) { return fminf(fmaxf(o0, 1e-6f), 1.0f - 1e-6f); }
__device__ inline float bank_opacity(float o0, float da) {
  const float c = bank_clamped(o0);
  return 1.0f / (1.0f + expf(-(logf(c / (1.0f - c)) + da)));
}

// Decoder-head activation of the means (GaussianParameterHeads.forward, blocks.py:174-181), each
// product and sum rounded on its own as torch forms them: (tanh(x) * e, tanh(y) * e,
// sigmoid(z) * z_extent + z_min).
__device__ inline float head_sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ inline void head_means(const gsb_scene& sc, const float raw[3], float m[3]) {
  m[0] = __fmul_rn(tanhf(raw[0]), sc.head_xy_extent);
  m[1] = __fmul_rn(tanhf(raw[1]), sc.head_xy_extent);
  m[2] = __fadd_rn(__fmul_rn(head_sigmoid(raw[2]), sc.head_z_extent), sc.head_z_min);
}

// Mean at view time t (velocity) or with the bank offset of basis phi (NULL: none).
__device__ inline void mean_at(const gsb_scene& sc, size_t pg, float t, const float* phi, float m[3]) {
#pragma unroll
  for (int k = 0; k < 3; ++k) m[k] = sc.means[pg * 3 + k];
  if (sc.flags & GSB_SCENE_HEAD) {
    const float raw[3] = {m[0], m[1], m[2]};
    head_means(sc, raw, m);
  }
#pragma unroll
  for (int k = 0; k < 3; ++k)
    if (sc.flags & GSB_SCENE_VELOCITY) m[k] = __fadd_rn(m[k], __fmul_rn(t, sc.velocity[pg * 3 + k]));
  size_t row;
  if (phi && bank_row(sc, pg, row)) {
    float dm[3];
    bank_combine<3>(sc.bank_mu, row, sc.bank_basis, phi, dm);
#pragma unroll
    for (int k = 0; k < 3; ++k) m[k] = __fadd_rn(m[k], dm[k]);
  }
}

// Parameters of Gaussian pg at one view (time t, bank basis phi or NULL); rot (may be NULL)
// receives the bank rotation's intermediates of a bank Gaussian.
__device__ inline GaussParams load_params(const gsb_scene& sc, size_t pg, float t, const float* phi,
                                          BankRotation* rot = nullptr) {
  GaussParams p;
  const bool head = sc.flags & GSB_SCENE_HEAD;
  const bool raw = (sc.flags & GSB_SCENE_RAW) || head;
  mean_at(sc, pg, t, phi, p.m);
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const float s = sc.scales[pg * 3 + k];
    p.s[k] = raw ? (head ? __fmul_rn(expf(s), sc.head_scale_init) : expf(s)) : s;
  }
  const float4 q4 = reinterpret_cast<const float4*>(sc.quats)[pg];
  p.q[0] = q4.x, p.q[1] = q4.y, p.q[2] = q4.z, p.q[3] = q4.w;
  p.qn_inv = 1.0f;
  if (raw) {
    const float n = sqrtf(q4.x * q4.x + q4.y * q4.y + q4.z * q4.z + q4.w * q4.w);
    p.qn_inv = 1.0f / (head ? fmaxf(n, 1e-12f) : n);  // F.normalize's eps (blocks.py:183)
#pragma unroll
    for (int k = 0; k < 4; ++k) p.q[k] *= p.qn_inv;
  }
  const float o = sc.opacities[pg];
  p.o = raw ? 1.0f / (1.0f + expf(-o)) : o;
  size_t row;
  if (phi && bank_row(sc, pg, row)) {
    float r[3], da;
    bank_combine<3>(sc.bank_rot, row, sc.bank_basis, phi, r);
    BankRotation R;
    bank_rotation(p.q, r, R);
#pragma unroll
    for (int k = 0; k < 4; ++k) p.q[k] = R.q[k];
    if (rot) *rot = R;
    bank_combine<1>(sc.bank_alpha, row, sc.bank_basis, phi, &da);
    p.o = bank_opacity(o, da);
  }
  return p;
}

// Rotation of common.py:169-179 (q = r, i, j, k; not renormalised).
__device__ inline void quat_rot(const float q[4], float R[9]) {
  const float r = q[0], i = q[1], j = q[2], k = q[3];
  R[0] = 1.0f - 2.0f * (j * j + k * k);
  R[1] = 2.0f * (i * j - r * k);
  R[2] = 2.0f * (i * k + r * j);
  R[3] = 2.0f * (i * j + r * k);
  R[4] = 1.0f - 2.0f * (i * i + k * k);
  R[5] = 2.0f * (j * k - r * i);
  R[6] = 2.0f * (i * k - r * j);
  R[7] = 2.0f * (j * k + r * i);
  R[8] = 1.0f - 2.0f * (i * i + j * j);
}

// Everything the forward computes for one (view, Gaussian); the backward recomputes it.
struct Proj {
  bool front;
  float d[3];          // mean_t - camera centre (world)
  float x, y, z;       // camera coordinates
  float zs, xp, yp;    // z_safe, x_project, y_project
  float Rq[9];         // Gaussian rotation
  float M[9];          // Rq diag(s)
  float cc[9];         // camera-space covariance
  float J00, J01, J02, J10, J11, J12;  // d pixel / d camera point (J01 = J10 = 0 for pinhole)
  float c00, c01, c11; // 2-D covariance incl. the 0.3 low-pass
  float det_raw, det;
  float A, B, C;
  float mx, my;
  float o_eff;
};

__device__ inline void project(const GaussParams& p, const Camera& cam, float near_plane, Proj& P) {
#pragma unroll
  for (int k = 0; k < 3; ++k) P.d[k] = __fsub_rn(p.m[k], cam.t[k]);
  P.x = cam_coord(P.d, cam.R, 0);
  P.y = cam_coord(P.d, cam.R, 1);
  P.z = cam_coord(P.d, cam.R, 2);
  quat_rot(p.q, P.Rq);
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j) P.M[i * 3 + j] = P.Rq[i * 3 + j] * p.s[j];
  float S[9];
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int k = 0; k < 3; ++k)
      S[i * 3 + k] = P.M[i * 3 + 0] * P.M[k * 3 + 0] + P.M[i * 3 + 1] * P.M[k * 3 + 1] + P.M[i * 3 + 2] * P.M[k * 3 + 2];
  // cc = Rcw^T S Rcw, Rcw[j][k] = cam.R[j*3+k]
  float T1[9];
#pragma unroll
  for (int j = 0; j < 3; ++j)
#pragma unroll
    for (int b = 0; b < 3; ++b)
      T1[j * 3 + b] = S[j * 3 + 0] * cam.R[0 * 3 + b] + S[j * 3 + 1] * cam.R[1 * 3 + b] + S[j * 3 + 2] * cam.R[2 * 3 + b];
#pragma unroll
  for (int a = 0; a < 3; ++a)
#pragma unroll
    for (int b = 0; b < 3; ++b)
      P.cc[a * 3 + b] = cam.R[0 * 3 + a] * T1[0 * 3 + b] + cam.R[1 * 3 + a] * T1[1 * 3 + b] + cam.R[2 * 3 + a] * T1[2 * 3 + b];
  P.front = P.z > near_plane;
  P.zs = P.front ? fmaxf(P.z, near_plane) : 1.0f;
  P.xp = P.front ? P.x : 0.0f;
  P.yp = P.front ? P.y : 0.0f;
  P.o_eff = p.o * (P.front ? 1.0f : 0.0f);
  const float* c = P.cc;
  if (cam.lens == GSB_LENS_PINHOLE) {  // common.py:200-215
    const float fx = cam.k.fx, fy = cam.k.fy;
    const float zs2 = P.zs * P.zs;
    P.J00 = fx / P.zs;
    P.J01 = P.J10 = 0.0f;
    P.J02 = -(fx * P.xp) / zs2;
    P.J11 = fy / P.zs;
    P.J12 = -(fy * P.yp) / zs2;
    P.c00 = P.J00 * P.J00 * c[0] + 2.0f * P.J00 * P.J02 * c[2] + P.J02 * P.J02 * c[8] + 0.3f;
    P.c11 = P.J11 * P.J11 * c[4] + 2.0f * P.J11 * P.J12 * c[5] + P.J12 * P.J12 * c[8] + 0.3f;
    P.c01 = P.J00 * P.J11 * c[1] + P.J00 * P.J12 * c[2] + P.J02 * P.J11 * c[5] + P.J02 * P.J12 * c[8];
    P.mx = __fadd_rn(__fdiv_rn(__fmul_rn(fx, P.xp), P.zs), cam.k.cx);
    P.my = __fadd_rn(__fdiv_rn(__fmul_rn(fy, P.yp), P.zs), cam.k.cy);
  } else {  // projection.py:164-214, 253-263; behind the near plane the Jacobian is zero
    float coef[5];
    lens_coefficients(cam, coef);
    const LensProjection<float> lp = lens_project<float>(P.xp, P.yp, P.zs, cam, coef);
    const float m = P.front ? 1.0f : 0.0f;
    P.J00 = lp.J[0] * m, P.J01 = lp.J[1] * m, P.J02 = lp.J[2] * m;
    P.J10 = lp.J[3] * m, P.J11 = lp.J[4] * m, P.J12 = lp.J[5] * m;
    const float u[3] = {P.J00, P.J01, P.J02}, v[3] = {P.J10, P.J11, P.J12};
    float tu[3], tv[3];  // (J cc) rows
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      tu[k] = u[0] * c[0 * 3 + k] + u[1] * c[1 * 3 + k] + u[2] * c[2 * 3 + k];
      tv[k] = v[0] * c[0 * 3 + k] + v[1] * c[1 * 3 + k] + v[2] * c[2 * 3 + k];
    }
    P.c00 = tu[0] * u[0] + tu[1] * u[1] + tu[2] * u[2] + 0.3f;
    P.c11 = tv[0] * v[0] + tv[1] * v[1] + tv[2] * v[2] + 0.3f;
    P.c01 = tu[0] * v[0] + tu[1] * v[1] + tu[2] * v[2];
    P.mx = lp.mx;
    P.my = lp.my;
  }
  P.det_raw = P.c00 * P.c11 - P.c01 * P.c01;
  P.det = fmaxf(P.det_raw, 1e-6f);
  P.A = P.c11 / P.det;
  P.C = P.c00 / P.det;
  const float inv01 = -P.c01 / P.det;
  P.B = inv01 + inv01;
}

// The K x 3 SH coefficients of Gaussian pg: 16-byte loads when the rows allow them (K = 4, 16 and
// an aligned array), so the load queue holds a quarter of the requests.
template <int K>
__device__ inline void load_sh(const gsb_scene& sc, size_t pg, float sh[K * 3]) {
  const float* src = sc.colors + pg * size_t(K) * 3;
  if ((K * 3) % 4 == 0 && (reinterpret_cast<uintptr_t>(sc.colors) & 15) == 0) {
    const float4* s4 = reinterpret_cast<const float4*>(src);
#pragma unroll
    for (int i = 0; i < (K * 3) / 4; ++i) {
      const float4 v = __ldg(s4 + i);
      sh[4 * i] = v.x, sh[4 * i + 1] = v.y, sh[4 * i + 2] = v.z, sh[4 * i + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < K * 3; ++i) sh[i] = __ldg(src + i);
  }
}

template <int K>
__device__ inline void eval_color(const gsb_scene& sc, size_t pg, const float d[3], bool clamp, float rgb[3]) {
  const float inv = rsqrtf(d[0] * d[0] + d[1] * d[1] + d[2] * d[2]);
  float Y[K];
  sh_basis<K>(d[0] * inv, d[1] * inv, d[2] * inv, Y);
  float sh[K * 3];
  load_sh<K>(sc, pg, sh);
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    float v = 0.5f;
#pragma unroll
    for (int k = 0; k < K; ++k) v += Y[k] * sh[k * 3 + c];
    rgb[c] = (clamp && v < 0.0f) ? 0.0f : v;  // torch.clamp(min=0): NaN stays NaN
  }
}

__device__ inline void load_color(const gsb_scene& sc, size_t pg, const float d[3], float rgb[3]) {
  if (sc.flags & GSB_SCENE_HEAD) {  // rgb = sigmoid(raw) (blocks.py:185)
#pragma unroll
    for (int c = 0; c < 3; ++c) rgb[c] = head_sigmoid(sc.colors[pg * 3 + c]);
    return;
  }
  if (!(sc.flags & GSB_SCENE_RAW)) {
    rgb[0] = sc.colors[pg * 3 + 0], rgb[1] = sc.colors[pg * 3 + 1], rgb[2] = sc.colors[pg * 3 + 2];
    return;
  }
  const bool clamp = sc.flags & GSB_SCENE_SH_CLAMP;
  switch (sc.sh_degree) {
    case 0: eval_color<1>(sc, pg, d, clamp, rgb); break;
    case 1: eval_color<4>(sc, pg, d, clamp, rgb); break;
    case 2: eval_color<9>(sc, pg, d, clamp, rgb); break;
    default: eval_color<16>(sc, pg, d, clamp, rgb); break;
  }
}

// ---- stage 1 kernels: depth keys and inverse permutation -------------------------------------

constexpr int kKeyThreads = 256;
// Gaussians per thread.  Measured on one B200 (depth order ms, 16 x 32768 / 8 x 200k): 8: 0.0838 /
// 0.1799, 4: 0.0821 / 0.1794, 2: 0.0800 / 0.1753 -- more blocks hide the latency of the shared
// digit counts.
constexpr int kKeyItems = 2;

// Depth sort keys of view blockIdx.y (the order-preserving bits of the camera z, common.py:190-195)
// with the Gaussian index as value, plus the view's four 8-bit digit histograms for the
// segmented radix sort (warp-aggregated shared-memory counts, one global add per non-zero bin).
// BANK: the scene has a dynamic bank (compiled out of the other instances).
template <bool BANK>
__global__ void __launch_bounds__(kKeyThreads) depth_key_kernel(gsb_scene sc, gsb_views vw,
                                                                uint32_t* __restrict__ keys,
                                                                uint32_t* __restrict__ vals,
                                                                uint32_t* __restrict__ hist) {
  __shared__ uint32_t s_hist[4][256];
  for (int i = threadIdx.x; i < 4 * 256; i += kKeyThreads) s_hist[i / 256][i % 256] = 0u;
  __syncthreads();
  const int b = blockIdx.y;
  const size_t G = sc.n_gaussians;
  const size_t set0 = size_t(b / vw.views_per_set) * G;
  const float t = vw.times ? vw.times[b] : 0.0f;
  const float* phi = BANK ? view_basis(sc, vw, b) : nullptr;
  const float* c2w = vw.camera_to_world + b * 16;
  float R[9], centre[3];
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    centre[k] = c2w[k * 4 + 3];
#pragma unroll
    for (int j = 0; j < 3; ++j) R[k * 3 + j] = c2w[k * 4 + j];
  }
  const size_t g0 = size_t(blockIdx.x) * kKeyThreads * kKeyItems + threadIdx.x;
#pragma unroll 2
  for (int it = 0; it < kKeyItems; ++it) {
    const size_t g = g0 + size_t(it) * kKeyThreads;
    const bool valid = g < G;
    uint32_t key = 0u;
    if (valid) {
      float m[3], d[3];
      mean_at(sc, set0 + g, t, phi, m);
#pragma unroll
      for (int k = 0; k < 3; ++k) d[k] = __fsub_rn(m[k], centre[k]);
      key = float_sort_key(cam_coord(d, R, 2));
      keys[size_t(b) * G + g] = key;
      vals[size_t(b) * G + g] = uint32_t(g);
    }
    count_digits4(s_hist, key, valid);
  }
  __syncthreads();
  flush_digits4(s_hist, hist + size_t(b) * 4 * 256);
}

__global__ void invert_order_kernel(const uint32_t* __restrict__ sorted_vals, int32_t n_views, int32_t G,
                                    int32_t* __restrict__ sorted_ids, int32_t* __restrict__ rank_of) {
  const size_t total = size_t(n_views) * G;
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < total; i += size_t(gridDim.x) * blockDim.x) {
    const size_t b = i / G;
    const int32_t r = int32_t(i - b * G);
    const int32_t g = int32_t(sorted_vals[i]);
    sorted_ids[i] = g;
    if (g >= 0 && g < G) rank_of[b * G + g] = r;
  }
}

// ---- stage 2: projection + bounds ------------------------------------------------------------

// Four CTAs per SM (64 registers, a few bytes of spill): the kernel is latency-bound on its
// scattered record stores and the float64 tile bounds, and occupancy beats the spill.  Measured on
// one B200 (ms, 16 x 128^2 / 8 x 384^2): 2 CTAs (91 registers) 0.090 / 0.406, 3 CTAs 0.082 / 0.344,
// 4 CTAs 0.079 / 0.336.
template <bool BANK>
__global__ void __launch_bounds__(256, 4) preprocess_fwd_kernel(gsb_scene sc, gsb_views vw, RenderConsts rc,
                                                             const int32_t* __restrict__ rank_of,
                                                             float* __restrict__ records, int4* __restrict__ rects,
                                                             uint32_t* __restrict__ counts, float* __restrict__ cov_out,
                                                             int32_t* __restrict__ status) {
  const size_t G = sc.n_gaussians;
  const size_t total = size_t(vw.n_views) * G;
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < total; i += size_t(gridDim.x) * blockDim.x) {
    const int b = int(i / G);
    const size_t g = i - size_t(b) * G;
    const size_t pg = size_t(b / vw.views_per_set) * G + g;
    const float t = vw.times ? vw.times[b] : 0.0f;
    const Camera cam = load_camera(vw, b);
    const GaussParams p = load_params(sc, pg, t, BANK ? view_basis(sc, vw, b) : nullptr);
    Proj P;
    project(p, cam, rc.near_plane, P);
    float rgb[3];
    load_color(sc, pg, P.d, rgb);

    // Non-finite inputs (NaN / inf parameters, overflowing scales) show up as non-finite projected
    // values: counted here (status word 2), first offender in word 1, GSB_ERR_NONFINITE in word 0.
    // Such a Gaussian gets no tile and is never blended (the host reports it as the reference's
    // trainers report a non-finite render).
    const bool finite = isfinite(P.mx) && isfinite(P.my) && isfinite(P.A) && isfinite(P.B) && isfinite(P.C) &&
                        isfinite(P.o_eff) && isfinite(P.z) && isfinite(rgb[0]) && isfinite(rgb[1]) &&
                        isfinite(rgb[2]);
    TileRect rect;
    float tau_f;
    uint32_t count = 0;
    if (!finite) {
      if (status) {
        record_error(status, GSB_ERR_NONFINITE, int(i));
        atomicAdd(status + 2, 1);
      }
      rect = TileRect{1, 1, 0, 0};
      tau_f = -1.0f;
    } else if (rc.compat) {
      rect = compat_rect(P.mx, P.my, P.c00, P.c11, P.o_eff, rc.bound_scale, rc.tiled_threshold, vw.height, vw.width,
                         rc.tile);
      count = rect.count();
      tau_f = __int_as_float(0x7f800000);  // +inf: every listed pair is blended
    } else {
      ExactShape es;
      rect = TileRect{1, 1, 0, 0};
      if (exact_shape(P.mx, P.my, P.A, P.B, P.C, P.o_eff, rc.alpha_cutoff, vw.height, vw.width, rc.pixel_center,
                      &es)) {
        rect = exact_rect_of(es, rc.tile);
        // with the ellipse rows the pairs are counted afterwards in rank order (pairs_kernel: the
        // rows of a block's Gaussians spread over its lanes)
        if (!rc.ellipse) count = rect.count();
        tau_f = __double2float_ru(es.L);
      } else {
        tau_f = -1.0f;  // never blended
      }
    }
    const size_t slot = size_t(b) * G + size_t(rank_of[i]);
    float4* rec = reinterpret_cast<float4*>(records + slot * GSB_RECORD_FLOATS);
    rec[0] = make_float4(P.mx, P.my, P.A, P.B);
    rec[1] = make_float4(P.C, P.o_eff, P.z, tau_f);
    rec[2] = make_float4(rgb[0], rgb[1], rgb[2], 0.0f);
    rec[3] = cull_extents(P.A, P.B, P.C, tau_f);
    rects[slot] = make_int4(rect.tx0, rect.ty0, rect.tx1, rect.ty1);
    counts[slot] = count;
    if (cov_out) {
      cov_out[slot * 3 + 0] = P.c00;
      cov_out[slot * 3 + 1] = P.c01;
      cov_out[slot * 3 + 2] = P.c11;
    }
  }
}

// ---- stage 7: backward -----------------------------------------------------------------------

// d loss / d quaternion components (r, i, j, k) from d loss / d R of quat_rot.
__device__ inline void quat_rot_vjp(const float q[4], const float G[9], float dq[4]) {
  const float r = q[0], i = q[1], j = q[2], k = q[3];
  dq[0] = 2.0f * (-k * G[1] + j * G[2] + k * G[3] - i * G[5] - j * G[6] + i * G[7]);
  dq[1] = 2.0f * (j * G[1] + k * G[2] + j * G[3] - 2.0f * i * G[4] - r * G[5] + k * G[6] + r * G[7] - 2.0f * i * G[8]);
  dq[2] = 2.0f * (-2.0f * j * G[0] + i * G[1] + r * G[2] + i * G[3] + k * G[5] - r * G[6] + k * G[7] - 2.0f * j * G[8]);
  dq[3] = 2.0f * (-2.0f * k * G[0] - r * G[1] + i * G[2] + r * G[3] - 2.0f * k * G[4] + j * G[5] + i * G[6] + j * G[7]);
}

// Colour of one view: d loss / d SH coefficients (accumulated into acol, K = 0: plain rgb) and
// the part of d loss / d mean that flows through the view direction d / |d| (added to dmt).
template <int K>
__device__ inline void sh_backward(const gsb_scene& sc, size_t pg, const float d[3], const float dcol[3],
                                   bool clamp_sh, float* acol, float dmt[3]) {
  if (K == 0) {
    if (acol)
      for (int c = 0; c < 3; ++c) acol[c] += dcol[c];
    return;
  }
  constexpr int KC = K > 0 ? K : 1;
  const float n2 = d[0] * d[0] + d[1] * d[1] + d[2] * d[2];
  const float inv = rsqrtf(n2);
  const float dir[3] = {d[0] * inv, d[1] * inv, d[2] * inv};
  float Y[KC];
  sh_basis<KC>(dir[0], dir[1], dir[2], Y);
  const float* sh = sc.colors + pg * size_t(KC) * 3;
  float dc[3];
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    float v = 0.5f;
#pragma unroll
    for (int k = 0; k < KC; ++k) v += Y[k] * sh[k * 3 + c];
    dc[c] = (clamp_sh && !(v >= 0.0f)) ? 0.0f : dcol[c];
  }
  if (acol) {
#pragma unroll
    for (int k = 0; k < KC; ++k)
#pragma unroll
      for (int c = 0; c < 3; ++c) acol[k * 3 + c] += dc[c] * Y[k];
  }
  if (KC > 1) {
    float dY[KC][3];
    sh_basis_grad<KC>(dir[0], dir[1], dir[2], dY);
    float ddir[3] = {0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int k = 1; k < KC; ++k) {
      const float w = dc[0] * sh[k * 3 + 0] + dc[1] * sh[k * 3 + 1] + dc[2] * sh[k * 3 + 2];
      ddir[0] += w * dY[k][0];
      ddir[1] += w * dY[k][1];
      ddir[2] += w * dY[k][2];
    }
    const float dd = dir[0] * ddir[0] + dir[1] * ddir[1] + dir[2] * ddir[2];
#pragma unroll
    for (int k = 0; k < 3; ++k) dmt[k] += (ddir[k] - dir[k] * dd) * inv;
  }
}

// d loss / d (J rows u, v) and d loss / d camera covariance from d loss / d inverse 2-D covariance.
struct CovGrad {
  float du[3], dv[3], dcc[9];
};

__device__ inline void cov_backward(const Proj& P, float dA, float dB, float dC, CovGrad& cg) {
  // inverse covariance -> covariance (det clamped at 1e-6: no gradient through the clamp)
  const float det = P.det;
  const float ddet = (P.det_raw >= 1e-6f) ? -(dA * P.A + dB * P.B + dC * P.C) / det : 0.0f;
  const float g00 = dC / det + ddet * P.c11;
  const float g11 = dA / det + ddet * P.c00;
  const float g01 = -2.0f * dB / det - 2.0f * ddet * P.c01;  // total over the two off-diagonals
  // covariance = J cc J^T, J rows u = (J00, J01, J02), v = (J10, J11, J12)
  const float u[3] = {P.J00, P.J01, P.J02}, v[3] = {P.J10, P.J11, P.J12};
  float cu[3], cv[3];
#pragma unroll
  for (int a = 0; a < 3; ++a) {
    cu[a] = P.cc[a * 3 + 0] * u[0] + P.cc[a * 3 + 1] * u[1] + P.cc[a * 3 + 2] * u[2];
    cv[a] = P.cc[a * 3 + 0] * v[0] + P.cc[a * 3 + 1] * v[1] + P.cc[a * 3 + 2] * v[2];
  }
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    cg.du[k] = 2.0f * g00 * cu[k] + g01 * cv[k];
    cg.dv[k] = 2.0f * g11 * cv[k] + g01 * cu[k];
  }
#pragma unroll
  for (int a = 0; a < 3; ++a)
#pragma unroll
    for (int c = 0; c < 3; ++c)
      cg.dcc[a * 3 + c] = g00 * u[a] * u[c] + g11 * v[a] * v[c] + 0.5f * g01 * (u[a] * v[c] + v[a] * u[c]);
}

// Jacobian and means2D -> camera-space point, pinhole (common.py:205-229).
__device__ inline void pinhole_point_backward(const Proj& P, const Camera& cam, float dmx, float dmy,
                                              const CovGrad& cg, float dmc[3]) {
  const float fx = cam.k.fx, fy = cam.k.fy, zs = P.zs;
  const float izs = 1.0f / zs, izs2 = izs * izs, izs3 = izs2 * izs;
  dmc[0] = cg.du[2] * (-fx * izs2) + dmx * fx * izs;
  dmc[1] = cg.dv[2] * (-fy * izs2) + dmy * fy * izs;
  dmc[2] = cg.du[0] * (-fx * izs2) + cg.du[2] * (2.0f * fx * P.xp * izs3) + cg.dv[1] * (-fy * izs2) +
           cg.dv[2] * (2.0f * fy * P.yp * izs3) + dmx * (-fx * P.xp * izs2) + dmy * (-fy * P.yp * izs2);
}

// The same through a lens: forward-mode derivatives of the pixel and of every Jacobian entry
// along the camera-space x, y, z.
__device__ inline void lens_point_backward(const Proj& P, const Camera& cam, float dmx, float dmy, const CovGrad& cg,
                                           float dmc[3]) {
  Dual3 coef[5];
  lens_coefficients(cam, coef);
  const LensProjection<Dual3> lp = lens_project<Dual3>(dual(P.xp, 1.0f, 0.0f, 0.0f), dual(P.yp, 0.0f, 1.0f, 0.0f),
                                                       dual(P.zs, 0.0f, 0.0f, 1.0f), cam, coef);
  const float dJ[6] = {cg.du[0], cg.du[1], cg.du[2], cg.dv[0], cg.dv[1], cg.dv[2]};
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    float acc = dmx * lp.mx.d[k] + dmy * lp.my.d[k];
#pragma unroll
    for (int e = 0; e < 6; ++e) acc += dJ[e] * lp.J[e].d[k];
    dmc[k] = acc;
  }
}

// Backward of normalize4: d loss / d x from d loss / d y, y = x / max(n, 1e-12), n = |x|.
__device__ inline void normalize4_vjp(const float y[4], float n, const float dy[4], float dx[4]) {
  if (n >= 1e-12f) {
    const float dot = y[0] * dy[0] + y[1] * dy[1] + y[2] * dy[2] + y[3] * dy[3];
#pragma unroll
    for (int k = 0; k < 4; ++k) dx[k] = (dy[k] - y[k] * dot) / n;
  } else {
#pragma unroll
    for (int k = 0; k < 4; ++k) dx[k] = dy[k] / 1e-12f;
  }
}

// Backward of quat_mul: d loss / d l and d loss / d r from d loss / d (l (x) r).
__device__ inline void quat_mul_vjp(const float l[4], const float r[4], const float du[4], float dl[4], float dr[4]) {
  dl[0] = du[0] * r[0] + du[1] * r[1] + du[2] * r[2] + du[3] * r[3];
  dl[1] = -du[0] * r[1] + du[1] * r[0] - du[2] * r[3] + du[3] * r[2];
  dl[2] = -du[0] * r[2] + du[1] * r[3] + du[2] * r[0] - du[3] * r[1];
  dl[3] = -du[0] * r[3] - du[1] * r[2] + du[2] * r[1] + du[3] * r[0];
  dr[0] = du[0] * l[0] + du[1] * l[1] + du[2] * l[2] + du[3] * l[3];
  dr[1] = -du[0] * l[1] + du[1] * l[0] + du[2] * l[3] - du[3] * l[2];
  dr[2] = -du[0] * l[2] - du[1] * l[3] + du[2] * l[0] + du[3] * l[1];
  dr[3] = -du[0] * l[3] + du[1] * l[2] - du[2] * l[1] + du[3] * l[0];
}

// Backward of v = (cos(a/2), r s(a)), a = |r|, through the branch bank_rotation took (torch.where
// routes the gradient to the chosen branch; the norm's gradient is 0 at r = 0).
__device__ inline void axis_angle_vjp(const BankRotation& R, const float dv[4], float dr[3]) {
  const float a = R.angle;
  const float dvr = dv[1] * R.r[0] + dv[2] * R.r[1] + dv[3] * R.r[2];
  const float ds = a < 1e-6f ? -a / 24.0f : (0.5f * cosf(R.half) * a - sinf(R.half)) / (a * a);
  const float da = dv[0] * (-0.5f * sinf(R.half)) + dvr * ds;
  const float ia = a > 0.0f ? 1.0f / a : 0.0f;
#pragma unroll
  for (int k = 0; k < 3; ++k) dr[k] = dv[k + 1] * R.s + da * R.r[k] * ia;
}

// K = SH coefficients per channel (1, 4, 9, 16) or 0 for plain rgb; LENS: some view has a
// non-pinhole lens (the dual-number lens backward is compiled into these instances only); BANK:
// the scene has a dynamic bank (activated values, K = 0): the gradients of its coefficients are
// summed over the set's views in registers, GSB_BANK_MAX_BASIS x 7 per Gaussian.  LPG: lanes per
// Gaussian; lane j of a group takes views j, j + LPG, ... of the set and the group's sums are then
// combined by shuffles, so a set of few Gaussians seen by many views still fills the GPU.
template <int K, bool LENS, bool BANK, int LPG>
__global__ void __launch_bounds__(128) preprocess_bwd_kernel(gsb_scene sc, gsb_views vw, RenderConsts rc,
                                                             const int32_t* __restrict__ rank_of,
                                                             const float* __restrict__ grad2d, gsb_scene_grads gr) {
  static_assert(LPG == 1 || (!BANK && 32 % LPG == 0), "lane groups tile a warp; the bank keeps one lane");
  const size_t G = sc.n_gaussians;
  const size_t first = rc.bwd_first;
  const size_t total = rc.bwd_count ? size_t(rc.bwd_count) : size_t(sc.n_sets) * G - first;
  const bool head = sc.flags & GSB_SCENE_HEAD;
  const bool raw = (sc.flags & GSB_SCENE_RAW) || head;
  const bool vel = sc.flags & GSB_SCENE_VELOCITY;
  const bool clamp_sh = sc.flags & GSB_SCENE_SH_CLAMP;
  constexpr int KC = K > 0 ? K : 1;
  constexpr int NB = BANK ? GSB_BANK_MAX_BASIS : 1;
  const int M = sc.bank_basis;
  const size_t lanes_total = total * LPG;
  // the trip count is uniform over a block: every lane reaches the group shuffles below
  for (size_t t0 = blockIdx.x * size_t(blockDim.x); t0 < lanes_total; t0 += size_t(gridDim.x) * blockDim.x) {
    const size_t tix = t0 + threadIdx.x;
    const bool valid = tix < lanes_total;
    const size_t pg = first + (valid ? tix / LPG : 0);
    const int sub = int(tix % LPG);
    const int s = int(pg / G);
    const size_t g = pg - size_t(s) * G;
    float am[3] = {0, 0, 0}, av[3] = {0, 0, 0}, as[3] = {0, 0, 0}, aq[4] = {0, 0, 0, 0}, ao = 0.0f;
    float acol[KC * 3];
#pragma unroll
    for (int k = 0; k < KC * 3; ++k) acol[k] = 0.0f;
    size_t row = 0;
    const bool banked = BANK && bank_row(sc, pg, row);
    float amu[NB][3], arot[NB][3], aal[NB];
#pragma unroll
    for (int m = 0; m < NB; ++m) amu[m][0] = amu[m][1] = amu[m][2] = arot[m][0] = arot[m][1] = arot[m][2] = aal[m] = 0.0f;
    const int b0 = s * vw.views_per_set;
    const int b1 = valid ? min(b0 + vw.views_per_set, vw.n_views) : b0;
    for (int b = b0 + sub; b < b1; b += LPG) {
      const size_t slot = size_t(b) * G + size_t(rank_of[size_t(b) * G + g]);
      const float* g2 = grad2d + slot * GSB_GRAD2D_FLOATS;
      float dmx = g2[0], dmy = g2[1], dA = g2[2], dB = g2[3], dC = g2[4], dO = g2[5];
      const float dcol[3] = {g2[6], g2[7], g2[8]};
      const float dzo = g2[9];
      const float t = vw.times ? vw.times[b] : 0.0f;
      const Camera cam = load_camera(vw, b);
      const float* phi = BANK ? view_basis(sc, vw, b) : nullptr;
      BankRotation R;
      const GaussParams p = load_params(sc, pg, t, phi, &R);
      Proj P;
      project(p, cam, rc.near_plane, P);
      if (!P.front) continue;  // opacity * 0: no gradient reaches this Gaussian from this view
      float dmt[3] = {0.0f, 0.0f, 0.0f};
      sh_backward<K>(sc, pg, P.d, dcol, clamp_sh, acol, dmt);
      CovGrad cg;
      cov_backward(P, dA, dB, dC, cg);
      float dmc[3];
      if (!LENS || cam.lens == GSB_LENS_PINHOLE) pinhole_point_backward(P, cam, dmx, dmy, cg, dmc);
      else lens_point_backward(P, cam, dmx, dmy, cg, dmc);
      dmc[2] += dzo;
      // camera -> world: mc = Rcw^T d, cc = Rcw^T S Rcw
#pragma unroll
      for (int j = 0; j < 3; ++j)
        dmt[j] += cam.R[j * 3 + 0] * dmc[0] + cam.R[j * 3 + 1] * dmc[1] + cam.R[j * 3 + 2] * dmc[2];
      const float* dcc = cg.dcc;
      float T2[9], dS[9];
#pragma unroll
      for (int a = 0; a < 3; ++a)
#pragma unroll
        for (int k = 0; k < 3; ++k)
          T2[a * 3 + k] = dcc[a * 3 + 0] * cam.R[k * 3 + 0] + dcc[a * 3 + 1] * cam.R[k * 3 + 1] + dcc[a * 3 + 2] * cam.R[k * 3 + 2];
#pragma unroll
      for (int j = 0; j < 3; ++j)
#pragma unroll
        for (int k = 0; k < 3; ++k)
          dS[j * 3 + k] = cam.R[j * 3 + 0] * T2[0 * 3 + k] + cam.R[j * 3 + 1] * T2[1 * 3 + k] + cam.R[j * 3 + 2] * T2[2 * 3 + k];
      // S = M M^T -> dM = (dS + dS^T) M
      float dRq[9];
      float dsv[3] = {0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) {
          float dm = 0.0f;
#pragma unroll
          for (int k = 0; k < 3; ++k) dm += (dS[i * 3 + k] + dS[k * 3 + i]) * P.M[k * 3 + j];
          dRq[i * 3 + j] = dm * p.s[j];
          dsv[j] += dm * P.Rq[i * 3 + j];
        }
      float dq[4];
      quat_rot_vjp(p.q, dRq, dq);
      if (raw) {
        const float dot = p.q[0] * dq[0] + p.q[1] * dq[1] + p.q[2] * dq[2] + p.q[3] * dq[3];
#pragma unroll
        for (int k = 0; k < 4; ++k) aq[k] += (dq[k] - p.q[k] * dot) * p.qn_inv;
#pragma unroll
        for (int k = 0; k < 3; ++k) as[k] += dsv[k] * p.s[k];
        ao += dO * p.o * (1.0f - p.o);
      } else if (banked) {
        // quat_t = normalize(q0 (x) normalize(v(r))), r = sum_m phi_m bank_rot[m]
        const float4 q4 = reinterpret_cast<const float4*>(sc.quats)[pg];
        const float q0[4] = {q4.x, q4.y, q4.z, q4.w};
        float du[4], dq0[4], dqa[4], dv[4], dr[3];
        normalize4_vjp(R.q, R.un, dq, du);
        quat_mul_vjp(q0, R.qa, du, dq0, dqa);
        normalize4_vjp(R.qa, R.vn, dqa, dv);
        axis_angle_vjp(R, dv, dr);
#pragma unroll
        for (int k = 0; k < 4; ++k) aq[k] += dq0[k];
#pragma unroll
        for (int k = 0; k < 3; ++k) as[k] += dsv[k];
        // opacity_t = sigmoid(logit(clamp(o0)) + sum_m phi_m bank_alpha[m]); clamp passes the
        // gradient inside its range
        const float o0 = sc.opacities[pg];
        const float c = bank_clamped(o0);
        const float dz = dO * p.o * (1.0f - p.o);
        if (o0 >= 1e-6f && o0 <= 1.0f - 1e-6f) ao += dz / (c * (1.0f - c));
#pragma unroll
        for (int m = 0; m < NB; ++m) {
          if (m >= M) break;
          const float f = phi[m];
#pragma unroll
          for (int k = 0; k < 3; ++k) {
            amu[m][k] = fmaf(f, dmt[k], amu[m][k]);
            arot[m][k] = fmaf(f, dr[k], arot[m][k]);
          }
          aal[m] = fmaf(f, dz, aal[m]);
        }
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) aq[k] += dq[k];
#pragma unroll
        for (int k = 0; k < 3; ++k) as[k] += dsv[k];
        ao += dO;
      }
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        am[k] += dmt[k];
        av[k] += t * dmt[k];
      }
    }
    if (LPG > 1) {  // the group's partial sums -> lane 0 of the group
#pragma unroll
      for (int o = LPG / 2; o > 0; o >>= 1) {
        auto add = [&](float& x) { x += __shfl_xor_sync(0xffffffffu, x, o); };
#pragma unroll
        for (int k = 0; k < 3; ++k) add(am[k]), add(av[k]), add(as[k]);
#pragma unroll
        for (int k = 0; k < 4; ++k) add(aq[k]);
        add(ao);
#pragma unroll
        for (int k = 0; k < KC * 3; ++k) add(acol[k]);
      }
    }
    if (!valid || sub != 0) continue;
    if (head && K == 0) {  // the head's view-independent activations, applied to the view sums
      const float* rm = sc.means + pg * 3;
      const float tx = tanhf(rm[0]), ty = tanhf(rm[1]), sz = head_sigmoid(rm[2]);
      am[0] *= sc.head_xy_extent * (1.0f - tx * tx);
      am[1] *= sc.head_xy_extent * (1.0f - ty * ty);
      am[2] *= sc.head_z_extent * sz * (1.0f - sz);
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        const float v = head_sigmoid(sc.colors[pg * 3 + c]);
        acol[c] *= v * (1.0f - v);
      }
    }
    if (gr.means)
      for (int k = 0; k < 3; ++k) gr.means[pg * 3 + k] = am[k];
    if (gr.scales)
      for (int k = 0; k < 3; ++k) gr.scales[pg * 3 + k] = as[k];
    if (gr.quats)
      for (int k = 0; k < 4; ++k) gr.quats[pg * 4 + k] = aq[k];
    if (gr.opacities) gr.opacities[pg] = ao;
    if (gr.colors)
      for (int k = 0; k < KC * 3; ++k) gr.colors[pg * KC * 3 + k] = acol[k];
    if (gr.velocity && vel)
      for (int k = 0; k < 3; ++k) gr.velocity[pg * 3 + k] = av[k];
    if (banked) {
#pragma unroll
      for (int m = 0; m < NB; ++m) {
        if (m >= M) break;
        const size_t o = row * size_t(M) + size_t(m);
        if (gr.bank_mu)
          for (int k = 0; k < 3; ++k) gr.bank_mu[o * 3 + k] = amu[m][k];
        if (gr.bank_rot)
          for (int k = 0; k < 3; ++k) gr.bank_rot[o * 3 + k] = arot[m][k];
        if (gr.bank_alpha) gr.bank_alpha[o] = aal[m];
      }
    }
  }
}

// ---- camera gradients --------------------------------------------------------------------------
//
// d loss / d camera of each view, summed over its Gaussians: intrinsics (fx, fy, cx, cy),
// camera_to_world rotation (mc = R^T d and cc = R^T S R, d = mean_t - centre) and centre
// (-d loss / d d), and the lens distortion coefficients (forward-mode duals over the point and
// the five coefficients).  One thread per (view, Gaussian), blockIdx.y = view; a block reduction
// then one atomic per value per block.

constexpr int kCamValues = 4 + 9 + 3 + 5;

template <int K, bool LENS>
__global__ void __launch_bounds__(128) camera_bwd_kernel(gsb_scene sc, gsb_views vw, RenderConsts rc,
                                                         const int32_t* __restrict__ rank_of,
                                                         const float* __restrict__ grad2d, gsb_camera_grads out) {
  const int b = blockIdx.y;
  const size_t G = sc.n_gaussians;
  const size_t g = blockIdx.x * size_t(blockDim.x) + threadIdx.x;
  float acc[kCamValues];
#pragma unroll
  for (int i = 0; i < kCamValues; ++i) acc[i] = 0.0f;
  if (g < G) {
    const size_t pg = size_t(b / vw.views_per_set) * G + g;
    const size_t slot = size_t(b) * G + size_t(rank_of[size_t(b) * G + g]);
    const float* g2 = grad2d + slot * GSB_GRAD2D_FLOATS;
    const float dmx = g2[0], dmy = g2[1], dA = g2[2], dB = g2[3], dC = g2[4];
    const float dcol[3] = {g2[6], g2[7], g2[8]};
    const float t = vw.times ? vw.times[b] : 0.0f;
    const Camera cam = load_camera(vw, b);
    const GaussParams p = load_params(sc, pg, t, view_basis(sc, vw, b));
    Proj P;
    project(p, cam, rc.near_plane, P);
    if (P.front) {
      float dmt[3] = {0.0f, 0.0f, 0.0f};
      sh_backward<K>(sc, pg, P.d, dcol, sc.flags & GSB_SCENE_SH_CLAMP, nullptr, dmt);
      CovGrad cg;
      cov_backward(P, dA, dB, dC, cg);
      float dmc[3];
      if (!LENS || cam.lens == GSB_LENS_PINHOLE) {
        pinhole_point_backward(P, cam, dmx, dmy, cg, dmc);
        const float izs = 1.0f / P.zs, izs2 = izs * izs;
        acc[0] = dmx * P.xp * izs + cg.du[0] * izs - cg.du[2] * P.xp * izs2;  // fx (common.py:210-229)
        acc[1] = dmy * P.yp * izs + cg.dv[1] * izs - cg.dv[2] * P.yp * izs2;  // fy
      } else {
        Dual<8> coef[5];
#pragma unroll
        for (int i = 0; i < 5; ++i) coef[i] = seed<8>(cam.dist[i], 3 + i);
        const LensProjection<Dual<8>> lp =
            lens_project<Dual<8>>(seed<8>(P.xp, 0), seed<8>(P.yp, 1), seed<8>(P.zs, 2), cam, coef);
        const float dJ[6] = {cg.du[0], cg.du[1], cg.du[2], cg.dv[0], cg.dv[1], cg.dv[2]};
        float dv8[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          float a = dmx * lp.mx.d[k] + dmy * lp.my.d[k];
#pragma unroll
          for (int e = 0; e < 6; ++e) a += dJ[e] * lp.J[e].d[k];
          dv8[k] = a;
        }
        dmc[0] = dv8[0], dmc[1] = dv8[1], dmc[2] = dv8[2];
#pragma unroll
        for (int i = 0; i < 5; ++i) acc[16 + i] = dv8[3 + i];
        // pixel = f xd + c, J = diag(f) U
        acc[0] = dmx * lp.xd.v + cg.du[0] * lp.U[0].v + cg.du[1] * lp.U[1].v + cg.du[2] * lp.U[2].v;
        acc[1] = dmy * lp.yd.v + cg.dv[0] * lp.U[3].v + cg.dv[1] * lp.U[4].v + cg.dv[2] * lp.U[5].v;
      }
      acc[2] = dmx;
      acc[3] = dmy;
      dmc[2] += g2[9];  // depth output
      // rotation: d_j dmc_k from the mean, 2 (S R dcc)_jk from the covariance (S = M M^T)
      float SR[9];
#pragma unroll
      for (int j = 0; j < 3; ++j)
#pragma unroll
        for (int a = 0; a < 3; ++a) {
          float s = 0.0f;
#pragma unroll
          for (int i = 0; i < 3; ++i) {
            const float Sji = P.M[j * 3 + 0] * P.M[i * 3 + 0] + P.M[j * 3 + 1] * P.M[i * 3 + 1] + P.M[j * 3 + 2] * P.M[i * 3 + 2];
            s += Sji * cam.R[i * 3 + a];
          }
          SR[j * 3 + a] = s;
        }
#pragma unroll
      for (int j = 0; j < 3; ++j)
#pragma unroll
        for (int k = 0; k < 3; ++k) {
          float c = 0.0f;
#pragma unroll
          for (int a = 0; a < 3; ++a) c += SR[j * 3 + a] * cg.dcc[a * 3 + k];
          acc[4 + j * 3 + k] = P.d[j] * dmc[k] + 2.0f * c;
        }
      // centre: d = mean_t - centre enters the camera point and the SH direction
#pragma unroll
      for (int j = 0; j < 3; ++j)
        acc[13 + j] = -(dmt[j] + cam.R[j * 3 + 0] * dmc[0] + cam.R[j * 3 + 1] * dmc[1] + cam.R[j * 3 + 2] * dmc[2]);
    }
  }
  // block reduction: warps, then the 4 warp partials
  __shared__ float part[4][kCamValues];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int i = 0; i < kCamValues; ++i) {
    float v = acc[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) part[warp][i] = v;
  }
  __syncthreads();
  if (threadIdx.x < kCamValues) {
    const int i = threadIdx.x;
    const float v = part[0][i] + part[1][i] + part[2][i] + part[3][i];
    if (v != 0.0f) {
      float* dst = nullptr;
      if (i < 4) dst = out.intrinsics ? out.intrinsics + b * 4 + i : nullptr;
      else if (i < 13) dst = out.camera_to_world ? out.camera_to_world + b * 16 + ((i - 4) / 3) * 4 + (i - 4) % 3 : nullptr;
      else if (i < 16) dst = out.camera_to_world ? out.camera_to_world + b * 16 + (i - 13) * 4 + 3 : nullptr;
      else dst = out.distortion ? out.distortion + b * 5 + (i - 16) : nullptr;
      if (dst) atomicAdd(dst, v);
    }
  }
}

// ---- host launchers --------------------------------------------------------------------------

static int grid_for(size_t n, int threads) {
  const size_t blocks = (n + threads - 1) / threads;
  return int(std::min<size_t>(blocks, size_t(148) * 64));
}

gsb_status launch_depth_keys(const gsb_scene& sc, const gsb_views& vw, uint32_t* keys, uint32_t* vals, uint32_t* hist,
                             cudaStream_t st) {
  const dim3 grid(unsigned((size_t(sc.n_gaussians) + kKeyThreads * kKeyItems - 1) / (kKeyThreads * kKeyItems)),
                  unsigned(vw.n_views));
  note_launch();
  if (sc.flags & GSB_SCENE_BANK) depth_key_kernel<true><<<grid, kKeyThreads, 0, st>>>(sc, vw, keys, vals, hist);
  else depth_key_kernel<false><<<grid, kKeyThreads, 0, st>>>(sc, vw, keys, vals, hist);
  return launch_status();
}

gsb_status launch_invert_order(const uint32_t* sorted_vals, int32_t B, int32_t G, int32_t* sorted_ids,
                               int32_t* rank_of, cudaStream_t st) {
  note_launch();
  invert_order_kernel<<<grid_for(size_t(B) * G, 256), 256, 0, st>>>(sorted_vals, B, G, sorted_ids, rank_of);
  return launch_status();
}

gsb_status launch_preprocess_fwd(const gsb_scene& sc, const gsb_views& vw, const RenderConsts& rc,
                                 const int32_t* rank_of, float* records, int4* rects, uint32_t* counts, float* cov,
                                 cudaStream_t st, int32_t* status) {
  const size_t n = size_t(vw.n_views) * sc.n_gaussians;
  note_launch();
  if (sc.flags & GSB_SCENE_BANK)
    preprocess_fwd_kernel<true>
        <<<grid_for(n, 256), 256, 0, st>>>(sc, vw, rc, rank_of, records, rects, counts, cov, status);
  else
    preprocess_fwd_kernel<false>
        <<<grid_for(n, 256), 256, 0, st>>>(sc, vw, rc, rank_of, records, rects, counts, cov, status);
  return launch_status();
}

template <int K, bool LENS, int LPG>
static void bwd_launch_lpg(const gsb_scene& sc, const gsb_views& vw, const RenderConsts& rc, const int32_t* rank_of,
                           const float* grad2d, const gsb_scene_grads& gr, cudaStream_t st) {
  const size_t n = rc.bwd_count ? size_t(rc.bwd_count) : size_t(sc.n_sets) * sc.n_gaussians;
  const int grid = grid_for(n * LPG, 128);
  preprocess_bwd_kernel<K, LENS, false, LPG><<<grid, 128, 0, st>>>(sc, vw, rc, rank_of, grad2d, gr);
}

// Lanes per Gaussian: 4 when a set has 4 views or more, else 1.  Measured on one B200 (ms, 16
// views per set x 32768 Gaussians SH1 / 8 views x 200k SH3): one lane 0.049 / 0.283, four 0.044 /
// 0.213; eight lanes 0.045 / 0.255 and sixteen (one view each) 0.059 on the first, where the
// shuffles of the group sums cost more than the extra parallelism gains.
template <int K, bool LENS>
static void bwd_launch_k(const gsb_scene& sc, const gsb_views& vw, const RenderConsts& rc, const int32_t* rank_of,
                         const float* grad2d, const gsb_scene_grads& gr, cudaStream_t st) {
  if (std::min(vw.views_per_set, vw.n_views) >= 4) bwd_launch_lpg<K, LENS, 4>(sc, vw, rc, rank_of, grad2d, gr, st);
  else bwd_launch_lpg<K, LENS, 1>(sc, vw, rc, rank_of, grad2d, gr, st);
}

template <bool LENS>
static void launch_bwd_for_degree(int deg, int grid, const gsb_scene& sc, const gsb_views& vw, const RenderConsts& rc,
                                  const int32_t* rank_of, const float* grad2d, const gsb_scene_grads& gr,
                                  cudaStream_t st) {
  if (sc.flags & GSB_SCENE_BANK) {  // activated values only (checked at the entry points)
    preprocess_bwd_kernel<0, LENS, true, 1><<<grid, 128, 0, st>>>(sc, vw, rc, rank_of, grad2d, gr);
    return;
  }
  switch (deg) {
    case -1: bwd_launch_k<0, LENS>(sc, vw, rc, rank_of, grad2d, gr, st); break;
    case 0: bwd_launch_k<1, LENS>(sc, vw, rc, rank_of, grad2d, gr, st); break;
    case 1: bwd_launch_k<4, LENS>(sc, vw, rc, rank_of, grad2d, gr, st); break;
    case 2: bwd_launch_k<9, LENS>(sc, vw, rc, rank_of, grad2d, gr, st); break;
    default: bwd_launch_k<16, LENS>(sc, vw, rc, rank_of, grad2d, gr, st); break;
  }
}

template <bool LENS>
static void launch_camera_for_degree(int deg, dim3 grid, const gsb_scene& sc, const gsb_views& vw,
                                     const RenderConsts& rc, const int32_t* rank_of, const float* grad2d,
                                     const gsb_camera_grads& out, cudaStream_t st) {
  switch (deg) {
    case -1: camera_bwd_kernel<0, LENS><<<grid, 128, 0, st>>>(sc, vw, rc, rank_of, grad2d, out); break;
    case 0: camera_bwd_kernel<1, LENS><<<grid, 128, 0, st>>>(sc, vw, rc, rank_of, grad2d, out); break;
    case 1: camera_bwd_kernel<4, LENS><<<grid, 128, 0, st>>>(sc, vw, rc, rank_of, grad2d, out); break;
    case 2: camera_bwd_kernel<9, LENS><<<grid, 128, 0, st>>>(sc, vw, rc, rank_of, grad2d, out); break;
    default: camera_bwd_kernel<16, LENS><<<grid, 128, 0, st>>>(sc, vw, rc, rank_of, grad2d, out); break;
  }
}

gsb_status launch_camera_bwd(const gsb_scene& sc, const gsb_views& vw, const RenderConsts& rc, const int32_t* rank_of,
                             const float* grad2d, const gsb_camera_grads& out, cudaStream_t st) {
  const int B = vw.n_views;
  if (out.intrinsics && cudaMemsetAsync(out.intrinsics, 0, size_t(B) * 4 * sizeof(float), st)) return GSB_ERR_CUDA;
  if (out.camera_to_world && cudaMemsetAsync(out.camera_to_world, 0, size_t(B) * 16 * sizeof(float), st))
    return GSB_ERR_CUDA;
  if (out.distortion && cudaMemsetAsync(out.distortion, 0, size_t(B) * 5 * sizeof(float), st)) return GSB_ERR_CUDA;
  const bool raw = sc.flags & GSB_SCENE_RAW;
  const int deg = raw ? sc.sh_degree : -1;
  if (deg < -1 || deg > 3) return GSB_ERR_ARG;
  const dim3 grid(unsigned((size_t(sc.n_gaussians) + 127) / 128), unsigned(B));
  note_launch();
  if (vw.lens_models) launch_camera_for_degree<true>(deg, grid, sc, vw, rc, rank_of, grad2d, out, st);
  else launch_camera_for_degree<false>(deg, grid, sc, vw, rc, rank_of, grad2d, out, st);
  return launch_status();
}

gsb_status launch_preprocess_bwd(const gsb_scene& sc, const gsb_views& vw, const RenderConsts& rc,
                                 const int32_t* rank_of, const float* grad2d, const gsb_scene_grads& gr,
                                 cudaStream_t st) {
  const size_t n = rc.bwd_count ? size_t(rc.bwd_count) : size_t(sc.n_sets) * sc.n_gaussians;
  const int grid = grid_for(n, 128);
  const bool raw = sc.flags & GSB_SCENE_RAW;
  const int deg = raw ? sc.sh_degree : -1;
  if (deg < -1 || deg > 3) return GSB_ERR_ARG;
  note_launch();
  if (vw.lens_models) launch_bwd_for_degree<true>(deg, grid, sc, vw, rc, rank_of, grad2d, gr, st);
  else launch_bwd_for_degree<false>(deg, grid, sc, vw, rc, rank_of, grad2d, gr, st);
  return launch_status();
}

}  // namespace gsb
