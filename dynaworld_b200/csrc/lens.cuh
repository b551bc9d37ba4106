// Central lens models of the reference's camera_model projection
// (src/train/renderers/projection.py:75-214): normalised coordinates x/z, y/z and their Jacobian,
// radial-tangential (Brown-Conrady k1, k2, p1, p2, k3) and OpenCV fisheye (Kannala-Brandt k1..k4)
// distortion with the reference's closed-form lens Jacobians, and
// pixel = (fx xd + cx, fy yd + cy), J = diag(fx, fy) L N (2 x 3, d pixel / d camera point).
//
// Written once over a scalar type T: float for the forward, Dual<N> (value + N derivatives) for
// the backward -- Dual<3> along the camera-space point (x, y, z), Dual<8> along the point and the
// five distortion coefficients -- which then differentiates exactly the expressions the
// reference's autograd differentiates: the pixel position and every Jacobian entry.
#pragma once

#include "gsb_common.cuh"

namespace gsb {

template <int N>
struct Dual {
  float v, d[N];
};
using Dual3 = Dual<3>;

template <int N>
__device__ inline Dual<N> seed(float v, int slot) {  // slot < 0: a constant
  Dual<N> r;
  r.v = v;
#pragma unroll
  for (int k = 0; k < N; ++k) r.d[k] = (k == slot) ? 1.0f : 0.0f;
  return r;
}
__device__ inline Dual3 dual(float v, float d0, float d1, float d2) { return Dual3{v, {d0, d1, d2}}; }

template <int N>
__device__ inline Dual<N> operator+(const Dual<N>& a, const Dual<N>& b) {
  Dual<N> r;
  r.v = a.v + b.v;
#pragma unroll
  for (int k = 0; k < N; ++k) r.d[k] = a.d[k] + b.d[k];
  return r;
}
template <int N>
__device__ inline Dual<N> operator-(const Dual<N>& a, const Dual<N>& b) {
  Dual<N> r;
  r.v = a.v - b.v;
#pragma unroll
  for (int k = 0; k < N; ++k) r.d[k] = a.d[k] - b.d[k];
  return r;
}
template <int N>
__device__ inline Dual<N> operator-(const Dual<N>& a) {
  Dual<N> r;
  r.v = -a.v;
#pragma unroll
  for (int k = 0; k < N; ++k) r.d[k] = -a.d[k];
  return r;
}
template <int N>
__device__ inline Dual<N> operator*(const Dual<N>& a, const Dual<N>& b) {
  Dual<N> r;
  r.v = a.v * b.v;
#pragma unroll
  for (int k = 0; k < N; ++k) r.d[k] = a.d[k] * b.v + a.v * b.d[k];
  return r;
}
template <int N>
__device__ inline Dual<N> operator/(const Dual<N>& a, const Dual<N>& b) {
  Dual<N> r;
  r.v = a.v / b.v;
  const float ib = 1.0f / b.v;
#pragma unroll
  for (int k = 0; k < N; ++k) r.d[k] = (a.d[k] - r.v * b.d[k]) * ib;
  return r;
}
template <int N>
__device__ inline Dual<N> operator+(const Dual<N>& a, float b) {
  Dual<N> r = a;
  r.v = a.v + b;
  return r;
}
template <int N>
__device__ inline Dual<N> operator+(float a, const Dual<N>& b) { return b + a; }
template <int N>
__device__ inline Dual<N> operator-(float a, const Dual<N>& b) { return (-b) + a; }
template <int N>
__device__ inline Dual<N> operator*(float a, const Dual<N>& b) {
  Dual<N> r;
  r.v = a * b.v;
#pragma unroll
  for (int k = 0; k < N; ++k) r.d[k] = a * b.d[k];
  return r;
}
template <int N>
__device__ inline Dual<N> operator*(const Dual<N>& a, float b) { return b * a; }
template <int N>
__device__ inline Dual<N> operator/(float a, const Dual<N>& b) {
  Dual<N> r;
  r.v = a / b.v;
  const float s = -r.v / b.v;
#pragma unroll
  for (int k = 0; k < N; ++k) r.d[k] = s * b.d[k];
  return r;
}

__device__ inline float value_of(float x) { return x; }
template <int N>
__device__ inline float value_of(const Dual<N>& x) { return x.v; }

__device__ inline float lens_sqrt(float x) { return sqrtf(x); }
template <int N>
__device__ inline Dual<N> lens_sqrt(const Dual<N>& x) {
  Dual<N> r;
  r.v = sqrtf(x.v);
  const float s = 0.5f / r.v;
#pragma unroll
  for (int k = 0; k < N; ++k) r.d[k] = s * x.d[k];
  return r;
}
__device__ inline float lens_atan(float x) { return atanf(x); }
template <int N>
__device__ inline Dual<N> lens_atan(const Dual<N>& x) {
  Dual<N> r;
  r.v = atanf(x.v);
  const float s = 1.0f / (1.0f + x.v * x.v);
#pragma unroll
  for (int k = 0; k < N; ++k) r.d[k] = s * x.d[k];
  return r;
}
// torch.clamp(x, min=lo): the gradient passes where x >= lo
__device__ inline float clamp_min(float x, float lo) { return fmaxf(x, lo); }
template <int N>
__device__ inline Dual<N> clamp_min(const Dual<N>& x, float lo) { return x.v >= lo ? x : seed<N>(lo, -1); }

template <typename T>
struct Constant {
  __device__ static T of(float v) { return v; }
};
template <int N>
struct Constant<Dual<N>> {
  __device__ static Dual<N> of(float v) { return seed<N>(v, -1); }
};

template <typename T>
struct LensJ {
  T xd, yd;                // distorted normalised coordinates
  T L00, L01, L10, L11;    // d(xd, yd) / d(x, y)
};

// projection.py:93-116
template <typename T>
__device__ inline LensJ<T> radial_tangential(T x, T y, const T c[5]) {
  const T k1 = c[0], k2 = c[1], p1 = c[2], p2 = c[3], k3 = c[4];
  LensJ<T> o;
  const T r2 = x * x + y * y;
  const T r4 = r2 * r2;
  const T r6 = r4 * r2;
  const T radial = 1.0f + k1 * r2 + k2 * r4 + k3 * r6;
  o.xd = x * radial + (2.0f * p1) * x * y + p2 * (r2 + 2.0f * x * x);
  o.yd = y * radial + p1 * (r2 + 2.0f * y * y) + (2.0f * p2) * x * y;
  const T rdr2 = k1 + (2.0f * k2) * r2 + (3.0f * k3) * r4;
  const T rdx = 2.0f * x * rdr2;
  const T rdy = 2.0f * y * rdr2;
  o.L00 = radial + x * rdx + (2.0f * p1) * y + (6.0f * p2) * x;
  o.L01 = x * rdy + (2.0f * p1) * x + (2.0f * p2) * y;
  o.L10 = y * rdx + (2.0f * p1) * x + (2.0f * p2) * y;
  o.L11 = radial + y * rdy + (6.0f * p1) * y + (2.0f * p2) * x;
  return o;
}

// projection.py:119-161
template <typename T>
__device__ inline LensJ<T> opencv_fisheye(T x, T y, const T c[5]) {
  const T k1 = c[0], k2 = c[1], k3 = c[2], k4 = c[3];
  constexpr float kEps2 = 1.0e-8f * 1.0e-8f;
  LensJ<T> o;
  const T r2 = x * x + y * y;
  const T radius = lens_sqrt(clamp_min(r2, kEps2));
  const T theta = lens_atan(radius);
  const T t2 = theta * theta;
  const T t4 = t2 * t2;
  const T t6 = t4 * t2;
  const T t8 = t4 * t4;
  const T theta_d = theta * (1.0f + k1 * t2 + k2 * t4 + k3 * t6 + k4 * t8);
  const bool valid = value_of(r2) > kEps2;
  const T scale = valid ? theta_d / radius : Constant<T>::of(1.0f);
  o.xd = scale * x;
  o.yd = scale * y;
  const T dtd = 1.0f + (3.0f * k1) * t2 + (5.0f * k2) * t4 + (7.0f * k3) * t6 + (9.0f * k4) * t8;
  const T dtdr = 1.0f / (1.0f + radius * radius);
  const T dsdr = valid ? (dtd * dtdr * radius - theta_d) / (radius * radius) : Constant<T>::of(0.0f);
  const T inv_r = valid ? 1.0f / radius : Constant<T>::of(0.0f);
  const T dsdx = dsdr * x * inv_r;
  const T dsdy = dsdr * y * inv_r;
  o.L00 = scale + x * dsdx;
  o.L01 = x * dsdy;
  o.L10 = y * dsdx;
  o.L11 = scale + y * dsdy;
  return o;
}

template <typename T>
struct LensProjection {
  T mx, my;        // pixel position
  T J[6];          // d pixel / d camera point, row-major 2 x 3
  T xd, yd;        // distorted normalised coordinates (d pixel / d (fx, fy))
  T U[6];          // L N: J with the focal lengths factored out (d J / d (fx, fy))
};

// Camera-space point (xp, yp, zs) of a Gaussian in front of the near plane (x_project,
// y_project, z_safe of projection.py:75-90) -> pixel and Jacobian (projection.py:164-214);
// ``coef`` are the lens's distortion coefficients.
template <typename T>
__device__ inline LensProjection<T> lens_project(T xp, T yp, T zs, const Camera& cam, const T coef[5]) {
  const T xn = xp / zs, yn = yp / zs;
  const T n00 = 1.0f / zs;                 // norm_jacobian[0][0] = [1][1]
  const T n02 = -xp / (zs * zs);
  const T n12 = -yp / (zs * zs);
  const LensJ<T> l = cam.lens == GSB_LENS_OPENCV_FISHEYE ? opencv_fisheye(xn, yn, coef) : radial_tangential(xn, yn, coef);
  const float fx = cam.k.fx, fy = cam.k.fy;
  LensProjection<T> p;
  p.U[0] = l.L00 * n00;
  p.U[1] = l.L01 * n00;
  p.U[2] = l.L00 * n02 + l.L01 * n12;
  p.U[3] = l.L10 * n00;
  p.U[4] = l.L11 * n00;
  p.U[5] = l.L10 * n02 + l.L11 * n12;
  const T a00 = fx * l.L00, a01 = fx * l.L01, a10 = fy * l.L10, a11 = fy * l.L11;  // diag(f) L
  p.J[0] = a00 * n00;
  p.J[1] = a01 * n00;
  p.J[2] = a00 * n02 + a01 * n12;
  p.J[3] = a10 * n00;
  p.J[4] = a11 * n00;
  p.J[5] = a10 * n02 + a11 * n12;
  p.xd = l.xd;
  p.yd = l.yd;
  p.mx = fx * l.xd + cam.k.cx;
  p.my = fy * l.yd + cam.k.cy;
  return p;
}

// The coefficients of a view as constants of type T.
template <typename T>
__device__ inline void lens_coefficients(const Camera& cam, T coef[5]) {
#pragma unroll
  for (int i = 0; i < 5; ++i) coef[i] = Constant<T>::of(cam.dist[i]);
}

}  // namespace gsb
