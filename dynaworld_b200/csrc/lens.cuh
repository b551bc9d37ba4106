// Central lens models of the reference's camera_model projection
// (src/train/renderers/projection.py:75-214): normalised coordinates x/z, y/z and their Jacobian,
// radial-tangential (Brown-Conrady k1, k2, p1, p2, k3) and OpenCV fisheye (Kannala-Brandt k1..k4)
// distortion with the reference's closed-form lens Jacobians, and
// pixel = (fx xd + cx, fy yd + cy), J = diag(fx, fy) L N (2 x 3, d pixel / d camera point).
//
// Written once over a scalar type T: float for the forward, Dual3 (value + derivatives along the
// three camera coordinates) for the backward, which then differentiates exactly the expressions
// the reference's autograd differentiates -- the pixel position and every Jacobian entry.
#pragma once

#include "gsb_common.cuh"

namespace gsb {

struct Dual3 {
  float v, d[3];
};

__device__ inline Dual3 dual(float v, float d0, float d1, float d2) { return Dual3{v, {d0, d1, d2}}; }
__device__ inline Dual3 operator+(Dual3 a, Dual3 b) { return dual(a.v + b.v, a.d[0] + b.d[0], a.d[1] + b.d[1], a.d[2] + b.d[2]); }
__device__ inline Dual3 operator-(Dual3 a, Dual3 b) { return dual(a.v - b.v, a.d[0] - b.d[0], a.d[1] - b.d[1], a.d[2] - b.d[2]); }
__device__ inline Dual3 operator-(Dual3 a) { return dual(-a.v, -a.d[0], -a.d[1], -a.d[2]); }
__device__ inline Dual3 operator*(Dual3 a, Dual3 b) {
  return dual(a.v * b.v, a.d[0] * b.v + a.v * b.d[0], a.d[1] * b.v + a.v * b.d[1], a.d[2] * b.v + a.v * b.d[2]);
}
__device__ inline Dual3 operator/(Dual3 a, Dual3 b) {
  const float q = a.v / b.v, ib = 1.0f / b.v;
  return dual(q, (a.d[0] - q * b.d[0]) * ib, (a.d[1] - q * b.d[1]) * ib, (a.d[2] - q * b.d[2]) * ib);
}
__device__ inline Dual3 operator+(Dual3 a, float b) { return dual(a.v + b, a.d[0], a.d[1], a.d[2]); }
__device__ inline Dual3 operator+(float a, Dual3 b) { return b + a; }
__device__ inline Dual3 operator-(float a, Dual3 b) { return dual(a - b.v, -b.d[0], -b.d[1], -b.d[2]); }
__device__ inline Dual3 operator*(float a, Dual3 b) { return dual(a * b.v, a * b.d[0], a * b.d[1], a * b.d[2]); }
__device__ inline Dual3 operator*(Dual3 a, float b) { return b * a; }
__device__ inline Dual3 operator/(float a, Dual3 b) {
  const float q = a / b.v, s = -q / b.v;
  return dual(q, s * b.d[0], s * b.d[1], s * b.d[2]);
}

__device__ inline float value_of(float x) { return x; }
__device__ inline float value_of(const Dual3& x) { return x.v; }
__device__ inline float lens_sqrt(float x) { return sqrtf(x); }
__device__ inline Dual3 lens_sqrt(Dual3 x) {
  const float r = sqrtf(x.v), s = 0.5f / r;
  return dual(r, s * x.d[0], s * x.d[1], s * x.d[2]);
}
__device__ inline float lens_atan(float x) { return atanf(x); }
__device__ inline Dual3 lens_atan(Dual3 x) {
  const float s = 1.0f / (1.0f + x.v * x.v);
  return dual(atanf(x.v), s * x.d[0], s * x.d[1], s * x.d[2]);
}
// torch.clamp(x, min=lo): the gradient passes where x >= lo
__device__ inline float clamp_min(float x, float lo) { return fmaxf(x, lo); }
__device__ inline Dual3 clamp_min(Dual3 x, float lo) { return x.v >= lo ? x : dual(lo, 0.0f, 0.0f, 0.0f); }
template <typename T>
__device__ inline T constant(float v);
template <>
__device__ inline float constant<float>(float v) { return v; }
template <>
__device__ inline Dual3 constant<Dual3>(float v) { return dual(v, 0.0f, 0.0f, 0.0f); }

template <typename T>
struct LensJ {
  T xd, yd;                // distorted normalised coordinates
  T L00, L01, L10, L11;    // d(xd, yd) / d(x, y)
};

// projection.py:93-116
template <typename T>
__device__ inline LensJ<T> radial_tangential(T x, T y, const float c[5]) {
  const float k1 = c[0], k2 = c[1], p1 = c[2], p2 = c[3], k3 = c[4];
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
__device__ inline LensJ<T> opencv_fisheye(T x, T y, const float c[5]) {
  const float k1 = c[0], k2 = c[1], k3 = c[2], k4 = c[3];
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
  const T scale = valid ? theta_d / radius : constant<T>(1.0f);
  o.xd = scale * x;
  o.yd = scale * y;
  const T dtd = 1.0f + (3.0f * k1) * t2 + (5.0f * k2) * t4 + (7.0f * k3) * t6 + (9.0f * k4) * t8;
  const T dtdr = 1.0f / (1.0f + radius * radius);
  const T dsdr = valid ? (dtd * dtdr * radius - theta_d) / (radius * radius) : constant<T>(0.0f);
  const T inv_r = valid ? 1.0f / radius : constant<T>(0.0f);
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
};

// Camera-space point (xp, yp, zs) of a Gaussian in front of the near plane (x_project,
// y_project, z_safe of projection.py:75-90) -> pixel and Jacobian (projection.py:164-214).
template <typename T>
__device__ inline LensProjection<T> lens_project(T xp, T yp, T zs, const Camera& cam) {
  const T xn = xp / zs, yn = yp / zs;
  const T n00 = 1.0f / zs;                 // norm_jacobian[0][0] = [1][1]
  const T n02 = -xp / (zs * zs);
  const T n12 = -yp / (zs * zs);
  const LensJ<T> l = cam.lens == GSB_LENS_OPENCV_FISHEYE ? opencv_fisheye(xn, yn, cam.dist)
                                                         : radial_tangential(xn, yn, cam.dist);
  const float fx = cam.k.fx, fy = cam.k.fy;
  const T a00 = fx * l.L00, a01 = fx * l.L01, a10 = fy * l.L10, a11 = fy * l.L11;  // diag(f) L
  LensProjection<T> p;
  p.J[0] = a00 * n00;
  p.J[1] = a01 * n00;
  p.J[2] = a00 * n02 + a01 * n12;
  p.J[3] = a10 * n00;
  p.J[4] = a11 * n00;
  p.J[5] = a10 * n02 + a11 * n12;
  p.mx = fx * l.xd + cam.k.cx;
  p.my = fy * l.yd + cam.k.cy;
  return p;
}

}  // namespace gsb
