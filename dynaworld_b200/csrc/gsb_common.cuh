// Shared device helpers of libgsb200 (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "gsb200.h"

namespace gsb {

// Every workspace starts with this header; kernels record the first error in `status`.
struct WorkspaceHeader {
  int32_t status;
  int32_t detail;
  uint32_t pad[62];
};
static_assert(sizeof(WorkspaceHeader) == 256, "header is 256 bytes");

constexpr size_t kAlign = 256;
__host__ __device__ inline size_t align_up(size_t x, size_t a = kAlign) { return (x + a - 1) / a * a; }

// Bump allocator over a caller-owned workspace (host side; no device allocation).
struct Carver {
  char* base;
  size_t used;
  size_t cap;
  explicit Carver(void* p, size_t c) : base(static_cast<char*>(p)), used(0), cap(c) {}
  template <typename T>
  T* take(size_t count) {
    size_t off = align_up(used);
    used = off + align_up(count * sizeof(T));
    return (base && used <= cap) ? reinterpret_cast<T*>(base + off) : nullptr;
  }
  bool ok() const { return used <= cap; }
};

__device__ inline void record_error(int32_t* status, int code, int detail = 0) {
  if (status && atomicCAS(status, 0, code) == 0) status[1] = detail;
}

// IEEE-754 float -> uint32 whose unsigned order is the float order; -0 == +0, NaN last.
__device__ __host__ inline uint32_t float_sort_key(float f) {
  uint32_t u;
#ifdef __CUDA_ARCH__
  u = __float_as_uint(f);
#else
  memcpy(&u, &f, 4);
#endif
  if ((u & 0x7fffffffu) == 0u) u = 0u;                      // -0 -> +0
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) u = 0x7fc00000u;  // NaN
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Warp-aggregated counts of the four 8-bit digits of each lane's key into a block's histograms
// (the segmented sort's counts, taken by the kernel that writes the keys).  Every lane of the warp
// calls it; lanes with valid = false count nothing.
__device__ inline void count_digits4(uint32_t (*s_hist)[256], uint32_t key, bool valid) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint32_t digit = valid ? (key >> (8 * p)) & 0xffu : 0xffffffffu;
    const uint32_t peers = __match_any_sync(0xffffffffu, digit);
    if (valid && lane == __ffs(peers) - 1) atomicAdd(&s_hist[p][digit], uint32_t(__popc(peers)));
  }
}

// Adds a block's four digit histograms to the segment's [4][256] counts in global memory.
__device__ inline void flush_digits4(const uint32_t (*s_hist)[256], uint32_t* __restrict__ hist) {
  for (int i = threadIdx.x; i < 4 * 256; i += blockDim.x) {
    const uint32_t c = s_hist[i / 256][i % 256];
    if (c) atomicAdd(hist + i, c);
  }
}

// Culling extents of the ellipse {q <= tau}, q = A dx^2 + B dx dy + C dy^2, that the raster's
// warp-block test reads from the record's fourth float4: half widths sqrt(tau (A^-1)_ii) (with a
// relative and an absolute margin) and the slopes of the lines through its extreme points;
// +inf half widths mark a conic that is never culled.
__device__ inline float4 cull_extents(float A, float B, float C, float tau) {
  const float det = A * C - 0.25f * B * B;
  if (!(det > 0.0f) || !(tau >= 0.0f) || !isfinite(tau))
    return make_float4(__int_as_float(0x7f800000), __int_as_float(0x7f800000), 0.0f, 0.0f);
  const float ex = sqrtf(tau * C / det) * 1.0001f + 0.01f;
  const float ey = sqrtf(tau * A / det) * 1.0001f + 0.01f;
  return make_float4(ex, ey, -0.5f * B / C, -0.5f * B / A);
}

// List length on a log scale in 8 bits (exact below 16, then 8 steps per power of two), so that
// one 8-bit radix pass orders the tiles (the raster launch order, longest lists first).
__device__ inline uint32_t length_class(uint32_t len) {
  if (len < 8u) return len;
  const int e = 31 - __clz(len);  // 3 .. 31
  return uint32_t(e - 2) * 8u + ((len >> (e - 3)) & 7u);  // 8 .. 239, non-decreasing in len
}

// log2(fl32(1 + 1e-6)) = log2(1 + 2^-20): the per-Gaussian transmittance growth of dense.py:225.
constexpr double kLog2F0 = 1.3757959012e-06;

struct Intrinsics {
  float fx, fy, cx, cy;
};

// Camera of one view, as read from device arrays.
struct Camera {
  float R[9];  // camera_to_world rotation, row-major: R[j*3+k] = c2w[j][k]
  float t[3];  // camera centre (world)
  Intrinsics k;
  int lens;       // GSB_LENS_*
  float dist[5];  // distortion coefficients (non-pinhole lenses)
};

__device__ inline Camera load_camera(const gsb_views& vw, int b) {
  Camera c;
  const float* m = vw.camera_to_world + b * 16;
#pragma unroll
  for (int j = 0; j < 3; ++j) {
#pragma unroll
    for (int k = 0; k < 3; ++k) c.R[j * 3 + k] = m[j * 4 + k];
    c.t[j] = m[j * 4 + 3];
  }
  c.k.fx = vw.intrinsics[b * 4 + 0];
  c.k.fy = vw.intrinsics[b * 4 + 1];
  c.k.cx = vw.intrinsics[b * 4 + 2];
  c.k.cy = vw.intrinsics[b * 4 + 3];
  c.lens = vw.lens_models ? vw.lens_models[b] : GSB_LENS_PINHOLE;
#pragma unroll
  for (int i = 0; i < 5; ++i) c.dist[i] = (c.lens != GSB_LENS_PINHOLE) ? vw.distortion[b * 5 + i] : 0.0f;
  return c;
}

// Camera-space coordinate k of world point m: fma(d2,R2k, fma(d1,R1k, d0*R0k)), d = fl32(m - t).
// Same rounding as the reference's float32 (m - t) @ R (common.py:39-51) on FMA CPUs, so depth
// keys, and hence the sort order, agree bit for bit.
__device__ inline float cam_coord(const float d[3], const float R[9], int k) {
  return __fmaf_rn(d[2], R[6 + k], __fmaf_rn(d[1], R[3 + k], __fmul_rn(d[0], R[k])));
}

}  // namespace gsb
