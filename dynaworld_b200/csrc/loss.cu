// Fused reconstruction loss: value per image and d loss / d prediction in one pass.
//
// Restates reconstruction_loss_per_image (src/train/losses.py:58-85) with standard_gs =
// l1_weight * mean|pred - target| + dssim_weight * (1 - SSIM)/2, where SSIM (losses.py:21-44) is
// the per-image mean of the SSIM map built from reflect-padded 11x11 box means (losses.py:13-18,
// avg_pool2d after F.pad(mode="reflect")), C1 = 1e-4, C2 = 9e-4, clamped to [-1, 1].
//
// One CTA per 32x32 output tile of one image plane.  The five window means are separable sums
// over a shared-memory copy of the (reflected) input; the SSIM gradient needs the adjoint of the
// window operator, which for reflect padding folds the zero-padded window sums at the mirrored
// positions -q and 2(N-1)-q back onto q:
//   (W^T g)(q) = sum_{m in {q, -q, 2(N-1)-q} valid} sum_k w_k g(m + k)   (g = 0 off the image).
// The kernel assumes the final clamp of the SSIM mean is inactive; a finishing kernel computes the
// per-image loss and a fix-up kernel rewrites the gradient of any image whose mean left [-1, 1].
#include <cmath>
#include <mutex>

#include "gsb_common.cuh"
#include "gsb_internal.h"

namespace gsb {

constexpr int kLossTile = 32;
// 384 threads, three CTAs per SM: with its two regions reused (65 KB of shared memory per tile) and
// at most 56 registers a thread, three tiles share an SM and one's barriers overlap the others'
// work.  Measured on one B200, 8 x 1920x1080 loss: 100 KB and 512 threads (two CTAs per SM) 1.81 ms;
// 65 KB, 512 threads, two CTAs 1.85; three CTAs of 512 (40 registers) 1.63; three of 384 1.60.
// (Earlier, at 100 KB: 16 x 128^2 / 8 x 384^2, 256 threads 0.068 / 0.216 ms, 512 0.062 / 0.192,
// 1024 0.064 / 0.201.)
constexpr int kLossThreads = 384;
constexpr int kLossCtasPerSm = 3;

struct LossArgs {
  int B, C, H, W;
  int type;  // 0 standard_gs, 1 l1, 2 mse, 3 l1_mse
  float c1, c2;
  float c_l1, c_mse, c_ssim;  // gradient coefficients (already divided by C*H*W)
  float w[16];                // window taps, w[k + half]
  int box;                    // every tap equal (the box window): running sums
  int plane_base;             // first image plane (image * C + channel) of this launch
  const float* pred;
  const float* target;
  float* dpred;
  double* acc;  // [B, 3]: sum |d|, sum d^2, sum ssim
};

__device__ __forceinline__ int reflect_idx(int i, int n) {
  i = i < 0 ? -i : i;
  i = i >= n ? 2 * (n - 1) - i : i;
  return min(max(i, 0), n - 1);
}

// SSIM of one window from its five means m = (mu_x, mu_y, E[x^2], E[y^2], E[xy]) (losses.py:29-44,
// the denominator clamped at 1e-12), and its derivatives with respect to the three window means
// that depend on the prediction: d / d mu_x (through mu_x and the variances), d / d E[x^2],
// d / d E[xy].
__device__ __forceinline__ float ssim_point(const float m[5], float c1, float c2, float& d_mx, float& d_mxx,
                                            float& d_mxy) {
  const float mux = m[0], muy = m[1];
  const float mux2 = mux * mux, muy2 = muy * muy, muxy = mux * muy;
  const float sxx = m[2] - mux2, syy = m[3] - muy2, sxy = m[4] - muxy;
  const float A1 = 2.0f * muxy + c1, A2 = 2.0f * sxy + c2;
  const float B1 = mux2 + muy2 + c1, B2 = sxx + syy + c2;
  const float Draw = B1 * B2;
  const float Dc = fmaxf(Draw, 1e-12f);
  const float rD = 1.0f / Dc;  // one division; the quotients below are products with it
  const float s = (A1 * A2) * rD;
  const float dsdD = Draw >= 1e-12f ? -s * rD : 0.0f;
  const float ds_mu = (2.0f * muy * A2) * rD + dsdD * (2.0f * mux * B2);  // explicit mu_x
  const float ds_sxx = dsdD * B1;
  const float ds_sxy = 2.0f * A1 * rD;
  d_mx = ds_mu - 2.0f * mux * ds_sxx - muy * ds_sxy;
  d_mxx = ds_sxx;
  d_mxy = ds_sxy;
  return s;
}

// Shared-memory floats of the loss kernel's two regions (see loss_kernel).
template <int HW>
__host__ __device__ constexpr int loss_region_a() {
  constexpr int R = kLossTile + 4 * HW, M = kLossTile + 2 * HW;
  return 2 * R * R > 3 * M * M ? 2 * R * R : 3 * M * M;
}
template <int HW>
__host__ __device__ constexpr int loss_region_b() {
  constexpr int R = kLossTile + 4 * HW, M = kLossTile + 2 * HW;
  return 5 * R * M > 3 * M * kLossTile ? 5 * R * M : 3 * M * kLossTile;
}

template <int HW>
__global__ void __launch_bounds__(kLossThreads, kLossCtasPerSm) loss_kernel(LossArgs a) {
  constexpr int R = kLossTile + 4 * HW;  // input rows/cols held
  constexpr int M = kLossTile + 2 * HW;  // window-mean rows/cols computed
  // Two regions, each reused once its first tenant is dead: the inputs (read by the horizontal
  // pass only; the last pass reads its pixels from global memory) give way to the derivative maps
  // the vertical pass writes, the horizontal sums (read by the vertical pass only) to the
  // horizontal adjoint.
  extern __shared__ float smem[];
  float* xs = smem;                               // [R][R]
  float* ys = xs + R * R;                         // [R][R]
  float* gm = smem;                               // [3][M][M], after the horizontal pass
  float* hs = smem + loss_region_a<HW>();         // [5][R][M]
  float* ha = hs;                                 // [3][M][kLossTile], after the vertical pass
  __shared__ double s_red[3][kLossThreads / 32];

  const int plane = a.plane_base + int(blockIdx.z), b = plane / a.C;
  const int x0 = blockIdx.x * kLossTile, y0 = blockIdx.y * kLossTile;
  const int H = a.H, W = a.W;
  const size_t poff = size_t(plane) * H * W;
  const bool ssim = a.type == 0;
  const int tid = threadIdx.x;

  for (int i = tid; i < R * R; i += kLossThreads) {
    const int r = i / R, c = i - r * R;
    const int gy = reflect_idx(y0 - 2 * HW + r, H), gx = reflect_idx(x0 - 2 * HW + c, W);
    xs[i] = a.pred[poff + size_t(gy) * W + gx];
    ys[i] = a.target[poff + size_t(gy) * W + gx];
  }
  __syncthreads();

  float sum_s = 0.0f;  // a thread's few values in float; the block sums them in double
  if (ssim) {
    // horizontal window sums for input rows r in [0,R), mean columns c in [0,M)
    if (a.box) {
      // Box window: a thread keeps running sums along kBoxRun columns of one row (the sum at
      // column c + 1 is the one at c plus input column c + 2 HW + 1 minus input column c), scaled
      // by the tap when stored; about a third of the per-tap loop's instructions.
      constexpr int kBoxRun = 6;
      constexpr int kRuns = (M + kBoxRun - 1) / kBoxRun;
      const float wk = a.w[0];
      for (int i = tid; i < R * kRuns; i += kLossThreads) {
        const int r = i / kRuns, c0 = (i - r * kRuns) * kBoxRun;
        const float* xr = xs + r * R;
        const float* yr = ys + r * R;
        float s0 = 0, s1 = 0, s2 = 0, s3 = 0, s4 = 0;
#pragma unroll
        for (int k = 0; k <= 2 * HW; ++k) {
          const float x = xr[c0 + k], y = yr[c0 + k];
          s0 += x;
          s1 += y;
          s2 = fmaf(x, x, s2);
          s3 = fmaf(y, y, s3);
          s4 = fmaf(x, y, s4);
        }
        const int c_end = min(c0 + kBoxRun, M);
        for (int c = c0;; ++c) {
          const int o = r * M + c;
          hs[0 * R * M + o] = s0 * wk;
          hs[1 * R * M + o] = s1 * wk;
          hs[2 * R * M + o] = s2 * wk;
          hs[3 * R * M + o] = s3 * wk;
          hs[4 * R * M + o] = s4 * wk;
          if (c + 1 >= c_end) break;
          const float xo = xr[c], yo = yr[c], xi = xr[c + 2 * HW + 1], yi = yr[c + 2 * HW + 1];
          s0 += xi - xo;
          s1 += yi - yo;
          s2 += fmaf(xi, xi, -xo * xo);
          s3 += fmaf(yi, yi, -yo * yo);
          s4 += fmaf(xi, yi, -xo * yo);
        }
      }
    } else
    for (int i = tid; i < R * M; i += kLossThreads) {
      const int r = i / M, c = i - r * M;
      float s0 = 0, s1 = 0, s2 = 0, s3 = 0, s4 = 0;
#pragma unroll
      for (int k = -HW; k <= HW; ++k) {
        const float wk = a.w[k + HW];
        const float x = xs[r * R + c + HW + k], y = ys[r * R + c + HW + k];
        s0 = fmaf(wk, x, s0);
        s1 = fmaf(wk, y, s1);
        s2 = fmaf(wk, x * x, s2);
        s3 = fmaf(wk, y * y, s3);
        s4 = fmaf(wk, x * y, s4);
      }
      hs[0 * R * M + i] = s0;
      hs[1 * R * M + i] = s1;
      hs[2 * R * M + i] = s2;
      hs[3 * R * M + i] = s3;
      hs[4 * R * M + i] = s4;
    }
    __syncthreads();
    // vertical sums -> SSIM map and its derivatives w.r.t. the three prediction moments
    if (a.box) {
      // Box window: a thread keeps the five column sums of kRunV consecutive mean rows as running
      // sums (add the row entering the window, drop the one leaving it).  (Shorter runs, 5 / 4 / 4 / 2
      // in the four passes for about one item per thread, were measured slower: 8 x 1920x1080
      // loss 1.94 -> 2.02 ms.)
      constexpr int kRunV = 6;
      constexpr int kRunsV = (M + kRunV - 1) / kRunV;
      const float wk = a.w[0];
      for (int i = tid; i < M * kRunsV; i += kLossThreads) {
        const int c = i % M, r0 = (i / M) * kRunV;
        const int r_end = min(r0 + kRunV, M);
        float m[5] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int t = 0; t <= 2 * HW; ++t)
#pragma unroll
          for (int q = 0; q < 5; ++q) m[q] += hs[q * R * M + (r0 + t) * M + c];
        for (int r = r0;; ++r) {
          const int gy = y0 - HW + r, gx = x0 - HW + c;
          float d_mx = 0.0f, d_mxx = 0.0f, d_mxy = 0.0f;
          if (gy >= 0 && gy < H && gx >= 0 && gx < W) {
            const float mm[5] = {m[0] * wk, m[1] * wk, m[2] * wk, m[3] * wk, m[4] * wk};
            const float sv = ssim_point(mm, a.c1, a.c2, d_mx, d_mxx, d_mxy);
            if (r >= HW && r < HW + kLossTile && c >= HW && c < HW + kLossTile) sum_s += sv;
          }
          const int o = r * M + c;
          gm[0 * M * M + o] = d_mx;
          gm[1 * M * M + o] = d_mxx;
          gm[2 * M * M + o] = d_mxy;
          if (r + 1 >= r_end) break;
#pragma unroll
          for (int q = 0; q < 5; ++q) m[q] += hs[q * R * M + (r + 2 * HW + 1) * M + c] - hs[q * R * M + r * M + c];
        }
      }
    } else {
      for (int i = tid; i < M * M; i += kLossThreads) {
        const int r = i / M, c = i - r * M;
        const int gy = y0 - HW + r, gx = x0 - HW + c;
        float d_mx = 0.0f, d_mxx = 0.0f, d_mxy = 0.0f;
        if (gy >= 0 && gy < H && gx >= 0 && gx < W) {
          float m[5] = {0, 0, 0, 0, 0};
#pragma unroll
          for (int k = -HW; k <= HW; ++k) {
            const float wk = a.w[k + HW];
            const int row = (r + HW + k) * M + c;
#pragma unroll
            for (int q = 0; q < 5; ++q) m[q] = fmaf(wk, hs[q * R * M + row], m[q]);
          }
          const float sv = ssim_point(m, a.c1, a.c2, d_mx, d_mxx, d_mxy);
          if (r >= HW && r < HW + kLossTile && c >= HW && c < HW + kLossTile) sum_s += sv;
        }
        gm[0 * M * M + i] = d_mx;
        gm[1 * M * M + i] = d_mxx;
        gm[2 * M * M + i] = d_mxy;
      }
    }
    __syncthreads();
    // horizontal adjoint: rows r in [0,M), output columns cq in [0,kLossTile).  The window operator
    // of reflect padding folds the zero-padded window sums at the mirrored positions -q and
    // 2(W-1)-q back onto q; gm is zero off the image, so the direct term needs no bounds and, for
    // the box window, is a running sum along the row.  The mirrored terms exist only within HW of
    // the image's left and right edges.
    auto mirror_h = [&](int r, int qx, float& acc0, float& acc1, float& acc2) {
      const int ms[2] = {(qx >= 1 && qx <= HW) ? -qx : INT32_MIN,
                         (qx >= W - 1 - HW && qx <= W - 2) ? 2 * (W - 1) - qx : INT32_MIN};
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        if (ms[t] == INT32_MIN) continue;
#pragma unroll
        for (int k = -HW; k <= HW; ++k) {
          const int gi = ms[t] + k;
          if (gi < 0 || gi >= W) continue;
          const int col = gi - x0 + HW;
          const float wk = a.w[k + HW];
          acc0 = fmaf(wk, gm[0 * M * M + r * M + col], acc0);
          acc1 = fmaf(wk, gm[1 * M * M + r * M + col], acc1);
          acc2 = fmaf(wk, gm[2 * M * M + r * M + col], acc2);
        }
      }
    };
    if (a.box) {
      constexpr int kRunH = 8;
      constexpr int kRunsH = kLossTile / kRunH;
      const float wk = a.w[0];
      for (int i = tid; i < M * kRunsH; i += kLossThreads) {
        const int r = i / kRunsH, c0 = (i - r * kRunsH) * kRunH;
        const float* q0 = gm + 0 * M * M + r * M;
        const float* q1 = gm + 1 * M * M + r * M;
        const float* q2 = gm + 2 * M * M + r * M;
        float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f;
#pragma unroll
        for (int t = 0; t <= 2 * HW; ++t) s0 += q0[c0 + t], s1 += q1[c0 + t], s2 += q2[c0 + t];
#pragma unroll
        for (int j = 0; j < kRunH; ++j) {
          const int cq = c0 + j, qx = x0 + cq;
          float acc0 = 0.0f, acc1 = 0.0f, acc2 = 0.0f;
          if (qx < W) {
            acc0 = s0 * wk, acc1 = s1 * wk, acc2 = s2 * wk;
            if (qx <= HW || qx >= W - 1 - HW) mirror_h(r, qx, acc0, acc1, acc2);
          }
          const int o = r * kLossTile + cq;
          ha[0 * M * kLossTile + o] = acc0;
          ha[1 * M * kLossTile + o] = acc1;
          ha[2 * M * kLossTile + o] = acc2;
          if (j + 1 < kRunH) {
            s0 += q0[cq + 2 * HW + 1] - q0[cq];
            s1 += q1[cq + 2 * HW + 1] - q1[cq];
            s2 += q2[cq + 2 * HW + 1] - q2[cq];
          }
        }
      }
    } else {
      for (int i = tid; i < M * kLossTile; i += kLossThreads) {
        const int r = i / kLossTile, cq = i - r * kLossTile;
        const int qx = x0 + cq;
        float acc0 = 0, acc1 = 0, acc2 = 0;
        if (qx < W) {
#pragma unroll
          for (int k = -HW; k <= HW; ++k) {
            const int col = cq + HW + k;  // gm is zero off the image
            const float wk = a.w[k + HW];
            acc0 = fmaf(wk, gm[0 * M * M + r * M + col], acc0);
            acc1 = fmaf(wk, gm[1 * M * M + r * M + col], acc1);
            acc2 = fmaf(wk, gm[2 * M * M + r * M + col], acc2);
          }
          mirror_h(r, qx, acc0, acc1, acc2);
        }
        ha[0 * M * kLossTile + i] = acc0;
        ha[1 * M * kLossTile + i] = acc1;
        ha[2 * M * kLossTile + i] = acc2;
      }
    }
    __syncthreads();
  }

  // vertical adjoint + gradient + L1/L2 sums over the output tile: column cq, kRunQ consecutive
  // output rows per thread (running sums of ha down the column for the box window; ha is zero off
  // the image; the mirrored terms only within HW of the top and bottom edges)
  float sum_l1 = 0.0f, sum_l2 = 0.0f;
  constexpr int kRunQ = 4;
  for (int i = tid; i < kLossTile * (kLossTile / kRunQ); i += kLossThreads) {
    const int cq = i % kLossTile, rq0 = (i / kLossTile) * kRunQ;
    const int qx = x0 + cq;
    if (qx >= W) continue;
    const float* h0 = ha + 0 * M * kLossTile + cq;
    const float* h1 = ha + 1 * M * kLossTile + cq;
    const float* h2 = ha + 2 * M * kLossTile + cq;
    float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f;
    if (ssim && a.box && a.dpred) {
#pragma unroll
      for (int t = 0; t <= 2 * HW; ++t)
        s0 += h0[(rq0 + t) * kLossTile], s1 += h1[(rq0 + t) * kLossTile], s2 += h2[(rq0 + t) * kLossTile];
    }
#pragma unroll
    for (int j = 0; j < kRunQ; ++j) {
      const int rq = rq0 + j, qy = y0 + rq;
      if (qy >= H) break;
      const float x = a.pred[poff + size_t(qy) * W + qx];
      const float y = a.target[poff + size_t(qy) * W + qx];
      const float d = x - y;
      sum_l1 += fabsf(d);
      sum_l2 += d * d;
      if (!a.dpred) continue;
      const float sgn = d > 0.0f ? 1.0f : (d < 0.0f ? -1.0f : 0.0f);
      float grad = a.c_l1 * sgn + a.c_mse * 2.0f * d;
      if (ssim) {
        float v0 = 0, v1 = 0, v2 = 0;
        if (a.box) {
          const float wk = a.w[0];
          v0 = s0 * wk, v1 = s1 * wk, v2 = s2 * wk;
          if (j + 1 < kRunQ) {
            const int in = (rq + 2 * HW + 1) * kLossTile, out = rq * kLossTile;
            s0 += h0[in] - h0[out];
            s1 += h1[in] - h1[out];
            s2 += h2[in] - h2[out];
          }
        } else {
#pragma unroll
          for (int k = -HW; k <= HW; ++k) {
            const int row = rq + HW + k;
            const float wk = a.w[k + HW];
            v0 = fmaf(wk, h0[row * kLossTile], v0);
            v1 = fmaf(wk, h1[row * kLossTile], v1);
            v2 = fmaf(wk, h2[row * kLossTile], v2);
          }
        }
        if (qy <= HW || qy >= H - 1 - HW) {
          const int ms[2] = {(qy >= 1 && qy <= HW) ? -qy : INT32_MIN,
                             (qy >= H - 1 - HW && qy <= H - 2) ? 2 * (H - 1) - qy : INT32_MIN};
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            if (ms[t] == INT32_MIN) continue;
#pragma unroll
            for (int k = -HW; k <= HW; ++k) {
              const int gi = ms[t] + k;
              if (gi < 0 || gi >= H) continue;
              const int row = gi - y0 + HW;
              const float wk = a.w[k + HW];
              v0 = fmaf(wk, h0[row * kLossTile], v0);
              v1 = fmaf(wk, h1[row * kLossTile], v1);
              v2 = fmaf(wk, h2[row * kLossTile], v2);
            }
          }
        }
        grad += a.c_ssim * (v0 + 2.0f * x * v1 + y * v2);
      }
      a.dpred[poff + size_t(qy) * W + qx] = grad;
    }
  }

  // block reduction of the three sums, one double atomic per quantity
  const int lane = tid & 31, warp = tid >> 5;
  double v[3] = {double(sum_l1), double(sum_l2), double(sum_s)};
#pragma unroll
  for (int q = 0; q < 3; ++q) {
    for (int o = 16; o > 0; o >>= 1) v[q] += __shfl_down_sync(0xffffffffu, v[q], o);
    if (lane == 0) s_red[q][warp] = v[q];
  }
  __syncthreads();
  if (tid < 3) {
    double t = 0.0;
    for (int w = 0; w < kLossThreads / 32; ++w) t += s_red[tid][w];
    atomicAdd(a.acc + b * 3 + tid, t);
  }
}

struct LossFinish {
  int B;
  int type;
  double n;  // C*H*W
  float l1_weight, dssim_weight, mse_weight;
  int dssim_half;
};

__global__ void loss_finish_kernel(LossFinish f, const double* __restrict__ acc, float* __restrict__ loss,
                                   int32_t* __restrict__ clamp_hit) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= f.B) return;
  const double l1 = acc[b * 3 + 0] / f.n, mse = acc[b * 3 + 1] / f.n, s = acc[b * 3 + 2] / f.n;
  const float l1f = float(l1), msef = float(mse);
  float out;
  int hit = 0;
  switch (f.type) {
    case 1: out = l1f; break;
    case 2: out = msef; break;
    case 3: out = f.l1_weight * l1f + f.mse_weight * msef; break;
    default: {
      const float sf = float(s);
      const float sc = fminf(fmaxf(sf, -1.0f), 1.0f);
      hit = (sf >= -1.0f && sf <= 1.0f) ? 0 : 1;
      out = f.l1_weight * l1f + f.dssim_weight * ((1.0f - sc) * (f.dssim_half ? 0.5f : 1.0f));
    }
  }
  loss[b] = out;
  clamp_hit[b] = hit;
}

// Gradient of an image whose SSIM mean was clamped: the SSIM term contributes nothing.
__global__ void loss_fixup_kernel(int B, int C, int H, int W, float c_l1, const int32_t* __restrict__ clamp_hit,
                                  const float* __restrict__ pred, const float* __restrict__ target,
                                  float* __restrict__ dpred) {
  const size_t per = size_t(C) * H * W;
  const size_t total = per * B;
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < total; i += size_t(gridDim.x) * blockDim.x) {
    if (!clamp_hit[i / per]) continue;
    const float d = pred[i] - target[i];
    dpred[i] = c_l1 * (d > 0.0f ? 1.0f : (d < 0.0f ? -1.0f : 0.0f));
  }
}

// out[b] = scale[b] * in[b]: image blockIdx.y, 16-byte accesses when the planes allow them.
__global__ void scale_planes_kernel(const float* __restrict__ in, const float* __restrict__ scale,
                                    float* __restrict__ out, int64_t per) {
  const int64_t b = blockIdx.y;
  const float s = scale[b];
  const float* src = in + b * per;
  float* dst = out + b * per;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  const int64_t first = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if ((per & 3) == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
    const float4* s4 = reinterpret_cast<const float4*>(src);
    float4* d4 = reinterpret_cast<float4*>(dst);
    for (int64_t i = first; i < per / 4; i += stride) {
      const float4 v = s4[i];
      d4[i] = make_float4(v.x * s, v.y * s, v.z * s, v.w * s);
    }
  } else {
    for (int64_t i = first; i < per; i += stride) dst[i] = src[i] * s;
  }
}

// ---- host ------------------------------------------------------------------------------------

size_t loss_workspace(int32_t n_images) {
  Carver c(nullptr, 0);
  c.take<WorkspaceHeader>(1);
  c.take<double>(size_t(n_images) * 3);
  c.take<int32_t>(n_images);
  return c.used;
}

// Largest grid.z of a launch: image planes beyond it go to further launches of the same kernel.
constexpr int64_t kMaxGridZ = 65535;

template <int HW>
static gsb_status launch_loss_t(const LossArgs& a, cudaStream_t st) {
  const size_t smem = sizeof(float) * size_t(loss_region_a<HW>() + loss_region_b<HW>());
  // The shared-memory opt-in is a per-device function attribute: set once per device.
  static std::mutex mu;
  static bool ready[64] = {};
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    (void)cudaGetLastError();
    return GSB_ERR_CUDA;
  }
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 0 || dev >= 64 || !ready[dev]) {
      if (cudaFuncSetAttribute(loss_kernel<HW>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem))) {
        (void)cudaGetLastError();
        return GSB_ERR_CUDA;
      }
      if (dev >= 0 && dev < 64) ready[dev] = true;
    }
  }
  const int64_t planes = int64_t(a.B) * a.C;
  for (int64_t p0 = 0; p0 < planes; p0 += kMaxGridZ) {
    LossArgs c = a;
    c.plane_base = int(p0);
    const dim3 grid((a.W + kLossTile - 1) / kLossTile, (a.H + kLossTile - 1) / kLossTile,
                    unsigned(std::min(kMaxGridZ, planes - p0)));
    note_launch();
    loss_kernel<HW><<<grid, kLossThreads, smem, st>>>(c);
  }
  return launch_status();
}

gsb_status loss_fwd_bwd(const gsb_loss_options& o, int32_t B, int32_t C, int32_t H, int32_t W, const float* pred,
                        const float* target, float* loss, float* dpred, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (!pred || !target || !loss) return GSB_ERR_ARG;
  if (B <= 0 || C <= 0 || H <= 0 || W <= 0) return GSB_ERR_SHAPE;
  if (int64_t(B) * C > INT32_MAX || (H + kLossTile - 1) / kLossTile > 65535) return GSB_ERR_SHAPE;
  if (o.type < 0 || o.type > 3) return GSB_ERR_ARG;
  const int ws_size = o.window_size;
  const int half = ws_size / 2;
  if (o.type == 0) {
    if (ws_size < 3 || ws_size > 15 || (ws_size % 2) == 0) return GSB_ERR_ARG;
    if (half >= H || half >= W) return GSB_ERR_SHAPE;  // reflect padding needs pad < size
  }
  Carver c(ws, ws_bytes);
  c.take<WorkspaceHeader>(1);
  double* acc = c.take<double>(size_t(B) * 3);
  int32_t* hit = c.take<int32_t>(B);
  if (!c.ok() || !ws) return GSB_ERR_WORKSPACE;
  if (cudaMemsetAsync(acc, 0, size_t(B) * 3 * sizeof(double), st)) return GSB_ERR_CUDA;

  const double n = double(C) * H * W;
  LossArgs a{};
  a.B = B, a.C = C, a.H = H, a.W = W, a.type = o.type, a.c1 = o.c1, a.c2 = o.c2;
  a.c_l1 = (o.type == 0 || o.type == 3) ? float(o.l1_weight / n) : (o.type == 1 ? float(1.0 / n) : 0.0f);
  a.c_mse = o.type == 3 ? float(o.mse_weight / n) : (o.type == 2 ? float(1.0 / n) : 0.0f);
  a.c_ssim = o.type == 0 ? float(-o.dssim_weight * (o.dssim_half ? 0.5 : 1.0) / n) : 0.0f;
  if (o.type == 0) {
    if (o.window == 1) {
      double sum = 0.0, t[16];
      for (int k = -half; k <= half; ++k) sum += t[k + half] = std::exp(-(double(k) * k) / (2.0 * o.sigma * o.sigma));
      for (int k = 0; k < ws_size; ++k) a.w[k] = float(t[k] / sum);
    } else {
      for (int k = 0; k < ws_size; ++k) a.w[k] = 1.0f / float(ws_size);
      a.box = 1;
    }
  }
  a.pred = pred, a.target = target, a.dpred = dpred, a.acc = acc;
  gsb_status s;
  switch (o.type == 0 ? half : 0) {
    case 0: s = launch_loss_t<0>(a, st); break;
    case 1: s = launch_loss_t<1>(a, st); break;
    case 2: s = launch_loss_t<2>(a, st); break;
    case 3: s = launch_loss_t<3>(a, st); break;
    case 4: s = launch_loss_t<4>(a, st); break;
    case 5: s = launch_loss_t<5>(a, st); break;
    case 6: s = launch_loss_t<6>(a, st); break;
    default: s = launch_loss_t<7>(a, st); break;
  }
  if (s != GSB_OK) return s;
  LossFinish f{B, o.type, n, o.l1_weight, o.dssim_weight, o.mse_weight, o.dssim_half};
  note_launch();
  loss_finish_kernel<<<(B + 127) / 128, 128, 0, st>>>(f, acc, loss, hit);
  if (dpred && o.type == 0) {
    const size_t total = size_t(B) * C * H * W;
    const int grid = int(std::min<size_t>((total + 255) / 256, 148u * 16u));
    note_launch();
    loss_fixup_kernel<<<grid, 256, 0, st>>>(B, C, H, W, a.c_l1, hit, pred, target, dpred);
  }
  return launch_status();
}

gsb_status scale_planes(const float* in, const float* scale, float* out, int32_t B, int64_t per, cudaStream_t st) {
  if (!in || !scale || !out || B < 0 || per < 0) return GSB_ERR_ARG;
  const int64_t total = per * B;
  if (total == 0) return GSB_OK;
  if (B > 65535) return GSB_ERR_SHAPE;
  const dim3 grid(unsigned(std::min<int64_t>((per / 4 + 255) / 256 + 1, 64)), unsigned(B));
  note_launch();
  scale_planes_kernel<<<grid, 256, 0, st>>>(in, scale, out, per);
  return launch_status();
}

// ---- allocation-free loss entry ----------------------------------------------------------------
//
// gsb_loss_fwd_bwd needs a small device workspace (three double sums and one flag per image) that
// its caller allocates.  Some callers have no way to allocate device memory: a plugin or binding
// that is handed its input and output buffers by a host framework which owns the device allocator
// and offers no call to obtain more.  For them gsb_loss_fwd_bwd_noalloc keeps that workspace in the
// fixed array below, which is part of the library image: every GPU that loads the library holds it
// (about 112 KiB) until the process exits.  Host code cannot use the array's name as a device
// address (on the host it names a stand-in, not device memory), so the entry point looks the
// address up once per device with cudaGetSymbolAddress, with that device current, and caches it.

constexpr int32_t kNoAllocMaxImages = GSB_LOSS_NOALLOC_MAX_IMAGES;
constexpr size_t kNoAllocAlign = 256;
constexpr size_t noalloc_round(size_t x) { return (x + kNoAllocAlign - 1) / kNoAllocAlign * kNoAllocAlign; }
// Same carving as loss_workspace(): header, per-image double sums, per-image clamp flags.
constexpr size_t kNoAllocBytes = noalloc_round(sizeof(WorkspaceHeader)) +
                                 noalloc_round(size_t(kNoAllocMaxImages) * 3 * sizeof(double)) +
                                 noalloc_round(size_t(kNoAllocMaxImages) * sizeof(int32_t));

static __device__ __align__(256) unsigned char g_loss_scratch[kNoAllocBytes];

constexpr int kNoAllocMaxDevices = 128;
static std::mutex g_loss_scratch_mu;
static void* g_loss_scratch_addr[kNoAllocMaxDevices] = {};

// Device address of g_loss_scratch on the current device (looked up on first use per device).
static gsb_status loss_scratch_address(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) return GSB_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_loss_scratch_mu);
  if (g_loss_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_loss_scratch);
    if (e != cudaSuccess || p == nullptr) return GSB_ERR_CUDA;
    g_loss_scratch_addr[dev] = p;
  }
  *out = g_loss_scratch_addr[dev];
  return GSB_OK;
}

}  // namespace gsb

extern "C" GSB_API gsb_status gsb_loss_fwd_bwd_noalloc(const gsb_loss_options* lopts, int32_t n_images,
                                                       int32_t channels, int32_t height, int32_t width,
                                                       const float* pred, const float* target, float* loss,
                                                       float* dpred, void* stream) {
  using namespace gsb;
  if (!lopts) return GSB_ERR_ARG;
  if (n_images <= 0 || n_images > kNoAllocMaxImages) return GSB_ERR_SHAPE;  // scratch holds at most this many
  if (loss_workspace(n_images) > kNoAllocBytes) return GSB_ERR_WORKSPACE;
  void* scratch = nullptr;
  const gsb_status s = loss_scratch_address(&scratch);
  if (s != GSB_OK) return s;
  // loss_fwd_bwd clears the per-image sums before its kernels run, so nothing carries over
  // from the previous call that used the array.
  return loss_fwd_bwd(*lopts, n_images, channels, height, width, pred, target, loss, dpred, scratch, kNoAllocBytes,
                      static_cast<cudaStream_t>(stream));
}
