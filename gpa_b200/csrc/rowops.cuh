// Per-row (one warp per token row) helpers of the level kernels: vectors of up
// to 256 values held lane-strided in registers.
#pragma once
#include "level.cuh"

namespace gpa {
namespace {

constexpr int kRowsPerTile = 64;
constexpr int kMaxPerLane = 8;  // vectors up to 256 long per warp row

GPA_DEV int64_t row(int u, int T, int t) { return (int64_t)u * T + t; }

// softmax over the lane-strided vector x[0..n) held in registers
template <int N>
GPA_DEV void warp_softmax(float (&x)[N], int n) {
  const int lane = threadIdx.x & 31;
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < N; ++i)
    if (lane + 32 * i < n) mx = fmaxf(mx, x[i]);
  mx = warp_max(mx);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < N; ++i)
    if (lane + 32 * i < n) {
      x[i] = __expf(x[i] - mx);
      s += x[i];
    }
  s = warp_sum(s);
  const float inv = 1.f / s;
#pragma unroll
  for (int i = 0; i < N; ++i)
    if (lane + 32 * i < n) x[i] *= inv;
}

template <int N>
GPA_DEV float warp_norm(const float (&x)[N], int n) {
  const int lane = threadIdx.x & 31;
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < N; ++i)
    if (lane + 32 * i < n) s += x[i] * x[i];
  return sqrtf(warp_sum(s));
}

template <int N>
GPA_DEV float warp_dot(const float (&x)[N], const float (&y)[N], int n) {
  const int lane = threadIdx.x & 31;
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < N; ++i)
    if (lane + 32 * i < n) s += x[i] * y[i];
  return warp_sum(s);
}

template <int N>
GPA_DEV void load_vec(float (&x)[N], const float* p, int n) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < N; ++i) x[i] = lane + 32 * i < n ? p[lane + 32 * i] : 0.f;
}

template <int N>
GPA_DEV void store_vec(float* p, const float (&x)[N], int n) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < N; ++i)
    if (lane + 32 * i < n) p[lane + 32 * i] = x[i];
}

// unit-normalisation backward: y = x / max(|x|, eps)
template <int N>
GPA_DEV void unit_bwd(float (&dx)[N], const float (&y)[N], const float (&dy)[N], float nrm,
                      int n) {
  if (nrm > kUnitEps) {
    const float yd = warp_dot(y, dy, n);
    const float inv = 1.f / nrm;
#pragma unroll
    for (int i = 0; i < N; ++i) dx[i] = (dy[i] - y[i] * yd) * inv;
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) dx[i] = dy[i] / kUnitEps;
  }
}

template <int N>
GPA_DEV void softmax_bwd(float (&dx)[N], const float (&y)[N], const float (&dy)[N], int n) {
  const float yd = warp_dot(y, dy, n);
#pragma unroll
  for (int i = 0; i < N; ++i) dx[i] = y[i] * (dy[i] - yd);
}

GPA_DEV float block_sum(float x, float* red) {
  x = warp_sum(x);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = x;
  __syncthreads();
  float s = 0.f;
  if (threadIdx.x < 32) {
    s = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    s = warp_sum(s);
  }
  return s;  // valid in warp 0
}

// softmax over the incoming edges' logits for head h
// The product reader's gain e^{clamp(g, -4, 4)} and whether g lies inside the clamp
// (src/gpa/attention.py:234)
GPA_DEV float product_gain(float g) { return __expf(fminf(fmaxf(g, -4.f), 4.f)); }
GPA_DEV float product_gain_live(float g) { return g >= -4.f && g <= 4.f ? 1.f : 0.f; }

GPA_DEV void edge_weights(const BridgeIn& in, const float* edge_logits, int H, int h,
                          float* w) {
  float mx = -INFINITY;
  for (int a = 0; a < in.n; ++a) mx = fmaxf(mx, edge_logits[in.edge[a] * H + h]);
  float s = 0.f;
  for (int a = 0; a < in.n; ++a) {
    w[a] = __expf(edge_logits[in.edge[a] * H + h] - mx);
    s += w[a];
  }
  for (int a = 0; a < in.n; ++a) w[a] /= s;
}

}  // namespace
}  // namespace gpa
