// Shared device helpers for the DenseGPA b200 kernels (sm_100a).
//
// Conventions used by every kernel in this library:
//  * "unit" u = b * H + h indexes one independent (batch, head) recurrence.
//  * Internal activations are fp32, unit-major: row (u, t) of an [U, T, X]
//    buffer starts at ((u * T) + t) * X.  Chunk tiles are therefore contiguous.
//  * Key-major states: S[K][V] row-major, matching GPAState's inner [D, M],
//    outer [M, Dv] and relation [M_i, M_j] layouts.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#define GPA_DEV __device__ __forceinline__

namespace gpa {

constexpr int kMaxChunk = 64;
constexpr float kUnitEps = 1e-6f;      // F.normalize eps (src/gpa/ops.py:17)
constexpr float kCenterEps = 1e-5f;    // centred-variance eps (src/gpa/attention.py:240)

enum InputDType : int { kF32 = 0, kBF16 = 1, kF16 = 2 };

GPA_DEV float load_in(const void* p, int64_t i, int dt) {
  if (dt == kBF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dt == kF16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

GPA_DEV void store_out(void* p, int64_t i, float x, int dt) {
  if (dt == kBF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16(x);
  else if (dt == kF16) reinterpret_cast<__half*>(p)[i] = __float2half(x);
  else reinterpret_cast<float*>(p)[i] = x;
}

GPA_DEV float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

GPA_DEV float warp_max(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}

GPA_DEV float softplus(float x) {
  // torch.nn.functional.softplus (beta=1, threshold=20)
  return x > 20.f ? x : log1pf(expf(x));
}

GPA_DEV float sigmoid(float x) { return 1.f / (1.f + expf(-x)); }

// exact-erf GELU and its derivative (F.gelu default, src/gpa/attention.py:243)
GPA_DEV float gelu(float x) { return 0.5f * x * (1.f + erff(x * 0.70710678118654752f)); }
GPA_DEV float gelu_grad(float x) {
  return 0.5f * (1.f + erff(x * 0.70710678118654752f)) +
         x * expf(-0.5f * x * x) * 0.39894228040143268f;
}

// Block-wide SIMT GEMM over shared (or global) operands described by accessors.
//   for every (i, j) in [0,m) x [0,n):  epi(i, j, sum_k a(i, k) * b(k, j))
// Each thread owns TM x TN register tiles; tiles are strided over the block.
template <int TM, int TN, class FA, class FB, class EPI>
GPA_DEV void block_gemm(int m, int n, int k, FA a, FB b, EPI epi) {
  const int tn = (n + TN - 1) / TN, tm = (m + TM - 1) / TM;
  for (int tile = threadIdx.x; tile < tm * tn; tile += blockDim.x) {
    const int i0 = (tile / tn) * TM, j0 = (tile % tn) * TN;
    float acc[TM][TN];
#pragma unroll
    for (int r = 0; r < TM; ++r)
#pragma unroll
      for (int c = 0; c < TN; ++c) acc[r][c] = 0.f;
    for (int kk = 0; kk < k; ++kk) {
      float av[TM], bv[TN];
#pragma unroll
      for (int r = 0; r < TM; ++r) av[r] = (i0 + r < m) ? a(i0 + r, kk) : 0.f;
#pragma unroll
      for (int c = 0; c < TN; ++c) bv[c] = (j0 + c < n) ? b(kk, j0 + c) : 0.f;
#pragma unroll
      for (int r = 0; r < TM; ++r)
#pragma unroll
        for (int c = 0; c < TN; ++c) acc[r][c] = fmaf(av[r], bv[c], acc[r][c]);
    }
#pragma unroll
    for (int r = 0; r < TM; ++r)
#pragma unroll
      for (int c = 0; c < TN; ++c)
        if (i0 + r < m && j0 + c < n) epi(i0 + r, j0 + c, acc[r][c]);
  }
}

// Cooperative copy of a dense row-major [rows x cols] fp32 tile (global -> shared).
GPA_DEV void load_tile(float* dst, const float* src, int rows, int cols, int src_ld) {
  const int n = rows * cols;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int r = i / cols, c = i - r * cols;
    dst[i] = src[(int64_t)r * src_ld + c];
  }
}

GPA_DEV void store_tile(float* dst, const float* src, int rows, int cols, int dst_ld) {
  const int n = rows * cols;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int r = i / cols, c = i - r * cols;
    dst[(int64_t)r * dst_ld + c] = src[i];
  }
}

// Lag-block geometry.  The first block of a call resumes a partially filled
// block: it holds chunk - offset tokens (src/gpa/attention.py:397); the rest
// hold chunk tokens; the last may be partial.  Block n of the GDN scans is
// exactly lag block n, so boundary state n is the state at its start.
struct Blocks {
  int T, C, first, nb;
  __host__ __device__ int start(int n) const { return n == 0 ? 0 : first + (n - 1) * C; }
  __host__ __device__ int end(int n) const {
    const int e = first + n * C;
    return e < T ? e : T;
  }
  __host__ __device__ int block_of(int t) const { return t < first ? 0 : 1 + (t - first) / C; }
};

// Kernel accounting: every launch in this library is bracketed by a Launch
// scope.  It always counts launches; when profiling is on (off by default, so
// graph capture sees no extra nodes) it records CUDA events on the launch
// stream and accumulates per-kernel device time.
struct Launch {
  Launch(const char* name, cudaStream_t st);
  ~Launch();
  int slot;
  cudaStream_t st;
};

inline Blocks make_blocks(int T, int C, int offset) {
  Blocks b;
  b.T = T;
  b.C = C;
  b.first = (C - offset) < T ? (C - offset) : T;
  b.nb = T == 0 ? 0 : 1 + (T - b.first + C - 1) / C;
  return b;
}

}  // namespace gpa
