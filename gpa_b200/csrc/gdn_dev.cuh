// Device helpers shared by the SIMT (gdn.cu) and tensor-core (gdn_tc.cu) GDN kernels.
#pragma once
#include "gdn.cuh"

namespace gpa {
namespace {

GPA_DEV int64_t row(int u, int T, int t) { return (int64_t)u * T + t; }

GPA_DEV float gate_at(const float* p, const ScanDesc& d, int u, int t) {
  return p[(int64_t)u * d.g_su + (int64_t)t * d.g_st];
}

// G[t] = inclusive cumsum of g over the block; bt[t] = beta.
GPA_DEV void load_gates(const ScanDesc& d, int u, int t0, int c, float* G, float* bt) {
  if (threadIdx.x < 32) {
    float carry = 0.f;
    for (int base = 0; base < c; base += 32) {
      const int t = base + threadIdx.x;
      float x = t < c ? gate_at(d.g, d, u, t0 + t) : 0.f;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, x, o);
        if ((int)threadIdx.x >= o) x += y;
      }
      if (t < c) {
        G[t] = x + carry;
        if (bt) bt[t] = gate_at(d.beta, d, u, t0 + t);
      }
      carry += __shfl_sync(0xffffffffu, x, 31);
    }
  }
}

// A[t][s] = b_t exp(G_t - G_s) k_t.k_s for s < t (0 elsewhere); Atil without b_t.
GPA_DEV void build_a(const float* Ks, int K, int c, const float* G, const float* bt, float* A,
                     float* Atil) {
  block_gemm<2, 2>(
      c, c, K, [&](int t, int kk) { return Ks[t * K + kk]; },
      [&](int kk, int s) { return Ks[s * K + kk]; },
      [&](int t, int s, float acc) {
        const float at = s < t ? __expf(G[t] - G[s]) * acc : 0.f;
        if (Atil) Atil[t * kAStride + s] = at;
        A[t * kAStride + s] = bt[t] * at;
      });
}

// In place: X <- (I + A)^-1 X for X [c x ncol] with row stride ld (A strictly lower).
GPA_DEV void forward_subst(const float* A, float* X, int c, int ncol, int ld) {
  for (int col = threadIdx.x; col < ncol; col += blockDim.x) {
    for (int t = 1; t < c; ++t) {
      const float* a = A + t * kAStride;
      float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
      int s = 0;
      for (; s + 3 < t; s += 4) {
        s0 = fmaf(a[s], X[s * ld + col], s0);
        s1 = fmaf(a[s + 1], X[(s + 1) * ld + col], s1);
        s2 = fmaf(a[s + 2], X[(s + 2) * ld + col], s2);
        s3 = fmaf(a[s + 3], X[(s + 3) * ld + col], s3);
      }
      for (; s < t; ++s) s0 = fmaf(a[s], X[s * ld + col], s0);
      X[t * ld + col] -= (s0 + s1) + (s2 + s3);
    }
  }
}

// In place: Y <- (I + A)^-T Y (back substitution, A strictly lower).
GPA_DEV void backward_subst(const float* A, float* Y, int c, int ncol, int ld) {
  for (int col = threadIdx.x; col < ncol; col += blockDim.x) {
    for (int t = c - 2; t >= 0; --t) {
      float s0 = 0.f, s1 = 0.f;
      int s = t + 1;
      for (; s + 1 < c; s += 2) {
        s0 = fmaf(A[s * kAStride + t], Y[s * ld + col], s0);
        s1 = fmaf(A[(s + 1) * kAStride + t], Y[(s + 1) * ld + col], s1);
      }
      for (; s < c; ++s) s0 = fmaf(A[s * kAStride + t], Y[s * ld + col], s0);
      Y[t * ld + col] -= s0 + s1;
    }
  }
}

// T = (I + A)^-1 for a strictly lower 64x64 A (row stride kAStride), into Tm (same stride).
GPA_DEV void invert_unit_lower(const float* A, float* Tm) {
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < kMaxChunk * kAStride; i += blockDim.x) Tm[i] = 0.f;
  __syncthreads();
  if (w < 4 && lane < 16) {
    const int b0 = 16 * w, j = lane;
    float x[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      float s = (r == j) ? 1.f : 0.f;
#pragma unroll
      for (int q = 0; q < r; ++q) s -= A[(b0 + r) * kAStride + b0 + q] * x[q];
      x[r] = s;
    }
#pragma unroll
    for (int r = 0; r < 16; ++r) Tm[(b0 + r) * kAStride + b0 + j] = x[r];
  }
  __syncthreads();
  // Off-diagonal 16 x 16 blocks by distance dd = ib - jb: X = sum_{jb <= kb < ib}
  // A[ib][kb] T[kb][jb], then T[ib][jb] = -T[ib][ib] X.  One warp owns block (ib, jb) for both
  // products, so X is parked in that block of Tm (which nothing else reads during step dd)
  // between two warp barriers.  A lane computes rows r and r + 8, columns c .. c + 3 of a
  // block: 6 shared loads per 8 FMAs.
  for (int dd = 1; dd < 4; ++dd) {
    const int nblk = 4 - dd;
    if (w < nblk) {
      const int jb = w, ib = jb + dd, r = lane >> 2, c = (lane & 3) << 2;
      float* blk = Tm + (16 * ib) * kAStride + 16 * jb;  // block (ib, jb)
      float x[2][4] = {};
      for (int kb = jb; kb < ib; ++kb) {
        const float* a0 = A + (16 * ib + r) * kAStride + 16 * kb;
        const float* t = Tm + (16 * kb) * kAStride + 16 * jb + c;
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const float u0 = a0[q], u1 = a0[8 * kAStride + q];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float tv = t[q * kAStride + k];
            x[0][k] = fmaf(u0, tv, x[0][k]);
            x[1][k] = fmaf(u1, tv, x[1][k]);
          }
        }
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        blk[r * kAStride + c + k] = x[0][k];
        blk[(r + 8) * kAStride + c + k] = x[1][k];
      }
      __syncwarp();
      const float* d0 = Tm + (16 * ib + r) * kAStride + 16 * ib;
      float y[2][4] = {};
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        const float u0 = d0[q], u1 = d0[8 * kAStride + q];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float xv = blk[q * kAStride + c + k];
          y[0][k] = fmaf(u0, xv, y[0][k]);
          y[1][k] = fmaf(u1, xv, y[1][k]);
        }
      }
      __syncwarp();
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        blk[r * kAStride + c + k] = -y[0][k];
        blk[(r + 8) * kAStride + c + k] = -y[1][k];
      }
    }
    __syncthreads();
  }
}

}  // namespace
}  // namespace gpa
