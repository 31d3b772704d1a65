// Positional moments (positional_mode "moments", src/gpa/attention.py:277-283, 318-322;
// src/gpa/ops.py:86-132): per level j and unit, the additive state
//   P_t = P_0 + sum_{s <= t} delta_s w_s^T     [D x M],  delta_s = rope(u(k_s), pos_s) - u(k_s)
// (u(k) the level's unit key, w the level's write) is read by the rotated unit query,
// corr_t = q_t^T P_t, and corr enters the level's base logits as g_m tanh(corr / (1 + n)).
// fp32 SIMT kernels shared by both precisions, over the lag-block partition of the call:
//   k_mom_state       CTA per unit, sequential over blocks: P at every block start (saved) and
//                     the final state
//   k_mom_out         CTA per (unit, block): corr = Q P_n + mask(Q Delta^T) W
//   k_mom_grad_state  CTA per unit, reverse: G at every block end, G_end(n) = dP_final +
//                     sum_{tau in later blocks} q_tau dcorr_tau^T, and dP_0
//   k_mom_bwd         CTA per (unit, block): dq, dw and the unit-key gradient through the
//                     rotation (written, for the caller to add after its own writers)
#include "level.cuh"

namespace gpa {
namespace {

GPA_DEV int64_t row(int u, int T, int t) { return (int64_t)u * T + t; }

constexpr int kMomThreads = 256;
constexpr int kMomRows = 64;  // tokens per block (chunk <= 64)

// rows [t0, t0 + c) of the unit key -> delta rows (rope(u) - u) in a [kMomRows x D] tile;
// rows >= c zero.  Pairs (d, d ^ 1) are read by the same thread.
GPA_DEV void delta_tile(float* Dt, const float* nk, int64_t r0, int c, int D, int64_t pos0) {
  for (int i = threadIdx.x; i < kMomRows * (D >> 1); i += blockDim.x) {
    const int t = i / (D >> 1), d = 2 * (i - t * (D >> 1));
    float e = 0.f, o = 0.f;
    if (t < c) {
      e = nk[(r0 + t) * D + d];
      o = nk[(r0 + t) * D + d + 1];
    }
    float cs, sn;
    rope_cs(pos0 + t, d, D, cs, sn);
    Dt[t * D + d] = t < c ? e * cs - o * sn - e : 0.f;
    Dt[t * D + d + 1] = t < c ? e * sn + o * cs - o : 0.f;
  }
}

GPA_DEV void load_rows(float* dst, const float* src, int c, int W) {
  for (int i = threadIdx.x; i < kMomRows * W; i += blockDim.x)
    dst[i] = i / W < c ? src[i] : 0.f;
}

constexpr int kMomRegs = 64;  // P entries per thread: D * M <= 128 * 128 over 256 threads

__global__ void __launch_bounds__(kMomThreads) k_mom_state(int U, Blocks bl, int D, int M,
                                                            int64_t pos0, const float* nk,
                                                            const float* w, const float* P0,
                                                            float* Pb, float* Pout) {
  const int u = blockIdx.x, T = bl.T, DM = D * M;
  extern __shared__ float sm[];
  float* Dt = sm;                     // [64 x D] delta rows
  float* Wt = Dt + kMomRows * D;      // [64 x M] write rows
  float p[kMomRegs];
#pragma unroll
  for (int r = 0; r < kMomRegs; ++r) {
    const int e = threadIdx.x + r * kMomThreads;
    p[r] = e < DM ? P0[(int64_t)u * DM + e] : 0.f;
  }
  for (int n = 0; n < bl.nb; ++n) {
    const int t0 = bl.start(n), c = bl.end(n) - t0;
    const int64_t r0 = row(u, T, t0);
    float* snap = Pb + ((int64_t)u * (bl.nb + 1) + n) * DM;
#pragma unroll
    for (int r = 0; r < kMomRegs; ++r) {
      const int e = threadIdx.x + r * kMomThreads;
      if (e < DM) snap[e] = p[r];
    }
    delta_tile(Dt, nk, r0, c, D, pos0 + t0);
    load_rows(Wt, w + r0 * M, c, M);
    __syncthreads();
#pragma unroll
    for (int r = 0; r < kMomRegs; ++r) {
      const int e = threadIdx.x + r * kMomThreads;
      if (e < DM) {
        const int d = e / M, m = e - d * M;
        float acc = 0.f;
        for (int t = 0; t < c; ++t) acc += Dt[t * D + d] * Wt[t * M + m];
        p[r] += acc;
      }
    }
    __syncthreads();
  }
  float* last = Pb + ((int64_t)u * (bl.nb + 1) + bl.nb) * DM;
#pragma unroll
  for (int r = 0; r < kMomRegs; ++r) {
    const int e = threadIdx.x + r * kMomThreads;
    if (e < DM) {
      last[e] = p[r];
      Pout[(int64_t)u * DM + e] = p[r];
    }
  }
}

// Rows t = tg, tg + nt, ... (< c) of column `col` for thread group tg of nt; at most 32 rows.
constexpr int kMomRowsPerThread = 32;

__global__ void __launch_bounds__(kMomThreads) k_mom_out(int U, Blocks bl, int D, int M,
                                                          int64_t pos0, const float* qh,
                                                          const float* nk, const float* w,
                                                          const float* Pb, float* corr) {
  const int u = blockIdx.x / bl.nb, n = blockIdx.x % bl.nb, T = bl.T;
  const int t0 = bl.start(n), c = bl.end(n) - t0;
  const int64_t r0 = row(u, T, t0);
  extern __shared__ float sm[];
  float* Qt = sm;                       // [64 x D]
  float* Dt = Qt + kMomRows * D;        // [64 x D]
  float* Wt = Dt + kMomRows * D;        // [64 x M]
  float* At = Wt + kMomRows * M;        // [64 x 64]  A[t][s] = q_t . delta_s (s <= t)
  load_rows(Qt, qh + r0 * D, c, D);
  delta_tile(Dt, nk, r0, c, D, pos0 + t0);
  load_rows(Wt, w + r0 * M, c, M);
  __syncthreads();
  for (int i = threadIdx.x; i < kMomRows * kMomRows; i += blockDim.x) {
    const int t = i / kMomRows, s = i - t * kMomRows;
    float a = 0.f;
    if (s <= t && t < c)
      for (int d = 0; d < D; ++d) a += Qt[t * D + d] * Dt[s * D + d];
    At[i] = a;
  }
  __syncthreads();
  const float* P = Pb + ((int64_t)u * (bl.nb + 1) + n) * D * M;
  const int nt = blockDim.x / M, m = threadIdx.x % M, tg = threadIdx.x / M;
  if (tg >= nt) return;
  float acc[kMomRowsPerThread];
#pragma unroll
  for (int k = 0; k < kMomRowsPerThread; ++k) acc[k] = 0.f;
  for (int d = 0; d < D; ++d) {
    const float pv = P[d * M + m];
#pragma unroll
    for (int k = 0; k < kMomRowsPerThread; ++k) {
      const int t = tg + k * nt;
      if (t < c) acc[k] += Qt[t * D + d] * pv;
    }
  }
  for (int s = 0; s < c; ++s) {
    const float wv = Wt[s * M + m];
#pragma unroll
    for (int k = 0; k < kMomRowsPerThread; ++k) {
      const int t = tg + k * nt;
      if (t < c) acc[k] += At[t * kMomRows + s] * wv;
    }
  }
#pragma unroll
  for (int k = 0; k < kMomRowsPerThread; ++k) {
    const int t = tg + k * nt;
    if (t < c) corr[(r0 + t) * M + m] = acc[k];
  }
}

// Reverse over blocks: G_end(n) = dP_final + sum over later blocks of Q^T dcorr (saved per
// block) and dP_0 = G_end(-1).  P-sized accumulator in registers, as in k_mom_state.
__global__ void __launch_bounds__(kMomThreads) k_mom_grad_state(int U, Blocks bl, int D, int M,
                                                                 const float* qh,
                                                                 const float* dcorr,
                                                                 const float* dPfinal,
                                                                 float* Gend, float* dP0) {
  const int u = blockIdx.x, T = bl.T, DM = D * M;
  extern __shared__ float sm[];
  float* Qt = sm;                   // [64 x D]
  float* Ct = Qt + kMomRows * D;    // [64 x M]
  float g[kMomRegs];
#pragma unroll
  for (int r = 0; r < kMomRegs; ++r) {
    const int e = threadIdx.x + r * kMomThreads;
    g[r] = e < DM && dPfinal ? dPfinal[(int64_t)u * DM + e] : 0.f;
  }
  for (int n = bl.nb - 1; n >= 0; --n) {
    const int t0 = bl.start(n), c = bl.end(n) - t0;
    const int64_t r0 = row(u, T, t0);
    float* snap = Gend + ((int64_t)u * bl.nb + n) * DM;
#pragma unroll
    for (int r = 0; r < kMomRegs; ++r) {
      const int e = threadIdx.x + r * kMomThreads;
      if (e < DM) snap[e] = g[r];
    }
    load_rows(Qt, qh + r0 * D, c, D);
    load_rows(Ct, dcorr + r0 * M, c, M);
    __syncthreads();
#pragma unroll
    for (int r = 0; r < kMomRegs; ++r) {
      const int e = threadIdx.x + r * kMomThreads;
      if (e < DM) {
        const int d = e / M, m = e - d * M;
        float acc = 0.f;
        for (int t = 0; t < c; ++t) acc += Qt[t * D + d] * Ct[t * M + m];
        g[r] += acc;
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < kMomRegs; ++r) {
    const int e = threadIdx.x + r * kMomThreads;
    if (e < DM) dP0[(int64_t)u * DM + e] = g[r];
  }
}

// Per block, with P_n the state at its start, G the gradient at its end,
// E[t][s] = w_s . dcorr_t and A[t][s] = q_t . delta_s (s <= t):
//   dq_t     = P_n dcorr_t + sum_{s <= t} E[t][s] delta_s              (added into dq)
//   ddelta_s = G w_s + sum_{tau >= s} E[tau][s] q_tau                  -> dkey = R^T ddelta - ddelta
//   dw_s     = G^T delta_s + sum_{tau >= s} A[tau][s] dcorr_tau        (added into dw)
__global__ void __launch_bounds__(kMomThreads) k_mom_bwd(int U, Blocks bl, int D, int M,
                                                          int64_t pos0, const float* qh,
                                                          const float* nk, const float* w,
                                                          const float* Pb, const float* dcorr,
                                                          const float* Gend, float* dq,
                                                          float* dw, float* dkey) {
  const int u = blockIdx.x / bl.nb, n = blockIdx.x % bl.nb, T = bl.T;
  const int t0 = bl.start(n), c = bl.end(n) - t0;
  const int64_t r0 = row(u, T, t0);
  extern __shared__ float sm[];
  float* Qt = sm;                       // [64 x D]
  float* Dt = Qt + kMomRows * D;        // [64 x D]
  float* Wt = Dt + kMomRows * D;        // [64 x M]
  float* Ct = Wt + kMomRows * M;        // [64 x M] dcorr rows
  float* At = Ct + kMomRows * M;        // [64 x 64]
  float* Et = At + kMomRows * kMomRows; // [64 x 64]
  load_rows(Qt, qh + r0 * D, c, D);
  delta_tile(Dt, nk, r0, c, D, pos0 + t0);
  load_rows(Wt, w + r0 * M, c, M);
  load_rows(Ct, dcorr + r0 * M, c, M);
  __syncthreads();
  for (int i = threadIdx.x; i < kMomRows * kMomRows; i += blockDim.x) {
    const int t = i / kMomRows, s = i - t * kMomRows;
    float a = 0.f, e = 0.f;
    if (s <= t && t < c) {
      for (int d = 0; d < D; ++d) a += Qt[t * D + d] * Dt[s * D + d];
      for (int m = 0; m < M; ++m) e += Wt[s * M + m] * Ct[t * M + m];
    }
    At[i] = a;
    Et[i] = e;
  }
  __syncthreads();
  const float* P = Pb + ((int64_t)u * (bl.nb + 1) + n) * D * M;
  const float* G = Gend + ((int64_t)u * bl.nb + n) * D * M;
  {  // dq and ddelta: column d of a thread group, rows t = tg + k nt
    const int nt = blockDim.x / D, d = threadIdx.x % D, tg = threadIdx.x / D;
    const bool live = tg < nt;
    float aq[kMomRowsPerThread], ad[kMomRowsPerThread];
#pragma unroll
    for (int k = 0; k < kMomRowsPerThread; ++k) aq[k] = ad[k] = 0.f;
    if (live) {
      for (int m = 0; m < M; ++m) {
        const float pv = P[d * M + m], gv = G[d * M + m];
#pragma unroll
        for (int k = 0; k < kMomRowsPerThread; ++k) {
          const int t = tg + k * nt;
          if (t < c) {
            aq[k] += pv * Ct[t * M + m];
            ad[k] += gv * Wt[t * M + m];
          }
        }
      }
      for (int s = 0; s < c; ++s) {
        const float ds_ = Dt[s * D + d], qs = Qt[s * D + d];
#pragma unroll
        for (int k = 0; k < kMomRowsPerThread; ++k) {
          const int t = tg + k * nt;
          if (t < c) {
            if (s <= t) aq[k] += Et[t * kMomRows + s] * ds_;  // dq_t += E[t][s] delta_s
            if (s >= t) ad[k] += Et[s * kMomRows + t] * qs;   // ddelta_t += E[s][t] q_s
          }
        }
      }
    }
    // dkey = R^T ddelta - ddelta; the pair partner d ^ 1 is thread threadIdx.x ^ 1 (D even)
#pragma unroll
    for (int k = 0; k < kMomRowsPerThread; ++k) {
      const int t = tg + k * nt;
      const float other = __shfl_xor_sync(0xffffffffu, ad[k], 1);
      if (live && t < c) {
        const int64_t o = (r0 + t) * D + d;
        dq[o] += aq[k];
        float cs, sn;
        rope_cs(pos0 + t0 + t, d, D, cs, sn);
        // forward: e' = e c - o s, o' = e s + o c  ->  de = c de' + s do', do = -s de' + c do'
        const float rt = (d & 1) == 0 ? cs * ad[k] + sn * other : -sn * other + cs * ad[k];
        dkey[o] = rt - ad[k];
      }
    }
  }
  {  // dw: column m of a thread group, rows s = tg + k nt
    const int nt = blockDim.x / M, m = threadIdx.x % M, tg = threadIdx.x / M;
    if (tg >= nt) return;
    float aw[kMomRowsPerThread];
#pragma unroll
    for (int k = 0; k < kMomRowsPerThread; ++k) aw[k] = 0.f;
    for (int d = 0; d < D; ++d) {
      const float gv = G[d * M + m];
#pragma unroll
      for (int k = 0; k < kMomRowsPerThread; ++k) {
        const int s = tg + k * nt;
        if (s < c) aw[k] += gv * Dt[s * D + d];
      }
    }
    for (int tau = 0; tau < c; ++tau) {
      const float cv = Ct[tau * M + m];
#pragma unroll
      for (int k = 0; k < kMomRowsPerThread; ++k) {
        const int s = tg + k * nt;
        if (s < c && tau >= s) aw[k] += At[tau * kMomRows + s] * cv;
      }
    }
#pragma unroll
    for (int k = 0; k < kMomRowsPerThread; ++k) {
      const int s = tg + k * nt;
      if (s < c) dw[(r0 + s) * M + m] += aw[k];
    }
  }
}

size_t mom_state_smem(int D, int M) { return 4 * (size_t)kMomRows * (D + M); }
size_t mom_out_smem(int D, int M) {
  return 4 * ((size_t)kMomRows * (2 * D + M) + (size_t)kMomRows * kMomRows);
}
size_t mom_bwd_smem(int D, int M) {
  return 4 * ((size_t)kMomRows * (2 * D + 2 * M) + 2 * (size_t)kMomRows * kMomRows);
}

template <class K>
cudaError_t mom_launch(const char* name, K kern, int grid, size_t smem, cudaStream_t st,
                       auto&&... args) {
  if (smem > 227 * 1024) return cudaErrorInvalidConfiguration;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  Launch scope_(name, st);
  kern<<<grid, kMomThreads, smem, st>>>(args...);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_moments_fwd(int U, const Blocks& bl, int D, int M, int64_t pos0,
                               const float* qh, const float* nk, const float* w, const float* P0,
                               float* Pb, float* corr, float* Pout, cudaStream_t st) {
  if (!U || !bl.T) return cudaSuccess;
  cudaError_t e = mom_launch("mom_state", k_mom_state, U, mom_state_smem(D, M), st, U, bl, D, M,
                             pos0, nk, w, P0, Pb, Pout);
  if (e != cudaSuccess) return e;
  return mom_launch("mom_out", k_mom_out, U * bl.nb, mom_out_smem(D, M), st, U, bl, D, M, pos0,
                    qh, nk, w, Pb, corr);
}

cudaError_t launch_moments_bwd(int U, const Blocks& bl, int D, int M, int64_t pos0,
                               const float* qh, const float* nk, const float* w, const float* Pb,
                               const float* dcorr, const float* dPfinal, float* Gend, float* dP0,
                               float* dq, float* dw, float* dkey, cudaStream_t st) {
  if (!U || !bl.T) return cudaSuccess;
  cudaError_t e = mom_launch("mom_grad_state", k_mom_grad_state, U, mom_state_smem(D, M), st, U,
                             bl, D, M, qh, dcorr, dPfinal, Gend, dP0);
  if (e != cudaSuccess) return e;
  return mom_launch("mom_bwd", k_mom_bwd, U * bl.nb, mom_bwd_smem(D, M), st, U, bl, D, M, pos0,
                    qh, nk, w, Pb, dcorr, Gend, dq, dw, dkey);
}

}  // namespace gpa
