// Chunked GDN scan kernels (see gdn.cuh for the math and the kernel list).
#include "gdn.cuh"
#include "gdn_dev.cuh"

namespace gpa {
namespace {

// ------------------------------------------------------------------ forward

// grid (U*NB, nscan). U and Wk of every block.
__global__ void __launch_bounds__(256) gdn_fwd_chunk_kernel(ScanBatch b, int U, Blocks bl) {
  const ScanDesc& d = b.s[blockIdx.y];
  const int u = blockIdx.x / bl.nb, n = blockIdx.x % bl.nb;
  const int t0 = bl.start(n), c = bl.end(n) - t0, T = bl.T;
  const int K = d.K, V = d.V, ldx = V + K;
  extern __shared__ float sm[];
  float* Ks = sm;                        // 64*K
  float* X = Ks + kMaxChunk * K;         // 64*(V+K)
  float* A = X + kMaxChunk * ldx;        // 64*65
  float* G = A + kMaxChunk * kAStride;   // 64
  float* bt = G + kMaxChunk;             // 64
  load_tile(Ks, d.k + row(u, T, t0) * K, c, K, K);
  load_gates(d, u, t0, c, G, bt);
  __syncthreads();
  for (int i = threadIdx.x; i < c * ldx; i += blockDim.x) {
    const int t = i / ldx, col = i - t * ldx;
    X[i] = col < V ? bt[t] * d.v[row(u, T, t0 + t) * V + col]
                   : bt[t] * __expf(G[t]) * Ks[t * K + (col - V)];
  }
  build_a(Ks, K, c, G, bt, A, nullptr);
  __syncthreads();
  forward_subst(A, X, c, ldx, ldx);
  __syncthreads();
  for (int i = threadIdx.x; i < c * ldx; i += blockDim.x) {
    const int t = i / ldx, col = i - t * ldx;
    if (col < V) d.Ub[row(u, T, t0 + t) * V + col] = X[i];
    else d.Wk[row(u, T, t0 + t) * K + (col - V)] = X[i];
  }
}

// grid (U*nvs, nscan). Sequential over blocks; state slice [K x VS] in shared memory.
__global__ void __launch_bounds__(256) gdn_fwd_state_kernel(ScanBatch b, int U, Blocks bl) {
  const ScanDesc& d = b.s[blockIdx.y];
  const int K = d.K, V = d.V, T = bl.T;
  const int nvs = (V + kVSlice - 1) / kVSlice;
  if ((int)blockIdx.x >= U * nvs) return;
  const int u = blockIdx.x / nvs, v0 = (blockIdx.x % nvs) * kVSlice;
  const int vw = min(kVSlice, V - v0);
  extern __shared__ float sm[];
  float* S = sm;                          // K*VS
  float* Wks = S + K * kVSlice;           // 64*K
  float* Ks = Wks + kMaxChunk * K;        // 64*K
  float* Wc = Ks + kMaxChunk * K;         // 64*VS
  float* G = Wc + kMaxChunk * kVSlice;    // 64
  for (int i = threadIdx.x; i < K * vw; i += blockDim.x) {
    const int k = i / vw, v = i - k * vw;
    S[k * kVSlice + v] = d.S0[((int64_t)u * K + k) * V + v0 + v];
  }
  __syncthreads();
  for (int n = 0; n < bl.nb; ++n) {
    const int t0 = bl.start(n), c = bl.end(n) - t0;
    float* sb = d.Sb + ((int64_t)u * (bl.nb + 1) + n) * K * V;
    for (int i = threadIdx.x; i < K * vw; i += blockDim.x) {
      const int k = i / vw, v = i - k * vw;
      sb[k * V + v0 + v] = S[k * kVSlice + v];
    }
    load_tile(Wks, d.Wk + row(u, T, t0) * K, c, K, K);
    load_tile(Ks, d.k + row(u, T, t0) * K, c, K, K);
    for (int i = threadIdx.x; i < c * vw; i += blockDim.x) {
      const int t = i / vw, v = i - t * vw;
      Wc[t * kVSlice + v] = d.Ub[row(u, T, t0 + t) * V + v0 + v];
    }
    load_gates(d, u, t0, c, G, nullptr);
    __syncthreads();
    // W = U - Wk S
    block_gemm<2, 4>(
        c, vw, K, [&](int t, int kk) { return Wks[t * K + kk]; },
        [&](int kk, int v) { return S[kk * kVSlice + v]; },
        [&](int t, int v, float acc) {
          const float w = Wc[t * kVSlice + v] - acc;
          d.W[row(u, T, t0 + t) * V + v0 + v] = w;
          Wc[t * kVSlice + v] = w * __expf(G[c - 1] - G[t]);
        });
    __syncthreads();
    const float gc = __expf(G[c - 1]);
    // S = e^{G_c} S + K^T diag(lambda) W
    block_gemm<2, 4>(
        K, vw, c, [&](int k, int t) { return Ks[t * K + k]; },
        [&](int t, int v) { return Wc[t * kVSlice + v]; },
        [&](int k, int v, float acc) { S[k * kVSlice + v] = fmaf(gc, S[k * kVSlice + v], acc); });
    __syncthreads();
  }
  float* sb = d.Sb + ((int64_t)u * (bl.nb + 1) + bl.nb) * K * V;
  for (int i = threadIdx.x; i < K * vw; i += blockDim.x) {
    const int k = i / vw, v = i - k * vw;
    sb[k * V + v0 + v] = S[k * kVSlice + v];
    if (d.S_final) d.S_final[((int64_t)u * K + k) * V + v0 + v] = S[k * kVSlice + v];
  }
}

// grid (U*NB*nvs, nscan).  O = e^G (Q S_n) + (Q K^T o Gamma) W.
__global__ void __launch_bounds__(256) gdn_fwd_out_kernel(ScanBatch b, int U, Blocks bl) {
  const ScanDesc& d = b.s[blockIdx.y];
  const int K = d.K, V = d.V, T = bl.T;
  const int nvs = (V + kVSlice - 1) / kVSlice;
  if ((int)blockIdx.x >= U * bl.nb * nvs || !d.q || !d.O) return;
  const int vs = blockIdx.x % nvs, un = blockIdx.x / nvs;
  const int u = un / bl.nb, n = un % bl.nb;
  const int v0 = vs * kVSlice, vw = min(kVSlice, V - v0);
  const int t0 = bl.start(n), c = bl.end(n) - t0;
  extern __shared__ float sm[];
  float* Qs = sm;                          // 64*K
  float* Ks = Qs + kMaxChunk * K;          // 64*K
  float* Ss = Ks + kMaxChunk * K;          // K*VS
  float* Ws = Ss + K * kVSlice;            // 64*VS
  float* P = Ws + kMaxChunk * kVSlice;     // 64*65
  float* G = P + kMaxChunk * kAStride;     // 64
  load_tile(Qs, d.q + row(u, T, t0) * K, c, K, K);
  load_tile(Ks, d.k + row(u, T, t0) * K, c, K, K);
  const float* sb = d.Sb + ((int64_t)u * (bl.nb + 1) + n) * K * V;
  for (int i = threadIdx.x; i < K * vw; i += blockDim.x) {
    const int k = i / vw, v = i - k * vw;
    Ss[k * kVSlice + v] = sb[k * V + v0 + v];
  }
  for (int i = threadIdx.x; i < c * vw; i += blockDim.x) {
    const int t = i / vw, v = i - t * vw;
    Ws[t * kVSlice + v] = d.W[row(u, T, t0 + t) * V + v0 + v];
  }
  load_gates(d, u, t0, c, G, nullptr);
  __syncthreads();
  block_gemm<2, 2>(
      c, c, K, [&](int t, int kk) { return Qs[t * K + kk]; },
      [&](int kk, int s) { return Ks[s * K + kk]; },
      [&](int t, int s, float acc) {
        P[t * kAStride + s] = s <= t ? __expf(G[t] - G[s]) * acc : 0.f;
      });
  __syncthreads();
  for (int t = threadIdx.x; t < c; t += blockDim.x) {
    const float e = __expf(G[t]);
    for (int kk = 0; kk < K; ++kk) Qs[t * K + kk] *= e;
  }
  __syncthreads();
  block_gemm<2, 4>(
      c, vw, K + c,
      [&](int t, int kk) { return kk < K ? Qs[t * K + kk] : P[t * kAStride + (kk - K)]; },
      [&](int kk, int v) { return kk < K ? Ss[kk * kVSlice + v] : Ws[(kk - K) * kVSlice + v]; },
      [&](int t, int v, float acc) { d.O[row(u, T, t0 + t) * V + v0 + v] = acc; });
}

// ----------------------------------------------------------------- backward

GPA_DEV float dO_scale_of(const ScanDesc& d, int u) { return d.dO_scale ? d.dO_scale[u] : 1.f; }

// grid (U*NB*nvs, nscan). Read-path gradients of O = e^G Q S_n + P W.
__global__ void __launch_bounds__(256) gdn_bwd_local_kernel(ScanBatch b, int U, Blocks bl) {
  const ScanDesc& d = b.s[blockIdx.y];
  const int K = d.K, V = d.V, T = bl.T;
  const int nvs = (V + kVSlice - 1) / kVSlice;
  if ((int)blockIdx.x >= U * bl.nb * nvs) return;
  const int vs = blockIdx.x % nvs, un = blockIdx.x / nvs;
  const int u = un / bl.nb, n = un % bl.nb;
  const int v0 = vs * kVSlice, vw = min(kVSlice, V - v0);
  const int t0 = bl.start(n), c = bl.end(n) - t0;
  extern __shared__ float sm[];
  float* Qs = sm;                          // 64*K
  float* Ks = Qs + kMaxChunk * K;          // 64*K
  float* Ss = Ks + kMaxChunk * K;          // K*VS
  float* Ws = Ss + K * kVSlice;            // 64*VS
  float* dOs = Ws + kMaxChunk * kVSlice;   // 64*VS
  float* P = dOs + kMaxChunk * kVSlice;    // 64*65
  float* dP = P + kMaxChunk * kAStride;    // 64*65
  float* G = dP + kMaxChunk * kAStride;    // 64
  float* racc = G + kMaxChunk;             // 64
  float* rsum = racc + kMaxChunk;          // 64
  float* csum = rsum + kMaxChunk;          // 64
  const float sc = dO_scale_of(d, u);
  load_tile(Qs, d.q + row(u, T, t0) * K, c, K, K);
  load_tile(Ks, d.k + row(u, T, t0) * K, c, K, K);
  const float* sb = d.Sb + ((int64_t)u * (bl.nb + 1) + n) * K * V;
  for (int i = threadIdx.x; i < K * vw; i += blockDim.x) {
    const int k = i / vw, v = i - k * vw;
    Ss[k * kVSlice + v] = sb[k * V + v0 + v];
  }
  for (int i = threadIdx.x; i < c * vw; i += blockDim.x) {
    const int t = i / vw, v = i - t * vw;
    Ws[t * kVSlice + v] = d.W[row(u, T, t0 + t) * V + v0 + v];
    dOs[t * kVSlice + v] = sc * d.dO[row(u, T, t0 + t) * V + v0 + v];
  }
  for (int t = threadIdx.x; t < kMaxChunk; t += blockDim.x) racc[t] = rsum[t] = csum[t] = 0.f;
  load_gates(d, u, t0, c, G, nullptr);
  __syncthreads();
  block_gemm<2, 2>(
      c, c, K, [&](int t, int kk) { return Qs[t * K + kk]; },
      [&](int kk, int s) { return Ks[s * K + kk]; },
      [&](int t, int s, float acc) {
        P[t * kAStride + s] = s <= t ? __expf(G[t] - G[s]) * acc : 0.f;
      });
  block_gemm<2, 2>(
      c, c, vw, [&](int t, int v) { return dOs[t * kVSlice + v]; },
      [&](int v, int s) { return Ws[s * kVSlice + v]; },
      [&](int t, int s, float acc) { dP[t * kAStride + s] = s <= t ? acc : 0.f; });
  // rowsum(dO o (Q S)) for the e^G term
  block_gemm<2, 4>(
      c, vw, K, [&](int t, int kk) { return Qs[t * K + kk]; },
      [&](int kk, int v) { return Ss[kk * kVSlice + v]; },
      [&](int t, int v, float acc) { atomicAdd(&racc[t], acc * dOs[t * kVSlice + v]); });
  __syncthreads();
  for (int i = threadIdx.x; i < c * c; i += blockDim.x) {
    const int t = i / c, s = i - t * c;
    if (s <= t) {
      const float e = dP[t * kAStride + s] * P[t * kAStride + s];
      atomicAdd(&rsum[t], e);
      atomicAdd(&csum[s], e);
    }
  }
  __syncthreads();
  for (int t = threadIdx.x; t < c; t += blockDim.x)
    atomicAdd(&d.sc_dG[row(u, T, t0 + t)], __expf(G[t]) * racc[t] + rsum[t] - csum[t]);
  // dX = dP o Gamma
  for (int i = threadIdx.x; i < c * c; i += blockDim.x) {
    const int t = i / c, s = i - t * c;
    if (s <= t) dP[t * kAStride + s] *= __expf(G[t] - G[s]);
  }
  __syncthreads();
  if (d.dq) {
    block_gemm<2, 4>(
        c, K, vw + c,
        [&](int t, int kk) {
          return kk < vw ? __expf(G[t]) * dOs[t * kVSlice + kk] : dP[t * kAStride + (kk - vw)];
        },
        [&](int kk, int k) { return kk < vw ? Ss[k * kVSlice + kk] : Ks[(kk - vw) * K + k]; },
        [&](int t, int k, float acc) { atomicAdd(&d.dq[row(u, T, t0 + t) * K + k], acc); });
  }
  // dK (read part) = dX^T Q
  block_gemm<2, 4>(
      c, K, c, [&](int s, int t) { return dP[t * kAStride + s]; },
      [&](int t, int k) { return Qs[t * K + k]; },
      [&](int s, int k, float acc) { atomicAdd(&d.sc_dK[row(u, T, t0 + s) * K + k], acc); });
  // dW_local = P^T dO
  block_gemm<2, 4>(
      c, vw, c, [&](int s, int t) { return P[t * kAStride + s]; },
      [&](int t, int v) { return dOs[t * kVSlice + v]; },
      [&](int s, int v, float acc) { d.sc_dW[row(u, T, t0 + s) * V + v0 + v] = acc; });
}

// grid (U*nvs, nscan). Reverse sweep: D = dS at block ends; dW = dW_local + lambda K D.
__global__ void __launch_bounds__(256) gdn_bwd_state_kernel(ScanBatch b, int U, Blocks bl) {
  const ScanDesc& d = b.s[blockIdx.y];
  const int K = d.K, V = d.V, T = bl.T;
  const int nvs = (V + kVSlice - 1) / kVSlice;
  if ((int)blockIdx.x >= U * nvs) return;
  const int u = blockIdx.x / nvs, v0 = (blockIdx.x % nvs) * kVSlice;
  const int vw = min(kVSlice, V - v0);
  extern __shared__ float sm[];
  float* D = sm;                           // K*VS
  float* Ks = D + K * kVSlice;             // 64*K
  float* Qs = Ks + kMaxChunk * K;          // 64*K (pre-scaled by e^G)
  float* Wks = Qs + kMaxChunk * K;         // 64*K
  float* dOs = Wks + kMaxChunk * K;        // 64*VS
  float* dWs = dOs + kMaxChunk * kVSlice;  // 64*VS
  float* G = dWs + kMaxChunk * kVSlice;    // 64
  const float sc = dO_scale_of(d, u);
  const int64_t KV = (int64_t)K * V;
  for (int i = threadIdx.x; i < K * vw; i += blockDim.x) {
    const int k = i / vw, v = i - k * vw;
    float x = d.ext ? d.ext[((int64_t)u * (bl.nb + 1) + bl.nb) * KV + k * V + v0 + v] : 0.f;
    if (d.dS_final) x += d.dS_final[(int64_t)u * KV + k * V + v0 + v];
    D[k * kVSlice + v] = x;
  }
  __syncthreads();
  for (int n = bl.nb - 1; n >= 0; --n) {
    const int t0 = bl.start(n), c = bl.end(n) - t0;
    float* de = d.Dend + ((int64_t)u * bl.nb + n) * KV;
    for (int i = threadIdx.x; i < K * vw; i += blockDim.x) {
      const int k = i / vw, v = i - k * vw;
      de[k * V + v0 + v] = D[k * kVSlice + v];
    }
    load_tile(Ks, d.k + row(u, T, t0) * K, c, K, K);
    load_tile(Wks, d.Wk + row(u, T, t0) * K, c, K, K);
    load_gates(d, u, t0, c, G, nullptr);
    if (d.dO) load_tile(Qs, d.q + row(u, T, t0) * K, c, K, K);
    for (int i = threadIdx.x; i < c * vw; i += blockDim.x) {
      const int t = i / vw, v = i - t * vw;
      dOs[t * kVSlice + v] = d.dO ? sc * d.dO[row(u, T, t0 + t) * V + v0 + v] : 0.f;
      dWs[t * kVSlice + v] = d.dO ? d.sc_dW[row(u, T, t0 + t) * V + v0 + v] : 0.f;
    }
    __syncthreads();
    if (d.dO) {
      for (int i = threadIdx.x; i < c * K; i += blockDim.x) Qs[i] *= __expf(G[i / K]);
    }
    // dW = dW_local + lambda * (K D)
    block_gemm<2, 4>(
        c, vw, K, [&](int t, int kk) { return Ks[t * K + kk]; },
        [&](int kk, int v) { return D[kk * kVSlice + v]; },
        [&](int t, int v, float acc) {
          const float w = fmaf(__expf(G[c - 1] - G[t]), acc, dWs[t * kVSlice + v]);
          dWs[t * kVSlice + v] = w;
          d.sc_dW[row(u, T, t0 + t) * V + v0 + v] = w;
        });
    __syncthreads();
    const float gc = __expf(G[c - 1]);
    const float* ext = d.ext ? d.ext + ((int64_t)u * (bl.nb + 1) + n) * KV : nullptr;
    const bool has_o = d.dO != nullptr;
    // D <- e^{G_c} D + Q^T diag(e^G) dO - Wk^T dW + ext_n
    block_gemm<2, 4>(
        K, vw, 2 * c,
        [&](int k, int tt) {
          return tt < c ? (has_o ? Qs[tt * K + k] : 0.f) : -Wks[(tt - c) * K + k];
        },
        [&](int tt, int v) { return tt < c ? dOs[tt * kVSlice + v] : dWs[(tt - c) * kVSlice + v]; },
        [&](int k, int v, float acc) {
          float x = fmaf(gc, D[k * kVSlice + v], acc);
          if (ext) x += ext[k * V + v0 + v];
          D[k * kVSlice + v] = x;
        });
    __syncthreads();
  }
  for (int i = threadIdx.x; i < K * vw; i += blockDim.x) {
    const int k = i / vw, v = i - k * vw;
    d.dS0[((int64_t)u * K + k) * V + v0 + v] = D[k * kVSlice + v];
  }
}

// grid (U*NB*nvs, nscan). State-update terms and the U path (V-sliced partials).
__global__ void __launch_bounds__(256) gdn_bwd_chunk_v_kernel(ScanBatch b, int U, Blocks bl) {
  const ScanDesc& d = b.s[blockIdx.y];
  const int K = d.K, V = d.V, T = bl.T;
  const int nvs = (V + kVSlice - 1) / kVSlice;
  if ((int)blockIdx.x >= U * bl.nb * nvs) return;
  const int vs = blockIdx.x % nvs, un = blockIdx.x / nvs;
  const int u = un / bl.nb, n = un % bl.nb;
  const int v0 = vs * kVSlice, vw = min(kVSlice, V - v0);
  const int t0 = bl.start(n), c = bl.end(n) - t0;
  const int64_t KV = (int64_t)K * V;
  extern __shared__ float sm[];
  float* Ks = sm;                           // 64*K
  float* Ss = Ks + kMaxChunk * K;           // K*VS
  float* Ds = Ss + K * kVSlice;             // K*VS
  float* Ws = Ds + K * kVSlice;             // 64*VS
  float* dWs = Ws + kMaxChunk * kVSlice;    // 64*VS
  float* Us = dWs + kMaxChunk * kVSlice;    // 64*VS
  float* A = Us + kMaxChunk * kVSlice;      // 64*65
  float* G = A + kMaxChunk * kAStride;      // 64
  float* bt = G + kMaxChunk;                // 64
  float* dlam = bt + kMaxChunk;             // 64
  float* red = dlam + kMaxChunk;            // 32
  load_tile(Ks, d.k + row(u, T, t0) * K, c, K, K);
  const float* sb = d.Sb + ((int64_t)u * (bl.nb + 1) + n) * KV;
  const float* de = d.Dend + ((int64_t)u * bl.nb + n) * KV;
  for (int i = threadIdx.x; i < K * vw; i += blockDim.x) {
    const int k = i / vw, v = i - k * vw;
    Ss[k * kVSlice + v] = sb[k * V + v0 + v];
    Ds[k * kVSlice + v] = de[k * V + v0 + v];
  }
  for (int i = threadIdx.x; i < c * vw; i += blockDim.x) {
    const int t = i / vw, v = i - t * vw;
    const int64_t r = row(u, T, t0 + t) * V + v0 + v;
    Ws[t * kVSlice + v] = d.W[r];
    dWs[t * kVSlice + v] = d.sc_dW[r];
    Us[t * kVSlice + v] = d.Ub[r];
  }
  load_gates(d, u, t0, c, G, bt);
  for (int t = threadIdx.x; t < kMaxChunk; t += blockDim.x) dlam[t] = 0.f;
  if (threadIdx.x < 32) red[threadIdx.x] = 0.f;
  __syncthreads();
  build_a(Ks, K, c, G, bt, A, nullptr);
  // WD = W D^T  -> dK += lambda WD ; dlambda_t = sum_k K_tk WD_tk
  block_gemm<2, 4>(
      c, K, vw, [&](int t, int v) { return Ws[t * kVSlice + v]; },
      [&](int v, int k) { return Ds[k * kVSlice + v]; },
      [&](int t, int k, float acc) {
        atomicAdd(&d.sc_dK[row(u, T, t0 + t) * K + k], __expf(G[c - 1] - G[t]) * acc);
        atomicAdd(&dlam[t], Ks[t * K + k] * acc);
      });
  // <D, S>
  {
    float part = 0.f;
    for (int i = threadIdx.x; i < K * vw; i += blockDim.x) {
      const int k = i / vw, v = i - k * vw;
      part += Ds[k * kVSlice + v] * Ss[k * kVSlice + v];
    }
    part = warp_sum(part);
    if ((threadIdx.x & 31) == 0) atomicAdd(&red[0], part);
  }
  // dWk (partial) = -dW S^T
  block_gemm<2, 4>(
      c, K, vw, [&](int t, int v) { return dWs[t * kVSlice + v]; },
      [&](int v, int k) { return Ss[k * kVSlice + v]; },
      [&](int t, int k, float acc) { atomicAdd(&d.sc_dWk[row(u, T, t0 + t) * K + k], -acc); });
  __syncthreads();
  // dG from the state update (lambda and gamma_c terms)
  if (threadIdx.x < 32) {
    float tot = 0.f;
    for (int t = threadIdx.x; t < c; t += 32) {
      const float lam = __expf(G[c - 1] - G[t]);
      const float x = dlam[t] * lam;
      tot += x;
      atomicAdd(&d.sc_dG[row(u, T, t0 + t)], -x);
    }
    tot = warp_sum(tot);
    if (threadIdx.x == 0)
      atomicAdd(&d.sc_dG[row(u, T, t0 + c - 1)], tot + __expf(G[c - 1]) * red[0]);
  }
  // dRu = (I + A)^-T dW   (in place)
  backward_subst(A, dWs, c, vw, kVSlice);
  __syncthreads();
  // dV = b dRu ; db += rowsum(dRu o V)
  for (int i = threadIdx.x; i < c * vw; i += blockDim.x) {
    const int t = i / vw, v = i - t * vw;
    const int64_t r = row(u, T, t0 + t) * V + v0 + v;
    const float y = dWs[t * kVSlice + v];
    atomicAdd(&d.dv[r], bt[t] * y);
    atomicAdd(&d.sc_db[row(u, T, t0 + t)], y * d.v[r]);
  }
  // dA (partial) = -dRu U^T, strictly lower
  float* dA = d.sc_dA + ((int64_t)u * bl.nb + n) * kMaxChunk * kMaxChunk;
  block_gemm<2, 2>(
      c, c, vw, [&](int t, int v) { return dWs[t * kVSlice + v]; },
      [&](int v, int s) { return Us[s * kVSlice + v]; },
      [&](int t, int s, float acc) {
        if (s < t) atomicAdd(&dA[t * kMaxChunk + s], -acc);
      });
}

// grid (U*NB, nscan). Wk path, dA consequences, final dK / dg / dbeta.
__global__ void __launch_bounds__(256) gdn_bwd_chunk_k_kernel(ScanBatch b, int U, Blocks bl) {
  const ScanDesc& d = b.s[blockIdx.y];
  const int K = d.K, T = bl.T;
  if ((int)blockIdx.x >= U * bl.nb) return;
  const int u = blockIdx.x / bl.nb, n = blockIdx.x % bl.nb;
  const int t0 = bl.start(n), c = bl.end(n) - t0;
  extern __shared__ float sm[];
  float* Ks = sm;                             // 64*K
  float* Wks = Ks + kMaxChunk * K;            // 64*K
  float* dWk = Wks + kMaxChunk * K;           // 64*K  (-> dRw in place)
  float* A = dWk + kMaxChunk * K;             // 64*65
  float* At = A + kMaxChunk * kAStride;       // 64*65  (Atil)
  float* dA = At + kMaxChunk * kAStride;      // 64*65
  float* G = dA + kMaxChunk * kAStride;       // 64
  float* bt = G + kMaxChunk;                  // 64
  float* dG = bt + kMaxChunk;                 // 64
  float* db = dG + kMaxChunk;                 // 64
  load_tile(Ks, d.k + row(u, T, t0) * K, c, K, K);
  load_tile(Wks, d.Wk + row(u, T, t0) * K, c, K, K);
  load_tile(dWk, d.sc_dWk + row(u, T, t0) * K, c, K, K);
  const float* dAg = d.sc_dA + ((int64_t)u * bl.nb + n) * kMaxChunk * kMaxChunk;
  for (int i = threadIdx.x; i < c * c; i += blockDim.x) {
    const int t = i / c, s = i - t * c;
    dA[t * kAStride + s] = dAg[t * kMaxChunk + s];
  }
  load_gates(d, u, t0, c, G, bt);
  for (int t = threadIdx.x; t < c; t += blockDim.x) {
    dG[t] = d.sc_dG[row(u, T, t0 + t)];
    db[t] = d.sc_db[row(u, T, t0 + t)];
  }
  __syncthreads();
  build_a(Ks, K, c, G, bt, A, At);
  __syncthreads();
  backward_subst(A, dWk, c, K, K);  // dRw
  __syncthreads();
  // rw_t = dRw_t . k_t ; db += e^G rw ; dG += b e^G rw
  if (threadIdx.x < 32 * 8) {
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int t = w; t < c; t += 8) {
      float x = 0.f;
      for (int k = lane; k < K; k += 32) x += dWk[t * K + k] * Ks[t * K + k];
      x = warp_sum(x);
      if (lane == 0) {
        const float e = __expf(G[t]);
        db[t] += e * x;
        dG[t] += bt[t] * e * x;
      }
    }
  }
  // dA += -(dRw Wk^T), strictly lower
  block_gemm<2, 2>(
      c, c, K, [&](int t, int k) { return dWk[t * K + k]; },
      [&](int k, int s) { return Wks[s * K + k]; },
      [&](int t, int s, float acc) {
        if (s < t) dA[t * kAStride + s] -= acc;
        else dA[t * kAStride + s] = 0.f;
      });
  __syncthreads();
  // dA consequences: db += rowsum(dA o Atil); dG += rowsum(dA o A) - colsum(dA o A)
  if (threadIdx.x < c) {
    const int t = threadIdx.x;
    float r1 = 0.f, r2 = 0.f, c2 = 0.f;
    for (int s = 0; s < t; ++s) {
      r1 += dA[t * kAStride + s] * At[t * kAStride + s];
      r2 += dA[t * kAStride + s] * A[t * kAStride + s];
    }
    for (int s = t + 1; s < c; ++s) c2 += dA[s * kAStride + t] * A[s * kAStride + t];
    db[t] += r1;
    dG[t] += r2 - c2;
  }
  __syncthreads();
  // Mm = dA o b_t Gamma  (= dA o A / k_t.k_s ... computed directly)
  for (int i = threadIdx.x; i < c * c; i += blockDim.x) {
    const int t = i / c, s = i - t * c;
    if (s < t) dA[t * kAStride + s] *= bt[t] * __expf(G[t] - G[s]);
  }
  __syncthreads();
  // dK_total = sc_dK + b e^G dRw + Mm K + Mm^T K
  block_gemm<2, 4>(
      c, K, 2 * c,
      [&](int t, int ss) {
        return ss < c ? (ss < t ? dA[t * kAStride + ss] : 0.f)
                      : ((ss - c) > t ? dA[(ss - c) * kAStride + t] : 0.f);
      },
      [&](int ss, int k) { return Ks[(ss < c ? ss : ss - c) * K + k]; },
      [&](int t, int k, float acc) {
        const int64_t r = row(u, T, t0 + t) * K + k;
        const float x = acc + d.sc_dK[r] + bt[t] * __expf(G[t]) * dWk[t * K + k];
        atomicAdd(&d.dk[r], x);
      });
  __syncthreads();
  // dg = reverse cumsum of dG over the block; dbeta
  if (threadIdx.x == 0) {
    float acc = 0.f;
    for (int t = c - 1; t >= 0; --t) {
      acc += dG[t];
      dG[t] = acc;
    }
  }
  __syncthreads();
  if (d.dg64) {
    if (threadIdx.x == 0) {
      double sg = 0.0, sb = 0.0;
      for (int t = 0; t < c; ++t) {
        sg += dG[t];
        sb += db[t];
      }
      atomicAdd(&d.dg64[(int64_t)u * d.dg_su], sg);
      atomicAdd(&d.dbeta64[(int64_t)u * d.dg_su], sb);
    }
    return;
  }
  for (int t = threadIdx.x; t < c; t += blockDim.x) {
    const int64_t gi = (int64_t)u * d.dg_su + (int64_t)(t0 + t) * d.dg_st;
    atomicAdd(&d.dg[gi], dG[t]);
    atomicAdd(&d.dbeta[gi], db[t]);
  }
}

// ----------------------------------------------------------- shared memory

int max_kv(const ScanBatch& b, int* K, int* V) {
  *K = 0;
  *V = 0;
  for (int i = 0; i < b.n; ++i) {
    *K = b.s[i].K > *K ? b.s[i].K : *K;
    *V = b.s[i].V > *V ? b.s[i].V : *V;
  }
  return 0;
}

constexpr int C = kMaxChunk, VS = kVSlice, AS = kMaxChunk * kAStride;
size_t smem_fwd_chunk(int K, int V) { return sizeof(float) * (C * K + C * (V + K) + AS + 2 * C); }
size_t smem_fwd_state(int K, int) { return sizeof(float) * (K * VS + 2 * C * K + C * VS + C); }
size_t smem_fwd_out(int K, int) { return sizeof(float) * (2 * C * K + K * VS + C * VS + AS + C); }
size_t smem_bwd_local(int K, int) {
  return sizeof(float) * (2 * C * K + K * VS + 2 * C * VS + 2 * AS + 4 * C);
}
size_t smem_bwd_state(int K, int) { return sizeof(float) * (K * VS + 3 * C * K + 2 * C * VS + C); }
size_t smem_bwd_chunk_v(int K, int) {
  return sizeof(float) * (C * K + 2 * K * VS + 3 * C * VS + AS + 3 * C + 32);
}
size_t smem_bwd_chunk_k(int K, int) { return sizeof(float) * (3 * C * K + 3 * AS + 4 * C); }

template <class Kern>
cudaError_t launch(const char* name, Kern k, dim3 grid, size_t smem, cudaStream_t st,
                   const ScanBatch& b, int U, const Blocks& bl) {
  if (grid.x == 0 || grid.y == 0) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  Launch scope(name, st);
  k<<<grid, 256, smem, st>>>(b, U, bl);
  return cudaGetLastError();
}

}  // namespace

int gdn_max_smem_bytes() { return 227 * 1024; }

cudaError_t gdn_forward(const ScanBatch& b, int U, const Blocks& bl, bool with_output,
                        cudaStream_t st) {
  if (b.tc) return tc_forward(b, U, bl, with_output, st);
  int K, V;
  max_kv(b, &K, &V);
  const int nvs = (V + VS - 1) / VS;
  cudaError_t e = launch("gdn_fwd_chunk", gdn_fwd_chunk_kernel, dim3(U * bl.nb, b.n), smem_fwd_chunk(K, V), st, b,
                         U, bl);
  if (e != cudaSuccess) return e;
  e = launch("gdn_fwd_state", gdn_fwd_state_kernel, dim3(U * nvs, b.n), smem_fwd_state(K, V), st, b, U, bl);
  if (e != cudaSuccess || !with_output) return e;
  return gdn_output(b, U, bl, st);
}

cudaError_t gdn_output(const ScanBatch& b, int U, const Blocks& bl, cudaStream_t st) {
  if (b.tc) return tc_output(b, U, bl, st);
  int K, V;
  max_kv(b, &K, &V);
  const int nvs = (V + VS - 1) / VS;
  return launch("gdn_fwd_out", gdn_fwd_out_kernel, dim3(U * bl.nb * nvs, b.n), smem_fwd_out(K, V), st, b, U, bl);
}

cudaError_t gdn_backward_local(const ScanBatch& b, int U, const Blocks& bl, cudaStream_t st) {
  if (b.tc) return tc_backward_local(b, U, bl, st);
  int K, V;
  max_kv(b, &K, &V);
  const int nvs = (V + VS - 1) / VS;
  return launch("gdn_bwd_local", gdn_bwd_local_kernel, dim3(U * bl.nb * nvs, b.n), smem_bwd_local(K, V), st, b, U,
                bl);
}

cudaError_t gdn_backward_rest(const ScanBatch& b, int U, const Blocks& bl, cudaStream_t st) {
  if (b.tc) return tc_backward_rest(b, U, bl, st);
  int K, V;
  max_kv(b, &K, &V);
  const int nvs = (V + VS - 1) / VS;
  // recompute U (into Ub scratch) and Wk
  cudaError_t e = launch("gdn_fwd_chunk", gdn_fwd_chunk_kernel, dim3(U * bl.nb, b.n), smem_fwd_chunk(K, V), st, b,
                         U, bl);
  if (e != cudaSuccess) return e;
  e = launch("gdn_bwd_state", gdn_bwd_state_kernel, dim3(U * nvs, b.n), smem_bwd_state(K, V), st, b, U, bl);
  if (e != cudaSuccess) return e;
  e = launch("gdn_bwd_chunk_v", gdn_bwd_chunk_v_kernel, dim3(U * bl.nb * nvs, b.n), smem_bwd_chunk_v(K, V), st, b, U,
             bl);
  if (e != cudaSuccess) return e;
  return launch("gdn_bwd_chunk_k", gdn_bwd_chunk_k_kernel, dim3(U * bl.nb, b.n), smem_bwd_chunk_k(K, V), st, b, U,
                bl);
}

}  // namespace gpa
