// Tensor-core GDN scan kernels (bf16 operands, fp32 accumulation and fp32 state).
//
// Same chunk algebra and phase split as the SIMT kernels in gdn.cu (see
// gdn.cuh), with three differences that the tensor cores make worthwhile:
//   * T = (I + A)^-1 of a block is formed explicitly (16x16 diagonal blocks by
//     warp forward substitution, off-diagonal blocks by block substitution) so
//     that U, Wk, T^T dW, T^T dWk become tile GEMMs;
//   * one CTA covers the full value width of a block (no value slices), so
//     every per-token gradient is written by exactly one CTA: no atomics;
//   * operands are bf16 tiles in shared memory fed to mma.sync m16n8k16 with
//     fp32 accumulators; states S and dS stay fp32 and are rounded to bf16
//     only as GEMM operands.
// Used when the input dtype is bf16 / fp16 and every width is a multiple of 16.
#include "gdn.cuh"
#include "gdn_dev.cuh"
#include "mma.cuh"
#include "tc5.cuh"
#include "tc_util.cuh"

namespace gpa {
namespace {

using tc::Acc;
using tc::bf16;
using tc::Carve;
using tc::for_tiles;
using tc::ld2;
using tc::st2;
using tc::ld16;
using tc::LDT;
using tc::mma_acc;
using tc::quad_sum;
using tc::tile_split;
using tc::tile_to_bf16;
using tc::tiles_n;
using tc::TileJob;

constexpr int C = kMaxChunk;  // 64 rows per block tile (zero padded)
constexpr int kThreads = 512;  // 16 warps: global-load latency of the tile loads is the limiter

// Gates of one block in registers of warp 0 (t = lane, lane + 32), fetched before the tile
// loads so that their latency overlaps them; gate_finish writes the inclusive cumsum G and
// beta, padded: rows >= c keep G = G[c-1] and beta = 0.
struct GateRegs {
  float g0, g1, b0, b1;
};

GPA_DEV GateRegs gate_fetch(const ScanDesc& d, int u, int t0, int c, bool beta) {
  GateRegs r{0.f, 0.f, 0.f, 0.f};
  if (threadIdx.x < 32) {
    const int t = threadIdx.x;
    if (t < c) {
      r.g0 = gate_at(d.g, d, u, t0 + t);
      if (beta) r.b0 = gate_at(d.beta, d, u, t0 + t);
    }
    if (t + 32 < c) {
      r.g1 = gate_at(d.g, d, u, t0 + t + 32);
      if (beta) r.b1 = gate_at(d.beta, d, u, t0 + t + 32);
    }
  }
  return r;
}

// Ends with __syncthreads (G, bt visible to the block).
GPA_DEV void gate_finish(const GateRegs& r, int c, float* G, float* bt) {
  static_assert(C == 64, "two gates per lane");
  if (threadIdx.x < 32) {
    const int t = threadIdx.x;
    float x0 = r.g0, x1 = r.g1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y0 = __shfl_up_sync(0xffffffffu, x0, o);
      const float y1 = __shfl_up_sync(0xffffffffu, x1, o);
      if (t >= o) {
        x0 += y0;
        x1 += y1;
      }
    }
    x1 += __shfl_sync(0xffffffffu, x0, 31);
    const float last = __shfl_sync(0xffffffffu, c - 1 < 32 ? x0 : x1, (c - 1) & 31);
    G[t] = t < c ? x0 : last;
    G[t + 32] = t + 32 < c ? x1 : last;
    if (bt) {
      bt[t] = t < c ? r.b0 : 0.f;
      bt[t + 32] = t + 32 < c ? r.b1 : 0.f;
    }
  }
  __syncthreads();
}

// The 10 of the 4 x 4 tiles (16 x 16) of a 64 x 64 block on or below the diagonal, round-robin
// over the warps: body(m0, n0).  A product with a lower-triangular block operand reads no other.
template <class Body>
GPA_DEV void for_lower_tiles(Body body) {
  static_assert(C == 64, "4 x 4 tiles of 16 x 16");
  for (int i = threadIdx.x >> 5; i < 10; i += blockDim.x >> 5) {
    const int mi = i < 1 ? 0 : i < 3 ? 1 : i < 6 ? 2 : 3;
    body(16 * mi, 16 * (i - mi * (mi + 1) / 2));
  }
}

// A[t][s] = b_t exp(G_t - G_s) k_t.k_s (s < t); k split hi/lo
GPA_DEV void tc_build_a(const bf16* Ks, const bf16* Kl, int ldk, int K, const float* G,
                        const float* bt, float* A) {
  for_lower_tiles([&](int m0, int n0) {  // the upper tiles are never read
    Acc<1, 1> acc;
    acc.zero();
    tc::mma_acc3<1, 1, false, true>(acc, Ks, Kl, ldk, Ks, Kl, ldk, m0, n0, K);
    acc.each(m0, n0, [&](int t, int s, float& v) {
      const float at = s < t ? __expf(G[t] - G[s]) * v : 0.f;
      A[t * kAStride + s] = bt[t] * at;
    });
  });
}

// ------------------------------------------------------------------ forward

struct LFwdChunk {
  // after the inversion, the A + Fpad region holds the hi/lo factor of one product at a time
  size_t Ks, Kl, Vs, A, Fpad, Tm, Fh, Fl, G, bt, total;
  __host__ __device__ LFwdChunk(int K, int V) {
    Carve c;
    Ks = c.take(2 * C * ld16(K));
    Kl = c.take(2 * C * ld16(K));
    Vs = c.take(2 * C * ld16(V));
    A = c.take(4 * C * kAStride);
    Fpad = c.take(4 * 768);
    Tm = c.take(4 * C * kAStride);
    G = c.take(4 * C);
    bt = c.take(4 * C);
    total = c.off;
    Fh = A;
    Fl = A + 2 * C * LDT;  // 2 * 2 * C * LDT <= 4 * C * kAStride + 4 * 768
  }
};

// grid (U*NB, nscan): U = T diag(b) V and Wk = T diag(b e^G) K of every block.
__global__ void __launch_bounds__(kThreads) tc_fwd_chunk(ScanBatch b, int U, Blocks bl) {
  const ScanDesc& d = b.s[blockIdx.y];
  const int u = blockIdx.x / bl.nb, n = blockIdx.x % bl.nb, T = bl.T;
  const int t0 = bl.start(n), c = bl.end(n) - t0, K = d.K, V = d.V;
  const int ldk = ld16(K), ldv = ld16(V);
  extern __shared__ __align__(16) unsigned char smem[];
  const LFwdChunk L(K, V);
  bf16* Ks = (bf16*)(smem + L.Ks);
  bf16* Kl = (bf16*)(smem + L.Kl);
  bf16* Vs = (bf16*)(smem + L.Vs);
  float* A = (float*)(smem + L.A);
  float* Tm = (float*)(smem + L.Tm);
  bf16* Fh = (bf16*)(smem + L.Fh);
  bf16* Fl = (bf16*)(smem + L.Fl);
  float* G = (float*)(smem + L.G);
  float* bt = (float*)(smem + L.bt);
  {
    const GateRegs gr = gate_fetch(d, u, t0, c, true);
    const TileJob jobs[] = {tc::job(Ks, Kl, ldk, d.k + row(u, T, t0) * K, K, c, K, C),
                            tc::job(Vs, nullptr, ldv, d.v + row(u, T, t0) * V, V, c, V, C)};
    tc::load_tiles<false>(jobs);
    gate_finish(gr, c, G, bt);
  }
  tc_build_a(Ks, Kl, ldk, K, G, bt, A);
  __syncthreads();
  invert_unit_lower(A, Tm);  // ends with __syncthreads: A is free below
  float* Ts = d.Tsv + ((int64_t)u * bl.nb + n) * C * C;
  for (int i = threadIdx.x; i < C * C; i += blockDim.x) Ts[i] = Tm[(i / C) * kAStride + (i % C)];
  for (int i = threadIdx.x; i < C * C / 2; i += blockDim.x) {
    const int t = 2 * i / C, s = 2 * i - t * C;
    tc::split2(Tm[t * kAStride + s] * bt[s], Tm[t * kAStride + s + 1] * bt[s + 1],
               Fh + t * LDT + s, Fl + t * LDT + s);
  }
  __syncthreads();
  tiles_n<1, 2>(C, V, [&]<int NI>(int m0, int n0) {
    Acc<1, NI> acc;
    acc.zero();
    tc::mma_acc3<1, NI, false, false>(acc, Fh, Fl, LDT, Vs, nullptr, ldv, m0, n0, m0 + 16);
    acc.each2(m0, n0, [&](int, int t, int col, float& v0, float& v1) {
      if (t < c) st2(d.Ub + row(u, T, t0 + t) * V + col, v0, v1);
    });
  });
  __syncthreads();
  for (int i = threadIdx.x; i < C * C / 2; i += blockDim.x) {
    const int t = 2 * i / C, s = 2 * i - t * C;
    tc::split2(Tm[t * kAStride + s] * bt[s] * __expf(G[s]),
               Tm[t * kAStride + s + 1] * bt[s + 1] * __expf(G[s + 1]), Fh + t * LDT + s,
               Fl + t * LDT + s);
  }
  __syncthreads();
  tiles_n<1, 2>(C, K, [&]<int NI>(int m0, int n0) {
    Acc<1, NI> acc;
    acc.zero();
    tc::mma_acc3<1, NI, false, false>(acc, Fh, Fl, LDT, Ks, Kl, ldk, m0, n0, m0 + 16);
    acc.each2(m0, n0, [&](int, int t, int col, float& v0, float& v1) {
      if (t < c) st2(d.Wk + row(u, T, t0 + t) * K + col, v0, v1);
    });
  });
}

// The state sweeps are split over value columns: W = U - Wk S and S <- e^{G_c} S + K^T
// diag(lambda) W (and the same for D, dW) never mix columns, so each CTA carries one slice
// of VS columns of the state.  VS keeps the shared memory of a CTA at or under 113 KB (two
// CTAs per SM) for widths up to 128.
constexpr int kStateThreads = 256;

__host__ __device__ inline int state_slice(int K, int V) {
  const int cap = K > 64 ? 32 : 64;  // V is a multiple of 16
  for (int vs = cap; vs > 16; vs >>= 1)
    if (V % vs == 0) return vs;
  return 16;
}

__host__ __device__ inline int state_slices(int K, int V) { return V / state_slice(K, V); }

// 16x32 tiles when they keep every warp busy, else 16x16
template <class Body>
GPA_DEV void tiles_spread(int M, int N, Body body) {
  if (N % 32 == 0 && (M / 16) * (N / 32) >= (int)(blockDim.x >> 5))
    tc::for_tiles<1, 2>(M, N, [&](int m0, int n0) { body.template operator()<2>(m0, n0); });
  else
    tc::for_tiles<1, 1>(M, N, [&](int m0, int n0) { body.template operator()<1>(m0, n0); });
}

struct LFwdState {
  size_t Sf, Sb, Wkh, Wkl, Ks, Kl, Wch, Wcl, G, lam, total;
  __host__ __device__ LFwdState(int K, int V) {
    const int VS = state_slice(K, V);
    Carve c;
    Sf = c.take(4 * K * (VS + 8));  // padded rows: the accumulator-layout float2 accesses
                                    // of a half-warp hit 16 distinct bank pairs
    Sb = c.take(2 * K * ld16(VS));
    Wkh = c.take(2 * C * ld16(K));
    Wkl = c.take(2 * C * ld16(K));
    Ks = c.take(2 * C * ld16(K));
    Kl = c.take(2 * C * ld16(K));
    Wch = c.take(2 * C * ld16(VS));
    Wcl = c.take(2 * C * ld16(VS));
    G = c.take(4 * C);
    lam = c.take(4 * C);
    total = c.off;
  }
};

// grid (U * slices, nscan): sequential over blocks, one column slice of the state [K x VS]
// fp32 in shared memory.
__global__ void __launch_bounds__(kStateThreads, 2) tc_fwd_state(ScanBatch b, int U, Blocks bl) {
  const ScanDesc& d = b.s[blockIdx.y];
  const int K = d.K, V = d.V, VS = state_slice(K, V), nvs = V / VS;
  const int u = blockIdx.x / nvs, v0 = (blockIdx.x % nvs) * VS, T = bl.T;
  const int ldk = ld16(K), lds = ld16(VS);
  const int64_t KV = (int64_t)K * V;
  extern __shared__ __align__(16) unsigned char smem[];
  const LFwdState L(K, V);
  float* Sf = (float*)(smem + L.Sf);
  const int lsf = VS + 8;
  bf16* Sb = (bf16*)(smem + L.Sb);
  bf16* Wkh = (bf16*)(smem + L.Wkh);
  bf16* Wkl = (bf16*)(smem + L.Wkl);
  bf16* Ks = (bf16*)(smem + L.Ks);
  bf16* Kl = (bf16*)(smem + L.Kl);
  bf16* Wch = (bf16*)(smem + L.Wch);
  bf16* Wcl = (bf16*)(smem + L.Wcl);
  float* G = (float*)(smem + L.G);
  float* lam = (float*)(smem + L.lam);
  const int q4 = VS >> 2;  // float4 per slice row
  // state slice rows k: global [k * V + v0, + VS)
  auto put_slice = [&](float* dst) {
    for (int i = threadIdx.x; i < K * q4; i += blockDim.x) {
      const int k = i / q4, j = (i - k * q4) << 2;
      *reinterpret_cast<float4*>(dst + (int64_t)k * V + v0 + j) =
          *reinterpret_cast<const float4*>(Sf + k * lsf + j);
    }
  };
  for (int i = threadIdx.x; i < K * q4; i += blockDim.x) {
    const int k = i / q4, j = (i - k * q4) << 2;
    const float4 x = *reinterpret_cast<const float4*>(d.S0 + u * KV + (int64_t)k * V + v0 + j);
    *reinterpret_cast<float4*>(Sf + k * lsf + j) = x;
    tc::put4(Sb, nullptr, k * lds + j, x);
  }
  __syncthreads();
  GateRegs gr = gate_fetch(d, u, bl.start(0), bl.end(0) - bl.start(0), false);
  for (int n = 0; n < bl.nb; ++n) {
    const int t0 = bl.start(n), c = bl.end(n) - t0;
    put_slice(d.Sb + ((int64_t)u * (bl.nb + 1) + n) * KV);
    const TileJob jobs[] = {tc::job(Wkh, Wkl, ldk, d.Wk + row(u, T, t0) * K, K, c, K, C),
                            tc::job(Ks, Kl, ldk, d.k + row(u, T, t0) * K, K, c, K, C)};
    tc::load_tiles(jobs);
    gate_finish(gr, c, G, nullptr);
    if (n + 1 < bl.nb) gr = gate_fetch(d, u, bl.start(n + 1), bl.end(n + 1) - bl.start(n + 1), false);
    for (int t = threadIdx.x; t < C; t += blockDim.x) lam[t] = __expf(G[c - 1] - G[t]);
    __syncthreads();
    // W = U - Wk S (slice columns)
    tiles_spread(C, VS, [&]<int NI>(int m0, int n0) {
      Acc<1, NI> acc;
      float2 ub[Acc<1, NI>::kPairs];
      acc.each2(m0, n0, [&](int p, int t, int col, float&, float&) {
        ub[p] = t < c ? ld2(d.Ub + row(u, T, t0 + t) * V + v0 + col) : make_float2(0.f, 0.f);
      });
      acc.zero();
      tc::mma_acc3<1, NI, false, false>(acc, Wkh, Wkl, ldk, Sb, nullptr, lds, m0, n0, K);
      acc.each2(m0, n0, [&](int p, int t, int col, float& x0, float& x1) {
        const float w0 = t < c ? ub[p].x - x0 : 0.f, w1 = t < c ? ub[p].y - x1 : 0.f;
        if (t < c)
          *reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<bf16*>(d.W) + row(u, T, t0 + t) * V +
                                             v0 + col) = __floats2bfloat162_rn(w0, w1);
        tc::split2(w0 * lam[t], w1 * lam[t], Wch + t * lds + col, Wcl + t * lds + col);
      });
    });
    __syncthreads();
    const float gc = __expf(G[c - 1]);
    // S = e^{G_c} S + K^T diag(lambda) W
    tiles_spread(K, VS, [&]<int NI>(int m0, int n0) {
      Acc<1, NI> acc;
      acc.each2(m0, n0, [&](int, int k, int col, float& x0, float& x1) {
        const float2 sv = *reinterpret_cast<const float2*>(Sf + k * lsf + col);
        x0 = gc * sv.x;
        x1 = gc * sv.y;
      });
      tc::mma_acc3<1, NI, true, false>(acc, Ks, Kl, ldk, Wch, Wcl, lds, m0, n0, C);
      acc.each2(m0, n0, [&](int, int k, int col, float& x0, float& x1) {
        *reinterpret_cast<float2*>(Sf + k * lsf + col) = make_float2(x0, x1);
        *reinterpret_cast<__nv_bfloat162*>(Sb + k * lds + col) = __floats2bfloat162_rn(x0, x1);
      });
    });
    __syncthreads();
  }
  put_slice(d.Sb + ((int64_t)u * (bl.nb + 1) + bl.nb) * KV);
  if (d.S_final) put_slice(d.S_final + u * KV);
}

struct LFwdOut {
  size_t Qs, Ks, Ss, Wh, Ph, Pl, G, total;
  __host__ __device__ LFwdOut(int K, int V) {
    Carve c;
    Qs = c.take(2 * C * ld16(K));
    Ks = c.take(2 * C * ld16(K));
    Ss = c.take(2 * K * ld16(V));
    Wh = c.take(2 * C * ld16(V));
    Ph = c.take(2 * C * LDT);
    Pl = c.take(2 * C * LDT);
    G = c.take(4 * C);
    total = c.off;
  }
};

// grid (U*NB, nscan): O = e^G (Q S_n) + (Q K^T o Gamma) W
__global__ void __launch_bounds__(kThreads) tc_fwd_out(ScanBatch b, int U, Blocks bl) {
  const ScanDesc& d = b.s[blockIdx.y];
  if (!d.q || !d.O) return;
  const int u = blockIdx.x / bl.nb, n = blockIdx.x % bl.nb, T = bl.T;
  const int t0 = bl.start(n), c = bl.end(n) - t0, K = d.K, V = d.V;
  const int ldk = ld16(K), ldv = ld16(V);
  const int64_t KV = (int64_t)K * V;
  extern __shared__ __align__(16) unsigned char smem[];
  const LFwdOut L(K, V);
  bf16* Qs = (bf16*)(smem + L.Qs);
  bf16* Ks = (bf16*)(smem + L.Ks);
  bf16* Ss = (bf16*)(smem + L.Ss);
  bf16* Wh = (bf16*)(smem + L.Wh);
  bf16* Ph = (bf16*)(smem + L.Ph);
  bf16* Pl = (bf16*)(smem + L.Pl);
  float* G = (float*)(smem + L.G);
  {
    const GateRegs gr = gate_fetch(d, u, t0, c, false);
    const TileJob jobs[] = {
        tc::job(Qs, nullptr, ldk, d.q + row(u, T, t0) * K, K, c, K, C),
        tc::job(Ks, nullptr, ldk, d.k + row(u, T, t0) * K, K, c, K, C),
        tc::job(Ss, nullptr, ldv, d.Sb + ((int64_t)u * (bl.nb + 1) + n) * KV, V, K, V, K)};
    tc::copy_bf16_tile(Wh, ldv, reinterpret_cast<const bf16*>(d.W) + row(u, T, t0) * V, V, c, V, C);
    tc::load_tiles<false>(jobs);
    gate_finish(gr, c, G, nullptr);
  }
  for_lower_tiles([&](int m0, int n0) {  // P is lower triangular
    Acc<1, 1> acc;
    acc.zero();
    mma_acc<1, 1, false, true>(acc, Qs, ldk, Ks, ldk, m0, n0, K);
    acc.each2(m0, n0, [&](int, int t, int s, float& v0, float& v1) {
      tc::split2(s <= t ? __expf(G[t] - G[s]) * v0 : 0.f,
                 s + 1 <= t ? __expf(G[t] - G[s + 1]) * v1 : 0.f, Ph + t * LDT + s,
                 Pl + t * LDT + s);
    });
  });
  __syncthreads();
  tiles_n<1, 2>(C, V, [&]<int NI>(int m0, int n0) {
    Acc<1, NI> acc;
    acc.zero();
    mma_acc<1, NI, false, false>(acc, Qs, ldk, Ss, ldv, m0, n0, K);
    acc.each(m0, n0, [&](int t, int, float& v) { v *= __expf(G[t]); });
    tc::mma_acc3<1, NI, false, false>(acc, Ph, Pl, LDT, Wh, nullptr, ldv, m0, n0, m0 + 16);
    acc.each2(m0, n0, [&](int, int t, int col, float& v0, float& v1) {
      if (t < c) st2(d.O + row(u, T, t0 + t) * V + col, v0, v1);
    });
  });
}

// ----------------------------------------------------------------- backward

GPA_DEV float dscale(const ScanDesc& d, int u) { return d.dO_scale ? d.dO_scale[u] : 1.f; }

struct LBwdLocal {
  size_t Qs, Ks, Ss, Wh, dOs, Ph, Pl, dXh, dXl, G, racc, rs, cs, total;
  __host__ __device__ LBwdLocal(int K, int V) {
    Carve c;
    Qs = c.take(2 * C * ld16(K));
    Ks = c.take(2 * C * ld16(K));
    Ss = c.take(2 * K * ld16(V));
    Wh = c.take(2 * C * ld16(V));
    dOs = c.take(2 * C * ld16(V));
    Ph = c.take(2 * C * LDT);
    Pl = c.take(2 * C * LDT);
    dXh = c.take(2 * C * LDT);
    dXl = c.take(2 * C * LDT);
    G = c.take(4 * C);
    racc = c.take(4 * C);
    rs = c.take(4 * C);
    cs = c.take(4 * C);
    total = c.off;
  }
};

// grid (U*NB, nscan): read-path gradients of O = e^G Q S_n + P W.
__global__ void __launch_bounds__(kThreads, 2) tc_bwd_local(ScanBatch b, int U, Blocks bl) {
  const ScanDesc& d = b.s[blockIdx.y];
  const int u = blockIdx.x / bl.nb, n = blockIdx.x % bl.nb, T = bl.T;
  const int t0 = bl.start(n), c = bl.end(n) - t0, K = d.K, V = d.V;
  const int ldk = ld16(K), ldv = ld16(V);
  const int64_t KV = (int64_t)K * V;
  extern __shared__ __align__(16) unsigned char smem[];
  const LBwdLocal L(K, V);
  bf16* Qs = (bf16*)(smem + L.Qs);
  bf16* Ks = (bf16*)(smem + L.Ks);
  bf16* Ss = (bf16*)(smem + L.Ss);
  bf16* Wh = (bf16*)(smem + L.Wh);
  bf16* dOs = (bf16*)(smem + L.dOs);
  bf16* Ph = (bf16*)(smem + L.Ph);
  bf16* Pl = (bf16*)(smem + L.Pl);
  bf16* dXh = (bf16*)(smem + L.dXh);
  bf16* dXl = (bf16*)(smem + L.dXl);
  float* G = (float*)(smem + L.G);
  float* racc = (float*)(smem + L.racc);
  float* rs = (float*)(smem + L.rs);
  float* cs = (float*)(smem + L.cs);
  for (int t = threadIdx.x; t < C; t += blockDim.x) racc[t] = rs[t] = cs[t] = 0.f;
  {
    const GateRegs gr = gate_fetch(d, u, t0, c, false);
    const TileJob jobs[] = {
        tc::job(Qs, nullptr, ldk, d.q + row(u, T, t0) * K, K, c, K, C),
        tc::job(Ks, nullptr, ldk, d.k + row(u, T, t0) * K, K, c, K, C),
        tc::job(Ss, nullptr, ldv, d.Sb + ((int64_t)u * (bl.nb + 1) + n) * KV, V, K, V, K),
        tc::job(dOs, nullptr, ldv, d.dO + row(u, T, t0) * V, V, c, V, C, dscale(d, u))};
    tc::copy_bf16_tile(Wh, ldv, reinterpret_cast<const bf16*>(d.W) + row(u, T, t0) * V, V, c, V, C);
    tc::load_tiles(jobs);
    gate_finish(gr, c, G, nullptr);
  }
  // P = (Q K^T) o Gamma and dP = dO W^T on the same tile: rowsum / colsum of P o dP and
  // dX = dP o Gamma straight from the accumulators (both lower triangular: the products
  // below read no upper tile of P or dX)
  for_lower_tiles([&](int m0, int n0) {
    Acc<1, 1> pa, da;
    pa.zero();
    mma_acc<1, 1, false, true>(pa, Qs, ldk, Ks, ldk, m0, n0, K);
    pa.each2(m0, n0, [&](int, int t, int s, float& v0, float& v1) {
      v0 = s <= t ? __expf(G[t] - G[s]) * v0 : 0.f;
      v1 = s + 1 <= t ? __expf(G[t] - G[s + 1]) * v1 : 0.f;
      tc::split2(v0, v1, Ph + t * LDT + s, Pl + t * LDT + s);
    });
    da.zero();
    mma_acc<1, 1, false, true>(da, dOs, ldv, Wh, ldv, m0, n0, V);  // dO is bf16 already
    const int lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
    float rsum[2] = {0.f, 0.f}, csum[2][2] = {};
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int t = m0 + g + 8 * h, s = n0 + 8 * j + 2 * q;
        float x[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float dp = s + e <= t ? da.v[0][j][2 * h + e] : 0.f;
          const float pr = pa.v[0][j][2 * h + e] * dp;
          rsum[h] += pr;
          csum[j][e] += pr;
          x[e] = s + e <= t ? dp * __expf(G[t] - G[s + e]) : 0.f;
        }
        tc::split2(x[0], x[1], dXh + t * LDT + s, dXl + t * LDT + s);
      }
    const float r0s = quad_sum(rsum[0]), r1s = quad_sum(rsum[1]);
    if (q == 0) {
      atomicAdd(&rs[m0 + g], r0s);
      atomicAdd(&rs[m0 + g + 8], r1s);
    }
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float x = csum[j][h];
        x += __shfl_xor_sync(0xffffffffu, x, 4);
        x += __shfl_xor_sync(0xffffffffu, x, 8);
        x += __shfl_xor_sync(0xffffffffu, x, 16);
        if (g == 0) atomicAdd(&cs[n0 + 8 * j + 2 * q + h], x);
      }
  });
  // racc = rowsum(dO o (Q S_n)) = rowsum(Q o (dO S_n^T)): taken from dq's first product when
  // dq is wanted, else from Q S_n
  auto racc_add = [&](int m0, float part0, float part1) {
    const int g = (threadIdx.x & 31) >> 2;
    const float p0 = quad_sum(part0), p1 = quad_sum(part1);
    if ((threadIdx.x & 3) == 0) {
      atomicAdd(&racc[m0 + g], p0);
      atomicAdd(&racc[m0 + g + 8], p1);
    }
  };
  if (!d.dq) {
    tiles_n<1, 2>(C, V, [&]<int NI>(int m0, int n0) {
      Acc<1, NI> acc;
      acc.zero();
      mma_acc<1, NI, false, false>(acc, Qs, ldk, Ss, ldv, m0, n0, K);
      float part[2] = {0.f, 0.f};
      acc.each2(m0, n0, [&](int, int t, int col, float& v0, float& v1) {
        const float2 o2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(dOs + t * ldv + col));
        part[(t - m0) >> 3 & 1] += v0 * o2.x + v1 * o2.y;
      });
      racc_add(m0, part[0], part[1]);
    });
  }
  __syncthreads();  // dX, P / dP sums
  if (d.dq) {
    tiles_n<1, 2>(C, K, [&]<int NI>(int m0, int n0) {
      Acc<1, NI> acc;
      float2 dq[Acc<1, NI>::kPairs];
      acc.each2(m0, n0, [&](int p, int t, int col, float&, float&) {
        if (t < c) dq[p] = ld2(d.dq + row(u, T, t0 + t) * K + col);
      });
      acc.zero();
      mma_acc<1, NI, false, true>(acc, dOs, ldv, Ss, ldv, m0, n0, V);
      float part[2] = {0.f, 0.f};
      acc.each2(m0, n0, [&](int, int t, int col, float& v0, float& v1) {
        const float2 q2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(Qs + t * ldk + col));
        part[(t - m0) >> 3 & 1] += v0 * q2.x + v1 * q2.y;
        const float e = __expf(G[t]);
        v0 *= e;
        v1 *= e;
      });
      racc_add(m0, part[0], part[1]);
      tc::mma_acc3<1, NI, false, false>(acc, dXh, dXl, LDT, Ks, nullptr, ldk, m0, n0, m0 + 16);
      acc.each2(m0, n0, [&](int p, int t, int col, float& v0, float& v1) {
        if (t < c) st2(d.dq + row(u, T, t0 + t) * K + col, dq[p].x + v0, dq[p].y + v1);
      });
    });
    __syncthreads();  // racc
  }
  for (int t = threadIdx.x; t < c; t += blockDim.x)
    d.sc_dG[row(u, T, t0 + t)] = __expf(G[t]) * racc[t] + rs[t] - cs[t];
  tiles_n<1, 2>(C, K, [&]<int NI>(int m0, int n0) {
    Acc<1, NI> acc;
    acc.zero();
    tc::mma_acc3<1, NI, true, false>(acc, dXh, dXl, LDT, Qs, nullptr, ldk, m0, n0, C, m0);
    acc.each2(m0, n0, [&](int, int s, int col, float& v0, float& v1) {
      if (s < c) st2(d.sc_dK + row(u, T, t0 + s) * K + col, v0, v1);
    });
  });
  tiles_n<1, 2>(C, V, [&]<int NI>(int m0, int n0) {
    Acc<1, NI> acc;
    acc.zero();
    tc::mma_acc3<1, NI, true, false>(acc, Ph, Pl, LDT, dOs, nullptr, ldv, m0, n0, C, m0);
    acc.each2(m0, n0, [&](int, int s, int col, float& v0, float& v1) {
      if (s < c) st2(d.sc_dW + row(u, T, t0 + s) * V + col, v0, v1);
    });
  });
}

struct LBwdState {
  size_t Dh, Dl, Ks, Qg, Wknh, Wknl, dOs, dWh, dWl, G, lam, eG, total;
  __host__ __device__ LBwdState(int K, int V) {
    const int VS = state_slice(K, V);
    Carve c;
    Dh = c.take(2 * K * ld16(VS));
    Dl = c.take(2 * K * ld16(VS));
    Ks = c.take(2 * C * ld16(K));
    Qg = c.take(2 * C * ld16(K));
    Wknh = c.take(2 * C * ld16(K));
    Wknl = c.take(2 * C * ld16(K));
    dOs = c.take(2 * C * ld16(VS));
    dWh = c.take(2 * C * ld16(VS));
    dWl = c.take(2 * C * ld16(VS));
    G = c.take(4 * C);
    lam = c.take(4 * C);
    eG = c.take(4 * C);
    total = c.off;
  }
};

// grid (U * slices, nscan): reverse sweep over one column slice; D = dS at block ends;
// dW = dW_local + lambda K D.  D is carried as a hi/lo bf16 pair (~16 significant bits).
__global__ void __launch_bounds__(kStateThreads, 2) tc_bwd_state(ScanBatch b, int U, Blocks bl) {
  const ScanDesc& d = b.s[blockIdx.y];
  const int K = d.K, V = d.V, VS = state_slice(K, V), nvs = V / VS;
  const int u = blockIdx.x / nvs, v0 = (blockIdx.x % nvs) * VS, T = bl.T;
  const int ldk = ld16(K), lds = ld16(VS);
  const int64_t KV = (int64_t)K * V;
  extern __shared__ __align__(16) unsigned char smem[];
  const LBwdState L(K, V);
  bf16* Dh = (bf16*)(smem + L.Dh);
  bf16* Dl = (bf16*)(smem + L.Dl);
  bf16* Ks = (bf16*)(smem + L.Ks);
  bf16* Qg = (bf16*)(smem + L.Qg);
  bf16* Wknh = (bf16*)(smem + L.Wknh);
  bf16* Wknl = (bf16*)(smem + L.Wknl);
  bf16* dOs = (bf16*)(smem + L.dOs);
  bf16* dWh = (bf16*)(smem + L.dWh);
  bf16* dWl = (bf16*)(smem + L.dWl);
  float* G = (float*)(smem + L.G);
  float* lam = (float*)(smem + L.lam);
  float* eG = (float*)(smem + L.eG);
  const float sc = dscale(d, u);
  const int q4 = VS >> 2;
  for (int i = threadIdx.x; i < K * q4; i += blockDim.x) {
    const int k = i / q4, j = (i - k * q4) << 2;
    const int64_t o = (int64_t)k * V + v0 + j;
    float4 x = d.ext ? *reinterpret_cast<const float4*>(d.ext + ((int64_t)u * (bl.nb + 1) + bl.nb) * KV + o)
                     : make_float4(0.f, 0.f, 0.f, 0.f);
    if (d.dS_final) {
      const float4 y = *reinterpret_cast<const float4*>(d.dS_final + u * KV + o);
      x.x += y.x;
      x.y += y.y;
      x.z += y.z;
      x.w += y.w;
    }
    tc::put4(Dh, Dl, k * lds + j, x);
  }
  // D (hi + lo) -> fp32 rows of a global [K x V] array, this slice's columns
  auto get_slice = [&](float* dst) {
    for (int i = threadIdx.x; i < K * q4; i += blockDim.x) {
      const int k = i / q4, j = (i - k * q4) << 2, o = k * lds + j;
      const uint2 h = *reinterpret_cast<const uint2*>(Dh + o), l = *reinterpret_cast<const uint2*>(Dl + o);
      const float2 h01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&h.x));
      const float2 h23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&h.y));
      const float2 l01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&l.x));
      const float2 l23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&l.y));
      *reinterpret_cast<float4*>(dst + (int64_t)k * V + v0 + j) =
          make_float4(h01.x + l01.x, h01.y + l01.y, h23.x + l23.x, h23.y + l23.y);
    }
  };
  __syncthreads();
  GateRegs gr = gate_fetch(d, u, bl.start(bl.nb - 1), bl.end(bl.nb - 1) - bl.start(bl.nb - 1),
                           false);
  for (int n = bl.nb - 1; n >= 0; --n) {
    const int t0 = bl.start(n), c = bl.end(n) - t0;
    if (n > 0 && threadIdx.x == 0) {
      // the rows block n - 1 reads, towards L2 while this block computes (the sweep otherwise
      // waits on DRAM at every block start)
      const int p0 = bl.start(n - 1), pc = bl.end(n - 1) - p0;
      const int64_t pr = row(u, T, p0);
      tc5::prefetch_l2(d.k + pr * K, (uint32_t)(pc * K * 4));
      tc5::prefetch_l2(d.q + pr * K, (uint32_t)(pc * K * 4));
      tc5::prefetch_l2(d.Wk + pr * K, (uint32_t)(pc * K * 4));
      tc5::prefetch_l2(d.dO + pr * V, (uint32_t)(pc * V * 4));
      tc5::prefetch_l2(d.sc_dW + pr * V, (uint32_t)(pc * V * 4));
      if (d.ext) tc5::prefetch_l2(d.ext + ((int64_t)u * (bl.nb + 1) + n - 1) * KV, (uint32_t)(KV * 4));
    }
    get_slice(d.Dend + ((int64_t)u * bl.nb + n) * KV);
    gate_finish(gr, c, G, nullptr);
    for (int t = threadIdx.x; t < C; t += blockDim.x) {
      lam[t] = __expf(G[c - 1] - G[t]);
      eG[t] = __expf(G[t]);
    }
    __syncthreads();
    if (n > 0) gr = gate_fetch(d, u, bl.start(n - 1), bl.end(n - 1) - bl.start(n - 1), false);
    {
      const TileJob jobs[] = {
          tc::job(Ks, nullptr, ldk, d.k + row(u, T, t0) * K, K, c, K, C),
          tc::job(Qg, nullptr, ldk, d.q + row(u, T, t0) * K, K, c, K, C, 1.f, eG),
          tc::job(Wknh, Wknl, ldk, d.Wk + row(u, T, t0) * K, K, c, K, C, -1.f),
          tc::job(dOs, nullptr, lds, d.dO + row(u, T, t0) * V + v0, V, c, VS, C, sc)};
      tc::load_tiles(jobs);
    }
    __syncthreads();
    // dW = dW_local + lambda (K D)
    tiles_spread(C, VS, [&]<int NI>(int m0, int n0) {
      Acc<1, NI> acc;
      float2 dw[Acc<1, NI>::kPairs];
      acc.each2(m0, n0, [&](int p, int t, int col, float&, float&) {
        dw[p] = t < c ? ld2(d.sc_dW + row(u, T, t0 + t) * V + v0 + col) : make_float2(0.f, 0.f);
      });
      acc.zero();
      tc::mma_acc3<1, NI, false, false>(acc, Ks, nullptr, ldk, Dh, Dl, lds, m0, n0, K);
      acc.each2(m0, n0, [&](int p, int t, int col, float& x0, float& x1) {
        const float w0 = t < c ? dw[p].x + lam[t] * x0 : 0.f;
        const float w1 = t < c ? dw[p].y + lam[t] * x1 : 0.f;
        if (t < c) st2(d.sc_dW + row(u, T, t0 + t) * V + v0 + col, w0, w1);
        tc::split2(w0, w1, dWh + t * lds + col, dWl + t * lds + col);
      });
    });
    __syncthreads();
    const float gc = __expf(G[c - 1]);
    const float* ext = d.ext ? d.ext + ((int64_t)u * (bl.nb + 1) + n) * KV + v0 : nullptr;
    // D <- e^{G_c} D + (e^G Q)^T dO - Wk^T dW + ext_n
    tiles_spread(K, VS, [&]<int NI>(int m0, int n0) {
      Acc<1, NI> acc;
      acc.each2(m0, n0, [&](int, int k, int col, float& x0, float& x1) {
        const int o = k * lds + col;
        const float2 h = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(Dh + o));
        const float2 l = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(Dl + o));
        const float2 e = ext ? ld2(ext + (int64_t)k * V + col) : make_float2(0.f, 0.f);
        x0 = gc * (h.x + l.x) + e.x;
        x1 = gc * (h.y + l.y) + e.y;
      });
      mma_acc<1, NI, true, false>(acc, Qg, ldk, dOs, lds, m0, n0, C);
      tc::mma_acc3<1, NI, true, false>(acc, Wknh, Wknl, ldk, dWh, dWl, lds, m0, n0, C);
      __syncwarp();
      acc.each2(m0, n0, [&](int, int k, int col, float& x0, float& x1) {
        tc::split2(x0, x1, Dh + k * lds + col, Dl + k * lds + col);
      });
    });
    __syncthreads();
  }
  get_slice(d.dS0 + u * KV);
}

struct LBwdChunk {
  // T (hi/lo) and the per-token vectors are fixed; a pool X holds, stage by stage,
  //   1 state terms: dWh, dWl, Sb, Db, Wb   2 U path: dWh, dWl, Uh, Ul
  //   3 Wk path: Wkh, Wkl, dWkh, dWkl       4 dA: Mh, Ml, Mmb, Ks, Kl (A = b e^G K K^T is
  //   recomputed in the dA epilogue exactly as the forward formed it)
  // so that every shape with K, V <= 128 but (128, 128) fits two CTAs per SM.
  size_t Th, Tl, G, bt, dG, db, dlam, rw, red, X, total;
  size_t dWh, dWl, Sb, Db, Wb, Uh, Ul, Wkh, Wkl, dWkh, dWkl, Mh, Ml, dAf, Ks, Kl, Mmb;
  __host__ __device__ LBwdChunk(int K, int V) {
    Carve c;
    const size_t sK = 2 * C * ld16(K), sV = 2 * C * ld16(V), sS = 2 * K * ld16(V);
    const size_t sT = 2 * C * LDT;
    Th = c.take(sT);
    Tl = c.take(sT);
    G = c.take(4 * C);
    bt = c.take(4 * C);
    dG = c.take(4 * C);
    db = c.take(4 * C);
    dlam = c.take(4 * C);
    rw = c.take(4 * C);
    red = c.take(4 * 32);
    Carve s1, s2, s3, s4;
    dWh = s1.take(sV);
    dWl = s1.take(sV);
    Sb = s1.take(sS);
    Db = s1.take(sS);
    Wb = s1.take(sV);
    s2.take(2 * sV);  // dW stays
    Uh = s2.take(sV);
    Ul = s2.take(sV);
    Wkh = s3.take(sK);
    Wkl = s3.take(sK);
    dWkh = s3.take(sK);
    dWkl = s3.take(sK);
    Mh = s4.take(sT);
    Ml = s4.take(sT);
    dAf = s4.take(sT);  // Mmb
    Ks = s4.take(sK);
    Kl = s4.take(sK);
    size_t pool = s1.off;
    pool = pool > s2.off ? pool : s2.off;
    pool = pool > s3.off ? pool : s3.off;
    pool = pool > s4.off ? pool : s4.off;
    X = c.take(pool);
    size_t* const in_pool[] = {&dWh, &dWl, &Sb, &Db, &Wb, &Uh, &Ul, &Wkh, &Wkl,
                               &dWkh, &dWkl, &Mh, &Ml, &dAf, &Ks, &Kl};
    for (size_t* q : in_pool) *q += X;
    Mmb = dAf;  // the dA epilogue writes Mm while other warps still read Mh, Ml
    total = c.off;
  }
};

// grid (U*NB, nscan): the whole block backward after the state sweep (dW and D known):
// state-update terms, U path, Wk path, dA consequences, final dK / dg / dbeta.
// The dA of both paths is formed as -T^T (dW U^T + dWk Wk^T) (strictly lower part); that
// C x C sum stays in each warp's accumulator tiles across the U and Wk stages.  Launched
// with 256 threads (two CTAs per SM) or 512.
__global__ void __launch_bounds__(kThreads) tc_bwd_chunk(ScanBatch b, int U, Blocks bl) {
  const ScanDesc& d = b.s[blockIdx.y];
  const int u = blockIdx.x / bl.nb, n = blockIdx.x % bl.nb, T = bl.T;
  const int t0 = bl.start(n), c = bl.end(n) - t0, K = d.K, V = d.V;
  const int ldk = ld16(K), ldv = ld16(V);
  const int64_t KV = (int64_t)K * V;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  extern __shared__ __align__(16) unsigned char smem[];
  const LBwdChunk L(K, V);
  bf16* Ks = (bf16*)(smem + L.Ks);
  bf16* Kl = (bf16*)(smem + L.Kl);
  bf16* Th = (bf16*)(smem + L.Th);
  bf16* Tl = (bf16*)(smem + L.Tl);
  bf16* Mh = (bf16*)(smem + L.Mh);
  bf16* Ml = (bf16*)(smem + L.Ml);
  float* G = (float*)(smem + L.G);
  float* bt = (float*)(smem + L.bt);
  float* dG = (float*)(smem + L.dG);
  float* db = (float*)(smem + L.db);
  float* dlam = (float*)(smem + L.dlam);
  float* rw = (float*)(smem + L.rw);
  float* red = (float*)(smem + L.red);
  bf16* dWh = (bf16*)(smem + L.dWh);
  bf16* dWl = (bf16*)(smem + L.dWl);
  bf16* Sb = (bf16*)(smem + L.Sb);
  bf16* Db = (bf16*)(smem + L.Db);
  bf16* Wb = (bf16*)(smem + L.Wb);
  bf16* Uh = (bf16*)(smem + L.Uh);
  bf16* Ul = (bf16*)(smem + L.Ul);
  bf16* Wkh = (bf16*)(smem + L.Wkh);
  bf16* Wkl = (bf16*)(smem + L.Wkl);
  bf16* dWkh = (bf16*)(smem + L.dWkh);
  bf16* dWkl = (bf16*)(smem + L.dWkl);
  bf16* Mmb = (bf16*)(smem + L.Mmb);
  const float* sg = d.Sb + ((int64_t)u * (bl.nb + 1) + n) * KV;
  const float* dg = d.Dend + ((int64_t)u * bl.nb + n) * KV;
  const int64_t r0 = row(u, T, t0);

  // M = dW U^T + dWk Wk^T: 16 accumulator tiles of 16 x 16, tile w + i nw of each warp
  constexpr int kMT = 2;  // 8 or 16 warps
  Acc<1, 1> macc[kMT];
  for (int t = threadIdx.x; t < C; t += blockDim.x) {
    dG[t] = t < c ? d.sc_dG[r0 + t] : 0.f;
    db[t] = dlam[t] = rw[t] = 0.f;
  }
  if (threadIdx.x < 32) red[threadIdx.x] = 0.f;
  if (threadIdx.x == 32) {
    // rows the later stages read (U and V path, Wk path, the K tile, the dK accumulator):
    // start them towards L2 now so that those stages wait on L2, not DRAM
    tc5::prefetch_l2(d.k + r0 * K, (uint32_t)(c * K * 4));
    tc5::prefetch_l2(d.Ub + r0 * V, (uint32_t)(c * V * 4));
    tc5::prefetch_l2(d.v + r0 * V, (uint32_t)(c * V * 4));
    tc5::prefetch_l2(d.Wk + r0 * K, (uint32_t)(c * K * 4));
    tc5::prefetch_l2(d.dk + r0 * K, (uint32_t)(c * K * 4));
  }
  float dsp = 0.f;  // this thread's part of <D, S>
  {  // gates, T of the block as the forward formed it, and the state-term operands
    const GateRegs gr = gate_fetch(d, u, t0, c, true);
    const TileJob jobs[] = {tc::job(Th, Tl, LDT, d.Tsv + ((int64_t)u * bl.nb + n) * C * C, C, C, C, C),
                            tc::job(dWh, dWl, ldv, d.sc_dW + r0 * V, V, c, V, C)};
    tc::copy_bf16_tile(Wb, ldv, reinterpret_cast<const bf16*>(d.W) + r0 * V, V, c, V, C);
    tc::load_tiles(jobs);
    const TileJob js = tc::job(Sb, nullptr, ldv, sg, V, K, V, K);
    const TileJob jd = tc::job(Db, nullptr, ldv, dg, V, K, V, K);
    tc::tile_pair(js, &jd, &dsp);  // S and D tiles; <D, S> from their fp32 values
    gate_finish(gr, c, G, bt);
  }
  __syncthreads();
  {  // <D, S> in fp32 (red was zeroed before the barrier)
    const float part = warp_sum(dsp);
    if (lane == 0) atomicAdd(&red[0], part);
  }

  // ---- state-update terms: WD = W D^T, <D, S>, dWk = -dW S^T
  // sc_dK += lambda WD ; dlambda_t = sum_k K_tk WD_tk
  tiles_n<1, 2>(C, K, [&]<int NI>(int m0, int n0) {
    Acc<1, NI> acc;
    float2 dk[Acc<1, NI>::kPairs], kk[Acc<1, NI>::kPairs];
    acc.each2(m0, n0, [&](int p, int t, int col, float&, float&) {
      kk[p] = make_float2(0.f, 0.f);
      if (t < c) {
        dk[p] = ld2(d.sc_dK + (r0 + t) * K + col);
        kk[p] = ld2(d.k + (r0 + t) * K + col);
      }
    });
    acc.zero();
    mma_acc<1, NI, false, true>(acc, Wb, ldv, Db, ldv, m0, n0, V);
    float part[2] = {0.f, 0.f};
    acc.each2(m0, n0, [&](int p, int t, int col, float& v0, float& v1) {
      if (t < c) {
        const float lm = __expf(G[c - 1] - G[t]);
        st2(d.sc_dK + (r0 + t) * K + col, dk[p].x + lm * v0, dk[p].y + lm * v1);
      }
      part[(t - m0) >> 3 & 1] += v0 * kk[p].x + v1 * kk[p].y;
    });
    const int g = lane >> 2;
    const float p0 = quad_sum(part[0]), p1 = quad_sum(part[1]);
    if ((lane & 3) == 0) {
      atomicAdd(&dlam[m0 + g], p0);
      atomicAdd(&dlam[m0 + g + 8], p1);
    }
  });
  // dWk = -dW S^T, staged through global memory (L2) for the Wk path
  tiles_n<1, 2>(C, K, [&]<int NI>(int m0, int n0) {
    Acc<1, NI> acc;
    acc.zero();
    tc::mma_acc3<1, NI, false, true>(acc, dWh, dWl, ldv, Sb, nullptr, ldv, m0, n0, V);
    acc.each2(m0, n0, [&](int, int t, int col, float& v0, float& v1) {
      if (t < c) st2(d.sc_dWk + (r0 + t) * K + col, -v0, -v1);
    });
  });
  __syncthreads();
  if (w == 0) {  // dG from the state update (lambda and gamma_c terms)
    float tot = 0.f;
    for (int t = lane; t < c; t += 32) {
      const float x = dlam[t] * __expf(G[c - 1] - G[t]);
      tot += x;
      dG[t] -= x;
    }
    tot = warp_sum(tot);
    if (lane == 0) dG[c - 1] += tot + __expf(G[c - 1]) * red[0];
  }

  // ---- U path: dRu = T^T dW ; dV += b dRu ; db += rowsum(dRu o V) ; M = dW U^T
  tile_split(Uh, Ul, ldv, d.Ub + r0 * V, V, c, V, C);
  __syncthreads();
  tiles_n<1, 2>(C, V, [&]<int NI>(int m0, int n0) {
    Acc<1, NI> acc;
    float2 vv[Acc<1, NI>::kPairs];
    acc.each2(m0, n0, [&](int p, int t, int col, float&, float&) {
      if (t < c) vv[p] = ld2(d.v + (r0 + t) * V + col);
    });
    acc.zero();
    tc::mma_acc3<1, NI, true, false>(acc, Th, Tl, LDT, dWh, dWl, ldv, m0, n0, C, m0);  // T^T: upper
    float part[2] = {0.f, 0.f};
    acc.each2(m0, n0, [&](int p, int t, int col, float& v0, float& v1) {
      if (t < c) {
        atomicAdd(reinterpret_cast<float2*>(d.dv + (r0 + t) * V + col),
                  make_float2(bt[t] * v0, bt[t] * v1));
        part[(t - m0) >> 3 & 1] += v0 * vv[p].x + v1 * vv[p].y;
      }
    });
    const int g = lane >> 2;
    const float p0 = quad_sum(part[0]), p1 = quad_sum(part[1]);
    if ((lane & 3) == 0) {
      atomicAdd(&db[m0 + g], p0);
      atomicAdd(&db[m0 + g + 8], p1);
    }
  });
#pragma unroll
  for (int i = 0; i < kMT; ++i) {
    const int tl = w + i * nw;
    macc[i].zero();
    if (tl < 16)
      tc::mma_acc3<1, 1, false, true>(macc[i], dWh, dWl, ldv, Uh, Ul, ldv, 16 * (tl >> 2),
                                      16 * (tl & 3), V);
  }
  __syncthreads();

  // ---- Wk path: dRw = T^T dWk ; sc_dK += b e^G dRw ; rw = rowsum(dRw o K) ; M += dWk Wk^T
  {
    const TileJob jobs[] = {tc::job(Wkh, Wkl, ldk, d.Wk + r0 * K, K, c, K, C),
                            tc::job(dWkh, dWkl, ldk, d.sc_dWk + r0 * K, K, c, K, C)};
    tc::load_tiles(jobs);
  }
  __syncthreads();
  tiles_n<1, 2>(C, K, [&]<int NI>(int m0, int n0) {
    Acc<1, NI> acc;
    float2 dk[Acc<1, NI>::kPairs], kk[Acc<1, NI>::kPairs];
    acc.each2(m0, n0, [&](int p, int t, int col, float&, float&) {
      kk[p] = make_float2(0.f, 0.f);
      if (t < c) {
        dk[p] = ld2(d.sc_dK + (r0 + t) * K + col);
        kk[p] = ld2(d.k + (r0 + t) * K + col);
      }
    });
    acc.zero();
    tc::mma_acc3<1, NI, true, false>(acc, Th, Tl, LDT, dWkh, dWkl, ldk, m0, n0, C, m0);
    float part[2] = {0.f, 0.f};
    acc.each2(m0, n0, [&](int p, int t, int col, float& v0, float& v1) {
      if (t < c) {
        const float be = bt[t] * __expf(G[t]);
        st2(d.sc_dK + (r0 + t) * K + col, dk[p].x + be * v0, dk[p].y + be * v1);
      }
      part[(t - m0) >> 3 & 1] += v0 * kk[p].x + v1 * kk[p].y;
    });
    const int g = lane >> 2;
    const float p0 = quad_sum(part[0]), p1 = quad_sum(part[1]);
    if ((lane & 3) == 0) {
      atomicAdd(&rw[m0 + g], p0);
      atomicAdd(&rw[m0 + g + 8], p1);
    }
  });
#pragma unroll
  for (int i = 0; i < kMT; ++i) {
    const int tl = w + i * nw;
    if (tl < 16)
      tc::mma_acc3<1, 1, false, true>(macc[i], dWkh, dWkl, ldk, Wkh, Wkl, ldk, 16 * (tl >> 2),
                                      16 * (tl & 3), K);
  }
  __syncthreads();  // Wk, dWk are dead: M, A and K of the block go into the pool
  for (int t = threadIdx.x; t < C; t += blockDim.x) {
    const float e = __expf(G[t]);
    db[t] += e * rw[t];
    dG[t] += bt[t] * e * rw[t];
    rw[t] = dlam[t] = 0.f;  // reused below for the row / column sums of dA o A
  }
  {
    const TileJob jobs[] = {tc::job(Ks, Kl, ldk, d.k + r0 * K, K, c, K, C)};
    tc::load_tiles(jobs);
  }
#pragma unroll
  for (int i = 0; i < kMT; ++i) {
    const int tl = w + i * nw;
    if (tl < 16)
      macc[i].each2(16 * (tl >> 2), 16 * (tl & 3), [&](int, int t, int s, float& v0, float& v1) {
        tc::split2(v0, v1, Mh + t * LDT + s, Ml + t * LDT + s);
      });
  }
  __syncthreads();
  // dA = -T^T M (strictly lower, real rows), straight from the accumulators: the row and
  // column sums of dA o A (into rw, dlam) and Mm = dA o b_t e^{G_t - G_s} (bf16, into Mmb).
  // A = b_t e^{G_t - G_s} k_t.k_s of the same tile is formed again beside it (the forward's
  // tc_build_a product on the same split K tiles: the same values).
  // Only the 10 tiles on or below the diagonal are formed (T^T is upper triangular: the
  // product for row tile m0 runs over k >= m0); the dK products below read no upper tile of Mm.
  float* rsum = rw;
  float* csum = dlam;
  for_lower_tiles([&](int m0, int n0) {
    Acc<1, 1> acc, ak;
    acc.zero();
    ak.zero();
    tc::mma_acc3<1, 1, true, false>(acc, Th, Tl, LDT, Mh, Ml, LDT, m0, n0, C, m0);
    tc::mma_acc3<1, 1, false, true>(ak, Ks, Kl, ldk, Ks, Kl, ldk, m0, n0, K);
    float rp[2] = {0.f, 0.f}, cp[2][2] = {};
    acc.each2(m0, n0, [&](int p, int t, int s, float& v0, float& v1) {
      const float d0 = (s < t && t < c) ? -v0 : 0.f, d1 = (s + 1 < t && t < c) ? -v1 : 0.f;
      const float k0 = ak.v[0][p >> 1][2 * (p & 1)], k1 = ak.v[0][p >> 1][2 * (p & 1) + 1];
      const float a0 = bt[t] * (s < t ? __expf(G[t] - G[s]) * k0 : 0.f);
      const float a1 = bt[t] * (s + 1 < t ? __expf(G[t] - G[s + 1]) * k1 : 0.f);
      const float p0 = d0 * a0, p1 = d1 * a1;
      rp[(t - m0) >> 3] += p0 + p1;
      cp[(p >> 1) & 1][0] += p0;
      cp[(p >> 1) & 1][1] += p1;
      const float f = bt[t];
      *reinterpret_cast<__nv_bfloat162*>(Mmb + t * LDT + s) =
          __floats2bfloat162_rn(d0 * f * __expf(G[t] - G[s]), d1 * f * __expf(G[t] - G[s + 1]));
    });
    const int g = lane >> 2, q = lane & 3;
    const float r0s = quad_sum(rp[0]), r1s = quad_sum(rp[1]);
    if (q == 0) {
      atomicAdd(&rsum[m0 + g], r0s);
      atomicAdd(&rsum[m0 + g + 8], r1s);
    }
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float x = cp[j][e];
        x += __shfl_xor_sync(0xffffffffu, x, 4);
        x += __shfl_xor_sync(0xffffffffu, x, 8);
        x += __shfl_xor_sync(0xffffffffu, x, 16);
        if (g == 0) atomicAdd(&csum[n0 + 8 * j + 2 * q + e], x);
      }
  });
  __syncthreads();
  // A = b_t A~ (A~ without b_t): rowsum(dA o A~) = rowsum(dA o A) / b_t (b_t > 0 on real rows)
  for (int t = threadIdx.x; t < C; t += blockDim.x) {
    if (t < c) db[t] += rsum[t] / bt[t];
    dG[t] += rsum[t] - csum[t];
  }
  // dK = sc_dK + Mm K + Mm^T K
  tiles_n<1, 2>(C, K, [&]<int NI>(int m0, int n0) {
    Acc<1, NI> acc;
    float2 a[Acc<1, NI>::kPairs], s2[Acc<1, NI>::kPairs];
    acc.each2(m0, n0, [&](int p, int t, int col, float&, float&) {
      if (t < c) {
        a[p] = ld2(d.dk + (r0 + t) * K + col);
        s2[p] = ld2(d.sc_dK + (r0 + t) * K + col);
      }
    });
    acc.zero();
    // Mm is strictly lower: Mm K needs k < m0 + 16, Mm^T K needs k >= m0
    tc::mma_acc3<1, NI, false, false>(acc, Mmb, nullptr, LDT, Ks, Kl, ldk, m0, n0, m0 + 16);
    tc::mma_acc3<1, NI, true, false>(acc, Mmb, nullptr, LDT, Ks, Kl, ldk, m0, n0, C, m0);
    acc.each2(m0, n0, [&](int p, int t, int col, float& v0, float& v1) {
      if (t < c) st2(d.dk + (r0 + t) * K + col, a[p].x + s2[p].x + v0, a[p].y + s2[p].y + v1);
    });
  });
  // dg_t = sum_{s >= t} dG_s (reverse cumsum over the block), then per-token or scalar output
  if (w == 0) {
    const int ta = 2 * lane, tb = 2 * lane + 1;
    const float x0 = ta < c ? dG[ta] : 0.f, x1 = tb < c ? dG[tb] : 0.f;
    const float pr = x0 + x1;
    float suf = pr;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_down_sync(0xffffffffu, suf, o);
      if (lane + o < 32) suf += y;
    }
    const float after = suf - pr;
    const float g0 = x0 + x1 + after, g1 = x1 + after;
    if (d.dg64) {
      float sg_ = (ta < c ? g0 : 0.f) + (tb < c ? g1 : 0.f);
      float sb_ = (ta < c ? db[ta] : 0.f) + (tb < c ? db[tb] : 0.f);
      sg_ = warp_sum(sg_);
      sb_ = warp_sum(sb_);
      if (lane == 0) {
        atomicAdd(&d.dg64[(int64_t)u * d.dg_su], (double)sg_);
        atomicAdd(&d.dbeta64[(int64_t)u * d.dg_su], (double)sb_);
      }
    } else {
      if (ta < c) {
        const int64_t gi = (int64_t)u * d.dg_su + (int64_t)(t0 + ta) * d.dg_st;
        d.dg[gi] += g0;
        d.dbeta[gi] += db[ta];
      }
      if (tb < c) {
        const int64_t gi = (int64_t)u * d.dg_su + (int64_t)(t0 + tb) * d.dg_st;
        d.dg[gi] += g1;
        d.dbeta[gi] += db[tb];
      }
    }
  }
}

template <class Kern>
cudaError_t tc_launch(const char* name, Kern k, dim3 grid, size_t smem, cudaStream_t st,
                      const ScanBatch& b, int U, const Blocks& bl, int threads = kThreads) {
  if (grid.x == 0 || grid.y == 0) return cudaSuccess;
  if (smem > 227 * 1024) return cudaErrorInvalidConfiguration;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  Launch scope(name, st);
  k<<<grid, threads, smem, st>>>(b, U, bl);
  return cudaGetLastError();
}

// Launch one kernel per group of scans with the same (K, V): each group gets the shared
// memory its own shape needs, so narrow scans fit more CTAs per SM.
// gx: CTAs per scan along x; with `sliced`, times the state slices of the group's shape.
// A group whose layout is at most `half_kb` KB runs 256 threads per CTA (0: never): at
// 113 KB two such CTAs share an SM, at 74 KB three (more CTAs in flight than two of 512).
template <class Lay, class Kern>
cudaError_t tc_launch_groups(const char* name, Kern k, int gx, const ScanBatch& b, int U,
                             const Blocks& bl, cudaStream_t st, bool sliced = false,
                             int half_kb = 0) {
  bool done[kMaxScans] = {};
  for (int i = 0; i < b.n; ++i) {
    if (done[i]) continue;
    ScanBatch sub;
    sub.tc = b.tc;
    sub.n = 0;
    for (int j = i; j < b.n; ++j)
      if (!done[j] && b.s[j].K == b.s[i].K && b.s[j].V == b.s[i].V) {
        sub.s[sub.n++] = b.s[j];
        done[j] = true;
      }
    const int K = b.s[i].K, V = b.s[i].V;
    const int x = sliced ? gx * state_slices(K, V) : gx;
    const size_t smem = Lay(K, V).total;
    const int threads =
        sliced ? kStateThreads : (smem <= (size_t)half_kb * 1024 ? kThreads / 2 : kThreads);
    const cudaError_t e = tc_launch(name, k, dim3(x, sub.n), smem, st, sub, U, bl, threads);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace

bool tc_supported(int K, int V) {
  return K % 16 == 0 && V % 16 == 0 && K <= 128 && V <= 128;
}

cudaError_t tc_forward(const ScanBatch& b, int U, const Blocks& bl, bool with_output,
                       cudaStream_t st) {
  cudaError_t e = tc5_wy_enabled() ? tc5_fwd_chunk_launch(b, U, bl, st)
                                   : tc_launch_groups<LFwdChunk>("tc_fwd_chunk", tc_fwd_chunk,
                                                                 U * bl.nb, b, U, bl, st, false, 74);
  if (e != cudaSuccess) return e;
  e = tc5_sweeps_enabled() ? tc5_fwd_state_launch(b, U, bl, st)
                           : tc_launch_groups<LFwdState>("tc_fwd_state", tc_fwd_state, U, b, U,
                                                         bl, st, true);
  if (e != cudaSuccess || !with_output) return e;
  return tc_output(b, U, bl, st);
}

cudaError_t tc_output(const ScanBatch& b, int U, const Blocks& bl, cudaStream_t st) {
  if (tc5_out_enabled()) return tc5_fwd_out_launch(b, U, bl, st);
  return tc_launch_groups<LFwdOut>("tc_fwd_out", tc_fwd_out, U * bl.nb, b, U, bl, st, false, 74);
}

cudaError_t tc_backward_local(const ScanBatch& b, int U, const Blocks& bl, cudaStream_t st) {
  return tc_launch_groups<LBwdLocal>("tc_bwd_local", tc_bwd_local, U * bl.nb, b, U, bl, st);
}

// U and Wk of every block come from the forward (kept in the saved buffer).
cudaError_t tc_backward_rest(const ScanBatch& b, int U, const Blocks& bl, cudaStream_t st) {
  cudaError_t e = tc5_sweeps_enabled()
                      ? tc5_bwd_state_launch(b, U, bl, st)
                      : tc_launch_groups<LBwdState>("tc_bwd_state", tc_bwd_state, U, b, U, bl, st, true);
  if (e != cudaSuccess) return e;
  return tc_launch_groups<LBwdChunk>("tc_bwd_chunk", tc_bwd_chunk, U * bl.nb, b, U, bl, st,
                                     false, 113);
}

}  // namespace gpa
