// Tensor-core (bf16 mma.sync, fp32 accumulate) variants of the per-token level
// kernels, used with bf16 / fp16 inputs when every width is a multiple of 16.
// Each CTA handles 64 tokens of one unit; per-head weights are staged in
// shared memory as bf16 (the reference applies them in the activation dtype,
// src/gpa/attention.py:177, 243-254), per-row softmax / norm work stays on
// warps.  Formulas are those of the SIMT kernels in level.cu.
#include "level.cuh"
#include "rowops.cuh"
#include "tc_util.cuh"

namespace gpa {
namespace {

using tc::Acc;
using tc::bf16;
using tc::Carve;
using tc::for_tiles;
using tc::ld16;
using tc::mma_acc;
using tc::quad_sum;
using tc::tile_split;
using tc::tile_to_bf16;
using tc::tiles_n;

constexpr int R = kRowsPerTile;  // 64 tokens per CTA

template <int N>
GPA_DEV void store_bf16_row(bf16* dst, const float (&x)[N], int n) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < N; ++i)
    if (lane + 32 * i < n) dst[lane + 32 * i] = __float2bfloat16(x[i]);
}

template <int N>
GPA_DEV void store_split_row(bf16* hi, bf16* lo, const float (&x)[N], int n) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < N; ++i)
    if (lane + 32 * i < n) tc::split_bf16(x[i], hi + lane + 32 * i, lo + lane + 32 * i);
}

template <class Lay>
size_t smem_of(int a, int b, int c) { return Lay(a, b, c).total; }

// ------------------------------------------------------------------ prep

struct LPrep {
  size_t Kb, Cb, St, Wg4, total;
  __host__ __device__ LPrep(int D, int M, int) {
    Carve c;
    Kb = c.take(2 * R * ld16(D));
    Cb = c.take(2 * M * ld16(D));
    St = c.take(4 * R * (M + 8));  // row stride M + 8: conflict-free accumulator float2 stores
    Wg4 = c.take(4 * 4 * D);
    total = c.off;
  }
};

template <int NPL>
__global__ void __launch_bounds__(512) tk_level_prep(int U, int T, int H, int D, int M,
                                                     const float* key, const float* C,
                                                     const float* Wg, const float* gbias,
                                                     float beta_max, int pos_none, float* nk,
                                                     float* kn, float* slot, float* ns, float* sn,
                                                     float* raw4, float* gates) {
  const int ntile = (T + R - 1) / R;
  const int u = blockIdx.x / ntile, t0 = (blockIdx.x % ntile) * R;
  const int c = min(R, T - t0), h = u % H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  extern __shared__ __align__(16) unsigned char smem[];
  const LPrep L(D, M, 0);
  bf16* Kb = (bf16*)(smem + L.Kb);
  bf16* Cb = (bf16*)(smem + L.Cb);
  float* St = (float*)(smem + L.St);
  tile_to_bf16(Kb, ld16(D), key + row(u, T, t0) * D, D, c, D, R);
  tile_to_bf16(Cb, ld16(D), C + (int64_t)h * M * D, D, M, D, M);
  float* Wg4 = (float*)(smem + L.Wg4);
  for (int i = threadIdx.x; i < D; i += blockDim.x)
    *reinterpret_cast<float4*>(Wg4 + 4 * i) = *reinterpret_cast<const float4*>(Wg + ((int64_t)h * D + i) * 4);
  __syncthreads();
  for (int t = warp; t < c; t += nw) {
    float kx[NPL];
    load_vec(kx, key + row(u, T, t0 + t) * D, D);
    const float nrm = warp_norm(kx, D);
    const float inv = 1.f / fmaxf(nrm, kUnitEps);
    float r[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
      const int d = lane + 32 * i;
      if (d >= D) break;
      const float x = kx[i] * inv;
      nk[row(u, T, t0 + t) * D + d] = x;
      const float4 w4 = *reinterpret_cast<const float4*>(Wg4 + 4 * d);
      r[0] += x * w4.x;
      r[1] += x * w4.y;
      r[2] += x * w4.z;
      r[3] += x * w4.w;
    }
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) r[cc] = warp_sum(r[cc]) + gbias[h * 4 + cc];
    if (lane == 0) {
      const int64_t o = row(u, T, t0 + t);
      kn[o] = nrm;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) raw4[o * 4 + cc] = r[cc];
      gates[o * 4 + 0] = pos_none ? 0.f : -fminf(softplus(r[0]), 10.f);
      gates[o * 4 + 1] = beta_max * sigmoid(r[1]);
      gates[o * 4 + 2] = pos_none ? 0.f : -fminf(softplus(r[2]), 10.f);
      gates[o * 4 + 3] = beta_max * sigmoid(r[3]);
    }
  }
  __syncthreads();
  // slot = k C^T
  tiles_n<1, 2>(R, M, [&]<int NI>(int m0, int n0) {
    Acc<1, NI> acc;
    acc.zero();
    mma_acc<1, NI, false, true>(acc, Kb, ld16(D), Cb, ld16(D), m0, n0, D);
    acc.each2(m0, n0, [&](int, int t, int m, float& v0, float& v1) {
      *reinterpret_cast<float2*>(St + t * (M + 8) + m) = make_float2(v0, v1);
      if (t < c) tc::st2(slot + row(u, T, t0 + t) * M + m, v0, v1);
    });
  });
  __syncthreads();
  for (int t = warp; t < c; t += nw) {
    float x[NPL];
    load_vec(x, St + t * (M + 8), M);
    const float nrm = warp_norm(x, M);
    const float inv = 1.f / fmaxf(nrm, kUnitEps);
#pragma unroll
    for (int i = 0; i < NPL; ++i) x[i] *= inv;
    store_vec(ns + row(u, T, t0 + t) * M, x, M);
    if (lane == 0) sn[row(u, T, t0 + t)] = nrm;
  }
}

// ------------------------------------------------------------------ post

GPA_DEV const float* frozen_at(const float* bnd, const float* fz, int u, int n, int nb, int post,
                               int64_t sz) {
  if (n == 0 && fz) return fz + (int64_t)u * sz;
  return bnd + ((int64_t)u * (nb + 1) + n + post) * sz;
}

struct LPost {
  size_t Af, Bf, Nk, Wf, Wb, total;
  __host__ __device__ LPost(int D, int Dv, int M) {
    Carve c;
    Af = c.take(2 * D * ld16(M));
    Bf = c.take(2 * M * ld16(Dv));
    Nk = c.take(2 * R * ld16(D));
    Wf = c.take(4 * R * (M + 8));  // row stride M + 8
    Wb = c.take(2 * R * ld16(M));
    total = c.off;
  }
};

template <int NPL>
__global__ void __launch_bounds__(512) tk_level_post(
    int U, Blocks bl, int post, int H, int D, int Dv, int M, int with_residual, const float* nk,
    const float* key, const float* val, const float* Abnd, const float* Bbnd, const float* fzA,
    const float* fzB, const float* residual_raw, int j, float* write, float* bsum,
    float* key_next, float* val_next) {
  const int u = blockIdx.x / bl.nb, n = blockIdx.x % bl.nb, T = bl.T;
  const int t0 = bl.start(n), c = bl.end(n) - t0, h = u % H;
  const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  extern __shared__ __align__(16) unsigned char smem[];
  const LPost L(D, Dv, M);
  bf16* Af = (bf16*)(smem + L.Af);
  bf16* Bf = (bf16*)(smem + L.Bf);
  bf16* Nk = (bf16*)(smem + L.Nk);
  float* Wf = (float*)(smem + L.Wf);
  bf16* Wb = (bf16*)(smem + L.Wb);
  const int lm = ld16(M), ld = ld16(D), lv = ld16(Dv);
  tile_to_bf16(Af, lm, frozen_at(Abnd, fzA, u, n, bl.nb, post, (int64_t)D * M), M, D, M, D);
  if (with_residual)
    tile_to_bf16(Bf, lv, frozen_at(Bbnd, fzB, u, n, bl.nb, post, (int64_t)M * Dv), Dv, M, Dv, M);
  tile_to_bf16(Nk, ld, nk + row(u, T, t0) * D, D, c, D, R);
  __syncthreads();
  tiles_n<1, 2>(R, M, [&]<int NI>(int m0, int n0) {
    Acc<1, NI> acc;
    acc.zero();
    mma_acc<1, NI, false, false>(acc, Nk, ld, Af, lm, m0, n0, D);
    acc.each2(m0, n0, [&](int, int t, int m, float& v0, float& v1) {
      *reinterpret_cast<float2*>(Wf + t * (M + 8) + m) = make_float2(v0, v1);
    });
  });
  __syncthreads();
  for (int t = warp; t < R; t += nw) {
    float x[NPL];
    if (t < c) {
      load_vec(x, Wf + t * (M + 8), M);
      warp_softmax(x, M);
      store_vec(write + row(u, T, t0 + t) * M, x, M);
    } else {
#pragma unroll
      for (int i = 0; i < NPL; ++i) x[i] = 0.f;
    }
    store_vec(Wf + t * (M + 8), x, M);
    store_bf16_row(Wb + t * lm, x, M);
  }
  __syncthreads();
  for (int m = threadIdx.x; m < M; m += blockDim.x) {
    float s = 0.f;
    for (int t = 0; t < c; ++t) s += Wf[t * (M + 8) + m];
    bsum[((int64_t)u * bl.nb + n) * M + m] = s;
  }
  if (!with_residual) return;
  const float ek = 1.f + .25f * tanhf(residual_raw[(j * H + h) * 2 + 0]);
  const float ev = 1.f + .25f * tanhf(residual_raw[(j * H + h) * 2 + 1]);
  // rk = write A_f^T, key_{j+1} = key - ek rk
  tiles_n<1, 2>(R, D, [&]<int NI>(int m0, int n0) {
    Acc<1, NI> acc;
    float2 kk[Acc<1, NI>::kPairs];
    acc.each2(m0, n0, [&](int p, int t, int d, float&, float&) {
      if (t < c) kk[p] = tc::ld2(key + row(u, T, t0 + t) * D + d);
    });
    acc.zero();
    mma_acc<1, NI, false, true>(acc, Wb, lm, Af, lm, m0, n0, M);
    acc.each2(m0, n0, [&](int p, int t, int d, float& v0, float& v1) {
      if (t < c) tc::st2(key_next + row(u, T, t0 + t) * D + d, kk[p].x - ek * v0, kk[p].y - ek * v1);
    });
  });
  // rv = write B_f, val_{j+1} = val - ev rv
  tiles_n<1, 2>(R, Dv, [&]<int NI>(int m0, int n0) {
    Acc<1, NI> acc;
    float2 xv[Acc<1, NI>::kPairs];
    acc.each2(m0, n0, [&](int p, int t, int vv, float&, float&) {
      if (t < c) xv[p] = tc::ld2(val + row(u, T, t0 + t) * Dv + vv);
    });
    acc.zero();
    mma_acc<1, NI, false, false>(acc, Wb, lm, Bf, lv, m0, n0, M);
    acc.each2(m0, n0, [&](int p, int t, int vv, float& v0, float& v1) {
      if (t < c) tc::st2(val_next + row(u, T, t0 + t) * Dv + vv, xv[p].x - ev * v0, xv[p].y - ev * v1);
    });
  });
}

// Cooperative staging of the reader inputs of a 64-token tile (all warps, float4, every
// incoming message's loads in flight together): inc[t][m] = sum_a w_a msg_a[t][m] and, when
// given, a second [rows x M] fp32 tile; rows t >= c are zero.
GPA_DEV void stage_incoming(float* inc, const BridgeIn& in, const float* w, int64_t r0, int c,
                            int M, int ld) {  // ld: row stride of inc
  const int m4 = M >> 2;
  for (int i = threadIdx.x; i < R * m4; i += blockDim.x) {
    const int t = i / m4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (t < c) {
      float4 x[kMaxIn];
      float f[kMaxIn];  // edge weight, times the source norm for the product reader
#pragma unroll
      for (int a = 0; a < kMaxIn; ++a)
        if (a < in.n) {
          x[a] = *reinterpret_cast<const float4*>(in.msg[a] + r0 * M + 4 * i);
          f[a] = in.mode != GPA_B200_READER_TANH ? w[a] * in.ln[a][r0 + t] : w[a];
        }
#pragma unroll
      for (int a = 0; a < kMaxIn; ++a)
        if (a < in.n) {
          acc.x += f[a] * x[a].x;
          acc.y += f[a] * x[a].y;
          acc.z += f[a] * x[a].z;
          acc.w += f[a] * x[a].w;
        }
    }
    *reinterpret_cast<float4*>(inc + t * ld + 4 * i - t * M) = acc;
  }
}

GPA_DEV void stage_rows(float* dst, const float* src, int c, int M) {
  const int m4 = M >> 2;
  for (int i = threadIdx.x; i < R * m4; i += blockDim.x)
    *reinterpret_cast<float4*>(dst + 4 * i) =
        i / m4 < c ? *reinterpret_cast<const float4*>(src + 4 * i) : make_float4(0.f, 0.f, 0.f, 0.f);
}

// reader_row_fwd with the row's logits and weighted incoming message in shared memory; for
// the product reader base += e^{clamp(g)} (M inc - log1p(counts) when marginal), cnt the
// row's counts
template <int N>
GPA_DEV void reader_row_fwd_s(float (&base)[N], const float* lg, const float* incr,
                              int M, bool has_in, float rg, int mode, const float* cnt) {
  load_vec(base, lg, M);
  if (has_in && mode != GPA_B200_READER_TANH) {
    float inc[N], cn[N];
    load_vec(inc, incr, M);
    if (mode == GPA_B200_READER_MARGINAL) load_vec(cn, cnt, M);
    const float ge = product_gain(rg);
#pragma unroll
    for (int i = 0; i < N; ++i)
      base[i] += ge * (M * inc[i] - (mode == GPA_B200_READER_MARGINAL ? log1pf(cn[i]) : 0.f));
  } else if (has_in) {
    const int lane = threadIdx.x & 31;
    float inc[N];
    load_vec(inc, incr, M);
    float mean = 0.f;
#pragma unroll
    for (int i = 0; i < N; ++i)
      if (lane + 32 * i < M) mean += inc[i];
    mean = warp_sum(mean) / M;
    float var = 0.f;
#pragma unroll
    for (int i = 0; i < N; ++i)
      if (lane + 32 * i < M) {
        inc[i] -= mean;
        var += inc[i] * inc[i];
      }
    var = warp_sum(var) / M;
    const float sd = rsqrtf(var + kCenterEps);
#pragma unroll
    for (int i = 0; i < N; ++i) base[i] += rg * tanhf(inc[i] * sd);
  }
  warp_softmax(base, M);
}

// reader_row_bwd up to dz (the gradient of the weighted incoming message), which the caller
// scatters to the messages and edge weights.  Product reader: dz = e^{clamp(g)} M db, and the
// gain's gradient sum db (M inc - log1p(counts)) e^{g} inside the clamp (cnt: the row's counts).
template <int N>
GPA_DEV void reader_row_bwd_s(float (&db)[N], float (&dz)[N], const float (&r)[N],
                              const float (&dr)[N],
                              const float* incr, int M, bool has_in, float rg, float& rg_acc,
                              int mode, const float* cnt) {
  const int lane = threadIdx.x & 31;
  softmax_bwd(db, r, dr, M);
#pragma unroll
  for (int i = 0; i < N; ++i) dz[i] = 0.f;
  if (!has_in) return;
  if (mode != GPA_B200_READER_TANH) {
    float inc[N], cn[N];
    load_vec(inc, incr, M);
    if (mode == GPA_B200_READER_MARGINAL) load_vec(cn, cnt, M);
    const float ge = product_gain(rg);
    float gp = 0.f;
#pragma unroll
    for (int i = 0; i < N; ++i) {
      const float t = M * inc[i] - (mode == GPA_B200_READER_MARGINAL ? log1pf(cn[i]) : 0.f);
      if (lane + 32 * i < M) gp += db[i] * t;
      dz[i] = ge * M * db[i];
    }
    rg_acc += warp_sum(gp) * ge * product_gain_live(rg);
    return;
  }
  float inc[N];
  load_vec(inc, incr, M);
  float mean = 0.f;
#pragma unroll
  for (int i = 0; i < N; ++i)
    if (lane + 32 * i < M) mean += inc[i];
  mean = warp_sum(mean) / M;
  float var = 0.f;
#pragma unroll
  for (int i = 0; i < N; ++i)
    if (lane + 32 * i < M) {
      inc[i] -= mean;
      var += inc[i] * inc[i];
    }
  var = warp_sum(var) / M;
  const float sd = rsqrtf(var + kCenterEps);
  float rgp = 0.f, dsum = 0.f;
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const float tz = tanhf(inc[i] * sd);
    if (lane + 32 * i < M) rgp += db[i] * tz;
    dz[i] = rg * db[i] * (1.f - tz * tz);
    if (lane + 32 * i < M) dsum += dz[i] * inc[i];
  }
  rg_acc += warp_sum(rgp);
  dsum = warp_sum(dsum);
  const float dvar = dsum * -0.5f * sd * sd * sd;
  float dmean = 0.f;
#pragma unroll
  for (int i = 0; i < N; ++i) {
    dz[i] = dz[i] * sd + dvar * 2.f * inc[i] / M;
    if (lane + 32 * i < M) dmean += dz[i];
  }
  dmean = warp_sum(dmean) / M;
#pragma unroll
  for (int i = 0; i < N; ++i) dz[i] -= dmean;
}

// ------------------------------------------------------------------ bridge

struct LBridge {
  size_t Rf, ARQ, Hb, Wbuf, Of, total;
  __host__ __device__ LBridge(int D, int M, int) {
    Carve c;
    Rf = c.take(4 * R * (M + 8));  // fp32 tiles with row stride M + 8
    ARQ = c.take(2 * R * ld16(M + D));
    Hb = c.take(2 * R * ld16(2 * M));
    const size_t w1 = 2 * M * ld16(2 * M), w2 = 2 * (2 * M) * ld16(M), w3 = 2 * (M + D) * ld16(M);
    size_t w = w1 > w2 ? w1 : w2;
    w = w > w3 ? w : w3;
    Wbuf = c.take(w);
    Of = c.take(4 * R * (M + 8));
    total = c.off;
  }
};

template <int NPL>
__global__ void __launch_bounds__(512) tk_bridge(
    int U, int T, int H, int D, int M, int L, int j, BridgeIn in, const float* edge_logits,
    const float* relation_gain, const float* route_up, const float* route_down,
    const float* route_mlp_gain, const float* Wrs, const float* Wqs, float qs,
    const float* logits, const float* qf, float* r_out, float* hp_out, float* mlp_out,
    float* route_out, float* qoh, float* qon) {
  const int ntile = (T + R - 1) / R;
  const int u = blockIdx.x / ntile, t0 = (blockIdx.x % ntile) * R;
  const int c = min(R, T - t0), h = u % H;
  const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  extern __shared__ __align__(16) unsigned char smem[];
  const LBridge Lb(D, M, 0);
  float* Rf = (float*)(smem + Lb.Rf);
  bf16* ARQ = (bf16*)(smem + Lb.ARQ);  // [route bf16 | q bf16]
  bf16* Hb = (bf16*)(smem + Lb.Hb);
  bf16* Wbuf = (bf16*)(smem + Lb.Wbuf);
  float* Of = (float*)(smem + Lb.Of);
  const int la = ld16(M + D), lh = ld16(2 * M), lm = ld16(M);
  float w[kMaxIn];
  edge_weights(in, edge_logits, H, h, w);
  const float rg = relation_gain[j * H + h];
  {
    float* Lg = (float*)(smem + Lb.Hb);  // Hb and Of are free until their GEMMs
    stage_rows(Lg, logits + row(u, T, t0) * M, c, M);
    if (in.n > 0) stage_incoming(Of, in, w, row(u, T, t0), c, M, M + 8);
  }
  __syncthreads();
  for (int t = warp; t < R; t += nw) {
    float x[NPL];
    if (t < c) {
      const int64_t o = row(u, T, t0 + t);
      reader_row_fwd_s(x, (const float*)(smem + Lb.Hb) + t * M, Of + t * (M + 8), M, in.n > 0, rg,
                       in.mode, in.counts ? in.counts + o * M : nullptr);
      store_vec(r_out + o * M, x, M);
    } else {
#pragma unroll
      for (int i = 0; i < NPL; ++i) x[i] = 0.f;
    }
    store_vec(Rf + t * (M + 8), x, M);
    store_bf16_row(ARQ + t * la, x, M);
  }
  tile_to_bf16(ARQ + M, la, qf + row(u, T, t0) * D, D, c, D, R);
  tile_to_bf16(Wbuf, lh, route_up + (int64_t)h * M * 2 * M, 2 * M, M, 2 * M, M);
  __syncthreads();  // the staged rows in Hb are dead below
  // hp = r U ; hidden = gelu(hp)
  tiles_n<1, 2>(R, 2 * M, [&]<int NI>(int m0, int n0) {
    Acc<1, NI> acc;
    acc.zero();
    mma_acc<1, NI, false, false>(acc, ARQ, la, Wbuf, lh, m0, n0, M);
    acc.each2(m0, n0, [&](int, int t, int rr, float& v0, float& v1) {
      if (t < c) tc::st2(hp_out + row(u, T, t0 + t) * 2 * M + rr, v0, v1);
      *reinterpret_cast<__nv_bfloat162*>(Hb + t * lh + rr) = __floats2bfloat162_rn(gelu(v0), gelu(v1));
    });
  });
  __syncthreads();
  tile_to_bf16(Wbuf, lm, route_down + (int64_t)h * 2 * M * M, M, 2 * M, M, 2 * M);
  __syncthreads();
  const float mg = route_mlp_gain[j * H + h];
  // mlp = hidden D ; route = r + mg mlp
  tiles_n<1, 2>(R, M, [&]<int NI>(int m0, int n0) {
    Acc<1, NI> acc;
    acc.zero();
    mma_acc<1, NI, false, false>(acc, Hb, lh, Wbuf, lm, m0, n0, 2 * M);
    acc.each2(m0, n0, [&](int, int t, int m, float& v0, float& v1) {
      const float2 rf = *reinterpret_cast<const float2*>(Rf + t * (M + 8) + m);
      const float route0 = rf.x + mg * v0, route1 = rf.y + mg * v1;
      if (t < c) {
        const int64_t o = row(u, T, t0 + t) * M + m;
        tc::st2(mlp_out + o, v0, v1);
        tc::st2(route_out + o, route0, route1);
      }
      *reinterpret_cast<__nv_bfloat162*>(ARQ + t * la + m) = __floats2bfloat162_rn(route0, route1);
    });
  });
  __syncthreads();
  tile_to_bf16(Wbuf, lm, Wrs + (int64_t)h * M * M, M, M, M, M);
  tile_to_bf16(Wbuf + M * lm, lm, Wqs + (int64_t)h * D * M, M, D, M, D, qs);
  __syncthreads();
  // qo = route W_rs + qs q W_qs
  tiles_n<1, 2>(R, M, [&]<int NI>(int m0, int n0) {
    Acc<1, NI> acc;
    acc.zero();
    mma_acc<1, NI, false, false>(acc, ARQ, la, Wbuf, lm, m0, n0, M + D);
    acc.each2(m0, n0, [&](int, int t, int m, float& v0, float& v1) {
      *reinterpret_cast<float2*>(Of + t * (M + 8) + m) = make_float2(v0, v1);
    });
  });
  __syncthreads();
  for (int t = warp; t < c; t += nw) {
    const int64_t o = row(u, T, t0 + t);
    float x[NPL];
    load_vec(x, Of + t * (M + 8), M);
    const float a = warp_norm(x, M);
    const float ia = 1.f / fmaxf(a, kUnitEps);
#pragma unroll
    for (int i = 0; i < NPL; ++i) x[i] *= ia;
    store_vec(qoh + o * M, x, M);
    if ((threadIdx.x & 31) == 0) qon[o] = a;
  }
}

struct LBridgeBwd {
  size_t Qb, Ql, Rf, Rb, Hb, Hl, Wbuf, red, qn, total;
  __host__ __device__ LBridgeBwd(int D, int M, int) {
    Carve c;
    Qb = c.take(2 * R * ld16(M));
    Ql = c.take(2 * R * ld16(M));
    Rf = c.take(4 * R * M);
    Rb = c.take(2 * R * ld16(M));
    Hb = c.take(2 * R * ld16(2 * M));
    Hl = c.take(2 * R * ld16(2 * M));
    const size_t w1 = 2 * (M + D) * ld16(M), w2 = 2 * (2 * M) * ld16(M), w3 = 2 * M * ld16(2 * M);
    size_t w = w1 > w2 ? w1 : w2;
    w = w > w3 ? w : w3;
    w = w > 4 * R * M ? w : 4 * R * M;  // also holds the dz rows of the reader backward
    Wbuf = c.take(w);
    red = c.take(4 * 32);
    qn = c.take(4 * R);
    total = c.off;
  }
};

template <int NPL>
__global__ void __launch_bounds__(512) tk_bridge_bwd(
    int U, int T, int H, int D, int M, int L, int j, BridgeIn in, const float* edge_logits,
    const float* relation_gain, const float* route_up, const float* route_down,
    const float* route_mlp_gain, const float* Wrs, const float* Wqs, float qs,
    const float* logits, const float* r_in, const float* hp, const float* mlp, const float* qoh,
    const float* qon, const float* dqoh, float* dqo_out, float* droute_out, float* dhp_out,
    float* dlogits, float* dq_direct, double* scal, double* scalE, int E) {
  const int ntile = (T + R - 1) / R;
  const int u = blockIdx.x / ntile, t0 = (blockIdx.x % ntile) * R;
  const int c = min(R, T - t0), h = u % H;
  const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5, lane = threadIdx.x & 31;
  extern __shared__ __align__(16) unsigned char smem[];
  const LBridgeBwd Lb(D, M, 0);
  bf16* Qb = (bf16*)(smem + Lb.Qb);
  bf16* Ql = (bf16*)(smem + Lb.Ql);
  float* Rf = (float*)(smem + Lb.Rf);
  bf16* Rb = (bf16*)(smem + Lb.Rb);
  bf16* Hb = (bf16*)(smem + Lb.Hb);
  bf16* Hl = (bf16*)(smem + Lb.Hl);
  bf16* Wbuf = (bf16*)(smem + Lb.Wbuf);
  float* red = (float*)(smem + Lb.red);
  float* qn = (float*)(smem + Lb.qn);
  const int lm = ld16(M), lh = ld16(2 * M);
  // qoh, dqoh and qon of the tile staged in Rf / Hb / qn (free until their GEMMs)
  stage_rows(Rf, qoh + row(u, T, t0) * M, c, M);
  stage_rows((float*)Hb, dqoh + row(u, T, t0) * M, c, M);
  for (int t = threadIdx.x; t < R; t += blockDim.x) qn[t] = t < c ? qon[row(u, T, t0 + t)] : 0.f;
  __syncthreads();
  for (int t = warp; t < R; t += nw) {
    float dx[NPL];
    if (t < c) {
      const int64_t o = row(u, T, t0 + t);
      float y[NPL], dy[NPL];
      load_vec(y, Rf + t * M, M);
      load_vec(dy, (const float*)Hb + t * M, M);
      unit_bwd(dx, y, dy, qn[t], M);
      store_vec(dqo_out + o * M, dx, M);
    } else {
#pragma unroll
      for (int i = 0; i < NPL; ++i) dx[i] = 0.f;
    }
    store_split_row(Qb + t * lm, Ql + t * lm, dx, M);
  }
  tile_to_bf16(Wbuf, lm, Wrs + (int64_t)h * M * M, M, M, M, M);
  tile_to_bf16(Wbuf + M * lm, lm, Wqs + (int64_t)h * D * M, M, D, M, D, qs);
  __syncthreads();  // staged rows in Rf / Hb are dead below
  // droute = dqo W_rs^T
  tiles_n<1, 2>(R, M, [&]<int NI>(int m0, int n0) {
    Acc<1, NI> acc;
    acc.zero();
    tc::mma_acc3<1, NI, false, true>(acc, Qb, Ql, lm, Wbuf, nullptr, lm, m0, n0, M);
    acc.each2(m0, n0, [&](int, int t, int m, float& v0, float& v1) {
      *reinterpret_cast<float2*>(Rf + t * M + m) = make_float2(v0, v1);
      *reinterpret_cast<__nv_bfloat162*>(Rb + t * lm + m) = __floats2bfloat162_rn(v0, v1);
      if (t < c) tc::st2(droute_out + row(u, T, t0 + t) * M + m, v0, v1);
    });
  });
  // dq_direct += qs dqo W_qs^T
  tiles_n<1, 2>(R, D, [&]<int NI>(int m0, int n0) {
    Acc<1, NI> acc;
    float2 dq[Acc<1, NI>::kPairs];
    acc.each2(m0, n0, [&](int p, int t, int d, float&, float&) {
      if (t < c) dq[p] = tc::ld2(dq_direct + row(u, T, t0 + t) * D + d);
    });
    acc.zero();
    tc::mma_acc3<1, NI, false, true>(acc, Qb, Ql, lm, Wbuf + M * lm, nullptr, lm, m0, n0, M);
    acc.each2(m0, n0, [&](int p, int t, int d, float& v0, float& v1) {
      if (t < c) tc::st2(dq_direct + row(u, T, t0 + t) * D + d, dq[p].x + v0, dq[p].y + v1);
    });
  });
  __syncthreads();
  {
    float part = 0.f;
    const float* mr = mlp + row(u, T, t0) * M;  // c rows, contiguous
    for (int i = 4 * threadIdx.x; i < c * M; i += 4 * blockDim.x) {
      const float4 a = *reinterpret_cast<const float4*>(mr + i);
      const float4 r4 = *reinterpret_cast<const float4*>(Rf + i);
      part += a.x * r4.x + a.y * r4.y + a.z * r4.z + a.w * r4.w;
    }
    const float s = block_sum(part, red);
    if (threadIdx.x == 0) atomicAdd(&scal[((int64_t)u * L + j) * kNScal + kS_MlpGain], (double)s);
  }
  tile_to_bf16(Wbuf, lm, route_down + (int64_t)h * 2 * M * M, M, 2 * M, M, 2 * M);
  __syncthreads();
  const float mg = route_mlp_gain[j * H + h];
  // dhp = mg (droute D^T) o gelu'(hp)
  tiles_n<1, 2>(R, 2 * M, [&]<int NI>(int m0, int n0) {
    Acc<1, NI> acc;
    float2 hv[Acc<1, NI>::kPairs];
    acc.each2(m0, n0, [&](int p, int t, int rr, float&, float&) {
      if (t < c) hv[p] = tc::ld2(hp + row(u, T, t0 + t) * 2 * M + rr);
    });
    acc.zero();
    mma_acc<1, NI, false, true>(acc, Rb, lm, Wbuf, lm, m0, n0, M);
    acc.each2(m0, n0, [&](int p, int t, int rr, float& v0, float& v1) {
      float x0 = 0.f, x1 = 0.f;
      if (t < c) {
        x0 = mg * v0 * gelu_grad(hv[p].x);
        x1 = mg * v1 * gelu_grad(hv[p].y);
        tc::st2(dhp_out + row(u, T, t0 + t) * 2 * M + rr, x0, x1);
      }
      tc::split2(x0, x1, Hb + t * lh + rr, Hl + t * lh + rr);
    });
  });
  __syncthreads();
  tile_to_bf16(Wbuf, lh, route_up + (int64_t)h * M * 2 * M, 2 * M, M, 2 * M, M);
  __syncthreads();
  // dr = droute + dhp U^T
  tiles_n<1, 2>(R, M, [&]<int NI>(int m0, int n0) {
    Acc<1, NI> acc;
    acc.zero();
    tc::mma_acc3<1, NI, false, true>(acc, Hb, Hl, lh, Wbuf, nullptr, lh, m0, n0, 2 * M);
    acc.each2(m0, n0, [&](int, int t, int m, float& v0, float& v1) {
      float2* p = reinterpret_cast<float2*>(Rf + t * M + m);
      const float2 x = *p;
      *p = make_float2(x.x + v0, x.y + v1);
    });
  });
  __syncthreads();
  float w[kMaxIn];
  edge_weights(in, edge_logits, H, h, w);
  const float rg = relation_gain[j * H + h];
  // reader backward: incoming and route rows staged in Hb / Hl, dz rows into Wbuf
  float* Inc = (float*)Hb;
  float* Rr = (float*)Hl;
  float* DZ = (float*)Wbuf;
  if (in.n > 0) stage_incoming(Inc, in, w, row(u, T, t0), c, M, M);
  stage_rows(Rr, r_in + row(u, T, t0) * M, c, M);
  __syncthreads();
  float rg_acc = 0.f;
  for (int t = warp; t < R; t += nw) {
    float dz[NPL];
    if (t < c) {
      float r[NPL], dr[NPL], db[NPL];
      load_vec(r, Rr + t * M, M);
      load_vec(dr, Rf + t * M, M);
      reader_row_bwd_s(db, dz, r, dr, Inc + t * M, M, in.n > 0, rg, rg_acc, in.mode,
                       in.counts ? in.counts + row(u, T, t0 + t) * M : nullptr);
      store_vec(dlogits + row(u, T, t0 + t) * M, db, M);
    } else {
#pragma unroll
      for (int i = 0; i < NPL; ++i) dz[i] = 0.f;
    }
    store_vec(DZ + t * M, dz, M);
  }
  if (in.n == 0) return;
  if (lane == 0) atomicAdd(&scal[((int64_t)u * L + j) * kNScal + kS_RelGain], (double)rg_acc);
  __syncthreads();
  if (in.mode != GPA_B200_READER_TANH) {
    // product reader, a warp per row: with s_a = dz . msg_a and the source norm n_a of the row,
    // dmsg_a = w_a n_a dz, d edge-weight_a += n_a s_a, dn_a += w_a s_a
    for (int a = 0; a < in.n; ++a) {
      float part = 0.f;
      for (int t = warp; t < c; t += nw) {
        const int64_t o = row(u, T, t0 + t);
        float z[NPL], x[NPL], dm[NPL];
        load_vec(z, DZ + t * M, M);
        load_vec(x, in.msg[a] + o * M, M);
        const float na = in.ln[a][o], s = warp_dot(z, x, M);
#pragma unroll
        for (int i = 0; i < NPL; ++i) dm[i] = w[a] * na * z[i];
        store_vec(in.dmsg[a] + o * M, dm, M);
        if (lane == 0) {
          part += na * s;
          in.dln[a][o] += w[a] * s;
        }
      }
      const float tot = block_sum(part, red);
      if (threadIdx.x == 0)
        atomicAdd(&scalE[((int64_t)u * E + in.edge[a]) * kNEdge + kE_W], (double)tot);
    }
    return;
  }
  // dmsg_a = w_a dz ; d edge-weight_a = sum dz o msg_a
  const int m4 = M >> 2;
  const int64_t r0 = row(u, T, t0) * M;
  for (int a = 0; a < in.n; ++a) {
    float part = 0.f;
    for (int i = threadIdx.x; i < c * m4; i += blockDim.x) {
      const float4 z = *reinterpret_cast<const float4*>(DZ + 4 * i);
      const float4 x = *reinterpret_cast<const float4*>(in.msg[a] + r0 + 4 * i);
      *reinterpret_cast<float4*>(in.dmsg[a] + r0 + 4 * i) =
          make_float4(w[a] * z.x, w[a] * z.y, w[a] * z.z, w[a] * z.w);
      part += z.x * x.x + z.y * x.y + z.z * x.z + z.w * x.w;
    }
    const float tot = block_sum(part, red);
    if (threadIdx.x == 0)
      atomicAdd(&scalE[((int64_t)u * E + in.edge[a]) * kNEdge + kE_W], (double)tot);
  }
}

// ------------------------------------------------------------- post backward

struct LPostBwd {
  // Bf is dead once dW is formed: dLb takes its place; Wf and dWf are dead after the
  // softmax backward rows: Nk is loaded there (the M = 64 layout then fits two CTAs per SM)
  size_t Af, Bf, dLb, Wb, Wf, dWf, Nk, dKb, dVb, red, total;
  __host__ __device__ LPostBwd(int D, int Dv, int M) {
    Carve c;
    Af = c.take(2 * D * ld16(M));
    const size_t sb = 2 * M * ld16(Dv), sl = 2 * R * ld16(M);
    Bf = dLb = c.take(sb > sl ? sb : sl);
    Wb = c.take(2 * R * ld16(M));
    const size_t sw = 2 * 4 * R * M, sn = 2 * R * ld16(D);
    Wf = Nk = c.take(sw > sn ? sw : sn);
    dWf = Wf + 4 * R * M;
    dKb = c.take(2 * R * ld16(D));
    dVb = c.take(2 * R * ld16(Dv));
    red = c.take(4 * 34);
    total = c.off;
  }
};

template <int NPL>
__global__ void __launch_bounds__(512) tk_post_bwd(
    int U, Blocks bl, int post, int offset, int H, int D, int Dv, int M, int L, int j,
    int with_residual, const float* nk, const float* write, const float* Abnd, const float* Bbnd,
    const float* fzA, const float* fzB, const float* residual_raw, const float* dkey,
    const float* dval, float* dwrite, float* dnk, float* extA, float* extB, float* dfzA,
    float* dfzB, double* scal) {
  const int u = blockIdx.x / bl.nb, n = blockIdx.x % bl.nb, T = bl.T;
  const int t0 = bl.start(n), c = bl.end(n) - t0, h = u % H;
  const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  extern __shared__ __align__(16) unsigned char smem[];
  const LPostBwd Lp(D, Dv, M);
  bf16* Af = (bf16*)(smem + Lp.Af);
  bf16* Bf = (bf16*)(smem + Lp.Bf);
  bf16* Wb = (bf16*)(smem + Lp.Wb);
  float* Wf = (float*)(smem + Lp.Wf);
  float* dWf = (float*)(smem + Lp.dWf);
  bf16* dKb = (bf16*)(smem + Lp.dKb);
  bf16* dVb = (bf16*)(smem + Lp.dVb);
  bf16* Nk = (bf16*)(smem + Lp.Nk);
  bf16* dLb = (bf16*)(smem + Lp.dLb);
  float* red = (float*)(smem + Lp.red);
  const int lm = ld16(M), ld = ld16(D), lv = ld16(Dv);
  const bool fz0 = (n == 0 && offset != 0);
  const float ek = 1.f + .25f * tanhf(residual_raw[(j * H + h) * 2 + 0]);
  const float ev = 1.f + .25f * tanhf(residual_raw[(j * H + h) * 2 + 1]);
  tile_to_bf16(Af, lm, frozen_at(Abnd, fz0 ? fzA : nullptr, u, n, bl.nb, post, (int64_t)D * M), M,
               D, M, D);
  tile_to_bf16(Wb, lm, write + row(u, T, t0) * M, M, c, M, R);
  for (int i = 4 * threadIdx.x; i < R * M; i += 4 * blockDim.x) {
    const bool in = i < c * M;  // rows t < c are contiguous from t0
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 a = in ? *reinterpret_cast<const float4*>(write + row(u, T, t0) * M + i) : z;
    const float4 b4 = in ? *reinterpret_cast<const float4*>(dwrite + row(u, T, t0) * M + i) : z;
    *reinterpret_cast<float4*>(Wf + i) = a;
    *reinterpret_cast<float4*>(dWf + i) = b4;
  }
  if (with_residual) {
    tile_to_bf16(Bf, lv, frozen_at(Bbnd, fz0 ? fzB : nullptr, u, n, bl.nb, post, (int64_t)M * Dv),
                 Dv, M, Dv, M);
    tile_to_bf16(dKb, ld, dkey + row(u, T, t0) * D, D, c, D, R, -ek);
    tile_to_bf16(dVb, lv, dval + row(u, T, t0) * Dv, Dv, c, Dv, R, -ev);
  }
  if (threadIdx.x < 34) red[threadIdx.x] = 0.f;
  __syncthreads();
  if (with_residual) {
    // d eta_k = -sum dk . (write A_f^T) ; d eta_v = -sum dv . (write B_f)
    float pk = 0.f, pv = 0.f;
    tiles_n<1, 2>(R, D, [&]<int NI>(int m0, int n0) {
      Acc<1, NI> acc;
      float2 dk[Acc<1, NI>::kPairs];
      acc.each2(m0, n0, [&](int p, int t, int d, float&, float&) {
        dk[p] = t < c ? tc::ld2(dkey + row(u, T, t0 + t) * D + d) : make_float2(0.f, 0.f);
      });
      acc.zero();
      mma_acc<1, NI, false, true>(acc, Wb, lm, Af, lm, m0, n0, M);
      acc.each2(m0, n0, [&](int p, int, int, float& v0, float& v1) {
        pk += v0 * dk[p].x + v1 * dk[p].y;
      });
    });
    tiles_n<1, 2>(R, Dv, [&]<int NI>(int m0, int n0) {
      Acc<1, NI> acc;
      float2 dv[Acc<1, NI>::kPairs];
      acc.each2(m0, n0, [&](int p, int t, int vv, float&, float&) {
        dv[p] = t < c ? tc::ld2(dval + row(u, T, t0 + t) * Dv + vv) : make_float2(0.f, 0.f);
      });
      acc.zero();
      mma_acc<1, NI, false, false>(acc, Wb, lm, Bf, lv, m0, n0, M);
      acc.each2(m0, n0, [&](int p, int, int, float& v0, float& v1) {
        pv += v0 * dv[p].x + v1 * dv[p].y;
      });
    });
    pk = warp_sum(pk);
    pv = warp_sum(pv);
    if ((threadIdx.x & 31) == 0) {
      atomicAdd(&red[32], pk);
      atomicAdd(&red[33], pv);
    }
    // dW += (-ek dk) A_f + (-ev dv) B_f^T
    tiles_n<1, 2>(R, M, [&]<int NI>(int m0, int n0) {
      Acc<1, NI> acc;
      acc.each2(m0, n0, [&](int, int t, int m, float& v0, float& v1) {
        const float2 x = *reinterpret_cast<const float2*>(dWf + t * M + m);
        v0 = x.x;
        v1 = x.y;
      });
      mma_acc<1, NI, false, false>(acc, dKb, ld, Af, lm, m0, n0, D);
      mma_acc<1, NI, false, true>(acc, dVb, lv, Bf, lv, m0, n0, Dv);
      acc.each2(m0, n0, [&](int, int t, int m, float& v0, float& v1) {
        *reinterpret_cast<float2*>(dWf + t * M + m) = make_float2(v0, v1);
      });
    });
  }
  __syncthreads();
  if (with_residual && threadIdx.x == 0) {
    atomicAdd(&scal[((int64_t)u * L + j) * kNScal + kS_EtaK], -(double)red[32]);
    atomicAdd(&scal[((int64_t)u * L + j) * kNScal + kS_EtaV], -(double)red[33]);
  }
  for (int t = warp; t < R; t += nw) {
    float y[NPL], dy[NPL], dx[NPL];
    load_vec(y, Wf + t * M, M);
    load_vec(dy, dWf + t * M, M);
    softmax_bwd(dx, y, dy, M);
    store_bf16_row(dLb + t * lm, dx, M);
  }
  __syncthreads();  // Wf / dWf are dead: the Nk tile goes there
  tile_to_bf16(Nk, ld, nk + row(u, T, t0) * D, D, c, D, R);
  // dnk = dlw A_f^T
  tiles_n<1, 2>(R, D, [&]<int NI>(int m0, int n0) {
    Acc<1, NI> acc;
    acc.zero();
    mma_acc<1, NI, false, true>(acc, dLb, lm, Af, lm, m0, n0, M);
    acc.each2(m0, n0, [&](int, int t, int d, float& v0, float& v1) {
      if (t < c) tc::st2(dnk + row(u, T, t0 + t) * D + d, v0, v1);
    });
  });
  __syncthreads();  // Nk
  float* ta = fz0 ? dfzA + (int64_t)u * D * M
                  : extA + ((int64_t)u * (bl.nb + 1) + n + post) * D * M;
  float* tb = fz0 ? dfzB + (int64_t)u * M * Dv
                  : extB + ((int64_t)u * (bl.nb + 1) + n + post) * M * Dv;
  // dA_f += nk^T dlw + (-ek dk)^T write
  tiles_n<1, 2>(D, M, [&]<int NI>(int m0, int n0) {
    Acc<1, NI> acc;
    float2 pa[Acc<1, NI>::kPairs];
    acc.each2(m0, n0, [&](int p, int d, int m, float&, float&) { pa[p] = tc::ld2(ta + d * M + m); });
    acc.zero();
    mma_acc<1, NI, true, false>(acc, Nk, ld, dLb, lm, m0, n0, R);
    if (with_residual) mma_acc<1, NI, true, false>(acc, dKb, ld, Wb, lm, m0, n0, R);
    acc.each2(m0, n0, [&](int p, int d, int m, float& v0, float& v1) {
      tc::st2(ta + d * M + m, pa[p].x + v0, pa[p].y + v1);
    });
  });
  if (with_residual) {
    // dB_f += write^T (-ev dv)
    tiles_n<1, 2>(M, Dv, [&]<int NI>(int m0, int n0) {
      Acc<1, NI> acc;
      float2 pb[Acc<1, NI>::kPairs];
      acc.each2(m0, n0, [&](int p, int m, int vv, float&, float&) {
        pb[p] = tc::ld2(tb + m * Dv + vv);
      });
      acc.zero();
      mma_acc<1, NI, true, false>(acc, Wb, lm, dVb, lv, m0, n0, R);
      acc.each2(m0, n0, [&](int p, int m, int vv, float& v0, float& v1) {
        tc::st2(tb + m * Dv + vv, pb[p].x + v0, pb[p].y + v1);
      });
    });
  }
}

// ------------------------------------------------------------- prep backward

struct LPrepBwd {
  size_t Dsb, Cb, Wg4, total;
  __host__ __device__ LPrepBwd(int D, int M, int) {
    Carve c;
    Dsb = c.take(2 * R * ld16(M));
    Cb = c.take(2 * M * ld16(D));
    Wg4 = c.take(4 * 4 * D);
    total = c.off;
  }
};

template <int NPL>
__global__ void __launch_bounds__(512, 2) tk_prep_bwd(int U, int T, int H, int D, int M,
                                                   const float* C, const float* Wg,
                                                   float beta_max, int pos_none, const float* raw4,
                                                   const float* nk, const float* kn,
                                                   const float* ns, const float* sn,
                                                   const float* dgates, const float* dnk,
                                                   const float* dns, float* dslot, float* d4out,
                                                   float* dkey) {
  const int ntile = (T + R - 1) / R;
  const int u = blockIdx.x / ntile, t0 = (blockIdx.x % ntile) * R;
  const int c = min(R, T - t0), h = u % H;
  const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5, lane = threadIdx.x & 31;
  extern __shared__ __align__(16) unsigned char smem[];
  const LPrepBwd Lp(D, M, 0);
  bf16* Dsb = (bf16*)(smem + Lp.Dsb);
  bf16* Cb = (bf16*)(smem + Lp.Cb);
  const int lm = ld16(M);
  tile_to_bf16(Cb, ld16(D), C + (int64_t)h * M * D, D, M, D, M);
  float* Wg4 = (float*)(smem + Lp.Wg4);
  for (int i = threadIdx.x; i < D; i += blockDim.x)
    *reinterpret_cast<float4*>(Wg4 + 4 * i) = *reinterpret_cast<const float4*>(Wg + ((int64_t)h * D + i) * 4);
  __syncthreads();
  for (int t = warp; t < R; t += nw) {
    float base[NPL];
    if (t < c) {
      const int64_t o = row(u, T, t0 + t);
      // every global read of the row first (the stores below may alias the inputs)
      const float4 r4 = *reinterpret_cast<const float4*>(raw4 + o * 4);
      const float4 g4 = *reinterpret_cast<const float4*>(dgates + o * 4);
      float y[NPL], dy[NPL], dx[NPL];
      load_vec(y, ns + o * M, M);
      load_vec(dy, dns + o * M, M);
      load_vec(base, dslot + o * M, M);
      float a[NPL], da[NPL], dkx[NPL], cur[NPL];
      load_vec(a, nk + o * D, D);
      load_vec(da, dnk + o * D, D);
      load_vec(cur, dkey + o * D, D);
      const float sno = sn[o], kno = kn[o];
      float d4[4] = {0.f, 0.f, 0.f, 0.f};
      const float r4v[4] = {r4.x, r4.y, r4.z, r4.w};
      const float dg[4] = {g4.x, g4.y, g4.z, g4.w};
      if (!pos_none) {
        if (softplus(r4v[0]) <= 10.f) d4[0] = -dg[0] * sigmoid(r4v[0]);
        if (softplus(r4v[2]) <= 10.f) d4[2] = -dg[2] * sigmoid(r4v[2]);
      }
      const float s1 = sigmoid(r4v[1]), s3 = sigmoid(r4v[3]);
      d4[1] = dg[1] * beta_max * s1 * (1.f - s1);
      d4[3] = dg[3] * beta_max * s3 * (1.f - s3);
      if (lane < 4) d4out[o * 4 + lane] = d4[lane];
      unit_bwd(dx, y, dy, sno, M);
#pragma unroll
      for (int i = 0; i < NPL; ++i) base[i] += dx[i];
      store_vec(dslot + o * M, base, M);
#pragma unroll
      for (int i = 0; i < NPL; ++i) {
        const int d = lane + 32 * i;
        if (d < D) {
          const float4 w4 = *reinterpret_cast<const float4*>(Wg4 + d * 4);
          da[i] += d4[0] * w4.x + d4[1] * w4.y + d4[2] * w4.z + d4[3] * w4.w;
        }
      }
      unit_bwd(dkx, a, da, kno, D);
#pragma unroll
      for (int i = 0; i < NPL; ++i) cur[i] += dkx[i];
      store_vec(dkey + o * D, cur, D);
    } else {
#pragma unroll
      for (int i = 0; i < NPL; ++i) base[i] = 0.f;
    }
    store_bf16_row(Dsb + t * lm, base, M);
  }
  __syncthreads();
  // dkey += dslot C
  tiles_n<1, 2>(R, D, [&]<int NI>(int m0, int n0) {
    Acc<1, NI> acc;
    float2 dk[Acc<1, NI>::kPairs];
    acc.each2(m0, n0, [&](int p, int t, int d, float&, float&) {
      if (t < c) dk[p] = tc::ld2(dkey + row(u, T, t0 + t) * D + d);
    });
    acc.zero();
    mma_acc<1, NI, false, false>(acc, Dsb, lm, Cb, ld16(D), m0, n0, M);
    acc.each2(m0, n0, [&](int p, int t, int d, float& v0, float& v1) {
      if (t < c) tc::st2(dkey + row(u, T, t0 + t) * D + d, dk[p].x + v0, dk[p].y + v1);
    });
  });
}

// -------------------------------------------- parameter-gradient reductions

constexpr int kOTile = 64;     // output tile unit (P and Q)
constexpr int kORows = 64;     // token rows per step
constexpr int kOSplit = 2048;  // tokens per CTA of a 64 x 64 output tile

// out[h] (P x Q) += cscale * scale[h] * sum_{b,t} X^T Y over the rows of head h; P, Q
// multiples of 16.  Operands are hi/lo bf16 pairs (sums run over every token).  A CTA owns a
// (64 WP) x (64 WQ) output tile, WP * WQ <= 2: wide X or Y operands are read by fewer CTAs
// (a 128 x 64 tile reads 192 values per token where two 64 x 64 tiles read 256).
template <int WP, int WQ>
struct LOuter {
  size_t Xh, Xl, Yh, Yl, total;
  __host__ __device__ LOuter(int, int, int) {
    Carve c;
    Xh = c.take(2 * kORows * ld16(kOTile * WP));
    Xl = c.take(2 * kORows * ld16(kOTile * WP));
    Yh = c.take(2 * kORows * ld16(kOTile * WQ));
    Yl = c.take(2 * kORows * ld16(kOTile * WQ));
    total = c.off;
  }
};

template <int WP, int WQ>
__global__ void __launch_bounds__(256, 2) tk_head_outer(int B, int T, int H, const float* X,
                                                        int P, int xmode, const float* Y, int Q,
                                                        const float* scale,
                                                        int64_t scale_stride, float cscale,
                                                        float* out, int split) {
  constexpr int TP = kOTile * WP, TQ = kOTile * WQ;
  const int h = blockIdx.x;
  const int tq = (Q + TQ - 1) / TQ;
  const int p0 = (blockIdx.y / tq) * TP, q0 = (blockIdx.y % tq) * TQ;
  const int pw = min(TP, P - p0), qw = min(TQ, Q - q0);
  const int64_t total = (int64_t)B * T;
  const int64_t r0 = (int64_t)blockIdx.z * split;
  const int64_t r1 = min(total, r0 + split);
  extern __shared__ __align__(16) unsigned char smem[];
  const LOuter<WP, WQ> Lo(0, 0, 0);
  bf16* Xh = (bf16*)(smem + Lo.Xh);
  bf16* Xl = (bf16*)(smem + Lo.Xl);
  bf16* Yh = (bf16*)(smem + Lo.Yh);
  bf16* Yl = (bf16*)(smem + Lo.Yl);
  const int lx = ld16(TP), ly = ld16(TQ);
  // the output tile is (TP / 16) x (TQ / 16) tiles of 16 x 16; warp w owns tiles w + 8 i
  constexpr int kT = 2 * WP * WQ, kTN = TQ / 16;
  const int w = threadIdx.x >> 5;
  Acc<1, 1> acc[kT];
  int tm[kT], tn[kT];
  bool act[kT];
#pragma unroll
  for (int i = 0; i < kT; ++i) {
    const int idx = w + 8 * i;
    tm[i] = (idx / kTN) * 16;
    tn[i] = (idx % kTN) * 16;
    act[i] = tm[i] < pw && tn[i] < qw;
    acc[i].zero();
  }
  // Each thread moves 4 WP float4 of X and 4 WQ of Y per 64-row step; the next step's values
  // are loaded into registers while the current step's MMAs run.
  constexpr int kPX = kORows * (TP / 4) / 256, kPY = kORows * (TQ / 4) / 256;
  float4 xn[kPX], yn[kPY];
  auto fetch = [&](int64_t rr) {
    const int rows = (int)min((int64_t)kORows, r1 - rr);
    const int b0 = (int)(rr / T), t0 = (int)(rr - (int64_t)b0 * T);  // one division per step
    auto at = [&](int rw) {  // token row of step row rw (rows of a step cross few sequence ends)
      int b = b0, t = t0 + rw;
      while (t >= T) {
        t -= T;
        ++b;
      }
      return row(b * H + h, T, t);
    };
#pragma unroll
    for (int j = 0; j < kPX; ++j) {
      const int i = threadIdx.x + j * 256;
      const int rw = i / (TP / 4), cc = (i % (TP / 4)) * 4;
      xn[j] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (rw < rows && cc < pw) xn[j] = *reinterpret_cast<const float4*>(X + at(rw) * P + p0 + cc);
    }
#pragma unroll
    for (int j = 0; j < kPY; ++j) {
      const int i = threadIdx.x + j * 256;
      const int rw = i / (TQ / 4), cc = (i % (TQ / 4)) * 4;
      yn[j] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (rw < rows && cc < qw) yn[j] = *reinterpret_cast<const float4*>(Y + at(rw) * Q + q0 + cc);
    }
  };
  if (r0 < r1) fetch(r0);
  for (int64_t rr = r0; rr < r1; rr += kORows) {
    __syncthreads();  // the previous step's MMAs are done with the tiles
#pragma unroll
    for (int j = 0; j < kPX; ++j) {
      const int i = threadIdx.x + j * 256;
      const int rw = i / (TP / 4), cc = (i % (TP / 4)) * 4;
      float4 xv = xn[j];
      if (xmode == 1) {
        xv.x = gelu(xv.x);
        xv.y = gelu(xv.y);
        xv.z = gelu(xv.z);
        xv.w = gelu(xv.w);
      }
      tc::put4(Xh, Xl, rw * lx + cc, xv);
    }
#pragma unroll
    for (int j = 0; j < kPY; ++j) {
      const int i = threadIdx.x + j * 256;
      const int rw = i / (TQ / 4), cc = (i % (TQ / 4)) * 4;
      tc::put4(Yh, Yl, rw * ly + cc, yn[j]);
    }
    __syncthreads();
    if (rr + kORows < r1) fetch(rr + kORows);
#pragma unroll
    for (int i = 0; i < kT; ++i)
      if (act[i])
        tc::mma_acc3<1, 1, true, false>(acc[i], Xh, Xl, lx, Yh, Yl, ly, tm[i], tn[i], kORows);
  }
  const float s = cscale * (scale ? scale[(int64_t)h * scale_stride] : 1.f);
  float* o = out + (int64_t)h * P * Q;
#pragma unroll
  for (int i = 0; i < kT; ++i)
    if (act[i])
      acc[i].each(tm[i], tn[i], [&](int p, int q, float& v) {
        atomicAdd(&o[(p0 + p) * Q + q0 + q], s * v);
      });
}

// per-lane registers of a warp-held row of n <= 256 values; the row kernels are compiled for
// each count so that their per-row loops have no predicated-off iterations
inline int npl_of(int n) { return n <= 32 ? 1 : n <= 64 ? 2 : n <= 128 ? 4 : 8; }
#define TK_NPL(kern, n) \
  (npl_of(n) == 1 ? kern<1> : npl_of(n) == 2 ? kern<2> : npl_of(n) == 4 ? kern<4> : kern<8>)

template <class Kern, class... Args>
cudaError_t tk_launch(const char* name, Kern k, dim3 grid, size_t smem, cudaStream_t st,
                      Args... args) {
  if (grid.x == 0 || grid.y == 0 || grid.z == 0) return cudaSuccess;
  if (smem > 227 * 1024) return cudaErrorInvalidConfiguration;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  // a CTA that needs more than half of an SM's shared memory runs alone on its SM: give it
  // 16 warps (the per-row loops and tiles adapt to blockDim); head_outer's tiling is fixed
  // at 8 warps and its shared memory is small
  const int threads = smem > 113 * 1024 ? 512 : 256;
  Launch scope(name, st);
  k<<<grid, threads, smem, st>>>(args...);
  return cudaGetLastError();
}

}  // namespace

cudaError_t tc_level_prep(int U, int T, int H, int D, int M, const float* key, const float* C,
                          const float* Wg, const float* gbias, float beta_max, int pos_none,
                          float* nk, float* kn, float* slot, float* ns, float* sn, float* raw4,
                          float* gates, cudaStream_t st) {
  const int ntile = (T + R - 1) / R;
  return tk_launch("tc_level_prep", TK_NPL(tk_level_prep, D > M ? D : M), dim3(U * ntile), smem_of<LPrep>(D, M, 0), st,
                   U, T, H, D, M, key, C, Wg, gbias, beta_max, pos_none, nk, kn, slot, ns, sn,
                   raw4, gates);
}

cudaError_t tc_level_post(int U, const Blocks& bl, int post, int H, int D, int Dv, int M,
                          int with_residual, const float* nk, const float* key, const float* val,
                          const float* Abnd, const float* Bbnd, const float* fzA, const float* fzB,
                          const float* residual_raw, int j, float* write, float* bsum,
                          float* key_next, float* val_next, cudaStream_t st) {
  return tk_launch("tc_level_post", TK_NPL(tk_level_post, M), dim3(U * bl.nb), smem_of<LPost>(D, Dv, M), st,
                   U, bl, post, H, D, Dv, M, with_residual, nk, key, val, Abnd, Bbnd, fzA, fzB,
                   residual_raw, j, write, bsum, key_next, val_next);
}

cudaError_t tc_bridge(int U, int T, int H, int D, int M, int L, int j, const BridgeIn& in,
                      const float* edge_logits, const float* relation_gain, const float* route_up,
                      const float* route_down, const float* route_mlp_gain, const float* Wrs,
                      const float* Wqs, float qs, const float* logits, const float* qf, float* r,
                      float* hp, float* mlp, float* route, float* qoh, float* qon,
                      cudaStream_t st) {
  const int ntile = (T + R - 1) / R;
  return tk_launch("tc_bridge", TK_NPL(tk_bridge, M), dim3(U * ntile), smem_of<LBridge>(D, M, 0), st, U, T,
                   H, D, M, L, j, in, edge_logits, relation_gain, route_up, route_down,
                   route_mlp_gain, Wrs, Wqs, qs, logits, qf, r, hp, mlp, route, qoh, qon);
}

cudaError_t tc_bridge_bwd(int U, int T, int H, int D, int M, int L, int j, const BridgeIn& in,
                          const float* edge_logits, const float* relation_gain,
                          const float* route_up, const float* route_down,
                          const float* route_mlp_gain, const float* Wrs, const float* Wqs,
                          float qs, const float* logits, const float* r, const float* hp,
                          const float* mlp, const float* qoh, const float* qon, const float* dqoh,
                          float* dqo, float* droute, float* dhp, float* dlogits, float* dq_direct,
                          double* scal, double* scalE, int E, cudaStream_t st) {
  const int ntile = (T + R - 1) / R;
  return tk_launch("tc_bridge_bwd", TK_NPL(tk_bridge_bwd, M), dim3(U * ntile), smem_of<LBridgeBwd>(D, M, 0),
                   st, U, T, H, D, M, L, j, in, edge_logits, relation_gain, route_up, route_down,
                   route_mlp_gain, Wrs, Wqs, qs, logits, r, hp, mlp, qoh, qon, dqoh, dqo, droute,
                   dhp, dlogits, dq_direct, scal, scalE, E);
}

cudaError_t tc_post_bwd(int U, const Blocks& bl, int post, int offset, int H, int D, int Dv,
                        int M, int L, int j, int with_residual, const float* nk,
                        const float* write, const float* Abnd, const float* Bbnd,
                        const float* fzA, const float* fzB, const float* residual_raw,
                        const float* dkey, const float* dval, float* dwrite, float* dnk,
                        float* extA, float* extB, float* dfzA, float* dfzB, double* scal,
                        cudaStream_t st) {
  return tk_launch("tc_post_bwd", TK_NPL(tk_post_bwd, M), dim3(U * bl.nb), smem_of<LPostBwd>(D, Dv, M), st,
                   U, bl, post, offset, H, D, Dv, M, L, j, with_residual, nk, write, Abnd, Bbnd,
                   fzA, fzB, residual_raw, dkey, dval, dwrite, dnk, extA, extB, dfzA, dfzB, scal);
}

cudaError_t tc_prep_bwd(int U, int T, int H, int D, int M, const float* C, const float* Wg,
                        float beta_max, int pos_none, const float* raw4, const float* nk,
                        const float* kn, const float* ns, const float* sn, const float* dgates,
                        const float* dnk, const float* dns, float* dslot, float* d4, float* dkey,
                        cudaStream_t st) {
  const int ntile = (T + R - 1) / R;
  return tk_launch("tc_prep_bwd", TK_NPL(tk_prep_bwd, D > M ? D : M), dim3(U * ntile), smem_of<LPrepBwd>(D, M, 0), st, U,
                   T, H, D, M, C, Wg, beta_max, pos_none, raw4, nk, kn, ns, sn, dgates, dnk, dns,
                   dslot, d4, dkey);
}

cudaError_t tc_head_outer(int B, int T, int H, const float* X, int P, int xmode, const float* Y,
                          int Q, const float* scale, int64_t scale_stride, float cscale,
                          float* out, cudaStream_t st) {
  if (tc5_outer_enabled())
    return tc5_head_outer_launch(B, T, H, X, P, xmode, Y, Q, scale, scale_stride, cscale, out, st);
  const int64_t total = (int64_t)B * T;
  // the wider operand gets the 128-wide side of the CTA tile; half the tokens per CTA keep
  // the CTA count (and its work) as with 64 x 64 tiles
  const int wp = P >= 2 * kOTile && P >= Q ? 2 : 1, wq = wp == 1 && Q >= 2 * kOTile ? 2 : 1;
  const int split = kOSplit / (wp * wq);
  const int tp = (P + kOTile * wp - 1) / (kOTile * wp), tq = (Q + kOTile * wq - 1) / (kOTile * wq);
  dim3 grid(H, tp * tq, (unsigned)((total + split - 1) / split));
  if (wp == 2)
    return tk_launch("tc_head_outer", tk_head_outer<2, 1>, grid, smem_of<LOuter<2, 1>>(0, 0, 0), st,
                     B, T, H, X, P, xmode, Y, Q, scale, scale_stride, cscale, out, split);
  if (wq == 2)
    return tk_launch("tc_head_outer", tk_head_outer<1, 2>, grid, smem_of<LOuter<1, 2>>(0, 0, 0), st,
                     B, T, H, X, P, xmode, Y, Q, scale, scale_stride, cscale, out, split);
  return tk_launch("tc_head_outer", tk_head_outer<1, 1>, grid, smem_of<LOuter<1, 1>>(0, 0, 0), st,
                   B, T, H, X, P, xmode, Y, Q, scale, scale_stride, cscale, out, split);
}

}  // namespace gpa
