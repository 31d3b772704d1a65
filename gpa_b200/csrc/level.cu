// Level, relation-reader and output kernels of the DenseGPA core (SIMT fp32).
//
// Reference formulas (src/gpa/attention.py): gates :161-174, slot :176-184,
// residual :190-194, base logits :196-204, relation gates :206-223, dense
// reader (bridge) :225-262, lag-block writes :314-316, output mix :340-341.
#include "level.cuh"
#include "rowops.cuh"

namespace gpa {
namespace {

// ------------------------------------------------------------------ forward

// x rounded to the input dtype (the reference rounds its rotated queries back to it)
GPA_DEV float round_in(float x, int dt) {
  if (dt == GPA_B200_BF16) return __bfloat162float(__float2bfloat16(x));
  if (dt == GPA_B200_F16) return __half2float(__float2half(x));
  return x;
}

// one warp per (u, t): fp32 copies, unit-normalised q; with rope_pos0 >= 0 the query is first
// rotated (adjacent pairs, token t at rope_pos0 + t; src/gpa/ops.py:117-132)
__global__ void k_input(const void* q, const void* k, const void* v, int dt, int B, int T, int H,
                        int D, int Dv, float* qf, float* qh, float* qn, float* key0, float* val0,
                        int64_t rope_pos0) {
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  const int U = B * H;
  if (w >= U * T) return;
  const int u = w / T, t = w - u * T, b = u / H, h = u - b * H;
  const int64_t src = ((int64_t)b * T + t) * H + h;
  float ss = 0.f;
  for (int i = 0; i < (D + 31) / 32; ++i) {  // warp-uniform trip count (pair shuffles)
    const int d = lane + 32 * i;
    float x = d < D ? load_in(q, src * D + d, dt) : 0.f;
    if (rope_pos0 >= 0) {
      const float other = __shfl_xor_sync(0xffffffffu, x, 1);
      float c, s;
      rope_cs(rope_pos0 + t, d, D, c, s);
      x = round_in((d & 1) == 0 ? x * c - other * s : other * s + x * c, dt);
    }
    if (d < D) {
      qf[(int64_t)w * D + d] = x;
      ss += x * x;
      key0[(int64_t)w * D + d] = load_in(k, src * D + d, dt);
    }
  }
  const float nrm = sqrtf(warp_sum(ss));
  const float inv = 1.f / fmaxf(nrm, kUnitEps);
  for (int d = lane; d < D; d += 32) qh[(int64_t)w * D + d] = qf[(int64_t)w * D + d] * inv;
  if (lane == 0) qn[w] = nrm;
  for (int d = lane; d < Dv; d += 32) val0[(int64_t)w * Dv + d] = load_in(v, src * Dv + d, dt);
}

// CTA per (u, 64-token tile): u(k), slot = k C^T, u(slot), gates.
__global__ void __launch_bounds__(256) k_level_prep(int U, int T, int H, int D, int M,
                                                    const float* key, const float* C,
                                                    const float* Wg, const float* gbias,
                                                    float beta_max, int pos_none, float* nk,
                                                    float* kn, float* slot, float* ns, float* sn,
                                                    float* raw4, float* gates) {
  const int ntile = (T + kRowsPerTile - 1) / kRowsPerTile;
  const int u = blockIdx.x / ntile, t0 = (blockIdx.x % ntile) * kRowsPerTile;
  const int c = min(kRowsPerTile, T - t0), h = u % H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  extern __shared__ float sm[];
  float* Kt = sm;                       // 64*D
  float* St = Kt + kRowsPerTile * D;    // 64*M
  load_tile(Kt, key + row(u, T, t0) * D, c, D, D);
  __syncthreads();
  const float* wg = Wg + (int64_t)h * D * 4;
  for (int t = warp; t < c; t += nw) {
    float ss = 0.f;
    for (int d = lane; d < D; d += 32) ss += Kt[t * D + d] * Kt[t * D + d];
    const float nrm = sqrtf(warp_sum(ss));
    const float inv = 1.f / fmaxf(nrm, kUnitEps);
    float r[4] = {0.f, 0.f, 0.f, 0.f};
    for (int d = lane; d < D; d += 32) {
      const float x = Kt[t * D + d] * inv;
      nk[row(u, T, t0 + t) * D + d] = x;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) r[cc] += x * wg[d * 4 + cc];
    }
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) r[cc] = warp_sum(r[cc]) + gbias[h * 4 + cc];
    if (lane == 0) {
      const int64_t o = row(u, T, t0 + t);
      kn[o] = nrm;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) raw4[o * 4 + cc] = r[cc];
      const float gi = pos_none ? 0.f : -fminf(softplus(r[0]), 10.f);
      const float go = pos_none ? 0.f : -fminf(softplus(r[2]), 10.f);
      gates[o * 4 + 0] = gi;
      gates[o * 4 + 1] = beta_max * sigmoid(r[1]);
      gates[o * 4 + 2] = go;
      gates[o * 4 + 3] = beta_max * sigmoid(r[3]);
    }
  }
  const float* Ch = C + (int64_t)h * M * D;
  block_gemm<2, 4>(
      c, M, D, [&](int t, int d) { return Kt[t * D + d]; },
      [&](int d, int m) { return Ch[m * D + d]; },
      [&](int t, int m, float acc) {
        St[t * M + m] = acc;
        slot[row(u, T, t0 + t) * M + m] = acc;
      });
  __syncthreads();
  for (int t = warp; t < c; t += nw) {
    float ss = 0.f;
    for (int m = lane; m < M; m += 32) ss += St[t * M + m] * St[t * M + m];
    const float nrm = sqrtf(warp_sum(ss));
    const float inv = 1.f / fmaxf(nrm, kUnitEps);
    for (int m = lane; m < M; m += 32) ns[row(u, T, t0 + t) * M + m] = St[t * M + m] * inv;
    if (lane == 0) sn[row(u, T, t0 + t)] = nrm;
  }
}

GPA_DEV const float* frozen_ptr(const float* bnd, const float* fz, int u, int n, int nb, int post,
                                int64_t sz) {
  if (n == 0 && fz) return fz + (int64_t)u * sz;
  return bnd + ((int64_t)u * (nb + 1) + n + post) * sz;
}

// CTA per (u, lag block): writes from the frozen snapshots, residual key/value.
__global__ void __launch_bounds__(256) k_level_post(
    int U, Blocks bl, int post, int H, int D, int Dv, int M, int with_residual, const float* nk,
    const float* key, const float* val, const float* Abnd, const float* Bbnd, const float* fzA,
    const float* fzB, const float* residual_raw, int j, float* write, float* bsum,
    float* key_next, float* val_next) {
  const int u = blockIdx.x / bl.nb, n = blockIdx.x % bl.nb, T = bl.T;
  const int t0 = bl.start(n), c = bl.end(n) - t0, h = u % H;
  const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  extern __shared__ float sm[];
  float* As = sm;               // D*M
  float* Bs = As + D * M;       // M*Dv
  float* Wr = Bs + M * Dv;      // 64*M
  const float* Af = frozen_ptr(Abnd, fzA, u, n, bl.nb, post, (int64_t)D * M);
  const float* Bf = frozen_ptr(Bbnd, fzB, u, n, bl.nb, post, (int64_t)M * Dv);
  load_tile(As, Af, D, M, M);
  if (with_residual) load_tile(Bs, Bf, M, Dv, Dv);
  __syncthreads();
  const float* nkb = nk + row(u, T, t0) * D;
  block_gemm<2, 4>(
      c, M, D, [&](int t, int d) { return nkb[t * D + d]; },
      [&](int d, int m) { return As[d * M + m]; },
      [&](int t, int m, float acc) { Wr[t * M + m] = acc; });
  __syncthreads();
  for (int t = warp; t < c; t += nw) {
    float x[kMaxPerLane];
    load_vec(x, Wr + t * M, M);
    warp_softmax(x, M);
    store_vec(Wr + t * M, x, M);
    store_vec(write + row(u, T, t0 + t) * M, x, M);
  }
  __syncthreads();
  for (int m = threadIdx.x; m < M; m += blockDim.x) {
    float s = 0.f;
    for (int t = 0; t < c; ++t) s += Wr[t * M + m];
    bsum[((int64_t)u * bl.nb + n) * M + m] = s;
  }
  if (!with_residual) return;
  const float ek = 1.f + .25f * tanhf(residual_raw[(j * H + h) * 2 + 0]);
  const float ev = 1.f + .25f * tanhf(residual_raw[(j * H + h) * 2 + 1]);
  block_gemm<2, 4>(
      c, D, M, [&](int t, int m) { return Wr[t * M + m]; },
      [&](int m, int d) { return As[d * M + m]; },
      [&](int t, int d, float acc) {
        const int64_t o = row(u, T, t0 + t) * D + d;
        key_next[o] = key[o] - ek * acc;
      });
  block_gemm<2, 4>(
      c, Dv, M, [&](int t, int m) { return Wr[t * M + m]; },
      [&](int m, int v) { return Bs[m * Dv + v]; },
      [&](int t, int v, float acc) {
        const int64_t o = row(u, T, t0 + t) * Dv + v;
        val_next[o] = val[o] - ev * acc;
      });
}

// CTA per (u, lag block): counts = n0 + cumsum(write); logits; u(local); u(write).
// dst[i] = src[i], i < n: float4 when `vec` (n, and both pointers' offsets, multiples of 4
// floats; the caller checks M % 4 == 0), else scalar
GPA_DEV void copy_rows(float* dst, const float* src, int n, bool vec) {
  if (vec) {
    for (int i = 4 * threadIdx.x; i < n; i += 4 * blockDim.x)
      *reinterpret_cast<float4*>(dst + i) = *reinterpret_cast<const float4*>(src + i);
  } else {
    for (int i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
  }
}

// Sum over the earlier lag blocks (before < 0: the later ones) of per-block vectors
// [U, NB, M], all threads: partial sums in `part` (blockDim floats), result in pre[M].
GPA_DEV void block_prefix(const float* bsum, int u, int nb, int first, int last, int M,
                          float* pre, float* part) {
  const int G = blockDim.x / M;  // thread groups per slot (M <= blockDim)
  const int m = threadIdx.x % M, g = threadIdx.x / M;
  float acc = 0.f;
  if (g < G) {
    const float* base = bsum + (int64_t)u * nb * M + m;
    int p = first + g;
    for (; p + 3 * G < last; p += 4 * G)
      acc += (base[(int64_t)p * M] + base[(int64_t)(p + G) * M]) +
             (base[(int64_t)(p + 2 * G) * M] + base[(int64_t)(p + 3 * G) * M]);
    for (; p < last; p += G) acc += base[(int64_t)p * M];
  }
  part[threadIdx.x] = acc;
  __syncthreads();
  for (int mm = threadIdx.x; mm < M; mm += blockDim.x) {
    float s = 0.f;
    for (int i = 0; i < G; ++i) s += part[i * M + mm];
    pre[mm] = s;
  }
  __syncthreads();
}

// CTA per (u, lag block), level j: running counts from the incoming cache and the earlier
// blocks, base logits, the normalised local distribution and write (relation queries / keys).
// The block's write tile is staged in shared memory (rows t < c contiguous from t0).
template <int NPL>  // registers per lane of an M-long row
__global__ void __launch_bounds__(256) k_counts(int U, Blocks bl, int H, int M, float read_scale,
                                                const float* count_gain_raw, int j,
                                                const float* n0, const float* bsum,
                                                const float* write, const float* raw,
                                                float* counts, float* logits, float* lh,
                                                float* ln, float* wh, float* wn, float* n_final,
                                                const float* corr, const float* moment_gain) {
  const int u = blockIdx.x / bl.nb, n = blockIdx.x % bl.nb, T = bl.T;
  const int t0 = bl.start(n), c = bl.end(n) - t0, h = u % H;
  const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  extern __shared__ __align__(16) float smc[];
  float* Wt = smc;                     // [64 x M] write rows of the block
  float* Ct = Wt + kRowsPerTile * M;   // [64 x M] counts
  float* pre = Ct + kRowsPerTile * M;  // [M]
  float* part = pre + M;               // [blockDim]
  const int64_t r0 = row(u, T, t0) * M;
  const bool vec = M % 4 == 0;
  copy_rows(Wt, write + r0, c * M, vec);
  block_prefix(bsum, u, bl.nb, 0, n, M, pre, part);
  for (int m = threadIdx.x; m < M; m += blockDim.x) {
    float acc = n0[(int64_t)u * M + m] + pre[m];
    for (int t = 0; t < c; ++t) {
      acc += Wt[t * M + m];
      Ct[t * M + m] = acc;
    }
    if (n == bl.nb - 1) n_final[(int64_t)u * M + m] = acc;
  }
  __syncthreads();
  copy_rows(counts + r0, Ct, c * M, vec);
  const float gain = softplus(count_gain_raw[j * H + h]);
  for (int t = warp; t < c; t += nw) {
    const int64_t o = row(u, T, t0 + t);
    float x[NPL], w[NPL], cn[NPL];
    load_vec(x, raw + o * M, M);
    load_vec(cn, Ct + t * M, M);
    load_vec(w, Wt + t * M, M);
#pragma unroll
    for (int i = 0; i < NPL; ++i) x[i] = read_scale * x[i] + gain * log1pf(cn[i]);
    if (corr) {  // positional moments: + g_m tanh(corr / (1 + n)) (src/gpa/attention.py:202-203)
      float cr[NPL];
      load_vec(cr, corr + o * M, M);
      const float mg = moment_gain[j * H + h];
#pragma unroll
      for (int i = 0; i < NPL; ++i) x[i] += mg * tanhf(cr[i] / (1.f + cn[i]));
    }
    store_vec(logits + o * M, x, M);
    warp_softmax(x, M);
    const float a = warp_norm(x, M);
    const float ia = 1.f / fmaxf(a, kUnitEps);
#pragma unroll
    for (int i = 0; i < NPL; ++i) x[i] *= ia;
    store_vec(lh + o * M, x, M);
    const float b = warp_norm(w, M);
    const float ib = 1.f / fmaxf(b, kUnitEps);
#pragma unroll
    for (int i = 0; i < NPL; ++i) w[i] *= ib;
    store_vec(wh + o * M, w, M);
    if ((threadIdx.x & 31) == 0) {
      ln[o] = a;
      wn[o] = b;
    }
  }
}

__global__ void k_rel_gates(int U, int H, int E, int pos_none, const float* decay_raw,
                            const float* beta_raw, float* ge, float* be) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= E * U) return;
  const int e = i / U, u = i - e * U, h = u % H;
  ge[i] = pos_none ? 0.f : -softplus(decay_raw[e * H + h]);
  be[i] = sigmoid(beta_raw[e * H + h]);
}

// CTA per (u, 64-token tile), target level j: dense reader, route MLP, query projection.
__global__ void __launch_bounds__(256) k_bridge(
    int U, int T, int H, int D, int M, int L, int j, BridgeIn in, const float* edge_logits,
    const float* relation_gain, const float* route_up, const float* route_down,
    const float* route_mlp_gain, const float* Wrs, const float* Wqs, float qs,
    const float* logits, const float* qf, float* r_out, float* hp_out, float* mlp_out,
    float* route_out, float* qoh, float* qon) {
  const int ntile = (T + kRowsPerTile - 1) / kRowsPerTile;
  const int u = blockIdx.x / ntile, t0 = (blockIdx.x % ntile) * kRowsPerTile;
  const int c = min(kRowsPerTile, T - t0), h = u % H;
  const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  extern __shared__ float sm[];
  float* Rt = sm;                          // 64*M
  float* Hd = Rt + kRowsPerTile * M;       // 64*2M
  float* Mt = Hd + kRowsPerTile * 2 * M;   // 64*M
  float w[kMaxIn];
  edge_weights(in, edge_logits, H, h, w);
  const float rg = relation_gain[j * H + h];
  for (int t = warp; t < c; t += nw) {
    const int64_t o = row(u, T, t0 + t);
    float base[kMaxPerLane];
    load_vec(base, logits + o * M, M);
    if (in.n > 0 && in.mode != GPA_B200_READER_TANH) {
      // product reader: base += e^{clamp(g)} (M sum_a w_a n_a msg_a - log1p(counts) if marginal)
      float inc[kMaxPerLane], cn[kMaxPerLane];
#pragma unroll
      for (int i = 0; i < kMaxPerLane; ++i) inc[i] = 0.f;
      for (int a = 0; a < in.n; ++a) {
        float x[kMaxPerLane];
        load_vec(x, in.msg[a] + o * M, M);
        const float f = w[a] * in.ln[a][o];
#pragma unroll
        for (int i = 0; i < kMaxPerLane; ++i) inc[i] += f * x[i];
      }
      const bool marg = in.mode == GPA_B200_READER_MARGINAL;
      if (marg) load_vec(cn, in.counts + o * M, M);
      const float ge = product_gain(rg);
#pragma unroll
      for (int i = 0; i < kMaxPerLane; ++i)
        base[i] += ge * (M * inc[i] - (marg ? log1pf(cn[i]) : 0.f));
    } else if (in.n > 0) {
      float inc[kMaxPerLane];
#pragma unroll
      for (int i = 0; i < kMaxPerLane; ++i) inc[i] = 0.f;
      for (int a = 0; a < in.n; ++a) {
        float x[kMaxPerLane];
        load_vec(x, in.msg[a] + o * M, M);
#pragma unroll
        for (int i = 0; i < kMaxPerLane; ++i) inc[i] += w[a] * x[i];
      }
      const int lane = threadIdx.x & 31;
      float mean = 0.f;
#pragma unroll
      for (int i = 0; i < kMaxPerLane; ++i)
        if (lane + 32 * i < M) mean += inc[i];
      mean = warp_sum(mean) / M;
      float var = 0.f;
#pragma unroll
      for (int i = 0; i < kMaxPerLane; ++i)
        if (lane + 32 * i < M) {
          inc[i] -= mean;
          var += inc[i] * inc[i];
        }
      var = warp_sum(var) / M;
      const float sd = rsqrtf(var + kCenterEps);
#pragma unroll
      for (int i = 0; i < kMaxPerLane; ++i) base[i] += rg * tanhf(inc[i] * sd);
    }
    warp_softmax(base, M);
    store_vec(Rt + t * M, base, M);
    store_vec(r_out + o * M, base, M);
  }
  __syncthreads();
  const float* Uh = route_up + (int64_t)h * M * 2 * M;
  const float* Dh = route_down + (int64_t)h * 2 * M * M;
  block_gemm<2, 4>(
      c, 2 * M, M, [&](int t, int m) { return Rt[t * M + m]; },
      [&](int m, int r) { return Uh[m * 2 * M + r]; },
      [&](int t, int r, float acc) {
        hp_out[row(u, T, t0 + t) * 2 * M + r] = acc;
        Hd[t * 2 * M + r] = gelu(acc);
      });
  __syncthreads();
  const float mg = route_mlp_gain[j * H + h];
  block_gemm<2, 4>(
      c, M, 2 * M, [&](int t, int r) { return Hd[t * 2 * M + r]; },
      [&](int r, int m) { return Dh[r * M + m]; },
      [&](int t, int m, float acc) {
        mlp_out[row(u, T, t0 + t) * M + m] = acc;
        Mt[t * M + m] = acc;
      });
  __syncthreads();
  for (int i = threadIdx.x; i < c * M; i += blockDim.x) {
    const int t = i / M, m = i - t * M;
    const float x = Rt[i] + mg * Mt[i];
    Rt[i] = x;
    route_out[row(u, T, t0 + t) * M + m] = x;
  }
  __syncthreads();
  const float* Wr = Wrs + (int64_t)h * M * M;
  const float* Wq = Wqs + (int64_t)h * D * M;
  const float* qb = qf + row(u, T, t0) * D;
  block_gemm<2, 4>(
      c, M, M + D,
      [&](int t, int kk) { return kk < M ? Rt[t * M + kk] : qs * qb[t * D + (kk - M)]; },
      [&](int kk, int nn) { return kk < M ? Wr[kk * M + nn] : Wq[(kk - M) * M + nn]; },
      [&](int t, int nn, float acc) { Mt[t * M + nn] = acc; });
  __syncthreads();
  for (int t = warp; t < c; t += nw) {
    const int64_t o = row(u, T, t0 + t);
    float x[kMaxPerLane];
    load_vec(x, Mt + t * M, M);
    const float a = warp_norm(x, M);
    const float ia = 1.f / fmaxf(a, kUnitEps);
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) x[i] *= ia;
    store_vec(qoh + o * M, x, M);
    if ((threadIdx.x & 31) == 0) qon[o] = a;
  }
}

struct YPtrs {
  const float* y[kMaxLevels];
};

// one warp per (u, t): out = sum_j softmax_L(output_logits)_j y_j
__global__ void k_mix(int B, int T, int H, int Dv, int L, const float* output_logits, YPtrs yp,
                      void* out, int dt) {
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  const int U = B * H;
  if (w >= U * T) return;
  const int u = w / T, t = w - u * T, b = u / H, h = u - b * H;
  float ow[kMaxLevels];
  float mx = -INFINITY, s = 0.f;
  for (int j = 0; j < L; ++j) mx = fmaxf(mx, output_logits[j * H + h]);
  for (int j = 0; j < L; ++j) {
    ow[j] = __expf(output_logits[j * H + h] - mx);
    s += ow[j];
  }
  const int64_t dst = (((int64_t)b * T + t) * H + h) * Dv;
  // Dv <= 128: every level's values of the row are loaded before the first store
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int j = 0; j < L; ++j) {
    const float wj = ow[j] / s;
    const float* yj = yp.y[j] + (int64_t)w * Dv;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (lane + 32 * i < Dv) acc[i] += wj * yj[lane + 32 * i];
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (lane + 32 * i < Dv) store_out(out, dst + lane + 32 * i, acc[i], dt);
}

__global__ void k_copy(float* dst, const float* src, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = src[i];
}

__global__ void k_to_bthx(const float* src, void* dst, int dt, int B, int T, int H, int X) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)B * T * H * X) return;
  const int64_t x = i % X, r = i / X;  // r = (b*T + t)*H + h
  const int64_t h = r % H, bt = r / H, t = bt % T, b = bt / T;
  store_out(dst, i, src[(((b * H + h) * T) + t) * X + x], dt);
}

__global__ void k_add(float* dst, const float* src, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] += src[i];
}

__global__ void k_boundary(float* dst, const float* src, int U, int nb1, int idx, int64_t sz,
                           int scatter_add) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)U * sz) return;
  const int64_t u = i / sz, r = i - u * sz;
  const int64_t b = (u * nb1 + idx) * sz + r;
  if (scatter_add) dst[b] += src[i];
  else dst[i] = src[b];
}

// ----------------------------------------------------------------- backward

__global__ void k_scales(int U, int H, int L, const float* output_logits, float* ow_scale) {
  const int u = blockIdx.x * blockDim.x + threadIdx.x;
  if (u >= U) return;
  const int h = u % H;
  float mx = -INFINITY, s = 0.f;
  for (int j = 0; j < L; ++j) mx = fmaxf(mx, output_logits[j * H + h]);
  for (int j = 0; j < L; ++j) s += __expf(output_logits[j * H + h] - mx);
  for (int j = 0; j < L; ++j) ow_scale[j * U + u] = __expf(output_logits[j * H + h] - mx) / s;
}

// one warp per (u, t): fp32 unit-major dout; per-unit sum of dout . y_j
__global__ void k_mix_bwd(int B, int T, int H, int Dv, int L, const void* dout, int dt, YPtrs yp,
                          float* dout_f, double* scal) {
  // 256 threads: a warp per row; the CTA's rows (consecutive, mostly one unit) are summed in
  // shared memory first, so each level takes one double atomic per unit run, not per row
  __shared__ float red[8][kMaxLevels];
  const int wi = threadIdx.x >> 5;
  const int w = blockIdx.x * (blockDim.x >> 5) + wi, lane = threadIdx.x & 31;
  const int U = B * H;
  if (w < U * T) {
    const int u = w / T, t = w - u * T, b = u / H, h = u - b * H;
    const int64_t src = (((int64_t)b * T + t) * H + h) * Dv;
    float acc[kMaxLevels];
    for (int j = 0; j < L; ++j) acc[j] = 0.f;
    float g[4];  // Dv <= 128: the row's gradient is loaded before any store
#pragma unroll
    for (int i = 0; i < 4; ++i) g[i] = lane + 32 * i < Dv ? load_in(dout, src + lane + 32 * i, dt) : 0.f;
    for (int j = 0; j < L; ++j) {
      const float* yj = yp.y[j] + (int64_t)w * Dv;
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (lane + 32 * i < Dv) acc[j] += g[i] * yj[lane + 32 * i];
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (lane + 32 * i < Dv) dout_f[(int64_t)w * Dv + lane + 32 * i] = g[i];
    for (int j = 0; j < L; ++j) {
      const float s = warp_sum(acc[j]);
      if (lane == 0) red[wi][j] = s;
    }
  }
  __syncthreads();
  if (threadIdx.x < L) {
    const int j = threadIdx.x, w0 = blockIdx.x * (blockDim.x >> 5);
    int r = 0;
    while (r < 8 && w0 + r < U * T) {
      const int ur = (w0 + r) / T;
      double s = 0.0;
      int e = r;
      for (; e < 8 && w0 + e < U * T && (w0 + e) / T == ur; ++e) s += red[e][j];
      atomicAdd(&scal[((int64_t)ur * L + j) * kNScal + kS_OutW], s);
      r = e;
    }
  }
}

// CTA per (u, 64-token tile), level j: backward of the reader / route MLP / projections.
__global__ void __launch_bounds__(256) k_bridge_bwd(
    int U, int T, int H, int D, int M, int L, int j, BridgeIn in, const float* edge_logits,
    const float* relation_gain, const float* route_up, const float* route_down,
    const float* route_mlp_gain, const float* Wrs, const float* Wqs, float qs,
    const float* logits, const float* r_in, const float* hp, const float* mlp, const float* qoh,
    const float* qon, const float* dqoh, float* dqo_out, float* droute_out, float* dhp_out,
    float* dlogits, float* dq_direct, double* scal, double* scalE, int E) {
  const int ntile = (T + kRowsPerTile - 1) / kRowsPerTile;
  const int u = blockIdx.x / ntile, t0 = (blockIdx.x % ntile) * kRowsPerTile;
  const int c = min(kRowsPerTile, T - t0), h = u % H;
  const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5, lane = threadIdx.x & 31;
  extern __shared__ float sm[];
  float* Q = sm;                          // 64*M   dqo
  float* R = Q + kRowsPerTile * M;        // 64*M   droute -> dr
  float* Hd = R + kRowsPerTile * M;       // 64*2M  dhp
  float* red = Hd + kRowsPerTile * 2 * M; // 32
  float* ew = red + 32;                   // kMaxIn accumulators
  if (threadIdx.x < kMaxIn) ew[threadIdx.x] = 0.f;
  for (int t = warp; t < c; t += nw) {
    const int64_t o = row(u, T, t0 + t);
    float y[kMaxPerLane], dy[kMaxPerLane], dx[kMaxPerLane];
    load_vec(y, qoh + o * M, M);
    load_vec(dy, dqoh + o * M, M);
    unit_bwd(dx, y, dy, qon[o], M);
    store_vec(Q + t * M, dx, M);
    store_vec(dqo_out + o * M, dx, M);
  }
  __syncthreads();
  const float* Wr = Wrs + (int64_t)h * M * M;
  const float* Wq = Wqs + (int64_t)h * D * M;
  block_gemm<2, 4>(
      c, M, M, [&](int t, int nn) { return Q[t * M + nn]; },
      [&](int nn, int m) { return Wr[m * M + nn]; },
      [&](int t, int m, float acc) {
        R[t * M + m] = acc;
        droute_out[row(u, T, t0 + t) * M + m] = acc;
      });
  block_gemm<2, 4>(
      c, D, M, [&](int t, int nn) { return Q[t * M + nn]; },
      [&](int nn, int d) { return Wq[d * M + nn]; },
      [&](int t, int d, float acc) { dq_direct[row(u, T, t0 + t) * D + d] += qs * acc; });
  __syncthreads();
  {
    float part = 0.f;
    for (int i = threadIdx.x; i < c * M; i += blockDim.x) {
      const int t = i / M, m = i - t * M;
      part += R[i] * mlp[row(u, T, t0 + t) * M + m];
    }
    const float s = block_sum(part, red);
    if (threadIdx.x == 0) atomicAdd(&scal[((int64_t)u * L + j) * kNScal + kS_MlpGain], (double)s);
  }
  const float mg = route_mlp_gain[j * H + h];
  const float* Uh = route_up + (int64_t)h * M * 2 * M;
  const float* Dh = route_down + (int64_t)h * 2 * M * M;
  block_gemm<2, 4>(
      c, 2 * M, M, [&](int t, int m) { return R[t * M + m]; },
      [&](int m, int rr) { return Dh[rr * M + m]; },
      [&](int t, int rr, float acc) {
        const float x = mg * acc * gelu_grad(hp[row(u, T, t0 + t) * 2 * M + rr]);
        Hd[t * 2 * M + rr] = x;
        dhp_out[row(u, T, t0 + t) * 2 * M + rr] = x;
      });
  __syncthreads();
  block_gemm<2, 4>(
      c, M, 2 * M, [&](int t, int rr) { return Hd[t * 2 * M + rr]; },
      [&](int rr, int m) { return Uh[m * 2 * M + rr]; },
      [&](int t, int m, float acc) { R[t * M + m] += acc; });
  __syncthreads();
  float w[kMaxIn];
  edge_weights(in, edge_logits, H, h, w);
  const float rg = relation_gain[j * H + h];
  float rg_acc = 0.f, ew_acc[kMaxIn];
  for (int a = 0; a < kMaxIn; ++a) ew_acc[a] = 0.f;
  for (int t = warp; t < c; t += nw) {
    const int64_t o = row(u, T, t0 + t);
    float r[kMaxPerLane], dr[kMaxPerLane], db[kMaxPerLane];
    load_vec(r, r_in + o * M, M);
    load_vec(dr, R + t * M, M);
    softmax_bwd(db, r, dr, M);
    store_vec(dlogits + o * M, db, M);
    if (in.n > 0 && in.mode != GPA_B200_READER_TANH) {
      // product reader: dinc = e^{clamp(g)} M db; with s_a = dinc . msg_a and the source norm
      // n_a, dmsg_a = w_a n_a dinc, d edge-weight_a += n_a s_a, dn_a += w_a s_a
      float inc[kMaxPerLane], cn[kMaxPerLane], dz[kMaxPerLane];
#pragma unroll
      for (int i = 0; i < kMaxPerLane; ++i) inc[i] = 0.f;
      for (int a = 0; a < in.n; ++a) {
        float x[kMaxPerLane];
        load_vec(x, in.msg[a] + o * M, M);
        const float f = w[a] * in.ln[a][o];
#pragma unroll
        for (int i = 0; i < kMaxPerLane; ++i) inc[i] += f * x[i];
      }
      const bool marg = in.mode == GPA_B200_READER_MARGINAL;
      if (marg) load_vec(cn, in.counts + o * M, M);
      const float ge = product_gain(rg);
      float gp = 0.f;
#pragma unroll
      for (int i = 0; i < kMaxPerLane; ++i) {
        const float tm = M * inc[i] - (marg ? log1pf(cn[i]) : 0.f);
        if (lane + 32 * i < M) gp += db[i] * tm;
        dz[i] = ge * M * db[i];
      }
      rg_acc += warp_sum(gp) * ge * product_gain_live(rg);
      for (int a = 0; a < in.n; ++a) {
        float x[kMaxPerLane], dm[kMaxPerLane];
        load_vec(x, in.msg[a] + o * M, M);
        const float na = in.ln[a][o], s = warp_dot(dz, x, M);
#pragma unroll
        for (int i = 0; i < kMaxPerLane; ++i) dm[i] = w[a] * na * dz[i];
        store_vec(in.dmsg[a] + o * M, dm, M);
        ew_acc[a] += na * s;
        if (lane == 0) in.dln[a][o] += w[a] * s;
      }
    } else if (in.n > 0) {
      float inc[kMaxPerLane];
#pragma unroll
      for (int i = 0; i < kMaxPerLane; ++i) inc[i] = 0.f;
      for (int a = 0; a < in.n; ++a) {
        float x[kMaxPerLane];
        load_vec(x, in.msg[a] + o * M, M);
#pragma unroll
        for (int i = 0; i < kMaxPerLane; ++i) inc[i] += w[a] * x[i];
      }
      float mean = 0.f;
#pragma unroll
      for (int i = 0; i < kMaxPerLane; ++i)
        if (lane + 32 * i < M) mean += inc[i];
      mean = warp_sum(mean) / M;
      float var = 0.f;
#pragma unroll
      for (int i = 0; i < kMaxPerLane; ++i)
        if (lane + 32 * i < M) {
          inc[i] -= mean;  // centred
          var += inc[i] * inc[i];
        }
      var = warp_sum(var) / M;
      const float sd = rsqrtf(var + kCenterEps);
      float dz[kMaxPerLane], tz[kMaxPerLane];
      float rgp = 0.f, dsum = 0.f;
#pragma unroll
      for (int i = 0; i < kMaxPerLane; ++i) {
        tz[i] = tanhf(inc[i] * sd);
        if (lane + 32 * i < M) rgp += db[i] * tz[i];
        dz[i] = rg * db[i] * (1.f - tz[i] * tz[i]);
        if (lane + 32 * i < M) dsum += dz[i] * inc[i];
      }
      rg_acc += warp_sum(rgp);
      dsum = warp_sum(dsum);
      const float dvar = dsum * -0.5f * sd * sd * sd;
      float dmean = 0.f;
#pragma unroll
      for (int i = 0; i < kMaxPerLane; ++i) {
        dz[i] = dz[i] * sd + dvar * 2.f * inc[i] / M;  // dcc
        if (lane + 32 * i < M) dmean += dz[i];
      }
      dmean = warp_sum(dmean) / M;
#pragma unroll
      for (int i = 0; i < kMaxPerLane; ++i) dz[i] -= dmean;  // dinc
      for (int a = 0; a < in.n; ++a) {
        float x[kMaxPerLane], dm[kMaxPerLane];
        load_vec(x, in.msg[a] + o * M, M);
#pragma unroll
        for (int i = 0; i < kMaxPerLane; ++i) dm[i] = w[a] * dz[i];
        store_vec(in.dmsg[a] + o * M, dm, M);
        ew_acc[a] += warp_dot(dz, x, M);
      }
    }
  }
  if (lane == 0 && in.n > 0) {
    atomicAdd(&scal[((int64_t)u * L + j) * kNScal + kS_RelGain], (double)rg_acc);
    for (int a = 0; a < in.n; ++a)
      atomicAdd(&scalE[((int64_t)u * E + in.edge[a]) * kNEdge + kE_W], (double)ew_acc[a]);
  }
}

// one warp per (u, t), level j: logits / local-softmax / count-log backward.
// Row vectors of NPL values per lane (M <= 32 * NPL), sized to the level's width so that
// every row read can be in flight at once without spending occupancy.
template <int NPL>
struct RowV {
  float v[NPL];
  GPA_DEV void load(const float* p, int n) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int i = 0; i < NPL; ++i) v[i] = lane + 32 * i < n ? p[lane + 32 * i] : 0.f;
  }
  GPA_DEV void store(float* p, int n) const {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int i = 0; i < NPL; ++i)
      if (lane + 32 * i < n) p[lane + 32 * i] = v[i];
  }
  GPA_DEV float dot(const RowV& o, int n) const {
    const int lane = threadIdx.x & 31;
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NPL; ++i)
      if (lane + 32 * i < n) s += v[i] * o.v[i];
    return warp_sum(s);
  }
};

// Warp per token row, 8 rows per CTA: every global read of a row is issued before its
// stores (which may alias), and the per-block count gradients of the CTA's rows are summed
// in shared memory before one atomic per slot and block.
template <int NPL>
__global__ void __launch_bounds__(256) k_logits_bwd(
    int U, Blocks bl, int H, int M, int L, int j, float read_scale, const float* count_gain_raw,
    const float* logits, const float* counts, const float* lh, const float* ln, const float* wh,
    const float* wn, const float* dlh, const float* dwh, const float* dlogits, float* dwrite,
    float* draw, float* dn, float* dnsum, double* scal, ProductBwd pb, MomentBwd mb) {
  __shared__ float red_dn[8][32 * NPL];
  __shared__ int blk[8];
  __shared__ float red_cg[8];  // count-gain partial of each warp's row (one atomic per unit run)
  __shared__ float red_mg[8];  // the same for the moment gain
  const int T = bl.T;
  const int wi = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int w = blockIdx.x * (blockDim.x >> 5) + wi;
  const bool live = w < U * T;
  const int u = live ? w / T : 0, t = live ? w - u * T : 0, h = u % H;
  const int64_t o = (int64_t)w * M;
  if (live) {
    RowV<NPL> x, y, dy, dlg, cn, y2, dy2, dw;
    x.load(logits + o, M);
    y.load(lh + o, M);
    dy.load(dlh + o, M);
    dlg.load(dlogits + o, M);
    cn.load(counts + o, M);
    y2.load(wh + o, M);
    dy2.load(dwh + o, M);
    dw.load(dwrite + o, M);
    const float lno = ln[w], wno = wn[w];
    const float gain = softplus(count_gain_raw[j * H + h]);
    // local = softmax(logits)
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < NPL; ++i)
      if (lane + 32 * i < M) mx = fmaxf(mx, x.v[i]);
    mx = warp_max(mx);
    float se = 0.f;
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
      x.v[i] = lane + 32 * i < M ? __expf(x.v[i] - mx) : 0.f;
      se += x.v[i];
    }
    const float inv = 1.f / warp_sum(se);
#pragma unroll
    for (int i = 0; i < NPL; ++i) x.v[i] *= inv;
    // dlocal = unit backward of lh
    RowV<NPL> d1;
    if (lno > kUnitEps) {
      const float yd = y.dot(dy, M), il = 1.f / lno;
#pragma unroll
      for (int i = 0; i < NPL; ++i) d1.v[i] = (dy.v[i] - y.v[i] * yd) * il;
    } else {
#pragma unroll
      for (int i = 0; i < NPL; ++i) d1.v[i] = dy.v[i] / kUnitEps;
    }
    if (pb.dln) {  // the norm |softmax(logits)| read by the product reader: d/dp = lh
      const float dl_n = pb.dln[w];
#pragma unroll
      for (int i = 0; i < NPL; ++i) d1.v[i] += dl_n * y.v[i];
    }
    const float ge = pb.marginal ? product_gain(pb.relation_gain[j * H + h]) : 0.f;
    const float xd = x.dot(d1, M);
    RowV<NPL> dr, dnv, cr, dcr;
    if (mb.corr) cr.load(mb.corr + o, M);
    const float mg = mb.corr ? mb.moment_gain[j * H + h] : 0.f;
    float cg = 0.f, mgp = 0.f;
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
      const float dl = dlg.v[i] + x.v[i] * (d1.v[i] - xd);
      dr.v[i] = read_scale * dl;
      if (lane + 32 * i < M) cg += dl * log1pf(cn.v[i]);
      dnv.v[i] = (gain * dl - ge * dlg.v[i]) / (1.f + cn.v[i]);
      if (mb.corr) {  // + g_m tanh(corr / (1 + n)): gradients of corr, n and g_m
        const float inv = 1.f / (1.f + cn.v[i]), th = tanhf(cr.v[i] * inv);
        const float dth = dl * mg * (1.f - th * th);
        dcr.v[i] = dth * inv;
        dnv.v[i] -= dth * cr.v[i] * inv * inv;
        if (lane + 32 * i < M) mgp += dl * th;
      }
    }
    if (mb.corr) dcr.store(mb.dcorr + o, M);
    mgp = warp_sum(mgp);
    if (lane == 0) red_mg[wi] = mgp;
    dr.store(draw + o, M);
    dnv.store(dn + o, M);
    cg = warp_sum(cg);
    if (lane == 0) red_cg[wi] = cg;
    if (wno > kUnitEps) {
      const float yd = y2.dot(dy2, M), iw = 1.f / wno;
#pragma unroll
      for (int i = 0; i < NPL; ++i) dw.v[i] += (dy2.v[i] - y2.v[i] * yd) * iw;
    } else {
#pragma unroll
      for (int i = 0; i < NPL; ++i) dw.v[i] += dy2.v[i] / kUnitEps;
    }
    dw.store(dwrite + o, M);
    dnv.store(&red_dn[wi][0], M);
    if (lane == 0) blk[wi] = u * bl.nb + bl.block_of(t);
  } else if (lane == 0) {
    blk[wi] = -1;
  }
  __syncthreads();
  if (threadIdx.x == 0) {  // consecutive live rows of one unit: one double atomic per run
    const int w0 = blockIdx.x * (blockDim.x >> 5);
    int r = 0;
    while (r < 8 && w0 + r < U * T) {
      const int ur = (w0 + r) / T;
      double s = 0.0;
      int e = r;
      double sm_ = 0.0;
      for (; e < 8 && w0 + e < U * T && (w0 + e) / T == ur; ++e) {
        s += red_cg[e];
        sm_ += red_mg[e];
      }
      atomicAdd(&scal[((int64_t)ur * L + j) * kNScal + kS_CountGain], s);
      if (mb.corr) atomicAdd(&scal[((int64_t)ur * L + j) * kNScal + kS_MomentGain], sm_);
      r = e;
    }
  }
  // rows of the CTA that share (unit, block) are consecutive: one atomic per run and slot
  for (int m = threadIdx.x; m < M; m += blockDim.x) {
    int r = 0;
    while (r < 8) {
      const int b = blk[r];
      float s = 0.f;
      int e = r;
      for (; e < 8 && blk[e] == b; ++e) s += red_dn[e][m];
      if (b >= 0) atomicAdd(&dnsum[(int64_t)b * M + m], s);
      r = e;
    }
  }
}

// CTA per (u, lag block): dwrite += suffix sums of dn; dn0.  The block's dn and dwrite
// rows are staged in shared memory (rows t < c contiguous from t0).
__global__ void __launch_bounds__(256) k_counts_bwd(int U, Blocks bl, int M, const float* dn,
                                                    const float* dnsum, const float* dn_final,
                                                    float* dwrite, float* dn0) {
  const int u = blockIdx.x / bl.nb, n = blockIdx.x % bl.nb, T = bl.T;
  const int t0 = bl.start(n), c = bl.end(n) - t0;
  extern __shared__ __align__(16) float smc[];
  float* Dn = smc;                     // [64 x M]
  float* Dw = Dn + kRowsPerTile * M;   // [64 x M]
  float* suf = Dw + kRowsPerTile * M;  // [M]
  float* part = suf + M;               // [blockDim]
  const int64_t r0 = row(u, T, t0) * M;
  const bool vec = M % 4 == 0;
  copy_rows(Dn, dn + r0, c * M, vec);
  copy_rows(Dw, dwrite + r0, c * M, vec);
  block_prefix(dnsum, u, bl.nb, n + 1, bl.nb, M, suf, part);
  for (int m = threadIdx.x; m < M; m += blockDim.x) {
    float acc = (dn_final ? dn_final[(int64_t)u * M + m] : 0.f) + suf[m];
    for (int t = c - 1; t >= 0; --t) {
      acc += Dn[t * M + m];
      Dw[t * M + m] += acc;
    }
    if (n == 0) dn0[(int64_t)u * M + m] = acc;
  }
  __syncthreads();
  copy_rows(dwrite + r0, Dw, c * M, vec);
}

// CTA per (u, lag block), level j: residual + write backward; frozen-snapshot gradients.
__global__ void __launch_bounds__(256) k_post_bwd(
    int U, Blocks bl, int post, int offset, int H, int D, int Dv, int M, int L, int j,
    int with_residual, const float* nk, const float* write, const float* Abnd, const float* Bbnd,
    const float* fzA, const float* fzB, const float* residual_raw, const float* dkey,
    const float* dval, float* dwrite, float* dnk, float* extA, float* extB, float* dfzA,
    float* dfzB, double* scal) {
  const int u = blockIdx.x / bl.nb, n = blockIdx.x % bl.nb, T = bl.T;
  const int t0 = bl.start(n), c = bl.end(n) - t0, h = u % H;
  const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  extern __shared__ float sm[];
  float* As = sm;              // D*M
  float* Bs = As + D * M;      // M*Dv
  float* Wr = Bs + M * Dv;     // 64*M
  float* dW = Wr + kRowsPerTile * M;  // 64*M
  float* red = dW + kRowsPerTile * M; // 32 + 2
  const bool fz0 = (n == 0 && offset != 0);
  const float* Af = frozen_ptr(Abnd, fz0 ? fzA : nullptr, u, n, bl.nb, post, (int64_t)D * M);
  const float* Bf = frozen_ptr(Bbnd, fz0 ? fzB : nullptr, u, n, bl.nb, post, (int64_t)M * Dv);
  load_tile(As, Af, D, M, M);
  if (with_residual) load_tile(Bs, Bf, M, Dv, Dv);
  load_tile(Wr, write + row(u, T, t0) * M, c, M, M);
  load_tile(dW, dwrite + row(u, T, t0) * M, c, M, M);
  if (threadIdx.x < 34) red[threadIdx.x] = 0.f;
  __syncthreads();
  const float ek = 1.f + .25f * tanhf(residual_raw[(j * H + h) * 2 + 0]);
  const float ev = 1.f + .25f * tanhf(residual_raw[(j * H + h) * 2 + 1]);
  const float* dk = dkey + row(u, T, t0) * D;
  const float* dv = dval + row(u, T, t0) * Dv;
  if (with_residual) {
    // d eta_k = -sum dk . (A_f write), d eta_v = -sum dv . (write B_f)
    float pk = 0.f, pv = 0.f;
    block_gemm<2, 4>(
        c, D, M, [&](int t, int m) { return Wr[t * M + m]; },
        [&](int m, int d) { return As[d * M + m]; },
        [&](int t, int d, float acc) { pk += acc * dk[t * D + d]; });
    block_gemm<2, 4>(
        c, Dv, M, [&](int t, int m) { return Wr[t * M + m]; },
        [&](int m, int v) { return Bs[m * Dv + v]; },
        [&](int t, int v, float acc) { pv += acc * dv[t * Dv + v]; });
    pk = warp_sum(pk);
    pv = warp_sum(pv);
    if ((threadIdx.x & 31) == 0) {
      atomicAdd(&red[32], pk);
      atomicAdd(&red[33], pv);
    }
    // dW += -ek dk A_f - ev dv B_f^T
    block_gemm<2, 4>(
        c, M, D + Dv,
        [&](int t, int kk) { return kk < D ? -ek * dk[t * D + kk] : -ev * dv[t * Dv + (kk - D)]; },
        [&](int kk, int m) { return kk < D ? As[kk * M + m] : Bs[m * Dv + (kk - D)]; },
        [&](int t, int m, float acc) { dW[t * M + m] += acc; });
  }
  __syncthreads();
  if (with_residual && threadIdx.x == 0) {
    atomicAdd(&scal[((int64_t)u * L + j) * kNScal + kS_EtaK], -(double)red[32]);
    atomicAdd(&scal[((int64_t)u * L + j) * kNScal + kS_EtaV], -(double)red[33]);
  }
  // dlw = softmax backward (in place in dW)
  for (int t = warp; t < c; t += nw) {
    float y[kMaxPerLane], dy[kMaxPerLane], dx[kMaxPerLane];
    load_vec(y, Wr + t * M, M);
    load_vec(dy, dW + t * M, M);
    softmax_bwd(dx, y, dy, M);
    store_vec(dW + t * M, dx, M);
  }
  __syncthreads();
  const float* nkb = nk + row(u, T, t0) * D;
  // dnk = dlw A_f^T
  block_gemm<2, 4>(
      c, D, M, [&](int t, int m) { return dW[t * M + m]; },
      [&](int m, int d) { return As[d * M + m]; },
      [&](int t, int d, float acc) { dnk[row(u, T, t0 + t) * D + d] = acc; });
  // dA_f = -ek dk^T write + nk^T dlw ;  dB_f = -ev write^T dv
  float* ta = fz0 ? dfzA + (int64_t)u * D * M
                  : extA + ((int64_t)u * (bl.nb + 1) + n + post) * D * M;
  float* tb = fz0 ? dfzB + (int64_t)u * M * Dv
                  : extB + ((int64_t)u * (bl.nb + 1) + n + post) * M * Dv;
  block_gemm<2, 4>(
      D, M, with_residual ? 2 * c : c,
      [&](int d, int tt) { return tt < c ? nkb[tt * D + d] : -ek * dk[(tt - c) * D + d]; },
      [&](int tt, int m) { return tt < c ? dW[tt * M + m] : Wr[(tt - c) * M + m]; },
      [&](int d, int m, float acc) { ta[d * M + m] += acc; });
  if (with_residual) {
    block_gemm<2, 4>(
        M, Dv, c, [&](int m, int t) { return Wr[t * M + m]; },
        [&](int t, int v) { return -ev * dv[t * Dv + v]; },
        [&](int m, int v, float acc) { tb[m * Dv + v] += acc; });
  }
}

// CTA per (u, 64-token tile), level j: gates / slot / unit-norm backward into dkey.
__global__ void __launch_bounds__(256) k_prep_bwd(int U, int T, int H, int D, int M,
                                                  const float* C, const float* Wg, float beta_max,
                                                  int pos_none, const float* raw4,
                                                  const float* nk, const float* kn,
                                                  const float* ns, const float* sn,
                                                  const float* dgates, const float* dnk,
                                                  const float* dns, float* dslot, float* d4out,
                                                  float* dkey) {
  const int ntile = (T + kRowsPerTile - 1) / kRowsPerTile;
  const int u = blockIdx.x / ntile, t0 = (blockIdx.x % ntile) * kRowsPerTile;
  const int c = min(kRowsPerTile, T - t0), h = u % H;
  const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5, lane = threadIdx.x & 31;
  extern __shared__ float sm[];
  float* Ds = sm;  // 64*M  dslot (total)
  const float* wg = Wg + (int64_t)h * D * 4;
  for (int t = warp; t < c; t += nw) {
    const int64_t o = row(u, T, t0 + t);
    float d4[4];
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) d4[cc] = 0.f;
    const float* r4 = raw4 + o * 4;
    const float* dg = dgates + o * 4;
    if (!pos_none) {
      if (softplus(r4[0]) <= 10.f) d4[0] = -dg[0] * sigmoid(r4[0]);
      if (softplus(r4[2]) <= 10.f) d4[2] = -dg[2] * sigmoid(r4[2]);
    }
    {
      const float s1 = sigmoid(r4[1]), s3 = sigmoid(r4[3]);
      d4[1] = dg[1] * beta_max * s1 * (1.f - s1);
      d4[3] = dg[3] * beta_max * s3 * (1.f - s3);
    }
    if (lane < 4) d4out[o * 4 + lane] = d4[lane];
    // dslot = dslot_value + unit_bwd(ns, dns)
    float y[kMaxPerLane], dy[kMaxPerLane], dx[kMaxPerLane], base[kMaxPerLane];
    load_vec(y, ns + o * M, M);
    load_vec(dy, dns + o * M, M);
    unit_bwd(dx, y, dy, sn[o], M);
    load_vec(base, dslot + o * M, M);
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) base[i] += dx[i];
    store_vec(Ds + t * M, base, M);
    store_vec(dslot + o * M, base, M);
    // dnk_total = dnk + d4 Wg^T ; dkey += unit_bwd(nk, dnk_total)
    float a[kMaxPerLane], da[kMaxPerLane], dkx[kMaxPerLane];
    load_vec(a, nk + o * D, D);
    load_vec(da, dnk + o * D, D);
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      const int d = lane + 32 * i;
      if (d < D)
        da[i] += d4[0] * wg[d * 4] + d4[1] * wg[d * 4 + 1] + d4[2] * wg[d * 4 + 2] +
                 d4[3] * wg[d * 4 + 3];
    }
    unit_bwd(dkx, a, da, kn[o], D);
    float cur[kMaxPerLane];
    load_vec(cur, dkey + o * D, D);
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) cur[i] += dkx[i];
    store_vec(dkey + o * D, cur, D);
  }
  __syncthreads();
  const float* Ch = C + (int64_t)h * M * D;
  block_gemm<2, 4>(
      c, D, M, [&](int t, int m) { return Ds[t * M + m]; },
      [&](int m, int d) { return Ch[m * D + d]; },
      [&](int t, int d, float acc) { dkey[row(u, T, t0 + t) * D + d] += acc; });
}

// out[h] += scale[h] * sum_{b, t} X^T Y over the rows of head h.
constexpr int kHoTile = 32;
constexpr int kHoRows = 64;
constexpr int kHoSplit = 2048;  // tokens per CTA
__global__ void __launch_bounds__(256) k_head_outer(int B, int T, int H, const float* X, int P,
                                                    int xmode, const float* Y, int Q,
                                                    const float* scale, int64_t scale_stride,
                                                    float cscale, float* out) {
  const int h = blockIdx.x;
  const int tq = (Q + kHoTile - 1) / kHoTile;
  const int p0 = (blockIdx.y / tq) * kHoTile, q0 = (blockIdx.y % tq) * kHoTile;
  const int pw = min(kHoTile, P - p0), qw = min(kHoTile, Q - q0);
  const int64_t total = (int64_t)B * T;
  const int64_t r0 = (int64_t)blockIdx.z * kHoSplit;
  const int64_t r1 = min(total, r0 + kHoSplit);
  __shared__ float Xs[kHoRows * kHoTile], Ys[kHoRows * kHoTile], Acc[kHoTile * kHoTile];
  for (int i = threadIdx.x; i < kHoTile * kHoTile; i += blockDim.x) Acc[i] = 0.f;
  for (int64_t rr = r0; rr < r1; rr += kHoRows) {
    const int rows = (int)min((int64_t)kHoRows, r1 - rr);
    __syncthreads();
    for (int i = threadIdx.x; i < rows * kHoTile; i += blockDim.x) {
      const int rw = i / kHoTile, cc = i - rw * kHoTile;
      const int64_t g = rr + rw;  // (b, t) flattened
      const int b = (int)(g / T), t = (int)(g - (int64_t)b * T);
      const int64_t o = row(b * H + h, T, t);
      float x = 0.f;
      if (cc < pw) {
        if (xmode == 2) x = 1.f;
        else {
          x = X[o * P + p0 + cc];
          if (xmode == 1) x = gelu(x);
        }
      }
      Xs[i] = x;
      Ys[i] = cc < qw ? Y[o * Q + q0 + cc] : 0.f;
    }
    __syncthreads();
    block_gemm<2, 2>(
        pw, qw, rows, [&](int p, int r) { return Xs[r * kHoTile + p]; },
        [&](int r, int q) { return Ys[r * kHoTile + q]; },
        [&](int p, int q, float acc) { Acc[p * kHoTile + q] += acc; });
  }
  __syncthreads();
  const float s = cscale * (scale ? scale[(int64_t)h * scale_stride] : 1.f);
  float* o = out + (int64_t)h * P * Q;
  for (int i = threadIdx.x; i < pw * qw; i += blockDim.x) {
    const int p = i / qw, q = i - p * qw;
    atomicAdd(&o[(p0 + p) * Q + q0 + q], s * Acc[p * kHoTile + q]);
  }
}

// Gate parameter gradients of one level, one CTA per (head, batch row, 1024-token chunk):
// gw[h] (D x 4) += sum_t x_t^T y_t and gb[h] += sum_t y_t, x = u(k) rows [U,T,D], y = the four
// gate-logit gradients [U,T,4] (the gate_weight / gate_bias products of the reference's
// _gates, src/gpa/attention.py:161-174).  A warp takes every eighth row: lane l holds the
// columns l, l + 32, ... of x (coalesced) and the row's y (one broadcast 16-byte load).
constexpr int kGateCols = 4;     // D <= 128
constexpr int kGateRows = 1024;  // tokens per CTA
__global__ void __launch_bounds__(256) k_gate_grad(int T, int H, const float* X, int D,
                                                   const float* Y, float* gw, float* gb) {
  const int h = blockIdx.x, b = blockIdx.y;
  const int t0 = blockIdx.z * kGateRows, t1 = min(T, t0 + kGateRows);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t u = (int64_t)b * H + h;
  float acc[kGateCols][4] = {}, bsum[4] = {0.f, 0.f, 0.f, 0.f};
  for (int t = t0 + w; t < t1; t += 8) {
    const int64_t o = u * T + t;
    const float4 y = *reinterpret_cast<const float4*>(Y + o * 4);
    const float yv[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
    for (int i = 0; i < kGateCols; ++i) {
      const int d = lane + 32 * i;
      const float x = d < D ? X[o * D + d] : 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] += x * yv[j];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) bsum[j] += yv[j];
  }
  __shared__ float red[8][32 * kGateCols][4];
  __shared__ float rb[8][4];
#pragma unroll
  for (int i = 0; i < kGateCols; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) red[w][lane + 32 * i][j] = acc[i][j];
  if (lane == 0)
#pragma unroll
    for (int j = 0; j < 4; ++j) rb[w][j] = bsum[j];
  __syncthreads();
  for (int i = threadIdx.x; i < D * 4; i += blockDim.x) {
    const int d = i >> 2, j = i & 3;
    float s = 0.f;
#pragma unroll
    for (int ww = 0; ww < 8; ++ww) s += red[ww][d][j];
    atomicAdd(&gw[((int64_t)h * D + d) * 4 + j], s);
  }
  if (threadIdx.x < 4) {
    float s = 0.f;
#pragma unroll
    for (int ww = 0; ww < 8; ++ww) s += rb[ww][threadIdx.x];
    atomicAdd(&gb[h * 4 + threadIdx.x], s);
  }
}

// one warp per (u, t): final input gradients in the input layout / dtype.
__global__ void k_input_bwd(int B, int T, int H, int D, int Dv, int dt, const float* qh,
                            const float* qn, const float* dqh, const float* dq_direct,
                            const float* dkey, const float* dval, void* dq, void* dk, void* dv,
                            int64_t rope_pos0) {
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  const int U = B * H;
  if (w >= U * T) return;
  const int u = w / T, t = w - u * T, b = u / H, h = u - b * H;
  const int64_t dst = ((int64_t)b * T + t) * H + h;
  // every operand of the row is loaded before the reduction (D, Dv <= 128: 4 per lane)
  float y[4], dy[4], dd[4], dkv[4], dvv[4];
  const float nrm = qn[w];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int d = lane + 32 * i;
    const int64_t o = (int64_t)w * D + d;
    const bool in = d < D;
    y[i] = in ? qh[o] : 0.f;
    dy[i] = in ? dqh[o] : 0.f;
    dd[i] = in ? dq_direct[o] : 0.f;
    dkv[i] = in ? dkey[o] : 0.f;
    dvv[i] = d < Dv ? dval[(int64_t)w * Dv + d] : 0.f;
  }
  float yd = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) yd += y[i] * dy[i];
  yd = warp_sum(yd);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int d = lane + 32 * i;
    const float g = nrm > kUnitEps ? (dy[i] - y[i] * yd) / nrm : dy[i] / kUnitEps;
    float gq = g + dd[i];
    if (rope_pos0 >= 0) {  // through the rotation: R^T of the rotated query's gradient
      const float other = __shfl_xor_sync(0xffffffffu, gq, 1);
      float c, s;
      rope_cs(rope_pos0 + t, d, D, c, s);
      gq = (d & 1) == 0 ? c * gq + s * other : -s * other + c * gq;
    }
    if (d < D) {
      store_out(dq, dst * D + d, gq, dt);
      store_out(dk, dst * D + d, dkv[i], dt);
    }
    if (d < Dv) store_out(dv, dst * Dv + d, dvv[i], dt);
  }
}

// per head: scalar parameter gradients from per-unit sums.
__global__ void k_fold(FoldArgs a) {
  const int h = blockIdx.x * blockDim.x + threadIdx.x;
  if (h >= a.H) return;
  const int H = a.H, L = a.L, E = a.E;
  auto S = [&](int j, int slot) {
    double s = 0.0;
    for (int b = 0; b < a.B; ++b) s += a.scal[((int64_t)(b * H + h) * L + j) * kNScal + slot];
    return (float)s;
  };
  auto SE = [&](int e, int slot) {
    double s = 0.0;
    for (int b = 0; b < a.B; ++b) s += a.scalE[((int64_t)(b * H + h) * E + e) * kNEdge + slot];
    return (float)s;
  };
  float ow[kMaxLevels], dow[kMaxLevels];
  float mx = -INFINITY, ssum = 0.f;
  for (int j = 0; j < L; ++j) mx = fmaxf(mx, a.output_logits[j * H + h]);
  for (int j = 0; j < L; ++j) {
    ow[j] = __expf(a.output_logits[j * H + h] - mx);
    ssum += ow[j];
  }
  float dot = 0.f;
  for (int j = 0; j < L; ++j) {
    ow[j] /= ssum;
    dow[j] = S(j, kS_OutW);
    dot += ow[j] * dow[j];
  }
  for (int j = 0; j < L; ++j) {
    a.g_output_logits[j * H + h] += ow[j] * (dow[j] - dot);
    const float tk = tanhf(a.residual_raw[(j * H + h) * 2]);
    const float tv = tanhf(a.residual_raw[(j * H + h) * 2 + 1]);
    a.g_residual_raw[(j * H + h) * 2] += S(j, kS_EtaK) * .25f * (1.f - tk * tk);
    a.g_residual_raw[(j * H + h) * 2 + 1] += S(j, kS_EtaV) * .25f * (1.f - tv * tv);
    a.g_count_gain_raw[j * H + h] += S(j, kS_CountGain) * sigmoid(a.count_gain_raw[j * H + h]);
    a.g_route_mlp_gain[j * H + h] += S(j, kS_MlpGain);
    a.g_relation_gain[j * H + h] += S(j, kS_RelGain);
    if (a.g_moment_gain) a.g_moment_gain[j * H + h] += S(j, kS_MomentGain);
    // edge-logit softmax over the edges into j
    float w[kMaxIn], dw[kMaxIn];
    int ids[kMaxIn], n = 0;
    for (int e = 0; e < E; ++e)
      if (a.edge_dst[e] == j) ids[n++] = e;
    if (n) {
      float m2 = -INFINITY, s2 = 0.f, d2 = 0.f;
      for (int i = 0; i < n; ++i) m2 = fmaxf(m2, a.edge_logits[ids[i] * H + h]);
      for (int i = 0; i < n; ++i) {
        w[i] = __expf(a.edge_logits[ids[i] * H + h] - m2);
        s2 += w[i];
      }
      for (int i = 0; i < n; ++i) {
        w[i] /= s2;
        dw[i] = SE(ids[i], kE_W);
        d2 += w[i] * dw[i];
      }
      for (int i = 0; i < n; ++i) a.g_edge_logits[ids[i] * H + h] += w[i] * (dw[i] - d2);
    }
  }
  for (int e = 0; e < E; ++e) {
    const float sd = sigmoid(a.relation_decay_raw[e * H + h]);
    if (!a.pos_none) a.g_relation_decay_raw[e * H + h] += -SE(e, kE_G) * sd;
    const float sb = sigmoid(a.relation_beta_raw[e * H + h]);
    a.g_relation_beta_raw[e * H + h] += SE(e, kE_B) * sb * (1.f - sb);
  }
}

int blocks_for(int64_t n, int per) { return (int)((n + per - 1) / per); }

template <class Kern, class... Args>
cudaError_t launch_smem(const char* name, Kern k, int grid, size_t smem, cudaStream_t st,
                        Args... args) {
  if (grid <= 0) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  Launch scope(name, st);
  k<<<grid, 256, smem, st>>>(args...);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_input(const void* q, const void* k, const void* v, int dt, int B, int T, int H,
                         int D, int Dv, float* qf, float* qh, float* qn, float* key0, float* val0,
                         int64_t rope_pos0, cudaStream_t st) {
  const int rows = B * T * H;
  if (!rows) return cudaSuccess;
  Launch scope_("input", st);
  k_input<<<blocks_for(rows, 8), 256, 0, st>>>(q, k, v, dt, B, T, H, D, Dv, qf, qh, qn, key0,
                                                val0, rope_pos0);
  return cudaGetLastError();
}

cudaError_t launch_level_prep(int U, int T, int H, int D, int M, const float* key, const float* C,
                              const float* Wg, const float* gbias, float beta_max, int pos_none,
                              float* nk, float* kn, float* slot, float* ns, float* sn, float* raw4,
                              float* gates, cudaStream_t st) {
  const int ntile = (T + kRowsPerTile - 1) / kRowsPerTile;
  const size_t smem = sizeof(float) * kRowsPerTile * (D + M);
  return launch_smem("level_prep", k_level_prep, U * ntile, smem, st, U, T, H, D, M, key, C, Wg, gbias,
                     beta_max, pos_none, nk, kn, slot, ns, sn, raw4, gates);
}

cudaError_t launch_level_post(int U, const Blocks& bl, int post, int H, int D, int Dv, int M,
                              int with_residual, const float* nk, const float* key, const float* val,
                              const float* Abnd, const float* Bbnd, const float* fzA,
                              const float* fzB, const float* residual_raw, int j, float* write,
                              float* bsum, float* key_next, float* val_next, cudaStream_t st) {
  const size_t smem = sizeof(float) * (D * M + M * Dv + kRowsPerTile * M);
  return launch_smem("level_post", k_level_post, U * bl.nb, smem, st, U, bl, post, H, D, Dv, M, with_residual,
                     nk, key, val, Abnd, Bbnd, fzA, fzB, residual_raw, j, write, bsum, key_next,
                     val_next);
}

cudaError_t launch_counts(int U, const Blocks& bl, int H, int M, float read_scale,
                          const float* count_gain_raw, int j, const float* n0, const float* bsum,
                          const float* write, const float* raw, float* counts, float* logits,
                          float* lh, float* ln, float* wh, float* wn, float* n_final,
                          const float* corr, const float* moment_gain, cudaStream_t st) {
  if (!U || !bl.nb) return cudaSuccess;
  Launch scope_("counts", st);
  const auto kern = M <= 32    ? k_counts<1>
                    : M <= 64  ? k_counts<2>
                    : M <= 128 ? k_counts<4>
                               : k_counts<8>;
  const size_t smem = (2 * kRowsPerTile * M + M + 256) * sizeof(float);
  if (smem > 48 * 1024) {
    const cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  kern<<<U * bl.nb, 256, smem, st>>>(U, bl, H, M, read_scale, count_gain_raw, j, n0, bsum, write, raw,
                                    counts, logits, lh, ln, wh, wn, n_final, corr, moment_gain);
  return cudaGetLastError();
}

cudaError_t launch_rel_gates(int U, int H, int E, int pos_none, const float* decay_raw,
                             const float* beta_raw, float* ge, float* be, cudaStream_t st) {
  if (!E || !U) return cudaSuccess;
  Launch scope_("rel_gates", st);
  k_rel_gates<<<blocks_for((int64_t)E * U, 256), 256, 0, st>>>(U, H, E, pos_none, decay_raw,
                                                                beta_raw, ge, be);
  return cudaGetLastError();
}

cudaError_t launch_bridge(int U, int T, int H, int D, int M, int L, int j, const BridgeIn& in,
                          const float* edge_logits, const float* relation_gain,
                          const float* route_up, const float* route_down,
                          const float* route_mlp_gain, const float* Wrs, const float* Wqs,
                          float qs, const float* logits, const float* qf, float* r, float* hp,
                          float* mlp, float* route, float* qoh, float* qon, cudaStream_t st) {
  const int ntile = (T + kRowsPerTile - 1) / kRowsPerTile;
  const size_t smem = sizeof(float) * kRowsPerTile * 4 * M;
  return launch_smem("bridge", k_bridge, U * ntile, smem, st, U, T, H, D, M, L, j, in, edge_logits,
                     relation_gain, route_up, route_down, route_mlp_gain, Wrs, Wqs, qs, logits, qf,
                     r, hp, mlp, route, qoh, qon);
}

cudaError_t launch_mix(int B, int T, int H, int Dv, int L, const float* output_logits,
                       const float* const* y, void* out, int dt, cudaStream_t st) {
  const int rows = B * T * H;
  if (!rows) return cudaSuccess;
  YPtrs yp;
  for (int j = 0; j < L; ++j) yp.y[j] = y[j];
  Launch scope_("mix", st);
  k_mix<<<blocks_for(rows, 8), 256, 0, st>>>(B, T, H, Dv, L, output_logits, yp, out, dt);
  return cudaGetLastError();
}

cudaError_t launch_copy(float* dst, const float* src, int64_t n, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  Launch scope_("copy", st);
  k_copy<<<blocks_for(n, 256), 256, 0, st>>>(dst, src, n);
  return cudaGetLastError();
}

cudaError_t launch_to_bthx(const float* src, void* dst, int dt, int B, int T, int H, int X,
                           cudaStream_t st) {
  const int64_t n = (int64_t)B * T * H * X;
  if (n <= 0) return cudaSuccess;
  Launch scope_("to_bthx", st);
  k_to_bthx<<<blocks_for(n, 256), 256, 0, st>>>(src, dst, dt, B, T, H, X);
  return cudaGetLastError();
}

cudaError_t launch_add(float* dst, const float* src, int64_t n, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  Launch scope_("add", st);
  k_add<<<blocks_for(n, 256), 256, 0, st>>>(dst, src, n);
  return cudaGetLastError();
}

cudaError_t launch_gather_boundary(float* dst, const float* src, int U, int nb1, int idx,
                                   int64_t sz, cudaStream_t st) {
  const int64_t n = (int64_t)U * sz;
  if (n <= 0) return cudaSuccess;
  Launch scope_("boundary", st);
  k_boundary<<<blocks_for(n, 256), 256, 0, st>>>(dst, src, U, nb1, idx, sz, 0);
  return cudaGetLastError();
}

cudaError_t launch_scatter_add_boundary(float* dst, const float* src, int U, int nb1, int idx,
                                        int64_t sz, cudaStream_t st) {
  const int64_t n = (int64_t)U * sz;
  if (n <= 0) return cudaSuccess;
  Launch scope_("boundary", st);
  k_boundary<<<blocks_for(n, 256), 256, 0, st>>>(dst, src, U, nb1, idx, sz, 1);
  return cudaGetLastError();
}

cudaError_t launch_scales(int U, int H, int L, const float* output_logits, float* ow_scale,
                          cudaStream_t st) {
  Launch scope_("scales", st);
  k_scales<<<blocks_for(U, 128), 128, 0, st>>>(U, H, L, output_logits, ow_scale);
  return cudaGetLastError();
}

cudaError_t launch_mix_bwd(int B, int T, int H, int Dv, int L, const void* dout, int dt,
                           const float* const* y, float* dout_f, double* scal, cudaStream_t st) {
  const int rows = B * T * H;
  if (!rows) return cudaSuccess;
  YPtrs yp;
  for (int j = 0; j < L; ++j) yp.y[j] = y[j];
  Launch scope_("mix_bwd", st);
  k_mix_bwd<<<blocks_for(rows, 8), 256, 0, st>>>(B, T, H, Dv, L, dout, dt, yp, dout_f, scal);
  return cudaGetLastError();
}

cudaError_t launch_bridge_bwd(int U, int T, int H, int D, int M, int L, int j, const BridgeIn& in,
                              const float* edge_logits, const float* relation_gain,
                              const float* route_up, const float* route_down,
                              const float* route_mlp_gain, const float* Wrs, const float* Wqs,
                              float qs, const float* logits, const float* r, const float* hp,
                              const float* mlp, const float* qoh, const float* qon,
                              const float* dqoh, float* dqo, float* droute, float* dhp,
                              float* dlogits, float* dq_direct, double* scal, double* scalE,
                              int E, cudaStream_t st) {
  const int ntile = (T + kRowsPerTile - 1) / kRowsPerTile;
  const size_t smem = sizeof(float) * (kRowsPerTile * 4 * M + 32 + kMaxIn);
  return launch_smem("bridge_bwd", k_bridge_bwd, U * ntile, smem, st, U, T, H, D, M, L, j, in, edge_logits,
                     relation_gain, route_up, route_down, route_mlp_gain, Wrs, Wqs, qs, logits, r,
                     hp, mlp, qoh, qon, dqoh, dqo, droute, dhp, dlogits, dq_direct, scal, scalE,
                     E);
}

cudaError_t launch_logits_bwd(int U, const Blocks& bl, int H, int M, int L, int j,
                              float read_scale, const float* count_gain_raw, const float* logits,
                              const float* counts, const float* lh, const float* ln,
                              const float* wh, const float* wn, const float* dlh,
                              const float* dwh, const float* dlogits, float* dwrite, float* draw,
                              float* dn, float* dnsum, double* scal, ProductBwd pb, MomentBwd mb,
                              cudaStream_t st) {
  const int rows = U * bl.T;
  if (!rows) return cudaSuccess;
  Launch scope_("logits_bwd", st);
  if (M <= 64)
    k_logits_bwd<2><<<blocks_for(rows, 8), 256, 0, st>>>(U, bl, H, M, L, j, read_scale,
                                                     count_gain_raw, logits, counts, lh, ln, wh,
                                                     wn, dlh, dwh, dlogits, dwrite, draw, dn,
                                                     dnsum, scal, pb, mb);
  else if (M <= 128)
    k_logits_bwd<4><<<blocks_for(rows, 8), 256, 0, st>>>(U, bl, H, M, L, j, read_scale,
                                                     count_gain_raw, logits, counts, lh, ln, wh,
                                                     wn, dlh, dwh, dlogits, dwrite, draw, dn,
                                                     dnsum, scal, pb, mb);
  else
    k_logits_bwd<8><<<blocks_for(rows, 8), 256, 0, st>>>(U, bl, H, M, L, j, read_scale,
                                                     count_gain_raw, logits, counts, lh, ln, wh,
                                                     wn, dlh, dwh, dlogits, dwrite, draw, dn,
                                                     dnsum, scal, pb, mb);
  return cudaGetLastError();
}

cudaError_t launch_counts_bwd(int U, const Blocks& bl, int M, const float* dn, const float* dnsum,
                              const float* dn_final, float* dwrite, float* dn0, cudaStream_t st) {
  if (!U || !bl.nb) return cudaSuccess;
  Launch scope_("counts_bwd", st);
  const size_t smem = (2 * kRowsPerTile * M + M + 256) * sizeof(float);
  if (smem > 48 * 1024) {
    const cudaError_t e =
        cudaFuncSetAttribute(k_counts_bwd, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  k_counts_bwd<<<U * bl.nb, 256, smem, st>>>(U, bl, M, dn, dnsum, dn_final, dwrite, dn0);
  return cudaGetLastError();
}

cudaError_t launch_post_bwd(int U, const Blocks& bl, int post, int offset, int H, int D, int Dv,
                            int M, int L, int j, int with_residual, const float* nk,
                            const float* write, const float* Abnd, const float* Bbnd,
                            const float* fzA, const float* fzB, const float* residual_raw,
                            const float* dkey, const float* dval, float* dwrite, float* dnk,
                            float* extA, float* extB, float* dfzA, float* dfzB, double* scal,
                            cudaStream_t st) {
  const size_t smem = sizeof(float) * (D * M + M * Dv + 2 * kRowsPerTile * M + 34);
  return launch_smem("post_bwd", k_post_bwd, U * bl.nb, smem, st, U, bl, post, offset, H, D, Dv, M, L, j,
                     with_residual, nk, write, Abnd, Bbnd, fzA, fzB, residual_raw, dkey, dval,
                     dwrite, dnk, extA, extB, dfzA, dfzB, scal);
}

cudaError_t launch_prep_bwd(int U, int T, int H, int D, int M, const float* C, const float* Wg,
                            float beta_max, int pos_none, const float* raw4, const float* nk,
                            const float* kn, const float* ns, const float* sn, const float* dgates,
                            const float* dnk, const float* dns, float* dslot, float* d4,
                            float* dkey, cudaStream_t st) {
  const int ntile = (T + kRowsPerTile - 1) / kRowsPerTile;
  const size_t smem = sizeof(float) * kRowsPerTile * M;
  return launch_smem("prep_bwd", k_prep_bwd, U * ntile, smem, st, U, T, H, D, M, C, Wg, beta_max, pos_none,
                     raw4, nk, kn, ns, sn, dgates, dnk, dns, dslot, d4, dkey);
}

cudaError_t launch_gate_grad(int B, int T, int H, const float* X, int D, const float* Y, float* gw,
                             float* gb, cudaStream_t st) {
  if (!B || !T) return cudaSuccess;
  if (D > 32 * kGateCols) return cudaErrorInvalidValue;
  dim3 grid(H, B, (unsigned)((T + kGateRows - 1) / kGateRows));
  Launch scope_("gate_grad", st);
  k_gate_grad<<<grid, 256, 0, st>>>(T, H, X, D, Y, gw, gb);
  return cudaGetLastError();
}

cudaError_t launch_head_outer(int B, int T, int H, const float* X, int P, int xmode,
                              const float* Y, int Q, const float* scale, int64_t scale_stride,
                              float cscale, float* out, cudaStream_t st) {
  const int64_t total = (int64_t)B * T;
  if (!total) return cudaSuccess;
  const int tp = (P + kHoTile - 1) / kHoTile, tq = (Q + kHoTile - 1) / kHoTile;
  dim3 grid(H, tp * tq, (unsigned)((total + kHoSplit - 1) / kHoSplit));
  Launch scope_("head_outer", st);
  k_head_outer<<<grid, 256, 0, st>>>(B, T, H, X, P, xmode, Y, Q, scale, scale_stride, cscale,
                                     out);
  return cudaGetLastError();
}

cudaError_t launch_input_bwd(int B, int T, int H, int D, int Dv, int dt, const float* qh,
                             const float* qn, const float* dqh, const float* dq_direct,
                             const float* dkey, const float* dval, void* dq, void* dk, void* dv,
                             int64_t rope_pos0, cudaStream_t st) {
  const int rows = B * T * H;
  if (!rows) return cudaSuccess;
  Launch scope_("input_bwd", st);
  k_input_bwd<<<blocks_for(rows, 8), 256, 0, st>>>(B, T, H, D, Dv, dt, qh, qn, dqh, dq_direct,
                                                    dkey, dval, dq, dk, dv, rope_pos0);
  return cudaGetLastError();
}

cudaError_t launch_fold(const FoldArgs& a, cudaStream_t st) {
  Launch scope_("fold", st);
  k_fold<<<blocks_for(a.H, 64), 64, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace gpa
