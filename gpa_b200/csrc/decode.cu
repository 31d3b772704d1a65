// One-token decode step for lag-block caches (chunk_size >= 2), fused into a single kernel
// per call: one CTA per (batch, head) unit walks the whole layer for its token and updates
// the cache in place.  The chunk offset lives in device memory; the last CTA to finish
// advances it (a completion counter beside the offset tells it that every CTA has read the
// old value), so a step is one launch and a sequence of steps can be captured once in a CUDA
// graph and replayed.
//
// Per unit and level j (src/gpa/attention.py:299-345 with a one-token block):
//   slot = C_j k, gates from u(k); A <- GDN(A, u(k), slot) and raw = u(q)^T A;
//   write = softmax(u(k)^T A_f) with A_f the frozen snapshot (the pre-update A when the
//   token opens a block); counts += write; logits = raw + softplus(c_j) log1p(n);
//   k <- k - eta_k A_f write, v <- v - eta_v write^T B_f.
// then the relation GDN steps of every edge, the dense reader per level
// (src/gpa/attention.py:225-262), the outer GDN steps B <- GDN(B, u(slot), v_j) read with
// u(qo_j), and the softmax(output_logits) mix.  All arithmetic is fp32.
//
// Each state matrix is read from HBM once into shared memory, updated there and written
// back once (the outer states, and the frozen snapshots when the token opens a block, are
// read a second time): the step is HBM-bound on the cache, 2 x 4 x 155,968 bytes per unit at
// the widths Dk = Dv = 128, slots (64, 64, 64, 128).
#include "decode.cuh"
#include "tc5.cuh"

namespace gpa {

__device__ int g_decode_status = 0;

namespace {

constexpr int kStepThreads = 256;

// ---------------------------------------------------------------- block helpers

// x rounded to the input dtype (the reference rounds its rotated query back to it)
GPA_DEV float round_in(float x, int dt) {
  if (dt == GPA_B200_BF16) return __bfloat162float(__float2bfloat16(x));
  if (dt == GPA_B200_F16) return __half2float(__float2half(x));
  return x;
}

GPA_DEV float block_sum_all(float x, float* red) {
  x = warp_sum(x);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = x;
  __syncthreads();
  float s = 0.f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += red[w];
  return s;
}

GPA_DEV float block_max_all(float x, float* red) {
  x = warp_max(x);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = x;
  __syncthreads();
  float s = -INFINITY;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s = fmaxf(s, red[w]);
  return s;
}

// dst = src / max(|src|, eps) (dst may alias src); ends synchronized
GPA_DEV void unit_vec(float* dst, const float* src, int n, float* red) {
  float ss = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) ss += src[i] * src[i];
  const float inv = 1.f / fmaxf(sqrtf(block_sum_all(ss, red)), kUnitEps);
  for (int i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i] * inv;
  __syncthreads();
}

// dst = softmax(src) (dst may alias src); ends synchronized
GPA_DEV void softmax_vec(float* dst, const float* src, int n, float* red) {
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < n; i += blockDim.x) mx = fmaxf(mx, src[i]);
  mx = block_max_all(mx, red);
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += __expf(src[i] - mx);
  const float inv = 1.f / block_sum_all(s, red);
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) dst[i] = __expf(src[i] - mx) * inv;
  __syncthreads();
}

GPA_DEV float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }

GPA_DEV void fma4(float4& a, float x, float4 b) {
  a.x += x * b.x;
  a.y += x * b.y;
  a.z += x * b.z;
  a.w += x * b.w;
}

// y[c] = sum_r x[r] S[r][c] for S [R x Cn] row-major (shared or global), Cn a multiple of 4
// and Cn / 4 <= blockDim: a thread owns 4 columns of a slice of the rows, four rows in
// flight; part: 4 * blockDim floats.  Ends synchronized.
GPA_DEV void colsum(const float* S, int R, int Cn, const float* x, float* y, float* part) {
  const int c4n = Cn >> 2, P = blockDim.x / c4n;
  const int c4 = threadIdx.x % c4n, pr = threadIdx.x / c4n;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (pr < P) {
    const float* col = S + 4 * c4;
    int r = pr;
    for (; r + 3 * P < R; r += 4 * P) {
      const float4 a0 = ld4(col + (int64_t)r * Cn), a1 = ld4(col + (int64_t)(r + P) * Cn);
      const float4 a2 = ld4(col + (int64_t)(r + 2 * P) * Cn), a3 = ld4(col + (int64_t)(r + 3 * P) * Cn);
      fma4(acc, x[r], a0);
      fma4(acc, x[r + P], a1);
      fma4(acc, x[r + 2 * P], a2);
      fma4(acc, x[r + 3 * P], a3);
    }
    for (; r < R; r += P) fma4(acc, x[r], ld4(col + (int64_t)r * Cn));
    *reinterpret_cast<float4*>(part + pr * Cn + 4 * c4) = acc;
  }
  __syncthreads();
  for (int c = threadIdx.x; c < Cn; c += blockDim.x) {
    float s = 0.f;
    for (int i = 0; i < P; ++i) s += part[i * Cn + c];
    y[c] = s;
  }
  __syncthreads();
}

// y[r] = sum_c S[r][c] x[c] for S [R x Cn] row-major, Cn a multiple of 4: a warp per row,
// float4 columns.  Ends synchronized.
GPA_DEV void rowdot(const float* S, int R, int Cn, const float* x, float* y) {
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int r0 = w; r0 < R; r0 += 4 * nw) {  // four rows of a warp in flight
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int c = 4 * lane; c < Cn; c += 128) {
      const float4 xv = ld4(x + c);
      float4 a[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        a[i] = r0 + i * nw < R ? ld4(S + (int64_t)(r0 + i * nw) * Cn + c) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] += a[i].x * xv.x + a[i].y * xv.y + a[i].z * xv.z + a[i].w * xv.w;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float s = warp_sum(acc[i]);
      if (lane == 0 && r0 + i * nw < R) y[r0 + i * nw] = s;
    }
  }
  __syncthreads();
}

// The mbarrier of the step's bulk state loads, its next phase parity, and whether every wait
// on it completed.
struct BulkLoad {
  uint64_t* bar;
  uint32_t parity;
  bool ok;
};

// shared <- global (n floats, 16-byte aligned rows of float4); optional copy to `also`.  When
// the matrix is 16-byte aligned and a whole number of 16-byte pieces it comes in as one bulk
// (TMA) copy: one load latency and no registers held.  Otherwise float4 loads, four in flight
// per thread.  A bulk wait that gives up (tc5::kWaitNs) clears bl.ok; the step then records
// GPA_B200_DEVICE_TIMEOUT and its results are not to be used.
GPA_DEV void load_mat(float* Ss, const float* g, int n, float* also, BulkLoad& bl) {
  if ((n & 3) == 0 && (reinterpret_cast<uintptr_t>(g) & 15) == 0) {
    tc5::fence_async_smem();  // every earlier access to Ss before the copy overwrites it
    __syncthreads();
    if (threadIdx.x == 0) {
      tc5::mbar_expect_tx(bl.bar, (uint32_t)n * 4u);
      tc5::bulk_g2s(Ss, g, (uint32_t)n * 4u, bl.bar);
    }
    if (!tc5::mbar_wait(bl.bar, bl.parity)) bl.ok = false;
    bl.parity ^= 1u;
    if (also)
      for (int i = 4 * threadIdx.x; i < n; i += 4 * blockDim.x)
        *reinterpret_cast<float4*>(also + i) = *reinterpret_cast<const float4*>(Ss + i);
    __syncthreads();
    return;
  }
  const int step = 4 * blockDim.x;
  for (int i0 = 4 * threadIdx.x; i0 < n; i0 += 4 * step) {  // four float4 in flight
    float4 x[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (i0 + j * step < n) x[j] = ld4(g + i0 + j * step);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (i0 + j * step < n) {
        *reinterpret_cast<float4*>(Ss + i0 + j * step) = x[j];
        if (also) *reinterpret_cast<float4*>(also + i0 + j * step) = x[j];
      }
  }
  __syncthreads();
}

// GDN update of the state already in shared memory (pre = kv^T S_old given):
// S <- e^g S + beta kv (val - e^g pre)^T, written back to global; y = qv^T S_new.
GPA_DEV void gdn_update(float* Ss, float* Sg, int K, int V, const float* kv, const float* val,
                        const float* pre, float g, float beta, const float* qv, float* y,
                        float* part) {
  const float eg = __expf(g);
  const int v4 = V >> 2;
  for (int i = threadIdx.x; i < K * v4; i += blockDim.x) {
    const int k = i / v4, c = (i - k * v4) << 2;
    float4 x = *reinterpret_cast<const float4*>(Ss + k * V + c);
    const float bk = beta * kv[k];
    x.x = eg * x.x + bk * (val[c] - eg * pre[c]);
    x.y = eg * x.y + bk * (val[c + 1] - eg * pre[c + 1]);
    x.z = eg * x.z + bk * (val[c + 2] - eg * pre[c + 2]);
    x.w = eg * x.w + bk * (val[c + 3] - eg * pre[c + 3]);
    *reinterpret_cast<float4*>(Ss + k * V + c) = x;
    *reinterpret_cast<float4*>(Sg + k * V + c) = x;
  }
  __syncthreads();
  colsum(Ss, K, V, qv, y, part);
}

// Offsets of one head's scalar parameters in shared memory: fetched together at kernel entry
// (one load latency for all of them) instead of one dependent global load per use.
struct HeadScalars {
  int E, L;
  GPA_DEV int edge_logit(int e) const { return e; }
  GPA_DEV int relation_decay(int e) const { return E + e; }
  GPA_DEV int relation_beta(int e) const { return 2 * E + e; }
  GPA_DEV int relation_gain(int j) const { return 3 * E + j; }
  GPA_DEV int count_gain(int j) const { return 3 * E + L + j; }
  GPA_DEV int route_mlp_gain(int j) const { return 3 * E + 2 * L + j; }
  GPA_DEV int output_logit(int j) const { return 3 * E + 3 * L + j; }
  GPA_DEV int residual(int j, int c) const { return 3 * E + 4 * L + 2 * j + c; }
  GPA_DEV int gate_bias(int j, int c) const { return 3 * E + 6 * L + 4 * j + c; }
  GPA_DEV int moment_gain(int j) const { return 3 * E + 10 * L + j; }
  GPA_DEV int count() const { return 3 * E + 11 * L; }
};

struct StepSmem {
  size_t Ss, q, qn, key, kn, val, tmp, tmp2, pre, yb, part, red, slot, write, logits, valin, qo,
      gates, hs, mdel, mcor, wu, lqu, bar, total;
  int msg_off[kMaxEdges];
  __host__ __device__ StepSmem(const StepArgs& a) {
    size_t off = 0;
    auto take = [&](size_t nfloat) {
      off = (off + 3) & ~size_t(3);
      const size_t r = off;
      off += nfloat;
      return r;
    };
    int mx = 0, big = 0;
    for (int j = 0; j < a.L; ++j) {
      mx = a.M[j] > mx ? a.M[j] : mx;
      const int s1 = a.D * a.M[j], s2 = a.M[j] * a.Dv;
      big = s1 > big ? s1 : big;
      big = s2 > big ? s2 : big;
    }
    for (int e = 0; e < a.E; ++e) {
      const int s3 = a.M[a.es[e]] * a.M[a.ed[e]];
      big = s3 > big ? s3 : big;
    }
    const int w = a.D > a.Dv ? a.D : a.Dv;
    const int wide = (w > 2 * mx ? w : 2 * mx);
    Ss = take(big);
    q = take(a.D);
    qn = take(a.D);
    key = take(a.D);
    kn = take(a.D);
    val = take(a.Dv);
    tmp = take(wide);
    tmp2 = take(wide);
    pre = take(w > mx ? w : mx);
    yb = take(a.Dv);
    part = take(4 * kStepThreads);
    red = take(32);
    slot = take(a.L * mx);
    write = take(a.L * mx);
    logits = take(a.L * mx);
    valin = take(a.L * a.Dv);
    qo = take(a.L * mx);
    gates = take(a.L * 4);
    for (int e = 0; e < a.E; ++e) msg_off[e] = (int)take(a.M[a.ed[e]]);
    hs = take(3 * kMaxEdges + 11 * kMaxLevels);  // this head's scalars (HeadScalars)
    mdel = take(a.D);  // positional moments: delta of the level key, moment reads
    mcor = take(mx);
    wu = take(a.L * mx);   // u(write_i) of every level (relation keys)
    lqu = take(a.L * mx);  // u(softmax(logits_i)) of every level (relation queries)
    bar = take(4);  // the bulk loads' mbarrier (16-byte aligned)
    total = off * sizeof(float);
  }
};

__global__ void __launch_bounds__(kStepThreads) k_decode_step(StepArgs a) {
  extern __shared__ __align__(16) float sm[];
  const StepSmem Lm(a);
  const int u = blockIdx.x, h = u % a.H, D = a.D, Dv = a.Dv, L = a.L;
  const int o = *a.offset;
  int mx = 0;
  for (int j = 0; j < L; ++j) mx = a.M[j] > mx ? a.M[j] : mx;
  float* Ss = sm + Lm.Ss;
  float* q = sm + Lm.q;
  float* qn = sm + Lm.qn;
  float* key = sm + Lm.key;
  float* kn = sm + Lm.kn;
  float* val = sm + Lm.val;
  float* tmp = sm + Lm.tmp;
  float* tmp2 = sm + Lm.tmp2;
  float* part = sm + Lm.part;
  float* red = sm + Lm.red;
  BulkLoad bl{reinterpret_cast<uint64_t*>(sm + Lm.bar), 0u, true};
  float* hs = sm + Lm.hs;
  const HeadScalars hx{a.E, L};
  for (int i = threadIdx.x; i < hx.count(); i += blockDim.x) {
    const int E = a.E, H = a.H;
    float x;
    if (i < E) x = a.p.edge_logits[i * H + h];
    else if (i < 2 * E) x = a.p.relation_decay_raw[(i - E) * H + h];
    else if (i < 3 * E) x = a.p.relation_beta_raw[(i - 2 * E) * H + h];
    else {
      const int r = i - 3 * E, kind = r / L, j = r - kind * L;
      if (kind == 0) x = a.p.relation_gain[j * H + h];
      else if (kind == 1) x = a.p.count_gain_raw[j * H + h];
      else if (kind == 2) x = a.p.route_mlp_gain[j * H + h];
      else if (kind == 3) x = a.p.output_logits[j * H + h];
      else if (kind < 6) {
        const int q = r - 4 * L;  // residual_raw: 2 per level
        x = a.p.residual_raw[((q >> 1) * H + h) * 2 + (q & 1)];
      } else if (kind < 10) {
        const int q = r - 6 * L;  // gate_bias: 4 per level
        x = a.p.gate_bias[q >> 2][h * 4 + (q & 3)];
      } else {
        x = a.moments ? a.p.moment_gain[j * H + h] : 0.f;
      }
    }
    hs[i] = x;
  }
  if (threadIdx.x == 0) {
    tc5::mbar_init(bl.bar, 1);
    tc5::mbar_fence_init();
  }
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    q[i] = load_in(a.q, (int64_t)u * D + i, a.dt);
    key[i] = load_in(a.k, (int64_t)u * D + i, a.dt);
  }
  for (int i = threadIdx.x; i < Dv; i += blockDim.x) val[i] = load_in(a.v, (int64_t)u * Dv + i, a.dt);
  __syncthreads();
  const int pos = a.offset[2];
  if (a.moments) {  // rotated query at the cache position, rounded to the input dtype
    for (int i = threadIdx.x; i < D / 2; i += blockDim.x) {
      const float e = q[2 * i], od = q[2 * i + 1];
      float c, s;
      rope_cs(pos, 2 * i, D, c, s);
      q[2 * i] = round_in(e * c - od * s, a.dt);
      q[2 * i + 1] = round_in(e * s + od * c, a.dt);
    }
    __syncthreads();
  }
  unit_vec(qn, q, D, red);

  // ------------------------------------------------ level chain
  for (int j = 0; j < L; ++j) {
    const int M = a.M[j];
    float* slot = sm + Lm.slot + j * mx;
    float* write = sm + Lm.write + j * mx;
    float* logits = sm + Lm.logits + j * mx;
    float* gates = sm + Lm.gates + 4 * j;
    unit_vec(kn, key, D, red);
    rowdot(a.p.center[j] + (int64_t)h * M * D, M, D, key, slot);  // slot = C k
    {  // gates from u(k)
      const float* wg = a.p.gate_weight[j] + (int64_t)h * D * 4;
      float r[4] = {0.f, 0.f, 0.f, 0.f};
      for (int d = threadIdx.x; d < D; d += blockDim.x) {
        const float4 w4 = *reinterpret_cast<const float4*>(wg + 4 * d);
        r[0] += kn[d] * w4.x;
        r[1] += kn[d] * w4.y;
        r[2] += kn[d] * w4.z;
        r[3] += kn[d] * w4.w;
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) r[c] = warp_sum(r[c]);
      __syncthreads();
      if ((threadIdx.x & 31) == 0)
        for (int c = 0; c < 4; ++c) part[4 * (threadIdx.x >> 5) + c] = r[c];
      __syncthreads();
      if (threadIdx.x == 0) {
        for (int c = 0; c < 4; ++c) {
          float t = hs[hx.gate_bias(j, c)];
          for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += part[4 * w + c];
          r[c] = t;
        }
        gates[0] = a.pos_none ? 0.f : -fminf(softplus(r[0]), 10.f);
        gates[1] = a.beta_max * sigmoid(r[1]);
        gates[2] = a.pos_none ? 0.f : -fminf(softplus(r[2]), 10.f);
        gates[3] = a.beta_max * sigmoid(r[3]);
      }
      __syncthreads();
    }
    const int64_t szA = (int64_t)D * M, szB = (int64_t)M * Dv;
    float* Ag = a.s.inner[j] + u * szA;
    float* Bg = a.s.outer[j] + u * szB;
    float* rk = tmp;  // [D]
    if (o != 0) {     // write and rk from the frozen inner snapshot
      load_mat(Ss, a.s.frozen_inner[j] + u * szA, (int)szA, nullptr, bl);
      colsum(Ss, D, M, kn, write, part);
      softmax_vec(write, write, M, red);
      rowdot(Ss, D, M, write, rk);
    }
    // inner GDN step; the pre-update A is the frozen snapshot when the token opens a block
    load_mat(Ss, Ag, (int)szA, o == 0 ? a.s.frozen_inner[j] + u * szA : nullptr, bl);
    float* pre = sm + Lm.pre;  // u(k)^T A_old [M]
    colsum(Ss, D, M, kn, pre, part);
    if (o == 0) {
      softmax_vec(write, pre, M, red);
      rowdot(Ss, D, M, write, rk);
    }
    gdn_update(Ss, Ag, D, M, kn, slot, pre, gates[0], gates[1], qn, logits, part);  // logits <- raw
    float* mcor = sm + Lm.mcor;
    if (a.moments) {  // P += delta w^T (delta = rope(u(k)) - u(k)), corr = u(q)^T P
      float* mdel = sm + Lm.mdel;
      for (int i = threadIdx.x; i < D / 2; i += blockDim.x) {
        const float e = kn[2 * i], od = kn[2 * i + 1];
        float c, s;
        rope_cs(pos, 2 * i, D, c, s);
        mdel[2 * i] = e * c - od * s - e;
        mdel[2 * i + 1] = e * s + od * c - od;
      }
      float* Pg = a.s.moment[j] + u * szA;
      load_mat(Ss, Pg, (int)szA, nullptr, bl);  // ends synchronized (mdel visible too)
      for (int i = threadIdx.x; i < D * M; i += blockDim.x) {
        const int d = i / M, m = i - d * M;
        const float x = Ss[i] + mdel[d] * write[m];
        Ss[i] = x;
        Pg[i] = x;
      }
      __syncthreads();
      colsum(Ss, D, M, qn, mcor, part);
    }
    {  // counts and base logits
      const float cg = softplus(hs[hx.count_gain(j)]);
      const float mg = hs[hx.moment_gain(j)];
      float* n = a.s.count[j] + (int64_t)u * M;
      for (int m = threadIdx.x; m < M; m += blockDim.x) {
        const float nn = n[m] + write[m];
        n[m] = nn;
        logits[m] = a.read_scale * logits[m] + cg * log1pf(nn);
        if (a.moments) logits[m] += mg * tanhf(mcor[m] / (1.f + nn));
      }
    }
    // rv = write^T B_f
    float* rv = tmp2;
    load_mat(Ss, o == 0 ? Bg : a.s.frozen_outer[j] + u * szB, (int)szB,
             o == 0 ? a.s.frozen_outer[j] + u * szB : nullptr, bl);
    colsum(Ss, M, Dv, write, rv, part);
    float* vin = sm + Lm.valin + j * Dv;
    const float ek = 1.f + .25f * tanhf(hs[hx.residual(j, 0)]);
    const float ev = 1.f + .25f * tanhf(hs[hx.residual(j, 1)]);
    for (int i = threadIdx.x; i < Dv; i += blockDim.x) {
      vin[i] = val[i];
      val[i] -= ev * rv[i];
    }
    for (int i = threadIdx.x; i < D; i += blockDim.x) key[i] -= ek * rk[i];
    __syncthreads();
  }

  // ------------------------------------------------ relations
  // the relation keys u(write_i) and queries u(softmax(logits_i)) of every level, once (each
  // level sends L - 1 edges); lnorm[i] = |softmax(logits_i)| (the product reader's factor)
  float lnorm[kMaxLevels];
  if (a.E > 0)
    for (int i = 0; i < L; ++i) {
      const int Mi = a.M[i];
      float* lqi = sm + Lm.lqu + i * mx;
      unit_vec(sm + Lm.wu + i * mx, sm + Lm.write + i * mx, Mi, red);
      softmax_vec(lqi, sm + Lm.logits + i * mx, Mi, red);
      float ss = 0.f;
      for (int m = threadIdx.x; m < Mi; m += blockDim.x) ss += lqi[m] * lqi[m];
      lnorm[i] = sqrtf(block_sum_all(ss, red));
      const float inv = 1.f / fmaxf(lnorm[i], kUnitEps);
      for (int m = threadIdx.x; m < Mi; m += blockDim.x) lqi[m] *= inv;
      __syncthreads();
    }
  for (int e = 0; e < a.E; ++e) {
    const int i = a.es[e], j = a.ed[e], Mi = a.M[i], Mj = a.M[j];
    const float* kv = sm + Lm.wu + i * mx;   // u(write_i)
    const float* lq = sm + Lm.lqu + i * mx;  // u(softmax(logits_i))
    const int64_t sz = (int64_t)Mi * Mj;
    float* Rg = a.s.relation[e] + u * sz;
    load_mat(Ss, Rg, (int)sz, nullptr, bl);
    float* prebuf = sm + Lm.pre;
    colsum(Ss, Mi, Mj, kv, prebuf, part);
    const float g = a.pos_none ? 0.f : -softplus(hs[hx.relation_decay(e)]);
    const float b = sigmoid(hs[hx.relation_beta(e)]);
    gdn_update(Ss, Rg, Mi, Mj, kv, sm + Lm.write + j * mx, prebuf, g, b, lq,
               sm + Lm.msg_off[e], part);
  }

  // ------------------------------------------------ dense reader and outer steps
  for (int j = 0; j < L; ++j) {
    const int M = a.M[j];
    float* base = tmp;  // [M]
    float* logits = sm + Lm.logits + j * mx;
    float* inc = tmp2;  // [M]
    int nin = 0;
    float wmax = -INFINITY;
    for (int e = 0; e < a.E; ++e)
      if (a.ed[e] == j) {
        ++nin;
        wmax = fmaxf(wmax, hs[hx.edge_logit(e)]);
      }
    for (int m = threadIdx.x; m < M; m += blockDim.x) base[m] = logits[m];
    if (nin > 0 && a.reader != GPA_B200_READER_TANH) {
      // base += e^{clamp(g)} (M sum_e w_e |softmax(logits_src)| msg_e - log1p(counts) if
      // marginal), with this token's counts
      float ws = 0.f;
      for (int e = 0; e < a.E; ++e)
        if (a.ed[e] == j) ws += __expf(hs[hx.edge_logit(e)] - wmax);
      const float ge = __expf(fminf(fmaxf(hs[hx.relation_gain(j)], -4.f), 4.f));
      const bool marg = a.reader == GPA_B200_READER_MARGINAL;
      const float* cnt = a.s.count[j] + (int64_t)u * M;
      for (int m = threadIdx.x; m < M; m += blockDim.x) {
        float x = 0.f;
        for (int e = 0; e < a.E; ++e)
          if (a.ed[e] == j)
            x += (__expf(hs[hx.edge_logit(e)] - wmax) / ws) * lnorm[a.es[e]] * sm[Lm.msg_off[e] + m];
        base[m] += ge * (M * x - (marg ? log1pf(cnt[m]) : 0.f));
      }
      __syncthreads();
    } else if (nin > 0) {
      float ws = 0.f;
      for (int e = 0; e < a.E; ++e)
        if (a.ed[e] == j) ws += __expf(hs[hx.edge_logit(e)] - wmax);
      for (int m = threadIdx.x; m < M; m += blockDim.x) {
        float x = 0.f;
        for (int e = 0; e < a.E; ++e)
          if (a.ed[e] == j) x += (__expf(hs[hx.edge_logit(e)] - wmax) / ws) * sm[Lm.msg_off[e] + m];
        inc[m] = x;
      }
      __syncthreads();
      float s = 0.f;
      for (int m = threadIdx.x; m < M; m += blockDim.x) s += inc[m];
      const float mean = block_sum_all(s, red) / M;
      float vs = 0.f;
      for (int m = threadIdx.x; m < M; m += blockDim.x) vs += (inc[m] - mean) * (inc[m] - mean);
      const float sd = rsqrtf(block_sum_all(vs, red) / M + kCenterEps);
      const float rg = hs[hx.relation_gain(j)];
      for (int m = threadIdx.x; m < M; m += blockDim.x) base[m] += rg * tanhf((inc[m] - mean) * sd);
      __syncthreads();
    }
    softmax_vec(base, base, M, red);  // route
    float* hid = tmp2;                // [2M]
    colsum(a.p.route_up[j] + (int64_t)h * M * 2 * M, M, 2 * M, base, hid, part);
    for (int r = threadIdx.x; r < 2 * M; r += blockDim.x) hid[r] = gelu(hid[r]);
    __syncthreads();
    float* mlp = sm + Lm.qo + j * mx;  // scratch until qo is formed
    colsum(a.p.route_down[j] + (int64_t)h * 2 * M * M, 2 * M, M, hid, mlp, part);
    const float mg = hs[hx.route_mlp_gain(j)];
    for (int m = threadIdx.x; m < M; m += blockDim.x) base[m] += mg * mlp[m];
    __syncthreads();
    float* qo = sm + Lm.qo + j * mx;
    colsum(a.p.route_weight[j] + (int64_t)h * M * M, M, M, base, qo, part);
    colsum(a.p.query_weight[j] + (int64_t)h * D * M, D, M, q, hid, part);
    for (int m = threadIdx.x; m < M; m += blockDim.x) qo[m] += a.query_scale * hid[m];
    __syncthreads();
  }
  float ow[kMaxLevels];
  {
    float mxl = -INFINITY, s = 0.f;
    for (int j = 0; j < L; ++j) mxl = fmaxf(mxl, hs[hx.output_logit(j)]);
    for (int j = 0; j < L; ++j) {
      ow[j] = __expf(hs[hx.output_logit(j)] - mxl);
      s += ow[j];
    }
    for (int j = 0; j < L; ++j) ow[j] /= s;
  }
  float outacc[4] = {0.f, 0.f, 0.f, 0.f};  // Dv <= 4 * blockDim
  for (int j = 0; j < L; ++j) {
    const int M = a.M[j];
    float* kv = tmp;   // u(slot_j)
    float* qv = tmp2;  // u(qo_j)
    unit_vec(kv, sm + Lm.slot + j * mx, M, red);
    unit_vec(qv, sm + Lm.qo + j * mx, M, red);
    const int64_t szB = (int64_t)M * Dv;
    float* Bg = a.s.outer[j] + u * szB;
    load_mat(Ss, Bg, (int)szB, nullptr, bl);
    float* pre = sm + Lm.pre;
    colsum(Ss, M, Dv, kv, pre, part);
    const float* gt = sm + Lm.gates + 4 * j;
    float* yv = sm + Lm.yb;
    gdn_update(Ss, Bg, M, Dv, kv, sm + Lm.valin + j * Dv, pre, gt[2], gt[3], qv, yv, part);
    for (int i = threadIdx.x, c = 0; i < Dv; i += blockDim.x, ++c) outacc[c] += ow[j] * yv[i];
  }
  for (int i = threadIdx.x, c = 0; i < Dv; i += blockDim.x, ++c)
    store_out(a.out, (int64_t)u * Dv + i, outacc[c], a.dt);
  // Offset advance: every CTA read the offset on entry, before it counts itself done here, so
  // the last CTA to arrive may overwrite it.  It also resets the counter for the next step.
  __syncthreads();
  if (threadIdx.x == 0) {
    if (!bl.ok) atomicExch(&g_decode_status, GPA_B200_DEVICE_TIMEOUT);
    __threadfence();
    const unsigned done = atomicAdd(reinterpret_cast<unsigned*>(a.offset + 1), 1u);
    if (done == gridDim.x - 1) {
      a.offset[0] = (o + 1) % a.C;
      a.offset[2] = pos + 1;
      a.offset[1] = 0;
      __threadfence();
    }
  }
}

}  // namespace

size_t decode_step_smem(const StepArgs& a) { return StepSmem(a).total; }

int decode_device_status(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_decode_status, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    const int z = 0;
    if (cudaMemcpyToSymbol(g_decode_status, &z, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}

cudaError_t launch_decode_step(const StepArgs& a, cudaStream_t st) {
  const size_t smem = decode_step_smem(a);
  if (smem > 227 * 1024) return cudaErrorInvalidConfiguration;
  cudaError_t e = cudaFuncSetAttribute(k_decode_step, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  {
    Launch scope("decode_step", st);
    k_decode_step<<<a.U, kStepThreads, smem, st>>>(a);
  }
  return cudaGetLastError();
}

}  // namespace gpa
