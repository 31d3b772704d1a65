// State sweeps of the chunked GDN scans on the 5th-generation tensor cores (tcgen05, TMEM
// accumulators, bulk TMA copies of the next block's operands).
//
// The forward sweep carries the state S [K x V] of one unit across its blocks:
//   W = U - Wk S,            S <- e^{G_c} S + K^T diag(lambda) W,   lambda_t = e^{G_c - G_t}
// (the WY / UT chunk form of gdn.cuh).  Both products run transposed, so that a TMEM lane is a
// value column v of the state for both of them:
//   W^T [V x c]  = S^T Wk^T          (A = S^T, 128 rows v, reduction over k; B = Wk, rows t)
//   S'^T [V x K] = (lambda W)^T K    (A = (lambda W)^T, rows v, reduction over t; B = K, rows k)
// and S' = e^{G_c} S + S'^T^T is formed in the epilogue from the fp32 state each thread keeps in
// registers (thread (v, half) holds S[k][v] for half of the k).  The MMAs use M = 128 (rows v >=
// V are zero) and bf16 operands: Wk, K, lambda W as hi + lo pairs (three products: hi hi, hi lo,
// lo hi), S as hi only, the same precision split as the mma.sync sweep it replaces.
//
// Per block n of a unit (one CTA per unit and scan, 256 threads):
//   land the fp32 rows of Wk(n), K(n) (bulk copies issued during block n-1), convert them into
//   the bf16 operand tiles, issue the copies of block n+1, then
//   MMA 1 -> epilogue 1 (W = U - acc, W to global as bf16, lambda W to shared memory)
//   MMA 2 -> epilogue 2 (S update, boundary state to global, S^T hi to shared memory).
// One thread issues every MMA and commit; every wait on an mbarrier is bounded and a wait that
// gives up sets the library's device status to GPA_B200_DEVICE_TIMEOUT and ends the sweep.
#include "../../include/gpa_b200.h"
#include "gdn.cuh"
#include "gdn_dev.cuh"
#include "tc5.cuh"

#include <cuda_bf16.h>

#include <cstdlib>
#include <cstring>

namespace gpa {

__device__ int g_device_status = 0;

namespace {

using bf16 = __nv_bfloat16;
constexpr int C = kMaxChunk;       // 64 tokens per block tile
constexpr int kSweepThreads = 256;  // 8 warps: two per TMEM lane quarter
constexpr int kSweepCols = 256;     // TMEM columns: W^T at 0 (64), S^T at 64 (<= 128)
constexpr int kMaxScanWidth = 128;  // K, V <= 128 (checked by the API)

struct SweepGates {
  float g0, g1;
};

// gates of block (t0, c) in registers of warp 0 (t = lane, lane + 32)
GPA_DEV SweepGates sweep_gate_fetch(const ScanDesc& d, int u, int t0, int c) {
  SweepGates r{0.f, 0.f};
  if (threadIdx.x < 32) {
    const int t = threadIdx.x;
    if (t < c) r.g0 = gate_at(d.g, d, u, t0 + t);
    if (t + 32 < c) r.g1 = gate_at(d.g, d, u, t0 + t + 32);
  }
  return r;
}

// G = inclusive cumsum of g (rows >= c hold G[c-1]) and lambda_t = e^{G_{c-1} - G_t} (0 for
// t >= c), written to shared memory by warp 0; the caller synchronizes.
GPA_DEV void sweep_gate_finish(const SweepGates& r, int c, float* G, float* lam) {
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
    lam[t] = t < c ? __expf(last - x0) : 0.f;
    lam[t + 32] = t + 32 < c ? __expf(last - x1) : 0.f;
  }
}

// 8 consecutive fp32 values -> their bf16 hi and lo parts as two 16-byte groups
GPA_DEV void split8(const float (&x)[8], uint4& hi, uint4& lo) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 p = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
    const float2 f = __bfloat1622float2(p);
    const __nv_bfloat162 q = __floats2bfloat162_rn(x[2 * i] - f.x, x[2 * i + 1] - f.y);
    h[i] = *reinterpret_cast<const uint32_t*>(&p);
    l[i] = *reinterpret_cast<const uint32_t*>(&q);
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

GPA_DEV uint4 pack8(const float (&x)[8]) {
  uint32_t h[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 p = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
    h[i] = *reinterpret_cast<const uint32_t*>(&p);
  }
  return make_uint4(h[0], h[1], h[2], h[3]);
}

// fp32 rows [c x K] staged in shared memory (row stride K) -> bf16 hi / lo operand tiles of 64
// rows t (rows >= c zero): K-major (rows t, reduction k) when kmajor, else MN-major with the
// rows k and the reduction over t.  A thread converts 8 consecutive k of one row per step;
// the 8 lanes of a shared-memory phase take 8 different t (conflict-free 16-byte stores).
GPA_DEV void stage_to_tiles(const float* raw, int c, int K, bool kmajor, unsigned char* hi,
                            unsigned char* lo) {
  // item i: row t = 8 * (i / (8 * k8n)) + j and column group k8 = (i / 8 + j) % k8n with
  // j = i % 8: the 8 lanes of a shared-memory phase read 8 rows at 8 different column groups
  // (2-way bank conflicts at most) and write 8 different core-matrix rows (none)
  const int k8n = K >> 3, n = C * k8n;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int j = i & 7, g = i >> 3, tq = g / k8n;
    const int t = 8 * tq + j, k8 = (g - tq * k8n + j) % k8n;
    float x[8];
    if (t < c) {
      const float4 a = *reinterpret_cast<const float4*>(raw + t * K + 8 * k8);
      const float4 b = *reinterpret_cast<const float4*>(raw + t * K + 8 * k8 + 4);
      x[0] = a.x, x[1] = a.y, x[2] = a.z, x[3] = a.w, x[4] = b.x, x[5] = b.y, x[6] = b.z, x[7] = b.w;
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) x[q] = 0.f;
    }
    uint4 h, l;
    split8(x, h, l);
    // the 8 k of this group form one core-matrix row in both layouts
    const uint32_t o = kmajor ? tc5::kmajor_off(t, 8 * k8, K) : tc5::mnmajor_off(8 * k8, t, C);
    *reinterpret_cast<uint4*>(hi + o) = h;
    if (lo) *reinterpret_cast<uint4*>(lo + o) = l;
  }
}

// A global load issued exactly here (the compiler may not sink it to the value's first use):
// the U values of the next block are in flight during this block's MMA 2 and epilogue 2.
GPA_DEV float ld_pinned(const float* p) {
  float x;
  asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(x) : "l"(p));
  return x;
}

struct LFwdSweep {
  uint32_t St, WkH, WkL, WtH, WtL, KbH, KbL, rawWk, rawK, G, lam, bar, slot, total;
  __host__ __device__ LFwdSweep(int K, int V) {
    uint32_t o = 0;
    auto take = [&](uint32_t b) {
      o = (o + 127u) & ~127u;
      const uint32_t r = o;
      o += b;
      return r;
    };
    St = take(128 * K * 2);   // S^T hi: A of MMA 1, K-major, rows v (128), reduction k
    WkH = take(C * K * 2);    // Wk: B of MMA 1, K-major, rows t, reduction k
    WkL = take(C * K * 2);
    WtH = take(128 * C * 2);  // (lambda W)^T: A of MMA 2, K-major, rows v, reduction t
    WtL = take(128 * C * 2);
    KbH = take(K * C * 2);    // K: B of MMA 2, MN-major, rows k, reduction t
    KbL = take(K * C * 2);
    rawWk = take(C * K * 4);  // fp32 rows of the next block, landed by bulk copies
    rawK = take(C * K * 4);
    G = take(C * 4);
    lam = take(C * 4);
    bar = take(2 * 8);
    slot = take(16);
    total = o;
    (void)V;
  }
};

GPA_DEV void fail_status() { atomicExch(&g_device_status, GPA_B200_DEVICE_TIMEOUT); }

// grid (U, nscan), 256 threads.  KMAX bounds the key width K (64: two CTAs per SM).
//
// Per block n: MMA 1 (W^T) -> epilogue 1 (issues the U loads of block n+1 when done) -> MMA 2
// (S^T), during which the landed fp32 Wk rows of block n+1 become its MMA-1 operand -> epilogue
// 2 -> the K rows of block n+1 become its MMA-2 operand -> the bulk copies of block n+2 start.
template <int KMAX>
__global__ void __launch_bounds__(kSweepThreads, KMAX <= 64 ? 2 : 1)
    tc5_fwd_state(ScanBatch b, int U, Blocks bl) {
  const ScanDesc& d = b.s[blockIdx.y];
  const int u = blockIdx.x, K = d.K, V = d.V, T = bl.T;
  extern __shared__ __align__(1024) unsigned char sm[];
  const LFwdSweep L(K, V);
  unsigned char* St = sm + L.St;
  unsigned char* WkH = sm + L.WkH;
  unsigned char* WkL = sm + L.WkL;
  unsigned char* WtH = sm + L.WtH;
  unsigned char* WtL = sm + L.WtL;
  unsigned char* KbH = sm + L.KbH;
  unsigned char* KbL = sm + L.KbL;
  float* rawWk = reinterpret_cast<float*>(sm + L.rawWk);
  float* rawK = reinterpret_cast<float*>(sm + L.rawK);
  float* G = reinterpret_cast<float*>(sm + L.G);
  float* lam = reinterpret_cast<float*>(sm + L.lam);
  uint64_t* bar_mma = reinterpret_cast<uint64_t*>(sm + L.bar);
  uint64_t* bar_tma = bar_mma + 1;
  uint32_t* slot = reinterpret_cast<uint32_t*>(sm + L.slot);
  constexpr int SH = KMAX / 2;  // state values per thread (max)
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q = warp & 3, half = warp >> 2;
  const int v = 32 * q + lane;
  const bool active = 32 * q < V;  // warp-uniform: the quarter holds state columns
  const bool vok = v < V;
  const int KH = K >> 1, k0 = half * KH;  // this thread's state rows k0 .. k0 + KH - 1
  const int64_t KV = (int64_t)K * V;
  bf16* Wout = reinterpret_cast<bf16*>(d.W);

  // A tiles: rows v >= V stay zero for the whole sweep
  for (uint32_t i = tid * 16; i < 128u * K * 2; i += blockDim.x * 16)
    *reinterpret_cast<uint4*>(St + i) = make_uint4(0, 0, 0, 0);
  for (uint32_t i = tid * 16; i < 128u * C * 2; i += blockDim.x * 16) {
    *reinterpret_cast<uint4*>(WtH + i) = make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4*>(WtL + i) = make_uint4(0, 0, 0, 0);
  }
  if (warp == 0) tc5::tmem_alloc(slot, kSweepCols);
  if (tid == 0) {
    tc5::mbar_init(bar_mma, 1);
    tc5::mbar_init(bar_tma, 1);
    tc5::mbar_fence_init();
  }
  auto issue_rows = [&](int n) {  // bulk copies of block n's fp32 rows of Wk and K
    const int t0 = bl.start(n), c = bl.end(n) - t0;
    const uint32_t bytes = (uint32_t)(c * K * 4);
    tc5::mbar_expect_tx(bar_tma, 2 * bytes);
    tc5::bulk_g2s(rawWk, d.Wk + row(u, T, t0) * K, bytes, bar_tma);
    tc5::bulk_g2s(rawK, d.k + row(u, T, t0) * K, bytes, bar_tma);
  };
  float ub[32];  // U[t][v] of this thread's 32 tokens of the coming epilogue 1
  auto load_u = [&](int n) {
    const int t0 = bl.start(n), c = bl.end(n) - t0;
    const float* up = d.Ub + row(u, T, t0 + 32 * half) * V + v;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      ub[j] = (active && vok && 32 * half + j < c) ? ld_pinned(up + (int64_t)j * V) : 0.f;
  };
  float s[SH];
#pragma unroll
  for (int i = 0; i < SH; ++i) s[i] = 0.f;
  tc5::fence_before_sync();
  __syncthreads();  // barriers initialised, tiles zeroed, TMEM allocated
  tc5::fence_after_sync();
  if (tid == 0) issue_rows(0);
  // initial state: S_0 into registers, the first boundary and the S^T hi tile
  if (active) {
    float* sb0 = d.Sb + (int64_t)u * (bl.nb + 1) * KV;
#pragma unroll
    for (int i = 0; i < SH; i += 8) {
      if (i < KH) {
        float x[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          x[j] = vok ? d.S0[(int64_t)u * KV + (int64_t)(k0 + i + j) * V + v] : 0.f;
          s[i + j] = x[j];
          if (vok) sb0[(int64_t)(k0 + i + j) * V + v] = x[j];
        }
        *reinterpret_cast<uint4*>(St + tc5::kmajor_off(v, k0 + i, K)) = pack8(x);
      }
    }
  }
  load_u(0);
  uint32_t tph = 0, mph = 0;
  bool ok = true, all_ok = true;
  {
    const int c0 = bl.end(0) - bl.start(0);
    sweep_gate_finish(sweep_gate_fetch(d, u, 0, c0), c0, G, lam);
    ok = tc5::mbar_wait(bar_tma, tph);
    tph ^= 1;
    stage_to_tiles(rawWk, c0, K, true, WkH, WkL);
    stage_to_tiles(rawK, c0, K, false, KbH, KbL);
  }
  SweepGates gr{0.f, 0.f};
  if (bl.nb > 1) gr = sweep_gate_fetch(d, u, bl.start(1), bl.end(1) - bl.start(1));
  tc5::fence_async_smem();
  tc5::fence_before_sync();
  all_ok = __syncthreads_and(ok);
  tc5::fence_after_sync();
  const uint32_t tbase = *slot;
  if (tid == 0 && all_ok && bl.nb > 1) issue_rows(1);
  const uint32_t id1 = tc5::idesc_bf16(128, C, false, false);
  const uint32_t id2 = tc5::idesc_bf16(128, K, false, true);
  for (int n = 0; all_ok && n < bl.nb; ++n) {
    const int t0 = bl.start(n), c = bl.end(n) - t0;
    const bool more = n + 1 < bl.nb;
    if (tid == 0) {  // MMA 1: W^T = S^T Wk^T (Wk hi and lo)
      const uint32_t a = tc5::saddr(St), bh = tc5::saddr(WkH), bl_ = tc5::saddr(WkL);
      for (int ks = 0; ks < K / 16; ++ks)
        tc5::mma(tbase, tc5::sdesc(a, K, ks), tc5::sdesc(bh, K, ks), id1, ks > 0);
      for (int ks = 0; ks < K / 16; ++ks)
        tc5::mma(tbase, tc5::sdesc(a, K, ks), tc5::sdesc(bl_, K, ks), id1, true);
      tc5::commit(bar_mma);
    }
    ok = ok && tc5::mbar_wait(bar_mma, mph);
    mph ^= 1;
    tc5::fence_after_sync();
    if (active) {  // epilogue 1: W = U - acc; W out (bf16); lambda W hi / lo -> (lambda W)^T
      float acc2[2][16];
      tc5::tmem_ld16(tc5::tmem_at(tbase, 32 * half), acc2[0]);
      tc5::tmem_ld16(tc5::tmem_at(tbase, 32 * half + 16), acc2[1]);
      tc5::tmem_wait_ld();
#pragma unroll
      for (int c16 = 0; c16 < 2; ++c16) {
        const float(&acc)[16] = acc2[c16];
#pragma unroll
        for (int j8 = 0; j8 < 2; ++j8) {
          float x[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int jj = 16 * c16 + 8 * j8 + j, t = 32 * half + jj;
            const float w = (vok && t < c) ? ub[jj] - acc[8 * j8 + j] : 0.f;
            if (vok && t < c) Wout[row(u, T, t0 + t) * V + v] = __float2bfloat16(w);
            x[j] = w * lam[t];
          }
          uint4 h, l;
          split8(x, h, l);
          const uint32_t o = tc5::kmajor_off(v, 32 * half + 16 * c16 + 8 * j8, C);
          *reinterpret_cast<uint4*>(WtH + o) = h;
          *reinterpret_cast<uint4*>(WtL + o) = l;
        }
      }
    }
    if (more) load_u(n + 1);
    tc5::fence_async_smem();
    tc5::fence_before_sync();
    __syncthreads();
    tc5::fence_after_sync();
    if (tid == 0 && ok) {  // MMA 2: S'^T = (lambda W)^T K (hi hi, hi lo, lo hi)
      const uint32_t ah = tc5::saddr(WtH), al = tc5::saddr(WtL);
      const uint32_t bh = tc5::saddr(KbH), bl_ = tc5::saddr(KbL);
      const uint32_t d2 = tbase + C;
      for (int ks = 0; ks < C / 16; ++ks) {
        tc5::mma(d2, tc5::sdesc(ah, C, ks), tc5::sdesc(bh, C, ks), id2, ks > 0);
        tc5::mma(d2, tc5::sdesc(ah, C, ks), tc5::sdesc(bl_, C, ks), id2, true);
        tc5::mma(d2, tc5::sdesc(al, C, ks), tc5::sdesc(bh, C, ks), id2, true);
      }
      tc5::commit(bar_mma);
    }
    int cn = 0;
    if (more) {  // while MMA 2 runs: the next block's Wk rows -> its MMA-1 operand
      cn = bl.end(n + 1) - bl.start(n + 1);
      ok = ok && tc5::mbar_wait(bar_tma, tph);
      tph ^= 1;
      stage_to_tiles(rawWk, cn, K, true, WkH, WkL);
    }
    ok = ok && tc5::mbar_wait(bar_mma, mph);
    mph ^= 1;
    tc5::fence_after_sync();
    const float gc = __expf(G[c - 1]);
    if (active) {  // epilogue 2: S <- e^{G_c} S + acc; boundary state out; S^T hi tile
      // (the boundary stores stay here: issued under the next MMA they slowed the sweep down)
      float* sbn = d.Sb + ((int64_t)u * (bl.nb + 1) + n + 1) * KV;
#pragma unroll
      for (int i = 0; i < SH; i += 16) {
        if (i < KH) {
          float acc[16];
          tc5::tmem_ld16(tc5::tmem_at(tbase, C + k0 + i), acc);
          tc5::tmem_wait_ld();
#pragma unroll
          for (int h8 = 0; h8 < 16; h8 += 8) {
            if (i + h8 < KH) {
              float x[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const float sv = gc * s[i + h8 + j] + acc[h8 + j];
                s[i + h8 + j] = sv;
                x[j] = sv;
                if (vok) sbn[(int64_t)(k0 + i + h8 + j) * V + v] = sv;
              }
              *reinterpret_cast<uint4*>(St + tc5::kmajor_off(v, k0 + i + h8, K)) = pack8(x);
            }
          }
        }
      }
    }
    if (more) {  // the next block's K rows -> its MMA-2 operand; its gates
      stage_to_tiles(rawK, cn, K, false, KbH, KbL);
      __syncthreads();  // every thread has read G[c - 1]
      sweep_gate_finish(gr, cn, G, lam);
      if (n + 2 < bl.nb) gr = sweep_gate_fetch(d, u, bl.start(n + 2), bl.end(n + 2) - bl.start(n + 2));
    }
    tc5::fence_async_smem();
    tc5::fence_before_sync();
    all_ok = __syncthreads_and(ok);
    tc5::fence_after_sync();
    if (tid == 0 && all_ok && n + 2 < bl.nb) issue_rows(n + 2);  // the staging rows were read
  }
  if (all_ok && d.S_final && active && vok) {
#pragma unroll
    for (int i = 0; i < SH; ++i)
      if (i < KH) d.S_final[(int64_t)u * KV + (int64_t)(k0 + i) * V + v] = s[i];
  }
  if (!all_ok && tid == 0) {
    fail_status();
    tc5::mbar_wait(bar_tma, tph);  // a bulk copy may still be landing: bounded wait
  }
  tc5::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc5::tmem_free(tbase, kSweepCols);
}

// ------------------------------------------------------------------ backward state sweep

// The reverse sweep carries D = dL/dS [K x V] from the last block to the first:
//   dW = dW_local + diag(lambda) K D                 (dW_local: the read path's, in sc_dW)
//   D <- e^{G_c} D + (e^G Q)^T dO - Wk^T dW + ext_n
// Dend[n] holds D at the end of block n, dS0 the gradient of the initial state.  As in the
// forward sweep both products run transposed, a TMEM lane being a value column v:
//   X^T  [V x c] = D^T K^T                      (A = D^T hi / lo, 128 rows v; B = K, rows t)
//   D'^T [V x K] = dO^T (e^G Q) + (-dW)^T Wk    (A = dO^T, (-dW)^T hi / lo, rows v, reduction
//                                                over t; B = e^G Q, Wk hi / lo, MN-major)
// and D' = e^{G_c} D + ext_n + D'^T^T is formed in the epilogue from the fp32 D each thread
// keeps in registers (four threads per column v, each holding D[k][v] for a quarter of the
// k).  Products per block: D hi K + D lo K, dO Qg, and dW hi Wk hi + dW hi Wk lo + dW lo Wk
// hi: the operand split of the mma.sync sweep, with D carried in fp32 instead of a bf16 hi /
// lo pair.
//
// Per block n of a unit (one CTA per unit and scan, 512 threads):
//   MMA 1 issued; while it runs the e^G Q and Wk rows of block n are converted into their
//   operand tiles (straight from global memory, bulk-prefetched into L2 one block ahead),
//   dO^T is packed and the dW_local values of the epilogue are loaded;
//   epilogue 1 (dW out, (-dW)^T hi / lo); MMA 2 issued; while it runs the fp32 K rows of
//   block n-1 (landed by a bulk copy) become the next MMA-1 operand; epilogue 2 (D update,
//   Dend[n-1] or dS0 out, D^T hi / lo).
struct LBwdSweep {
  uint32_t DtH, DtL, Kb, dOt, NWh, NWl, Qb, WkH, WkL, rawK, G, lam, eG, bar, slot, total;
  __host__ __device__ LBwdSweep(int K, int V) {
    uint32_t o = 0;
    auto take = [&](uint32_t b) {
      o = (o + 127u) & ~127u;
      const uint32_t r = o;
      o += b;
      return r;
    };
    DtH = take(128 * K * 2);  // D^T: A of MMA 1, K-major, rows v (128), reduction k
    DtL = take(128 * K * 2);
    Kb = take(C * K * 2);     // K: B of MMA 1, K-major, rows t, reduction k (hi only)
    dOt = take(128 * C * 2);  // dO^T: A of MMA 2, K-major, rows v, reduction t (hi only)
    NWh = take(128 * C * 2);  // (-dW)^T: A of MMA 2, K-major, rows v, reduction t
    NWl = take(128 * C * 2);
    Qb = take(K * C * 2);     // e^G Q: B of MMA 2, MN-major, rows k, reduction t (hi only)
    WkH = take(K * C * 2);    // Wk: B of MMA 2, MN-major, rows k, reduction t
    WkL = take(K * C * 2);
    rawK = take(C * K * 4);   // fp32 K rows of the next block, landed by a bulk copy
    G = take(C * 4);
    lam = take(C * 4);
    eG = take(C * 4);
    bar = take(2 * 8);
    slot = take(16);
    total = o;
    (void)V;
  }
};

constexpr int kBwdThreads = 512;              // 16 warps: four per TMEM lane quarter
constexpr int kBwdParts = kBwdThreads / 128;  // threads per state column

// fp32 rows [c x K] in global memory (row stride K) -> bf16 operand tiles as stage_to_tiles
// lays them out (rows >= c zero), each row times rowmul[t] when given; every load of the
// thread is in flight before the first conversion.  kBwdThreads threads, K <= 128.
constexpr int kGlobalItems = C * kMaxScanWidth / 8 / kBwdThreads;
GPA_DEV void global_rows_to_tiles(const float* src, int c, int K, bool kmajor, unsigned char* hi,
                                  unsigned char* lo, const float* rowmul) {
  const int k8n = K >> 3, n = C * k8n;
  float4 a[kGlobalItems], b[kGlobalItems];
#pragma unroll
  for (int q = 0; q < kGlobalItems; ++q) {
    const int i = threadIdx.x + q * kBwdThreads;
    const int j = i & 7, g = i >> 3, tq = g / k8n;
    const int t = 8 * tq + j, k8 = (g - tq * k8n + j) % k8n;
    if (i < n && t < c) {
      const float* p = src + (int64_t)t * K + 8 * k8;
      a[q] = *reinterpret_cast<const float4*>(p);
      b[q] = *reinterpret_cast<const float4*>(p + 4);
    } else {
      a[q] = b[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
#pragma unroll
  for (int q = 0; q < kGlobalItems; ++q) {
    const int i = threadIdx.x + q * kBwdThreads;
    if (i < n) {
      const int j = i & 7, g = i >> 3, tq = g / k8n;
      const int t = 8 * tq + j, k8 = (g - tq * k8n + j) % k8n;
      const float f = (rowmul && t < c) ? rowmul[t] : 1.f;
      const float x[8] = {a[q].x * f, a[q].y * f, a[q].z * f, a[q].w * f,
                          b[q].x * f, b[q].y * f, b[q].z * f, b[q].w * f};
      const uint32_t o = kmajor ? tc5::kmajor_off(t, 8 * k8, K) : tc5::mnmajor_off(8 * k8, t, C);
      uint4 h, l;
      split8(x, h, l);
      *reinterpret_cast<uint4*>(hi + o) = h;
      if (lo) *reinterpret_cast<uint4*>(lo + o) = l;
    }
  }
}

// G, lambda (sweep_gate_finish) and eG_t = e^{G_t} (0 for t >= c) of a block, by warp 0.
GPA_DEV void bwd_gate_finish(const SweepGates& r, int c, float* G, float* lam, float* eG) {
  sweep_gate_finish(r, c, G, lam);
  if (threadIdx.x < 32) {
    const int t = threadIdx.x;
    __syncwarp();
    eG[t] = t < c ? __expf(G[t]) : 0.f;
    eG[t + 32] = t + 32 < c ? __expf(G[t + 32]) : 0.f;
  }
}

// grid (U, nscan), 512 threads, one CTA per SM.  KMAX bounds the key width K.
// Thread (v, part) of lane quarter v / 32 owns column v for tokens 16 part .. + 15 in epilogue
// 1 and for a contiguous range of up to KMAX / 4 state rows (whole groups of 8) in epilogue 2.
template <int KMAX>
__global__ void __launch_bounds__(kBwdThreads, 1) tc5_bwd_state(ScanBatch b, int U, Blocks bl) {
  const ScanDesc& d = b.s[blockIdx.y];
  const int u = blockIdx.x, K = d.K, V = d.V, T = bl.T;
  extern __shared__ __align__(1024) unsigned char sm[];
  const LBwdSweep L(K, V);
  unsigned char* DtH = sm + L.DtH;
  unsigned char* DtL = sm + L.DtL;
  unsigned char* Kb = sm + L.Kb;
  unsigned char* dOt = sm + L.dOt;
  unsigned char* NWh = sm + L.NWh;
  unsigned char* NWl = sm + L.NWl;
  unsigned char* Qb = sm + L.Qb;
  unsigned char* WkH = sm + L.WkH;
  unsigned char* WkL = sm + L.WkL;
  float* rawK = reinterpret_cast<float*>(sm + L.rawK);
  float* G = reinterpret_cast<float*>(sm + L.G);
  float* lam = reinterpret_cast<float*>(sm + L.lam);
  float* eG = reinterpret_cast<float*>(sm + L.eG);
  uint64_t* bar_mma = reinterpret_cast<uint64_t*>(sm + L.bar);
  uint64_t* bar_tma = bar_mma + 1;
  uint32_t* slot = reinterpret_cast<uint32_t*>(sm + L.slot);
  constexpr int SH = KMAX / kBwdParts;  // D values per thread (max)
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q = warp & 3, part = warp >> 2;
  const int v = 32 * q + lane;
  const bool active = 32 * q < V;  // warp-uniform: the quarter holds state columns
  const bool vok = v < V;
  const int gp = (K / 8 + kBwdParts - 1) / kBwdParts;  // groups of 8 rows per part
  const int kb = 8 * gp * part;                        // this thread's first row of D
  const int kn = max(0, min(K - kb, 8 * gp));          // and how many it holds
  const int tb = 16 * part;                            // its first token of epilogue 1
  const int64_t KV = (int64_t)K * V;
  const int nb = bl.nb;
  const float sc = d.dO_scale ? d.dO_scale[u] : 1.f;

  // A tiles: rows v >= V stay zero for the whole sweep
  for (uint32_t i = tid * 16; i < 128u * K * 2; i += blockDim.x * 16) {
    *reinterpret_cast<uint4*>(DtH + i) = make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4*>(DtL + i) = make_uint4(0, 0, 0, 0);
  }
  for (uint32_t i = tid * 16; i < 128u * C * 2; i += blockDim.x * 16) {
    *reinterpret_cast<uint4*>(dOt + i) = make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4*>(NWh + i) = make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4*>(NWl + i) = make_uint4(0, 0, 0, 0);
  }
  if (warp == 0) tc5::tmem_alloc(slot, kSweepCols);
  if (tid == 0) {
    tc5::mbar_init(bar_mma, 1);
    tc5::mbar_init(bar_tma, 1);
    tc5::mbar_fence_init();
  }
  auto issue_k = [&](int n) {  // bulk copy of block n's fp32 K rows
    const int t0 = bl.start(n), c = bl.end(n) - t0;
    const uint32_t bytes = (uint32_t)(c * K * 4);
    tc5::mbar_expect_tx(bar_tma, bytes);
    tc5::bulk_g2s(rawK, d.k + row(u, T, t0) * K, bytes, bar_tma);
  };
  // D^T hi / lo of this thread's rows (8 at a time) into the MMA-1 operand; D to dst
  float dr[SH];
  auto put_state = [&](float* dst) {
#pragma unroll
    for (int i = 0; i < SH; i += 8) {
      if (i < kn) {
        float x[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          x[j] = dr[i + j];
          if (vok) dst[(int64_t)(kb + i + j) * V + v] = x[j];
        }
        uint4 h, l;
        split8(x, h, l);
        const uint32_t o = tc5::kmajor_off(v, kb + i, K);
        *reinterpret_cast<uint4*>(DtH + o) = h;
        *reinterpret_cast<uint4*>(DtL + o) = l;
      }
    }
  };
  tc5::fence_before_sync();
  __syncthreads();  // barriers initialised, tiles zeroed, TMEM allocated
  tc5::fence_after_sync();
  if (tid == 0) issue_k(nb - 1);
#pragma unroll
  for (int i = 0; i < SH; ++i) dr[i] = 0.f;
  if (active) {  // D at the end of the last block: dS_final + ext[nb]
    const float* e0 = d.ext ? d.ext + ((int64_t)u * (nb + 1) + nb) * KV : nullptr;
    const float* f0 = d.dS_final ? d.dS_final + (int64_t)u * KV : nullptr;
#pragma unroll
    for (int i = 0; i < SH; ++i) {
      if (i < kn && vok) {
        const int64_t o = (int64_t)(kb + i) * V + v;
        dr[i] = (e0 ? e0[o] : 0.f) + (f0 ? f0[o] : 0.f);
      }
    }
    put_state(d.Dend + ((int64_t)u * nb + nb - 1) * KV);
  }
  uint32_t tph = 0, mph = 0;
  bool ok = true, all_ok = true;
  {
    const int cl = bl.end(nb - 1) - bl.start(nb - 1);
    bwd_gate_finish(sweep_gate_fetch(d, u, bl.start(nb - 1), cl), cl, G, lam, eG);
    ok = tc5::mbar_wait(bar_tma, tph);
    tph ^= 1;
    stage_to_tiles(rawK, cl, K, true, Kb, nullptr);
  }
  SweepGates gr{0.f, 0.f};
  if (nb > 1) gr = sweep_gate_fetch(d, u, bl.start(nb - 2), bl.end(nb - 2) - bl.start(nb - 2));
  tc5::fence_async_smem();
  tc5::fence_before_sync();
  all_ok = __syncthreads_and(ok);
  tc5::fence_after_sync();
  const uint32_t tbase = *slot;
  if (tid == 0 && all_ok && nb > 1) issue_k(nb - 2);
  const uint32_t id1 = tc5::idesc_bf16(128, C, false, false);
  const uint32_t id2 = tc5::idesc_bf16(128, K, false, true);
  for (int n = nb - 1; all_ok && n >= 0; --n) {
    const int t0 = bl.start(n), c = bl.end(n) - t0;
    const int64_t r0 = row(u, T, t0);
    if (tid == 0) {
      // MMA 1: X^T = D^T K^T (D hi and lo)
      const uint32_t ah = tc5::saddr(DtH), al = tc5::saddr(DtL), bk = tc5::saddr(Kb);
      for (int ks = 0; ks < K / 16; ++ks)
        tc5::mma(tbase, tc5::sdesc(ah, K, ks), tc5::sdesc(bk, K, ks), id1, ks > 0);
      for (int ks = 0; ks < K / 16; ++ks)
        tc5::mma(tbase, tc5::sdesc(al, K, ks), tc5::sdesc(bk, K, ks), id1, true);
      tc5::commit(bar_mma);
      if (n > 0) {  // the rows block n - 1 reads, towards L2 while this block computes
        const int p0 = bl.start(n - 1), pc = bl.end(n - 1) - p0;
        const int64_t pr = row(u, T, p0);
        tc5::prefetch_l2(d.q + pr * K, (uint32_t)(pc * K * 4));
        tc5::prefetch_l2(d.Wk + pr * K, (uint32_t)(pc * K * 4));
        tc5::prefetch_l2(d.dO + pr * V, (uint32_t)(pc * V * 4));
        tc5::prefetch_l2(d.sc_dW + pr * V, (uint32_t)(pc * V * 4));
        if (d.ext) tc5::prefetch_l2(d.ext + ((int64_t)u * (nb + 1) + n - 1) * KV, (uint32_t)(KV * 4));
      }
    }
    // while MMA 1 runs: this thread's dO and dW_local values (loads issued first), the MMA-2
    // B operands of block n, dO^T
    float dw[16], o16[16];
    {
      const bool act = active && vok;
      const float* op = d.dO + row(u, T, t0 + tb) * V + v;
      const float* wp = d.sc_dW + row(u, T, t0 + tb) * V + v;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const bool in = act && tb + j < c;
        o16[j] = in ? ld_pinned(op + (int64_t)j * V) : 0.f;
        dw[j] = in ? ld_pinned(wp + (int64_t)j * V) : 0.f;
      }
    }
    global_rows_to_tiles(d.q + r0 * K, c, K, false, Qb, nullptr, eG);
    global_rows_to_tiles(d.Wk + r0 * K, c, K, false, WkH, WkL, nullptr);
    if (active) {
#pragma unroll
      for (int g8 = 0; g8 < 2; ++g8) {
        float x[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) x[j] = sc * o16[8 * g8 + j];
        *reinterpret_cast<uint4*>(dOt + tc5::kmajor_off(v, tb + 8 * g8, C)) = pack8(x);
      }
    }
    ok = ok && tc5::mbar_wait(bar_mma, mph);
    mph ^= 1;
    tc5::fence_after_sync();
    if (active) {  // epilogue 1: dW = dW_local + lambda X; dW out; (-dW)^T hi / lo
      float acc[16];
      tc5::tmem_ld16(tc5::tmem_at(tbase, tb), acc);
      tc5::tmem_wait_ld();
#pragma unroll
      for (int j8 = 0; j8 < 2; ++j8) {
        float x[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int jj = 8 * j8 + j, t = tb + jj;
          const bool in = vok && t < c;
          const float w = in ? dw[jj] + lam[t] * acc[jj] : 0.f;
          if (in) d.sc_dW[row(u, T, t0 + t) * V + v] = w;
          x[j] = -w;
        }
        uint4 h, l;
        split8(x, h, l);
        const uint32_t o = tc5::kmajor_off(v, tb + 8 * j8, C);
        *reinterpret_cast<uint4*>(NWh + o) = h;
        *reinterpret_cast<uint4*>(NWl + o) = l;
      }
    }
    tc5::fence_async_smem();
    tc5::fence_before_sync();
    __syncthreads();
    tc5::fence_after_sync();
    if (tid == 0 && ok) {  // MMA 2: D'^T = dO^T Qg + (-dW)^T Wk (hi hi, hi lo, lo hi)
      const uint32_t ao = tc5::saddr(dOt), ah = tc5::saddr(NWh), al = tc5::saddr(NWl);
      const uint32_t bq = tc5::saddr(Qb), bh = tc5::saddr(WkH), bl_ = tc5::saddr(WkL);
      const uint32_t d2 = tbase + C;
      for (int ks = 0; ks < C / 16; ++ks) {
        tc5::mma(d2, tc5::sdesc(ao, C, ks), tc5::sdesc(bq, C, ks), id2, ks > 0);
        tc5::mma(d2, tc5::sdesc(ah, C, ks), tc5::sdesc(bh, C, ks), id2, true);
        tc5::mma(d2, tc5::sdesc(ah, C, ks), tc5::sdesc(bl_, C, ks), id2, true);
        tc5::mma(d2, tc5::sdesc(al, C, ks), tc5::sdesc(bh, C, ks), id2, true);
      }
      tc5::commit(bar_mma);
    }
    // ext_n of this thread's D rows, 16 at a time in two alternating buffers: the first
    // group is loaded while MMA 2 runs, each next one before the current group is used
    const float* ext = (d.ext && active && vok) ? d.ext + ((int64_t)u * (nb + 1) + n) * KV + v : nullptr;
    float ea[16], eb[16];
    auto load_ext = [&](float (&e)[16], int i) {
#pragma unroll
      for (int j = 0; j < 16; ++j)
        e[j] = (ext && i + j < kn) ? ext[(int64_t)(kb + i + j) * V] : 0.f;
    };
    load_ext(ea, 0);
    int cn = 0;
    if (n > 0) {  // while MMA 2 runs: the K rows of block n - 1 -> its MMA-1 operand
      cn = bl.end(n - 1) - bl.start(n - 1);
      ok = ok && tc5::mbar_wait(bar_tma, tph);
      tph ^= 1;
      stage_to_tiles(rawK, cn, K, true, Kb, nullptr);
    }
    ok = ok && tc5::mbar_wait(bar_mma, mph);
    mph ^= 1;
    tc5::fence_after_sync();
    const float gc = __expf(G[c - 1]);
    if (active) {  // epilogue 2: D <- e^{G_c} D + acc + ext_n; Dend[n - 1] (or dS0); D^T tiles
#pragma unroll
      for (int i = 0; i < SH; i += 16) {
        if (i < kn) {
          float(&cur)[16] = ((i >> 4) & 1) ? eb : ea;
          float(&nxt)[16] = ((i >> 4) & 1) ? ea : eb;
          if (i + 16 < kn) load_ext(nxt, i + 16);
          float acc[16];
          tc5::tmem_ld16(tc5::tmem_at(tbase, C + kb + i), acc);
          tc5::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) dr[i + j] = gc * dr[i + j] + acc[j] + cur[j];
        }
      }
      put_state(n > 0 ? d.Dend + ((int64_t)u * nb + n - 1) * KV : d.dS0 + (int64_t)u * KV);
    }
    if (n > 0) {  // the gates of block n - 1
      __syncthreads();  // every thread has read G[c - 1] and lambda
      bwd_gate_finish(gr, cn, G, lam, eG);
      if (n >= 2) gr = sweep_gate_fetch(d, u, bl.start(n - 2), bl.end(n - 2) - bl.start(n - 2));
    }
    tc5::fence_async_smem();
    tc5::fence_before_sync();
    all_ok = __syncthreads_and(ok);
    tc5::fence_after_sync();
    if (tid == 0 && all_ok && n >= 2) issue_k(n - 2);  // the staging rows were read
  }
  if (!all_ok && tid == 0) {
    fail_status();
    tc5::mbar_wait(bar_tma, tph);  // a bulk copy may still be landing: bounded wait
  }
  tc5::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc5::tmem_free(tbase, kSweepCols);
}

// ------------------------------------------------------------------ WY / UT transform

// Per block of c <= 64 tokens of a (K, V) scan (gdn.cuh):
//   A = strict_lower(b_t e^{G_t - G_s} k_t . k_s),   T = (I + A)^-1,
//   U = T diag(b) V,   Wk = T diag(b e^G) K.
// The three products run on tcgen05 with M = 64 (rows t; TMEM lanes 0-15 of each quarter):
//   A  = K K^T   (A and B the same K-major K tile, hi / lo: hi hi + hi lo + lo hi)
//   U  = F V     (F = T diag(b), hi / lo, K-major; V hi, MN-major)
//   Wk = F' K    (F' = T diag(b e^G), hi / lo; K read through the MN-major view of its tile)
// T comes from the same SIMT unit-lower inversion as the mma.sync kernel.  Each CTA is one
// dependent chain (loads, MMA, epilogue, inversion, MMA, stores), so throughput comes from
// chains overlapping: three CTAs per SM (at most 80 registers; 73 KB of shared memory for
// K = 128, V = 64).
struct LFwdChunk5 {
  uint32_t Kh, Kl, Vh, A, Tm, G, bt, bar, slot, total, Fh, Fl, F2h, F2l;
  __host__ __device__ LFwdChunk5(int K, int V) {
    uint32_t o = 0;
    auto take = [&](uint32_t b) {
      o = (o + 127u) & ~127u;
      const uint32_t r = o;
      o += b;
      return r;
    };
    Kh = take(C * K * 2);  // K tile, K-major: rows t, reduction k
    Kl = take(C * K * 2);
    Vh = take(V * C * 2);  // V tile, MN-major: rows v, reduction t
    A = take(4 * C * kAStride);
    Tm = take(4 * C * kAStride);
    G = take(4 * C);
    bt = take(4 * C);
    bar = take(8);
    slot = take(16);
    total = o;
    Fh = A;  // F = T diag(b), K-major (rows t, reduction s), over A once T is formed
    Fl = A + C * C * 2;
    F2h = Tm;  // F' = T diag(b e^G) over T once every thread holds its T values in registers
    F2l = Tm + C * C * 2;
  }
};

// One operand tile built from `rows` (64 tokens, or K rows of a state) fp32 source rows of
// width W (src at the tile's first row; rows >= the valid count zero): K-major (rows = the
// source rows, reduction over w) or MN-major (rows w, reduction over the source rows); bf16 hi
// (+ lo when lo is set); each source row t times e^{rowexp[t]} when rowexp is set.
struct RowTile {
  const float* src;
  int W;
  bool kmajor;
  unsigned char* hi;
  unsigned char* lo;
  int rows = C;
  const float* rowexp = nullptr;
};

// Items of 8 consecutive w of one row a thread takes per pass: C * W / 8 / threads for W <=
// 128; a K x V state tile takes K / C passes.
constexpr int kRowItems = C * kMaxScanWidth / 8 / kSweepThreads;
static_assert(kRowItems * kSweepThreads * 8 == C * kMaxScanWidth, "row items cover the tile");
using RowRegs = float4[kRowItems][2];

// Item i of a tile: row t and column group w8 (8 columns).  The 8 lanes of a shared-memory
// phase take 8 rows at 8 different column groups (conflict-free 16-byte stores).
GPA_DEV void row_item(int i, int w8n, int& t, int& w8) {
  const int j = i & 7, g = i >> 3, tq = g / w8n;
  t = 8 * tq + j;
  w8 = (g - tq * w8n + j) % w8n;
}

// Issue every global load of this thread's items of pass `pass` of tile J (all in flight at
// once); source rows >= `valid` read as zero.
GPA_DEV void tile_fetch(const RowTile& J, int valid, RowRegs& v, int pass = 0) {
  const int w8n = J.W >> 3, n = J.rows * w8n;
#pragma unroll
  for (int q = 0; q < kRowItems; ++q) {
    const int i = threadIdx.x + (pass * kRowItems + q) * kSweepThreads;
    int t, w8;
    row_item(i, w8n, t, w8);
    if (i < n && t < valid) {
      const float* p = J.src + (int64_t)t * J.W + 8 * w8;
      v[q][0] = *reinterpret_cast<const float4*>(p);
      v[q][1] = *reinterpret_cast<const float4*>(p + 4);
    } else {
      v[q][0] = v[q][1] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
}

// Convert the fetched items of pass `pass` into the bf16 operand tile(s) of J.
GPA_DEV void tile_store(const RowTile& J, const RowRegs& v, int pass = 0) {
  const int w8n = J.W >> 3, n = J.rows * w8n;
#pragma unroll
  for (int q = 0; q < kRowItems; ++q) {
    const int i = threadIdx.x + (pass * kRowItems + q) * kSweepThreads;
    if (i >= n) continue;
    int t, w8;
    row_item(i, w8n, t, w8);
    const float4 a = v[q][0], b = v[q][1];
    float x[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    if (J.rowexp) {
      const float f = __expf(J.rowexp[t]);
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] *= f;
    }
    const uint32_t o =
        J.kmajor ? tc5::kmajor_off(t, 8 * w8, J.W) : tc5::mnmajor_off(8 * w8, t, J.rows);
    if (J.lo) {
      uint4 h, l;
      split8(x, h, l);
      *reinterpret_cast<uint4*>(J.hi + o) = h;
      *reinterpret_cast<uint4*>(J.lo + o) = l;
    } else {
      *reinterpret_cast<uint4*>(J.hi + o) = pack8(x);
    }
  }
}

// bf16 rows [C x W] (src at the tile's first row, row stride W; rows >= `valid` zero) -> the
// MN-major bf16 tile with rows w and the reduction over the C rows: each item is one 16-byte
// core-matrix row, loaded (all in flight) and stored as is.
GPA_DEV void bf16_rows_to_mn(const bf16* src, int valid, int W, unsigned char* dst) {
  const int w8n = W >> 3, n = C * w8n;
  uint4 v[kRowItems];
#pragma unroll
  for (int q = 0; q < kRowItems; ++q) {
    const int i = threadIdx.x + q * kSweepThreads;
    int t, w8;
    row_item(i, w8n, t, w8);
    v[q] = i < n && t < valid ? *reinterpret_cast<const uint4*>(src + (int64_t)t * W + 8 * w8)
                              : make_uint4(0u, 0u, 0u, 0u);
  }
#pragma unroll
  for (int q = 0; q < kRowItems; ++q) {
    const int i = threadIdx.x + q * kSweepThreads;
    if (i >= n) continue;
    int t, w8;
    row_item(i, w8n, t, w8);
    *reinterpret_cast<uint4*>(dst + tc5::mnmajor_off(8 * w8, t, C)) = v[q];
  }
}

// Warp 0: G = inclusive cumsum of g over the block (rows >= c hold G[c-1]) and, when bt is
// set, bt = beta (0 for rows >= c).  The caller synchronizes.
GPA_DEV void chunk_gates(const ScanDesc& d, int u, int t0, int c, float* G, float* bt) {
  if (threadIdx.x < 32) {
    const int t = threadIdx.x;
    float x0 = t < c ? gate_at(d.g, d, u, t0 + t) : 0.f;
    float x1 = t + 32 < c ? gate_at(d.g, d, u, t0 + t + 32) : 0.f;
    const float b0 = bt && t < c ? gate_at(d.beta, d, u, t0 + t) : 0.f;
    const float b1 = bt && t + 32 < c ? gate_at(d.beta, d, u, t0 + t + 32) : 0.f;
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
      bt[t] = b0;
      bt[t + 32] = b1;
    }
  }
}

// F / F' items a thread builds: C rows x C / 8 column groups over the threads
constexpr int kFItems = C * (C / 8) / kSweepThreads;
static_assert(kFItems * kSweepThreads == C * (C / 8), "F items cover the tile");

// grid (U * NB, nscan), 256 threads.  Epilogues: TMEM lanes 0-15 of quarter q hold rows
// t = 16 q + lane; the two warps of a quarter take alternate 16-column chunks.
__global__ void __launch_bounds__(kSweepThreads, 3) tc5_fwd_chunk(ScanBatch b, int U, Blocks bl) {
  const ScanDesc& d = b.s[blockIdx.y];
  const int u = blockIdx.x / bl.nb, n = blockIdx.x % bl.nb, T = bl.T;
  const int t0 = bl.start(n), c = bl.end(n) - t0, K = d.K, V = d.V;
  extern __shared__ __align__(1024) unsigned char sm[];
  const LFwdChunk5 L(K, V);
  unsigned char* Kh = sm + L.Kh;
  unsigned char* Kl = sm + L.Kl;
  unsigned char* Vh = sm + L.Vh;
  unsigned char* Fh = sm + L.Fh;
  unsigned char* Fl = sm + L.Fl;
  unsigned char* F2h = sm + L.F2h;
  unsigned char* F2l = sm + L.F2l;
  float* A = reinterpret_cast<float*>(sm + L.A);
  float* Tm = reinterpret_cast<float*>(sm + L.Tm);
  float* G = reinterpret_cast<float*>(sm + L.G);
  float* bt = reinterpret_cast<float*>(sm + L.bt);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + L.bar);
  uint32_t* slot = reinterpret_cast<uint32_t*>(sm + L.slot);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int half = warp >> 2, trow = 16 * (warp & 3) + (lane & 15);
  const bool rowlane = lane < 16;
  // 128 TMEM columns (three CTAs per SM fit the 512): U at [0, V) and Wk at [V, V + K) when
  // both fit, else U and then Wk at [0, ...) in two rounds
  const bool split = V + K > 128;
  const int wc = split ? 0 : V;
  constexpr uint32_t ncols = 128;
  const int64_t r0 = row(u, T, t0);
  const RowTile kt{d.k + r0 * K, K, true, Kh, Kl}, vt{d.v + r0 * V, V, false, Vh, nullptr};

  if (warp == 0) tc5::tmem_alloc(slot, ncols);
  if (tid == 0) {
    tc5::mbar_init(bar, 1);
    tc5::mbar_fence_init();
    tc5::prefetch_l2(d.v + r0 * V, (uint32_t)(c * V * 4));  // fetched after the K tile
  }
  {
    RowRegs kv;
    tile_fetch(kt, c, kv);  // K loads in flight while warp 0 fetches and scans the gates
    chunk_gates(d, u, t0, c, G, bt);
    tile_store(kt, kv);
  }
  tc5::fence_async_smem();
  tc5::fence_before_sync();
  __syncthreads();
  tc5::fence_after_sync();
  const uint32_t tb = *slot;
  uint32_t ph = 0;
  bool ok = true;
  if (tid == 0) {  // A = K K^T (hi hi + hi lo + lo hi)
    const uint32_t id = tc5::idesc_bf16(C, C, false, false);
    const uint32_t h = tc5::saddr(Kh), l = tc5::saddr(Kl);
    for (int ks = 0; ks < K / 16; ++ks) {
      tc5::mma(tb, tc5::sdesc(h, K, ks), tc5::sdesc(h, K, ks), id, ks > 0);
      tc5::mma(tb, tc5::sdesc(h, K, ks), tc5::sdesc(l, K, ks), id, true);
      tc5::mma(tb, tc5::sdesc(l, K, ks), tc5::sdesc(h, K, ks), id, true);
    }
    tc5::commit(bar);
  }
  RowRegs vv;
  tile_fetch(vt, c, vv);  // V loads in flight during MMA 1 and its epilogue
  ok = tc5::mbar_wait(bar, ph);
  ph ^= 1;
  tc5::fence_after_sync();
  for (int ci = half; ci < C / 16; ci += 2) {  // A[t][s] = b_t e^{G_t - G_s} (k_t . k_s), s < t
    float acc[16];
    tc5::tmem_ld16(tc5::tmem_at(tb, 16 * ci), acc);
    tc5::tmem_wait_ld();
    if (rowlane) {
      const float gt = G[trow], bb = bt[trow];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int s = 16 * ci + j;
        A[trow * kAStride + s] = s < trow ? bb * __expf(gt - G[s]) * acc[j] : 0.f;
      }
    }
  }
  tile_store(vt, vv);  // read by MMA 2 after the proxy fence below
  __syncthreads();
  invert_unit_lower(A, Tm);  // ends with __syncthreads: A is free below
  {
    // T out, then every thread's T values (F / F' items) into registers before F' overwrites T
    float* Ts = d.Tsv + ((int64_t)u * bl.nb + n) * C * C;
    for (int i = tid; i < C * C; i += blockDim.x) Ts[i] = Tm[(i / C) * kAStride + (i % C)];
    float x[kFItems][8];
#pragma unroll
    for (int q = 0; q < kFItems; ++q) {
      const int i = tid + q * kSweepThreads, j = i & 7, g = i >> 3, tq = g >> 3;
      const int t = 8 * tq + j, s8 = ((g & 7) + j) & 7;
#pragma unroll
      for (int e = 0; e < 8; ++e) x[q][e] = Tm[t * kAStride + 8 * s8 + e] * bt[8 * s8 + e];
    }
    __syncthreads();
    // F = T diag(b) and F' = T diag(b e^G), hi / lo, K-major (rows t, reduction s)
#pragma unroll
    for (int q = 0; q < kFItems; ++q) {
      const int i = tid + q * kSweepThreads, j = i & 7, g = i >> 3, tq = g >> 3;
      const int t = 8 * tq + j, s8 = ((g & 7) + j) & 7;
      const uint32_t o = tc5::kmajor_off(t, 8 * s8, C);
      uint4 h, l;
      split8(x[q], h, l);
      *reinterpret_cast<uint4*>(Fh + o) = h;
      *reinterpret_cast<uint4*>(Fl + o) = l;
      float y[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) y[e] = x[q][e] * __expf(G[8 * s8 + e]);
      split8(y, h, l);
      *reinterpret_cast<uint4*>(F2h + o) = h;
      *reinterpret_cast<uint4*>(F2l + o) = l;
    }
  }
  tc5::fence_async_smem();
  tc5::fence_before_sync();
  __syncthreads();
  tc5::fence_after_sync();
  const uint32_t fh = tc5::saddr(Fh), fl = tc5::saddr(Fl), f2h = tc5::saddr(F2h),
                 f2l = tc5::saddr(F2l), vh = tc5::saddr(Vh), kh = tc5::saddr(Kh), kl = tc5::saddr(Kl);
  auto issue_u = [&] {  // U = F V -> columns [0, V)
    const uint32_t idu = tc5::idesc_bf16(C, V, false, true);
    for (int ks = 0; ks < C / 16; ++ks) {
      tc5::mma(tb, tc5::sdesc(fh, C, ks), tc5::sdesc(vh, C, ks), idu, ks > 0);
      tc5::mma(tb, tc5::sdesc(fl, C, ks), tc5::sdesc(vh, C, ks), idu, true);
    }
  };
  auto issue_w = [&] {  // Wk = F' K -> columns [wc, wc + K)
    const uint32_t idw = tc5::idesc_bf16(C, K, false, true);
    for (int ks = 0; ks < C / 16; ++ks) {
      tc5::mma(tb + wc, tc5::sdesc(f2h, C, ks), tc5::sdesc_mn_view(kh, K, ks), idw, ks > 0);
      tc5::mma(tb + wc, tc5::sdesc(f2h, C, ks), tc5::sdesc_mn_view(kl, K, ks), idw, true);
      tc5::mma(tb + wc, tc5::sdesc(f2l, C, ks), tc5::sdesc_mn_view(kh, K, ks), idw, true);
    }
  };
  // rows of U and Wk out: 16-column chunks ci (U for ci < nu, then Wk), read through the
  // 16-lane TMEM shape so that every lane holds data: lane l of quarter q has rows
  // 16 q + l / 4 and + 8, columns 2 (l % 4) + {0, 1} and + 8 of the chunk, stored as float2
  // (8 rows x 32 contiguous bytes per store instruction).  Two chunks per wait.
  const int nu = V / 16, nch = nu + K / 16;
  const int er = 16 * (warp & 3) + (lane >> 2), ec = 2 * (lane & 3);
  auto chunk_col = [&](int ci) { return ci < nu ? 16 * ci : wc + 16 * (ci - nu); };
  auto chunk_out = [&](int ci, const float (&v)[8]) {
    if (!ok) return;
    float* base = ci < nu ? d.Ub + r0 * V + 16 * ci + ec : d.Wk + r0 * K + 16 * (ci - nu) + ec;
    const int ld = ci < nu ? V : K;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int t = er + 8 * h;
      if (t < c) {
        float* p = base + (int64_t)t * ld;
        *reinterpret_cast<float2*>(p) = make_float2(v[2 * h], v[2 * h + 1]);
        *reinterpret_cast<float2*>(p + 8) = make_float2(v[4 + 2 * h], v[5 + 2 * h]);
      }
    }
  };
  auto epilogue = [&](int lo, int hi) {  // chunks [lo, hi)
    for (int ci = lo + half; ci < hi; ci += 4) {
      const bool two = ci + 2 < hi;  // warp-uniform
      float a0[8], a1[8];
      tc5::tmem_ld16x16(tc5::tmem_at(tb, chunk_col(ci)), a0);
      if (two) tc5::tmem_ld16x16(tc5::tmem_at(tb, chunk_col(ci + 2)), a1);
      tc5::tmem_wait_ld();
      chunk_out(ci, a0);
      if (two) chunk_out(ci + 2, a1);
    }
  };
  if (tid == 0 && ok) {
    issue_u();
    if (!split) issue_w();
    tc5::commit(bar);
  }
  ok = ok && tc5::mbar_wait(bar, ph);
  ph ^= 1;
  tc5::fence_after_sync();
  epilogue(0, split ? nu : nch);
  if (split) {  // Wk reuses the columns once every warp has read U
    tc5::fence_before_sync();
    __syncthreads();
    tc5::fence_after_sync();
    if (tid == 0 && ok) {
      issue_w();
      tc5::commit(bar);
    }
    ok = ok && tc5::mbar_wait(bar, ph);
    tc5::fence_after_sync();
    epilogue(nu, nch);
  }
  tc5::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc5::tmem_free(tb, ncols);
  if (!ok && tid == 0) fail_status();
}

// Per block of c <= 64 tokens of a scan with output (gdn.cuh): O = e^G (Q S_n) + P W with
// P = (Q K^T) o Gamma, Gamma_ts = e^{G_t - G_s} for s <= t (else 0).  Two tcgen05 rounds, M = 64
// (rows t; TMEM lanes 0-15 of each quarter), 128 TMEM columns:
//   P = Q K^T            Q, K hi, K-major                                  -> columns [0, 64)
//   O = Qg S + P W       Qg = diag(e^G) Q hi, K-major; S hi, MN-major (rows v, reduction k);
//                        P hi / lo, K-major; W hi (bf16 in memory), MN-major -> [0, V)
// with the operand precision of the mma.sync kernel (Q, K, S, W single bf16; P split).  The
// S and W tiles are built while the first round runs; Qg takes the K tile's place after it.
struct LFwdOut5 {
  uint32_t Qh, Kq, Sh, Wt, Ph, Pl, G, bar, slot, total;
  __host__ __device__ LFwdOut5(int K, int V) {
    uint32_t o = 0;
    auto take = [&](uint32_t b) {
      o = (o + 127u) & ~127u;
      const uint32_t r = o;
      o += b;
      return r;
    };
    Qh = take(C * K * 2);
    Kq = take(C * K * 2);  // K, then Qg
    Sh = take(K * V * 2);
    Wt = take(C * V * 2);
    Ph = take(C * C * 2);
    Pl = take(C * C * 2);
    G = take(4 * C);
    bar = take(8);
    slot = take(16);
    total = o;
  }
};

// grid (U * NB, nscan), 256 threads; scans without output return at once.
__global__ void __launch_bounds__(kSweepThreads, 3) tc5_fwd_out(ScanBatch b, int U, Blocks bl) {
  const ScanDesc& d = b.s[blockIdx.y];
  if (!d.q || !d.O) return;
  const int u = blockIdx.x / bl.nb, n = blockIdx.x % bl.nb, T = bl.T;
  const int t0 = bl.start(n), c = bl.end(n) - t0, K = d.K, V = d.V;
  extern __shared__ __align__(1024) unsigned char sm[];
  const LFwdOut5 L(K, V);
  unsigned char* Qh = sm + L.Qh;
  unsigned char* Kq = sm + L.Kq;
  unsigned char* Sh = sm + L.Sh;
  unsigned char* Wt = sm + L.Wt;
  unsigned char* Ph = sm + L.Ph;
  unsigned char* Pl = sm + L.Pl;
  float* G = reinterpret_cast<float*>(sm + L.G);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + L.bar);
  uint32_t* slot = reinterpret_cast<uint32_t*>(sm + L.slot);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int half = warp >> 2, trow = 16 * (warp & 3) + (lane & 15);
  const bool rowlane = lane < 16;
  constexpr uint32_t ncols = 128;
  const int64_t r0 = row(u, T, t0), KV = (int64_t)K * V;
  const RowTile qt{d.q + r0 * K, K, true, Qh, nullptr};
  const RowTile kt{d.k + r0 * K, K, true, Kq, nullptr};
  const float* sn = d.Sb + ((int64_t)u * (bl.nb + 1) + n) * KV;
  const bf16* wn = reinterpret_cast<const bf16*>(d.W) + r0 * V;

  if (warp == 0) tc5::tmem_alloc(slot, ncols);
  if (tid == 0) {
    tc5::mbar_init(bar, 1);
    tc5::mbar_fence_init();
    // every region this block reads is contiguous: start them all towards L2 at once, so
    // that the tile loads below (one tile in registers at a time) wait on L2, not DRAM
    tc5::prefetch_l2(d.q + r0 * K, (uint32_t)(c * K * 4));
    tc5::prefetch_l2(sn, (uint32_t)(KV * 4));
    tc5::prefetch_l2(wn, (uint32_t)(c * V * 2));
  }
  {
    RowRegs r;
    tile_fetch(kt, c, r);
    chunk_gates(d, u, t0, c, G, nullptr);
    tile_store(kt, r);
    tile_fetch(qt, c, r);
    tile_store(qt, r);
  }
  tc5::fence_async_smem();
  tc5::fence_before_sync();
  __syncthreads();
  tc5::fence_after_sync();
  const uint32_t tb = *slot;
  uint32_t ph = 0;
  bool ok = true;
  if (tid == 0) {  // P = Q K^T
    const uint32_t id = tc5::idesc_bf16(C, C, false, false);
    const uint32_t qa = tc5::saddr(Qh), ka = tc5::saddr(Kq);
    for (int ks = 0; ks < K / 16; ++ks)
      tc5::mma(tb, tc5::sdesc(qa, K, ks), tc5::sdesc(ka, K, ks), id, ks > 0);
    tc5::commit(bar);
  }
  {  // S_n (K x V fp32 -> MN-major, reduction over k) and W (bf16 -> MN-major) under MMA 1
    const RowTile st{sn, V, false, Sh, nullptr, K};
    constexpr int per_pass = kRowItems * kSweepThreads;
    const int passes = (K * (V / 8) + per_pass - 1) / per_pass;
    for (int pass = 0; pass < passes; ++pass) {
      RowRegs r;
      tile_fetch(st, K, r, pass);
      tile_store(st, r, pass);
    }
    bf16_rows_to_mn(wn, c, V, Wt);
  }
  {
    RowRegs qv;
    tile_fetch(qt, c, qv);  // Q again (from L2) for Qg
    ok = tc5::mbar_wait(bar, ph);
    ph ^= 1;
    tc5::fence_after_sync();
    // MMA 1 has read K: Qg = diag(e^G) Q takes its tile
    const RowTile gq{d.q + r0 * K, K, true, Kq, nullptr, C, G};
    tile_store(gq, qv);
  }
  for (int ci = half; ci < C / 16; ci += 2) {  // P[t][s] = e^{G_t - G_s} (q_t . k_s), s <= t
    float acc[16];
    tc5::tmem_ld16(tc5::tmem_at(tb, 16 * ci), acc);
    tc5::tmem_wait_ld();
    if (rowlane) {
      const float gt = G[trow];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float x[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int s = 16 * ci + 8 * h + e;
          x[e] = s <= trow && trow < c ? __expf(gt - G[s]) * acc[8 * h + e] : 0.f;
        }
        uint4 hv, lv;
        split8(x, hv, lv);
        const uint32_t o = tc5::kmajor_off(trow, 16 * ci + 8 * h, C);
        *reinterpret_cast<uint4*>(Ph + o) = hv;
        *reinterpret_cast<uint4*>(Pl + o) = lv;
      }
    }
  }
  tc5::fence_async_smem();
  tc5::fence_before_sync();
  __syncthreads();
  tc5::fence_after_sync();
  if (tid == 0 && ok) {  // O = Qg S + Ph W + Pl W
    const uint32_t id = tc5::idesc_bf16(C, V, false, true);
    const uint32_t qg = tc5::saddr(Kq), sa = tc5::saddr(Sh), wa = tc5::saddr(Wt),
                   pha = tc5::saddr(Ph), pla = tc5::saddr(Pl);
    for (int ks = 0; ks < K / 16; ++ks)
      tc5::mma(tb, tc5::sdesc(qg, K, ks), tc5::sdesc(sa, K, ks), id, ks > 0);
    for (int ks = 0; ks < C / 16; ++ks) {
      tc5::mma(tb, tc5::sdesc(pha, C, ks), tc5::sdesc(wa, C, ks), id, true);
      tc5::mma(tb, tc5::sdesc(pla, C, ks), tc5::sdesc(wa, C, ks), id, true);
    }
    tc5::commit(bar);
  }
  ok = ok && tc5::mbar_wait(bar, ph);
  tc5::fence_after_sync();
  // O rows out through the 16-lane TMEM shape: lane l of quarter q holds rows 16 q + l / 4 and
  // + 8, columns 2 (l % 4) + {0, 1} and + 8 of a 16-column chunk; two chunks per wait
  const int er = 16 * (warp & 3) + (lane >> 2), ec = 2 * (lane & 3), nv = V / 16;
  auto chunk_out = [&](int ci, const float (&v)[8]) {
    if (!ok) return;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int t = er + 8 * h;
      if (t < c) {
        float* p = d.O + (r0 + t) * V + 16 * ci + ec;
        *reinterpret_cast<float2*>(p) = make_float2(v[2 * h], v[2 * h + 1]);
        *reinterpret_cast<float2*>(p + 8) = make_float2(v[4 + 2 * h], v[5 + 2 * h]);
      }
    }
  };
  for (int ci = half; ci < nv; ci += 4) {
    const bool two = ci + 2 < nv;  // warp-uniform
    float a0[8], a1[8];
    tc5::tmem_ld16x16(tc5::tmem_at(tb, 16 * ci), a0);
    if (two) tc5::tmem_ld16x16(tc5::tmem_at(tb, 16 * (ci + 2)), a1);
    tc5::tmem_wait_ld();
    chunk_out(ci, a0);
    if (two) chunk_out(ci + 2, a1);
  }
  tc5::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc5::tmem_free(tb, ncols);
  if (!ok && tid == 0) fail_status();
}

}  // namespace

size_t tc5_fwd_state_smem(int K, int V) { return LFwdSweep(K, V).total; }

int tc5_device_status(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_status, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    const int z = 0;
    if (cudaMemcpyToSymbol(g_device_status, &z, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}

bool tc5_sweeps_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("GPA_B200_SWEEPS");
    return !(e && std::strcmp(e, "mma") == 0);
  }();
  return on;
}

cudaError_t tc5_fwd_state_launch(const ScanBatch& b, int U, const Blocks& bl, cudaStream_t st) {
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
    const size_t smem = tc5_fwd_state_smem(b.s[i].K, b.s[i].V);
    if (smem > 227 * 1024) return cudaErrorInvalidConfiguration;
    const auto kern = b.s[i].K <= 64 ? tc5_fwd_state<64> : tc5_fwd_state<128>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    Launch scope("tc5_fwd_state", st);
    kern<<<dim3(U, sub.n), kSweepThreads, smem, st>>>(sub, U, bl);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t tc5_bwd_state_launch(const ScanBatch& b, int U, const Blocks& bl, cudaStream_t st) {
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
    const size_t smem = LBwdSweep(b.s[i].K, b.s[i].V).total;
    if (smem > 227 * 1024 || b.s[i].K > kMaxScanWidth || b.s[i].V > kMaxScanWidth)
      return cudaErrorInvalidConfiguration;
    const auto kern = b.s[i].K <= 64 ? tc5_bwd_state<64> : tc5_bwd_state<128>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    Launch scope("tc5_bwd_state", st);
    kern<<<dim3(U, sub.n), kBwdThreads, smem, st>>>(sub, U, bl);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

bool tc5_wy_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("GPA_B200_WY");
    return !(e && std::strcmp(e, "mma") == 0);
  }();
  return on;
}

// Opt-in (GPA_B200_OUT=tc5): its per-block chain of tile loads (one tile in registers at a
// time under the 80-register cap of three CTAs per SM, and the fp32 state snapshot converted
// every block) measured slower than the 512-thread mma.sync kernel.
bool tc5_out_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("GPA_B200_OUT");
    return e && std::strcmp(e, "tc5") == 0;
  }();
  return on;
}

cudaError_t tc5_fwd_out_launch(const ScanBatch& b, int U, const Blocks& bl, cudaStream_t st) {
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
    const size_t smem = LFwdOut5(b.s[i].K, b.s[i].V).total;
    if (smem > 227 * 1024 || b.s[i].K > kMaxScanWidth || b.s[i].V > kMaxScanWidth)
      return cudaErrorInvalidConfiguration;
    cudaError_t e = cudaFuncSetAttribute(tc5_fwd_out, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    Launch scope("tc5_fwd_out", st);
    tc5_fwd_out<<<dim3(U * bl.nb, sub.n), kSweepThreads, smem, st>>>(sub, U, bl);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t tc5_fwd_chunk_launch(const ScanBatch& b, int U, const Blocks& bl, cudaStream_t st) {
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
    const size_t smem = LFwdChunk5(b.s[i].K, b.s[i].V).total;
    if (smem > 227 * 1024 || b.s[i].K > kMaxScanWidth || b.s[i].V > kMaxScanWidth)
      return cudaErrorInvalidConfiguration;
    cudaError_t e = cudaFuncSetAttribute(tc5_fwd_chunk, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    Launch scope("tc5_fwd_chunk", st);
    tc5_fwd_chunk<<<dim3(U * bl.nb, sub.n), kSweepThreads, smem, st>>>(sub, U, bl);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace gpa
