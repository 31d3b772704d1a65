// Parameter-gradient reductions on the 5th-generation tensor cores:
//   out[h] (P x Q) += cscale * scale[h] * sum_{b,t} X^T Y      (X [U,T,P], Y [U,T,Q], fp32)
// over the rows of head h (units u = b H + h), as tc_head_outer in level_tc.cu.  A CTA owns a
// 128 x NQ tile of out and a run of `split` tokens; per 64-token step the threads convert the
// fp32 rows into bf16 hi / lo operand tiles (X^T as an MN-major A of 128 rows p, Y as an
// MN-major B of NQ rows q, the reduction over tokens), and one thread issues the three
// products hi hi + hi lo + lo hi into a TMEM accumulator (M = 128, N = NQ).  Two stages: step
// i's tiles are converted while step i-1's MMAs run, and step i+1's rows are loaded into
// registers meanwhile.  The epilogue adds the tile into out with atomics (split-K).
#include "../../include/gpa_b200.h"
#include "level.cuh"
#include "tc5.cuh"

#include <cuda_bf16.h>

#include <cstdlib>
#include <cstring>

namespace gpa {

__device__ int g_outer_status = 0;

namespace {

constexpr int kHoThreads = 256;
constexpr int kHoK = 64;    // tokens per step
constexpr int kHoP = 128;   // rows of the output tile (M of the MMA)
constexpr int kHoItems = kHoP * kHoK / 8 / kHoThreads;  // 8-wide items per thread and operand

GPA_DEV int64_t ho_row(int u, int T, int t) { return (int64_t)u * T + t; }

// 8 fp32 -> bf16 hi and lo parts (x = hi + lo to ~16 significant bits)
GPA_DEV void split8h(const float (&x)[8], uint4& hi, uint4& lo) {
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

template <int NQ>
struct LHo {
  // per stage: A hi / lo (128 rows p x 64 tokens), B hi / lo (NQ rows q x 64 tokens)
  static constexpr uint32_t kA = kHoP * kHoK * 2, kB = NQ * kHoK * 2;
  static constexpr uint32_t kStage = 2 * kA + 2 * kB;
  static constexpr uint32_t kBar = 2 * kStage, kSlot = kBar + 16, kTotal = kSlot + 16;
};

template <int NQ>
__global__ void __launch_bounds__(kHoThreads, 2) tc5_head_outer(
    int B, int T, int H, const float* X, int P, int xmode, const float* Y, int Q,
    const float* scale, int64_t scale_stride, float cscale, float* out, int split) {
  using Lo = LHo<NQ>;
  constexpr int kYItems = NQ * kHoK / 8 / kHoThreads;
  const int h = blockIdx.x;
  const int tq = (Q + NQ - 1) / NQ;
  const int p0 = (blockIdx.y / tq) * kHoP, q0 = (blockIdx.y % tq) * NQ;
  const int pw = min(kHoP, P - p0), qw = min(NQ, Q - q0);
  const int64_t total = (int64_t)B * T;
  const int64_t r0 = (int64_t)blockIdx.z * split;
  const int64_t r1 = min(total, r0 + split);
  const int nsteps = (int)((r1 - r0 + kHoK - 1) / kHoK);
  extern __shared__ __align__(1024) unsigned char sm[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + Lo::kBar);
  uint32_t* slot = reinterpret_cast<uint32_t*>(sm + Lo::kSlot);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (warp == 0) tc5::tmem_alloc(slot, 128);
  if (tid == 0) {
    tc5::mbar_init(&bar[0], 1);
    tc5::mbar_init(&bar[1], 1);
    tc5::mbar_fence_init();
  }
  // registers of one step: 8 consecutive p (or q) of one token per item
  float4 xr[kHoItems][2], yr[kYItems][2];
  auto token_row = [&](int64_t rr) {  // global row of step token rr of head h
    const int b = (int)(rr / T), t = (int)(rr - (int64_t)b * T);
    return ho_row(b * H + h, T, t);
  };
  auto fetch = [&](int step) {
    const int64_t base = r0 + (int64_t)step * kHoK;
#pragma unroll
    for (int j = 0; j < kHoItems; ++j) {
      const int i = tid + j * kHoThreads, t = i / (kHoP / 8), g = i - t * (kHoP / 8);
      xr[j][0] = xr[j][1] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (base + t < r1 && 8 * g < pw) {
        const float* p = X + token_row(base + t) * P + p0 + 8 * g;
        xr[j][0] = *reinterpret_cast<const float4*>(p);
        xr[j][1] = *reinterpret_cast<const float4*>(p + 4);
      }
    }
#pragma unroll
    for (int j = 0; j < kYItems; ++j) {
      const int i = tid + j * kHoThreads, t = i / (NQ / 8), g = i - t * (NQ / 8);
      yr[j][0] = yr[j][1] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (base + t < r1 && 8 * g < qw) {
        const float* p = Y + token_row(base + t) * Q + q0 + 8 * g;
        yr[j][0] = *reinterpret_cast<const float4*>(p);
        yr[j][1] = *reinterpret_cast<const float4*>(p + 4);
      }
    }
  };
  auto convert = [&](int s) {
    unsigned char* st = sm + s * Lo::kStage;
#pragma unroll
    for (int j = 0; j < kHoItems; ++j) {
      const int i = tid + j * kHoThreads, t = i / (kHoP / 8), g = i - t * (kHoP / 8);
      float x[8] = {xr[j][0].x, xr[j][0].y, xr[j][0].z, xr[j][0].w,
                    xr[j][1].x, xr[j][1].y, xr[j][1].z, xr[j][1].w};
      if (xmode == 1) {
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = gelu(x[e]);
      }
      uint4 hi, lo;
      split8h(x, hi, lo);
      const uint32_t o = tc5::mnmajor_off(8 * g, t, kHoK);  // rows p, reduction over tokens
      *reinterpret_cast<uint4*>(st + o) = hi;
      *reinterpret_cast<uint4*>(st + Lo::kA + o) = lo;
    }
#pragma unroll
    for (int j = 0; j < kYItems; ++j) {
      const int i = tid + j * kHoThreads, t = i / (NQ / 8), g = i - t * (NQ / 8);
      const float y[8] = {yr[j][0].x, yr[j][0].y, yr[j][0].z, yr[j][0].w,
                          yr[j][1].x, yr[j][1].y, yr[j][1].z, yr[j][1].w};
      uint4 hi, lo;
      split8h(y, hi, lo);
      const uint32_t o = tc5::mnmajor_off(8 * g, t, kHoK);
      *reinterpret_cast<uint4*>(st + 2 * Lo::kA + o) = hi;
      *reinterpret_cast<uint4*>(st + 2 * Lo::kA + Lo::kB + o) = lo;
    }
  };
  if (nsteps > 0) fetch(0);
  tc5::fence_before_sync();
  __syncthreads();
  tc5::fence_after_sync();
  const uint32_t tb = *slot;
  bool ok = true;
  const uint32_t id = tc5::idesc_bf16(kHoP, NQ, true, true);
  for (int i = 0; i < nsteps; ++i) {
    const int s = i & 1;
    // the MMAs of step i - 2 read this stage: wait for their commit
    if (i >= 2) ok = ok && tc5::mbar_wait(&bar[s], ((i - 2) >> 1) & 1);
    convert(s);
    tc5::fence_async_smem();
    tc5::fence_before_sync();
    __syncthreads();
    tc5::fence_after_sync();
    if (tid == 0 && ok) {
      const uint32_t a = tc5::saddr(sm + s * Lo::kStage);
      const uint32_t ah = a, al = a + Lo::kA, bh = a + 2 * Lo::kA, bl = bh + Lo::kB;
      for (int ks = 0; ks < kHoK / 16; ++ks) {
        tc5::mma(tb, tc5::sdesc(ah, kHoK, ks), tc5::sdesc(bh, kHoK, ks), id, i > 0 || ks > 0);
        tc5::mma(tb, tc5::sdesc(ah, kHoK, ks), tc5::sdesc(bl, kHoK, ks), id, true);
        tc5::mma(tb, tc5::sdesc(al, kHoK, ks), tc5::sdesc(bh, kHoK, ks), id, true);
      }
      tc5::commit(&bar[s]);
    }
    if (i + 1 < nsteps) fetch(i + 1);  // in flight while this step's MMAs run
  }
  // every MMA is done once the last step's commit has arrived
  if (nsteps > 0) ok = ok && tc5::mbar_wait(&bar[(nsteps - 1) & 1], ((nsteps - 1) >> 1) & 1);
  tc5::fence_after_sync();
  // epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 (rows p), its half of the columns
  const float sc = cscale * (scale ? scale[(int64_t)h * scale_stride] : 1.f);
  float* o = out + (int64_t)h * P * Q;
  const int p = 32 * (warp & 3) + lane, half = warp >> 2;
  for (int c = 16 * half; c < NQ; c += 32) {
    float v[16];
    tc5::tmem_ld16(tc5::tmem_at(tb, c), v);
    tc5::tmem_wait_ld();
    if (ok && nsteps > 0 && p < pw)
#pragma unroll
      for (int e = 0; e < 16; ++e)
        if (c + e < qw) atomicAdd(&o[(int64_t)(p0 + p) * Q + q0 + c + e], sc * v[e]);
  }
  tc5::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc5::tmem_free(tb, 128);
  if (!ok && tid == 0) atomicExch(&g_outer_status, GPA_B200_DEVICE_TIMEOUT);
}

constexpr int kHoSplit = 2048;  // tokens per CTA

template <int NQ>
cudaError_t ho_launch(int B, int T, int H, const float* X, int P, int xmode, const float* Y, int Q,
                      const float* scale, int64_t scale_stride, float cscale, float* out,
                      cudaStream_t st) {
  const int64_t total = (int64_t)B * T;
  const int tp = (P + kHoP - 1) / kHoP, tq = (Q + NQ - 1) / NQ;
  const dim3 grid(H, tp * tq, (unsigned)((total + kHoSplit - 1) / kHoSplit));
  if (!total || !H) return cudaSuccess;
  const size_t smem = LHo<NQ>::kTotal;
  cudaError_t e = cudaFuncSetAttribute(tc5_head_outer<NQ>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  Launch scope("tc5_head_outer", st);
  tc5_head_outer<NQ><<<grid, kHoThreads, smem, st>>>(B, T, H, X, P, xmode, Y, Q, scale,
                                                      scale_stride, cscale, out, kHoSplit);
  return cudaGetLastError();
}

}  // namespace

// Opt-in (GPA_B200_OUTER=tc5): the per-step hi / lo conversion of the fp32 rows by the SIMT
// threads costs more issue slots than the mma.sync kernel's MMA chains (11.1 ms per step at
// the benched shape against 8.3 for the mma.sync kernel).
bool tc5_outer_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("GPA_B200_OUTER");
    return e && std::strcmp(e, "tc5") == 0;
  }();
  return on;
}

cudaError_t tc5_head_outer_launch(int B, int T, int H, const float* X, int P, int xmode,
                                  const float* Y, int Q, const float* scale,
                                  int64_t scale_stride, float cscale, float* out,
                                  cudaStream_t st) {
  if (P % 8 || Q % 8 || P > 256 || Q > 256) return cudaErrorInvalidValue;
  // N = 64 tiles when Q fits one of them, else 128 (64-wide tiles throughout measured slower:
  // 11.9 ms per step, Y read twice)
  if (Q <= 64)
    return ho_launch<64>(B, T, H, X, P, xmode, Y, Q, scale, scale_stride, cscale, out, st);
  return ho_launch<128>(B, T, H, X, P, xmode, Y, Q, scale, scale_stride, cscale, out, st);
}

int outer_device_status(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_outer_status, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    const int z = 0;
    if (cudaMemcpyToSymbol(g_outer_status, &z, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}

}  // namespace gpa
