// Self-test of the tcgen05 building blocks in tc5.cuh: one CTA stages a bf16 A (M x Kd) and
// B (Kd x N) from global memory into the K-major or MN-major shared-memory layouts (A through a
// bulk TMA copy of a pre-tiled image when asked), runs the Kd / 16 MMAs into a TMEM
// accumulator and writes D = A B (fp32, M x N) back through tcgen05.ld (the 32-lane shape, or
// for M = 64 the 16-lane shape when asked).  The GPU tests compare
// D with a CPU product for every layout combination the scan kernels use.
#include "../../include/gpa_b200.h"
#include "tc5.cuh"

#include <cuda_bf16.h>

namespace gpa {
namespace {

using bf16 = __nv_bfloat16;

constexpr int kProbeThreads = 128;
constexpr int kProbeMaxK = 128, kProbeMaxN = 256;
// A tile (128 rows) and B tile (256 rows) at the maximum reduction width, an A staging image,
// then the barriers: every descriptor-reachable byte lies inside the allocation
constexpr size_t kProbeA = 128 * kProbeMaxK * 2, kProbeB = kProbeMaxN * kProbeMaxK * 2;
constexpr size_t kProbeSmem = 2 * kProbeA + kProbeB + 64;

__global__ void __launch_bounds__(kProbeThreads) k_umma_probe(int M, int mma_m, int N, int Kd,
                                                               int a_mn, int b_mn, int flags,
                                                               const bf16* A, const bf16* B,
                                                               const bf16* A_tiled, float* D,
                                                               int* status) {
  extern __shared__ __align__(1024) unsigned char sm[];
  unsigned char* As = sm;
  unsigned char* Bs = sm + kProbeA;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + 2 * kProbeA + kProbeB);
  uint32_t* slot = reinterpret_cast<uint32_t*>(bar + 2);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t ncols = N <= 32 ? 32 : N <= 64 ? 64 : N <= 128 ? 128 : 256;
  const bool a_bulk = flags & GPA_B200_UMMA_BULK_A, ld16 = flags & GPA_B200_UMMA_LD16;
  if (!a_bulk) {
    for (int i = tid; i < 128 * Kd; i += blockDim.x) {
      const int r = i / Kd, k = i - r * Kd;
      const bf16 v = r < M ? A[(size_t)r * Kd + k] : __float2bfloat16(0.f);
      const uint32_t o = a_mn ? tc5::mnmajor_off(r, k, Kd) : tc5::kmajor_off(r, k, Kd);
      *reinterpret_cast<bf16*>(As + o) = v;
    }
  }
  for (int i = tid; i < N * Kd; i += blockDim.x) {
    const int n = i / Kd, k = i - n * Kd;
    // b_mn == 2: B stored as the K-major tile of B itself (rows k, cols n), read through the
    // MN-major view of that tile
    const uint32_t o = b_mn == 2 ? tc5::kmajor_off(k, n, N)
                       : b_mn ? tc5::mnmajor_off(n, k, Kd) : tc5::kmajor_off(n, k, Kd);
    *reinterpret_cast<bf16*>(Bs + o) = B[(size_t)k * N + n];
  }
  if (warp == 0) tc5::tmem_alloc(slot, ncols);
  if (tid == 0) {
    tc5::mbar_init(&bar[0], 1);
    tc5::mbar_init(&bar[1], 1);
    tc5::mbar_fence_init();
  }
  tc5::fence_async_smem();
  tc5::fence_before_sync();
  __syncthreads();
  tc5::fence_after_sync();
  bool ok = true;
  if (a_bulk) {  // A arrives as one bulk copy of its pre-tiled image (128 rows x Kd)
    if (tid == 0) {
      tc5::mbar_expect_tx(&bar[1], (uint32_t)(128 * Kd * 2));
      tc5::bulk_g2s(As, A_tiled, (uint32_t)(128 * Kd * 2), &bar[1]);
    }
    ok = tc5::mbar_wait(&bar[1], 0);
  }
  const uint32_t taddr = *slot;
  if (tid == 0 && ok) {
    const uint32_t id = tc5::idesc_bf16(mma_m, N, a_mn != 0, b_mn != 0);
    for (int ks = 0; ks < Kd / 16; ++ks)
      tc5::mma(taddr, tc5::sdesc(tc5::saddr(As), Kd, ks),
               b_mn == 2 ? tc5::sdesc_mn_view(tc5::saddr(Bs), N, ks)
                         : tc5::sdesc(tc5::saddr(Bs), Kd, ks),
               id, ks > 0);
    tc5::commit(&bar[0]);
  }
  ok = ok && tc5::mbar_wait(&bar[0], 0);
  tc5::fence_after_sync();
  if (ld16) {  // M = 64 through the 16-lane shape: every thread holds 8 values per 16 columns
    const int r = 16 * warp + (lane >> 2), cc = 2 * (lane & 3);
    for (int c = 0; c < N; c += 16) {
      float v[8];
      tc5::tmem_ld16x16(tc5::tmem_at(taddr, c), v);
      tc5::tmem_wait_ld();
      for (int i = 0; i < 8; ++i) {
        const int row = r + 8 * ((i >> 1) & 1), col = c + cc + 8 * (i >> 2) + (i & 1);
        if (ok && row < M) D[(size_t)row * N + col] = v[i];
      }
    }
  } else {
    // M = 128: row = TMEM lane; M = 64: rows 16 q .. 16 q + 15 in lanes 0-15 of quarter q
    const int row = mma_m == 128 ? 32 * warp + lane : (lane < 16 ? 16 * warp + lane : -1);
    for (int c = 0; c < N; c += 16) {
      float v[16];
      tc5::tmem_ld16(tc5::tmem_at(taddr, c), v);
      tc5::tmem_wait_ld();
      if (ok && row >= 0 && row < M)
        for (int i = 0; i < 16; ++i) D[(size_t)row * N + c + i] = v[i];
    }
  }
  tc5::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc5::tmem_free(taddr, ncols);
  if (!ok && tid == 0) *status = GPA_B200_DEVICE_TIMEOUT;
}

}  // namespace

int umma_probe(int M, int mma_m, int N, int Kd, int a_mn, int b_mn, int flags, const void* A,
               const void* B, const void* A_tiled, float* D, int* status, cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(k_umma_probe, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kProbeSmem);
  if (e != cudaSuccess) return GPA_B200_LAUNCH_FAILURE;
  k_umma_probe<<<1, kProbeThreads, kProbeSmem, st>>>(
      M, mma_m, N, Kd, a_mn, b_mn, flags, static_cast<const bf16*>(A),
      static_cast<const bf16*>(B), static_cast<const bf16*>(A_tiled), D, status);
  return cudaGetLastError() == cudaSuccess ? GPA_B200_OK : GPA_B200_LAUNCH_FAILURE;
}

bool umma_probe_shape_ok(int M, int mma_m, int N, int Kd, int flags) {
  const bool ld16 = flags & GPA_B200_UMMA_LD16;
  return (mma_m == 64 || mma_m == 128) && M >= 1 && M <= mma_m && Kd >= 16 &&
         Kd <= kProbeMaxK && Kd % 16 == 0 && N >= 16 && N <= kProbeMaxN &&
         N % (mma_m == 128 || ld16 ? 16 : 8) == 0 && (!ld16 || mma_m == 64) &&
         (flags & ~(GPA_B200_UMMA_BULK_A | GPA_B200_UMMA_LD16)) == 0;
}

}  // namespace gpa
