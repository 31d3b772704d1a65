// Warp-level bf16 tensor-core tiles (mma.sync m16n8k16, fp32 accumulate) over
// shared-memory operands loaded with ldmatrix.
//
// Operand conventions (all bf16 in shared memory, row strides `ld` in elements,
// ld * 2 bytes a multiple of 16):
//   A (M x K):  TA == false  -> stored row-major A[m][k]
//               TA == true   -> stored as S[k][m] (A = S^T)
//   B (K x N):  TB == false  -> stored row-major B[k][n]
//               TB == true   -> stored as S[n][k] (B = S^T)
// A warp tile is (16*MI) x (16*NI); acc[mi][j][r] holds element
//   row = m0 + 16*mi + g + 8*(r >> 1),  col = n0 + 8*j + 2*q + (r & 1)
// with g = lane / 4, q = lane % 4 (the PTX m16n8 accumulator layout).
#pragma once
#include "common.cuh"

namespace gpa {
namespace tc {

using bf16 = __nv_bfloat16;

GPA_DEV uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

GPA_DEV void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_addr(p)));
}

GPA_DEV void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_addr(p)));
}

GPA_DEV void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <bool TA>
GPA_DEV void load_a(uint32_t (&a)[4], const bf16* A, int lda, int m0, int k0) {
  const int lane = threadIdx.x & 31;
  if (!TA) {
    ldsm_x4(a, A + (m0 + (lane & 15)) * lda + k0 + ((lane >> 4) << 3));
  } else {
    ldsm_x4_t(a, A + (k0 + (lane & 7) + ((lane >> 4) << 3)) * lda + m0 + (((lane >> 3) & 1) << 3));
  }
}

// two n8 fragments: b[0], b[1] for columns n0..n0+7, b[2], b[3] for n0+8..n0+15
template <bool TB>
GPA_DEV void load_b(uint32_t (&b)[4], const bf16* B, int ldb, int k0, int n0) {
  const int lane = threadIdx.x & 31;
  if (TB) {
    ldsm_x4(b, B + (n0 + (lane & 7) + ((lane >> 4) << 3)) * ldb + k0 + (((lane >> 3) & 1) << 3));
  } else {
    ldsm_x4_t(b, B + (k0 + (lane & 7) + (((lane >> 3) & 1) << 3)) * ldb + n0 + ((lane >> 4) << 3));
  }
}

template <int MI, int NI>
struct Acc {
  float v[MI][2 * NI][4];
  GPA_DEV void zero() {
#pragma unroll
    for (int i = 0; i < MI; ++i)
#pragma unroll
      for (int j = 0; j < 2 * NI; ++j)
#pragma unroll
        for (int r = 0; r < 4; ++r) v[i][j][r] = 0.f;
  }
  // Column pairs (col, col + 1) of the warp's elements, with a pair index p in
  // [0, kPairs) that is a compile-time constant after unrolling: f(p, row, col, v0, v1).
  // Epilogues that read global memory first gather every pair they need into a
  // float2[kPairs] (all loads in flight at once), then compute and store.
  static constexpr int kPairs = MI * 2 * NI * 2;
  template <class F>
  GPA_DEV void each2(int m0, int n0, F f) {
    const int lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
#pragma unroll
    for (int i = 0; i < MI; ++i)
#pragma unroll
      for (int j = 0; j < 2 * NI; ++j)
#pragma unroll
        for (int h = 0; h < 2; ++h)
          f((i * 2 * NI + j) * 2 + h, m0 + 16 * i + g + 8 * h, n0 + 8 * j + 2 * q, v[i][j][2 * h],
            v[i][j][2 * h + 1]);
  }
  // f(row, col, float& value) over the warp's elements
  template <class F>
  GPA_DEV void each(int m0, int n0, F f) {
    const int lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
#pragma unroll
    for (int i = 0; i < MI; ++i)
#pragma unroll
      for (int j = 0; j < 2 * NI; ++j)
#pragma unroll
        for (int r = 0; r < 4; ++r)
          f(m0 + 16 * i + g + 8 * (r >> 1), n0 + 8 * j + 2 * q + (r & 1), v[i][j][r]);
  }
};

// acc += A[m0:m0+16MI, kb:K] * B[kb:K, n0:n0+16NI] (kb a multiple of 16: a triangular
// operand skips its zero blocks)
template <int MI, int NI, bool TA, bool TB>
GPA_DEV void mma_acc(Acc<MI, NI>& acc, const bf16* A, int lda, const bf16* B, int ldb, int m0,
                     int n0, int K, int kb = 0) {
  for (int k0 = kb; k0 < K; k0 += 16) {
    uint32_t a[MI][4], b[NI][4];
#pragma unroll
    for (int i = 0; i < MI; ++i) load_a<TA>(a[i], A, lda, m0 + 16 * i, k0);
#pragma unroll
    for (int j = 0; j < NI; ++j) load_b<TB>(b[j], B, ldb, k0, n0 + 16 * j);
#pragma unroll
    for (int i = 0; i < MI; ++i)
#pragma unroll
      for (int j = 0; j < NI; ++j) {
        mma16816(acc.v[i][2 * j], a[i], b[j][0], b[j][1]);
        mma16816(acc.v[i][2 * j + 1], a[i], b[j][2], b[j][3]);
      }
  }
}

// Split-operand product: acc += Ah*Bh + Ah*Bl + Al*Bh, where x = xh + xl is an
// fp32 value carried as two bf16 (hi = bf16(x), lo = bf16(x - hi)); either lo
// may be null.  Products then carry ~16 significant bits instead of 8.  k runs over [kb, K).
template <int MI, int NI, bool TA, bool TB>
GPA_DEV void mma_acc3(Acc<MI, NI>& acc, const bf16* Ah, const bf16* Al, int lda, const bf16* Bh,
                      const bf16* Bl, int ldb, int m0, int n0, int K, int kb = 0) {
  for (int k0 = kb; k0 < K; k0 += 16) {
    uint32_t a[MI][4], b[NI][4], x[4];
#pragma unroll
    for (int i = 0; i < MI; ++i) load_a<TA>(a[i], Ah, lda, m0 + 16 * i, k0);
#pragma unroll
    for (int j = 0; j < NI; ++j) load_b<TB>(b[j], Bh, ldb, k0, n0 + 16 * j);
#pragma unroll
    for (int i = 0; i < MI; ++i)
#pragma unroll
      for (int j = 0; j < NI; ++j) {
        mma16816(acc.v[i][2 * j], a[i], b[j][0], b[j][1]);
        mma16816(acc.v[i][2 * j + 1], a[i], b[j][2], b[j][3]);
      }
    if (Bl) {
#pragma unroll
      for (int j = 0; j < NI; ++j) {
        load_b<TB>(x, Bl, ldb, k0, n0 + 16 * j);
#pragma unroll
        for (int i = 0; i < MI; ++i) {
          mma16816(acc.v[i][2 * j], a[i], x[0], x[1]);
          mma16816(acc.v[i][2 * j + 1], a[i], x[2], x[3]);
        }
      }
    }
    if (Al) {
#pragma unroll
      for (int i = 0; i < MI; ++i) {
        load_a<TA>(x, Al, lda, m0 + 16 * i, k0);
#pragma unroll
        for (int j = 0; j < NI; ++j) {
          mma16816(acc.v[i][2 * j], x, b[j][0], b[j][1]);
          mma16816(acc.v[i][2 * j + 1], x, b[j][2], b[j][3]);
        }
      }
    }
  }
}

GPA_DEV float2 ld2(const float* p) { return *reinterpret_cast<const float2*>(p); }
GPA_DEV void st2(float* p, float a, float b) { *reinterpret_cast<float2*>(p) = make_float2(a, b); }

// hi / lo bf16 pair of an fp32 value
GPA_DEV void split_bf16(float x, bf16* hi, bf16* lo) {
  const bf16 h = __float2bfloat16(x);
  *hi = h;
  *lo = __float2bfloat16(x - __bfloat162float(h));
}

// hi / lo bf16 pairs of two adjacent fp32 values (hi, lo 4-byte aligned)
GPA_DEV void split2(float a, float b, bf16* hi, bf16* lo) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  const float2 f = __bfloat1622float2(h);
  *reinterpret_cast<__nv_bfloat162*>(hi) = h;
  *reinterpret_cast<__nv_bfloat162*>(lo) = __floats2bfloat162_rn(a - f.x, b - f.y);
}

// Round-robin the (16MI x 16NI) tiles of an M x N output over the block's warps.
template <int MI, int NI, class Body>
GPA_DEV void for_tiles(int M, int N, Body body) {
  const int tm = M / (16 * MI), tn = N / (16 * NI);
  const int nw = blockDim.x >> 5;
  for (int t = threadIdx.x >> 5; t < tm * tn; t += nw) body((t / tn) * 16 * MI, (t % tn) * 16 * NI);
}

// sum of x over the 4 lanes that share a row (same g) of an accumulator
GPA_DEV float quad_sum(float x) {
  x += __shfl_xor_sync(0xffffffffu, x, 1);
  x += __shfl_xor_sync(0xffffffffu, x, 2);
  return x;
}

}  // namespace tc
}  // namespace gpa
