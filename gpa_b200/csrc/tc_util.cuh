// Tile utilities shared by the tensor-core kernels (gdn_tc.cu, level_tc.cu).
#pragma once
#include "mma.cuh"

namespace gpa {
namespace tc {

constexpr int LDT = kMaxChunk + 8;  // bf16 row stride of 64-wide tiles

__host__ __device__ __forceinline__ int ld16(int x) { return x + 8; }  // padded bf16 row stride

// Shared-memory carve-up identical on host (sizing) and device (pointers).
struct Carve {
  size_t off = 0;
  __host__ __device__ size_t take(size_t bytes) {
    off = (off + 15) & ~size_t(15);
    const size_t r = off;
    off += bytes;
    return r;
  }
};

// fp32 rows [rows x cols] (row stride src_ld) -> bf16 tile [rows_pad x ld]; zero padding.
// cols and src_ld are multiples of 4 and src is 16-byte aligned: float4 loads, 4 in flight
// per thread.  With `lo`, the tile is stored as a hi/lo pair.
constexpr int kLoadIlp = 4;

// four values -> one 8-byte store per tile (o a multiple of 4: tiles are 8-byte aligned)
GPA_DEV void put4(bf16* hi, bf16* lo, int o, float4 v) {
  union Pack {
    __nv_bfloat162 h[2];
    uint2 u;
  };
  Pack ph, pl;
  ph.h[0] = __floats2bfloat162_rn(v.x, v.y);
  ph.h[1] = __floats2bfloat162_rn(v.z, v.w);
  *reinterpret_cast<uint2*>(hi + o) = ph.u;
  if (lo) {
    const float2 f01 = __bfloat1622float2(ph.h[0]), f23 = __bfloat1622float2(ph.h[1]);
    pl.h[0] = __floats2bfloat162_rn(v.x - f01.x, v.y - f01.y);
    pl.h[1] = __floats2bfloat162_rn(v.z - f23.x, v.w - f23.y);
    *reinterpret_cast<uint2*>(lo + o) = pl.u;
  }
}

GPA_DEV void tile_load(bf16* hi, bf16* lo, int ld, const float* src, int src_ld, int rows,
                       int cols, int rows_pad, float scale) {
  const int c4 = cols >> 2, n4 = rows_pad * c4;
  for (int base = threadIdx.x; base < n4; base += blockDim.x * kLoadIlp) {
    float4 v[kLoadIlp];
#pragma unroll
    for (int j = 0; j < kLoadIlp; ++j) {
      const int i = base + j * blockDim.x;
      const int r = i / c4, cc = (i - r * c4) << 2;
      v[j] = (i < n4 && r < rows) ? *reinterpret_cast<const float4*>(src + (int64_t)r * src_ld + cc)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int j = 0; j < kLoadIlp; ++j) {
      const int i = base + j * blockDim.x;
      if (i >= n4) break;
      const int r = i / c4, cc = (i - r * c4) << 2;
      float4 x = v[j];
      x.x *= scale;
      x.y *= scale;
      x.z *= scale;
      x.w *= scale;
      put4(hi, lo, r * ld + cc, x);
    }
  }
}

GPA_DEV void tile_to_bf16(bf16* dst, int ld, const float* src, int src_ld, int rows, int cols,
                          int rows_pad, float scale = 1.f) {
  tile_load(dst, nullptr, ld, src, src_ld, rows, cols, rows_pad, scale);
}

GPA_DEV void tile_split(bf16* hi, bf16* lo, int ld, const float* src, int src_ld, int rows,
                        int cols, int rows_pad, float scale = 1.f) {
  tile_load(hi, lo, ld, src, src_ld, rows, cols, rows_pad, scale);
}

// One tile of a batched load: fp32 rows [rows x cols] (row stride src_ld) -> bf16 (hi, and lo
// when given) [rows_pad x ld], zero padded; each value times `scale` and, when given, the
// shared-memory row factor rowmul[r].
struct TileJob {
  bf16* hi;
  bf16* lo;
  int ld;
  const float* src;
  int src_ld, rows, cols, rows_pad;
  float scale;
  const float* rowmul;
};

GPA_DEV TileJob job(bf16* hi, bf16* lo, int ld, const float* src, int src_ld, int rows, int cols,
                    int rows_pad, float scale = 1.f, const float* rowmul = nullptr) {
  return TileJob{hi, lo, ld, src, src_ld, rows, cols, rows_pad, scale, rowmul};
}

// Load the tiles two at a time: each thread keeps kLoadIlp float4 of each of the two tiles in
// flight before converting any of them.  With `dot` (A and B of the same geometry), the
// thread's part of sum(A o B) over the fp32 values is added to *dot on the way.
GPA_DEV void tile_pair(const TileJob& A, const TileJob* B, float* dot = nullptr) {
  const int ca = A.cols >> 2, na = A.rows_pad * ca;
  const int cb = B ? B->cols >> 2 : 1, nb = B ? B->rows_pad * cb : 0;
  const int n = na > nb ? na : nb;
  for (int base = threadIdx.x; base < n; base += blockDim.x * kLoadIlp) {
    float4 va[kLoadIlp], vb[kLoadIlp];
#pragma unroll
    for (int q = 0; q < kLoadIlp; ++q) {
      const int i = base + q * blockDim.x;
      const int ra = i / ca, xa = (i - ra * ca) << 2;
      va[q] = (i < na && ra < A.rows)
                  ? *reinterpret_cast<const float4*>(A.src + (int64_t)ra * A.src_ld + xa)
                  : make_float4(0.f, 0.f, 0.f, 0.f);
      if (B) {
        const int rb = i / cb, xb = (i - rb * cb) << 2;
        vb[q] = (i < nb && rb < B->rows)
                    ? *reinterpret_cast<const float4*>(B->src + (int64_t)rb * B->src_ld + xb)
                    : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    if (dot) {
#pragma unroll
      for (int q = 0; q < kLoadIlp; ++q)
        *dot += va[q].x * vb[q].x + va[q].y * vb[q].y + va[q].z * vb[q].z + va[q].w * vb[q].w;
    }
#pragma unroll
    for (int q = 0; q < kLoadIlp; ++q) {
      const int i = base + q * blockDim.x;
      if (i < na) {
        const int r = i / ca, cc = (i - r * ca) << 2;
        const float f = A.rowmul ? A.scale * A.rowmul[r] : A.scale;
        float4 x = va[q];
        x.x *= f;
        x.y *= f;
        x.z *= f;
        x.w *= f;
        put4(A.hi, A.lo, r * A.ld + cc, x);
      }
      if (B && i < nb) {
        const int r = i / cb, cc = (i - r * cb) << 2;
        const float f = B->rowmul ? B->scale * B->rowmul[r] : B->scale;
        float4 x = vb[q];
        x.x *= f;
        x.y *= f;
        x.z *= f;
        x.w *= f;
        put4(B->hi, B->lo, r * B->ld + cc, x);
      }
    }
  }
}

// Paired loads help kernels with one CTA per SM; with two CTAs per SM (little L1 left beside
// their shared memory) one tile at a time measured faster.
template <bool kPaired = true, int N>
GPA_DEV void load_tiles(const TileJob (&jobs)[N]) {
  if (kPaired) {
#pragma unroll
    for (int j = 0; j < N; j += 2) tile_pair(jobs[j], j + 1 < N ? &jobs[j + 1] : nullptr);
  } else {
#pragma unroll
    for (int j = 0; j < N; ++j) tile_pair(jobs[j], nullptr);
  }
}

// bf16 rows [rows x cols] in global memory (row stride src_ld, cols % 8 == 0, 16-byte
// aligned rows) -> bf16 tile [rows_pad x ld]; rows >= `rows` zero.  16-byte copies, two in
// flight per thread.
GPA_DEV void copy_bf16_tile(bf16* dst, int ld, const bf16* src, int src_ld, int rows, int cols,
                            int rows_pad) {
  const int c8 = cols >> 3, n = rows_pad * c8;
  for (int base = threadIdx.x; base < n; base += 2 * blockDim.x) {
    uint4 v[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int i = base + j * blockDim.x, r = i / c8, cc = (i - r * c8) << 3;
      v[j] = (i < n && r < rows) ? *reinterpret_cast<const uint4*>(src + (int64_t)r * src_ld + cc)
                                 : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int i = base + j * blockDim.x, r = i / c8, cc = (i - r * c8) << 3;
      if (i < n) *reinterpret_cast<uint4*>(dst + r * ld + cc) = v[j];
    }
  }
}

template <int MI, int NI, class Body>
GPA_DEV void tiles_n(int M, int N, Body body) {
  // NI chosen at run time: 32-wide tiles when N allows and they still give every warp a
  // tile, else 16-wide
  if (N % 32 == 0 && (M / (16 * MI)) * (N / 32) >= (int)(blockDim.x >> 5))
    for_tiles<MI, 2>(M, N, [&](int m0, int n0) { body.template operator()<2>(m0, n0); });
  else
    for_tiles<MI, 1>(M, N, [&](int m0, int n0) { body.template operator()<1>(m0, n0); });
}

}  // namespace tc
}  // namespace gpa
