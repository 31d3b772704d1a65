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

GPA_DEV void put4(bf16* hi, bf16* lo, int o, float4 v) {
  __nv_bfloat162 h01 = __floats2bfloat162_rn(v.x, v.y), h23 = __floats2bfloat162_rn(v.z, v.w);
  *reinterpret_cast<__nv_bfloat162*>(hi + o) = h01;
  *reinterpret_cast<__nv_bfloat162*>(hi + o + 2) = h23;
  if (lo) {
    const float2 f01 = __bfloat1622float2(h01), f23 = __bfloat1622float2(h23);
    *reinterpret_cast<__nv_bfloat162*>(lo + o) = __floats2bfloat162_rn(v.x - f01.x, v.y - f01.y);
    *reinterpret_cast<__nv_bfloat162*>(lo + o + 2) = __floats2bfloat162_rn(v.z - f23.x, v.w - f23.y);
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

// Load the tiles one after another (kLoadIlp float4 in flight per thread).  Loading all
// tiles of a phase in one round (16 float4 per thread) measured slower on B200.
template <int N>
GPA_DEV void load_tiles(const TileJob (&jobs)[N]) {
#pragma unroll
  for (int j = 0; j < N; ++j) {
    const TileJob& J = jobs[j];
    const int c4 = J.cols >> 2, n4 = J.rows_pad * c4;
    for (int base = threadIdx.x; base < n4; base += blockDim.x * kLoadIlp) {
      float4 v[kLoadIlp];
#pragma unroll
      for (int q = 0; q < kLoadIlp; ++q) {
        const int i = base + q * blockDim.x;
        const int r = i / c4, cc = (i - r * c4) << 2;
        v[q] = (i < n4 && r < J.rows)
                   ? *reinterpret_cast<const float4*>(J.src + (int64_t)r * J.src_ld + cc)
                   : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int q = 0; q < kLoadIlp; ++q) {
        const int i = base + q * blockDim.x;
        if (i >= n4) break;
        const int r = i / c4, cc = (i - r * c4) << 2;
        const float f = J.rowmul ? J.scale * J.rowmul[r] : J.scale;
        float4 x = v[q];
        x.x *= f;
        x.y *= f;
        x.z *= f;
        x.w *= f;
        put4(J.hi, J.lo, r * J.ld + cc, x);
      }
    }
  }
}

// dst[i] = src[i] for n floats (n multiple of 4, 16-byte aligned), float4 copies
GPA_DEV void copy_f4(float* dst, const float* src, int n) {
  for (int i = threadIdx.x * 4; i < n; i += blockDim.x * 4)
    *reinterpret_cast<float4*>(dst + i) = *reinterpret_cast<const float4*>(src + i);
}

template <int MI, int NI, class Body>
GPA_DEV void tiles_n(int M, int N, Body body) {
  // NI chosen at run time: 32-wide tiles when N allows, else 16-wide
  if (N % 32 == 0) for_tiles<MI, 2>(M, N, [&](int m0, int n0) { body.template operator()<2>(m0, n0); });
  else for_tiles<MI, 1>(M, N, [&](int m0, int n0) { body.template operator()<1>(m0, n0); });
}

}  // namespace tc
}  // namespace gpa
