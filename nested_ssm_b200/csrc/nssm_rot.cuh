// Rotation kernel of B and C (rot_flat and the rotation inside the tiered step).
#pragma once

#include "nssm_device.cuh"

namespace nssm {

// Rotation of B and C by R (out[j][g][m] = sum_n R[g][m][n] x[j][g][n], fp32 accumulate,
// n in order).  Per group a small GEMM OUT[rows][m] = X[rows][n] R_g^T[n][m]: one CTA per
// (group g, tile of kRotTile rows of the stacked B;C row list, half of the outputs m)
// copies its 64 rows of R_g (32 KB, coalesced 128-bit loads) and the tile's rows (as fp32)
// into shared memory with rows padded to kRotLd floats, and every thread accumulates a
// 4-row x 4-output register tile, reading four n at a time.  Four CTAs fit an SM.
struct RotParams {
  const void* x0;
  const void* x1;
  int64_t xs0, xs1;
  void* o0;
  void* o1;
  int64_t os0, os1;
  const float* R;
  int T, G, dtype;      // rows [0, T) come from x0 / o0, rows [T, 2T) from x1 / o1
};

constexpr int kRotTile = 32;
constexpr int kRotThreads = 128;
constexpr int kRotHalf = 64;  // outputs m per CTA
constexpr int kRotLd = 132;   // padded row length: 16-byte aligned, rows 4 banks apart

__host__ __device__ constexpr int rot_smem_bytes(int N) { return (kRotHalf + kRotTile) * kRotLd * 4; }

// io values as fp32 / back, the io dtype fixed at compile time (bf16 or fp32)
template <bool IOBF>
__device__ __forceinline__ float rot_ld(const void* p, int64_t i) {
  if constexpr (IOBF) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  else return reinterpret_cast<const float*>(p)[i];
}
template <bool IOBF>
__device__ __forceinline__ void rot_st(void* p, int64_t i, float v) {
  if constexpr (IOBF) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else reinterpret_cast<float*>(p)[i] = v;
}

template <int N, bool IOBF>
__global__ void __launch_bounds__(kRotThreads, 4) rot_kernel(const RotParams p, int rows_total) {
  static_assert(N == 128, "tile mapping assumes dstate 128");
  extern __shared__ __align__(16) float rsm[];
  float* Rs = rsm;                       // [kRotHalf][kRotLd]: Rs[m - m0][n] = R[g][m][n]
  float* Xs = rsm + kRotHalf * kRotLd;   // [kRotTile][kRotLd]: Xs[r][n] = x[j0 + r][g][n]
  const int g = blockIdx.y;
  const int m0 = blockIdx.z * kRotHalf;
  const int tid = threadIdx.x;
  const int j0 = blockIdx.x * kRotTile;
  const int nr = min(kRotTile, rows_total - j0);

  // rows m0 .. m0+63 of R_g: a warp copies one 512-byte row per instruction
  {
    const float4* src = reinterpret_cast<const float4*>(p.R + ((int64_t)g * N + m0) * N);
    constexpr int kVec = kRotHalf * N / 4 / kRotThreads;   // float4 per thread (16)
    float4 v[kVec];
#pragma unroll
    for (int u = 0; u < kVec; ++u) v[u] = __ldg(src + tid + u * kRotThreads);
#pragma unroll
    for (int u = 0; u < kVec; ++u) {
      const int e = tid + u * kRotThreads;   // float4 index: row e / 32, column 4 * (e % 32)
      *reinterpret_cast<float4*>(Rs + (e / (N / 4)) * kRotLd + 4 * (e % (N / 4))) = v[u];
    }
  }
  // the tile's rows: a warp reads one row's 128 values (zeros past the end of the list)
  {
    const int warp = tid / 32, lane = tid % 32;
    constexpr int kRowsPerWarp = kRotTile / (kRotThreads / 32);
    float v[kRowsPerWarp][4];
#pragma unroll
    for (int u = 0; u < kRowsPerWarp; ++u) {
      const int r = warp * kRowsPerWarp + u;
      const int j = j0 + r;
      const bool second = j >= p.T;
      const void* x = second ? p.x1 : p.x0;
      const int64_t base = (int64_t)(second ? j - p.T : j) * (second ? p.xs1 : p.xs0) + (int64_t)g * N;
#pragma unroll
      for (int t = 0; t < 4; ++t)
        v[u][t] = r < nr ? rot_ld<IOBF>(x, base + lane + 32 * t) : 0.0f;   // strides may be odd
    }
#pragma unroll
    for (int u = 0; u < kRowsPerWarp; ++u)
#pragma unroll
      for (int t = 0; t < 4; ++t) Xs[(warp * kRowsPerWarp + u) * kRotLd + lane + 32 * t] = v[u][t];
  }
  __syncthreads();

  // thread tile: rows 4*rg .. 4*rg+3, outputs m0 + mg + 16*j (j = 0..3)
  const int rg = tid / 16, mg = tid % 16;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
#pragma unroll 4
  for (int n = 0; n < N; n += 4) {
    float4 xv[4], rv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) xv[i] = *reinterpret_cast<const float4*>(Xs + (4 * rg + i) * kRotLd + n);
#pragma unroll
    for (int j = 0; j < 4; ++j) rv[j] = *reinterpret_cast<const float4*>(Rs + (mg + 16 * j) * kRotLd + n);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float a = acc[i][j];
        a = fmaf(rv[j].x, xv[i].x, a);
        a = fmaf(rv[j].y, xv[i].y, a);
        a = fmaf(rv[j].z, xv[i].z, a);
        a = fmaf(rv[j].w, xv[i].w, a);
        acc[i][j] = a;
      }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = 4 * rg + i;
    if (r >= nr) break;
    const int j = j0 + r;
    const bool second = j >= p.T;
    const int row = second ? j - p.T : j;   // padded rows are rotated too (nobody reads them)
    void* o = second ? p.o1 : p.o0;
    const int64_t ob = (int64_t)row * (second ? p.os1 : p.os0) + (int64_t)g * N + m0;
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) rot_st<IOBF>(o, ob + mg + 16 * jj, acc[i][jj]);
  }
}

}  // namespace nssm
