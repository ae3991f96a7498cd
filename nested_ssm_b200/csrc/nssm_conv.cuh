// Decode-token conv of the Mamba2 mixer ahead of the tiered state update: the causal
// conv1d update of [x | B | C] with the per-slot conv state, the activation, the split, and
// the per-group rotation of B and C, in one launch.
//
// Per batch row b (slot s = idx[b]) and conv channel d, with window width K and a state of
// L >= K - 1 columns:  w_d = last K of [state[s][d][0..L), xbc[b][d]],
//   out[d] = act(bias[d] + sum_k weight[d][k] w_d[k])   (fp32, k in order),
//   state[s][d] <- last L of [state[s][d], xbc[b][d]].
// x = out[0, I), B = out[I, I+G*N), C = out[I+G*N, I+2*G*N); B and C are then rotated per
// group like rot_kernel (fp32 dot products, n in order) and written in the io dtype.
#pragma once

#include "nssm_rot.cuh"

namespace nssm {

struct ConvParams {
  const void* xbc;
  int64_t xbc_sb;
  void* state;
  int64_t state_ss;     // elements between slots
  int L, K;
  const void* weight;
  int w_dtype;
  const void* bias;
  int act;              // 0: none, 1: silu
  const float* R;       // [G][N][N] or NULL
  const int32_t* idx;
  int pad, S;
  int T, I, G, dtype;
  void* x_out;
  int64_t x_sb;
  void* b_out;
  void* c_out;
  int64_t bc_sb;
  int32_t* status;
};

constexpr int kConvTile = 32;     // batch rows per CTA
constexpr int kConvThreads = 128;
constexpr int kConvMaxK = 8;      // conv width and state length supported
constexpr int kConvMaxL = 8;

__host__ __device__ constexpr int conv_smem_bytes(int N) { return (N + kConvTile) * kRotLd * 4; }

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + expf(-v)); }

// a value as stored in the io dtype (the conv output is rounded before the rotation reads
// it, as the split tensors of the reference are)
__device__ __forceinline__ float round_io(float v, int dtype) {
  return dtype == NSSM_BF16 ? __bfloat162float(__float2bfloat16_rn(v)) : v;
}

// conv of one channel of one row (window position l of [state, x] holds weight tap
// k = l - (L + 1 - K)); updates the slot's state when `upd`
__device__ __forceinline__ float conv_channel(const ConvParams& p, int64_t srow, int b, int d, bool upd) {
  const float xin = ld_io(p.xbc, (int64_t)b * p.xbc_sb + d, p.dtype);
  const int64_t so = srow + (int64_t)d * p.L;
  float win[kConvMaxL + 1];
#pragma unroll
  for (int l = 0; l <= kConvMaxL; ++l)
    win[l] = l < p.L ? ld_io(p.state, so + l, p.dtype) : (l == p.L ? xin : 0.0f);
  float acc = 0.0f;
  const int off = p.L + 1 - p.K;
#pragma unroll
  for (int l = 0; l <= kConvMaxL; ++l) {
    const int k = l - off;
    if (l <= p.L && k >= 0) acc = fmaf(ld_io(p.weight, (int64_t)d * p.K + k, p.w_dtype), win[l], acc);
  }
  if (p.bias) acc = acc + ld_io(p.bias, d, p.w_dtype);
  if (upd) {
#pragma unroll
    for (int l = 0; l < kConvMaxL; ++l)
      if (l < p.L) st_io(p.state, so + l, p.dtype, win[l + 1]);
  }
  return p.act ? silu_f(acc) : acc;
}

// B and C channels.  grid (ceil(T / kConvTile), G, 2): z = 0 for B, 1 for C.  A CTA
// converts the tile's channels of group g (state updated), then rotates them (all 128
// outputs: thread tile of 4 rows x 8 outputs) or copies them out.
template <int N>
__global__ void __launch_bounds__(kConvThreads, 2) conv_step_kernel(const ConvParams p) {
  static_assert(N == 128, "tile mapping assumes dstate 128");
  extern __shared__ __align__(16) float csm_[];
  float* Rs = csm_;                  // [N][kRotLd]: Rs[m][n] = R[g][m][n]
  float* Xs = csm_ + N * kRotLd;     // [kConvTile][kRotLd]
  const int g = blockIdx.y;
  const int which = blockIdx.z;
  const int tid = threadIdx.x;
  const int b0 = blockIdx.x * kConvTile;
  const int nr = min(kConvTile, p.T - b0);
  const bool rot = p.R != nullptr;

  // R_g (coalesced 128-bit loads), issued first
  if (rot) {
    const float4* src = reinterpret_cast<const float4*>(p.R + (int64_t)g * N * N);
    constexpr int kVec = N * N / 4 / kConvThreads;   // 32 float4 per thread
#pragma unroll
    for (int u0 = 0; u0 < kVec; u0 += 8) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = __ldg(src + tid + (u0 + u) * kConvThreads);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int e = tid + (u0 + u) * kConvThreads;
        *reinterpret_cast<float4*>(Rs + (e / (N / 4)) * kRotLd + 4 * (e % (N / 4))) = v[u];
      }
    }
  }

  // the tile's B (or C) channels of group g into shared memory (state updated)
  {
    const int cbase = p.I + which * p.G * N + g * N;
    for (int e = tid; e < kConvTile * N; e += kConvThreads) {
      const int r = e / N, n = e - r * N;
      float v = 0.0f;
      if (r < nr) {
        const int b = b0 + r;
        const int slot = p.idx ? p.idx[b] : b;
        if (slot != p.pad && slot >= 0 && slot < p.S)
          v = round_io(conv_channel(p, (int64_t)slot * p.state_ss, b, cbase + n, true), p.dtype);
      }
      Xs[r * kRotLd + n] = v;
    }
  }
  __syncthreads();
  void* out = which ? p.c_out : p.b_out;
  if (!rot) {
    for (int e = tid; e < nr * N; e += kConvThreads) {
      const int r = e / N, n = e - r * N;
      st_io(out, (int64_t)(b0 + r) * p.bc_sb + (int64_t)g * N + n, p.dtype, Xs[r * kRotLd + n]);
    }
    return;
  }
  // thread tile: rows 4*rg .. 4*rg+3, outputs mg + 16*j (j = 0..7); n in order
  const int rg = tid / 16, mg = tid % 16;
  float acc[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
#pragma unroll 2
  for (int n = 0; n < N; n += 4) {
    float4 xv[4], rv[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) xv[i] = *reinterpret_cast<const float4*>(Xs + (4 * rg + i) * kRotLd + n);
#pragma unroll
    for (int j = 0; j < 8; ++j) rv[j] = *reinterpret_cast<const float4*>(Rs + (mg + 16 * j) * kRotLd + n);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) {
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
    const int64_t ob = (int64_t)(b0 + r) * p.bc_sb + (int64_t)g * N;
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) st_io(out, ob + mg + 16 * jj, p.dtype, acc[i][jj]);
  }
}

// x channels: one thread per 4 consecutive channels of one row.  With compile-time K and L
// (VEC) the state, weights and x move in 8-byte vectors (16 for fp32 weights); otherwise
// per element.  grid (ceil(I / (4 * kConvXThreads)), T).
constexpr int kConvXThreads = 256;

template <int K, int L, bool IOBF, bool WBF>
__global__ void __launch_bounds__(kConvXThreads) conv_x_kernel(const ConvParams p) {
  const int b = blockIdx.y;
  const int d0 = (blockIdx.x * kConvXThreads + threadIdx.x) * 4;
  if (d0 >= p.I) return;
  const int slot = p.idx ? p.idx[b] : b;
  if (slot == p.pad) return;
  if (slot < 0 || slot >= p.S) {
    if (p.status && d0 == 0) atomicOr(p.status, STATUS_BAD_SLOT);
    return;
  }
  const int64_t srow = (int64_t)slot * p.state_ss;
  if constexpr (K > 0) {
    // every access below is aligned (checked on the host): state rows of L elements start
    // at d0 * L, x rows at b * xbc_sb + d0
    constexpr int EB = IOBF ? 2 : 4;
    float win[4][L + 1];
    {
      // 4 * L state elements, contiguous
      const unsigned char* sp = static_cast<const unsigned char*>(p.state) + (srow + (int64_t)d0 * L) * EB;
      float sv[4 * L];
      if constexpr (IOBF) {
#pragma unroll
        for (int q = 0; q < L; ++q) {   // 4 * L bf16 = L x 8 bytes
          const uint2 u = reinterpret_cast<const uint2*>(sp)[q];
          sv[4 * q + 0] = __uint_as_float(u.x << 16);
          sv[4 * q + 1] = __uint_as_float(u.x & 0xffff0000u);
          sv[4 * q + 2] = __uint_as_float(u.y << 16);
          sv[4 * q + 3] = __uint_as_float(u.y & 0xffff0000u);
        }
      } else {
#pragma unroll
        for (int q = 0; q < L; ++q) {
          const float4 u = reinterpret_cast<const float4*>(sp)[q];
          sv[4 * q + 0] = u.x; sv[4 * q + 1] = u.y; sv[4 * q + 2] = u.z; sv[4 * q + 3] = u.w;
        }
      }
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int l = 0; l < L; ++l) win[c][l] = sv[c * L + l];
    }
    {
      const int64_t xo = (int64_t)b * p.xbc_sb + d0;
      float xv[4];
      if constexpr (IOBF) {
        const uint2 u = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(p.xbc) + xo);
        xv[0] = __uint_as_float(u.x << 16); xv[1] = __uint_as_float(u.x & 0xffff0000u);
        xv[2] = __uint_as_float(u.y << 16); xv[3] = __uint_as_float(u.y & 0xffff0000u);
      } else {
        const float4 u = *reinterpret_cast<const float4*>(static_cast<const float*>(p.xbc) + xo);
        xv[0] = u.x; xv[1] = u.y; xv[2] = u.z; xv[3] = u.w;
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) win[c][L] = xv[c];
    }
    float wv[4 * K];
#pragma unroll
    for (int e = 0; e < 4 * K; ++e) wv[e] = ld_io(p.weight, (int64_t)d0 * K + e, WBF ? NSSM_BF16 : NSSM_F32);
    float out[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float acc = 0.0f;
#pragma unroll
      for (int k = 0; k < K; ++k) acc = fmaf(wv[c * K + k], win[c][L + 1 - K + k], acc);
      if (p.bias) acc = acc + ld_io(p.bias, d0 + c, WBF ? NSSM_BF16 : NSSM_F32);
      out[c] = p.act ? silu_f(acc) : acc;
    }
    // state <- last L of the window
    unsigned char* sp = static_cast<unsigned char*>(p.state) + (srow + (int64_t)d0 * L) * EB;
    if constexpr (IOBF) {
#pragma unroll
      for (int q = 0; q < L; ++q) {
        const int e0 = 4 * q;
        uint32_t h[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const int e = e0 + t, c = e / L, l = e % L;
          h[t] = __float_as_uint(win[c][l + 1]) >> 16;   // bf16 values: exact
        }
        reinterpret_cast<uint2*>(sp)[q] = make_uint2(h[0] | (h[1] << 16), h[2] | (h[3] << 16));
      }
      const __nv_bfloat162 o01 = __floats2bfloat162_rn(out[0], out[1]);
      const __nv_bfloat162 o23 = __floats2bfloat162_rn(out[2], out[3]);
      *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p.x_out) + (int64_t)b * p.x_sb + d0) =
          make_uint2(*reinterpret_cast<const uint32_t*>(&o01), *reinterpret_cast<const uint32_t*>(&o23));
    } else {
#pragma unroll
      for (int q = 0; q < L; ++q) {
        float v4[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const int e = 4 * q + t, c = e / L, l = e % L;
          v4[t] = win[c][l + 1];
        }
        reinterpret_cast<float4*>(sp)[q] = make_float4(v4[0], v4[1], v4[2], v4[3]);
      }
      *reinterpret_cast<float4*>(static_cast<float*>(p.x_out) + (int64_t)b * p.x_sb + d0) =
          make_float4(out[0], out[1], out[2], out[3]);
    }
  } else {
    for (int c = 0; c < 4 && d0 + c < p.I; ++c) {
      const float v = conv_channel(p, srow, b, d0 + c, true);
      st_io(p.x_out, (int64_t)b * p.x_sb + d0 + c, p.dtype, v);
    }
  }
}

}  // namespace nssm
