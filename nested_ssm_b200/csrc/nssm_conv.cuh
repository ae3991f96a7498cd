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
  int64_t state_ss;     // element (s, d, l) at s * state_ss + d * state_sd + l * state_sl
  int64_t state_sd, state_sl;
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
  const int64_t so = srow + (int64_t)d * p.state_sd;
  float win[kConvMaxL + 1];
#pragma unroll
  for (int l = 0; l <= kConvMaxL; ++l)
    win[l] = l < p.L ? ld_io(p.state, so + l * p.state_sl, p.dtype) : (l == p.L ? xin : 0.0f);
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
      if (l < p.L) st_io(p.state, so + l * p.state_sl, p.dtype, win[l + 1]);
  }
  return p.act ? silu_f(acc) : acc;
}

// Four consecutive channels d0 .. d0+3 of one row with compile-time width K and state
// length L: the loads (state, x) and the compute + stores are separate steps so a thread
// can have several groups' loads in flight.  Every access is aligned (checked on the host).
template <int L, bool IOBF>
struct Conv4 {
  float s[4 * L];
  float x[4];
};

// LD: the state is channels-last ([slot][l][d], the HF / vLLM cache layout): each window
// position of the 4 channels is one vector; otherwise [slot][d][l]: the 4 channels' L
// positions are 4 * L consecutive elements.  c.s[ch * L + l] either way.
template <int L, bool IOBF, bool LD>
__device__ __forceinline__ void conv4_load(const ConvParams& p, int64_t srow, int b, int d0, Conv4<L, IOBF>& c) {
  constexpr int EB = IOBF ? 2 : 4;
  const int64_t xo = (int64_t)b * p.xbc_sb + d0;
  if constexpr (LD) {
#pragma unroll
    for (int l = 0; l < L; ++l) {
      const int64_t e = srow + (int64_t)l * p.state_sl + d0;
      float v[4];
      if constexpr (IOBF) {
        const uint2 u = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(p.state) + e);
        v[0] = __uint_as_float(u.x << 16); v[1] = __uint_as_float(u.x & 0xffff0000u);
        v[2] = __uint_as_float(u.y << 16); v[3] = __uint_as_float(u.y & 0xffff0000u);
      } else {
        const float4 u = *reinterpret_cast<const float4*>(static_cast<const float*>(p.state) + e);
        v[0] = u.x; v[1] = u.y; v[2] = u.z; v[3] = u.w;
      }
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) c.s[ch * L + l] = v[ch];
    }
  }
  const unsigned char* sp = static_cast<const unsigned char*>(p.state) + (srow + (int64_t)d0 * L) * EB;
  if constexpr (IOBF) {
#pragma unroll
    for (int q = 0; q < (LD ? 0 : L); ++q) {   // 4 * L bf16 = L x 8 bytes
      const uint2 u = reinterpret_cast<const uint2*>(sp)[q];
      c.s[4 * q + 0] = __uint_as_float(u.x << 16);
      c.s[4 * q + 1] = __uint_as_float(u.x & 0xffff0000u);
      c.s[4 * q + 2] = __uint_as_float(u.y << 16);
      c.s[4 * q + 3] = __uint_as_float(u.y & 0xffff0000u);
    }
    const uint2 u = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(p.xbc) + xo);
    c.x[0] = __uint_as_float(u.x << 16); c.x[1] = __uint_as_float(u.x & 0xffff0000u);
    c.x[2] = __uint_as_float(u.y << 16); c.x[3] = __uint_as_float(u.y & 0xffff0000u);
  } else {
#pragma unroll
    for (int q = 0; q < (LD ? 0 : L); ++q) {
      const float4 u = reinterpret_cast<const float4*>(sp)[q];
      c.s[4 * q + 0] = u.x; c.s[4 * q + 1] = u.y; c.s[4 * q + 2] = u.z; c.s[4 * q + 3] = u.w;
    }
    const float4 u = *reinterpret_cast<const float4*>(static_cast<const float*>(p.xbc) + xo);
    c.x[0] = u.x; c.x[1] = u.y; c.x[2] = u.z; c.x[3] = u.w;
  }
}

// 4 * K weights and 4 biases of channels d0 .. d0+3 as fp32
template <int K, bool WBF>
__device__ __forceinline__ void conv4_weights(const ConvParams& p, int d0, float* w, float* bias) {
  if constexpr (WBF) {
    const uint4* wp = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p.weight) + (int64_t)d0 * K);
#pragma unroll
    for (int q = 0; q < K / 2; ++q) {   // 8 bf16 per 16 bytes
      const uint4 u = wp[q];
      const uint32_t ww[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        w[8 * q + 2 * t] = __uint_as_float(ww[t] << 16);
        w[8 * q + 2 * t + 1] = __uint_as_float(ww[t] & 0xffff0000u);
      }
    }
    if (p.bias) {
      const uint2 u = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(p.bias) + d0);
      bias[0] = __uint_as_float(u.x << 16); bias[1] = __uint_as_float(u.x & 0xffff0000u);
      bias[2] = __uint_as_float(u.y << 16); bias[3] = __uint_as_float(u.y & 0xffff0000u);
    }
  } else {
    const float4* wp = reinterpret_cast<const float4*>(static_cast<const float*>(p.weight) + (int64_t)d0 * K);
#pragma unroll
    for (int q = 0; q < K; ++q) {
      const float4 u = wp[q];
      w[4 * q] = u.x; w[4 * q + 1] = u.y; w[4 * q + 2] = u.z; w[4 * q + 3] = u.w;
    }
    if (p.bias) {
      const float4 u = *reinterpret_cast<const float4*>(static_cast<const float*>(p.bias) + d0);
      bias[0] = u.x; bias[1] = u.y; bias[2] = u.z; bias[3] = u.w;
    }
  }
}

// conv outputs of the 4 channels (activated, fp32) and the state written back
template <int K, int L, bool IOBF, bool WBF, bool LD>
__device__ __forceinline__ void conv4_finish(const ConvParams& p, int64_t srow, int d0, const Conv4<L, IOBF>& c,
                                             float* out) {
  float w[4 * K], bias[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  conv4_weights<K, WBF>(p, d0, w, bias);
#pragma unroll
  for (int ch = 0; ch < 4; ++ch) {
    // window position l of [state, x] holds tap k = l - (L + 1 - K)
    float acc = 0.0f;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int l = L + 1 - K + k;
      acc = fmaf(w[ch * K + k], l < L ? c.s[ch * L + l] : c.x[ch], acc);
    }
    if (p.bias) acc = acc + bias[ch];
    out[ch] = p.act ? silu_f(acc) : acc;
  }
  // state <- last L of the window: element e = ch * L + l takes window position l + 1
  constexpr int EB = IOBF ? 2 : 4;
  auto nv = [&](int e) { const int ch = e / L, l = e % L; return l + 1 < L ? c.s[ch * L + l + 1] : c.x[ch]; };
  if constexpr (LD) {
#pragma unroll
    for (int l = 0; l < L; ++l) {
      const int64_t e = srow + (int64_t)l * p.state_sl + d0;
      if constexpr (IOBF) {
        uint32_t h[4];
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) h[ch] = __float_as_uint(nv(ch * L + l)) >> 16;   // bf16 values: exact
        *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p.state) + e) =
            make_uint2(h[0] | (h[1] << 16), h[2] | (h[3] << 16));
      } else {
        *reinterpret_cast<float4*>(static_cast<float*>(p.state) + e) =
            make_float4(nv(l), nv(L + l), nv(2 * L + l), nv(3 * L + l));
      }
    }
    return;
  }
  unsigned char* sp = static_cast<unsigned char*>(p.state) + (srow + (int64_t)d0 * L) * EB;
  if constexpr (IOBF) {
#pragma unroll
    for (int q = 0; q < L; ++q) {
      uint32_t h[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) h[t] = __float_as_uint(nv(4 * q + t)) >> 16;   // bf16 values: exact
      reinterpret_cast<uint2*>(sp)[q] = make_uint2(h[0] | (h[1] << 16), h[2] | (h[3] << 16));
    }
  } else {
#pragma unroll
    for (int q = 0; q < L; ++q)
      reinterpret_cast<float4*>(sp)[q] = make_float4(nv(4 * q), nv(4 * q + 1), nv(4 * q + 2), nv(4 * q + 3));
  }
}

// B and C channels.  grid (ceil(T / kConvTile), G, 2): z = 0 for B, 1 for C.  A CTA
// converts the tile's channels of group g (state updated), then rotates them (all 128
// outputs: thread tile of 4 rows x 8 outputs) or copies them out.
template <int N, int K, int L, bool IOBF, bool WBF, bool LD>
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

  // the tile's B (or C) channels of group g into shared memory (state updated), rounded
  // to the io dtype
  {
    const int cbase = p.I + which * p.G * N + g * N;
    if constexpr (K > 0) {
      // thread -> (row r, 4 channels) tasks, kTasks at a time with all loads first
      constexpr int kQ = N / 4;
      constexpr int kTasks = kConvTile * kQ / kConvThreads;   // 8
      Conv4<L, IOBF> cin[kTasks];
      int64_t srow[kTasks];
#pragma unroll
      for (int u = 0; u < kTasks; ++u) {
        const int e = tid + u * kConvThreads;
        const int r = e / kQ, d0 = cbase + 4 * (e % kQ);
        const int b = b0 + r;
        srow[u] = -1;
        if (r < nr) {
          const int slot = p.idx ? p.idx[b] : b;
          if (slot != p.pad && slot >= 0 && slot < p.S) {
            srow[u] = (int64_t)slot * p.state_ss;
            conv4_load<L, IOBF, LD>(p, srow[u], b, d0, cin[u]);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < kTasks; ++u) {
        const int e = tid + u * kConvThreads;
        const int r = e / kQ, n0 = 4 * (e % kQ);
        float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (srow[u] >= 0) {
          conv4_finish<K, L, IOBF, WBF, LD>(p, srow[u], cbase + n0, cin[u], o);
#pragma unroll
          for (int t = 0; t < 4; ++t) o[t] = round_io(o[t], p.dtype);
        }
        *reinterpret_cast<float4*>(Xs + r * kRotLd + n0) = make_float4(o[0], o[1], o[2], o[3]);
      }
    } else {
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
// the state, weights and x move in 8- or 16-byte vectors; otherwise per element.
// grid (ceil(I / (4 * kConvXThreads)), T).
constexpr int kConvXThreads = 256;

template <int K, int L, bool IOBF, bool WBF, bool LD>
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
    Conv4<L, IOBF> cin;
    conv4_load<L, IOBF, LD>(p, srow, b, d0, cin);
    float out[4];
    conv4_finish<K, L, IOBF, WBF, LD>(p, srow, d0, cin, out);
    if constexpr (IOBF) {
      const __nv_bfloat162 o01 = __floats2bfloat162_rn(out[0], out[1]);
      const __nv_bfloat162 o23 = __floats2bfloat162_rn(out[2], out[3]);
      *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p.x_out) + (int64_t)b * p.x_sb + d0) =
          make_uint2(*reinterpret_cast<const uint32_t*>(&o01), *reinterpret_cast<const uint32_t*>(&o23));
    } else {
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
