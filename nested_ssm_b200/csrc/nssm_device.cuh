// Device code of the tiered Mamba2 decode state op (sm_100a).
//
// One CTA owns one (batch row, head) tile.  Thread (row p, part) owns
// hot[p][part*PB/TPR ...) and cold[p][part*NC/TPR ...) of that head: the tile is
// read once with 16-byte vector loads (8-byte where a row split is not a
// multiple of 16 B), updated in registers and written back once.  Dot products
// over d_state are reduced across the TPR lanes of a row with warp shuffles.
// B and C of the head's group are staged in shared memory as fp32.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "nested_ssm.h"

// Minimum resident CTAs per SM requested from ptxas for the non-persistent step
// kernel (caps its registers).  Measured on B200: the untiered instance (320
// threads) is fastest at 2 (64 registers, 5.5 TB/s); the tiered fallback at 4.
#ifndef NSSM_STEP_MINB
#define NSSM_STEP_MINB 4
#endif
#ifndef NSSM_FRESH_MINB
#define NSSM_FRESH_MINB 2
#endif

namespace nssm {

enum ColdKind { COLD_F32 = 0, COLD_BF16 = 1, COLD_FP8 = 2, COLD_NONE = 3 };

// Error bits OR-ed into the caller's status word.
enum : int { STATUS_BAD_SLOT = 1 };

constexpr float kFp8Max = 448.0f;
constexpr float kScaleEps = 1e-12f;
constexpr int kRingChunk = 16;  // ring entries staged in shared memory at a time
constexpr int kMaxChunk = 256;  // largest flush period c supported

// ring_dt rows are padded to a multiple of 4 entries (16 bytes) so a slot-head's
// row can be moved with one bulk copy.
__host__ __device__ __forceinline__ int ring_dt_stride(int c) { return (c + 3) & ~3; }

template <int K> struct ColdTraits;
template <> struct ColdTraits<COLD_F32> { static constexpr int kBytes = 4; };
template <> struct ColdTraits<COLD_BF16> { static constexpr int kBytes = 2; };
template <> struct ColdTraits<COLD_FP8> { static constexpr int kBytes = 1; };
template <> struct ColdTraits<COLD_NONE> { static constexpr int kBytes = 1; };

// Kernel parameters (passed by value).
struct StepParams {
  // pool
  float* hot;
  void* cold;
  float* scale;
  float* glog;
  int32_t* t;
  void* ring_x;
  float* ring_dt;
  float* ring_b;
  int S, H, P, G, c;
  // inputs
  const void* x;
  int64_t x_sb, x_sh;
  const void* dt;
  int64_t dt_sb, dt_sh;
  int dt_dtype;
  int softplus;
  const void* B;
  int64_t B_sb;
  const void* C;
  int64_t C_sb;
  int io_dtype;
  const float* A;
  const float* D;
  const float* dt_bias;
  float dt_min;
  int mode;
  const int32_t* idx;
  int pad;
  void* out;
  int64_t out_sb, out_sh;
  int out_dtype;
  int32_t* status;
  // fused gated RMS norm of y (ngate != nullptr): out = weight * round(h * rstd_group)
  const void* ngate;
  int64_t ngate_sb;
  const void* nweight;
  int nweight_dtype;
  float neps;
};

__device__ __forceinline__ float ld_io(const void* p, int64_t i, int dtype) {
  if (dtype == NSSM_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

__device__ __forceinline__ void st_io(void* p, int64_t i, int dtype, float v) {
  if (dtype == NSSM_BF16)
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else
    reinterpret_cast<float*>(p)[i] = v;
}

// torch.nn.functional.softplus (beta 1, threshold 20)
__device__ __forceinline__ float softplus_f(float v) {
  return v > 20.0f ? v : log1pf(expf(v));
}

// ---- register-resident vector of raw bytes, loaded/stored with the widest
// aligned vector access.
template <int BYTES>
struct RawVec {
  static constexpr int kVB = (BYTES % 16 == 0) ? 16 : ((BYTES % 8 == 0) ? 8 : 4);
  static constexpr int kWords = BYTES / 4;
  uint32_t w[kWords > 0 ? kWords : 1];

  __device__ __forceinline__ void load(const void* src) {
    if constexpr (kVB == 16) {
      const uint4* s = reinterpret_cast<const uint4*>(src);
#pragma unroll
      for (int i = 0; i < BYTES / 16; ++i) {
        uint4 v = s[i];
        w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
      }
    } else if constexpr (kVB == 8) {
      const uint2* s = reinterpret_cast<const uint2*>(src);
#pragma unroll
      for (int i = 0; i < BYTES / 8; ++i) {
        uint2 v = s[i];
        w[2 * i] = v.x; w[2 * i + 1] = v.y;
      }
    } else {
      const uint32_t* s = reinterpret_cast<const uint32_t*>(src);
#pragma unroll
      for (int i = 0; i < BYTES / 4; ++i) w[i] = s[i];
    }
  }
  __device__ __forceinline__ void store(void* dst) const {
    if constexpr (kVB == 16) {
      uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
      for (int i = 0; i < BYTES / 16; ++i)
        d[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
    } else if constexpr (kVB == 8) {
      uint2* d = reinterpret_cast<uint2*>(dst);
#pragma unroll
      for (int i = 0; i < BYTES / 8; ++i) d[i] = make_uint2(w[2 * i], w[2 * i + 1]);
    } else {
      uint32_t* d = reinterpret_cast<uint32_t*>(dst);
#pragma unroll
      for (int i = 0; i < BYTES / 4; ++i) d[i] = w[i];
    }
  }
};

// Element k (of CPT) of a raw cold chunk, as fp32 (exact for all storage types).
template <int COLD, int CPT>
__device__ __forceinline__ void cold_to_float(const uint32_t* w, float* v) {
  if constexpr (COLD == COLD_F32) {
#pragma unroll
    for (int k = 0; k < CPT; ++k) v[k] = __uint_as_float(w[k]);
  } else if constexpr (COLD == COLD_BF16) {
#pragma unroll
    for (int k = 0; k < CPT / 2; ++k) {
      v[2 * k] = __uint_as_float(w[k] << 16);
      v[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
    }
  } else {
#pragma unroll
    for (int k = 0; k < CPT / 4; ++k) {
      const uint32_t word = w[k];
      __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(word & 0xffffu), __NV_E4M3);
      __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(word >> 16), __NV_E4M3);
      float2 a = __half22float2(*reinterpret_cast<__half2*>(&lo));
      float2 b = __half22float2(*reinterpret_cast<__half2*>(&hi));
      v[4 * k] = a.x; v[4 * k + 1] = a.y; v[4 * k + 2] = b.x; v[4 * k + 3] = b.y;
    }
  }
}

// Elements per 32-bit storage word and the conversion of one word to fp32.
template <int COLD> struct WordTraits { static constexpr int kPer = 1; };
template <> struct WordTraits<COLD_BF16> { static constexpr int kPer = 2; };
template <> struct WordTraits<COLD_FP8> { static constexpr int kPer = 4; };

template <int COLD>
__device__ __forceinline__ void word_to_float(uint32_t word, float* v) {
  if constexpr (COLD == COLD_F32) {
    v[0] = __uint_as_float(word);
  } else if constexpr (COLD == COLD_BF16) {
    v[0] = __uint_as_float(word << 16);
    v[1] = __uint_as_float(word & 0xffff0000u);
  } else {
    __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(word & 0xffffu), __NV_E4M3);
    __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(word >> 16), __NV_E4M3);
    const float2 a = __half22float2(*reinterpret_cast<__half2*>(&lo));
    const float2 b = __half22float2(*reinterpret_cast<__half2*>(&hi));
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
  }
}

// Pack CPT fp32 values (already divided by the row scale for fp8) to storage.
template <int COLD, int CPT>
__device__ __forceinline__ void float_to_cold(const float* v, uint32_t* w) {
  if constexpr (COLD == COLD_F32) {
#pragma unroll
    for (int k = 0; k < CPT; ++k) w[k] = __float_as_uint(v[k]);
  } else if constexpr (COLD == COLD_BF16) {
#pragma unroll
    for (int k = 0; k < CPT / 2; ++k) {
      __nv_bfloat162 b = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
      w[k] = *reinterpret_cast<uint32_t*>(&b);
    }
  } else {
#pragma unroll
    for (int k = 0; k < CPT / 4; ++k) {
      const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(v[4 * k], v[4 * k + 1]), __NV_SATFINITE, __NV_E4M3);
      const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(v[4 * k + 2], v[4 * k + 3]), __NV_SATFINITE, __NV_E4M3);
      w[k] = (lo & 0xffffu) | (hi << 16);
    }
  }
}

template <int TPR>
__device__ __forceinline__ float row_sum(float v) {
#pragma unroll
  for (int o = 1; o < TPR; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int TPR>
__device__ __forceinline__ float row_max(float v) {
#pragma unroll
  for (int o = 1; o < TPR; o <<= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Requantise CPT fp32 values of one row part; the row amax is shared across the
// TPR lanes of the row.  fp8: scale = amax/448 + 1e-12, q = e4m3_rne(v/scale)
// with IEEE division (matches torch's (v / sc).to(float8_e4m3fn)).
template <int COLD, int CPT, int TPR>
__device__ __forceinline__ float requantise(float* v, uint32_t* w) {
  float sc = 1.0f;
  if constexpr (COLD == COLD_FP8) {
    float m = 0.0f;
#pragma unroll
    for (int k = 0; k < CPT; ++k) m = fmaxf(m, fabsf(v[k]));
    m = row_max<TPR>(m);
    sc = __fadd_rn(__fdiv_rn(m, kFp8Max), kScaleEps);
#pragma unroll
    for (int k = 0; k < CPT; ++k) v[k] = __fdiv_rn(v[k], sc);
  }
  float_to_cold<COLD, CPT>(v, w);
  return sc;
}

// --------------------------------------------------------------------------
// The per-token kernel.  One CTA = one (batch row, head); T = blockDim.x threads
// (a multiple of 32, >= TPR*P).  Global memory is moved in 16-byte chunks with
// chunk index i = k*T + tid, so every warp instruction covers 512 contiguous
// bytes of the tile:
//   hot  f32 [P][PB]: LPR = PB/4 chunks per row.  T % LPR == 0, so a thread's
//        hot columns are fixed (tid % LPR) and the LPR lanes of a row are
//        consecutive lanes of one warp: row sums are warp shuffles.
//   cold     [P][NC]: CPR = NC*esize/16 chunks per row; per-chunk partial dot
//        products (and, in a flush, per-chunk amax) are combined in shared memory.
// PB hot columns, NC cold columns, COLD storage kind.  COLD_NONE with NC == 0 is
// the untiered (fresh) update of a full fp32 state held in `hot`.
// --------------------------------------------------------------------------
template <int PB, int NC, int COLD>
struct StepShape {
  static constexpr int N = PB + NC;
  static constexpr bool kCold = (COLD != COLD_NONE) && NC > 0;
  static constexpr int ESZ = ColdTraits<COLD>::kBytes;
  static constexpr int LPR = PB / 4;
  static constexpr int CPR = kCold ? (NC * ESZ) / 16 : 1;
  static constexpr int CE = 16 / ESZ;
  // shared floats: Bs,Cs[N] | yh,s_x,s_sco,s_sc[P] | pc[P*CPR] | s_esuf,s_dtj[c] | rb[ch*NC] sW[ch*P]
  __host__ __device__ static constexpr size_t smem_floats(int P, int c) {
    return 2 * (size_t)N + 4 * (size_t)P + (size_t)P * CPR + 2 * (size_t)c +
           (size_t)(c < kRingChunk ? c : kRingChunk) * (size_t)((kCold ? NC : 0) + P);
  }
};

template <int PB, int NC, int COLD, int TPR>
__global__ void __launch_bounds__(128 * TPR, (TPR == 2 ? NSSM_STEP_MINB : NSSM_FRESH_MINB)) tiered_step_kernel(const StepParams p) {
  using Sh = StepShape<PB, NC, COLD>;
  constexpr int N = Sh::N;
  constexpr bool kCold = Sh::kCold;
  constexpr int LPR = Sh::LPR;
  constexpr int CPR = Sh::CPR;
  constexpr int CE = Sh::CE;
  constexpr int HCH = (LPR + TPR - 1) / TPR;                 // hot chunks per thread (max)
  constexpr int KCH = kCold ? (CPR + TPR - 1) / TPR : 1;     // cold chunks per thread (max)
  constexpr int kPerW = WordTraits<COLD>::kPer;
  static_assert(PB % 4 == 0 && LPR <= 32 && (LPR & (LPR - 1)) == 0, "hot width must be 4 x power of two <= 128");
  static_assert(!kCold || (NC * Sh::ESZ) % 16 == 0, "cold row must be whole 16-byte chunks");

  const int T = blockDim.x;
  const int tid = threadIdx.x;
  const int h = blockIdx.x, b = blockIdx.y;
  const int Pn = p.P;
  const int c = p.c;

  extern __shared__ float smem[];
  float* Bs = smem;               // [N] B of the head's group
  float* Cs = Bs + N;             // [N]
  float* yh = Cs + N;             // [P] hot row sums
  float* s_x = yh + Pn;           // [P] x of each row
  float* s_sco = s_x + Pn;        // [P] old cold scale of each row
  float* s_sc = s_sco + Pn;       // [P] new cold scale (flush)
  float* pc = s_sc + Pn;          // [P*CPR] cold chunk partials / chunk amax
  float* s_esuf = pc + Pn * CPR;  // [c]
  float* s_dtj = s_esuf + c;      // [c]
  const int chunk = min(c, kRingChunk);
  float* rb = s_dtj + c;          // [chunk][NC] ring B (flush)
  float* sW = rb + chunk * (kCold ? NC : 0);   // [chunk][P] flush weights
  __shared__ float s_dt, s_dA, s_decay, s_glog_raw, s_eglog, s_etot;
  __shared__ int s_tnew;

  const int slot = p.idx ? p.idx[b] : b;
  if (slot == p.pad) return;
  if (slot < 0 || slot >= p.S) {
    if (tid == 0 && p.status) atomicOr(p.status, STATUS_BAD_SLOT);
    return;
  }
  const int HG = p.H / p.G;
  const int g = h / HG;
  const int64_t sh = (int64_t)slot * p.H + h;   // (slot, head)

  // ---- first batch of loads: the tile and every small input, issued together
  const int nh = Pn * LPR;
  const int hcol = tid % LPR;
  float4* hot4 = reinterpret_cast<float4*>(p.hot + sh * (int64_t)Pn * PB);
  float4 hv[HCH];
#pragma unroll
  for (int k = 0; k < HCH; ++k) {
    const int i = k * T + tid;
    if (i < nh) hv[k] = hot4[i];
  }
  const int ncc = Pn * CPR;
  uint4* cold16 = nullptr;
  uint4 cw[KCH];
  if constexpr (kCold) {
    cold16 = reinterpret_cast<uint4*>(reinterpret_cast<char*>(p.cold) + sh * (int64_t)Pn * NC * Sh::ESZ);
#pragma unroll
    for (int k = 0; k < KCH; ++k) {
      const int i = k * T + tid;
      if (i < ncc) cw[k] = cold16[i];
    }
  }
  if (tid < Pn) {
    s_x[tid] = ld_io(p.x, (int64_t)b * p.x_sb + (int64_t)h * p.x_sh + tid, p.io_dtype);
    if constexpr (COLD == COLD_FP8) s_sco[tid] = p.scale[sh * Pn + tid];
  }
  for (int n = tid; n < N; n += T) {
    Bs[n] = ld_io(p.B, (int64_t)b * p.B_sb + (int64_t)g * N + n, p.io_dtype);
    Cs[n] = ld_io(p.C, (int64_t)b * p.C_sb + (int64_t)g * N + n, p.io_dtype);
  }
  if constexpr (kCold) {
    if (tid < c - 1) s_dtj[tid] = p.ring_dt[sh * ring_dt_stride(c) + tid];   // this chunk's earlier dts (flush / corr)
  }
  if (tid == 0) {
    float d = ld_io(p.dt, (int64_t)b * p.dt_sb + (int64_t)h * p.dt_sh, p.dt_dtype);
    if (p.dt_bias) d += p.dt_bias[h];
    if (p.softplus) d = softplus_f(d);
    if (p.dt_min > 0.0f) d = fmaxf(d, p.dt_min);
    const float dA = d * p.A[h];
    s_dt = d;
    s_dA = dA;
    s_decay = expf(dA);
    if constexpr (kCold) {
      s_tnew = p.t[sh] + 1;
      const float gl = p.glog[sh];
      s_glog_raw = gl;
      s_eglog = expf((p.mode == NSSM_MODE_CORR) ? gl + dA : gl);   // corr reads G_t inclusive
    }
  }
  __syncthreads();
  const float dt = s_dt, decay = s_decay;

  // ---- hot update h <- h*exp(dt A) + (dt B) x, stored back; row sums of C.h
  {
    float dtB[4], ch[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      dtB[e] = dt * Bs[hcol * 4 + e];
      ch[e] = Cs[hcol * 4 + e];
    }
#pragma unroll
    for (int k = 0; k < HCH; ++k) {
      const int i = k * T + tid;
      float part = 0.0f;
      if (i < nh) {
        const float xp = s_x[i / LPR];
        float4 v = hv[k];
        v.x = fmaf(v.x, decay, dtB[0] * xp);
        v.y = fmaf(v.y, decay, dtB[1] * xp);
        v.z = fmaf(v.z, decay, dtB[2] * xp);
        v.w = fmaf(v.w, decay, dtB[3] * xp);
        hot4[i] = v;
        part = fmaf(v.x, ch[0], fmaf(v.y, ch[1], fmaf(v.z, ch[2], v.w * ch[3])));
      }
#pragma unroll
      for (int o = 1; o < LPR; o <<= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
      if (hcol == 0 && i < nh) yh[i / LPR] = part;
    }
  }

  if constexpr (!kCold) {
    __syncthreads();
    if (tid < Pn) {
      float y = yh[tid];
      if (p.D) y = fmaf(s_x[tid], p.D[h], y);
      st_io(p.out, (int64_t)b * p.out_sb + (int64_t)h * p.out_sh + tid, p.out_dtype, y);
    }
    return;
  } else {
    // ---- stale cold readout: per-chunk partials sum_e q[e] C[n]
    if (p.mode != NSSM_MODE_COLDOFF) {
#pragma unroll
      for (int k = 0; k < KCH; ++k) {
        const int i = k * T + tid;
        if (i < ncc) {
          const int cc = i % CPR;
          const float* Cc = Cs + PB + cc * CE;
          const uint32_t wv[4] = {cw[k].x, cw[k].y, cw[k].z, cw[k].w};
          float part = 0.0f;
#pragma unroll
          for (int wi = 0; wi < 4; ++wi) {
            float q[kPerW];
            word_to_float<COLD>(wv[wi], q);
#pragma unroll
            for (int e = 0; e < kPerW; ++e) part = fmaf(q[e], Cc[wi * kPerW + e], part);
          }
          pc[i] = part;
        }
      }
    }
    const int tnew = s_tnew;
    const bool flush = (tnew % c) == 0;
    const int pos = (tnew - 1) % c;
    const float A_h = p.A[h];
    const int warp = tid >> 5, lane = tid & 31, nwarps = T >> 5;

    // ---- exact rank-c correction (mode corr): sum over this chunk's tokens j <= t of
    //      exp(G_t - G_j) (C_cold . B_j) (dt_j x_j)
    if (p.mode == NSSM_MODE_CORR) {
      const int J = pos + 1;
      if (tid == 0) {
        s_dtj[J - 1] = dt;
        float suf = 0.0f;
        s_esuf[J - 1] = 1.0f;
        for (int j = J - 2; j >= 0; --j) {
          suf = suf + s_dtj[j + 1] * A_h;
          s_esuf[j] = expf(suf);
        }
      }
      __syncthreads();
      for (int j = warp; j < J; j += nwarps) {
        float sdot = 0.0f;
        for (int k = lane; k < NC; k += 32) {
          const float bj = (j == J - 1) ? Bs[PB + k]
              : p.ring_b[(((int64_t)slot * p.G + g) * c + j) * NC + k];
          sdot = fmaf(Cs[PB + k], bj, sdot);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sdot += __shfl_xor_sync(0xffffffffu, sdot, o);
        if (lane == 0) s_esuf[j] = s_esuf[j] * sdot;     // w_j = exp(G_t - G_j) s_j
      }
    }
    __syncthreads();

    // ---- y = C_hot.h + exp(glog) scale C_cold.cold (+ corr) + D x, one thread per row
    if (tid < Pn) {
      float y = yh[tid];
      if (p.mode != NSSM_MODE_COLDOFF) {
        float yc = 0.0f;
#pragma unroll
        for (int cc = 0; cc < CPR; ++cc) yc += pc[tid * CPR + cc];
        const float scl = (COLD == COLD_FP8) ? s_sco[tid] : 1.0f;
        y += (yc * scl) * s_eglog;
      }
      if (p.mode == NSSM_MODE_CORR) {
        const int J = pos + 1;
        float ycorr = 0.0f;
        for (int j = 0; j < J; ++j) {
          const float xj = (j == J - 1) ? s_x[tid] : ld_io(p.ring_x, (sh * c + j) * Pn + tid, p.io_dtype);
          ycorr = fmaf(s_esuf[j], s_dtj[j] * xj, ycorr);
        }
        y += ycorr;
      }
      if (p.D) y = fmaf(s_x[tid], p.D[h], y);
      st_io(p.out, (int64_t)b * p.out_sb + (int64_t)h * p.out_sh + tid, p.out_dtype, y);
    }

    if (!flush) {
      // ---- ring write at pos, glog += dA
      if (tid < Pn) st_io(p.ring_x, (sh * c + pos) * Pn + tid, p.io_dtype, s_x[tid]);
      if (h % HG == 0) {
        for (int k = tid; k < NC; k += T)
          p.ring_b[(((int64_t)slot * p.G + g) * c + pos) * NC + k] = Bs[PB + k];
      }
      if (tid == 0) {
        p.ring_dt[sh * ring_dt_stride(c) + pos] = dt;
        p.glog[sh] = s_glog_raw + s_dA;
        p.t[sh] = tnew;
      }
      return;
    }

    // ---- flush: cold <- exp(sum dA) cold + sum_j exp(suf_j) (dt_j x_j) B_j, requantised.
    // Operation order matches the oracle: acc = sum_j (W_j * B_j[n]) in j order,
    // v = (q * scale) * exp(tot) + acc; fp8 scale = amax/448 + 1e-12, q = rne(v / scale).
    __syncthreads();   // the row pass above may still read s_esuf / s_dtj (corr) and pc
    if (tid == 0) {
      s_dtj[c - 1] = dt;
      float tot = 0.0f;
      for (int j = 0; j < c; ++j) tot = tot + s_dtj[j] * A_h;
      s_etot = expf(tot);
      float suf = 0.0f;
      s_esuf[c - 1] = 1.0f;
      for (int j = c - 2; j >= 0; --j) {
        suf = suf + s_dtj[j + 1] * A_h;
        s_esuf[j] = expf(suf);
      }
      p.glog[sh] = 0.0f;
      p.t[sh] = tnew;
    }
    auto stage = [&](int j0) {   // ring chunk j0.. into shared memory (uniform over the CTA)
      const int jn = min(chunk, c - j0);
      __syncthreads();
      for (int e = tid; e < jn * NC; e += T) {
        const int jj = e / NC, k = e - jj * NC;
        const int j = j0 + jj;
        rb[jj * NC + k] = (j == c - 1) ? Bs[PB + k]
            : p.ring_b[(((int64_t)slot * p.G + g) * c + j) * NC + k];
      }
      for (int e = tid; e < jn * Pn; e += T) {
        const int jj = e / Pn, r = e - jj * Pn;
        const int j = j0 + jj;
        const float xj = (j == c - 1) ? s_x[r] : ld_io(p.ring_x, (sh * c + j) * Pn + r, p.io_dtype);
        sW[jj * Pn + r] = __fmul_rn(s_esuf[j], __fmul_rn(s_dtj[j], xj));
      }
      __syncthreads();
    };
    const bool one_chunk = c <= kRingChunk;
    if (one_chunk) stage(0);
    const float etot = s_etot;
    // v of cold chunk k (CE values), recomputed identically in both passes
    auto chunk_values = [&](int k, float* v) {
      const int i = k * T + tid;
      const int row = (i < ncc) ? i / CPR : 0;
      const int cc = (i < ncc) ? i - row * CPR : 0;
#pragma unroll
      for (int e = 0; e < CE; ++e) v[e] = 0.0f;
      for (int j0 = 0; j0 < c; j0 += chunk) {
        if (!one_chunk) stage(j0);
        const int jn = min(chunk, c - j0);
        for (int jj = 0; jj < jn; ++jj) {
          const float W = sW[jj * Pn + row];
          const float* bj = rb + jj * NC + cc * CE;
#pragma unroll
          for (int e = 0; e < CE; ++e) v[e] = __fadd_rn(v[e], __fmul_rn(W, bj[e]));
        }
      }
      const float scl = (COLD == COLD_FP8) ? s_sco[row] : 1.0f;
      // re-read the (L1/L2-resident) old chunk instead of keeping it in registers
      const uint4 cv = (i < ncc) ? cold16[i] : make_uint4(0u, 0u, 0u, 0u);
      const uint32_t wv[4] = {cv.x, cv.y, cv.z, cv.w};
#pragma unroll
      for (int wi = 0; wi < 4; ++wi) {
        float q[kPerW];
        word_to_float<COLD>(wv[wi], q);
#pragma unroll
        for (int e = 0; e < kPerW; ++e) {
          const float deq = (COLD == COLD_FP8) ? __fmul_rn(q[e], scl) : q[e];
          v[wi * kPerW + e] = __fadd_rn(__fmul_rn(deq, etot), v[wi * kPerW + e]);
        }
      }
    };
    if constexpr (COLD == COLD_FP8) {
      // pass 1: per-chunk amax -> per-row scale
#pragma unroll 1
      for (int k = 0; k < KCH; ++k) {
        float v[CE];
        chunk_values(k, v);
        float m = 0.0f;
#pragma unroll
        for (int e = 0; e < CE; ++e) m = fmaxf(m, fabsf(v[e]));
        const int i = k * T + tid;
        if (i < ncc) pc[i] = m;
      }
      __syncthreads();
      if (tid < Pn) {
        float m = 0.0f;
#pragma unroll
        for (int cc = 0; cc < CPR; ++cc) m = fmaxf(m, pc[tid * CPR + cc]);
        const float sc = __fadd_rn(__fdiv_rn(m, kFp8Max), kScaleEps);
        s_sc[tid] = sc;
        p.scale[sh * Pn + tid] = sc;
      }
      __syncthreads();
    }
    // pass 2 (or the only pass): quantise and store
#pragma unroll 1
    for (int k = 0; k < KCH; ++k) {
      float v[CE];
      chunk_values(k, v);
      const int i = k * T + tid;
      if constexpr (COLD == COLD_FP8) {
        const float sc = s_sc[(i < ncc) ? i / CPR : 0];
#pragma unroll
        for (int e = 0; e < CE; ++e) v[e] = __fdiv_rn(v[e], sc);
      }
      uint32_t w[4];
      float_to_cold<COLD, CE>(v, w);
      if (i < ncc) cold16[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

// --------------------------------------------------------------------------
// Prefill split: full fp32 state rows -> hot / quantised cold; glog = t = 0.
// --------------------------------------------------------------------------
struct SplitParams {
  float* hot;
  void* cold;
  float* scale;
  float* glog;
  int32_t* t;
  int S, H, P;
  const float* src;
  int64_t src_sb;
  const int32_t* idx;
  int pad;
  int32_t* status;
};

template <int PB, int NC, int COLD, int TPR>
__global__ void __launch_bounds__(512) prefill_split_kernel(const SplitParams p) {
  constexpr int N = PB + NC;
  constexpr int HPT = PB / TPR;
  constexpr int CPT = NC / TPR;
  constexpr int kCB = CPT * ColdTraits<COLD>::kBytes;
  const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
  const int row = tid / TPR, part = tid % TPR;
  const bool act = row < p.P;
  const int slot = p.idx ? p.idx[b] : b;
  if (slot == p.pad) return;
  if (slot < 0 || slot >= p.S) {
    if (tid == 0 && p.status) atomicOr(p.status, STATUS_BAD_SLOT);
    return;
  }
  const int64_t sh = (int64_t)slot * p.H + h;
  const int64_t prow = sh * p.P + row;
  const float* src = p.src + (int64_t)b * p.src_sb + ((int64_t)h * p.P + row) * N;
  float cv[CPT];
  if (act) {
    const float4* hs = reinterpret_cast<const float4*>(src + part * HPT);
    float4* hd = reinterpret_cast<float4*>(p.hot + prow * PB + part * HPT);
#pragma unroll
    for (int i = 0; i < HPT / 4; ++i) hd[i] = hs[i];
    const float4* cs = reinterpret_cast<const float4*>(src + PB + part * CPT);
#pragma unroll
    for (int i = 0; i < CPT / 4; ++i) {
      float4 v = cs[i];
      cv[4 * i] = v.x; cv[4 * i + 1] = v.y; cv[4 * i + 2] = v.z; cv[4 * i + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int k = 0; k < CPT; ++k) cv[k] = 0.0f;
  }
  RawVec<kCB> cw;
  const float sc = requantise<COLD, CPT, TPR>(cv, cw.w);
  if (act) {
    cw.store(reinterpret_cast<char*>(p.cold) + (prow * NC + part * CPT) * ColdTraits<COLD>::kBytes);
    if constexpr (COLD == COLD_FP8) {
      if (part == 0) p.scale[prow] = sc;
    }
  }
  if (tid == 0) {
    p.glog[sh] = 0.0f;
    p.t[sh] = 0;
  }
}

// --------------------------------------------------------------------------
// Materialise: exact full fp32 state = hot ++ (cold replayed through the ring
// entries since the last flush).  Read-only on the pool.
// --------------------------------------------------------------------------
struct MatParams {
  const float* hot;
  const void* cold;
  const float* scale;
  const int32_t* t;
  const void* ring_x;
  const float* ring_dt;
  const float* ring_b;
  int S, H, P, G, c, io_dtype;
  const float* A;
  const int32_t* idx;
  int pad;
  float* out;
  int64_t out_sb;
  int32_t* status;
};

template <int PB, int NC, int COLD, int TPR>
__global__ void __launch_bounds__(512) materialize_kernel(const MatParams p) {
  constexpr int N = PB + NC;
  constexpr int HPT = PB / TPR;
  constexpr int CPT = NC / TPR;
  constexpr int kCB = CPT * ColdTraits<COLD>::kBytes;
  extern __shared__ float smem[];
  float* s_esuf = smem;                 // [kMaxChunk]
  float* s_dtj = smem + kMaxChunk;      // [kMaxChunk]
  __shared__ float s_etot;
  const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
  const int row = tid / TPR, part = tid % TPR;
  const bool act = row < p.P;
  const int slot = p.idx ? p.idx[b] : b;
  if (slot == p.pad) return;
  if (slot < 0 || slot >= p.S) {
    if (tid == 0 && p.status) atomicOr(p.status, STATUS_BAD_SLOT);
    return;
  }
  const int HG = p.H / p.G, g = h / HG;
  const int64_t sh = (int64_t)slot * p.H + h;
  const int64_t prow = sh * p.P + row;
  const int c = p.c;
  const int k = p.t[sh] % c;
  const float A_h = p.A[h];
  if (tid == 0) {
    float tot = 0.0f;
    for (int j = 0; j < k; ++j) {
      const float dj = p.ring_dt[sh * ring_dt_stride(c) + j];
      s_dtj[j] = dj;
      tot = tot + dj * A_h;
    }
    s_etot = expf(tot);
    if (k > 0) {
      float suf = 0.0f;
      s_esuf[k - 1] = 1.0f;
      for (int j = k - 2; j >= 0; --j) {
        suf = suf + s_dtj[j + 1] * A_h;
        s_esuf[j] = expf(suf);
      }
    }
  }
  __syncthreads();
  if (!act) return;
  float* dst = p.out + (int64_t)b * p.out_sb + ((int64_t)h * p.P + row) * N;
  {
    const float4* hs = reinterpret_cast<const float4*>(p.hot + prow * PB + part * HPT);
    float4* hd = reinterpret_cast<float4*>(dst + part * HPT);
#pragma unroll
    for (int i = 0; i < HPT / 4; ++i) hd[i] = hs[i];
  }
  RawVec<kCB> cw;
  cw.load(reinterpret_cast<const char*>(p.cold) + (prow * NC + part * CPT) * ColdTraits<COLD>::kBytes);
  float cv[CPT];
  cold_to_float<COLD, CPT>(cw.w, cv);
  const float scl = (COLD == COLD_FP8) ? p.scale[prow] : 1.0f;
  float acc[CPT];
#pragma unroll
  for (int q = 0; q < CPT; ++q) acc[q] = 0.0f;
  for (int j = 0; j < k; ++j) {
    const float xj = ld_io(p.ring_x, (sh * c + j) * p.P + row, p.io_dtype);
    const float W = __fmul_rn(s_esuf[j], __fmul_rn(s_dtj[j], xj));
    const int64_t bbase = (((int64_t)slot * p.G + g) * c + j) * NC + part * CPT;
#pragma unroll
    for (int q = 0; q < CPT; ++q) acc[q] = __fadd_rn(acc[q], __fmul_rn(W, p.ring_b[bbase + q]));
  }
  const float etot = s_etot;
#pragma unroll
  for (int q = 0; q < CPT; ++q) {
    const float deq = (COLD == COLD_FP8) ? __fmul_rn(cv[q], scl) : cv[q];
    dst[PB + part * CPT + q] = (k > 0) ? __fadd_rn(__fmul_rn(deq, etot), acc[q]) : deq;
  }
}

// --------------------------------------------------------------------------
// Rotation: out[t][g][m] = sum_n R[g][m][n] x[t][g][n], fp32 accumulation in
// n order, rounded once to the io dtype.  One CTA = (block of rows, group,
// tensor); R[g] is staged transposed (padded) in shared memory.
// --------------------------------------------------------------------------
}  // namespace nssm
