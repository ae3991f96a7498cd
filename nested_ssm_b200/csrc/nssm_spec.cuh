// Self-speculative decoding on the tiered state: the hot-only draft step, the multi-token
// verify and the commit of the accepted tokens.
//
//   draft  (draft_step_kernel): one token of the hot-only model -- h <- h exp(dt A) +
//          (dt B_hot) x on a separate [S][H][P][pb] fp32 draft state (read from the pool's
//          hot slice on the first draft token), y = C_hot . h + D x; the pool is not touched.
//          The reference's cold="off" install (scale/v4_fused_decode.py:49-55 on the hot slice,
//          :140-142 no cold at all).
//   verify (verify_step_kernel): y of n tokens per row read against the committed tiered state
//          exactly as n successive decode tokens would read it (hot updated token by token in
//          registers, the stale cold slice read once, exp(glog) advanced by each token's dt A).
//          Read-only on the pool.  The window may end on a chunk boundary but not cross it:
//          (t % c) + n <= c.
//   commit (commit_step_kernel): the first k of those tokens made permanent -- the hot slice
//          replayed over them, their (x, dt, B_cold) written to the ring at t%c .. t%c+k-1,
//          glog and t advanced, and every row whose chunk is now complete named in flush_idx
//          for the FLUSH kernels that follow.  Commit of k tokens leaves the pool exactly as k
//          decode steps would (same arithmetic, same operation order).
#pragma once

#include "nssm_device.cuh"
#include "nssm_persistent.cuh"   // f2 and the packed fp32 helpers

namespace nssm {

enum : int { STATUS_SPEC_WINDOW = 4 };   // a window crosses a chunk boundary, or accept is out of range

struct SpecParams {
  StepParams sp;               // pool, per-row / per-head strides, token 0 of every input
  int ntok;                    // tokens per row in this call
  int64_t x_st, dt_st, B_st, C_st, out_st;   // element strides between a row's tokens
  const int32_t* accept;       // commit: tokens kept per batch row, 0..ntok
  int32_t* flush_idx;          // commit: slot of each row whose chunk completed, else -1
  float* draft;                // draft: [S][H][P][PB] fp32 draft state
  int from_pool;               // draft: read the pool's hot slice instead of the draft state
};

// dt of one (row, head, token): softplus(dt + dt_bias), clamped below, as the decode step
__device__ __forceinline__ float spec_dt(const StepParams& p, int b, int h, int64_t toff) {
  float d = ld_io(p.dt, (int64_t)b * p.dt_sb + (int64_t)h * p.dt_sh + toff, p.dt_dtype);
  if (p.dt_bias) d += p.dt_bias[h];
  if (p.softplus) d = softplus_f(d);
  if (p.dt_min > 0.0f) d = fmaxf(d, p.dt_min);
  return d;
}

// h <- h exp(dt A) + (dt B) x on the thread's hot chunks, and the row sums C . h into yh.
// Chunk i = k*T + tid holds hot[i / LPR][4 (i % LPR) ..]; the LPR lanes of a row are
// consecutive lanes of one warp (T % LPR == 0).
template <int PB, int HCH>
__device__ __forceinline__ void hot_token(float4 (&hv)[HCH], int T, int tid, int nh, float dt, float decay,
                                          const float* Bs, const float* Cs, const float* s_x, float* yh,
                                          bool sums) {
  constexpr int LPR = PB / 4;
  const int hcol = tid % LPR;
  float dtB[4], ch[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    dtB[e] = dt * Bs[hcol * 4 + e];
    ch[e] = Cs ? Cs[hcol * 4 + e] : 0.0f;
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
      hv[k] = v;
      part = fmaf(v.x, ch[0], fmaf(v.y, ch[1], fmaf(v.z, ch[2], v.w * ch[3])));
    }
    if (sums) {
#pragma unroll
      for (int o = 1; o < LPR; o <<= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
      if (hcol == 0 && i < nh) yh[i / LPR] = part;
    }
  }
}

// ---- draft ------------------------------------------------------------------
template <int PB, int N, int TPR>
__global__ void __launch_bounds__(128 * TPR) draft_step_kernel(const SpecParams q) {
  const StepParams& p = q.sp;
  constexpr int LPR = PB / 4;
  constexpr int HCH = (LPR + TPR - 1) / TPR;
  const int T = blockDim.x, tid = threadIdx.x;
  const int h = blockIdx.x, b = blockIdx.y;
  const int Pn = p.P;
  __shared__ float Bs[PB], Cs[PB], s_x[128], yh[128];
  __shared__ float s_dt, s_decay;

  const int slot = p.idx ? p.idx[b] : b;
  if (slot == p.pad) return;
  if (slot < 0 || slot >= p.S) {
    if (tid == 0 && p.status) atomicOr(p.status, STATUS_BAD_SLOT);
    return;
  }
  const int g = h / (p.H / p.G);
  const int64_t sh = (int64_t)slot * p.H + h;
  const float4* src = reinterpret_cast<const float4*>((q.from_pool ? p.hot : q.draft) + sh * (int64_t)Pn * PB);
  float4* dst = reinterpret_cast<float4*>(q.draft + sh * (int64_t)Pn * PB);
  const int nh = Pn * LPR;
  float4 hv[HCH];
#pragma unroll
  for (int k = 0; k < HCH; ++k) {
    const int i = k * T + tid;
    if (i < nh) hv[k] = src[i];
  }
  if (tid < Pn) s_x[tid] = ld_io(p.x, (int64_t)b * p.x_sb + (int64_t)h * p.x_sh + tid, p.io_dtype);
  for (int n = tid; n < PB; n += T) {
    Bs[n] = ld_io(p.B, (int64_t)b * p.B_sb + (int64_t)g * N + n, p.io_dtype);
    Cs[n] = ld_io(p.C, (int64_t)b * p.C_sb + (int64_t)g * N + n, p.io_dtype);
  }
  if (tid == 0) {
    const float d = spec_dt(p, b, h, 0);
    s_dt = d;
    s_decay = expf(d * p.A[h]);
  }
  __syncthreads();
  hot_token<PB, HCH>(hv, T, tid, nh, s_dt, s_decay, Bs, Cs, s_x, yh, true);
#pragma unroll
  for (int k = 0; k < HCH; ++k) {
    const int i = k * T + tid;
    if (i < nh) dst[i] = hv[k];
  }
  __syncthreads();
  if (tid < Pn) {
    float y = yh[tid];
    if (p.D) y = fmaf(s_x[tid], p.D[h], y);
    st_io(p.out, (int64_t)b * p.out_sb + (int64_t)h * p.out_sh + tid, p.out_dtype, y);
  }
}

// ---- verify -----------------------------------------------------------------
// Two threads per headdim row: thread 2r + u holds half u of row r's hot slice (fp32, PB/2
// values) and of its cold slice (decoded to fp32 once, the first ceil(CPR/2) 16-byte chunks for
// u = 0, the rest for u = 1).  Tokens are staged TC at a time (x, B_hot, C and the dt scalars,
// one round of loads); each thread then runs the hot recurrence of its half row through the
// staged tokens and forms both partial dot products, and one shuffle combines the pair.  Every
// lane of a warp reads the same B / C words (shared-memory broadcast).  Two block barriers per
// TC tokens.  Headdim <= 80 (the persistent kernels' limit, which verify shares): <= 160 threads.
constexpr int kVerifyTC = 16;

template <int PB, int NC, int COLD>
__host__ __device__ constexpr size_t verify_smem_floats(int P) {
  // per staged token: B_hot, C_hot [PB], C_cold [NC], x [P]; dt, dA, exp(dA), exp(glog) [4 TC]
  return (size_t)kVerifyTC * (2 * PB + NC + (size_t)P) + 4 * (size_t)kVerifyTC;
}

// 16 bytes of io values (8 bf16 or 4 fp32) as fp32 into shared memory
template <bool IOBF>
__device__ __forceinline__ void stage16(const void* src, float* dst) {
  const uint4 v = *reinterpret_cast<const uint4*>(src);
  if constexpr (IOBF) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 2; ++i)
      reinterpret_cast<float4*>(dst)[i] = make_float4(__uint_as_float(w[2 * i] << 16), __uint_as_float(w[2 * i] & 0xffff0000u),
                                                      __uint_as_float(w[2 * i + 1] << 16),
                                                      __uint_as_float(w[2 * i + 1] & 0xffff0000u));
  } else {
    *reinterpret_cast<float4*>(dst) = make_float4(__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z),
                                                  __uint_as_float(v.w));
  }
}

template <int PB, int NC, int COLD, bool IOBF>
__global__ void __launch_bounds__(160, 4) verify_step_kernel(const SpecParams q) {
  const StepParams& p = q.sp;
  using Sh = StepShape<PB, NC, COLD>;
  constexpr int N = Sh::N;
  constexpr int CPR = Sh::CPR;        // 16-byte cold chunks per row
  constexpr int CE = Sh::CE;          // values per chunk
  constexpr int K0 = (CPR + 1) / 2;   // chunks of half 0 (half 1 takes CPR - K0)
  constexpr int HQ = PB / 8;          // hot float4 per half row
  constexpr int kPerW = WordTraits<COLD>::kPer;
  constexpr int TC = kVerifyTC;
  static_assert(Sh::kCold, "tiered instances only");
  static_assert(PB % 8 == 0 && CE % 4 == 0, "half rows of whole float4s");

  const int tid = threadIdx.x;
  const int h = blockIdx.x, b = blockIdx.y;
  const int Pn = p.P, c = p.c;
  const int row = tid >> 1, u = tid & 1;
  const bool act = row < Pn;
  extern __shared__ __align__(16) float smem[];
  float* Bh = smem;                 // [TC][PB]
  float* Ch = Bh + TC * PB;         // [TC][PB]
  float* Cc = Ch + TC * PB;         // [TC][NC]
  float* s_x = Cc + TC * NC;        // [TC][P]
  float* s_dt = s_x + TC * Pn;      // [TC]
  float* s_dA = s_dt + TC;          // [TC]
  float* s_dec = s_dA + TC;         // [TC]
  float* s_eg = s_dec + TC;         // [TC]
  __shared__ int s_r;

  const int slot = p.idx ? p.idx[b] : b;
  if (slot == p.pad) return;
  if (slot < 0 || slot >= p.S) {
    if (tid == 0 && p.status) atomicOr(p.status, STATUS_BAD_SLOT);
    return;
  }
  const int g = h / (p.H / p.G);
  const int64_t sh = (int64_t)slot * p.H + h;
  const bool cold_read = p.mode != NSSM_MODE_COLDOFF;

  // ---- one round of loads: this thread's half row (hot fp32, raw cold chunks), the item's
  //      bookkeeping and the first staged tokens; the cold chunks are decoded afterwards
  float4 hv[HQ];
  uint4 craw[K0];
  float cv[K0 * CE];
  float scl = 0.0f;
  const int kn = u == 0 ? K0 : CPR - K0;
  if (act) {
    const float4* hot4 = reinterpret_cast<const float4*>(p.hot + (sh * Pn + row) * PB) + u * HQ;
#pragma unroll
    for (int k = 0; k < HQ; ++k) hv[k] = hot4[k];
    if (cold_read) {
      const uint4* c16 = reinterpret_cast<const uint4*>(static_cast<const char*>(p.cold) +
                                                        (sh * Pn + row) * (int64_t)(NC * Sh::ESZ)) + u * K0;
#pragma unroll
      for (int k = 0; k < K0; ++k)
        if (k < kn) craw[k] = c16[k];
      scl = (COLD == COLD_FP8) ? p.scale[sh * Pn + row] : 1.0f;
    }
  }
  float glog = 0.0f;   // thread 0: glog before the next token to be read
  if (tid == 0) {
    const int r = p.t[sh] % c;
    s_r = (r + q.ntok <= c) ? r : -1;
    glog = p.glog[sh];
  }
  const float A_h = p.A[h];
  const float Dh = p.D ? p.D[h] : 0.0f;
  const int T = blockDim.x;

  for (int j0 = 0; j0 < q.ntok; j0 += TC) {
    const int nt = min(TC, q.ntok - j0);
    // ---- stage the nt tokens: 16-byte chunks of x, B_hot and C, one per thread and pass
    {
      constexpr int EPC = IOBF ? 8 : 4;   // io values per 16-byte chunk
      constexpr int IOB = IOBF ? 2 : 4;
      const int xc = Pn / EPC, per = xc + PB / EPC + N / EPC;
      const char* xb = static_cast<const char*>(p.x);
      const char* bb = static_cast<const char*>(p.B);
      const char* cb = static_cast<const char*>(p.C);
      for (int e = tid; e < nt * per; e += T) {
        const int j = e / per, k = e - j * per;
        const int64_t tok = j0 + j;
        if (k < xc) {
          stage16<IOBF>(xb + ((int64_t)b * p.x_sb + tok * q.x_st + (int64_t)h * p.x_sh + k * EPC) * IOB,
                        s_x + j * Pn + k * EPC);
        } else if (k < xc + PB / EPC) {
          const int n0 = (k - xc) * EPC;
          stage16<IOBF>(bb + ((int64_t)b * p.B_sb + tok * q.B_st + (int64_t)g * N + n0) * IOB, Bh + j * PB + n0);
        } else {
          const int n0 = (k - xc - PB / EPC) * EPC;
          float* dst = n0 < PB ? Ch + j * PB + n0 : Cc + j * NC + (n0 - PB);
          stage16<IOBF>(cb + ((int64_t)b * p.C_sb + tok * q.C_st + (int64_t)g * N + n0) * IOB, dst);
        }
      }
    }
    if (tid < nt) {
      const float d = spec_dt(p, b, h, (j0 + tid) * q.dt_st);
      const float dA = d * A_h;
      s_dt[tid] = d;
      s_dA[tid] = dA;
      s_dec[tid] = expf(dA);
    }
    if (j0 == 0 && act && cold_read) {   // decode the cold chunks once
#pragma unroll
      for (int k = 0; k < K0; ++k) {
        if (k < kn) {
          const uint32_t wv[4] = {craw[k].x, craw[k].y, craw[k].z, craw[k].w};
#pragma unroll
          for (int wi = 0; wi < 4; ++wi) word_to_float<COLD>(wv[wi], cv + k * CE + wi * kPerW);
        }
      }
    }
    __syncthreads();
    if (s_r < 0) {   // uniform: the window crosses a chunk boundary
      if (tid == 0 && p.status) atomicOr(p.status, STATUS_SPEC_WINDOW);
      return;
    }
    if (tid == 0) {   // the stale read of token j: glog + dA_0 + ... + dA_{j-1}, summed in token order
      for (int j = 0; j < nt; ++j) {
        s_eg[j] = expf(glog);
        glog = glog + s_dA[j];
      }
    }
    __syncthreads();
    for (int j = 0; j < nt; ++j) {
      float yhot = 0.0f, ycold = 0.0f;
      float xp = 0.0f;
      if (act) {   // packed fp32 pairs: the same per-element rounding as the scalar form
        const float dt = s_dt[j], decay = s_dec[j];
        xp = s_x[j * Pn + row];
        const float2 dt2 = f2(dt, dt), x2 = f2(xp, xp), dec2 = f2(decay, decay);
        const float4* b4 = reinterpret_cast<const float4*>(Bh + j * PB) + u * HQ;
        const float4* c4 = reinterpret_cast<const float4*>(Ch + j * PB) + u * HQ;
        float2 yh2 = f2(0.0f, 0.0f);
#pragma unroll
        for (int k = 0; k < HQ; ++k) {
          const float4 bb = b4[k], cc = c4[k];
          const float4 v = hv[k];
          const float2 a = __ffma2_rn(f2(v.x, v.y), dec2, __fmul2_rn(__fmul2_rn(dt2, f2(bb.x, bb.y)), x2));
          const float2 d = __ffma2_rn(f2(v.z, v.w), dec2, __fmul2_rn(__fmul2_rn(dt2, f2(bb.z, bb.w)), x2));
          hv[k] = make_float4(a.x, a.y, d.x, d.y);
          yh2 = __ffma2_rn(a, f2(cc.x, cc.y), yh2);
          yh2 = __ffma2_rn(d, f2(cc.z, cc.w), yh2);
        }
        yhot = yh2.x + yh2.y;
        if (cold_read) {
          const float4* cc4 = reinterpret_cast<const float4*>(Cc + j * NC + u * K0 * CE);
          float2 yc2 = f2(0.0f, 0.0f);
#pragma unroll
          for (int k = 0; k < K0; ++k) {
            if (k < kn) {
#pragma unroll
              for (int v = 0; v < CE / 4; ++v) {
                const float4 cc = cc4[k * (CE / 4) + v];
                const float* qv = cv + k * CE + 4 * v;
                yc2 = __ffma2_rn(f2(qv[0], qv[1]), f2(cc.x, cc.y), yc2);
                yc2 = __ffma2_rn(f2(qv[2], qv[3]), f2(cc.z, cc.w), yc2);
              }
            }
          }
          ycold = yc2.x + yc2.y;
        }
      }
      yhot += __shfl_xor_sync(0xffffffffu, yhot, 1);
      ycold += __shfl_xor_sync(0xffffffffu, ycold, 1);
      if (act && u == 0) {
        float y = yhot;
        if (cold_read) y += (ycold * scl) * s_eg[j];
        if (p.D) y = fmaf(xp, Dh, y);
        st_io(p.out, (int64_t)b * p.out_sb + (j0 + j) * q.out_st + (int64_t)h * p.out_sh + row, p.out_dtype, y);
      }
    }
    __syncthreads();   // the next chunk restages
  }
}

// ---- commit -----------------------------------------------------------------
constexpr int kCommitTC = 16;   // tokens staged at a time

template <int PB, int N, int TPR, bool IOBF>
__global__ void __launch_bounds__(128 * TPR) commit_step_kernel(const SpecParams q) {
  constexpr int NC = N - PB;
  const StepParams& p = q.sp;
  constexpr int LPR = PB / 4;
  constexpr int HCH = (LPR + TPR - 1) / TPR;
  const int T = blockDim.x, tid = threadIdx.x;
  const int h = blockIdx.x, b = blockIdx.y;
  const int Pn = p.P, c = p.c;
  __shared__ __align__(16) float Bs[kCommitTC * PB];
  __shared__ __align__(16) float s_x[kCommitTC * 128];
  __shared__ float s_dt[kCommitTC], s_dA[kCommitTC], s_dec[kCommitTC];
  __shared__ int s_k, s_r;
  const bool lead = (h == 0 && tid == 0);   // writes the row's flush_idx entry

  const int slot = p.idx ? p.idx[b] : b;
  if (slot == p.pad) {
    if (lead) q.flush_idx[b] = -1;
    return;
  }
  if (slot < 0 || slot >= p.S) {
    if (lead) q.flush_idx[b] = -1;
    if (tid == 0 && p.status) atomicOr(p.status, STATUS_BAD_SLOT);
    return;
  }
  const int HG = p.H / p.G;
  const int g = h / HG;
  const int64_t sh = (int64_t)slot * p.H + h;
  const int cp = ring_dt_stride(c);
  // the hot slice is loaded with the bookkeeping, before the accept count is known (a row
  // that keeps no token only wastes the read)
  float4* hot4 = reinterpret_cast<float4*>(p.hot + sh * (int64_t)Pn * PB);
  const int nh = Pn * LPR;
  float4 hv[HCH];
#pragma unroll
  for (int kk = 0; kk < HCH; ++kk) {
    const int i = kk * T + tid;
    if (i < nh) hv[kk] = hot4[i];
  }
  int t0 = 0;
  if (tid == 0) {
    const int k = q.accept[b];
    t0 = p.t[sh];
    s_k = (k >= 0 && k <= q.ntok && t0 % c + k <= c) ? k : -1;
    s_r = t0 % c;
  }
  __syncthreads();
  const int k = s_k;
  const int r = s_r;
  if (k <= 0) {
    if (lead) q.flush_idx[b] = -1;
    if (k < 0 && tid == 0 && p.status) atomicOr(p.status, STATUS_SPEC_WINDOW);
    return;
  }
  const float A_h = p.A[h];
  float glog = 0.0f;
  if (tid == 0) glog = p.glog[sh];
  for (int j0 = 0; j0 < k; j0 += kCommitTC) {
    const int nt = min(kCommitTC, k - j0);
    // ---- stage the nt tokens in 16-byte chunks (x -> shared and the ring, B_hot -> shared,
    //      B_cold -> the ring by the group's first head) and their dt scalars
    {
      constexpr int EPC = IOBF ? 8 : 4;   // io values per 16-byte chunk
      constexpr int IOB = IOBF ? 2 : 4;
      const int xc = Pn / EPC;
      const int bcn = (h % HG == 0) ? N / EPC : PB / EPC;   // B chunks this CTA needs
      const int per = xc + bcn;
      const char* xb = static_cast<const char*>(p.x);
      const char* bb = static_cast<const char*>(p.B);
      for (int e = tid; e < nt * per; e += T) {
        const int j = e / per, kk = e - j * per;
        const int64_t tok = j0 + j;
        const int pos = r + j0 + j;
        if (kk < xc) {
          const uint4 v = *reinterpret_cast<const uint4*>(
              xb + ((int64_t)b * p.x_sb + tok * q.x_st + (int64_t)h * p.x_sh + kk * EPC) * IOB);
          *reinterpret_cast<uint4*>(static_cast<char*>(p.ring_x) + ((sh * c + pos) * Pn + kk * EPC) * IOB) = v;
          stage16<IOBF>(&v, s_x + j * Pn + kk * EPC);
        } else {
          const int n0 = (kk - xc) * EPC;
          const char* src = bb + ((int64_t)b * p.B_sb + tok * q.B_st + (int64_t)g * N + n0) * IOB;
          if (n0 < PB) {
            stage16<IOBF>(src, Bs + j * PB + n0);
          } else {
            stage16<IOBF>(src, p.ring_b + (((int64_t)slot * p.G + g) * c + pos) * NC + (n0 - PB));
          }
        }
      }
    }
    if (tid < nt) {
      const float d = spec_dt(p, b, h, (j0 + tid) * q.dt_st);
      const float dA = d * A_h;
      s_dt[tid] = d;
      s_dA[tid] = dA;
      s_dec[tid] = expf(dA);
      p.ring_dt[sh * cp + r + j0 + tid] = d;
    }
    __syncthreads();
    if (tid == 0)
      for (int j = 0; j < nt; ++j) glog = glog + s_dA[j];   // in token order, as the steps
    for (int j = 0; j < nt; ++j)
      hot_token<PB, HCH>(hv, T, tid, nh, s_dt[j], s_dec[j], Bs + j * PB, nullptr, s_x + j * Pn, nullptr, false);
    __syncthreads();   // the next chunk restages
  }
#pragma unroll
  for (int kk = 0; kk < HCH; ++kk) {
    const int i = kk * T + tid;
    if (i < nh) hot4[i] = hv[kk];
  }
  if (tid == 0) {
    const int t1 = t0 + k;
    const bool flush = (t1 % c) == 0;
    p.glog[sh] = flush ? 0.0f : glog;   // the FLUSH that follows re-bases the cold slice
    p.t[sh] = t1;
    if (h == 0) q.flush_idx[b] = flush ? slot : -1;
  }
}

}  // namespace nssm
