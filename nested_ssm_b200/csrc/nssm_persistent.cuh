// Persistent, TMA-pipelined kernels of the tiered step (sm_100a): the per-token
// STEP phase (hot update, stale readout, ring write, bookkeeping) and the FLUSH
// phase (rank-c replay of the ring into the cold slice + requantisation) of the
// slots whose token count reached a multiple of c.  A step launches STEP, then
// FLUSH on the same stream; FLUSH finds its work from the token counts STEP wrote.
//
// Grid = (#SMs x resident CTAs).  CTA k owns the contiguous range of work items
// [k*W/G, (k+1)*W/G) over (row, head), so it streams the tiles of consecutive heads of
// the same slot.  STEP: rows are the batch rows, W = batch*H.  FLUSH: rows are the batch
// rows at a chunk boundary, numbered in batch order, W = (their count)*H.
//
// Prologue (once per CTA): the slot and token count of every row in range and (STEP)
// every item's scalars (dt = softplus(dt_raw + dt_bias) clamped, dt*A, exp(dt*A),
// exp(glog), D) or (FLUSH) every item's suffix decays are computed in parallel into
// shared memory.
//
// Main loop: one elected thread keeps kStages items in flight with 1-D bulk copies
// (cp.async.bulk global->shared, no multicast) completing on a "full" mbarrier per
// stage.  Every warp owns a fixed band of headdim rows of every item, so row sums,
// the y pass, the replay and the row amax of the requantisation are warp-local: no
// CTA-wide barrier in the steady state.  A warp releases a stage by arriving on its
// "empty" mbarrier; the producer refills the stage once all warps arrived.
//
// Inside a band the tile is read in 16-byte chunks, consecutive lanes on
// consecutive chunks (conflict-free shared-memory reads, coalesced write-back).
#pragma once

#include "nssm_device.cuh"

// Pipeline depth, CTA size and resident CTAs per SM of the persistent kernels.
#ifndef NSSM_STEP_STAGES
#define NSSM_STEP_STAGES 3
#endif
#ifndef NSSM_FLUSH_STAGES
#define NSSM_FLUSH_STAGES 8
#endif
#ifndef NSSM_PTHREADS
#define NSSM_PTHREADS 256
#endif
#ifndef NSSM_STEP_P_MINB
#define NSSM_STEP_P_MINB 3
#endif
#ifndef NSSM_FLUSH_P_MINB
#define NSSM_FLUSH_P_MINB 3
#endif

namespace nssm {

constexpr int kMaxStages = NSSM_STEP_STAGES > NSSM_FLUSH_STAGES ? NSSM_STEP_STAGES : NSSM_FLUSH_STAGES;
__host__ __device__ constexpr int stages_for(int phase) { return phase == 0 ? NSSM_STEP_STAGES : NSSM_FLUSH_STAGES; }
constexpr int kPT = NSSM_PTHREADS;         // threads per CTA
constexpr int kPW = kPT / 32;              // warps per CTA
constexpr int kPMaxPersistent = 80;        // headdim bound of the persistent path (10 rows per warp)
constexpr int kRingInStage = 16;           // c up to this: the ring rides in the stage
constexpr int kRingF32Max = 8;             // c up to this: each warp keeps the ring B as fp32
constexpr uint32_t kSpinLimit = 1u << 26;  // default polls of a bounded mbarrier wait, then error + exit
enum : int { STATUS_TIMEOUT = 2 };
enum : int { PH_STEP = 0, PH_FLUSH = 1 };

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// 1-D bulk copy global -> this CTA's shared memory (16-byte aligned, size % 16 == 0)
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// 1-D bulk copy this CTA's shared memory -> global (16-byte aligned, size % 16 == 0)
__device__ __forceinline__ void bulk_s2g(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_u32(src)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// the shared-memory sources of all committed bulk stores have been read
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

// wait until at most the most recent bulk group of this thread still reads shared memory
__device__ __forceinline__ void bulk_wait_read_1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
// all committed bulk stores are complete
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait of at most `polls` tries; false on timeout.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t polls = kSpinLimit) {
  for (uint32_t it = 0; it < polls; ++it)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// Correctly rounded a / b given r = RN(1/b) (Markstein's FMA correction:
// q0 = RN(a r) is within one ulp of a/b, the residual a - b q0 is exact in one FMA,
// and RN(q0 + residual * r) is the correctly rounded quotient, barring underflow).
__device__ __forceinline__ float div_rn_fma(float a, float b, float r) {
  const float q0 = __fmul_rn(a, r);
  const float e = __fmaf_rn(-q0, b, a);
  return __fmaf_rn(e, r, q0);
}
// amax / 448 correctly rounded: Markstein's correction with rn(1/448); quotients far below
// the normal range (amax < 2^-100) take the full division
__device__ __forceinline__ float scale_div448(float m) {
  return m >= 0x1p-100f ? div_rn_fma(m, kFp8Max, 1.0f / kFp8Max) : __fdiv_rn(m, kFp8Max);
}

// Byte layout of the dynamic shared memory (computed on the host, passed in).
struct PLayout {
  int stage_bytes;
  int s_hot, s_cold, s_scale, s_x, s_b, s_c, s_rx, s_rb, s_rdt, s_gate;   // inside a stage (0 size if unused)
  int off_scal, off_head, off_yh, off_pc, off_sc, off_rcp, off_wsc, off_sw, off_rbw, off_fsc, off_bslot, off_bmeta,
      off_bpos, off_gbuf, off_nslot, off_bar;
  int total;
  int nst;          // pipeline stages
  int rpw;          // headdim rows per warp band
  int wsc_stride;   // floats of per-warp scratch (suffix decays / corr weights)
  int maxb;         // batch rows one CTA can touch
  int maxitems;     // items one CTA can own
};

__host__ __device__ inline int al(int v, int a) { return (v + a - 1) / a * a; }

constexpr int kScal = 8;   // per-item scalars (STEP): dt, dA, exp(dA), exp(glog), glog, D, A, -

template <int PB, int NC, int COLD>
__host__ inline PLayout make_playout(int phase, bool corr, int P, int H, int c, int io_bytes, int maxb,
                                     int maxitems, bool ring_in_stage, int nst, int norm_hg = 0) {
  constexpr int N = PB + NC;
  constexpr int ESZ = ColdTraits<COLD>::kBytes;
  constexpr int CPR = (NC * ESZ) / 16;
  const bool step = phase == PH_STEP;
  const bool ring = ring_in_stage && (!step || corr);
  PLayout L{};
  int o = 0;
  L.s_hot = o; o = al(o + (step ? P * PB * 4 : 0), 128);
  L.s_cold = o; o = al(o + P * NC * ESZ, 128);
  L.s_scale = o; o = al(o + (COLD == COLD_FP8 ? P * 4 : 0), 16);
  L.s_x = o; o = al(o + (step ? P * io_bytes : 0), 16);
  L.s_b = o; o = al(o + (step ? N * io_bytes : 0), 16);
  L.s_c = o; o = al(o + (step ? N * io_bytes : 0), 16);
  L.s_rx = o; o = al(o + (ring ? c * P * io_bytes : 0), 16);
  L.s_rb = o; o = al(o + (ring ? c * NC * 4 : 0), 16);      // ring B is fp32
  L.s_rdt = o; o = al(o + (ring ? ring_dt_stride(c) * 4 : 0), 16);
  L.s_gate = o; o = al(o + (step && norm_hg ? P * io_bytes : 0), 16);   // fused norm: the item's gate
  L.stage_bytes = al(o, 128);
  L.rpw = (P + kPW - 1) / kPW;
  L.wsc_stride = al(2 * c + 2, 4);
  L.nst = nst;
  int t = nst * L.stage_bytes;
  L.off_scal = t; t += (step ? maxitems * kScal * 4 : 0);
  L.off_head = t; t += H * 4;                    // A per head (FLUSH)
  L.off_yh = t; t += P * 4;
  L.off_pc = t; t += P * CPR * 4;
  L.off_sc = t; t += P * 4;
  L.off_rcp = t; t += P * 4;
  L.off_wsc = t; t += kPW * L.wsc_stride * 4;
  L.off_sw = t; t += (step ? 0 : c * P * 4);     // flush weights W_j[row] (rows are warp-private)
  L.off_rbw = t;
  // per-item suffix decays of the flush: exp(suf_j) [c], dt_j [c], exp(total)
  L.off_fsc = t; t += (!step && c <= kRingF32Max) ? maxitems * (2 * c + 1) * 4 : 0;
  L.off_bslot = t; t += maxb * 4;
  L.off_bmeta = t; t += maxb * 4;
  L.off_bpos = t; t += maxb * 4;
  L.off_gbuf = t; t += norm_hg * P * 4;          // fused norm: h of a (row, group) [heads][P]
  L.off_nslot = t; t += norm_hg ? 2 * kPW * 4 : 0;   // fused norm: per-warp sums of squares, 2 buffers
  t = al(t, 8);
  L.off_bar = t; t += 2 * nst * 8 + 8;           // full[stages], empty[stages], fused norm
  L.total = al(t, 128);
  L.maxb = maxb;
  L.maxitems = maxitems;
  return L;
}

struct PParams {
  StepParams sp;
  PLayout L;
  int items;          // batch * H
  int ring_in_stage;  // the ring rides in the stage (c <= kRingInStage, aligned)
  uint32_t polls;     // polls of a pipeline wait before it gives up (kSpinLimit by default)
  int inject_stuck;   // failure injection (tests only): CTA 0's first item never completes
};

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }

template <bool IOBF>
__device__ __forceinline__ float ldv(const void* p, int64_t i) {
  if constexpr (IOBF) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  else return reinterpret_cast<const float*>(p)[i];
}
template <bool IOBF>
__device__ __forceinline__ void stv(void* p, int64_t i, float v) {
  if constexpr (IOBF) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else reinterpret_cast<float*>(p)[i] = v;
}

// CNT consecutive io values starting at element n0 of a shared row, as fp32.
template <int CNT, bool IOBF>
__device__ __forceinline__ void ld_row(const unsigned char* row, int n0, float* v) {
  if constexpr (IOBF) {
    const unsigned char* s = row + n0 * 2;
    if constexpr (CNT % 8 == 0) {
#pragma unroll
      for (int q = 0; q < CNT / 8; ++q) {
        const uint4 w = reinterpret_cast<const uint4*>(s)[q];
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          v[8 * q + 2 * k] = __uint_as_float(ws[k] << 16);
          v[8 * q + 2 * k + 1] = __uint_as_float(ws[k] & 0xffff0000u);
        }
      }
    } else {
#pragma unroll
      for (int q = 0; q < CNT / 2; ++q) {
        const uint32_t w = reinterpret_cast<const uint32_t*>(s)[q];
        v[2 * q] = __uint_as_float(w << 16);
        v[2 * q + 1] = __uint_as_float(w & 0xffff0000u);
      }
    }
  } else {
    const float4* s = reinterpret_cast<const float4*>(row + n0 * 4);
#pragma unroll
    for (int q = 0; q < CNT / 4; ++q) {
      const float4 w = s[q];
      v[4 * q] = w.x; v[4 * q + 1] = w.y; v[4 * q + 2] = w.z; v[4 * q + 3] = w.w;
    }
  }
}

// CFIX > 0 compiles the kernel for that flush period (unrolled replay loops) and
// RPWC > 0 for headdim == 8 * RPWC (every warp band RPWC rows); 0 takes them from
// the parameters.
// NORM (STEP only) fuses the mixer's gated RMS norm into the y epilogue: CTAs take whole
// (row, SSM group) units, every warp keeps h = round(y) * silu(gate) of its rows for the
// group's heads in shared memory, and at the group's last head the warps' sums of squares meet
// through an mbarrier (a bounded wait) and each warp writes its rows of weight * round(h * rstd).
template <int PB, int NC, int COLD, bool IOBF, int PHASE, int CFIX, int RPWC, bool NORM = false>
__global__ void __launch_bounds__(kPT, PHASE == PH_STEP ? NSSM_STEP_P_MINB : NSSM_FLUSH_P_MINB)
    tiered_persistent_kernel(const __grid_constant__ PParams pp) {
  using Sh = StepShape<PB, NC, COLD>;
  constexpr int N = Sh::N;
  constexpr int LPR = Sh::LPR;     // hot 16-byte chunks per row
  constexpr int CPR = Sh::CPR;     // cold 16-byte chunks per row
  constexpr int CE = Sh::CE;       // cold elements per chunk
  constexpr int ESZ = Sh::ESZ;
  constexpr int kPerW = WordTraits<COLD>::kPer;
  constexpr int IOB = IOBF ? 2 : 4;
  constexpr bool STEP = PHASE == PH_STEP;
  constexpr int RPWMAX = RPWC > 0 ? RPWC : (kPMaxPersistent + kPW - 1) / kPW;   // rows per warp band
  constexpr int HQ = (RPWMAX * LPR + 31) / 32;                // hot chunks per lane
  constexpr int CQ = (RPWMAX * CPR + 31) / 32;                // cold chunks per lane (STEP)
  constexpr int CQF = (CPR + (32 / RPWMAX) - 1) / (32 / RPWMAX);   // column passes (FLUSH)
  // fp8 instances with a compile-time band of an even number of rows: a lane owns one cold
  // chunk column of two rows (rows rp and rp + RPWC/2 of the band), so the per-column data
  // (C'_cold in STEP, the ring's B'_cold in FLUSH) is read once for both rows; in FLUSH the
  // decay and the division by the new row scale are folded into one multiply each
  constexpr bool kPair = COLD == COLD_FP8 && RPWC > 0 && RPWC % 2 == 0 && (RPWC / 2) * CPR <= 32;
  constexpr int kHR = kPair ? RPWC / 2 : 1;
  static_assert(32 % LPR == 0, "hot row chunks must tile a warp");
  static_assert(COLD != COLD_NONE && NC > 0, "tiered instances only");
  static_assert(!NORM || PHASE == PH_STEP, "the norm is fused into STEP");
  static_assert(CE % 4 == 0 && PB % 4 == 0, "chunk shapes");

  const StepParams& p = pp.sp;
  const PLayout& L = pp.L;
  const int kStages = L.nst;
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int c = CFIX > 0 ? CFIX : p.c;
  const int Pn = RPWC > 0 ? kPW * RPWC : p.P;   // the RPWC instances run only for headdim == 8 * RPWC
  const int H = p.H;
  const int cp = ring_dt_stride(c);
  const int HG = H / p.G;
  const bool corr = (p.mode == NSSM_MODE_CORR);
  const bool ring_st = pp.ring_in_stage != 0 && (!STEP || corr);

  extern __shared__ __align__(128) unsigned char sm[];
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + L.off_bar);
  uint64_t* empty = full + L.nst;
  uint64_t* nbar = empty + L.nst;   // fused norm: the warps' sums of squares of a group
  const float* scal = reinterpret_cast<const float*>(sm + L.off_scal);
  float* sA = reinterpret_cast<float*>(sm + L.off_head);
  float* yh = reinterpret_cast<float*>(sm + L.off_yh);
  float* pc = reinterpret_cast<float*>(sm + L.off_pc);
  float* s_sc = reinterpret_cast<float*>(sm + L.off_sc);
  float* s_rcp = reinterpret_cast<float*>(sm + L.off_rcp);
  float* wsc = reinterpret_cast<float*>(sm + L.off_wsc) + warp * L.wsc_stride;   // per-warp scratch
  float* sW = reinterpret_cast<float*>(sm + L.off_sw);
  int* bslot = reinterpret_cast<int*>(sm + L.off_bslot);
  int* btn = reinterpret_cast<int*>(sm + L.off_bmeta);   // token count after this step
  int* bpos = reinterpret_cast<int*>(sm + L.off_bpos);   // ring position of this token, -(pos+1) if it flushes

  // FLUSH works on the rows at a chunk boundary only, numbered in batch order (every CTA
  // repeats the count from the token counts STEP wrote); their items are split evenly over
  // the grid, so a batch whose rows flush on different tokens (per-slot phases) spreads
  // each token's flushes over every SM.  Rows b0.. below are such compacted rows in FLUSH
  // and batch rows in STEP.  The count costs every CTA two loads per batch row (slot, then
  // its token count): two passes of 256 rows at B=448.
  const int batch = pp.items / H;
  auto flush_row = [&](int b, int& slot, int& tn) -> bool {
    slot = p.idx ? p.idx[b] : b;
    if (slot == p.pad || slot < 0 || slot >= p.S) return false;
    tn = p.t[(int64_t)slot * H];
    return tn > 0 && tn % c == 0;
  };
  int W = pp.items;
  if constexpr (!STEP) {
    int nfl = 0;
    for (int c0 = 0; c0 < batch; c0 += kPT) {
      int sl = -1, tn = 0;
      nfl += __syncthreads_count(c0 + tid < batch && flush_row(c0 + tid, sl, tn));
    }
    W = nfl * H;
  }
  int beg = (int)((long long)W * blockIdx.x / gridDim.x);
  int end = (int)((long long)W * (blockIdx.x + 1) / gridDim.x);
  if constexpr (NORM) {   // whole (row, group) units: a group's heads stay in one CTA
    const int U = W / HG;
    beg = (int)((long long)U * blockIdx.x / gridDim.x) * HG;
    end = (int)((long long)U * (blockIdx.x + 1) / gridDim.x) * HG;
  }
  if (beg >= end) return;
  const int b0 = beg / H;
  const int nb = (end - 1) / H - b0 + 1;
  const int nit = end - beg;

  // ---- prologue 1: slot and token count after this step of every row in range.  STEP
  // reads t and adds one; FLUSH takes the flushing rows numbered b0 .. b0 + nb - 1 (a
  // block-wide exclusive count by warp ballots).
  bool any = false;
  if constexpr (!STEP) {
    int* wcnt = reinterpret_cast<int*>(sm + L.off_pc);   // per-warp counts (pc is free here)
    int base = 0;
    for (int c0 = 0; c0 < batch && base < b0 + nb; c0 += kPT) {   // uniform over the CTA
      const int b = c0 + tid;
      int slot = -1, tn = 0;
      const bool f = b < batch && flush_row(b, slot, tn);
      const unsigned bal = __ballot_sync(0xffffffffu, f);
      if (lane == 0) wcnt[warp] = __popc(bal);
      __syncthreads();
      int pre = 0, tot = 0;
      for (int w = 0; w < kPW; ++w) {
        const int n = wcnt[w];
        pre += w < warp ? n : 0;
        tot += n;
      }
      if (f) {
        const int pos = base + pre + __popc(bal & ((1u << lane) - 1u));
        if (pos >= b0 && pos < b0 + nb) {
          bslot[pos - b0] = slot;
          btn[pos - b0] = tn;
          bpos[pos - b0] = -c;
        }
      }
      base += tot;
      __syncthreads();
    }
    any = true;
  }
  for (int j = tid; STEP && j < nb; j += kPT) {
    const int b = b0 + j;
    const int slot = p.idx ? p.idx[b] : b;
    int s = -1, tn = 0;
    if (slot != p.pad) {
      if (slot < 0 || slot >= p.S) {
        if (p.status) atomicOr(p.status, STATUS_BAD_SLOT);
      } else {
        const int hf = (j == 0) ? beg - b0 * H : 0;   // first head of row b owned here
        s = slot;
        tn = p.t[(int64_t)slot * H + hf] + 1;
      }
    }
    any |= s >= 0;
    bslot[j] = s;
    btn[j] = tn;
    const int ps = tn > 0 ? (tn - 1) % c : 0;
    bpos[j] = (ps == c - 1) ? -(ps + 1) : ps;
  }
  // nothing to do in this CTA's range (STEP: every row padded; FLUSH left above when no
  // row of the batch is at a chunk boundary -- c - 1 launches out of c in lockstep
  // batches): leave before any set-up
  if (!__syncthreads_or(any)) return;
  if (!STEP) {
    for (int h = tid; h < H; h += kPT) sA[h] = p.A[h];
  }
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kPW);
    }
    if (NORM) mbar_init(nbar, kPW);
    fence_mbar_init();
  }
  __syncthreads();

  // ---- prologue 2 (STEP): every item's scalars, in parallel
  if constexpr (STEP) {
    for (int it = tid; it < nit; it += kPT) {
      const int w = beg + it;
      const int b = w / H, h = w - (w / H) * H;
      const int slot = bslot[b - b0];
      if (slot < 0) continue;
      float d = ld_io(p.dt, (int64_t)b * p.dt_sb + (int64_t)h * p.dt_sh, p.dt_dtype);
      if (p.dt_bias) d += p.dt_bias[h];
      if (p.softplus) d = softplus_f(d);
      if (p.dt_min > 0.0f) d = fmaxf(d, p.dt_min);
      const float dA = d * p.A[h];
      const float gl = p.glog[(int64_t)slot * H + h];
      float* f = reinterpret_cast<float*>(sm + L.off_scal) + it * kScal;
      f[0] = d;
      f[1] = dA;
      f[2] = expf(dA);
      f[3] = expf(corr ? gl + dA : gl);   // corr reads G_t inclusive
      f[4] = gl;
      f[5] = p.D ? p.D[h] : 0.0f;
      f[6] = p.A[h];
    }
  }

  // ---- prologue 2 (FLUSH): every flushing item's suffix decays, in parallel (same
  // sequential order as the oracle: total and suffix sums accumulated j-wise)
  if constexpr (!STEP) {
    if (c <= kRingF32Max) {
      for (int it = tid; it < nit; it += kPT) {
        const int w = beg + it;
        const int b = w / H, h = w - (w / H) * H;
        const int slot = bslot[b - b0];
        if (slot < 0) continue;
        const float* rd = p.ring_dt + ((int64_t)slot * H + h) * cp;
        const float A_h = p.A[h];
        float dts[kRingF32Max];
#pragma unroll
        for (int j = 0; j < kRingF32Max; ++j) dts[j] = (j < c) ? rd[j] : 0.0f;
        float* fs = reinterpret_cast<float*>(sm + L.off_fsc) + it * (2 * c + 1);
        float tot = 0.0f;
#pragma unroll
        for (int j = 0; j < kRingF32Max; ++j)
          if (j < c) tot = tot + dts[j] * A_h;
        fs[2 * c] = expf(tot);
        float suf = 0.0f;
        fs[c - 1] = 1.0f;
        fs[2 * c - 1] = dts[c - 1];
#pragma unroll
        for (int j = kRingF32Max - 2; j >= 0; --j) {
          if (j <= c - 2) {
            suf = suf + dts[j + 1] * A_h;
            fs[j] = expf(suf);
            fs[c + j] = dts[j];
          }
        }
      }
    }
  }

  // item cursor over valid items: (b, h, group, head-in-group) advanced incrementally
  struct Cur { int b, h, g, hr; };
  auto first_valid = [&](Cur& q) {
    while (q.b * H + q.h < end && bslot[q.b - b0] < 0) { ++q.b; q.h = 0; q.g = 0; q.hr = 0; }
  };
  auto advance = [&](Cur& q) {
    ++q.h;
    if (++q.hr == HG) { q.hr = 0; ++q.g; }
    if (q.h == H) { q.h = 0; q.g = 0; q.hr = 0; ++q.b; }
    first_valid(q);
  };
  const int h_beg = beg - b0 * H;
  const Cur start{b0, h_beg, h_beg / HG, h_beg % HG};

  // ---- producer: bulk copies of item q into stage s (one thread).  `stuck` (failure
  // injection) announces 16 bytes more than the copies deliver, so that stage's phase
  // never completes and its waits run out.
  auto issue = [&](const Cur& q, int s, bool stuck = false) {
    const int j = q.b - b0, b = q.b, h = q.h, g = q.g;
    const int slot = bslot[j];
    const int64_t sh = (int64_t)slot * H + h;
    unsigned char* st = sm + s * L.stage_bytes;
    uint32_t bytes = (uint32_t)(Pn * NC * ESZ);
    if (COLD == COLD_FP8) bytes += Pn * 4;
    if (STEP) bytes += (uint32_t)(Pn * PB * 4 + Pn * IOB + 2 * N * IOB);
    if (ring_st) bytes += (uint32_t)(c * Pn * IOB + c * NC * 4 + cp * 4);
    if (NORM) bytes += (uint32_t)(Pn * IOB);
    mbar_expect_tx(&full[s], bytes + (stuck ? 16u : 0u));
    if (NORM)
      bulk_g2s(st + L.s_gate, static_cast<const char*>(p.ngate) + ((int64_t)b * p.ngate_sb + (int64_t)h * Pn) * IOB,
               Pn * IOB, &full[s]);
    bulk_g2s(st + L.s_cold, static_cast<const char*>(p.cold) + sh * Pn * NC * ESZ, Pn * NC * ESZ, &full[s]);
    if (COLD == COLD_FP8) bulk_g2s(st + L.s_scale, p.scale + sh * Pn, Pn * 4, &full[s]);
    if (STEP) {
      bulk_g2s(st + L.s_hot, p.hot + sh * Pn * PB, Pn * PB * 4, &full[s]);
      bulk_g2s(st + L.s_x, static_cast<const char*>(p.x) + ((int64_t)b * p.x_sb + (int64_t)h * p.x_sh) * IOB,
               Pn * IOB, &full[s]);
      bulk_g2s(st + L.s_b, static_cast<const char*>(p.B) + ((int64_t)b * p.B_sb + (int64_t)g * N) * IOB,
               N * IOB, &full[s]);
      bulk_g2s(st + L.s_c, static_cast<const char*>(p.C) + ((int64_t)b * p.C_sb + (int64_t)g * N) * IOB,
               N * IOB, &full[s]);
    }
    if (ring_st) {
      bulk_g2s(st + L.s_rx, static_cast<const char*>(p.ring_x) + sh * c * Pn * IOB, c * Pn * IOB, &full[s]);
      bulk_g2s(st + L.s_rb, p.ring_b + ((int64_t)slot * p.G + g) * c * NC, c * NC * 4, &full[s]);
      bulk_g2s(st + L.s_rdt, p.ring_dt + sh * cp, cp * 4, &full[s]);
    }
  };

  // ---- pipeline fill
  Cur pq = start;
  first_valid(pq);
  uint32_t n_issued = 0;
  const bool inject = STEP && pp.inject_stuck != 0 && blockIdx.x == 0;
  if (tid == 0) {
    for (int s = 0; s < kStages && pq.b * H + pq.h < end; ++s) {
      issue(pq, s, inject && s == 0);
      ++n_issued;
      advance(pq);
    }
  }
  __syncthreads();   // item scalars visible

  // this warp's band of headdim rows (compile-time when RPWC > 0: headdim == kPW * RPWC)
  const int rpw = RPWC > 0 ? RPWC : L.rpw;
  const int r0 = RPWC > 0 ? warp * RPWC : min(warp * rpw, Pn);
  const int nrow = RPWC > 0 ? RPWC : min(r0 + rpw, Pn) - r0;
  const int hcol = lane % LPR;
  const int nch = nrow * LPR;
  const int ncb = nrow * CPR;
  // FLUSH lane mapping: fcw chunk columns per pass, lane -> (row frr, column fcq)
  const int fcw = nrow > 0 ? 32 / nrow : 1;
  const int frr = nrow > 0 ? lane % nrow : 0;
  const int fcq = nrow > 0 ? lane / nrow : 0;
  const bool fok = nrow > 0 && fcq < fcw;
  bool ok = true;
  float nss = 0.0f;     // fused norm: this lane's row's sum of h^2 over the group's heads so far
  uint32_t npar = 0;    // fused norm: phase of nbar

  Cur q = start;
  first_valid(q);
  int s = 0;
  uint32_t par = 0;   // stage s / its phase parity for item k
  int s_prev = 0;
  uint32_t par_prev = 0;   // FLUSH: stage / parity of item k - 1 (released after item k)
  for (uint32_t k = 0; q.b * H + q.h < end; advance(q), ++k) {
    const int j0b = q.b - b0, b = q.b, h = q.h, g = q.g;
    const int slot = bslot[j0b], tnew = btn[j0b];
    const int64_t sh = (int64_t)slot * H + h;
    const unsigned char* st = sm + s * L.stage_bytes;
    // every lane waits on the stage's copies itself (acquire); the warp leaves together
    // if any lane's wait ran out, so no lane reaches the warp-wide shuffles alone
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(&full[s], par, pp.polls))) { ok = false; break; }
    const uint4* csm = reinterpret_cast<const uint4*>(st + L.s_cold);
    auto ring_x_at = [&](int j, int r) -> float {
      return ring_st ? ldv<IOBF>(st + L.s_rx, j * Pn + r) : ldv<IOBF>(p.ring_x, (sh * c + j) * Pn + r);
    };
    auto ring_dt_at = [&](int j) -> float {
      return ring_st ? reinterpret_cast<const float*>(st + L.s_rdt)[j] : p.ring_dt[sh * cp + j];
    };
    auto ring_b_at = [&](int j, int n) -> float {
      return ring_st ? reinterpret_cast<const float*>(st + L.s_rb)[j * NC + n]
                     : p.ring_b[(((int64_t)slot * p.G + g) * c + j) * NC + n];
    };

    if constexpr (STEP) {
      const int it = b * H + h - beg;
      const float* f = scal + it * kScal;
      const float dt = f[0], dA = f[1], decay = f[2], eglog = f[3], glraw = f[4], Dh = f[5], A_h = f[6];
      const int pcode = bpos[j0b];
      const bool flush = pcode < 0;
      const int pos = flush ? -pcode - 1 : pcode;
      const unsigned char* xr = st + L.s_x;
      const unsigned char* br = st + L.s_b;
      const unsigned char* cr = st + L.s_c;

      // ---- hot update of the band, written back to global; row sums of C.h
      {
        const float4* hs = reinterpret_cast<const float4*>(st + L.s_hot);
        float4* hg = reinterpret_cast<float4*>(p.hot + sh * Pn * PB);
        float bq[4], cq[4];
        ld_row<4, IOBF>(br, hcol * 4, bq);
        ld_row<4, IOBF>(cr, hcol * 4, cq);
        const float2 dtB01 = f2(dt * bq[0], dt * bq[1]), dtB23 = f2(dt * bq[2], dt * bq[3]);
        const float2 c01 = f2(cq[0], cq[1]), c23 = f2(cq[2], cq[3]);
        const float2 dec2 = f2(decay, decay);
#pragma unroll
        for (int u = 0; u < HQ; ++u) {
          if (u * 32 >= nch) break;   // uniform over the warp
          const int lc = u * 32 + lane;
          const int i = r0 * LPR + lc;
          float part = 0.0f;
          if (lc < nch) {
            const float xp = ldv<IOBF>(xr, i / LPR);
            const float2 x2 = f2(xp, xp);
            const float4 v = hs[i];
            const float2 a = __ffma2_rn(f2(v.x, v.y), dec2, __fmul2_rn(dtB01, x2));
            const float2 bb = __ffma2_rn(f2(v.z, v.w), dec2, __fmul2_rn(dtB23, x2));
            hg[i] = make_float4(a.x, a.y, bb.x, bb.y);
            const float2 pr = __ffma2_rn(a, c01, __fmul2_rn(bb, c23));
            part = pr.x + pr.y;
          }
#pragma unroll
          for (int o = 1; o < LPR; o <<= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
          if (hcol == 0 && lc < nch) yh[i / LPR] = part;
        }
      }
      // ---- stale cold readout of the band: per-chunk partials sum_e q[e] C[n]
      if constexpr (kPair) {
        // a lane owns one chunk column of two rows: C'_cold of the column is widened once
        const int rp = lane % kHR, cc = lane / kHR;
        if (p.mode != NSSM_MODE_COLDOFF && cc < CPR) {
          float cv[CE];
          ld_row<CE, IOBF>(cr, PB + cc * CE, cv);
#pragma unroll
          for (int hr = 0; hr < 2; ++hr) {
            const int i = (r0 + rp + hr * kHR) * CPR + cc;
            const uint4 q4 = csm[i];
            const uint32_t wv[4] = {q4.x, q4.y, q4.z, q4.w};
            float2 acc = f2(0.0f, 0.0f);
#pragma unroll
            for (int wi = 0; wi < 4; ++wi) {
              float qv[4];
              word_to_float<COLD>(wv[wi], qv);
              acc = __ffma2_rn(f2(qv[0], qv[1]), f2(cv[wi * 4], cv[wi * 4 + 1]), acc);
              acc = __ffma2_rn(f2(qv[2], qv[3]), f2(cv[wi * 4 + 2], cv[wi * 4 + 3]), acc);
            }
            pc[i] = acc.x + acc.y;
          }
        }
      } else if (p.mode != NSSM_MODE_COLDOFF) {
#pragma unroll
        for (int u = 0; u < CQ; ++u) {
          if (u * 32 >= ncb) break;
          const int lc = u * 32 + lane;
          if (lc < ncb) {
            const int i = r0 * CPR + lc;
            const int cc = i % CPR;
            float cv[CE];
            ld_row<CE, IOBF>(cr, PB + cc * CE, cv);
            const uint4 q4 = csm[i];
            const uint32_t wv[4] = {q4.x, q4.y, q4.z, q4.w};
            float2 acc = f2(0.0f, 0.0f);
#pragma unroll
            for (int wi = 0; wi < 4; ++wi) {
              float qv[kPerW];
              word_to_float<COLD>(wv[wi], qv);
              if constexpr (kPerW >= 2) {
#pragma unroll
                for (int e = 0; e < kPerW; e += 2)
                  acc = __ffma2_rn(f2(qv[e], qv[e + 1]), f2(cv[wi * kPerW + e], cv[wi * kPerW + e + 1]), acc);
              } else {
                acc.x = fmaf(qv[0], cv[wi], acc.x);
              }
            }
            pc[i] = acc.x + acc.y;
          }
        }
      }
      // ---- exact rank-c correction weights (mode corr), per warp:
      //      w_j = exp(G_t - G_j) (C_cold . B_j) for this chunk's tokens j <= t
      const int J = pos + 1;
      if (corr) {
        if (lane == 0) {
          float suf = 0.0f;
          wsc[J - 1] = 1.0f;
          wsc[c + J - 1] = dt;
          for (int j = J - 2; j >= 0; --j) {
            suf = suf + ((j + 1 == J - 1) ? dt : ring_dt_at(j + 1)) * A_h;
            wsc[j] = expf(suf);
            wsc[c + j] = ring_dt_at(j);
          }
        }
        __syncwarp();
        for (int j = 0; j < J; ++j) {
          float sd = 0.0f;
          for (int n = lane; n < NC; n += 32)
            sd = fmaf(ldv<IOBF>(cr, PB + n), (j == J - 1) ? ldv<IOBF>(br, PB + n) : ring_b_at(j, n), sd);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) sd += __shfl_xor_sync(0xffffffffu, sd, o);
          __syncwarp();
          if (lane == 0) wsc[j] = wsc[j] * sd;
        }
      }
      __syncwarp();

      // ---- y = C_hot.h + exp(glog) scale C_cold.cold (+ corr) + D x, one lane per row;
      //      this token into the ring at pos
      if (lane < nrow) {
        const int row = r0 + lane;
        const float xp = ldv<IOBF>(xr, row);
        float y = yh[row];
        if (p.mode != NSSM_MODE_COLDOFF) {
          float yc = 0.0f;
#pragma unroll
          for (int cc = 0; cc < CPR; ++cc) yc += pc[row * CPR + cc];
          const float scl = (COLD == COLD_FP8) ? reinterpret_cast<const float*>(st + L.s_scale)[row] : 1.0f;
          y += (yc * scl) * eglog;
        }
        if (corr) {
          float ycorr = 0.0f;
          for (int j = 0; j < J; ++j) {
            const float xj = (j == J - 1) ? xp : ring_x_at(j, row);
            ycorr = fmaf(wsc[j], wsc[c + j] * xj, ycorr);
          }
          y += ycorr;
        }
        if (p.D) y = fmaf(xp, Dh, y);
        if constexpr (NORM) {
          // h = round_out(y) * silu(gate), as the norm kernel computes it from the stored y
          const float yq = p.out_dtype == NSSM_BF16 ? __bfloat162float(__float2bfloat16_rn(y)) : y;
          const float z = ldv<IOBF>(st + L.s_gate, row);
          const float hv = yq * (z / (1.0f + expf(-z)));
          reinterpret_cast<float*>(sm + L.off_gbuf)[q.hr * Pn + row] = hv;
          nss = fmaf(hv, hv, nss);
        } else {
          st_io(p.out, (int64_t)b * p.out_sb + (int64_t)h * p.out_sh + row, p.out_dtype, y);
        }
        stv<IOBF>(p.ring_x, (sh * c + pos) * Pn + row, xp);
      }
      if constexpr (NORM) {
        if (q.hr == HG - 1) {   // the group's last head: rstd over its HG * P channels
          float ssw = nss;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) ssw += __shfl_xor_sync(0xffffffffu, ssw, o);
          float* nslot = reinterpret_cast<float*>(sm + L.off_nslot) + (npar ? kPW : 0);
          if (lane == 0) {
            nslot[warp] = ssw;
            mbar_arrive(nbar);
          }
          if (!__all_sync(0xffffffffu, mbar_wait_bounded(nbar, npar, pp.polls))) { ok = false; break; }
          float tot = 0.0f;
#pragma unroll
          for (int w2 = 0; w2 < kPW; ++w2) tot += nslot[w2];
          const float r = 1.0f / sqrtf(tot / (float)(HG * Pn) + p.neps);
          if (lane < nrow) {
            const int row = r0 + lane;
            const float* gb = reinterpret_cast<const float*>(sm + L.off_gbuf);
            for (int hr = 0; hr < HG; ++hr) {
              const int hh = g * HG + hr;
              const float hv = gb[hr * Pn + row] * r;
              const float hn = p.out_dtype == NSSM_BF16 ? __bfloat162float(__float2bfloat16_rn(hv)) : hv;
              const float wv = ld_io(p.nweight, (int64_t)hh * Pn + row, p.nweight_dtype);
              st_io(p.out, (int64_t)b * p.out_sb + (int64_t)hh * p.out_sh + row, p.out_dtype, wv * hn);
            }
          }
          nss = 0.0f;
          npar ^= 1u;
        }
      }
      if (q.hr == 0) {   // the group's B_cold, once per group, spread over the warps
        for (int n = tid; n < NC; n += kPT)
          p.ring_b[(((int64_t)slot * p.G + g) * c + pos) * NC + n] = ldv<IOBF>(br, PB + n);
      }
      if (tid == 0) {
        p.ring_dt[sh * cp + pos] = dt;
        p.glog[sh] = flush ? 0.0f : glraw + dA;   // the FLUSH phase re-bases the cold slice
        p.t[sh] = tnew;
      }
    } else {
      // ---- FLUSH of the band: cold <- exp(sum dA) cold + sum_j exp(suf_j) (dt_j x_j) B_j,
      // requantised; the ring holds all c tokens of the chunk.  acc = sum_j (W_j * B_j[n])
      // in j order as the oracle; fp8 scale = amax/448 + 1e-12 exactly as the oracle.  The
      // general instances also follow the oracle's v = (q * scale) * exp(tot) + acc and
      // q = rne(v / scale) (correctly rounded division); the paired fp8 instances fold
      // each into one multiply (below), which moves a stored code by one step, rarely.
      const float A_h = sA[h];
      const bool pre = c <= kRingF32Max;
      // exp(suf_j) [c], dt_j [c], exp(total): the prologue's table, or computed per warp
      const float* dec = pre ? reinterpret_cast<const float*>(sm + L.off_fsc) + (b * H + h - beg) * (2 * c + 1)
                             : wsc;
      if (!pre) {   // suffix decays (per warp; identical in every warp)
        // the c dts loaded by all lanes at once, the sums in j order by one lane, the
        // exponentials by all lanes again
        for (int j = lane; j < c; j += 32) wsc[c + j] = ring_dt_at(j);
        __syncwarp();
        if (lane == 0) {
          float tot = 0.0f;
          for (int j = 0; j < c; ++j) tot = tot + wsc[c + j] * A_h;
          wsc[2 * c] = expf(tot);
          float suf = 0.0f;
          for (int j = c - 2; j >= 0; --j) {
            suf = suf + wsc[c + j + 1] * A_h;
            wsc[j] = suf;
          }
        }
        __syncwarp();
        for (int j = lane; j < c - 1; j += 32) wsc[j] = expf(wsc[j]);
        if (lane == 0) wsc[c - 1] = 1.0f;
        __syncwarp();
      }
      // W_j[row] = exp(suf_j) * (dt_j * x_j[row]) for the band's rows; past kRingF32Max tokens
      // every (j, row) pair of the band goes over the lanes, so the ring loads are independent
      if (pre) {
        for (int j = 0; j < c; ++j) {
          if (lane < nrow) sW[j * Pn + r0 + lane] = __fmul_rn(dec[j], __fmul_rn(dec[c + j], ring_x_at(j, r0 + lane)));
        }
      } else {
        for (int i = lane; i < c * nrow; i += 32) {
          const int j = i / nrow, r = r0 + (i - j * nrow);
          sW[j * Pn + r] = __fmul_rn(dec[j], __fmul_rn(dec[c + j], ring_x_at(j, r)));
        }
      }
      __syncwarp();
      const float etot = dec[2 * c];
      const float* scl_s = reinterpret_cast<const float*>(st + L.s_scale);
      const float* rbp = ring_st ? reinterpret_cast<const float*>(st + L.s_rb)
                                 : p.ring_b + ((int64_t)slot * p.G + g) * c * NC;
      uint4* cst = reinterpret_cast<uint4*>(sm + s * L.stage_bytes + L.s_cold);   // requantised in place
      if constexpr (kPair) {
        // lane -> chunk column cc of rows rA = r0 + rp and rB = rA + RPWC/2: each B_j chunk
        // read from shared memory serves both rows
        const int rp = lane % kHR, cc = lane / kHR;
        const bool act = cc < CPR;
        const int rA = r0 + rp, rB = rA + kHR;
        float va[CE], vb[CE];
#pragma unroll
        for (int e = 0; e < CE; ++e) { va[e] = 0.0f; vb[e] = 0.0f; }
        if (act) {
#pragma unroll
          for (int j = 0; j < CFIX; ++j) {
            const float wa = sW[j * Pn + rA], wb = sW[j * Pn + rB];
            const float2 wa2 = f2(wa, wa), wb2 = f2(wb, wb);
            const float4* b4 = reinterpret_cast<const float4*>(rbp + j * NC + cc * CE);
#pragma unroll
            for (int e = 0; e < CE / 4; ++e) {
              const float4 bv = b4[e];
              const float2 lo = f2(bv.x, bv.y), hi = f2(bv.z, bv.w);
              float2 t = __ffma2_rn(wa2, lo, f2(va[4 * e], va[4 * e + 1]));
              va[4 * e] = t.x; va[4 * e + 1] = t.y;
              t = __ffma2_rn(wa2, hi, f2(va[4 * e + 2], va[4 * e + 3]));
              va[4 * e + 2] = t.x; va[4 * e + 3] = t.y;
              t = __ffma2_rn(wb2, lo, f2(vb[4 * e], vb[4 * e + 1]));
              vb[4 * e] = t.x; vb[4 * e + 1] = t.y;
              t = __ffma2_rn(wb2, hi, f2(vb[4 * e + 2], vb[4 * e + 3]));
              vb[4 * e + 2] = t.x; vb[4 * e + 3] = t.y;
            }
          }
        }
        // v = q * (scale * exp(tot)) + acc, one fused multiply-add per element (the
        // oracle rounds q * scale and the decay product separately: the two differ by an
        // fp32 ulp, which moves a stored fp8 code by one step in rare cases)
        const float sa = scl_s[rA], sb = scl_s[rB];
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          float* v = hr ? vb : va;
          const int row = hr ? rB : rA;
          const uint4 q4 = act ? csm[row * CPR + cc] : make_uint4(0u, 0u, 0u, 0u);
          const uint32_t wv[4] = {q4.x, q4.y, q4.z, q4.w};
          const float se = __fmul_rn(hr ? sb : sa, etot);
          const float2 se2 = f2(se, se);
          float m = 0.0f;
#pragma unroll
          for (int wi = 0; wi < 4; ++wi) {
            float qv[4];
            word_to_float<COLD>(wv[wi], qv);
#pragma unroll
            for (int e = 0; e < 4; e += 2) {
              const int x = wi * 4 + e;
              const float2 r2 = __ffma2_rn(f2(qv[e], qv[e + 1]), se2, f2(v[x], v[x + 1]));
              v[x] = r2.x;
              v[x + 1] = r2.y;
            }
          }
#pragma unroll
          for (int e = 0; e < CE; ++e) m = fmaxf(m, fabsf(v[e]));
          if (act) pc[row * CPR + cc] = m;
        }
        __syncwarp();
        if (lane < nrow) {
          const int row = r0 + lane;
          float m = 0.0f;
#pragma unroll
          for (int k = 0; k < CPR; ++k) m = fmaxf(m, pc[row * CPR + k]);
          const float sc = __fadd_rn(scale_div448(m), kScaleEps);
          s_sc[row] = sc;
          s_rcp[row] = __frcp_rn(sc);
          p.scale[sh * Pn + row] = sc;
        }
        __syncwarp();
        if (act) {
#pragma unroll
          for (int hr = 0; hr < 2; ++hr) {
            float* v = hr ? vb : va;
            const int row = hr ? rB : rA;
            // v * rn(1 / scale): within an fp32 ulp of v / scale, so a stored code can
            // differ by one step from the correctly rounded quotient's, rarely
            const float2 r2 = f2(s_rcp[row], s_rcp[row]);
#pragma unroll
            for (int e = 0; e < CE; e += 2) {
              const float2 qq = __fmul2_rn(f2(v[e], v[e + 1]), r2);
              v[e] = qq.x;
              v[e + 1] = qq.y;
            }
            uint32_t wq[4];
            float_to_cold<COLD, CE>(v, wq);
            cst[row * CPR + cc] = make_uint4(wq[0], wq[1], wq[2], wq[3]);
          }
        }
      } else {
        // lane -> (row frr of the band, chunk column u*fcw + fcq): the 8 lanes of a
        // shared-memory phase share a chunk column, so B_j reads are broadcasts
        float v[CQF][CE];
  #pragma unroll
        for (int u = 0; u < CQF; ++u) {
          if (u * fcw >= CPR) break;   // uniform
          const int cc0 = u * fcw + fcq;
          const bool act = fok && cc0 < CPR;
          const int cc = act ? cc0 : 0;
          const int row = r0 + (fok ? frr : 0);
          const int i = row * CPR + cc;
  #pragma unroll
          for (int e = 0; e < CE; ++e) v[u][e] = 0.0f;
  #pragma unroll 4
          for (int j = 0; j < c; ++j) {
            const float Wv = sW[j * Pn + row];
            const float2 W2 = f2(Wv, Wv);
            const float4* b4 = reinterpret_cast<const float4*>(rbp + j * NC + cc * CE);
  #pragma unroll
            for (int e = 0; e < CE / 4; ++e) {
              const float4 bv = b4[e];
              const float2 lo = __ffma2_rn(W2, f2(bv.x, bv.y), f2(v[u][4 * e], v[u][4 * e + 1]));
              const float2 hi = __ffma2_rn(W2, f2(bv.z, bv.w), f2(v[u][4 * e + 2], v[u][4 * e + 3]));
              v[u][4 * e] = lo.x; v[u][4 * e + 1] = lo.y; v[u][4 * e + 2] = hi.x; v[u][4 * e + 3] = hi.y;
            }
          }
          const float scl = (COLD == COLD_FP8) ? scl_s[row] : 1.0f;
          const uint4 q4 = csm[i];
          const uint32_t wv[4] = {q4.x, q4.y, q4.z, q4.w};
          const float2 e2 = f2(etot, etot), s2 = f2(scl, scl);
          float m = 0.0f;
  #pragma unroll
          for (int wi = 0; wi < 4; ++wi) {
            float qv[kPerW];
            word_to_float<COLD>(wv[wi], qv);
            if constexpr (kPerW >= 2) {
  #pragma unroll
              for (int e = 0; e < kPerW; e += 2) {
                const int x = wi * kPerW + e;
                float2 dq = f2(qv[e], qv[e + 1]);
                if constexpr (COLD == COLD_FP8) dq = __fmul2_rn(dq, s2);
                const float2 r2 = __fadd2_rn(__fmul2_rn(dq, e2), f2(v[u][x], v[u][x + 1]));
                v[u][x] = r2.x;
                v[u][x + 1] = r2.y;
              }
            } else {
              v[u][wi] = __fadd_rn(__fmul_rn(qv[0], etot), v[u][wi]);
            }
          }
  #pragma unroll
          for (int e = 0; e < CE; ++e) m = fmaxf(m, fabsf(v[u][e]));
          if (COLD == COLD_FP8 && act) pc[i] = m;
        }
        if constexpr (COLD == COLD_FP8) {
          __syncwarp();
          if (lane < nrow) {
            const int row = r0 + lane;
            float m = 0.0f;
  #pragma unroll
            for (int cc = 0; cc < CPR; ++cc) m = fmaxf(m, pc[row * CPR + cc]);
            const float sc = __fadd_rn(scale_div448(m), kScaleEps);
            s_sc[row] = sc;
            s_rcp[row] = __frcp_rn(sc);
            p.scale[sh * Pn + row] = sc;
          }
          __syncwarp();
        }
  #pragma unroll
        for (int u = 0; u < CQF; ++u) {
          if (u * fcw >= CPR) break;
          const int cc0 = u * fcw + fcq;
          if (fok && cc0 < CPR) {
            const int row = r0 + frr;
            if constexpr (COLD == COLD_FP8) {
              // correctly rounded v / scale, two lanes at a time (Markstein's correction)
              const float2 r2 = f2(s_rcp[row], s_rcp[row]);
              const float2 nsc2 = f2(-s_sc[row], -s_sc[row]);
  #pragma unroll
              for (int e = 0; e < CE; e += 2) {
                const float2 a = f2(v[u][e], v[u][e + 1]);
                const float2 q0 = __fmul2_rn(a, r2);
                const float2 rs = __ffma2_rn(q0, nsc2, a);
                const float2 qq = __ffma2_rn(rs, r2, q0);
                v[u][e] = qq.x;
                v[u][e + 1] = qq.y;
              }
            }
            uint32_t wq[4];
            float_to_cold<COLD, CE>(v[u], wq);
            cst[row * CPR + cc0] = make_uint4(wq[0], wq[1], wq[2], wq[3]);
          }
        }
      }
      // the band's requantised rows -> global in one bulk store
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && nrow > 0) {
        bulk_s2g(static_cast<char*>(p.cold) + (sh * Pn + r0) * NC * ESZ, cst + r0 * CPR,
                 (uint32_t)(nrow * NC * ESZ));
        bulk_commit();
      }
    }

    // ---- release a stage once this warp's bulk store has read it; the producer refills
    // it once every warp has.  STEP releases the stage it just used.  FLUSH releases the
    // previous item's stage, so the bulk store of a band overlaps the next item's work.
    // The producer (thread 0) waits for the stage to empty; its verdict is broadcast to
    // warp 0 so that the whole warp leaves together when that wait runs out.
    __syncwarp();
    bool prod_fail = false;
    if constexpr (STEP) {
      if (lane == 0) {
        bulk_wait_read_all();
        mbar_arrive(&empty[s]);
      }
      if (tid == 0 && pq.b * H + pq.h < end) {
        if (!mbar_wait_bounded(&empty[s], par, pp.polls)) {
          prod_fail = true;
        } else {
          fence_proxy_async_smem();
          issue(pq, s);
          ++n_issued;
          advance(pq);
        }
      }
    } else {
      if (k > 0) {
        if (lane == 0) {
          bulk_wait_read_1();
          mbar_arrive(&empty[s_prev]);
        }
        if (tid == 0 && pq.b * H + pq.h < end) {
          if (!mbar_wait_bounded(&empty[s_prev], par_prev, pp.polls)) {
            prod_fail = true;
          } else {
            fence_proxy_async_smem();
            issue(pq, s_prev);
            ++n_issued;
            advance(pq);
          }
        }
      }
      s_prev = s;
      par_prev = par;
    }
    if (warp == 0 && __shfl_sync(0xffffffffu, prod_fail, 0)) { ok = false; break; }
    if (++s == kStages) { s = 0; par ^= 1u; }
  }
  if (lane == 0) bulk_wait_all();   // this warp's bulk stores are complete before exit
  if (!ok) {
    if (lane == 0 && p.status) atomicOr(p.status, STATUS_TIMEOUT);
    if (tid == 0) {
      // a wait ran out: keep the CTA (and its shared memory) alive until the copies it
      // issued have landed.  Item n went to stage n % kStages as that stage's phase
      // n / kStages; only the last kStages items can still be in flight, and each is the
      // latest phase of its stage, so its parity identifies it (bounded again, with the
      // default poll count; the injected stuck phase, whose copies have all landed, with the
      // caller's).
      const uint32_t first = n_issued > (uint32_t)kStages ? n_issued - (uint32_t)kStages : 0u;
      for (uint32_t qn = first; qn < n_issued; ++qn)
        mbar_wait_bounded(&full[qn % kStages], (qn / kStages) & 1u, (inject && qn == 0) ? pp.polls : kSpinLimit);
    }
  }
}

}  // namespace nssm
