// Prefill chunked scan (SSD) on the 5th-generation tensor cores, warp-specialised.
//
// Work item = one (sequence, head); a persistent CTA walks items blockIdx.x, +gridDim.x, ...
// and each item's chunks of kQ = 128 tokens in order, as one stream of iterations.  Per
// chunk, with cs = cumsum(dt * A) inside the chunk (the published algorithm of mamba_ssm
// 2.3.2.post1 mamba_chunk_scan_combined, which the reference's lean prefill calls at
// scale/v4_native_decode.py:209-216):
//
//   MMA1  CB[l][s]    = sum_n C[l][n] B[s][n]                       M=128 N=128 K=128
//   MMA3  Yoff[l][p]  = sum_n C[l][n] Sprev[p][n]   (Sprev: bf16)   M=128 N=P   K=128
//   A     M[l][s] = bf16((CB * exp(cs_l - cs_s)) * dt_s) for s <= l, else 0;
//         B in place -> bf16(B[s][n] * exp(cs_last - cs_s) * dt_s)
//   MMA4  S[n][p]    += sum_s Bs[s][n] x[s][p]                      M=128 N=P   K=128
//   MMA2  Ydiag[l][p] = sum_s M[l][s] x[s][p]                       M=128 N=P   K=128
//   E     S (fp32, tensor memory) <- exp(cs_last) S before MMA4 accumulates into it;
//         Sprev = bf16(S); y = Yoff * exp(cs_l) + Ydiag + D x
//
// Warp roles (18 warps):
//   warp 0      producer: dt, softplus, clamp, in-chunk cumsum and the decay vectors of the
//               chunk (all lanes), then TMA tile loads of C, B, x into a two-slot stage ring.
//   warp 1      MMA issuer (one lane) and tensor-memory owner.
//   warps 2-9   A: the masked, decayed C.B tile M and the scaled B (two warps per TMEM
//               lane quadrant, one half of the columns each).
//   warps 10-17 E: state update and y epilogue (two warps per quadrant, each a share of
//               the 16-column blocks of P).
// Only the state crosses chunks, so chunk c+1's loads, MMA1 and A work run while E finishes
// chunk c; C.B^T is double-buffered in tensor memory so MMA1(c+1) runs while A reads chunk c's.
// Every hand-off is an mbarrier (tcgen05.commit for MMA completion, plain arrives for
// warps) and every wait is bounded: on timeout the CTA raises an abort flag that all roles
// poll, records STATUS_TIMEOUT and exits after freeing its tensor memory.
//
// Shared-memory operand layouts (16-byte chunk = 8 bf16 of a row):
//   C, B tile: two TMA boxes {64 n, 128 t} with 128-byte swizzle, [n half][t][128 B]: K-major
//       for MMA1 / MMA3 (8-row groups 1024 B, K steps +32 B, second half +16 KB); the scaled B
//       is also the MN-major A operand of MMA4 (M = n: halves 16 KB apart, K = t groups 1024 B).
//   X tile: P/16 boxes {16 p, 128 s} with 32-byte swizzle, [p group][s][32 B]: MN-major B
//       operand of MMA2 / MMA4 (16-column groups 4 KB apart, K groups of 8 rows 256 B).
//   M tile [16 chunks][128 rows l][16 B], no swizzle: K-major A operand of MMA2 (rows 16 B,
//       8-row groups 128 B, K chunks 2048 B).
//   Sprev [P/8 chunks][128 rows n][16 B], no swizzle: MN-major B operand of MMA3.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "nssm_persistent.cuh"
#include "nssm_tc.cuh"

namespace nssm {
namespace scan {

constexpr int kQ = 128;        // tokens per chunk
constexpr int kN = 128;        // d_state
constexpr int kWarps = 18;
constexpr int kThreads = kWarps * 32;
constexpr int kWA0 = 2, kWE0 = 10;       // first A warp, first E warp
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColCB0 = 0, kColCB1 = 128, kColYd = 256, kColS = 336, kColYo = 416;
constexpr int kOp = kQ * kN * 2;   // bytes of a 128 x 128 bf16 tile

struct ScanParams {
  int batch, T, H, G;
  const __nv_bfloat16* x;   // read by the epilogue for D x (the MMAs take x through TMA)
  int64_t x_sb, x_st;
  const void* dt;
  int64_t dt_sb, dt_st;
  int dt_bf16, softplus;
  float dt_lo, dt_hi;
  const float* A;
  const float* D;
  const float* dt_bias;
  const float* init;
  int64_t init_sb;
  __nv_bfloat16* y;
  int64_t y_sb, y_st;
  float* fin;
  int64_t fin_sb;
  int32_t* status;
};

constexpr int kVSlots = 3;                       // chunk vectors ring (dt, cs, fst, eoff, eT)
constexpr int kVBytes = 4 * kQ * 4 + 32;

template <int P>
struct Smem {
  static constexpr int kX = kQ * P * 2;                       // X: P/16 tiles of [128 s][16 p]
  static constexpr int kStage = 2 * kOp + kX;                 // C | B | X tiles of one chunk
  static constexpr int kM = 2 * kStage;
  static constexpr int kSp = kM + kOp;
  static constexpr int kVec = kSp + kN * P * 2;
  static constexpr int kBar = kVec + kVSlots * kVBytes;
  static constexpr int kBytes = kBar + 256;
  static constexpr uint32_t kTx = kStage;                     // TMA bytes per stage
  static_assert(kStage % 1024 == 0, "stage must keep 1 KB alignment");
};

// mbarrier slots (8 bytes each) at Smem::kBar
enum : int {
  B_FULL0 = 0, B_FULL1, B_EMPTY0, B_EMPTY1, B_CBFULL0, B_CBFULL1, B_CBFREE0, B_CBFREE1, B_MFULL, B_MFREE,
  B_SFULL, B_YFULL, B_SREADY, B_YDFREE, B_SPFULL, B_YOFREE, B_VFULL0, B_VFULL1, B_VFULL2, B_VEMPTY0,
  B_VEMPTY1, B_VEMPTY2, B_COUNT
};

// tcgen05 primitives (descriptors, MMA issue, commit, fences, tensor-memory loads): nssm_tc.cuh

// 3-D tiled TMA load global -> this CTA's shared memory (no multicast), completing on `bar`
__device__ __forceinline__ void tma_load3(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}
// descriptor layout types (bits 61-63)
constexpr uint64_t kSw128 = 2ull << 61, kSw32 = 6ull << 61;

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ float2 unpack_bf16(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}

// try_wait that lets the thread sleep up to 1 ms for the phase (instead of spinning and taking
// issue slots from the working warps); true once the phase with `parity` has completed
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
      : "memory");
  return ok != 0;
}
constexpr uint32_t kWaitTries = 4000;   // at most ~4 s per wait

// Bounded wait that also gives up once another role has raised the abort flag.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t par, volatile int* abort_flag) {
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait_sleep(bar, par)) return true;
    if (*abort_flag) return false;
    if (it >= kWaitTries) {
      *abort_flag = 1;
      return false;
    }
  }
}

// The same wait taken by every lane (each observes the phase, so the data it guards is
// visible to each), with one outcome for the whole warp so a warp never splits on it.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t par, volatile int* abort_flag) {
  const bool ok = wait_bar(bar, par, abort_flag);
  return __all_sync(0xffffffffu, ok);
}

// 2^x, flushing subnormal results to zero (one MUFU op)
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float load_dt(const ScanParams& p, int b, int t, int h) {
  const int64_t i = (int64_t)b * p.dt_sb + (int64_t)t * p.dt_st + h;
  return p.dt_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.dt)[i])
                   : reinterpret_cast<const float*>(p.dt)[i];
}

template <int P>
__global__ void __launch_bounds__(kThreads, 1)
    chunk_scan_kernel(const ScanParams p, const __grid_constant__ CUtensorMap tmC,
                      const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmX) {
  static_assert(P % 16 == 0 && P >= 32 && P <= 80, "headdim must be a multiple of 16 in [32, 80]");
  using L = Smem<P>;
  extern __shared__ __align__(1024) unsigned char smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + L::kBar + 8 * B_COUNT);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + L::kBar + 8 * B_COUNT + 4);
  const uint32_t sbase = smem_u32(smem);

  const int n_items = p.batch * p.H;
  const int nch = (p.T + kQ - 1) / kQ;
  const int my_items = blockIdx.x < n_items ? (n_items - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int total = my_items * nch;   // iterations of this CTA's stream
  const bool have_init = p.init != nullptr;

  if (tid == 0) {
    mbar_init(&bar[B_FULL0], 1);
    mbar_init(&bar[B_FULL1], 1);
    mbar_init(&bar[B_EMPTY0], 1);
    mbar_init(&bar[B_EMPTY1], 1);
    mbar_init(&bar[B_CBFULL0], 1);
    mbar_init(&bar[B_CBFULL1], 1);
    mbar_init(&bar[B_CBFREE0], 8);
    mbar_init(&bar[B_CBFREE1], 8);
    mbar_init(&bar[B_MFULL], 8);
    mbar_init(&bar[B_MFREE], 1);
    mbar_init(&bar[B_SFULL], 1);
    mbar_init(&bar[B_YFULL], 1);
    mbar_init(&bar[B_SREADY], 8);
    mbar_init(&bar[B_YDFREE], 8);
    mbar_init(&bar[B_SPFULL], 8);
    mbar_init(&bar[B_YOFREE], 8);
    for (int v = 0; v < kVSlots; ++v) {
      mbar_init(&bar[B_VFULL0 + v], 1);
      mbar_init(&bar[B_VEMPTY0 + v], 16);   // 8 A warps + 8 E warps
    }
    *s_abort = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(s_tmem)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }

  // E role: state rows n = erow (TMEM lane), 16-column blocks [eb0, eb0 + enb) of P (blocks
  // split between the two warps of a quadrant so every TMEM access is 16-column aligned).  The
  // running state lives in tensor memory (columns kColS): before chunk c's MMA4 the epilogue
  // scales it by exp(cs_last) of chunk c (or sets it to that times the initial state at an
  // item's first chunk), and MMA4 accumulates sum_s Bs[s][n] x[s][p] on top.
  constexpr int NB = P / 16, NB0 = (NB + 1) / 2, NB1 = NB - NB0;
  const bool is_e = warp >= kWE0;
  const int eq = warp & 3, ehalf = (warp - kWE0) >> 2;
  const int erow = 32 * eq + lane;
  const int eb0 = ehalf ? NB0 : 0, enb = ehalf ? NB1 : NB0;
  auto item_bh = [&](int k, int& b, int& h) {
    const int item = (int)blockIdx.x + k * (int)gridDim.x;
    b = item / p.H;
    h = item - b * p.H;
  };
  // 16 values of the initial state of this CTA's item k, row erow, columns 16*blk .. +15
  auto init_block = [&](int k, int blk, float* v) {
    int b, h;
    item_bh(k, b, h);
    const float* src = p.init + (int64_t)b * p.init_sb + ((int64_t)h * P + 16 * blk) * kN + erow;
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = src[(int64_t)i * kN];
  };
  auto sp_block = [&](int blk, const float* v) {   // bf16 of 16 state columns -> MMA3 operand
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      uint4 w;
      w.x = pack_bf16(v[8 * hh + 0], v[8 * hh + 1]);
      w.y = pack_bf16(v[8 * hh + 2], v[8 * hh + 3]);
      w.z = pack_bf16(v[8 * hh + 4], v[8 * hh + 5]);
      w.w = pack_bf16(v[8 * hh + 6], v[8 * hh + 7]);
      *reinterpret_cast<uint4*>(smem + L::kSp + (2 * blk + hh) * 2048 + erow * 16) = w;
    }
  };
  if (is_e && my_items > 0 && have_init) {
#pragma unroll
    for (int kb = 0; kb < NB0; ++kb)
      if (kb < enb) {
        float v[16];
        init_block(0, eb0 + kb, v);
        sp_block(eb0 + kb, v);
      }
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    for (int it = 0; it < total; ++it) {
      const int s = it & 1, vs = it % kVSlots;
      const int k = it / nch, c = it - k * nch;
      int b, h;
      item_bh(k, b, h);
      // the chunk's vectors first: they do not wait for the stage
      if (it >= kVSlots && !warp_wait(&bar[B_VEMPTY0 + vs], (uint32_t)((it / kVSlots - 1) & 1), s_abort)) break;
      float* v_dt = reinterpret_cast<float*>(smem + L::kVec + vs * kVBytes);
      float* v_cs = v_dt + kQ;
      float* v_fst = v_cs + kQ;
      float* v_eoff = v_fst + kQ;
      float* v_eT = v_eoff + kQ;
      const int t0 = c * kQ;
      const float A_h = p.A[h];
      const float bias = p.dt_bias ? p.dt_bias[h] : 0.0f;
      float d[4], cs[4];
      float run = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int t = t0 + 4 * lane + j;
        float v = 0.0f;
        if (t < p.T) {
          v = load_dt(p, b, t, h) + bias;
          if (p.softplus) v = softplus_f(v);
          v = fminf(fmaxf(v, p.dt_lo), p.dt_hi);
        }
        d[j] = v;
        run += v * A_h;
        cs[j] = run;
      }
      float inc = run;   // inclusive scan of the lane totals
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const float u = __shfl_up_sync(0xffffffffu, inc, off);
        if (lane >= off) inc += u;
      }
      const float base = inc - run;
#pragma unroll
      for (int j = 0; j < 4; ++j) cs[j] += base;
      // exponentials in base 2 of log2(e)-scaled cumsums (v_cs holds cs * log2 e)
#pragma unroll
      for (int j = 0; j < 4; ++j) cs[j] *= kLog2e;
      const float last = __shfl_sync(0xffffffffu, cs[3], 31);
      *reinterpret_cast<float4*>(v_dt + 4 * lane) = make_float4(d[0], d[1], d[2], d[3]);
      *reinterpret_cast<float4*>(v_cs + 4 * lane) = make_float4(cs[0], cs[1], cs[2], cs[3]);
      *reinterpret_cast<float4*>(v_fst + 4 * lane) =
          make_float4(ex2_ftz(last - cs[0]) * d[0], ex2_ftz(last - cs[1]) * d[1], ex2_ftz(last - cs[2]) * d[2],
                      ex2_ftz(last - cs[3]) * d[3]);
      *reinterpret_cast<float4*>(v_eoff + 4 * lane) =
          make_float4(ex2_ftz(cs[0]), ex2_ftz(cs[1]), ex2_ftz(cs[2]), ex2_ftz(cs[3]));
      if (lane == 0) *v_eT = ex2_ftz(last);
      __threadfence_block();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[B_VFULL0 + vs]);
      // then the tiles, once the stage's previous chunk has left the tensor cores
      if (it >= 2 && !warp_wait(&bar[B_EMPTY0 + s], (uint32_t)(((it >> 1) - 1) & 1), s_abort)) break;
      if (lane == 0) {
        const uint32_t st = sbase + s * L::kStage;
        const int g = h / (p.H / p.G);
        mbar_expect_tx(&bar[B_FULL0 + s], L::kTx);
        tma_load3(st, &tmC, kN * g, t0, b, &bar[B_FULL0 + s]);
        tma_load3(st + kOp / 2, &tmC, kN * g + 64, t0, b, &bar[B_FULL0 + s]);
        tma_load3(st + kOp, &tmB, kN * g, t0, b, &bar[B_FULL0 + s]);
        tma_load3(st + kOp + kOp / 2, &tmB, kN * g + 64, t0, b, &bar[B_FULL0 + s]);
#pragma unroll
        for (int j = 0; j < P / 16; ++j) tma_load3(st + 2 * kOp + 4096 * j, &tmX, P * h + 16 * j, t0, b, &bar[B_FULL0 + s]);
      }
      __syncwarp();
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdCB = idesc_bf16(128, 128, 0, 0);
      constexpr uint32_t kIdY = idesc_bf16(128, P, 0, 1);
      constexpr uint32_t kIdS = idesc_bf16(128, P, 1, 1);
      // x tile: MN-major with 32-byte swizzle, 16-column groups 4096 B apart (LBO), K groups of
      // 8 token rows 256 B apart (SBO); 16 K rows per MMA
      auto xdesc = [&](uint32_t st, int kk) { return sdesc(st + 2 * kOp + 512 * kk, 4096, 256) | kSw32; };
      // C and B: K-major, 128-byte swizzle (8-row groups 1024 B), two 64-column halves 16 KB
      // apart; K steps of 16 columns are +32 B inside a half
      auto kdesc = [&](uint32_t base, int kk) {
        return sdesc(base + (kk >> 2) * (kOp / 2) + (kk & 3) * 32, 16, 1024) | kSw128;
      };
      const uint32_t sM = sbase + L::kM, sSp = sbase + L::kSp;
      // C.B^T of chunk it into CB buffer it & 1 (both tensor-memory CB buffers let chunk it+1's
      // MMA1 run while the A warps still read chunk it's)
      auto issue_cb = [&](int it) -> bool {
        const int s = it & 1;
        const uint32_t st = sbase + s * L::kStage;
        if (!wait_bar(&bar[B_FULL0 + s], (uint32_t)((it >> 1) & 1), s_abort)) return false;
        if (it >= 2 && !wait_bar(&bar[B_CBFREE0 + s], (uint32_t)(((it >> 1) - 1) & 1), s_abort)) return false;
        tc_fence_after();
        const uint32_t cb = s ? kColCB1 : kColCB0;
#pragma unroll 1
        for (int kk = 0; kk < 8; ++kk) umma(tmem + cb, kdesc(st, kk), kdesc(st + kOp, kk), kIdCB, kk > 0);
        umma_commit(&bar[B_CBFULL0 + s]);
        return true;
      };
      bool ok = total == 0 || issue_cb(0);
      for (int it = 0; ok && it < total; ++it) {
        const int s = it & 1;
        const int c = it % nch;
        const uint32_t st = sbase + s * L::kStage, sC = st, sB = st + kOp;
        const uint32_t pprev = (uint32_t)((it - 1) & 1);
        if (it + 1 < total && !issue_cb(it + 1)) break;
        if (c > 0 || have_init) {
          if (it > 0 && !wait_bar(&bar[B_SPFULL], pprev, s_abort)) break;
          if (it > 0 && !wait_bar(&bar[B_YOFREE], pprev, s_abort)) break;
          tc_fence_after();
#pragma unroll 1
          for (int kk = 0; kk < 8; ++kk)
            umma(tmem + kColYo, kdesc(sC, kk), sdesc(sSp + 256 * kk, 128, 2048), kIdY, kk > 0);
        }
        if (!wait_bar(&bar[B_MFULL], (uint32_t)(it & 1), s_abort)) break;
        if (!wait_bar(&bar[B_SREADY], (uint32_t)(it & 1), s_abort)) break;
        tc_fence_after();
        // S already holds exp(cs_last) * S_prev (the epilogue scaled it): accumulate the chunk.
        // Scaled B as the MN-major A operand (M = n): 128-byte swizzle, n halves 16 KB apart
        // (LBO), K groups of 8 token rows 1024 B apart (SBO)
#pragma unroll 1
        for (int kk = 0; kk < 8; ++kk)
          umma(tmem + kColS, sdesc(sB + 2048 * kk, 16384, 1024) | kSw128, xdesc(st, kk), kIdS, 1u);
        umma_commit(&bar[B_SFULL]);
        if (it > 0 && !wait_bar(&bar[B_YDFREE], pprev, s_abort)) break;
        tc_fence_after();
#pragma unroll 1
        for (int kk = 0; kk < 8; ++kk) umma(tmem + kColYd, sdesc(sM + 4096 * kk, 2048, 128), xdesc(st, kk), kIdY, kk > 0);
        umma_commit(&bar[B_YFULL]);
        umma_commit(&bar[B_MFREE]);
        umma_commit(&bar[B_EMPTY0 + s]);
      }
    }
    __syncwarp();
  } else if (!is_e) {
    // ------------------------------------------------------------------ A: M tile, scaled B
    const int q = warp & 3, half = (warp - kWA0) >> 2;
    const int l = 32 * q + lane;
    const int a_idx = (warp - kWA0) * 32 + lane;   // 0..255
    for (int it = 0; it < total; ++it) {
      const int s = it & 1, vs = it % kVSlots;
      unsigned char* stg = smem + s * L::kStage;
      const float* v_dt = reinterpret_cast<const float*>(smem + L::kVec + vs * kVBytes);
      const float* v_cs = v_dt + kQ;
      const float* v_fst = v_cs + kQ;
      if (!warp_wait(&bar[B_VFULL0 + vs], (uint32_t)((it / kVSlots) & 1), s_abort)) break;
      if (!warp_wait(&bar[B_FULL0 + s], (uint32_t)((it >> 1) & 1), s_abort)) break;
      if (!warp_wait(&bar[B_CBFULL0 + s], (uint32_t)((it >> 1) & 1), s_abort)) break;
      if (it > 0 && !warp_wait(&bar[B_MFREE], (uint32_t)((it - 1) & 1), s_abort)) break;
      tc_fence_after();
      const float cs_l = v_cs[l];
      const uint32_t cb = (s ? kColCB1 : kColCB0) + ((uint32_t)(32 * q) << 16);
#pragma unroll 1
      for (int blk = 0; blk < 4; ++blk) {
        const int s0 = 64 * half + 16 * blk;
        uint4 w0 = make_uint4(0, 0, 0, 0), w1 = make_uint4(0, 0, 0, 0);
        if (s0 <= 32 * q + 31) {   // some s <= l in this block (warp-uniform)
          float v[16];
          tmem_ld16(tmem + cb + s0, v);
          float m[16];
#pragma unroll
          for (int k4 = 0; k4 < 4; ++k4) {
            const float4 c4 = *reinterpret_cast<const float4*>(v_cs + s0 + 4 * k4);
            const float4 d4 = *reinterpret_cast<const float4*>(v_dt + s0 + 4 * k4);
            const float cv[4] = {c4.x, c4.y, c4.z, c4.w}, dv[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int kx = 4 * k4 + j;
              m[kx] = (s0 + kx <= l) ? (v[kx] * ex2_ftz(cs_l - cv[j])) * dv[j] : 0.0f;
            }
          }
          w0 = make_uint4(pack_bf16(m[0], m[1]), pack_bf16(m[2], m[3]), pack_bf16(m[4], m[5]), pack_bf16(m[6], m[7]));
          w1 = make_uint4(pack_bf16(m[8], m[9]), pack_bf16(m[10], m[11]), pack_bf16(m[12], m[13]),
                          pack_bf16(m[14], m[15]));
        }
        unsigned char* mrow = smem + L::kM + (s0 >> 3) * 2048 + l * 16;
        *reinterpret_cast<uint4*>(mrow) = w0;
        *reinterpret_cast<uint4*>(mrow + 2048) = w1;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[B_CBFREE0 + s]);
      unsigned char* bt = stg + kOp;
#pragma unroll 1
      for (int k2 = 0; k2 < 8; ++k2) {
        // 16-byte chunk i of the swizzled tile holds 8 n of token row (i / 8) % 128
        const int i = a_idx + 256 * k2;
        const float f = v_fst[(i >> 3) & 127];
        uint4* qp = reinterpret_cast<uint4*>(bt + i * 16);
        uint4 w = *qp;
        const float2 a0 = unpack_bf16(w.x), a1 = unpack_bf16(w.y), a2 = unpack_bf16(w.z), a3 = unpack_bf16(w.w);
        w.x = pack_bf16(a0.x * f, a0.y * f);
        w.y = pack_bf16(a1.x * f, a1.y * f);
        w.z = pack_bf16(a2.x * f, a2.y * f);
        w.w = pack_bf16(a3.x * f, a3.y * f);
        *qp = w;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bar[B_MFULL]);
        mbar_arrive(&bar[B_VEMPTY0 + vs]);
      }
    }
  } else {
    // ------------------------------------------------------------------ E: state, y
    const uint32_t lane_base = (uint32_t)(32 * eq) << 16;
    // S <- scale * (S or the initial state of item k): the state MMA4 of the next chunk adds to
    if (total > 0 && warp_wait(&bar[B_VFULL0], 0u, s_abort)) {   // the state chunk 0's MMA4 adds to
      const float eT0 = *(reinterpret_cast<const float*>(smem + L::kVec) + 4 * kQ);
#pragma unroll
      for (int kb = 0; kb < NB0; ++kb)
        if (kb < enb) {
          float v[16];
          if (have_init) {
            init_block(0, eb0 + kb, v);
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = 0.0f;
          }
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] *= eT0;
          tmem_st16(tmem + lane_base + kColS + 16 * (eb0 + kb), v);
        }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[B_SREADY]);
    }
    for (int it = 0; it < total; ++it) {
      const int s = it & 1, vs = it % kVSlots;
      const int k = it / nch, c = it - k * nch;
      const bool last = c == nch - 1;
      int b, h;
      item_bh(k, b, h);
      const float* v_eoff = reinterpret_cast<const float*>(smem + L::kVec + vs * kVBytes) + 3 * kQ;
      // x of this thread's token row and column blocks, for D x (global, L2-resident: the
      // chunk's TMA load brought it in), fetched before the waits to hide its latency
      const int t = c * kQ + erow;
      const __nv_bfloat16* xrow =
          p.x + (int64_t)b * p.x_sb + (int64_t)(t < p.T ? t : 0) * p.x_st + (int64_t)h * P;
      uint4 xr[2 * NB0];
#pragma unroll
      for (int kb = 0; kb < NB0; ++kb)
        if (kb < enb) {
          xr[2 * kb] = __ldg(reinterpret_cast<const uint4*>(xrow + 16 * (eb0 + kb)));
          xr[2 * kb + 1] = __ldg(reinterpret_cast<const uint4*>(xrow + 16 * (eb0 + kb) + 8));
        }
      if (!warp_wait(&bar[B_VFULL0 + vs], (uint32_t)((it / kVSlots) & 1), s_abort)) break;
      if (!warp_wait(&bar[B_SFULL], (uint32_t)(it & 1), s_abort)) break;
      tc_fence_after();
      // S after chunk c: the bf16 copy for MMA3 of chunk c+1 (or the final state), then S
      // scaled for chunk it+1's MMA4 (at an item's last chunk: the next item's initial state)
      const bool more = it + 1 < total;
      float eT1 = 0.0f;
      if (more) {
        const int vs1 = (it + 1) % kVSlots;
        if (!warp_wait(&bar[B_VFULL0 + vs1], (uint32_t)(((it + 1) / kVSlots) & 1), s_abort)) break;
        eT1 = *(reinterpret_cast<const float*>(smem + L::kVec + vs1 * kVBytes) + 4 * kQ);
      }
      float* fin = p.fin ? p.fin + (int64_t)b * p.fin_sb + (int64_t)h * P * kN + erow : nullptr;
#pragma unroll 1
      for (int kb = 0; kb < NB0; ++kb) {
        if (kb < enb) {
          const int blk = eb0 + kb;
          float cur[16];
          tmem_ld16(tmem + lane_base + kColS + 16 * blk, cur);
          if (last) {
            if (fin) {
#pragma unroll
              for (int i = 0; i < 16; ++i) fin[(int64_t)(16 * blk + i) * kN] = cur[i];
            }
            if (more) {
              if (have_init) {
                init_block(k + 1, blk, cur);
                sp_block(blk, cur);
              } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) cur[i] = 0.0f;
              }
            }
          } else {
            sp_block(blk, cur);
          }
          if (more) {
#pragma unroll
            for (int i = 0; i < 16; ++i) cur[i] *= eT1;
            tmem_st16(tmem + lane_base + kColS + 16 * blk, cur);
          }
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bar[B_SPFULL]);
        if (more) mbar_arrive(&bar[B_SREADY]);
      }

      if (!warp_wait(&bar[B_YFULL], (uint32_t)(it & 1), s_abort)) break;
      tc_fence_after();
      const float el = v_eoff[erow];
      const float D_h = p.D ? p.D[h] : 0.0f;
      const bool prev = c > 0 || have_init;
      const uint32_t yo = kColYo;
      __nv_bfloat16* yrow = p.y + (int64_t)b * p.y_sb + (int64_t)(t < p.T ? t : 0) * p.y_st + (int64_t)h * P;
#pragma unroll
      for (int kb = 0; kb < NB0; ++kb) {
        if (kb < enb) {
          const int col = 16 * (eb0 + kb);
          float yd[16], yv[16];
          tmem_ld16(tmem + lane_base + kColYd + col, yd);
          if (prev) {
            tmem_ld16(tmem + lane_base + yo + col, yv);
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) yv[i] = 0.0f;
          }
          uint32_t o[8];
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const uint4 xw = xr[2 * kb + hh];
            const uint32_t xs[4] = {xw.x, xw.y, xw.z, xw.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float2 xv = unpack_bf16(xs[i]);
              const int j = 8 * hh + 2 * i;
              const float v0 = (yv[j] * el + yd[j]) + xv.x * D_h;
              const float v1 = (yv[j + 1] * el + yd[j + 1]) + xv.y * D_h;
              o[4 * hh + i] = pack_bf16(v0, v1);
            }
          }
          if (t < p.T) {
            uint4* dst = reinterpret_cast<uint4*>(yrow + col);
            dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
            dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bar[B_YDFREE]);
        mbar_arrive(&bar[B_YOFREE]);
        mbar_arrive(&bar[B_VEMPTY0 + vs]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (tid == 0 && *s_abort && p.status) atomicOr(p.status, STATUS_TIMEOUT);
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

}  // namespace scan
}  // namespace nssm
