// FLUSH phase on the 5th-generation tensor cores, for the flush periods whose rank-c update
// is compute-visible on the CUDA cores (c = 16 and 64; fp8 cold, bf16 io, compile-time c and
// headdim).  Per flushing (row, head) item, with W_j[p] = exp(sum_{k>j} dA_k) * (dt_j * x_j[p]):
//
//   U[p][n] = sum_j W_j[p] * B'_j[n]                      tcgen05.mma, fp32 accumulator in TMEM
//   v[p][n] = q[p][n] * (scale[p] * exp(sum_j dA_j)) + U[p][n]
//   scale'  = amax_n |v| / 448 + 1e-12,   q' = e4m3(v * rn(1 / scale'))
//
// (scale/v4_fused_decode.py:76-92, whose flush is a cuBLAS einsum, with the fp8 row scales of
// scale/vllm_v4_patch.py:106-114.)  The MMA is kind::f16 with M = 128 (rows p; headdim 80 or
// 64 of them are used), N = N - pb cold columns.  B'_j holds bf16 values exactly (the ring keeps
// the rotated bf16 B as fp32), so B is one bf16 operand; W is fp32 and is split into three bf16
// pieces W = W_hi + W_mid + W_lo (each the bf16 rounding of what the previous pieces leave; 24
// significant bits in all), whose products with B are exact in the fp32 accumulator.
//   c >= 16: three MMA chains of K = c, one per piece, the smallest piece first;
//   c <= 8 ("packed"): the pieces side by side in K, [W_hi | W_mid | W_lo | 0] against
//     [B; B; B; 0], K = 3c rounded up to 16: one or two MMAs per item.
//
// One CTA = 4 warps = the 128 tensor-memory lanes.  A persistent grid walks the flushing rows'
// items as the other FLUSH kernels do (every CTA counts and numbers the batch's flushing rows
// and takes an even share of their items).  Per item, in order:
//   thread 0 keeps the item's cold rows, row scales, ring x and ring dt in flight in a ring of
//     shared-memory stages (1-D bulk copies, no multicast);
//   thread 0 forms the decay sums in j order (the oracle's), all threads the exponentials;
//   all threads build the three A pieces (K-major, no swizzle: [c/8][128 rows][16 B]) and, when
//     the item's group changes, the B tile (MN-major: [N/8][c rows][16 B]) from the ring's B';
//   thread 0 issues the 3 * c/16 MMAs and commits them to an mbarrier;
//   every thread owning a row p < headdim loads its row of U from tensor memory (16 columns at
//     a time), adds the decayed old row, takes the row amax and scale in registers (one row per
//     thread: no reduction across threads) and requantises into the stage;
//   thread 0 writes the item's cold rows and scales back with two bulk stores.
// All waits are bounded; a wait that runs out sets bit 1 of the status word, and the CTA waits
// (bounded) for its copies and MMAs in flight, frees its tensor memory and leaves.
#pragma once

#include "nssm_persistent.cuh"
#include "nssm_tc.cuh"

namespace nssm {

constexpr int kFmThreads = 128;
constexpr int kFmRowsPerThread = 8;   // batch rows one thread counts per pass (1024 per pass)
constexpr uint32_t kFmTmemCols = 128;

// resident CTAs per SM the register budget is sized for (a row's NC values live in registers)
__host__ __device__ constexpr int fm_min_blocks(int c, int nc) { return (c <= 8 && nc <= 96) ? 4 : c <= 16 ? 3 : 2; }
// the three W pieces share one K range when 3c fits in two MMA K steps
__host__ __device__ constexpr bool fm_packed(int c) { return 3 * c <= 32; }
// K extent of the A tile(s): packed 3c rounded up to 16, else c per piece
__host__ __device__ constexpr int fm_k(int c) { return fm_packed(c) ? (3 * c + 15) / 16 * 16 : c; }
// bytes of the A operand (packed: one tile; else three piece tiles) and of the B tile
__host__ __device__ constexpr int fm_a_bytes(int c) { return (fm_packed(c) ? fm_k(c) : 3 * c) / 8 * 128 * 16; }
template <int NC> __host__ __device__ constexpr int fm_b_bytes(int c) { return NC / 8 * fm_k(c) * 16; }

struct FmLayout {
  int stage_bytes;
  int s_cold, s_scale, s_rx, s_rdt;   // inside a stage
  int off_a, off_b, off_tab, off_bslot, off_cnt, off_bar, off_tmem;
  int total, nst, maxb;
};

template <int NC, int CFIX, int P>
__host__ inline FmLayout make_fm_layout(int maxb, int nst) {
  constexpr int cp = (CFIX + 3) & ~3;
  FmLayout L{};
  int o = 0;
  L.s_cold = o; o = al(o + P * NC, 128);
  L.s_scale = o; o = al(o + P * 4, 16);
  L.s_rx = o; o = al(o + CFIX * P * 2, 16);
  L.s_rdt = o; o = al(o + cp * 4, 16);
  L.stage_bytes = al(o, 128);
  L.nst = nst;
  int t = nst * L.stage_bytes;
  L.off_a = t; t += fm_a_bytes(CFIX);                // A: pieces hi | mid | lo
  L.off_b = t; t += fm_b_bytes<NC>(CFIX);            // B tile
  L.off_tab = t; t += (3 * CFIX + 4) * 4;           // suffix sums, exp(suf_j), dt_j, exp(total)
  t = al(t, 16);
  L.off_bslot = t; t += maxb * 4;
  L.off_cnt = t; t += 32 * 4;
  t = al(t, 8);
  L.off_bar = t; t += (nst + 1) * 8;                // full[nst], mma
  L.off_tmem = t; t += 16;
  L.total = al(t, 128);
  L.maxb = maxb;
  return L;
}

// e4m3 pairs of a 32-bit word -> four fp32 values (exact)
__device__ __forceinline__ void fp8x4_to_f32(uint32_t w, float* v) {
  const __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w & 0xffffu), __NV_E4M3);
  const __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w >> 16), __NV_E4M3);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&lo));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&hi));
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}

// four fp32 values (already divided by the row scale) -> four e4m3 codes, saturating
__device__ __forceinline__ uint32_t f32x4_to_fp8x4(float a, float b, float c, float d) {
  const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
  const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(c, d), __NV_SATFINITE, __NV_E4M3);
  return (lo & 0xffffu) | (hi << 16);
}

struct FmParams {
  StepParams sp;
  FmLayout L;
  int batch;
  uint32_t polls;
};

__device__ __forceinline__ uint32_t bf16x2_bits(float a, float b) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// fp32 w = hi + mid + lo with each piece the bf16 rounding of what the previous ones leave
// (the residuals are exact in fp32); returned as bf16 bit patterns
__device__ __forceinline__ void split3_bf16(float w, uint16_t& hi, uint16_t& mid, uint16_t& lo) {
  const __nv_bfloat16 h = __float2bfloat16_rn(w);
  const float r1 = __fsub_rn(w, __bfloat162float(h));
  const __nv_bfloat16 m = __float2bfloat16_rn(r1);
  const float r2 = __fsub_rn(r1, __bfloat162float(m));
  const __nv_bfloat16 l = __float2bfloat16_rn(r2);
  hi = __bfloat16_as_ushort(h);
  mid = __bfloat16_as_ushort(m);
  lo = __bfloat16_as_ushort(l);
}

template <int PB, int NC, int CFIX, int P>
__global__ void __launch_bounds__(kFmThreads, fm_min_blocks(CFIX, NC)) flush_mma_kernel(const __grid_constant__ FmParams fp) {
  constexpr int NT = kFmThreads;
  constexpr int c = CFIX;
  constexpr int cp = (CFIX + 3) & ~3;
  constexpr bool PACK = fm_packed(CFIX);
  constexpr int KT = fm_k(CFIX);           // K rows of the B tile
  constexpr int KC = KT / 8;               // 16-byte K chunks of an A row (of one piece)
  constexpr int NB = NC / 16;              // 16-column blocks of a cold row
  static_assert(PACK ? (CFIX >= 1) : (CFIX % 16 == 0 && CFIX <= 128), "flush period vs the MMA's K = 16");
  static_assert(NC % 16 == 0 && NC >= 16 && NC <= 256, "cold width: the MMA's N");
  static_assert(P % 16 == 0 && P <= 128, "headdim rows within the 128 tensor-memory lanes");
  constexpr uint32_t kIdesc = idesc_bf16(128, NC, 0, 1);
  constexpr int kAPiece = KC * 128 * 16;   // bytes of one A piece

  const StepParams& p = fp.sp;
  const FmLayout& L = fp.L;
  const int kStages = L.nst;
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int H = p.H;
  const int HG = H / p.G;

  extern __shared__ __align__(128) unsigned char sm[];
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + L.off_bar);
  uint64_t* mma_bar = full + kStages;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sm + L.off_tmem);
  int* bslot = reinterpret_cast<int*>(sm + L.off_bslot);
  int* wcnt = reinterpret_cast<int*>(sm + L.off_cnt);
  float* tab = reinterpret_cast<float*>(sm + L.off_tab);   // [0,c): suffix sums -> exp; [c,2c): dt; [2c]: exp(total)
  unsigned char* sA = sm + L.off_a;
  unsigned char* sB = sm + L.off_b;

  // ---- the flushing rows, numbered in batch order; this CTA's share of their items.  One
  // pass: thread tid owns the contiguous rows [tid*R, tid*R + R) (R = ceil(batch / 128), at
  // most kFmRowsPerThread; larger batches loop over blocks of 128 * R rows), loads all of their
  // slots and then all of their token counts before using any (two memory round trips per
  // block, not per 128 rows), and a block-wide exclusive scan of the per-thread counts numbers
  // the flushing rows.  A launch where no row flushes leaves after that one pass.
  const int batch = fp.batch;
  const int R = min((batch + NT - 1) / NT, kFmRowsPerThread);
  const int blk_rows = R * NT;
  auto flags_of = [&](int r0, int* slots) -> uint32_t {   // bit k: row r0 + k flushes
    int sl[kFmRowsPerThread];
#pragma unroll
    for (int k = 0; k < kFmRowsPerThread; ++k) {
      const int b = r0 + k;
      sl[k] = (k < R && b < batch) ? (p.idx ? p.idx[b] : b) : -1;
    }
    int tn[kFmRowsPerThread];
#pragma unroll
    for (int k = 0; k < kFmRowsPerThread; ++k) {
      const bool v = sl[k] != p.pad && sl[k] >= 0 && sl[k] < p.S;
      tn[k] = v ? p.t[(int64_t)sl[k] * H] : 0;
      if (!v) sl[k] = -1;
    }
    uint32_t f = 0u;
#pragma unroll
    for (int k = 0; k < kFmRowsPerThread; ++k) {
      if (sl[k] >= 0 && tn[k] > 0 && tn[k] % c == 0) f |= 1u << k;
      if (slots) slots[k] = sl[k];
    }
    return f;
  };
  // exclusive prefix (over threads in order) of each thread's count, and the block total
  auto block_scan = [&](int v, int& total) -> int {
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    if (lane == 31) wcnt[warp] = incl;
    __syncthreads();
    int before = 0;
    total = 0;
    for (int w2 = 0; w2 < NT / 32; ++w2) {
      const int n = wcnt[w2];
      before += w2 < warp ? n : 0;
      total += n;
    }
    __syncthreads();
    return before + incl - v;
  };
  int nfl = 0;
  for (int bb = 0; bb < batch; bb += blk_rows) {
    int tot = 0;
    block_scan(__popc(flags_of(bb + tid * R, nullptr)), tot);
    nfl += tot;
  }
  const int W = nfl * H;
  const int beg = (int)((long long)W * blockIdx.x / gridDim.x);
  const int end = (int)((long long)W * (blockIdx.x + 1) / gridDim.x);
  if (beg >= end) return;
  const int b0 = beg / H;
  const int nb = (end - 1) / H - b0 + 1;
  {
    int base = 0;
    for (int bb = 0; bb < batch && base < b0 + nb; bb += blk_rows) {   // uniform over the CTA
      int sl[kFmRowsPerThread];
      const uint32_t f = flags_of(bb + tid * R, sl);
      int tot = 0;
      int pos = base + block_scan(__popc(f), tot);
#pragma unroll
      for (int k = 0; k < kFmRowsPerThread; ++k) {
        if (f & (1u << k)) {
          if (pos >= b0 && pos < b0 + nb) bslot[pos - b0] = sl[k];
          ++pos;
        }
      }
      base += tot;
    }
  }
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
    mbar_init(mma_bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(s_tmem, kFmTmemCols);

  // ---- producer: item w's cold rows, scales, ring x and ring dt into stage s (thread 0)
  auto issue = [&](int w, int s) {
    const int b = w / H, h = w - b * H;
    const int64_t sh = (int64_t)bslot[b - b0] * H + h;
    unsigned char* st = sm + s * L.stage_bytes;
    mbar_expect_tx(&full[s], (uint32_t)(P * NC + P * 4 + c * P * 2 + cp * 4));
    bulk_g2s(st + L.s_cold, static_cast<const char*>(p.cold) + sh * P * NC, P * NC, &full[s]);
    bulk_g2s(st + L.s_scale, p.scale + sh * P, P * 4, &full[s]);
    bulk_g2s(st + L.s_rx, static_cast<const char*>(p.ring_x) + sh * c * P * 2, c * P * 2, &full[s]);
    bulk_g2s(st + L.s_rdt, p.ring_dt + sh * cp, cp * 4, &full[s]);
  };
  tc_fence_before();
  __syncthreads();   // barriers initialised, row list and tensor-memory address visible
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  uint32_t n_issued = 0;
  int wq = beg;
  if (tid == 0) {
    for (int s = 0; s < kStages && wq < end; ++s, ++wq) {
      issue(wq, s);
      ++n_issued;
    }
  }

  const uint32_t a_base = smem_u32(sA), b_base = smem_u32(sB);
  const int row = tid;                      // this thread's tensor-memory lane = headdim row
  bool ok = true;
  bool mma_pending = false;
  int cur_group = -1;                       // (row, group) whose B tile is in shared memory
  int s = 0;
  uint32_t par = 0;
  uint32_t mpar = 0;
  for (int w = beg; w < end; ++w) {
    const int b = w / H, h = w - b * H;
    const int slot = bslot[b - b0];
    const int64_t sh = (int64_t)slot * H + h;
    const int grp = b * p.G + h / HG;
    unsigned char* st = sm + s * L.stage_bytes;
    if (!__syncthreads_and(mbar_wait_bounded(&full[s], par, fp.polls))) { ok = false; break; }

    // ---- decay sums in the oracle's order (thread 0), exponentials (all)
    const float* rdt = reinterpret_cast<const float*>(st + L.s_rdt);
    if (tid == 0) {
      const float A_h = p.A[h];
      float tot = 0.0f;
      for (int j = 0; j < c; ++j) tot = tot + rdt[j] * A_h;
      tab[3 * c] = tot;
      float suf = 0.0f;
      tab[c - 1] = 0.0f;
      for (int j = c - 2; j >= 0; --j) {
        suf = suf + rdt[j + 1] * A_h;
        tab[j] = suf;
      }
    }
    __syncthreads();
    if (tid < c) {
      tab[c + tid] = tid == c - 1 ? 1.0f : expf(tab[tid]);   // exp(suf_j)
      tab[2 * c + tid] = rdt[tid];                            // dt_j
    }
    if (tid == 0) tab[3 * c + 1] = expf(tab[3 * c]);
    // ---- B tile of the item's (row, group): ring B'_j[n] (bf16 values held exactly in fp32)
    // -> bf16, MN-major [N/8 chunks][KT rows][16 B]; packed: row k holds B'_{k mod c} for
    // k < 3c and zeros after
    if (grp != cur_group) {
      const float* rb = p.ring_b + ((int64_t)slot * p.G + h / HG) * c * NC;
      for (int q = tid; q < (NC / 8) * KT; q += NT) {
        const int k = q % KT, n8 = q / KT;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (!PACK || k < 3 * c) {
          const int j = PACK ? k % c : k;
          const float4 lo = *reinterpret_cast<const float4*>(rb + j * NC + n8 * 8);
          const float4 hi = *reinterpret_cast<const float4*>(rb + j * NC + n8 * 8 + 4);
          v.x = bf16x2_bits(lo.x, lo.y);
          v.y = bf16x2_bits(lo.z, lo.w);
          v.z = bf16x2_bits(hi.x, hi.y);
          v.w = bf16x2_bits(hi.z, hi.w);
        }
        *reinterpret_cast<uint4*>(sB + n8 * (KT * 16) + k * 16) = v;
      }
      cur_group = grp;
    }
    __syncthreads();   // tab complete
    // ---- A: W_j[row] split into three bf16 pieces, K-major [K/8 chunks][128 rows][16 B];
    // packed: one task per row writes [hi | mid | lo | 0] over K, else three piece tiles with
    // one task per (row, 8 consecutive j)
    const __nv_bfloat16* rx = reinterpret_cast<const __nv_bfloat16*>(st + L.s_rx);
    if constexpr (PACK) {
      for (int r = tid; r < P; r += NT) {
        uint16_t pc[3][CFIX];
#pragma unroll
        for (int j = 0; j < CFIX; ++j)
          split3_bf16(__fmul_rn(tab[c + j], __fmul_rn(tab[2 * c + j], __bfloat162float(rx[j * P + r]))), pc[0][j],
                      pc[1][j], pc[2][j]);
        uint32_t wds[KT / 2];
#pragma unroll
        for (int k2 = 0; k2 < KT / 2; ++k2) {
          uint32_t lohalf = 0u, hihalf = 0u;
          const int k0 = 2 * k2, k1 = 2 * k2 + 1;
          if (k0 < 3 * CFIX) lohalf = pc[k0 / CFIX][k0 % CFIX];
          if (k1 < 3 * CFIX) hihalf = pc[k1 / CFIX][k1 % CFIX];
          wds[k2] = lohalf | (hihalf << 16);
        }
#pragma unroll
        for (int k8 = 0; k8 < KC; ++k8)
          *reinterpret_cast<uint4*>(sA + k8 * 2048 + r * 16) =
              make_uint4(wds[4 * k8], wds[4 * k8 + 1], wds[4 * k8 + 2], wds[4 * k8 + 3]);
      }
    } else {
      for (int q = tid; q < P * KC; q += NT) {
        const int r = q % P, k8 = q / P;
        uint32_t ph[4], pm[4], pl[4];
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          uint16_t h0, m0, l0, h1, m1, l1;
          const int j = 8 * k8 + e;
          split3_bf16(__fmul_rn(tab[c + j], __fmul_rn(tab[2 * c + j], __bfloat162float(rx[j * P + r]))), h0, m0, l0);
          split3_bf16(__fmul_rn(tab[c + j + 1], __fmul_rn(tab[2 * c + j + 1], __bfloat162float(rx[(j + 1) * P + r]))),
                      h1, m1, l1);
          ph[e / 2] = (uint32_t)h0 | ((uint32_t)h1 << 16);
          pm[e / 2] = (uint32_t)m0 | ((uint32_t)m1 << 16);
          pl[e / 2] = (uint32_t)l0 | ((uint32_t)l1 << 16);
        }
        const int off = k8 * 2048 + r * 16;
        *reinterpret_cast<uint4*>(sA + off) = make_uint4(ph[0], ph[1], ph[2], ph[3]);
        *reinterpret_cast<uint4*>(sA + kAPiece + off) = make_uint4(pm[0], pm[1], pm[2], pm[3]);
        *reinterpret_cast<uint4*>(sA + 2 * kAPiece + off) = make_uint4(pl[0], pl[1], pl[2], pl[3]);
      }
    }
    fence_proxy_async_smem();   // the operands written by this thread -> the tensor core's view
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // ---- U = W_lo B + W_mid B + W_hi B (smallest first), fp32 in tensor memory
    if (tid == 0) {
      if constexpr (PACK) {
#pragma unroll
        for (int kk = 0; kk < KT / 16; ++kk)
          umma(tmem, sdesc(a_base + kk * 4096, 2048, 128), sdesc(b_base + kk * 256, 128, KT * 16), kIdesc,
               kk == 0 ? 0u : 1u);
      } else {
#pragma unroll
        for (int q = 2; q >= 0; --q)
#pragma unroll
          for (int kk = 0; kk < c / 16; ++kk)
            umma(tmem, sdesc(a_base + q * kAPiece + kk * 4096, 2048, 128), sdesc(b_base + kk * 256, 128, KT * 16),
                 kIdesc, (q == 2 && kk == 0) ? 0u : 1u);
      }
      umma_commit(mma_bar);
    }
    mma_pending = true;
    if (!__syncthreads_and(mbar_wait_bounded(mma_bar, mpar, fp.polls))) { ok = false; break; }
    mma_pending = false;
    mpar ^= 1u;
    tc_fence_after();

    // ---- epilogue: one headdim row per thread
    const float etot = tab[3 * c + 1];
    if (warp * 32 < P) {   // warp-uniform: the tensor-memory loads are warp-collective
      const bool mine = row < P;
      const float se = mine ? __fmul_rn(reinterpret_cast<const float*>(st + L.s_scale)[row], etot) : 0.0f;
      const float2 se2 = f2(se, se);
      const uint4* crow = reinterpret_cast<const uint4*>(st + L.s_cold + (mine ? row : 0) * NC);
      // U of this row straight into v (96 columns: two loads and one wait), then in place
      // v = q * se + U
      float v[NC];
      const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16);
      if constexpr (NC == 96) {
        tmem_ld96(taddr, v);
      } else {
#pragma unroll
        for (int blk = 0; blk < NB; ++blk) tmem_ld16(taddr + (uint32_t)(blk * 16), v + 16 * blk);
      }
      float mx[4] = {0.0f, 0.0f, 0.0f, 0.0f};   // independent partial maxima (no serial chain)
#pragma unroll
      for (int blk = 0; blk < NB; ++blk) {
        const uint4 q4 = mine ? crow[blk] : make_uint4(0u, 0u, 0u, 0u);
        const uint32_t wv[4] = {q4.x, q4.y, q4.z, q4.w};
        float* u = v + 16 * blk;
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
          float qv[4];
          fp8x4_to_f32(wv[wi], qv);
          const float2 a = __ffma2_rn(f2(qv[0], qv[1]), se2, f2(u[4 * wi], u[4 * wi + 1]));
          const float2 d = __ffma2_rn(f2(qv[2], qv[3]), se2, f2(u[4 * wi + 2], u[4 * wi + 3]));
          u[4 * wi] = a.x; u[4 * wi + 1] = a.y;
          u[4 * wi + 2] = d.x; u[4 * wi + 3] = d.y;
          mx[wi] = fmaxf(mx[wi], fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(d.x), fabsf(d.y))));
        }
      }
      if (mine) {
        const float m = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
        const float sc = __fadd_rn(scale_div448(m), kScaleEps);
        const float rc = __frcp_rn(sc);
        reinterpret_cast<float*>(st + L.s_scale)[row] = sc;
        const float2 r2 = f2(rc, rc);
        uint4* cw = reinterpret_cast<uint4*>(st + L.s_cold + row * NC);
#pragma unroll
        for (int blk = 0; blk < NB; ++blk) {
          float* vb = v + 16 * blk;
#pragma unroll
          for (int e = 0; e < 16; e += 2) {
            const float2 qq = __fmul2_rn(f2(vb[e], vb[e + 1]), r2);
            vb[e] = qq.x;
            vb[e + 1] = qq.y;
          }
          cw[blk] = make_uint4(f32x4_to_fp8x4(vb[0], vb[1], vb[2], vb[3]), f32x4_to_fp8x4(vb[4], vb[5], vb[6], vb[7]),
                               f32x4_to_fp8x4(vb[8], vb[9], vb[10], vb[11]),
                               f32x4_to_fp8x4(vb[12], vb[13], vb[14], vb[15]));
        }
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();   // the item's rows are requantised in the stage; tensor memory read
    if (tid == 0) {
      bulk_s2g(static_cast<char*>(p.cold) + sh * P * NC, st + L.s_cold, P * NC);
      bulk_s2g(p.scale + sh * P, st + L.s_scale, P * 4);
      bulk_commit();
      // the previous item's stores have read their stage: refill it
      if (w > beg && wq < end) {
        bulk_wait_read_1();
        const int sp = (s == 0 ? kStages : s) - 1;
        issue(wq, sp);
        ++wq;
        ++n_issued;
      }
    }
    if (++s == kStages) { s = 0; par ^= 1u; }
  }
  if (tid == 0) bulk_wait_all();   // the bulk stores are complete before exit
  if (!ok) {
    if (tid == 0) {
      if (p.status) atomicOr(p.status, STATUS_TIMEOUT);
      // copies in flight: only the last kStages issued items can be (each the latest phase of
      // its stage); an MMA in flight: its commit (both bounded, with the default poll count)
      const uint32_t first = n_issued > (uint32_t)kStages ? n_issued - (uint32_t)kStages : 0u;
      for (uint32_t qn = first; qn < n_issued; ++qn)
        mbar_wait_bounded(&full[qn % kStages], (qn / kStages) & 1u, kSpinLimit);
      if (mma_pending) mbar_wait_bounded(mma_bar, mpar, kSpinLimit);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_free(tmem, kFmTmemCols);
}

}  // namespace nssm
