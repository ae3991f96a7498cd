// FLUSH phase of the tiered step for fp8 cold rows, bf16 io and a compile-time flush period c
// and headdim (the production configuration): the rank-c replay of the ring into the cold
// slice of every (row, head) item whose token count reached a multiple of c, followed by the
// requantisation to fp8 with a fresh row scale.
//
//   v[p][n] = q[p][n] * (scale[p] * exp(sum_j dA_j)) + sum_j W_j[p] * B'_j[n],
//   W_j[p]  = exp(sum_{k>j} dA_k) * (dt_j * x_j[p]),
//   scale'  = amax_n |v[p][n]| / 448 + 1e-12,   q'[p][n] = e4m3(v[p][n] * rn(1 / scale'))
//
// (scale/v4_fused_decode.py:76-92 with the fp8 row scales of scale/vllm_v4_patch.py:106-114.)
//
// Work split and pipeline as in tiered_persistent_kernel's FLUSH phase: every CTA counts
// and numbers the batch's flushing rows and takes an even share of their items; thread 0
// keeps up to L.nst items in flight with 1-D bulk copies (cold rows, row scales, the ring's
// x, B' and dt: one item's whole working set) into a ring of shared-memory stages.
//
// Thread mapping: headdim / 16 warps, each owning a band of 16 headdim rows of every item.
// Lane = 4 cc + g: g picks the rows {g, g+4, g+8, g+12} of the band, cc one 16-byte chunk
// column (16 fp8 values) of the cold row (chunk columns >= (N-pb)/16 idle).  So each B'_j
// chunk a lane reads from shared memory serves four rows, the row amax is a 3-step shuffle
// over the lanes of one g, and every lane's 64 values stay in registers from the replay to
// the requantisation.  128-bit shared loads are served a quarter-warp at a time: a quarter
// holds two chunk columns x the four row groups, so a B'_j load is two conflict-free
// addresses broadcast to four lanes each, and a cold-row load eight distinct 16-byte chunks
// on distinct banks.  The band's requantised rows and its 16 row scales leave with two bulk
// stores straight from the stage.
#pragma once

#include "nssm_persistent.cuh"

namespace nssm {

constexpr int kFqRows = 16;      // headdim rows per warp band
constexpr int kFqMinBlocks = 3;  // resident CTAs per SM the register budget is sized for

__host__ __device__ constexpr int fq_warps(int P) { return P / kFqRows; }
// W scratch of one warp: per row group g the c float4s of its four rows, groups 4c + 4 floats
// apart (the padding puts the four groups' vectors on distinct banks)
__host__ __device__ constexpr int fq_sw_stride(int c) { return 4 * c + 4; }
__host__ __device__ constexpr int fq_sw_floats(int c) { return 4 * fq_sw_stride(c); }

// Byte layout of the quad-row FLUSH kernel's dynamic shared memory.
struct FqLayout {
  int stage_bytes;
  int s_cold, s_scale, s_rx, s_rb, s_rdt;   // inside a stage
  int off_fsc, off_sw, off_bslot, off_btn, off_cnt, off_bar;
  int total, nst, maxb, maxitems;
};

template <int NC, int CFIX, int P>
__host__ inline FqLayout make_fq_layout(int maxb, int maxitems, int nst) {
  constexpr int cp = (CFIX + 3) & ~3;
  FqLayout L{};
  int o = 0;
  L.s_cold = o; o = al(o + P * NC, 128);
  L.s_scale = o; o = al(o + P * 4, 16);
  L.s_rx = o; o = al(o + CFIX * P * 2, 16);
  L.s_rb = o; o = al(o + CFIX * NC * 4, 16);
  L.s_rdt = o; o = al(o + cp * 4, 16);
  L.stage_bytes = al(o, 128);
  L.nst = nst;
  int t = nst * L.stage_bytes;
  L.off_fsc = t; t += maxitems * (2 * CFIX + 1) * 4;       // per item: exp(suf_j), dt_j, exp(total)
  t = al(t, 16);
  L.off_sw = t; t += fq_warps(P) * fq_sw_floats(CFIX) * 4;   // per warp: W_j of its 16 rows
  L.off_bslot = t; t += maxb * 4;
  L.off_btn = t; t += maxb * 4;
  L.off_cnt = t; t += 32 * 4;                              // per-warp flushing-row counts
  t = al(t, 8);
  L.off_bar = t; t += 2 * nst * 8;
  L.total = al(t, 128);
  L.maxb = maxb;
  L.maxitems = maxitems;
  return L;
}

struct FqParams {
  StepParams sp;
  FqLayout L;
  int batch;
  uint32_t polls;
};

// e4m3 pairs of a 32-bit word -> four fp32 values (exact)
__device__ __forceinline__ void fp8x4_to_f32(uint32_t w, float* v) {
  const __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w & 0xffffu), __NV_E4M3);
  const __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w >> 16), __NV_E4M3);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&lo));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&hi));
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}

__device__ __forceinline__ uint32_t f32x4_to_fp8x4(float a, float b, float c, float d) {
  const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
  const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(c, d), __NV_SATFINITE, __NV_E4M3);
  return (lo & 0xffffu) | (hi << 16);
}

template <int PB, int NC, int CFIX, int P>
__global__ void __launch_bounds__(fq_warps(P) * 32, kFqMinBlocks) flush_quad_kernel(const __grid_constant__ FqParams fp) {
  constexpr int NW = fq_warps(P);
  constexpr int NT = NW * 32;
  constexpr int CPR = NC / 16;              // 16-byte fp8 chunk columns per cold row
  constexpr int c = CFIX;
  constexpr int cp = (CFIX + 3) & ~3;
  static_assert(P % kFqRows == 0 && NC % 16 == 0 && CPR <= 8, "quad-row flush shapes");
  static_assert(CFIX >= 1 && CFIX <= 16, "flush period");

  const StepParams& p = fp.sp;
  const FqLayout& L = fp.L;
  const int kStages = L.nst;
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane & 3, cc = lane >> 2;
  const bool act = cc < CPR;
  const int H = p.H;
  const int HG = H / p.G;

  extern __shared__ __align__(128) unsigned char sm[];
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + L.off_bar);
  uint64_t* empty = full + kStages;
  int* bslot = reinterpret_cast<int*>(sm + L.off_bslot);
  int* btn = reinterpret_cast<int*>(sm + L.off_btn);
  int* wcnt = reinterpret_cast<int*>(sm + L.off_cnt);
  constexpr int SWS = fq_sw_stride(CFIX);
  float* sW = reinterpret_cast<float*>(sm + L.off_sw) + warp * fq_sw_floats(CFIX);

  // ---- the flushing rows, numbered in batch order; this CTA's share of their items
  const int batch = fp.batch;
  auto flush_row = [&](int b, int& slot, int& tn) -> bool {
    slot = p.idx ? p.idx[b] : b;
    if (slot == p.pad || slot < 0 || slot >= p.S) return false;
    tn = p.t[(int64_t)slot * H];
    return tn > 0 && tn % c == 0;
  };
  int nfl = 0;
  for (int c0 = 0; c0 < batch; c0 += NT) {
    int sl = -1, tn = 0;
    nfl += __syncthreads_count(c0 + tid < batch && flush_row(c0 + tid, sl, tn));
  }
  const int W = nfl * H;
  const int beg = (int)((long long)W * blockIdx.x / gridDim.x);
  const int end = (int)((long long)W * (blockIdx.x + 1) / gridDim.x);
  if (beg >= end) return;
  const int b0 = beg / H;
  const int nb = (end - 1) / H - b0 + 1;
  const int nit = end - beg;
  {
    int base = 0;
    for (int c0 = 0; c0 < batch && base < b0 + nb; c0 += NT) {   // uniform over the CTA
      const int b = c0 + tid;
      int slot = -1, tn = 0;
      const bool f = b < batch && flush_row(b, slot, tn);
      const unsigned bal = __ballot_sync(0xffffffffu, f);
      if (lane == 0) wcnt[warp] = __popc(bal);
      __syncthreads();
      int pre = 0, tot = 0;
      for (int w = 0; w < NW; ++w) {
        const int n = wcnt[w];
        pre += w < warp ? n : 0;
        tot += n;
      }
      if (f) {
        const int pos = base + pre + __popc(bal & ((1u << lane) - 1u));
        if (pos >= b0 && pos < b0 + nb) {
          bslot[pos - b0] = slot;
          btn[pos - b0] = tn;
        }
      }
      base += tot;
      __syncthreads();
    }
  }
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NW);
    }
    fence_mbar_init();
  }
  // ---- every item's suffix decays (same sequential order as the oracle: total and
  // suffix sums accumulated j-wise)
  for (int it = tid; it < nit; it += NT) {
    const int w = beg + it;
    const int b = w / H, h = w - b * H;
    const int slot = bslot[b - b0];
    const float* rd = p.ring_dt + ((int64_t)slot * H + h) * cp;
    const float A_h = p.A[h];
    float dts[CFIX];
#pragma unroll
    for (int j = 0; j < CFIX; ++j) dts[j] = rd[j];
    float* fs = reinterpret_cast<float*>(sm + L.off_fsc) + it * (2 * c + 1);
    float tot = 0.0f;
#pragma unroll
    for (int j = 0; j < CFIX; ++j) tot = tot + dts[j] * A_h;
    fs[2 * c] = expf(tot);
    fs[c - 1] = 1.0f;
    fs[2 * c - 1] = dts[c - 1];
    float suf = 0.0f;
#pragma unroll
    for (int j = CFIX - 2; j >= 0; --j) {
      suf = suf + dts[j + 1] * A_h;
      fs[j] = expf(suf);
      fs[c + j] = dts[j];
    }
  }

  // ---- producer: item w = (flushing row b, head h) into stage s (one thread)
  auto issue = [&](int w, int s) {
    const int b = w / H, h = w - b * H;
    const int slot = bslot[b - b0];
    const int64_t sh = (int64_t)slot * H + h;
    unsigned char* st = sm + s * L.stage_bytes;
    const uint32_t bytes = (uint32_t)(P * NC + P * 4 + c * P * 2 + c * NC * 4 + cp * 4);
    mbar_expect_tx(&full[s], bytes);
    bulk_g2s(st + L.s_cold, static_cast<const char*>(p.cold) + sh * P * NC, P * NC, &full[s]);
    bulk_g2s(st + L.s_scale, p.scale + sh * P, P * 4, &full[s]);
    bulk_g2s(st + L.s_rx, static_cast<const char*>(p.ring_x) + sh * c * P * 2, c * P * 2, &full[s]);
    bulk_g2s(st + L.s_rb, p.ring_b + ((int64_t)slot * p.G + h / HG) * c * NC, c * NC * 4, &full[s]);
    bulk_g2s(st + L.s_rdt, p.ring_dt + sh * cp, cp * 4, &full[s]);
  };
  __syncthreads();   // barriers initialised, decay table and row list visible
  uint32_t n_issued = 0;
  int wq = beg;      // producer cursor (items are contiguous: every row in range flushes)
  if (tid == 0) {
    for (int s = 0; s < kStages && wq < end; ++s, ++wq) {
      issue(wq, s);
      ++n_issued;
    }
  }

  const int r0 = warp * kFqRows;
  bool ok = true;
  int s = 0;
  uint32_t par = 0;
  int s_prev = 0;
  uint32_t par_prev = 0;
  for (int w = beg; w < end; ++w) {
    const int it = w - beg;
    const int b = w / H, h = w - b * H;
    const int slot = bslot[b - b0];
    const int64_t sh = (int64_t)slot * H + h;
    unsigned char* st = sm + s * L.stage_bytes;
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(&full[s], par, fp.polls))) { ok = false; break; }
    const float* fs = reinterpret_cast<const float*>(sm + L.off_fsc) + it * (2 * c + 1);

    // W_j[row] for the band's 16 rows: (row, j) pairs over the lanes, stored so that a
    // lane's four rows {g, g+4, g+8, g+12} of one j are one 16-byte vector
    {
      const __nv_bfloat16* rx = reinterpret_cast<const __nv_bfloat16*>(st + L.s_rx);
#pragma unroll
      for (int q = lane; q < kFqRows * c; q += 32) {
        const int j = q / kFqRows, rl = q % kFqRows;
        const float x = __bfloat162float(rx[j * P + r0 + rl]);
        sW[(rl & 3) * SWS + j * 4 + (rl >> 2)] = __fmul_rn(fs[j], __fmul_rn(fs[c + j], x));
      }
    }
    __syncwarp();

    // replay: v[i][e] = sum_j W_j[row_i] B'_j[cc*16 + e] in j order
    float v[4][16];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int e = 0; e < 16; ++e) v[i][e] = 0.0f;
    const float* rb = reinterpret_cast<const float*>(st + L.s_rb);
    if (act) {
#pragma unroll
      for (int j = 0; j < CFIX; ++j) {
        const float4 w4 = *reinterpret_cast<const float4*>(sW + g * SWS + j * 4);
        const float wr[4] = {w4.x, w4.y, w4.z, w4.w};
        const float4* b4 = reinterpret_cast<const float4*>(rb + j * NC + cc * 16);
#pragma unroll
        for (int e4 = 0; e4 < 4; ++e4) {
          const float4 bv = b4[e4];
          const float2 lo = f2(bv.x, bv.y), hi = f2(bv.z, bv.w);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 w2 = f2(wr[i], wr[i]);
            float2 t = __ffma2_rn(w2, lo, f2(v[i][4 * e4], v[i][4 * e4 + 1]));
            v[i][4 * e4] = t.x; v[i][4 * e4 + 1] = t.y;
            t = __ffma2_rn(w2, hi, f2(v[i][4 * e4 + 2], v[i][4 * e4 + 3]));
            v[i][4 * e4 + 2] = t.x; v[i][4 * e4 + 3] = t.y;
          }
        }
      }
    }
    // decay: v += q * (scale * exp(total)) (one fused multiply-add per element; the
    // oracle rounds q * scale first, which moves a stored code by one step in rare cases)
    const float etot = fs[2 * c];
    const float* scl = reinterpret_cast<const float*>(st + L.s_scale);
    const uint4* csm = reinterpret_cast<const uint4*>(st + L.s_cold);
    float m[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int row = r0 + g + 4 * i;
      const float se = __fmul_rn(scl[row], etot);
      const float2 se2 = f2(se, se);
      const uint4 q4 = act ? csm[row * CPR + cc] : make_uint4(0u, 0u, 0u, 0u);
      const uint32_t wv[4] = {q4.x, q4.y, q4.z, q4.w};
      float mx = 0.0f;
#pragma unroll
      for (int wi = 0; wi < 4; ++wi) {
        float qv[4];
        fp8x4_to_f32(wv[wi], qv);
        float2 t = __ffma2_rn(f2(qv[0], qv[1]), se2, f2(v[i][4 * wi], v[i][4 * wi + 1]));
        v[i][4 * wi] = t.x; v[i][4 * wi + 1] = t.y;
        t = __ffma2_rn(f2(qv[2], qv[3]), se2, f2(v[i][4 * wi + 2], v[i][4 * wi + 3]));
        v[i][4 * wi + 2] = t.x; v[i][4 * wi + 3] = t.y;
      }
#pragma unroll
      for (int e = 0; e < 16; e += 2) mx = fmaxf(mx, fmaxf(fabsf(v[i][e]), fabsf(v[i][e + 1])));
      m[i] = mx;
    }
    // row amax over the 8 lanes of row group g (lanes g, g+4, ..., g+28; idle lanes hold zeros)
#pragma unroll
    for (int o = 4; o < 32; o <<= 1)
#pragma unroll
      for (int i = 0; i < 4; ++i) m[i] = fmaxf(m[i], __shfl_xor_sync(0xffffffffu, m[i], o));
    // lane (cc, g) forms the scale of the group's row (cc & 3) (correctly rounded amax / 448,
    // as the oracle) and its reciprocal; lanes cc < 4 hold the four, which are then broadcast
    const int ri = cc & 3;
    const float mi = ri == 0 ? m[0] : ri == 1 ? m[1] : ri == 2 ? m[2] : m[3];
    const float sc = __fadd_rn(scale_div448(mi), kScaleEps);
    const float rc = __frcp_rn(sc);
    float* scl_w = reinterpret_cast<float*>(st + L.s_scale);
    __syncwarp();   // every lane has read its rows' old scales
    if (cc < 4) scl_w[r0 + g + 4 * cc] = sc;
    uint4* cst = reinterpret_cast<uint4*>(st + L.s_cold);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float r = __shfl_sync(0xffffffffu, rc, 4 * i + g);
      const float2 r2 = f2(r, r);
#pragma unroll
      for (int e = 0; e < 16; e += 2) {
        const float2 qq = __fmul2_rn(f2(v[i][e], v[i][e + 1]), r2);
        v[i][e] = qq.x;
        v[i][e + 1] = qq.y;
      }
      if (act) {
        const int row = r0 + g + 4 * i;
        cst[row * CPR + cc] = make_uint4(f32x4_to_fp8x4(v[i][0], v[i][1], v[i][2], v[i][3]),
                                         f32x4_to_fp8x4(v[i][4], v[i][5], v[i][6], v[i][7]),
                                         f32x4_to_fp8x4(v[i][8], v[i][9], v[i][10], v[i][11]),
                                         f32x4_to_fp8x4(v[i][12], v[i][13], v[i][14], v[i][15]));
      }
    }
    // the band's requantised rows and row scales -> global, straight from the stage
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      bulk_s2g(static_cast<char*>(p.cold) + (sh * P + r0) * NC, st + L.s_cold + r0 * NC, kFqRows * NC);
      bulk_s2g(p.scale + sh * P + r0, st + L.s_scale + r0 * 4, kFqRows * 4);
      bulk_commit();
    }

    // ---- release the previous item's stage once this warp's bulk stores have read it; the
    // producer refills it once every warp has (its verdict broadcast to warp 0)
    bool prod_fail = false;
    if (w > beg) {
      if (lane == 0) {
        bulk_wait_read_1();
        mbar_arrive(&empty[s_prev]);
      }
      if (tid == 0 && wq < end) {
        if (!mbar_wait_bounded(&empty[s_prev], par_prev, fp.polls)) {
          prod_fail = true;
        } else {
          fence_proxy_async_smem();
          issue(wq, s_prev);
          ++wq;
          ++n_issued;
        }
      }
    }
    if (warp == 0 && __shfl_sync(0xffffffffu, prod_fail, 0)) { ok = false; break; }
    s_prev = s;
    par_prev = par;
    if (++s == kStages) { s = 0; par ^= 1u; }
  }
  if (lane == 0) bulk_wait_all();   // this warp's bulk stores are complete before exit
  if (!ok) {
    if (lane == 0 && p.status) atomicOr(p.status, STATUS_TIMEOUT);
    if (tid == 0) {
      // keep the CTA alive until its copies in flight have landed (only the last kStages
      // items can be; each is the latest phase of its stage)
      const uint32_t first = n_issued > (uint32_t)kStages ? n_issued - (uint32_t)kStages : 0u;
      for (uint32_t qn = first; qn < n_issued; ++qn)
        mbar_wait_bounded(&full[qn % kStages], (qn / kStages) & 1u, kSpinLimit);
    }
  }
}

}  // namespace nssm
