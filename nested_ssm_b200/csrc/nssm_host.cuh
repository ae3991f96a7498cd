// Host-side launch helpers shared by the translation units of libnested_ssm:
// validation results are reported through fail() (thread-local message), and each
// (dstate, hot width, cold dtype, io dtype) instance is launched by the templates
// below.  nssm_pb16/32/64.cu instantiate them per hot width (compiled in parallel);
// nssm_abi.cu holds the extern "C" entry points.
#pragma once

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

#include "nssm_persistent.cuh"
#include "nssm_flush_mma.cuh"
#include "nssm_spec.cuh"
#include "nssm_rot.cuh"
#include "nssm_conv.cuh"

namespace nssm_host {

int fail(int code, const char* fmt, ...);
int cuda_check(const char* what);
int occupancy(const void* fn, int smem, int threads, int* occ_out);
int ensure_smem_attr(const void* fn);   // opt the kernel in to the device's shared-memory maximum
int sm_count(int* out);
int smem_optin(int* out);
uint32_t wait_polls();   // polls of a bounded pipeline wait (nssm_set_wait_polls)
int inject_stuck();      // failure injection for tests (nssm_test_inject_stuck_copy)
// set by the step dispatch when the gated norm ran fused into STEP (this thread's last call)
extern thread_local bool g_norm_fused;

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int io_bytes(int dt) { return dt == NSSM_BF16 ? 2 : 4; }

inline int round_up(int v, int m) { return (v + m - 1) / m * m; }

using nssm::COLD_BF16;
using nssm::COLD_F32;
using nssm::COLD_FP8;
using nssm::COLD_NONE;

constexpr int kTPR = 2;        // threads per headdim row, tiered kernels
constexpr int kTPRFresh = 4;   // threads per headdim row, untiered kernel

template <int PB, int NC, int COLD>
size_t step_smem_bytes(int P, int c) {
  return sizeof(float) * nssm::StepShape<PB, NC, COLD>::smem_floats(P, c);
}

// ---- launchers ------------------------------------------------------------
template <int PB, int NC, int COLD, int TPR>
int launch_step(const nssm::StepParams& sp, int batch, cudaStream_t st) {
  dim3 grid(sp.H, batch);
  const int threads = round_up(sp.P * TPR, 32);
  nssm::tiered_step_kernel<PB, NC, COLD, TPR><<<grid, threads, step_smem_bytes<PB, NC, COLD>(sp.P, sp.c), st>>>(sp);
  return cuda_check("tiered_step_kernel launch");
}

// The persistent TMA-pipelined kernels move every per-item operand with 1-D bulk
// copies, so they need 16-byte aligned rows: headdim % 4 == 0 and <= 80, x / B / C
// bases and strides 16-byte aligned.  Anything else runs the simple kernel.
template <int PB, int NC, int COLD, bool IOBF, int PHASE, int CFIX, int RPWC, bool NORM = false>
inline int launch_phase(const nssm::StepParams& sp, int batch, cudaStream_t st, bool ring_ok, int sms, bool* done) {
  *done = false;
  const long long items = (long long)batch * sp.H;
  auto fn = nssm::tiered_persistent_kernel<PB, NC, COLD, IOBF, PHASE, CFIX, RPWC, NORM>;
  const int hg = sp.H / sp.G;
  const int iob = IOBF ? 2 : 4;
  const int minb = PHASE == nssm::PH_STEP ? NSSM_STEP_P_MINB : NSSM_FLUSH_P_MINB;
  int optin = 0;
  int rc = smem_optin(&optin);
  if (rc) return rc;
  for (int target = minb; target >= 1; --target) {
    long long grid = (long long)sms * target;
    if (grid > items) grid = items;
    // with the fused norm a CTA takes whole (row, group) units of hg items
    const long long per_cta = NORM ? (items / hg + grid - 1) / grid * hg : (items + grid - 1) / grid;
    const int maxb = (int)((per_cta + sp.H - 1) / sp.H) + 2;
    nssm::PParams pp{};
    pp.sp = sp;
    pp.items = (int)items;
    pp.ring_in_stage = ring_ok ? 1 : 0;
    pp.polls = wait_polls();
    pp.inject_stuck = PHASE == nssm::PH_STEP ? inject_stuck() : 0;
    // deepest pipeline (up to the phase's stage count) whose CTAs fit `target` per SM
    int nst = nssm::stages_for(PHASE);
    for (; nst >= 2; --nst) {
      pp.L = nssm::make_playout<PB, NC, COLD>(PHASE, sp.mode == NSSM_MODE_CORR, sp.P, sp.H, sp.c, iob, maxb,
                                              (int)per_cta, ring_ok, nst, NORM ? hg : 0);
      if (pp.L.total <= optin && (long long)target * (pp.L.total + 1024) <= 228 * 1024) break;
    }
    if (nst < 2) continue;
    int occ = 0;
    rc = occupancy(reinterpret_cast<const void*>(fn), pp.L.total, nssm::kPT, &occ);
    if (rc) return rc;
    if (occ >= target) {
      fn<<<(unsigned)grid, nssm::kPT, pp.L.total, st>>>(pp);
      *done = true;
      return cuda_check("tiered_persistent_kernel launch");
    }
  }
  return NSSM_OK;
}

// The tensor-core FLUSH kernel (fp8 cold, bf16 io, c in {4, 8, 16, 64}, compile-time headdim);
// *done stays false when its layout does not fit the device.
template <int PB, int NC, int CFIX, int P>
inline int launch_flush_mma(const nssm::StepParams& sp, int batch, cudaStream_t st, int sms, bool* done) {
  *done = false;
  const long long items = (long long)batch * sp.H;
  auto fn = nssm::flush_mma_kernel<PB, NC, CFIX, P>;
  int optin = 0;
  int rc = smem_optin(&optin);
  if (rc) return rc;
  for (int target = nssm::fm_min_blocks(CFIX, NC); target >= 1; --target) {
    long long grid = (long long)sms * target;
    if (grid > items) grid = items;
    const long long per_cta = (items + grid - 1) / grid;
    const int maxb = (int)((per_cta + sp.H - 1) / sp.H) + 2;
    nssm::FmParams fp{};
    fp.sp = sp;
    fp.batch = batch;
    fp.polls = wait_polls();
    int nst = 6;
    for (; nst >= 2; --nst) {
      fp.L = nssm::make_fm_layout<NC, CFIX, P>(maxb, nst);
      if (fp.L.total <= optin && (long long)target * (fp.L.total + 1024) <= 228 * 1024) break;
    }
    if (nst < 2) continue;
    // Residency from this kernel's own budgets: registers (its launch bounds reserve them for
    // fm_min_blocks CTAs), shared memory (checked above) and tensor memory (target x 128 of the
    // SM's 512 columns, so an allocation never waits).  The runtime's occupancy query reports
    // one CTA per SM for every kernel that allocates tensor memory, so it is not asked.
    static_assert(nssm::fm_min_blocks(CFIX, NC) * nssm::kFmTmemCols <= 512, "tensor memory per SM");
    rc = ensure_smem_attr(reinterpret_cast<const void*>(fn));
    if (rc) return rc;
    fn<<<(unsigned)grid, nssm::kFmThreads, fp.L.total, st>>>(fp);
    *done = true;
    return cuda_check("flush_mma_kernel launch");
  }
  return NSSM_OK;
}

// The FLUSH of the rows whose t is a multiple of c (after their STEP or commit).  The
// production configuration's is the tensor-core kernel (NSSM_LEGACY_FLUSH builds keep the
// banded FLUSH phase of the persistent kernel).
template <int PB, int NC, int COLD, bool IOBF, int CFIX, int RPWC>
inline int launch_flush_part(const nssm::StepParams& sp, int batch, cudaStream_t st, bool ring_ok, int sms) {
  bool done = false;
  int rc = NSSM_OK;
  if constexpr (COLD == nssm::COLD_FP8 && IOBF && (CFIX == 4 || CFIX == 8 || CFIX == 16 || CFIX == 64) &&
                (RPWC == 8 || RPWC == 10) && NC % 16 == 0) {
#ifndef NSSM_LEGACY_FLUSH
    const bool rows_ok = aligned16(sp.ring_x) && aligned16(sp.ring_dt);
    if (rows_ok) {
      rc = launch_flush_mma<PB, NC, CFIX, 8 * RPWC>(sp, batch, st, sms, &done);
      if (rc || done) return rc;
    }
#endif
  }
  rc = launch_phase<PB, NC, COLD, IOBF, nssm::PH_FLUSH, CFIX, RPWC>(sp, batch, st, ring_ok, sms, &done);
  if (rc) return rc;
  if (!done) return fail(NSSM_ERR_UNSUPPORTED, "flush phase does not fit this device");
  return NSSM_OK;
}

// Both phases of one step (FLUSH_ONLY: the FLUSH alone, after a commit).  The production
// configuration (fp8 cold, bf16 io) has instances compiled for c in {4, 8, 16, 64} and
// headdim in {64, 80}; anything else runs the instances that read c and headdim at run time.
template <int PB, int NC, int COLD, bool IOBF, int CFIX, int RPWC, bool FLUSH_ONLY = false>
inline int launch_both(const nssm::StepParams& sp, int batch, cudaStream_t st, bool ring_ok, int sms) {
  if constexpr (FLUSH_ONLY) return launch_flush_part<PB, NC, COLD, IOBF, CFIX, RPWC>(sp, batch, st, ring_ok, sms);
  bool done = false;
  int rc = NSSM_OK;
  // the fused norm runs in the production instances' STEP; elsewhere the step writes y and
  // the caller of the dispatch applies the norm kernel (g_norm_fused stays false)
  constexpr bool kNormable = COLD == nssm::COLD_FP8 && IOBF && RPWC > 0;
  if constexpr (kNormable) {
    if (sp.ngate) {
      rc = launch_phase<PB, NC, COLD, IOBF, nssm::PH_STEP, CFIX, RPWC, true>(sp, batch, st, ring_ok, sms, &done);
      if (rc) return rc;
      g_norm_fused = done;
    }
  }
  if (!done) rc = launch_phase<PB, NC, COLD, IOBF, nssm::PH_STEP, CFIX, RPWC>(sp, batch, st, ring_ok, sms, &done);
  if (rc) return rc;
  if (!done) return launch_step<PB, NC, COLD, kTPR>(sp, batch, st);
  return launch_flush_part<PB, NC, COLD, IOBF, CFIX, RPWC>(sp, batch, st, ring_ok, sms);
}

template <int PB, int NC, int COLD, bool IOBF, int RPWC, bool FLUSH_ONLY>
inline int launch_c(const nssm::StepParams& sp, int batch, cudaStream_t st, bool ring_ok, int sms) {
  switch (sp.c) {
    case 4: return launch_both<PB, NC, COLD, IOBF, 4, RPWC, FLUSH_ONLY>(sp, batch, st, ring_ok, sms);
    case 8: return launch_both<PB, NC, COLD, IOBF, 8, RPWC, FLUSH_ONLY>(sp, batch, st, ring_ok, sms);
    case 16: return launch_both<PB, NC, COLD, IOBF, 16, RPWC, FLUSH_ONLY>(sp, batch, st, ring_ok, sms);
    case 64: return launch_both<PB, NC, COLD, IOBF, 64, RPWC, FLUSH_ONLY>(sp, batch, st, ring_ok, sms);
  }
  return launch_both<PB, NC, COLD, IOBF, 0, 0, FLUSH_ONLY>(sp, batch, st, ring_ok, sms);
}

template <int PB, int NC, int COLD, bool IOBF, bool FLUSH_ONLY = false>
inline int launch_persistent(const nssm::StepParams& sp, int batch, cudaStream_t st, bool ring_ok) {
  const long long items = (long long)batch * sp.H;
  if (items > (1ll << 30)) {
    if constexpr (FLUSH_ONLY) return fail(NSSM_ERR_UNSUPPORTED, "batch too large for the persistent FLUSH");
    return launch_step<PB, NC, COLD, kTPR>(sp, batch, st);
  }
  int sms = 0;
  int rc = sm_count(&sms);
  if (rc) return rc;
  if constexpr (COLD == nssm::COLD_FP8 && IOBF) {
    if (sp.P == 80) return launch_c<PB, NC, COLD, IOBF, 10, FLUSH_ONLY>(sp, batch, st, ring_ok, sms);
    if (sp.P == 64) return launch_c<PB, NC, COLD, IOBF, 8, FLUSH_ONLY>(sp, batch, st, ring_ok, sms);
  }
  return launch_both<PB, NC, COLD, IOBF, 0, 0, FLUSH_ONLY>(sp, batch, st, ring_ok, sms);
}

// Whether the persistent TMA-pipelined kernels take this call (else the simple kernel runs):
// 16-byte aligned pool tiles and input rows, headdim % 4 == 0 and <= kPMaxPersistent.
template <int PB, int NC, int COLD>
inline bool persistent_ok(const nssm::StepParams& sp, bool* ring_ok) {
  constexpr int N = PB + NC;
  const int iob = io_bytes(sp.io_dtype);
  auto a16 = [](long long v) { return (v % 16) == 0; };
  const bool tma_ok = sp.P % 4 == 0 && sp.P <= nssm::kPMaxPersistent && aligned16(sp.hot) &&
                      aligned16(sp.cold) && (COLD != COLD_FP8 || aligned16(sp.scale)) && aligned16(sp.x) &&
                      a16(sp.x_sb * iob) && a16(sp.x_sh * iob) && a16((long long)sp.P * iob) &&
                      aligned16(sp.B) && aligned16(sp.C) && a16(sp.B_sb * iob) && a16(sp.C_sb * iob) &&
                      a16((long long)N * iob);
  *ring_ok = sp.c <= nssm::kRingInStage && aligned16(sp.ring_x) && aligned16(sp.ring_b) &&
             aligned16(sp.ring_dt) && a16((long long)sp.c * sp.P * iob) && a16((long long)sp.c * NC * 4);
  return tma_ok;
}

template <int PB, int NC, int COLD>
inline int launch_tiered(const nssm::StepParams& sp, int batch, cudaStream_t st) {
#ifdef NSSM_FORCE_SIMPLE
  return launch_step<PB, NC, COLD, kTPR>(sp, batch, st);
#endif
  bool ring_ok = false;
  if (!persistent_ok<PB, NC, COLD>(sp, &ring_ok)) return launch_step<PB, NC, COLD, kTPR>(sp, batch, st);
  if (sp.io_dtype == NSSM_BF16) return launch_persistent<PB, NC, COLD, true>(sp, batch, st, ring_ok);
  return launch_persistent<PB, NC, COLD, false>(sp, batch, st, ring_ok);
}

// ---- self-speculative decoding ---------------------------------------------
template <int PB, int NC>
int launch_draft(const nssm::SpecParams& q, int batch, cudaStream_t st) {
  dim3 grid(q.sp.H, batch);
  const int threads = round_up(q.sp.P * kTPR, 32);
  nssm::draft_step_kernel<PB, PB + NC, kTPR><<<grid, threads, 0, st>>>(q);
  return cuda_check("draft_step_kernel launch");
}

// The commit's FLUSH runs on the persistent kernels only; verify and commit refuse a call
// those kernels cannot take before launching anything.
template <int PB, int NC, int COLD>
int launch_verify(const nssm::SpecParams& q, int batch, cudaStream_t st) {
  bool ring_ok = false;
  if (!persistent_ok<PB, NC, COLD>(q.sp, &ring_ok))
    return fail(NSSM_ERR_UNSUPPORTED, "verify / commit need the persistent kernels' layout (16-byte aligned rows, "
                                      "headdim %% 4 == 0 and <= %d)", nssm::kPMaxPersistent);
  // the tokens are staged in 16-byte chunks: token strides and headdim in whole chunks
  const int iob = io_bytes(q.sp.io_dtype);
  const int epc = 16 / iob;
  if ((q.x_st * iob) % 16 || (q.B_st * iob) % 16 || (q.C_st * iob) % 16 || q.sp.P % epc)
    return fail(NSSM_ERR_UNSUPPORTED, "verify needs token strides of whole 16-byte chunks and headdim %% %d == 0", epc);
  dim3 grid(q.sp.H, batch);
  const int threads = round_up(q.sp.P * 2, 32);   // two threads per headdim row
  const size_t smem = sizeof(float) * nssm::verify_smem_floats<PB, NC, COLD>(q.sp.P);
  auto fn = q.sp.io_dtype == NSSM_BF16 ? nssm::verify_step_kernel<PB, NC, COLD, true>
                                       : nssm::verify_step_kernel<PB, NC, COLD, false>;
  if (smem > 48 * 1024) {
    int rc = ensure_smem_attr(reinterpret_cast<const void*>(fn));
    if (rc) return rc;
  }
  fn<<<grid, threads, smem, st>>>(q);
  return cuda_check("verify_step_kernel launch");
}

template <int PB, int NC, int COLD>
int launch_commit(const nssm::SpecParams& q, int batch, cudaStream_t st) {
  bool ring_ok = false;
  if (!persistent_ok<PB, NC, COLD>(q.sp, &ring_ok))
    return fail(NSSM_ERR_UNSUPPORTED, "verify / commit need the persistent kernels' layout (16-byte aligned rows, "
                                      "headdim %% 4 == 0 and <= %d)", nssm::kPMaxPersistent);
  // the tokens are staged in 16-byte chunks: token strides, headdim and the ring rows in whole chunks
  const int iob = io_bytes(q.sp.io_dtype);
  if ((q.x_st * iob) % 16 || (q.B_st * iob) % 16 || q.sp.P % (16 / iob) || !aligned16(q.sp.ring_x) ||
      !aligned16(q.sp.ring_b))
    return fail(NSSM_ERR_UNSUPPORTED, "commit needs token strides, headdim and ring rows of whole 16-byte chunks");
  dim3 grid(q.sp.H, batch);
  const int threads = round_up(q.sp.P * kTPR, 32);
  if (q.sp.io_dtype == NSSM_BF16)
    nssm::commit_step_kernel<PB, PB + NC, kTPR, true><<<grid, threads, 0, st>>>(q);
  else
    nssm::commit_step_kernel<PB, PB + NC, kTPR, false><<<grid, threads, 0, st>>>(q);
  int rc = cuda_check("commit_step_kernel launch");
  if (rc) return rc;
  nssm::StepParams fs = q.sp;   // FLUSH of the rows the commit completed (the others are -1)
  fs.idx = q.flush_idx;
  fs.pad = -1;
  if (fs.io_dtype == NSSM_BF16) return launch_persistent<PB, NC, COLD, true, true>(fs, batch, st, ring_ok);
  return launch_persistent<PB, NC, COLD, false, true>(fs, batch, st, ring_ok);
}

template <int PB, int NC, int COLD, int TPR>
int launch_split(const nssm::SplitParams& sp, int batch, cudaStream_t st) {
  dim3 grid(sp.H, batch);
  const int threads = round_up(sp.P * TPR, 32);
  nssm::prefill_split_kernel<PB, NC, COLD, TPR><<<grid, threads, 0, st>>>(sp);
  return cuda_check("prefill_split_kernel launch");
}

template <int PB, int NC, int COLD, int TPR>
int launch_mat(const nssm::MatParams& mp, int batch, cudaStream_t st) {
  dim3 grid(mp.H, batch);
  const int threads = round_up(mp.P * TPR, 32);
  nssm::materialize_kernel<PB, NC, COLD, TPR><<<grid, threads, 2 * nssm::kMaxChunk * sizeof(float), st>>>(mp);
  return cuda_check("materialize_kernel launch");
}

// Instances compiled: dstate 128, hot width 16/32/64, cold fp8/bf16/fp32.
enum Op { OP_STEP, OP_SPLIT, OP_MAT, OP_DRAFT, OP_VERIFY, OP_COMMIT };

template <int PB, int COLD>
int run_op(Op op, const void* params, int batch, cudaStream_t st) {
  constexpr int NC = 128 - PB;
  switch (op) {
    case OP_STEP: return launch_tiered<PB, NC, COLD>(*static_cast<const nssm::StepParams*>(params), batch, st);
    case OP_SPLIT: return launch_split<PB, NC, COLD, kTPR>(*static_cast<const nssm::SplitParams*>(params), batch, st);
    case OP_MAT: return launch_mat<PB, NC, COLD, kTPR>(*static_cast<const nssm::MatParams*>(params), batch, st);
    case OP_DRAFT: return launch_draft<PB, NC>(*static_cast<const nssm::SpecParams*>(params), batch, st);
    case OP_VERIFY: return launch_verify<PB, NC, COLD>(*static_cast<const nssm::SpecParams*>(params), batch, st);
    case OP_COMMIT: return launch_commit<PB, NC, COLD>(*static_cast<const nssm::SpecParams*>(params), batch, st);
  }
  return fail(NSSM_ERR_INVALID, "unknown op");
}

template <int PB>
int run_cold(Op op, int cold, const void* params, int batch, cudaStream_t st) {
  switch (cold) {
    case NSSM_F8E4M3: return run_op<PB, COLD_FP8>(op, params, batch, st);
    case NSSM_BF16: return run_op<PB, COLD_BF16>(op, params, batch, st);
    case NSSM_F32: return run_op<PB, COLD_F32>(op, params, batch, st);
  }
  return fail(NSSM_ERR_INVALID, "cold_dtype %d is not one of F32/BF16/F8E4M3", cold);
}

int dispatch_pb16(Op op, int cold, const void* params, int batch, cudaStream_t st);
int dispatch_pb32(Op op, int cold, const void* params, int batch, cudaStream_t st);
int dispatch_pb64(Op op, int cold, const void* params, int batch, cudaStream_t st);

}  // namespace nssm_host
