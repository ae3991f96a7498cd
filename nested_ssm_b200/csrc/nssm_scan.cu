// nssm_chunk_scan: the prefill chunked scan entry point (argument checks and launch of
// nssm::scan::chunk_scan_kernel).
#include <cuda_runtime.h>
#include <math.h>

#include "nested_ssm.h"
#include "nssm_scan.cuh"

namespace nssm_host {
int fail(int code, const char* fmt, ...);
}

namespace {

using nssm_host::fail;

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <int P>
int launch(const nssm::scan::ScanParams& sp, cudaStream_t st) {
  using L = nssm::scan::Smem<P>;
  static_assert(L::kBytes <= 232448, "shared memory beyond the per-CTA limit");
  cudaError_t e = cudaFuncSetAttribute(nssm::scan::chunk_scan_kernel<P>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       L::kBytes);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(NSSM_ERR_CUDA, "cudaFuncSetAttribute(chunk_scan_kernel): %s", cudaGetErrorString(e));
  }
  dim3 grid(sp.H, sp.batch);
  nssm::scan::chunk_scan_kernel<P><<<grid, nssm::scan::kThreads, L::kBytes, st>>>(sp);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(NSSM_ERR_CUDA, "chunk_scan_kernel launch: %s", cudaGetErrorString(e));
  return NSSM_OK;
}

}  // namespace

extern "C" {

size_t nssm_sizeof_scan_args(void) { return sizeof(nssm_scan_args); }

int nssm_chunk_scan(const nssm_scan_args* a, void* stream) {
  if (!a) return fail(NSSM_ERR_INVALID, "args is NULL");
  if (a->batch < 0 || a->batch > 65535) return fail(NSSM_ERR_INVALID, "batch %d outside [0, 65535]", a->batch);
  if (a->seqlen < 0) return fail(NSSM_ERR_INVALID, "seqlen %d < 0", a->seqlen);
  if (a->batch == 0 || a->seqlen == 0) return NSSM_OK;
  if (a->nheads <= 0 || a->nheads > 65535 || a->ngroups <= 0 || a->nheads % a->ngroups)
    return fail(NSSM_ERR_INVALID, "nheads %d / ngroups %d", a->nheads, a->ngroups);
  if (a->dstate != nssm::scan::kN) return fail(NSSM_ERR_UNSUPPORTED, "chunk scan compiled for dstate 128 only");
  if (a->chunk_size != nssm::scan::kQ) return fail(NSSM_ERR_UNSUPPORTED, "chunk scan compiled for chunk_size 128 only");
  if (a->headdim != 64 && a->headdim != 80)
    return fail(NSSM_ERR_UNSUPPORTED, "headdim %d not compiled (supported: 64, 80)", a->headdim);
  if (a->io_dtype != NSSM_BF16) return fail(NSSM_ERR_UNSUPPORTED, "chunk scan io_dtype must be BF16");
  if (a->dt_dtype != NSSM_F32 && a->dt_dtype != NSSM_BF16) return fail(NSSM_ERR_INVALID, "dt_dtype must be F32 or BF16");
  if (!a->x || !a->dt || !a->A || !a->B || !a->C || !a->y) return fail(NSSM_ERR_INVALID, "x/dt/A/B/C/y must be non-NULL");
  if (!(a->dt_min <= a->dt_max) || isnan(a->dt_min)) return fail(NSSM_ERR_INVALID, "dt limits [%g, %g]", a->dt_min, a->dt_max);
  // 16-byte cp.async / vector stores of 8 bf16: bases aligned, strides multiples of 8 elements
  if (!al16(a->x) || !al16(a->B) || !al16(a->C) || !al16(a->y))
    return fail(NSSM_ERR_INVALID, "x / B / C / y must be 16-byte aligned");
  if ((a->x_stride_b | a->x_stride_t | a->B_stride_b | a->B_stride_t | a->C_stride_b | a->C_stride_t | a->y_stride_b |
       a->y_stride_t) & 7)
    return fail(NSSM_ERR_INVALID, "x / B / C / y strides must be multiples of 8 elements");
  if (a->x_stride_t < (int64_t)a->nheads * a->headdim || a->y_stride_t < (int64_t)a->nheads * a->headdim ||
      a->B_stride_t < (int64_t)a->ngroups * a->dstate || a->C_stride_t < (int64_t)a->ngroups * a->dstate)
    return fail(NSSM_ERR_INVALID, "token strides smaller than a token's row");
  nssm::scan::ScanParams sp{};
  sp.batch = a->batch; sp.T = a->seqlen; sp.H = a->nheads; sp.G = a->ngroups;
  sp.x = static_cast<const __nv_bfloat16*>(a->x); sp.x_sb = a->x_stride_b; sp.x_st = a->x_stride_t;
  sp.dt = a->dt; sp.dt_sb = a->dt_stride_b; sp.dt_st = a->dt_stride_t; sp.dt_bf16 = a->dt_dtype == NSSM_BF16;
  sp.softplus = a->dt_softplus != 0; sp.dt_lo = a->dt_min; sp.dt_hi = a->dt_max;
  sp.A = a->A; sp.D = a->D; sp.dt_bias = a->dt_bias;
  sp.B = static_cast<const __nv_bfloat16*>(a->B); sp.B_sb = a->B_stride_b; sp.B_st = a->B_stride_t;
  sp.C = static_cast<const __nv_bfloat16*>(a->C); sp.C_sb = a->C_stride_b; sp.C_st = a->C_stride_t;
  sp.init = a->initial_states; sp.init_sb = a->init_stride_b;
  sp.y = static_cast<__nv_bfloat16*>(a->y); sp.y_sb = a->y_stride_b; sp.y_st = a->y_stride_t;
  sp.fin = a->final_states; sp.fin_sb = a->final_stride_b;
  sp.status = a->status;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return a->headdim == 64 ? launch<64>(sp, st) : launch<80>(sp, st);
}

}  // extern "C"
