// nssm_chunk_scan: the prefill chunked scan entry point (argument checks, the TMA tensor maps
// of the C / B / x tiles, and the persistent launch of nssm::scan::chunk_scan_kernel).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <math.h>

#include <mutex>

#include "nested_ssm.h"
#include "nssm_scan.cuh"

namespace nssm_host {
int fail(int code, const char* fmt, ...);
}

namespace {

using nssm_host::fail;

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

int get_encode(PFN_cuTensorMapEncodeTiled_v12000* out) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    else
      cudaGetLastError();
  });
  if (!g_encode) return fail(NSSM_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  *out = g_encode;
  return NSSM_OK;
}

// A [batch][T][width] bf16 tensor (token stride st, batch stride sb, in elements) as a 3-D map
// {width, T, batch} with box {box_w, 128, 1}: one 128-token tile of box_w columns, landing in
// shared memory as [128 tokens][box_w] with the given swizzle.
int encode_tiles(PFN_cuTensorMapEncodeTiled_v12000 enc, CUtensorMap* m, const void* base, int width, int T,
                 int batch, int64_t st, int64_t sb, int box_w, CUtensorMapSwizzle sw, const char* what) {
  cuuint64_t dims[3] = {(cuuint64_t)width, (cuuint64_t)T, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)st * 2, (cuuint64_t)(sb > 0 ? sb : st) * 2};
  cuuint32_t box[3] = {(cuuint32_t)box_w, (cuuint32_t)nssm::scan::kQ, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(NSSM_ERR_INVALID, "tensor map of %s rejected (CUresult %d)", what, (int)r);
  return NSSM_OK;
}

template <int P>
int launch(const nssm::scan::ScanParams& sp, const CUtensorMap& mC, const CUtensorMap& mB, const CUtensorMap& mX,
           cudaStream_t st) {
  using L = nssm::scan::Smem<P>;
  static_assert(L::kBytes <= 232448, "shared memory beyond the per-CTA limit");
  cudaError_t e = cudaFuncSetAttribute(nssm::scan::chunk_scan_kernel<P>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       L::kBytes);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(NSSM_ERR_CUDA, "cudaFuncSetAttribute(chunk_scan_kernel): %s", cudaGetErrorString(e));
  }
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    cudaGetLastError();
    return fail(NSSM_ERR_CUDA, "device query failed");
  }
  const int items = sp.batch * sp.H;
  const int grid = items < sms ? items : sms;   // one persistent CTA per SM (226 KB shared memory each)
  nssm::scan::chunk_scan_kernel<P><<<grid, nssm::scan::kThreads, L::kBytes, st>>>(sp, mC, mB, mX);
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
  if (a->seqlen < 0 || a->seqlen > (1 << 30)) return fail(NSSM_ERR_INVALID, "seqlen %d out of range", a->seqlen);
  if (a->batch == 0 || a->seqlen == 0) return NSSM_OK;
  if (a->nheads <= 0 || a->nheads > 65535 || a->ngroups <= 0 || a->nheads % a->ngroups)
    return fail(NSSM_ERR_INVALID, "nheads %d / ngroups %d", a->nheads, a->ngroups);
  if ((int64_t)a->batch * a->nheads > (1 << 30)) return fail(NSSM_ERR_INVALID, "batch * nheads too large");
  if (a->dstate != nssm::scan::kN) return fail(NSSM_ERR_UNSUPPORTED, "chunk scan compiled for dstate 128 only");
  if (a->chunk_size != nssm::scan::kQ) return fail(NSSM_ERR_UNSUPPORTED, "chunk scan compiled for chunk_size 128 only");
  if (a->headdim != 64 && a->headdim != 80)
    return fail(NSSM_ERR_UNSUPPORTED, "headdim %d not compiled (supported: 64, 80)", a->headdim);
  if (a->io_dtype != NSSM_BF16) return fail(NSSM_ERR_UNSUPPORTED, "chunk scan io_dtype must be BF16");
  if (a->dt_dtype != NSSM_F32 && a->dt_dtype != NSSM_BF16) return fail(NSSM_ERR_INVALID, "dt_dtype must be F32 or BF16");
  if (!a->x || !a->dt || !a->A || !a->B || !a->C || !a->y) return fail(NSSM_ERR_INVALID, "x/dt/A/B/C/y must be non-NULL");
  if (!(a->dt_min <= a->dt_max) || isnan(a->dt_min)) return fail(NSSM_ERR_INVALID, "dt limits [%g, %g]", a->dt_min, a->dt_max);
  // TMA tiles and 16-byte stores of 8 bf16: bases aligned, strides multiples of 8 elements
  if (!al16(a->x) || !al16(a->B) || !al16(a->C) || !al16(a->y))
    return fail(NSSM_ERR_INVALID, "x / B / C / y must be 16-byte aligned");
  if ((a->x_stride_b | a->x_stride_t | a->B_stride_b | a->B_stride_t | a->C_stride_b | a->C_stride_t | a->y_stride_b |
       a->y_stride_t) & 7)
    return fail(NSSM_ERR_INVALID, "x / B / C / y strides must be multiples of 8 elements");
  if (a->x_stride_t < (int64_t)a->nheads * a->headdim || a->y_stride_t < (int64_t)a->nheads * a->headdim ||
      a->B_stride_t < (int64_t)a->ngroups * a->dstate || a->C_stride_t < (int64_t)a->ngroups * a->dstate)
    return fail(NSSM_ERR_INVALID, "token strides smaller than a token's row");
  PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
  int rc = get_encode(&enc);
  if (rc) return rc;
  // C, B: two 64-column boxes (128-byte swizzle) per 128-column group tile; x: 16-column boxes
  // (32-byte swizzle)
  alignas(64) CUtensorMap mC, mB, mX;
  const int gw = a->ngroups * a->dstate, xw = a->nheads * a->headdim;
  if ((rc = encode_tiles(enc, &mC, a->C, gw, a->seqlen, a->batch, a->C_stride_t, a->C_stride_b, 64,
                         CU_TENSOR_MAP_SWIZZLE_128B, "C")) ||
      (rc = encode_tiles(enc, &mB, a->B, gw, a->seqlen, a->batch, a->B_stride_t, a->B_stride_b, 64,
                         CU_TENSOR_MAP_SWIZZLE_128B, "B")) ||
      (rc = encode_tiles(enc, &mX, a->x, xw, a->seqlen, a->batch, a->x_stride_t, a->x_stride_b, 16,
                         CU_TENSOR_MAP_SWIZZLE_32B, "x")))
    return rc;
  nssm::scan::ScanParams sp{};
  sp.batch = a->batch; sp.T = a->seqlen; sp.H = a->nheads; sp.G = a->ngroups;
  sp.x = static_cast<const __nv_bfloat16*>(a->x); sp.x_sb = a->x_stride_b; sp.x_st = a->x_stride_t;
  sp.dt = a->dt; sp.dt_sb = a->dt_stride_b; sp.dt_st = a->dt_stride_t; sp.dt_bf16 = a->dt_dtype == NSSM_BF16;
  sp.softplus = a->dt_softplus != 0; sp.dt_lo = a->dt_min; sp.dt_hi = a->dt_max;
  sp.A = a->A; sp.D = a->D; sp.dt_bias = a->dt_bias;
  sp.init = a->initial_states; sp.init_sb = a->init_stride_b;
  sp.y = static_cast<__nv_bfloat16*>(a->y); sp.y_sb = a->y_stride_b; sp.y_st = a->y_stride_t;
  sp.fin = a->final_states; sp.fin_sb = a->final_stride_b;
  sp.status = a->status;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return a->headdim == 64 ? launch<64>(sp, mC, mB, mX, st) : launch<80>(sp, mC, mB, mX, st);
}

}  // extern "C"
