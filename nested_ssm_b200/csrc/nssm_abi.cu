// extern "C" entry points of libnested_ssm: argument validation, dispatch to
// the compiled (dstate, hot width, cold dtype) instances, and launches on the
// caller's stream.  Nothing here allocates device memory or synchronises.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

#include "nssm_host.cuh"
#include "nssm_norm.cuh"

namespace nssm_host {

thread_local std::string g_last_error;
thread_local bool g_norm_fused = false;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_check(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(NSSM_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return NSSM_OK;
}

// Per-(kernel, smem size, device) cache of resident CTAs per SM.
struct OccEntry { const void* fn; int smem; int dev; int occ; };
OccEntry g_occ[64];
std::atomic<int> g_nocc{0};

int occupancy(const void* fn, int smem, int threads, int* occ_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return cuda_check("cudaGetDevice");
  const int n = g_nocc.load(std::memory_order_acquire);
  for (int i = 0; i < n && i < 64; ++i)
    if (g_occ[i].fn == fn && g_occ[i].smem == smem && g_occ[i].dev == dev) {
      *occ_out = g_occ[i].occ;
      return NSSM_OK;
    }
  // The attribute is one value per function: always opt in to the device maximum so
  // a later launch with a larger layout (another c / batch) stays legal.
  int optin = 0;
  if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
    return cuda_check("cudaDeviceGetAttribute(smem opt-in)");
  if (smem > optin) {
    *occ_out = 0;
    return NSSM_OK;
  }
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, optin) != cudaSuccess)
    return cuda_check("cudaFuncSetAttribute(persistent kernel)");
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, threads, smem) != cudaSuccess)
    return cuda_check("cudaOccupancyMaxActiveBlocksPerMultiprocessor");
  const int slot = g_nocc.fetch_add(1, std::memory_order_acq_rel);
  if (slot < 64) g_occ[slot] = OccEntry{fn, smem, dev, occ};
  *occ_out = occ;
  return NSSM_OK;
}

// Per-(kernel, device) record that the dynamic shared-memory opt-in was set.
struct AttrEntry { const void* fn; int dev; };
AttrEntry g_attr[64];
std::atomic<int> g_nattr{0};

int ensure_smem_attr(const void* fn) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return cuda_check("cudaGetDevice");
  const int n = g_nattr.load(std::memory_order_acquire);
  for (int i = 0; i < n && i < 64; ++i)
    if (g_attr[i].fn == fn && g_attr[i].dev == dev) return NSSM_OK;
  int optin = 0;
  if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
    return cuda_check("cudaDeviceGetAttribute(smem opt-in)");
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, optin) != cudaSuccess)
    return cuda_check("cudaFuncSetAttribute(max dynamic shared memory)");
  const int slot = g_nattr.fetch_add(1, std::memory_order_acq_rel);
  if (slot < 64) g_attr[slot] = AttrEntry{fn, dev};
  return NSSM_OK;
}

int smem_optin(int* out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return cuda_check("cudaGetDevice");
  if (cudaDeviceGetAttribute(out, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
    return cuda_check("cudaDeviceGetAttribute(smem opt-in)");
  return NSSM_OK;
}

std::atomic<uint32_t> g_wait_polls{nssm::kSpinLimit};

uint32_t wait_polls() { return g_wait_polls.load(std::memory_order_relaxed); }

std::atomic<int> g_inject_stuck{0};

int inject_stuck() { return g_inject_stuck.load(std::memory_order_relaxed); }

int sm_count(int* out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return cuda_check("cudaGetDevice");
  if (cudaDeviceGetAttribute(out, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return cuda_check("cudaDeviceGetAttribute(SM count)");
  return NSSM_OK;
}


}  // namespace nssm_host

namespace {

using namespace nssm_host;

int dispatch(Op op, int N, int pb, int cold, const void* params, int batch, cudaStream_t st) {
  if (N != 128) return fail(NSSM_ERR_UNSUPPORTED, "dstate %d not compiled (supported: 128)", N);
  switch (pb) {
    case 16: return dispatch_pb16(op, cold, params, batch, st);
    case 32: return dispatch_pb32(op, cold, params, batch, st);
    case 64: return dispatch_pb64(op, cold, params, batch, st);
  }
  return fail(NSSM_ERR_UNSUPPORTED, "hot_dim %d not compiled for dstate %d (supported: 16, 32, 64)", pb, N);
}

// ---- validation ---------------------------------------------------------
int check_pool(const nssm_pool* pl) {
  if (!pl) return fail(NSSM_ERR_INVALID, "pool is NULL");
  if (pl->num_slots <= 0 || pl->nheads <= 0 || pl->headdim <= 0 || pl->dstate <= 0 || pl->ngroups <= 0)
    return fail(NSSM_ERR_INVALID, "pool dims must be positive (S=%d H=%d P=%d N=%d G=%d)", pl->num_slots,
                pl->nheads, pl->headdim, pl->dstate, pl->ngroups);
  if (pl->nheads % pl->ngroups) return fail(NSSM_ERR_INVALID, "nheads %d not divisible by ngroups %d", pl->nheads, pl->ngroups);
  if (pl->hot_dim <= 0 || pl->hot_dim >= pl->dstate)
    return fail(NSSM_ERR_INVALID, "hot_dim %d must be in [1, dstate) (use nssm_fresh_step for an all-hot state)", pl->hot_dim);
  if (pl->chunk < 1 || pl->chunk > nssm::kMaxChunk)
    return fail(NSSM_ERR_INVALID, "chunk %d outside [1, %d]", pl->chunk, nssm::kMaxChunk);
  if (pl->headdim * kTPR > 128 * kTPR) return fail(NSSM_ERR_UNSUPPORTED, "headdim %d > 128", pl->headdim);
  if (pl->io_dtype != NSSM_F32 && pl->io_dtype != NSSM_BF16)
    return fail(NSSM_ERR_INVALID, "io_dtype %d must be F32 or BF16", pl->io_dtype);
  if (!pl->hot || !pl->cold || !pl->glog || !pl->t || !pl->ring_x || !pl->ring_dt || !pl->ring_b)
    return fail(NSSM_ERR_INVALID, "a pool buffer is NULL");
  if (pl->cold_dtype == NSSM_F8E4M3 && !pl->cold_scale) return fail(NSSM_ERR_INVALID, "fp8 cold needs cold_scale");
  if (!aligned16(pl->hot) || !aligned16(pl->cold) || (pl->cold_scale && !aligned16(pl->cold_scale)))
    return fail(NSSM_ERR_INVALID, "hot / cold / cold_scale must be 16-byte aligned");
  return NSSM_OK;
}

int check_args(const nssm_step_args* a, int H) {
  if (!a) return fail(NSSM_ERR_INVALID, "args is NULL");
  if (a->batch < 0) return fail(NSSM_ERR_INVALID, "batch %d < 0", a->batch);
  if (a->batch > 65535) return fail(NSSM_ERR_UNSUPPORTED, "batch %d > 65535 rows per call", a->batch);
  if (!a->x || !a->dt || !a->A || !a->B || !a->C || !a->out) return fail(NSSM_ERR_INVALID, "x/dt/A/B/C/out must be non-NULL");
  if (a->io_dtype != NSSM_F32 && a->io_dtype != NSSM_BF16) return fail(NSSM_ERR_INVALID, "io_dtype must be F32 or BF16");
  if (a->dt_dtype != NSSM_F32 && a->dt_dtype != NSSM_BF16) return fail(NSSM_ERR_INVALID, "dt_dtype must be F32 or BF16");
  if (a->out_dtype != NSSM_F32 && a->out_dtype != NSSM_BF16) return fail(NSSM_ERR_INVALID, "out_dtype must be F32 or BF16");
  if (a->mode < NSSM_MODE_STALE || a->mode > NSSM_MODE_COLDOFF) return fail(NSSM_ERR_INVALID, "mode %d unknown", a->mode);
  (void)H;
  return NSSM_OK;
}

// Rotate B and C into the workspace (if R given); fills sp.B / sp.C.
int launch_rot(const nssm::RotParams& rp, int rows_total, int G, cudaStream_t st) {
  // 80 KB of dynamic shared memory: opt in once per device
  static std::atomic<unsigned long long> attr_done{0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return cuda_check("cudaGetDevice");
  const unsigned long long bit = 1ull << (dev & 63);
  constexpr int smem = nssm::rot_smem_bytes(128);
  if (!(attr_done.load(std::memory_order_acquire) & bit)) {
    if (cudaFuncSetAttribute(nssm::rot_kernel<128, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
            cudaSuccess ||
        cudaFuncSetAttribute(nssm::rot_kernel<128, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
            cudaSuccess)
      return cuda_check("cudaFuncSetAttribute(rot_kernel)");
    attr_done.fetch_or(bit, std::memory_order_acq_rel);
  }
  dim3 grid((unsigned)((rows_total + nssm::kRotTile - 1) / nssm::kRotTile), (unsigned)G, 128 / nssm::kRotHalf);
  if (rp.dtype == NSSM_BF16)
    nssm::rot_kernel<128, true><<<grid, nssm::kRotThreads, smem, st>>>(rp, rows_total);
  else
    nssm::rot_kernel<128, false><<<grid, nssm::kRotThreads, smem, st>>>(rp, rows_total);
  return cuda_check("rot_kernel launch");
}

int maybe_rotate(const nssm_step_args* a, int G, int N, nssm::StepParams& sp, cudaStream_t st) {
  sp.B = a->B; sp.B_sb = a->B_stride_b;
  sp.C = a->C; sp.C_sb = a->C_stride_b;
  if (!a->R || a->batch == 0) return NSSM_OK;
  const size_t need = nssm_step_workspace_bytes(a->batch, G, N, a->io_dtype, 1);
  if (!a->workspace || a->workspace_bytes < need)
    return fail(NSSM_ERR_INVALID, "workspace of %zu bytes needed for the rotation (got %zu)", need, a->workspace_bytes);
  if (N != 128) return fail(NSSM_ERR_UNSUPPORTED, "rotation compiled for dstate 128 only");
  if (reinterpret_cast<uintptr_t>(a->R) % 16) return fail(NSSM_ERR_INVALID, "R must be 16-byte aligned");
  const size_t half = need / 2;
  nssm::RotParams rp{};
  rp.x0 = a->B; rp.xs0 = a->B_stride_b;
  rp.x1 = a->C; rp.xs1 = a->C_stride_b;
  rp.o0 = a->workspace; rp.os0 = (int64_t)G * N;
  rp.o1 = static_cast<char*>(a->workspace) + half; rp.os1 = (int64_t)G * N;
  rp.R = a->R; rp.T = a->batch; rp.G = G; rp.dtype = a->io_dtype;
  int rc = launch_rot(rp, 2 * a->batch, G, st);
  if (rc) return rc;
  sp.B = rp.o0; sp.B_sb = rp.os0;
  sp.C = rp.o1; sp.C_sb = rp.os1;
  return NSSM_OK;
}

template <int K, int L, bool IOBF, bool WBF, bool LD>
int launch_conv(const nssm::ConvParams& cp, int batch, int G, cudaStream_t st) {
  // the B/C kernel uses 84 KB of dynamic shared memory: opt in once per device
  static std::atomic<unsigned long long> attr_done{0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return cuda_check("cudaGetDevice");
  const unsigned long long bit = 1ull << (dev & 63);
  constexpr int smem = nssm::conv_smem_bytes(128);
  auto kbc = nssm::conv_step_kernel<128, K, L, IOBF, WBF, LD>;
  if (!(attr_done.load(std::memory_order_acquire) & bit)) {
    if (cudaFuncSetAttribute(kbc, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return cuda_check("cudaFuncSetAttribute(conv_step_kernel)");
    attr_done.fetch_or(bit, std::memory_order_acq_rel);
  }
  dim3 gx((unsigned)((cp.I + 4 * nssm::kConvXThreads - 1) / (4 * nssm::kConvXThreads)), (unsigned)batch);
  nssm::conv_x_kernel<K, L, IOBF, WBF, LD><<<gx, nssm::kConvXThreads, 0, st>>>(cp);
  int rc = cuda_check("conv_x_kernel launch");
  if (rc) return rc;
  dim3 grid((unsigned)((batch + nssm::kConvTile - 1) / nssm::kConvTile), (unsigned)G, 2);
  kbc<<<grid, nssm::kConvThreads, smem, st>>>(cp);
  return cuda_check("conv_step_kernel launch");
}

void fill_inputs(const nssm_step_args* a, nssm::StepParams& sp) {
  sp.x = a->x; sp.x_sb = a->x_stride_b; sp.x_sh = a->x_stride_h;
  sp.dt = a->dt; sp.dt_sb = a->dt_stride_b; sp.dt_sh = a->dt_stride_h; sp.dt_dtype = a->dt_dtype;
  sp.softplus = a->dt_softplus;
  sp.io_dtype = a->io_dtype;
  sp.A = a->A; sp.D = a->D; sp.dt_bias = a->dt_bias; sp.dt_min = a->dt_min;
  sp.mode = a->mode;
  sp.idx = a->state_batch_indices; sp.pad = a->pad_slot_id;
  sp.out = a->out; sp.out_sb = a->out_stride_b; sp.out_sh = a->out_stride_h; sp.out_dtype = a->out_dtype;
  sp.status = a->status;
}

// The gated norm requested with a step: validated here; fused into STEP when its gate rows
// can be bulk-copied (16-byte aligned), else applied by the norm kernel after the step.
int check_norm(const nssm_step_args* a, int H, int P, int G) {
  if (!a->norm_gate) return NSSM_OK;
  if (!a->norm_weight) return fail(NSSM_ERR_INVALID, "norm_gate given without norm_weight");
  if (a->out_dtype != a->io_dtype)
    return fail(NSSM_ERR_INVALID, "the fused norm needs out_dtype == io_dtype (gate and y share it)");
  if (a->norm_weight_dtype != NSSM_F32 && a->norm_weight_dtype != NSSM_BF16)
    return fail(NSSM_ERR_INVALID, "norm_weight_dtype must be F32 or BF16");
  if (a->norm_group_size != (H / G) * P)
    return fail(NSSM_ERR_INVALID, "norm_group_size %d must be one SSM group of a row, (nheads/ngroups)*headdim = %d",
                a->norm_group_size, (H / G) * P);
  if (a->out_stride_h != P) return fail(NSSM_ERR_INVALID, "the fused norm needs out rows [nheads*headdim] contiguous");
  if (!(a->norm_eps >= 0.0f)) return fail(NSSM_ERR_INVALID, "norm_eps must be >= 0");
  return NSSM_OK;
}

bool norm_fusable(const nssm_step_args* a) {
  const int iob = io_bytes(a->io_dtype);
  return aligned16(a->norm_gate) && (a->norm_gate_stride_b * iob) % 16 == 0;
}

int run_norm_after_step(const nssm_step_args* a, int H, int P, cudaStream_t st) {
  nssm::NormParams np{};
  np.y = a->out; np.y_sb = a->out_stride_b; np.gate = a->norm_gate; np.g_sb = a->norm_gate_stride_b;
  np.weight = a->norm_weight; np.w_dtype = a->norm_weight_dtype; np.eps = a->norm_eps;
  np.dim = H * P; np.gs = a->norm_group_size; np.dtype = a->out_dtype; np.out = a->out; np.o_sb = a->out_stride_b;
  if (np.gs > nssm::kNormThreads * nssm::kNormMaxPer) return fail(NSSM_ERR_UNSUPPORTED, "norm group size %d too large", np.gs);
  dim3 grid((unsigned)(np.dim / np.gs), (unsigned)a->batch);
  nssm::gated_rmsnorm_kernel<<<grid, nssm::kNormThreads, 0, st>>>(np);   // in place: reads a group, then writes it
  return cuda_check("gated_rmsnorm_kernel launch (after the step)");
}

void fill_pool(const nssm_pool* pool, nssm::StepParams& sp) {
  sp.hot = pool->hot; sp.cold = pool->cold; sp.scale = pool->cold_scale;
  sp.glog = pool->glog; sp.t = pool->t;
  sp.ring_x = pool->ring_x; sp.ring_dt = pool->ring_dt; sp.ring_b = pool->ring_b;
  sp.S = pool->num_slots; sp.H = pool->nheads; sp.P = pool->headdim; sp.G = pool->ngroups; sp.c = pool->chunk;
}

// Checks shared by the self-speculative entry points; fills sp (pool + token-0 inputs) and the
// token strides of q.
int spec_prepare(const nssm_pool* pool, const nssm_step_args* a, const nssm_token_args* tok, nssm::StepParams& sp,
                 nssm::SpecParams& q) {
  int rc = check_pool(pool);
  if (rc) return rc;
  rc = check_args(a, pool->nheads);
  if (rc) return rc;
  if (a->io_dtype != pool->io_dtype)
    return fail(NSSM_ERR_INVALID, "args io_dtype %d differs from the pool's ring dtype %d", a->io_dtype, pool->io_dtype);
  if (a->norm_gate) return fail(NSSM_ERR_INVALID, "the fused norm is a nssm_tiered_step option");
  if (tok) {
    if (tok->ntok < 1) return fail(NSSM_ERR_INVALID, "ntok %d < 1", tok->ntok);
    if (tok->ntok > pool->chunk)
      return fail(NSSM_ERR_INVALID, "ntok %d > chunk %d: a window cannot cross a chunk boundary", tok->ntok, pool->chunk);
    q.ntok = tok->ntok;
    q.x_st = tok->x_stride_t; q.dt_st = tok->dt_stride_t; q.B_st = tok->B_stride_t;
    q.C_st = tok->C_stride_t; q.out_st = tok->out_stride_t;
  }
  fill_pool(pool, sp);
  fill_inputs(a, sp);
  return NSSM_OK;
}

// R rotation of the ntok tokens' B and C (token-contiguous rows) into the workspace.
int spec_rotate(const nssm_step_args* a, int ntok, int G, int N, nssm::StepParams& sp, nssm::SpecParams& q,
                cudaStream_t st) {
  sp.B = a->B; sp.B_sb = a->B_stride_b;
  sp.C = a->C; sp.C_sb = a->C_stride_b;
  if (!a->R) return NSSM_OK;
  if (N != 128) return fail(NSSM_ERR_UNSUPPORTED, "rotation compiled for dstate 128 only");
  if (reinterpret_cast<uintptr_t>(a->R) % 16) return fail(NSSM_ERR_INVALID, "R must be 16-byte aligned");
  if (ntok > 1 && (a->B_stride_b != ntok * q.B_st || a->C_stride_b != ntok * q.C_st))
    return fail(NSSM_ERR_INVALID, "with R, B and C rows must be token-contiguous (stride_b == ntok * stride_t)");
  const int rows = a->batch * ntok;
  const size_t half = nssm_step_workspace_bytes(rows, G, N, a->io_dtype, 1) / 2;
  nssm::RotParams rp{};
  rp.x0 = a->B; rp.xs0 = ntok > 1 ? q.B_st : a->B_stride_b;
  rp.x1 = a->C; rp.xs1 = ntok > 1 ? q.C_st : a->C_stride_b;
  rp.o0 = a->workspace; rp.os0 = (int64_t)G * N;
  rp.o1 = static_cast<char*>(a->workspace) + half; rp.os1 = (int64_t)G * N;
  rp.R = a->R; rp.T = rows; rp.G = G; rp.dtype = a->io_dtype;
  int rc = launch_rot(rp, 2 * rows, G, st);
  if (rc) return rc;
  sp.B = rp.o0; sp.B_sb = (int64_t)ntok * G * N; q.B_st = (int64_t)G * N;
  sp.C = rp.o1; sp.C_sb = (int64_t)ntok * G * N; q.C_st = (int64_t)G * N;
  return NSSM_OK;
}

}  // namespace

extern "C" {

size_t nssm_spec_workspace_bytes(int32_t batch, int32_t ntok, int32_t ngroups, int32_t dstate, int32_t io_dtype,
                                 int32_t has_rotation) {
  if (batch <= 0 || ntok <= 0) return 0;
  const size_t rot = nssm_step_workspace_bytes(batch * ntok, ngroups, dstate, io_dtype, has_rotation);
  return rot + ((size_t)batch * 4 + 255) / 256 * 256;
}

int nssm_draft_step(const nssm_pool* pool, float* draft, int32_t from_pool, const nssm_step_args* args,
                    void* stream) {
  nssm::StepParams sp{};
  nssm::SpecParams q{};
  int rc = spec_prepare(pool, args, nullptr, sp, q);
  if (rc) return rc;
  if (!draft || !aligned16(draft)) return fail(NSSM_ERR_INVALID, "draft must be a 16-byte aligned device pointer");
  if (args->batch == 0) return NSSM_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (args->R) {
    const size_t need = nssm_step_workspace_bytes(args->batch, pool->ngroups, pool->dstate, args->io_dtype, 1);
    if (!args->workspace || args->workspace_bytes < need)
      return fail(NSSM_ERR_INVALID, "workspace of %zu bytes needed for the rotation (got %zu)", need,
                  args->workspace_bytes);
  }
  rc = spec_rotate(args, 1, pool->ngroups, pool->dstate, sp, q, st);
  if (rc) return rc;
  q.sp = sp;
  q.ntok = 1;
  q.draft = draft;
  q.from_pool = from_pool ? 1 : 0;
  return dispatch(OP_DRAFT, pool->dstate, pool->hot_dim, pool->cold_dtype, &q, args->batch, st);
}

int nssm_verify_step(const nssm_pool* pool, const nssm_step_args* args, const nssm_token_args* tok, void* stream) {
  if (!tok) return fail(NSSM_ERR_INVALID, "tok is NULL");
  nssm::StepParams sp{};
  nssm::SpecParams q{};
  int rc = spec_prepare(pool, args, tok, sp, q);
  if (rc) return rc;
  if (args->mode == NSSM_MODE_CORR) return fail(NSSM_ERR_UNSUPPORTED, "verify reads modes STALE and COLDOFF");
  if (args->batch == 0) return NSSM_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (args->R) {
    const size_t need = nssm_spec_workspace_bytes(args->batch, tok->ntok, pool->ngroups, pool->dstate, args->io_dtype, 1);
    if (!args->workspace || args->workspace_bytes < need)
      return fail(NSSM_ERR_INVALID, "workspace of %zu bytes needed (got %zu)", need, args->workspace_bytes);
  }
  rc = spec_rotate(args, tok->ntok, pool->ngroups, pool->dstate, sp, q, st);
  if (rc) return rc;
  q.sp = sp;
  return dispatch(OP_VERIFY, pool->dstate, pool->hot_dim, pool->cold_dtype, &q, args->batch, st);
}

int nssm_commit_step(const nssm_pool* pool, const nssm_step_args* args, const nssm_token_args* tok, void* stream) {
  if (!tok) return fail(NSSM_ERR_INVALID, "tok is NULL");
  if (!tok->accept) return fail(NSSM_ERR_INVALID, "tok->accept is NULL");
  nssm::StepParams sp{};
  nssm::SpecParams q{};
  int rc = spec_prepare(pool, args, tok, sp, q);
  if (rc) return rc;
  if (args->batch == 0) return NSSM_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t need = nssm_spec_workspace_bytes(args->batch, tok->ntok, pool->ngroups, pool->dstate, args->io_dtype,
                                                args->R ? 1 : 0);
  if (!args->workspace || args->workspace_bytes < need || !aligned16(args->workspace))
    return fail(NSSM_ERR_INVALID, "a 16-byte aligned workspace of %zu bytes is needed (got %zu)", need,
                args->workspace_bytes);
  rc = spec_rotate(args, tok->ntok, pool->ngroups, pool->dstate, sp, q, st);
  if (rc) return rc;
  q.sp = sp;
  q.accept = tok->accept;
  q.flush_idx = reinterpret_cast<int32_t*>(
      static_cast<char*>(args->workspace) +
      nssm_step_workspace_bytes(args->batch * tok->ntok, pool->ngroups, pool->dstate, args->io_dtype, args->R ? 1 : 0));
  return dispatch(OP_COMMIT, pool->dstate, pool->hot_dim, pool->cold_dtype, &q, args->batch, st);
}

size_t nssm_step_workspace_bytes(int32_t batch, int32_t ngroups, int32_t dstate, int32_t io_dtype,
                                 int32_t has_rotation) {
  if (!has_rotation || batch <= 0) return 0;
  size_t half = (size_t)batch * ngroups * dstate * io_bytes(io_dtype);
  half = (half + 255) / 256 * 256;
  return 2 * half;
}

int nssm_tiered_step(const nssm_pool* pool, const nssm_step_args* args, void* stream) {
  int rc = check_pool(pool);
  if (rc) return rc;
  rc = check_args(args, pool->nheads);
  if (rc) return rc;
  if (args->io_dtype != pool->io_dtype)
    return fail(NSSM_ERR_INVALID, "args io_dtype %d differs from the pool's ring dtype %d", args->io_dtype, pool->io_dtype);
  if (args->batch == 0) return NSSM_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  nssm::StepParams sp{};
  sp.hot = pool->hot; sp.cold = pool->cold; sp.scale = pool->cold_scale;
  sp.glog = pool->glog; sp.t = pool->t;
  sp.ring_x = pool->ring_x; sp.ring_dt = pool->ring_dt; sp.ring_b = pool->ring_b;
  sp.S = pool->num_slots; sp.H = pool->nheads; sp.P = pool->headdim; sp.G = pool->ngroups; sp.c = pool->chunk;
  fill_inputs(args, sp);
  rc = check_norm(args, pool->nheads, pool->headdim, pool->ngroups);
  if (rc) return rc;
  if (args->norm_gate && norm_fusable(args)) {
    sp.ngate = args->norm_gate; sp.ngate_sb = args->norm_gate_stride_b;
    sp.nweight = args->norm_weight; sp.nweight_dtype = args->norm_weight_dtype; sp.neps = args->norm_eps;
  }
  rc = maybe_rotate(args, pool->ngroups, pool->dstate, sp, st);
  if (rc) return rc;
  g_norm_fused = false;
  rc = dispatch(OP_STEP, pool->dstate, pool->hot_dim, pool->cold_dtype, &sp, args->batch, st);
  if (rc || !args->norm_gate || g_norm_fused) return rc;
  return run_norm_after_step(args, pool->nheads, pool->headdim, st);
}

int nssm_fresh_step(float* state, int32_t num_slots, int32_t nheads, int32_t headdim, int32_t dstate,
                    int32_t ngroups, const nssm_step_args* args, void* stream) {
  if (!state) return fail(NSSM_ERR_INVALID, "state is NULL");
  if (!aligned16(state)) return fail(NSSM_ERR_INVALID, "state must be 16-byte aligned");
  if (num_slots <= 0 || nheads <= 0 || headdim <= 0 || ngroups <= 0 || nheads % ngroups)
    return fail(NSSM_ERR_INVALID, "bad dims (S=%d H=%d P=%d G=%d)", num_slots, nheads, headdim, ngroups);
  if (dstate != 128) return fail(NSSM_ERR_UNSUPPORTED, "fresh step compiled for dstate 128 only");
  if (headdim > 128) return fail(NSSM_ERR_UNSUPPORTED, "headdim %d > 128", headdim);
  int rc = check_args(args, nheads);
  if (rc) return rc;
  if (args->norm_gate) return fail(NSSM_ERR_INVALID, "the fused norm is a tiered-step option (nssm_fresh_step has none)");
  if (args->batch == 0) return NSSM_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  nssm::StepParams sp{};
  sp.hot = state;
  sp.S = num_slots; sp.H = nheads; sp.P = headdim; sp.G = ngroups; sp.c = 1;
  fill_inputs(args, sp);
  sp.mode = NSSM_MODE_STALE;
  rc = maybe_rotate(args, ngroups, dstate, sp, st);
  if (rc) return rc;
  dim3 grid(nheads, args->batch);
  const int threads = round_up(headdim * kTPRFresh, 32);
  nssm::tiered_step_kernel<128, 0, COLD_NONE, kTPRFresh><<<grid, threads, step_smem_bytes<128, 0, COLD_NONE>(headdim, 1), st>>>(sp);
  return cuda_check("fresh step launch");
}

int nssm_prefill_split(const nssm_pool* pool, const float* state, int64_t state_stride_b, const int32_t* slots,
                       int32_t batch, int32_t pad_slot_id, void* stream) {
  int rc = check_pool(pool);
  if (rc) return rc;
  if (batch < 0 || batch > 65535) return fail(NSSM_ERR_INVALID, "batch %d outside [0, 65535]", batch);
  if (batch == 0) return NSSM_OK;
  if (!state) return fail(NSSM_ERR_INVALID, "state is NULL");
  if (!aligned16(state) || (state_stride_b % 4)) return fail(NSSM_ERR_INVALID, "state rows must be 16-byte aligned");
  nssm::SplitParams sp{};
  sp.hot = pool->hot; sp.cold = pool->cold; sp.scale = pool->cold_scale; sp.glog = pool->glog; sp.t = pool->t;
  sp.S = pool->num_slots; sp.H = pool->nheads; sp.P = pool->headdim;
  sp.src = state; sp.src_sb = state_stride_b; sp.idx = slots; sp.pad = pad_slot_id; sp.status = nullptr;
  return dispatch(OP_SPLIT, pool->dstate, pool->hot_dim, pool->cold_dtype, &sp, batch, static_cast<cudaStream_t>(stream));
}

int nssm_materialize(const nssm_pool* pool, const float* A, const int32_t* slots, int32_t batch,
                     int32_t pad_slot_id, float* out, int64_t out_stride_b, void* stream) {
  int rc = check_pool(pool);
  if (rc) return rc;
  if (batch < 0 || batch > 65535) return fail(NSSM_ERR_INVALID, "batch %d outside [0, 65535]", batch);
  if (batch == 0) return NSSM_OK;
  if (!A || !out) return fail(NSSM_ERR_INVALID, "A / out is NULL");
  if (!aligned16(out) || (out_stride_b % 4)) return fail(NSSM_ERR_INVALID, "out rows must be 16-byte aligned");
  nssm::MatParams mp{};
  mp.hot = pool->hot; mp.cold = pool->cold; mp.scale = pool->cold_scale; mp.t = pool->t;
  mp.ring_x = pool->ring_x; mp.ring_dt = pool->ring_dt; mp.ring_b = pool->ring_b;
  mp.S = pool->num_slots; mp.H = pool->nheads; mp.P = pool->headdim; mp.G = pool->ngroups; mp.c = pool->chunk;
  mp.io_dtype = pool->io_dtype; mp.A = A; mp.idx = slots; mp.pad = pad_slot_id; mp.out = out; mp.out_sb = out_stride_b;
  mp.status = nullptr;
  return dispatch(OP_MAT, pool->dstate, pool->hot_dim, pool->cold_dtype, &mp, batch, static_cast<cudaStream_t>(stream));
}

int nssm_rot_flat(const void* x, int64_t x_stride, int32_t dtype, const float* R, int32_t T, int32_t ngroups,
                  int32_t dstate, void* out, int64_t out_stride, void* stream) {
  if (T < 0 || T > (1 << 24)) return fail(NSSM_ERR_INVALID, "T %d out of range", T);
  if (T == 0) return NSSM_OK;
  if (!x || !R || !out) return fail(NSSM_ERR_INVALID, "x / R / out is NULL");
  if (dtype != NSSM_F32 && dtype != NSSM_BF16) return fail(NSSM_ERR_INVALID, "dtype must be F32 or BF16");
  if (dstate != 128) return fail(NSSM_ERR_UNSUPPORTED, "rotation compiled for dstate 128 only");
  if (ngroups <= 0 || ngroups > 65535) return fail(NSSM_ERR_INVALID, "ngroups %d", ngroups);
  if (reinterpret_cast<uintptr_t>(R) % 16) return fail(NSSM_ERR_INVALID, "R must be 16-byte aligned");
  nssm::RotParams rp{};
  rp.x0 = rp.x1 = x; rp.xs0 = rp.xs1 = x_stride;
  rp.o0 = rp.o1 = out; rp.os0 = rp.os1 = out_stride;
  rp.R = R; rp.T = T; rp.G = ngroups; rp.dtype = dtype;
  return launch_rot(rp, T, ngroups, static_cast<cudaStream_t>(stream));
}

int nssm_conv_step(const nssm_conv_args* a, void* stream) {
  if (!a) return fail(NSSM_ERR_INVALID, "args is NULL");
  if (a->batch < 0 || a->batch > 65535) return fail(NSSM_ERR_INVALID, "batch %d outside [0, 65535]", a->batch);
  if (a->batch == 0) return NSSM_OK;
  if (a->nheads <= 0 || a->headdim <= 0 || a->ngroups <= 0 || a->ngroups > 65535 || a->num_slots <= 0)
    return fail(NSSM_ERR_INVALID, "bad dims (H=%d P=%d G=%d S=%d)", a->nheads, a->headdim, a->ngroups, a->num_slots);
  if (a->dstate != 128) return fail(NSSM_ERR_UNSUPPORTED, "conv step compiled for dstate 128 only");
  if (a->width < 1 || a->width > nssm::kConvMaxK || a->state_len < a->width - 1 || a->state_len > nssm::kConvMaxL ||
      a->state_len < 1)
    return fail(NSSM_ERR_INVALID, "width %d / state_len %d unsupported (1 <= K <= 8, K-1 <= L <= 8, L >= 1)",
                a->width, a->state_len);
  if (a->io_dtype != NSSM_F32 && a->io_dtype != NSSM_BF16) return fail(NSSM_ERR_INVALID, "io_dtype must be F32 or BF16");
  if (a->weight_dtype != NSSM_F32 && a->weight_dtype != NSSM_BF16)
    return fail(NSSM_ERR_INVALID, "weight_dtype must be F32 or BF16");
  if (a->activation != 0 && a->activation != 1) return fail(NSSM_ERR_INVALID, "activation %d unknown", a->activation);
  if (!a->xbc || !a->conv_state || !a->weight || !a->x_out || !a->B_out || !a->C_out)
    return fail(NSSM_ERR_INVALID, "a required pointer is NULL");
  if (a->R && (reinterpret_cast<uintptr_t>(a->R) % 16)) return fail(NSSM_ERR_INVALID, "R must be 16-byte aligned");
  nssm::ConvParams cp{};
  cp.xbc = a->xbc; cp.xbc_sb = a->xbc_stride_b;
  cp.state = a->conv_state; cp.state_ss = a->state_stride_s; cp.L = a->state_len; cp.K = a->width;
  cp.state_sd = a->state_stride_d; cp.state_sl = a->state_stride_l;
  cp.weight = a->weight; cp.w_dtype = a->weight_dtype; cp.bias = a->bias; cp.act = a->activation;
  cp.R = a->R; cp.idx = a->state_batch_indices; cp.pad = a->pad_slot_id; cp.S = a->num_slots;
  cp.T = a->batch; cp.I = a->nheads * a->headdim; cp.G = a->ngroups; cp.dtype = a->io_dtype;
  cp.x_out = a->x_out; cp.x_sb = a->x_out_stride_b;
  cp.b_out = a->B_out; cp.c_out = a->C_out; cp.bc_sb = a->bc_out_stride_b;
  cp.status = a->status;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // vector paths for width 4 with state length 3 or 4 when every access is aligned; the
  // state either [slot][d][l] (DL) or channels-last [slot][l][d] (LD)
  const bool dl = a->state_stride_l == 1 && a->state_stride_d == a->state_len;
  const bool ld = a->state_stride_d == 1 && a->state_stride_l % 4 == 0 && a->state_stride_l >= cp.I + 2 * a->ngroups * 128;
  const bool vec = a->width == 4 && (a->state_len == 3 || a->state_len == 4) && cp.I % 4 == 0 && (dl || ld) &&
                   aligned16(a->xbc) && aligned16(a->conv_state) && aligned16(a->x_out) && aligned16(a->weight) &&
                   (!a->bias || aligned16(a->bias)) && a->xbc_stride_b % 4 == 0 && a->x_out_stride_b % 4 == 0 &&
                   a->state_stride_s % 4 == 0;
  const bool iobf = a->io_dtype == NSSM_BF16, wbf = a->weight_dtype == NSSM_BF16;
  const int B = a->batch, G = a->ngroups;
  if (!vec) return launch_conv<0, 0, false, false, false>(cp, B, G, st);
  if (ld) {
    if (a->state_len == 3) {
      if (iobf) return wbf ? launch_conv<4, 3, true, true, true>(cp, B, G, st) : launch_conv<4, 3, true, false, true>(cp, B, G, st);
      return wbf ? launch_conv<4, 3, false, true, true>(cp, B, G, st) : launch_conv<4, 3, false, false, true>(cp, B, G, st);
    }
    if (iobf) return wbf ? launch_conv<4, 4, true, true, true>(cp, B, G, st) : launch_conv<4, 4, true, false, true>(cp, B, G, st);
    return wbf ? launch_conv<4, 4, false, true, true>(cp, B, G, st) : launch_conv<4, 4, false, false, true>(cp, B, G, st);
  }
  if (a->state_len == 3) {
    if (iobf) return wbf ? launch_conv<4, 3, true, true, false>(cp, B, G, st) : launch_conv<4, 3, true, false, false>(cp, B, G, st);
    return wbf ? launch_conv<4, 3, false, true, false>(cp, B, G, st) : launch_conv<4, 3, false, false, false>(cp, B, G, st);
  }
  if (iobf) return wbf ? launch_conv<4, 4, true, true, false>(cp, B, G, st) : launch_conv<4, 4, true, false, false>(cp, B, G, st);
  return wbf ? launch_conv<4, 4, false, true, false>(cp, B, G, st) : launch_conv<4, 4, false, false, false>(cp, B, G, st);
}

int nssm_gated_rmsnorm(const void* y, int64_t y_stride, const void* gate, int64_t gate_stride, const void* weight,
                       int32_t weight_dtype, float eps, int32_t batch, int32_t dim, int32_t group_size,
                       int32_t io_dtype, void* out, int64_t out_stride, void* stream) {
  if (batch < 0 || batch > 65535) return fail(NSSM_ERR_INVALID, "batch %d outside [0, 65535]", batch);
  if (batch == 0) return NSSM_OK;
  if (!y || !gate || !weight || !out) return fail(NSSM_ERR_INVALID, "y / gate / weight / out is NULL");
  if (dim <= 0 || group_size <= 0 || dim % group_size || group_size > nssm::kNormThreads * nssm::kNormMaxPer)
    return fail(NSSM_ERR_INVALID, "dim %d / group_size %d unsupported (group_size divides dim, <= %d)", dim,
                group_size, nssm::kNormThreads * nssm::kNormMaxPer);
  if (dim / group_size > 65535) return fail(NSSM_ERR_INVALID, "too many groups");
  if ((io_dtype != NSSM_F32 && io_dtype != NSSM_BF16) || (weight_dtype != NSSM_F32 && weight_dtype != NSSM_BF16))
    return fail(NSSM_ERR_INVALID, "dtypes must be F32 or BF16");
  nssm::NormParams np{};
  np.y = y; np.y_sb = y_stride; np.gate = gate; np.g_sb = gate_stride; np.weight = weight; np.w_dtype = weight_dtype;
  np.eps = eps; np.dim = dim; np.gs = group_size; np.dtype = io_dtype; np.out = out; np.o_sb = out_stride;
  dim3 grid((unsigned)(dim / group_size), (unsigned)batch);
  nssm::gated_rmsnorm_kernel<<<grid, nssm::kNormThreads, 0, static_cast<cudaStream_t>(stream)>>>(np);
  return cuda_check("gated_rmsnorm_kernel launch");
}

size_t nssm_sizeof_conv_args(void) { return sizeof(nssm_conv_args); }

int32_t nssm_supported_hot_dims(int32_t dstate, int32_t* widths, int32_t cap) {
  static const int32_t k128[] = {16, 32, 64};
  if (dstate != 128) return 0;
  int32_t n = 0;
  for (int32_t w : k128) {
    if (widths && n < cap) widths[n] = w;
    ++n;
  }
  return n;
}

uint32_t nssm_set_wait_polls(uint32_t polls) {
  return g_wait_polls.exchange(polls ? polls : nssm::kSpinLimit, std::memory_order_relaxed);
}

int32_t nssm_test_inject_stuck_copy(int32_t enable) {
  return g_inject_stuck.exchange(enable ? 1 : 0, std::memory_order_relaxed);
}

size_t nssm_sizeof_pool(void) { return sizeof(nssm_pool); }
size_t nssm_sizeof_step_args(void) { return sizeof(nssm_step_args); }
size_t nssm_sizeof_token_args(void) { return sizeof(nssm_token_args); }
int32_t nssm_abi_version(void) { return NSSM_ABI_VERSION; }
const char* nssm_last_error(void) { return g_last_error.c_str(); }

}  // extern "C"
