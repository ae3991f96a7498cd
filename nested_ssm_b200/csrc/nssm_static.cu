// nssm_tiered_step_static: the tiered step for callers that cannot give the
// library any device memory.
//
// nssm_tiered_step needs a caller-owned workspace when it rotates B and C (the
// rotated copies live there between the rotation kernel and the state kernel).
// Some hosts have no way to hand one over: an inference server whose memory
// planner owns every device allocation and forbids extension code from calling
// cudaMalloc or a framework allocator, or a thin FFI binding (cgo, JNI) that
// passes only the model's own tensors.  This entry point takes the scratch from
// a fixed array in the library's static device memory instead, so a call makes
// no allocation of any kind.  It then runs exactly the nssm_tiered_step path.
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>

#include "nested_ssm.h"

namespace nssm_host {
int fail(int code, const char* fmt, ...);
}

namespace {

// One copy per device (static __device__ memory is instantiated in every
// context that loads the library).  Every byte the state kernel reads from it
// is written by the same call's rotation kernel first, so nothing here has to
// start at zero.
__device__ __align__(256) unsigned char g_step_scratch[NSSM_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::atomic<void*> g_scratch_ptr[kMaxDevices];
std::mutex g_setup_mu;

// Device address of g_step_scratch on the current device; looked up once per
// device (the first call), then read from the cache.  The cache lives as long as the
// process: a cudaDeviceReset unloads the array on that device and leaves the cached
// address stale, so callers do not use this entry point on a device after resetting it.
int scratch_on_current_device(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return nssm_host::fail(NSSM_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  }
  if (dev < 0 || dev >= kMaxDevices)
    return nssm_host::fail(NSSM_ERR_UNSUPPORTED, "device ordinal %d beyond the %d this entry point tracks", dev,
                           kMaxDevices);
  void* p = g_scratch_ptr[dev].load(std::memory_order_acquire);
  if (!p) {
    std::lock_guard<std::mutex> lk(g_setup_mu);
    p = g_scratch_ptr[dev].load(std::memory_order_relaxed);
    if (!p) {
      e = cudaGetSymbolAddress(&p, g_step_scratch);
      if (e != cudaSuccess || !p) {
        cudaGetLastError();
        return nssm_host::fail(NSSM_ERR_CUDA, "cudaGetSymbolAddress(static step scratch) on device %d: %s", dev,
                               cudaGetErrorString(e));
      }
      g_scratch_ptr[dev].store(p, std::memory_order_release);
    }
  }
  *out = p;
  return NSSM_OK;
}

}  // namespace

extern "C" {

int nssm_tiered_step_static(const nssm_pool* pool, const nssm_step_args* args, void* stream) {
  if (!pool || !args) return nssm_host::fail(NSSM_ERR_INVALID, "pool / args is NULL");
  nssm_step_args a = *args;
  a.workspace = nullptr;
  a.workspace_bytes = 0;
  if (a.R != nullptr && a.batch > 0) {
    const size_t need = nssm_step_workspace_bytes(a.batch, pool->ngroups, pool->dstate, a.io_dtype, 1);
    if (need > (size_t)NSSM_STATIC_SCRATCH_BYTES)
      return nssm_host::fail(NSSM_ERR_INVALID,
                             "batch %d needs %zu bytes of rotation scratch; the static scratch holds %zu "
                             "(use nssm_tiered_step with a workspace, or split the batch)",
                             a.batch, need, (size_t)NSSM_STATIC_SCRATCH_BYTES);
    void* p = nullptr;
    const int rc = scratch_on_current_device(&p);
    if (rc) return rc;
    a.workspace = p;
    a.workspace_bytes = NSSM_STATIC_SCRATCH_BYTES;
  }
  return nssm_tiered_step(pool, &a, stream);
}

}  // extern "C"
