// Tiered-step / prefill-split / materialise instances for hot width 16.
#include "nssm_host.cuh"

namespace nssm_host {

int dispatch_pb16(Op op, int cold, const void* params, int batch, cudaStream_t st) {
  return run_cold<16>(op, cold, params, batch, st);
}

}  // namespace nssm_host
