// Gated RMS norm of the mixer output (the step after the state op):
//   h = y * silu(gate)  (fp32),   per group of `gs` channels: h *= 1 / sqrt(mean(h^2) + eps),
//   out = weight * round_io(h)
// as transformers' Zamba2RMSNormGated (gate before the norm) that NemotronH uses, and the
// reference's restatement rmsnorm_fn(norm_before_gate=False) (scale/nemotron_retrofit.py:146-161).
#pragma once

#include "nssm_device.cuh"

namespace nssm {

struct NormParams {
  const void* y;
  int64_t y_sb;
  const void* gate;
  int64_t g_sb;
  const void* weight;
  int w_dtype;
  float eps;
  int dim, gs, dtype;
  void* out;
  int64_t o_sb;
};

constexpr int kNormThreads = 256;
constexpr int kNormMaxPer = 8;   // group_size <= kNormThreads * kNormMaxPer

// one CTA per (row, group)
__global__ void __launch_bounds__(kNormThreads) gated_rmsnorm_kernel(const NormParams p) {
  __shared__ float red[kNormThreads / 32];
  const int b = blockIdx.y, g = blockIdx.x;
  const int tid = threadIdx.x;
  const int64_t c0 = (int64_t)g * p.gs;
  float h[kNormMaxPer];
  float ss = 0.0f;
#pragma unroll
  for (int u = 0; u < kNormMaxPer; ++u) {
    const int i = tid + u * kNormThreads;
    h[u] = 0.0f;
    if (i < p.gs) {
      const float y = ld_io(p.y, (int64_t)b * p.y_sb + c0 + i, p.dtype);
      const float z = ld_io(p.gate, (int64_t)b * p.g_sb + c0 + i, p.dtype);
      h[u] = y * (z / (1.0f + expf(-z)));
      ss = fmaf(h[u], h[u], ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) tot += red[w];
  const float r = 1.0f / sqrtf(tot / (float)p.gs + p.eps);
#pragma unroll
  for (int u = 0; u < kNormMaxPer; ++u) {
    const int i = tid + u * kNormThreads;
    if (i < p.gs) {
      const float hn = (p.dtype == NSSM_BF16) ? __bfloat162float(__float2bfloat16_rn(h[u] * r)) : h[u] * r;
      st_io(p.out, (int64_t)b * p.o_sb + c0 + i, p.dtype, ld_io(p.weight, c0 + i, p.w_dtype) * hn);
    }
  }
}

}  // namespace nssm
