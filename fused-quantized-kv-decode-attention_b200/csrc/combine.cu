// Split-K combine: log-sum-exp merge of per-split (m, l, o) partials.
//
// Replaces gqa_sk_combine_par (kernels/decode_attn_gqa_sk_fast.cu:57-94).  Same
// algebra -- an empty split (m = -inf) gets weight 0 -- with m in log2 units
// (the partial kernels work in the log2 domain).  Launched with programmatic
// dependent launch: the CTAs are scheduled while the partial grid is still
// streaming and block in griddepcontrol.wait until it has completed, which
// hides the second launch's latency (the reference pays two full launches).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>

#include "device_common.cuh"
#include "kernels.h"

namespace fqkv {
namespace {

__global__ void __launch_bounds__(128) combine_kernel(const float* __restrict__ pm, const float* __restrict__ pl,
                                                      const float* __restrict__ po, __half* __restrict__ out,
                                                      int rows, int D, int S, int S_eff) {
  pdl_wait_primary();
  // one warp per row, each lane covers D/32 dims
  const int warps = blockDim.x >> 5;
  const int row = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* m = pm + size_t(row) * S;
  const float* l = pl + size_t(row) * S;
  float M = -INFINITY;
  for (int s = lane; s < S_eff; s += 32) M = fmaxf(M, m[s]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  float L = 0.f;
  float O[4] = {0.f, 0.f, 0.f, 0.f};
  const int per = D / 32;
  for (int s = 0; s < S_eff; ++s) {
    const float ms = m[s];
    const float w = (ms == -INFINITY) ? 0.f : ex2(ms - M);
    L += w * l[s];
    const float* os = po + (size_t(row) * S + s) * D;
    for (int e = 0; e < per; ++e) O[e] += w * os[lane + 32 * e];
  }
  for (int e = 0; e < per; ++e) out[size_t(row) * D + lane + 32 * e] = __float2half_rn(O[e] / L);
}

}  // namespace

cudaError_t launch_combine(const DecodeLaunch& a, cudaStream_t stream) {
  const int rows = a.B * a.Hq;
  const int warps = 4;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((rows + warps - 1) / warps);
  cfg.blockDim = dim3(32 * warps);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, combine_kernel, static_cast<const float*>(a.part_m),
                            static_cast<const float*>(a.part_l), static_cast<const float*>(a.part_o),
                            static_cast<__half*>(a.out), rows, a.D, a.S, a.S_eff);
}

}  // namespace fqkv
