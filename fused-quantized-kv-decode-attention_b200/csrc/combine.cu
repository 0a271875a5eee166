// Split-K combine: log-sum-exp merge of per-split (m, l, o) partials.
//
// Replaces gqa_sk_combine_par (kernels/decode_attn_gqa_sk_fast.cu:57-94).  Same
// algebra -- an empty split (m = -inf) gets weight 0 -- with m in log2 units
// (the partial kernels work in the log2 domain).  Launched with programmatic
// dependent launch: the CTAs are scheduled while the partial grid is still
// streaming and block in griddepcontrol.wait until it has completed, which
// hides the second launch's latency (the reference pays two full launches).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>

#include "device_common.cuh"
#include "kernels.h"

namespace fqkv {
namespace {

constexpr int kCombineThreads = 512;

// One CTA per row.  The split range is divided among kCombineThreads / D
// thread groups (thread = one dim of one group); every group merges its
// splits online -- (M, L, O) rescaled when M grows, branch-free, so the loads
// of consecutive splits are independent and in flight together -- and the
// groups' results are merged once through shared memory.
__global__ void __launch_bounds__(kCombineThreads) combine_kernel(const float* __restrict__ pm,
                                                                  const float* __restrict__ pl,
                                                                  const float* __restrict__ po,
                                                                  void* __restrict__ out, bool out_bf16, int D, int S,
                                                                  int S_eff, const TpOut tp) {
  pdl_launch_dependents();  // the next decode kernel may be scheduled now; it waits for this grid
  pdl_wait_primary();
  __shared__ float sm_o[kCombineThreads];
  __shared__ float sm_m[kCombineThreads / 64];
  __shared__ float sm_l[kCombineThreads / 64];
  const size_t row = blockIdx.x;
  const int tid = threadIdx.x;
  const float* m = pm + row * S;
  const float* l = pl + row * S;

  const int groups = kCombineThreads / D;
  const int gi = tid / D, d = tid - gi * D;
  float M = -INFINITY, L = 0.f, O = 0.f;
#pragma unroll 8
  for (int s = gi; s < S_eff; s += groups) {
    const float ms = m[s];
    const float ls = l[s];
    const float os = po[(row * S + s) * D + d];
    const float Mn = fmaxf(M, ms);
    const float a = (Mn == -INFINITY) ? 1.f : ex2(M - Mn);   // M = -inf: ex2 gives 0
    const float b = (ms == -INFINITY) ? 0.f : ex2(ms - Mn);  // an empty split weighs 0
    L = fmaf(L, a, b * ls);
    O = fmaf(O, a, b * os);
    M = Mn;
  }
  sm_o[tid] = O;
  if (d == 0) {
    sm_m[gi] = M;
    sm_l[gi] = L;
  }
  __syncthreads();
  if (gi == 0) {
    float Mt = -INFINITY;
    for (int g = 0; g < groups; ++g) Mt = fmaxf(Mt, sm_m[g]);
    float Ls = 0.f, Os = 0.f;
    for (int g = 0; g < groups; ++g) {
      const float w = (sm_m[g] == -INFINITY) ? 0.f : ex2(sm_m[g] - Mt);
      Ls = fmaf(w, sm_l[g], Ls);
      Os = fmaf(w, sm_o[g * D + d], Os);
    }
    const __half_raw h = __half_raw(__float2half_rn(Os / Ls));
    if (out_bf16) {
      static_cast<__nv_bfloat16*>(out)[row * D + d] = __float2bfloat16_rn(Os / Ls);
    } else if (tp.world == 0) {
      static_cast<__half_raw*>(out)[row * D + d] = h;
    } else {
      for (int p = 0; p < tp.world; ++p) tp.dst[p][tp.dst_off + row * D + d] = h;
    }
  }
  if (tp.world != 0) {  // tensor-parallel output: one arrival per row on every rank
    __threadfence_system();
    __syncthreads();
    if (tid == 0)
      for (int p = 0; p < tp.world; ++p) atomicAdd_system(tp.cnt[p] + tp.rank, 1ull);
  }
}

}  // namespace

cudaError_t launch_combine(const DecodeLaunch& a, cudaStream_t stream) {
  const int rows = a.B * a.Hq;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(rows);
  cfg.blockDim = dim3(kCombineThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, combine_kernel, static_cast<const float*>(a.part_m),
                            static_cast<const float*>(a.part_l), static_cast<const float*>(a.part_o),
                            a.out, a.out_bf16, a.D, a.S, a.S_eff, a.tp);
}

}  // namespace fqkv
