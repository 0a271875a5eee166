// Per-token symmetric KV quantizers, bit-exact with the reference's torch code.
//
// int8: qpt (notebooks/integration_and_benchmarks.ipynb lines 236-238,
//        tests/test_kernels.py:32-34)
// int4: quant_int4_per_token (notebook lines 292-299), element 2t in the low
//        nibble of byte t.
//
// The reference evaluates  s = (amax / Q).clamp(min=1e-8);  round(X / s)  on
// fp16 tensors, i.e. every operation is done in fp32 and rounded to fp16.  The
// kernel reproduces that sequence exactly:
//   s    = fp16( fp32(amax) / Q )            (IEEE division, round to nearest)
//   r    = fp16( fp32(x) / fp32(s) )         (second rounding to fp16)
//   code = rint(r) clamped to [-Q, Q];  NaN -> 0
// clamp(min=1e-8) never changes an fp16 value (1e-8 rounds to fp16 zero), and
// amax propagates NaN like torch.amax.  Divisions use __fdiv_rn so the result
// does not depend on fast-math flags.
//
// HBM-bound: one 16-byte load per lane (8 elements), D/8 lanes per token.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "kernels.h"

namespace fqkv {
namespace {

template <int Q>
__device__ __forceinline__ int quant_code(float x, float s) {
  const float r = __half2float(__float2half_rn(__fdiv_rn(x, s)));
  const float rr = rintf(r);
  if (isnan(rr)) return 0;
  return static_cast<int>(fminf(fmaxf(rr, -float(Q)), float(Q)));
}

template <int Q>
__device__ __forceinline__ __half quant_scale(float amax, bool any_nan) {
  const float a = any_nan ? __int_as_float(0x7fc00000) : amax;
  return __float2half_rn(__fdiv_rn(a, float(Q)));
}

// Vectorised path: D in {64, 128, 256}; LPR = D/8 lanes per token.
// Output placement: token `row` of the input (rows = groups x T tokens) goes
// to output row (row / T) * cap + pos + row % T, where pos is *pos_dev when
// given (a growing KV cache) else pos_host; tokens landing at or past `cap`
// are not written.  The plain quantizer uses T = cap = rows, pos = 0.
struct QuantPlace {
  int64_t T, cap, pos_host;
  const int* pos_dev;
};

template <bool kInt4, int D>
__global__ void __launch_bounds__(256) quantize_vec_kernel(const __half* __restrict__ X, void* __restrict__ codes,
                                                           __half* __restrict__ scales, int64_t rows,
                                                           QuantPlace pl) {
  constexpr int LPR = D / 8;
  constexpr int RPW = 32 / LPR;
  constexpr int Q = kInt4 ? 7 : 127;
  const int lane = threadIdx.x & 31;
  const int64_t warp_global = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t row = warp_global * RPW + lane / LPR;
  const int c = lane % LPR;
  const bool active = row < rows;
  uint4 raw = make_uint4(0, 0, 0, 0);
  if (active) raw = *reinterpret_cast<const uint4*>(X + row * D + 8 * c);
  const __half* hx = reinterpret_cast<const __half*>(&raw);
  float xf[8];
  float amax = 0.f;
  bool nan = false;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    xf[i] = __half2float(hx[i]);
    nan |= isnan(xf[i]);
    amax = fmaxf(amax, fabsf(xf[i]));
  }
#pragma unroll
  for (int off = 1; off < LPR; off <<= 1) {
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    nan |= __shfl_xor_sync(0xffffffffu, int(nan), off) != 0;
  }
  const __half sh = quant_scale<Q>(amax, nan);
  const float s = __half2float(sh);
  if (!active) return;
  const int64_t pos = (pl.pos_dev ? int64_t(*pl.pos_dev) : pl.pos_host) + row % pl.T;
  if (pos < 0 || pos >= pl.cap) return;
  const int64_t orow = (row / pl.T) * pl.cap + pos;
  if (c == 0) scales[orow] = sh;
  if (kInt4) {
    uint32_t packed = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) packed |= (uint32_t(quant_code<Q>(xf[i], s)) & 0xFu) << (4 * i);
    reinterpret_cast<uint32_t*>(codes)[(orow * D) / 8 + c] = packed;
  } else {
    uint32_t w0 = 0, w1 = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      w0 |= (uint32_t(quant_code<Q>(xf[i], s)) & 0xFFu) << (8 * i);
      w1 |= (uint32_t(quant_code<Q>(xf[4 + i], s)) & 0xFFu) << (8 * i);
    }
    reinterpret_cast<uint2*>(codes)[(orow * D) / 8 + c] = make_uint2(w0, w1);
  }
}

// Generic path: any D (even for int4), one warp per token, scalar accesses.
template <bool kInt4>
__global__ void __launch_bounds__(256) quantize_generic_kernel(const __half* __restrict__ X, void* __restrict__ codes,
                                                               __half* __restrict__ scales, int64_t rows, int D) {
  constexpr int Q = kInt4 ? 7 : 127;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (row >= rows) return;
  const __half* xr = X + row * D;
  float amax = 0.f;
  bool nan = false;
  for (int d = lane; d < D; d += 32) {
    const float x = __half2float(xr[d]);
    nan |= isnan(x);
    amax = fmaxf(amax, fabsf(x));
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    nan |= __shfl_xor_sync(0xffffffffu, int(nan), off) != 0;
  }
  const __half sh = quant_scale<Q>(amax, nan);
  const float s = __half2float(sh);
  if (lane == 0) scales[row] = sh;
  if (kInt4) {
    uint8_t* out = static_cast<uint8_t*>(codes) + row * (D / 2);
    for (int t = lane; t < D / 2; t += 32) {
      const int lo = quant_code<Q>(__half2float(xr[2 * t]), s);
      const int hi = quant_code<Q>(__half2float(xr[2 * t + 1]), s);
      out[t] = uint8_t((lo & 0xF) | ((hi & 0xF) << 4));
    }
  } else {
    int8_t* out = static_cast<int8_t*>(codes) + row * D;
    for (int d = lane; d < D; d += 32) out[d] = int8_t(quant_code<Q>(__half2float(xr[d]), s));
  }
}

template <bool kInt4>
cudaError_t launch_q(const void* X, void* codes, void* scales, int64_t rows, int D, cudaStream_t stream) {
  const __half* x = static_cast<const __half*>(X);
  __half* sc = static_cast<__half*>(scales);
  const bool aligned = (reinterpret_cast<uintptr_t>(X) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(codes) % (kInt4 ? 4 : 8) == 0);
  if (aligned && (D == 64 || D == 128 || D == 256)) {
    const int lpr = D / 8;
    const int64_t threads_needed = rows * lpr;
    const int64_t blocks = (threads_needed + 255) / 256;
    const QuantPlace pl{rows, rows, 0, nullptr};
    if (D == 64) quantize_vec_kernel<kInt4, 64><<<dim3(unsigned(blocks)), 256, 0, stream>>>(x, codes, sc, rows, pl);
    else if (D == 128) quantize_vec_kernel<kInt4, 128><<<dim3(unsigned(blocks)), 256, 0, stream>>>(x, codes, sc, rows, pl);
    else quantize_vec_kernel<kInt4, 256><<<dim3(unsigned(blocks)), 256, 0, stream>>>(x, codes, sc, rows, pl);
  } else {
    const int64_t blocks = (rows * 32 + 255) / 256;
    quantize_generic_kernel<kInt4><<<dim3(unsigned(blocks)), 256, 0, stream>>>(x, codes, sc, rows, D);
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_quantize_into(bool int4, const void* X, void* codes, void* scales, int64_t groups, int64_t T,
                                 int D, int64_t cap, int64_t pos_host, const int* pos_dev, cudaStream_t stream) {
  const __half* x = static_cast<const __half*>(X);
  __half* sc = static_cast<__half*>(scales);
  const int64_t rows = groups * T;
  const QuantPlace pl{T, cap, pos_host, pos_dev};
  const int64_t blocks = (rows * (D / 8) + 255) / 256;
  if (D == 64) {
    if (int4) quantize_vec_kernel<true, 64><<<dim3(unsigned(blocks)), 256, 0, stream>>>(x, codes, sc, rows, pl);
    else quantize_vec_kernel<false, 64><<<dim3(unsigned(blocks)), 256, 0, stream>>>(x, codes, sc, rows, pl);
  } else {
    if (int4) quantize_vec_kernel<true, 128><<<dim3(unsigned(blocks)), 256, 0, stream>>>(x, codes, sc, rows, pl);
    else quantize_vec_kernel<false, 128><<<dim3(unsigned(blocks)), 256, 0, stream>>>(x, codes, sc, rows, pl);
  }
  return cudaGetLastError();
}

cudaError_t launch_quantize(bool int4, const void* X, void* codes, void* scales, int64_t rows, int D,
                            cudaStream_t stream) {
  return int4 ? launch_q<true>(X, codes, scales, rows, D, stream) : launch_q<false>(X, codes, scales, rows, D, stream);
}

}  // namespace fqkv
