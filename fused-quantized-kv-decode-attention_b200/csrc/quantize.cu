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
// amax propagates NaN like torch.amax.
//
// The quotient x / s: for a scale s that is a normal fp16 number (the common
// case) it is computed with Markstein's FMA-corrected division (P. Markstein,
// "IA-64 and Elementary Functions", 2000): y ~ 1/s from the hardware
// reciprocal approximation (relative error < 2^-22), q0 = x*y, r = x - s*q0
// (one FMA), q1 = q0 + r*y (one FMA).  q1 - x/s = (q0 - x/s)(1 - s*y), about
// 2^-21 of an fp32 ulp.  With fp16 operands, x/s = (A/B) 2^k with integers
// A, B < 2^11; such a quotient is never an fp32 rounding midpoint and, when it
// is not one, lies at least 2^-12 ulp away from every midpoint (the distance
// is a nonzero integer over B 2^(24-e)).  So q1 rounds exactly as the IEEE
// quotient -- for every fp16 pair, checked on the GPU over all (amax, x)
// pairs by the quantizer tests.  With s normal, |x/s| <= Q (1 + 2^-10), so the
// rounded code needs no clamp.  Scales that are 0, subnormal, inf or NaN
// (all-zero / tiny tokens, non-finite inputs) take the IEEE __fdiv_rn path
// with the clamp and the NaN rule.
//
// HBM-bound: a persistent grid; each lane keeps 16-byte loads of kUnroll
// tokens in flight (streaming, evict-first), D/8 lanes per token.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>

#include "device_common.cuh"
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

// fp32 quotient x / s for a normal fp16 scale s (y = approximate 1/s), rounded as IEEE division.
__device__ __forceinline__ float quot_fast(float x, float s, float y) {
  const float q0 = x * y;
  return fmaf(fmaf(-s, q0, x), y, q0);
}

// Codes of two fp32 quotients with |q| <= 128: fp16(q) (the reference's rounding of X / s),
// then round half to even to an integer by one fp16 addition of 1536 = 1.5 * 2^10 (the sums
// lie in [1408, 1664], where fp16 spacing is 1 and 1536 is even); each code is then the low
// byte of its half's bit pattern (1536 + k has mantissa 512 + k: low byte = k mod 256).
__device__ __forceinline__ uint32_t code_pair_bits(float q_lo, float q_hi) {
  const __half2 r = __floats2half2_rn(q_lo, q_hi);
  const __half2 m = __hadd2(r, __half2half2(__ushort_as_half(0x6600u)));  // + 1536
  return *reinterpret_cast<const uint32_t*>(&m);  // byte 0: code(q_lo), byte 2: code(q_hi)
}

__device__ __forceinline__ float rcp_approx(float s) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(s));
  return y;
}

// s is a normal fp16 number: the fast division applies (see the file comment)
__device__ __forceinline__ bool normal_fp16_scale(float s) { return s >= 6.103515625e-05f && s <= 65504.f; }

template <int Q>
__device__ __forceinline__ __half quant_scale(float amax, bool any_nan) {
  const float a = any_nan ? __int_as_float(0x7fc00000) : amax;
  return __float2half_rn(__fdiv_rn(a, float(Q)));
}

// The same scale for a finite amax by the FMA-corrected division (amax and Q are
// fp16 values, so the argument of the file comment applies); inf / NaN take
// quant_scale's IEEE path.
template <int Q>
__device__ __forceinline__ __half quant_scale_fast(float amax, bool any_nan) {
  if (any_nan || !(amax <= 65504.f)) return quant_scale<Q>(amax, any_nan);
  constexpr float kY = 1.0f / float(Q);  // within half an ulp of 1/Q
  const float q0 = amax * kY;
  return __float2half_rn(fmaf(fmaf(-float(Q), q0, amax), kY, q0));
}

// Output placement: token `row` of the input (rows = groups x T tokens) goes
// to output row (row / T) * cap + pos + row % T, where pos is *pos_dev when
// given (a growing KV cache) else pos_host; tokens landing at or past `cap`
// are not written.  The plain quantizer uses T = cap = rows, pos = 0.
struct QuantPlace {
  int64_t T, cap, pos_host;
  const int* pos_dev;
};

// Tokens whose 16-byte loads each lane of the quantizer keeps in flight.
constexpr int kUnroll = 3;


// Vectorised path: D in {64, 128, 256}; LPR = D/8 lanes per token, each with 8
// consecutive elements.  Persistent: warp w handles tokens w*RPW + j + i*stride.
template <bool kInt4, int D, bool kPlace>
__global__ void __launch_bounds__(256, 4) quantize_vec_kernel(const __half* __restrict__ X, void* __restrict__ codes,
                                                           __half* __restrict__ scales, int64_t rows,
                                                           QuantPlace pl) {
  constexpr int LPR = D / 8;
  constexpr int RPW = 32 / LPR;
  constexpr int Q = kInt4 ? 7 : 127;
  const int lane = threadIdx.x & 31;
  const int c = lane % LPR;
  const int64_t warps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  const int64_t stride = warps * RPW;  // tokens covered by one pass of all warps
  const int64_t pos0 = kPlace ? (pl.pos_dev ? int64_t(*pl.pos_dev) : pl.pos_host) : 0;
  for (int64_t wbase = ((int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5) * RPW; wbase < rows;
       wbase += kUnroll * stride) {  // warp-uniform: every lane takes part in the shuffles below
    uint4 raw[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t row = wbase + lane / LPR + u * stride;
      raw[u] = row < rows ? __ldcs(reinterpret_cast<const uint4*>(X + row * D + 8 * c)) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t row = wbase + lane / LPR + u * stride;
      if (wbase + u * stride >= rows) break;  // warp-uniform
      const __half2* h2 = reinterpret_cast<const __half2*>(&raw[u]);
      // amax in fp16 (exact), NaN-propagating like torch.amax, reduced over the token's lanes
      // as packed fp16 pairs: one shuffle per step carries both the maximum and any NaN
      __half2 m2 = __habs2(h2[0]);
#pragma unroll
      for (int i = 1; i < 4; ++i) m2 = __hmax2_nan(m2, __habs2(h2[i]));
#pragma unroll
      for (int off = 1; off < LPR; off <<= 1) m2 = __hmax2_nan(m2, __shfl_xor_sync(0xffffffffu, m2, off));
      m2 = __hmax2_nan(m2, __lowhigh2highlow(m2));
      const bool nan = __hisnan(__low2half(m2));
      const float amax = __low2float(m2);
      const __half sh = quant_scale_fast<Q>(amax, nan);
      const float sc = __half2float(sh);
      if (row >= rows) continue;
      int64_t orow = row;
      if constexpr (kPlace) {  // append into a cache: group row / T, position pos0 + row % T
        const int64_t pos = pos0 + row % pl.T;
        if (pos < 0 || pos >= pl.cap) continue;
        orow = (row / pl.T) * pl.cap + pos;
      }
      if (c == 0) scales[orow] = sh;
      // cb[i]: codes of elements 2i (byte 0) and 2i + 1 (byte 2)
      uint32_t cb[4];
      if (normal_fp16_scale(sc)) {
        const float y = rcp_approx(sc);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(h2[i]);
          cb[i] = code_pair_bits(quot_fast(f.x, sc, y), quot_fast(f.y, sc, y));
        }
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(h2[i]);
          cb[i] = (uint32_t(quant_code<Q>(f.x, sc)) & 0xFFu) | ((uint32_t(quant_code<Q>(f.y, sc)) & 0xFFu) << 16);
        }
      }
      const uint32_t w0 = __byte_perm(cb[0], cb[1], 0x6420u);  // elements 0..3, one byte each
      const uint32_t w1 = __byte_perm(cb[2], cb[3], 0x6420u);  // elements 4..7
      if (kInt4) {
        // byte t = (code[2t] & 0xF) | (code[2t+1] << 4): even elements from bytes 0/2, odd from 1/3
        const uint32_t ev = __byte_perm(w0, w1, 0x6420u) & 0x0F0F0F0Fu;
        const uint32_t od = (__byte_perm(w0, w1, 0x7531u) << 4) & 0xF0F0F0F0u;
        __stcs(reinterpret_cast<unsigned int*>(codes) + (orow * D) / 8 + c, ev | od);
      } else {
        __stcs(reinterpret_cast<uint2*>(codes) + (orow * D) / 8 + c, make_uint2(w0, w1));
      }
    }
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

// Persistent grid of the vectorised quantizer: enough 256-thread CTAs for every
// token once (kUnroll tokens per lane), at most 4 per SM (64 registers per thread).
int64_t quant_blocks(int64_t rows, int D, int sm_count) {
  const int64_t warps_needed = (rows * (D / 8) + 31) / 32;
  const int64_t blocks = (warps_needed + kUnroll * 8 - 1) / (kUnroll * 8);
  return std::max<int64_t>(1, std::min<int64_t>(blocks, int64_t(sm_count) * 4));
}

template <bool kInt4>
cudaError_t launch_q(const void* X, void* codes, void* scales, int64_t rows, int D, int sm_count, cudaStream_t stream) {
  const __half* x = static_cast<const __half*>(X);
  __half* sc = static_cast<__half*>(scales);
  const bool aligned = (reinterpret_cast<uintptr_t>(X) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(codes) % (kInt4 ? 4 : 8) == 0);
  if (aligned && (D == 64 || D == 128 || D == 256)) {
    const unsigned blocks = unsigned(quant_blocks(rows, D, sm_count));
    const QuantPlace pl{rows, rows, 0, nullptr};
    if (D == 64) quantize_vec_kernel<kInt4, 64, false><<<blocks, 256, 0, stream>>>(x, codes, sc, rows, pl);
    else if (D == 128) quantize_vec_kernel<kInt4, 128, false><<<blocks, 256, 0, stream>>>(x, codes, sc, rows, pl);
    else quantize_vec_kernel<kInt4, 256, false><<<blocks, 256, 0, stream>>>(x, codes, sc, rows, pl);
  } else {
    const int64_t blocks = (rows * 32 + 255) / 256;
    quantize_generic_kernel<kInt4><<<dim3(unsigned(blocks)), 256, 0, stream>>>(x, codes, sc, rows, D);
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------------- RoPE + append
// One decode step of a Llama-style attention block after its (fused) q/k/v
// projection: rotary embedding of q and k exactly as transformers'
// apply_rotary_pos_emb evaluates it in the model dtype T (fp16 or bf16):
//   out_i = T( T(x_i * cos_i) + T(rot_i * sin_i) ),  rot = cat(-x[D/2:], x[:D/2])
// (each product is exact in fp32 and rounded once to T, the sum is an fp32
// add rounded to T -- torch's elementwise ops on T tensors), then the cast to
// fp16 the attention takes (x.to(float16)).  q goes to q_out [B, Hq, D] fp16;
// k (rotated) and v go to the cache at position pos: fp16 rows, or the
// reference quantizer's int8 codes + fp16 scale of the fp16 row (bit-exact with
// qpt).  One warp per head row; lane l holds elements l + 32m, so every
// rotate-half partner (i, i + D/2) is in the same lane.
template <typename T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <typename T>
__device__ __forceinline__ float round_t(float x);
template <>
__device__ __forceinline__ float round_t<__half>(float x) { return __half2float(__float2half_rn(x)); }
template <>
__device__ __forceinline__ float round_t<__nv_bfloat16>(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

struct RopeAppendArgs {
  const void* qkv;
  int64_t qkv_stride;        // elements between consecutive sequences' rows
  const void* cos_t;         // [table_rows, D] in T
  const void* sin_t;
  int64_t table_rows;
  int64_t pos_host;
  const int* pos_dev;
  __half* q_out;             // [B, Hq, D]
  void* k_cache;             // [B, Hkv, cap, D] f16 or i8
  void* v_cache;
  __half* k_scales;          // [B, Hkv, cap] (int8 cache)
  __half* v_scales;
  int B, Hq, Hkv, cap;
};

template <typename T, int D, bool kInt8>
__global__ void __launch_bounds__(256) rope_append_kernel(const RopeAppendArgs a) {
  pdl_wait_primary();
  pdl_launch_dependents();
  constexpr int M = D / 32;  // elements per lane
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int heads = a.Hq + 2 * a.Hkv;
  if (row >= int64_t(a.B) * heads) return;
  const int b = int(row / heads), slot = int(row % heads);
  const int64_t pos = a.pos_dev ? int64_t(*a.pos_dev) : a.pos_host;
  if (pos < 0 || pos >= a.table_rows) return;
  const T* x = static_cast<const T*>(a.qkv) + b * a.qkv_stride + int64_t(slot) * D;
  float v[M];
#pragma unroll
  for (int m = 0; m < M; ++m) v[m] = to_f<T>(x[lane + 32 * m]);
  const bool is_v = slot >= a.Hq + a.Hkv;
  if (!is_v) {
    const T* c = static_cast<const T*>(a.cos_t) + pos * D;
    const T* sn = static_cast<const T*>(a.sin_t) + pos * D;
    float r[M];
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const int i = lane + 32 * m;
      const float rot = m < M / 2 ? -v[m + M / 2] : v[m - M / 2];
      r[m] = round_t<T>(round_t<T>(v[m] * to_f<T>(c[i])) + round_t<T>(rot * to_f<T>(sn[i])));
    }
#pragma unroll
    for (int m = 0; m < M; ++m) v[m] = r[m];
  }
  __half h[M];
#pragma unroll
  for (int m = 0; m < M; ++m) h[m] = __float2half_rn(v[m]);  // x.to(float16)
  if (slot < a.Hq) {
    __half* q = a.q_out + (int64_t(b) * a.Hq + slot) * D;
#pragma unroll
    for (int m = 0; m < M; ++m) q[lane + 32 * m] = h[m];
    return;
  }
  if (pos >= a.cap) return;
  const int kh = is_v ? slot - a.Hq - a.Hkv : slot - a.Hq;
  const int64_t crow = (int64_t(b) * a.Hkv + kh) * a.cap + pos;
  if constexpr (!kInt8) {
    __half* dst = static_cast<__half*>(is_v ? a.v_cache : a.k_cache) + crow * D;
#pragma unroll
    for (int m = 0; m < M; ++m) dst[lane + 32 * m] = h[m];
  } else {
    float amax = 0.f;
    bool nan = false;
    float xf[M];
#pragma unroll
    for (int m = 0; m < M; ++m) {
      xf[m] = __half2float(h[m]);
      nan |= isnan(xf[m]);
      amax = fmaxf(amax, fabsf(xf[m]));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
      nan |= __shfl_xor_sync(0xffffffffu, int(nan), off) != 0;
    }
    const __half sh = quant_scale<127>(amax, nan);
    const float sc = __half2float(sh);
    int8_t* dst = static_cast<int8_t*>(is_v ? a.v_cache : a.k_cache) + crow * D;
#pragma unroll
    for (int m = 0; m < M; ++m) dst[lane + 32 * m] = int8_t(quant_code<127>(xf[m], sc));
    if (lane == 0) (is_v ? a.v_scales : a.k_scales)[crow] = sh;
  }
}

template <typename T, int D>
cudaError_t launch_rope_append_t(const RopeAppendArgs& a, bool int8, cudaStream_t stream) {
  const int64_t rows = int64_t(a.B) * (a.Hq + 2 * a.Hkv);
  const unsigned blocks = unsigned((rows * 32 + 255) / 256);
  if (int8) return launch_pdl(rope_append_kernel<T, D, true>, dim3(blocks), dim3(256), 0, stream, a);
  return launch_pdl(rope_append_kernel<T, D, false>, dim3(blocks), dim3(256), 0, stream, a);
}

}  // namespace

cudaError_t launch_rope_append(bool bf16, bool int8_cache, const void* qkv, int64_t qkv_stride, const void* cos_t,
                               const void* sin_t, int64_t table_rows, int64_t pos_host, const int* pos_dev,
                               void* q_out, void* k_cache, void* v_cache, void* k_scales, void* v_scales, int B,
                               int Hq, int Hkv, int D, int cap, cudaStream_t stream) {
  const RopeAppendArgs a{qkv,     qkv_stride, cos_t,   sin_t,   table_rows,
                         pos_host, pos_dev,   static_cast<__half*>(q_out), k_cache, v_cache,
                         static_cast<__half*>(k_scales), static_cast<__half*>(v_scales), B, Hq, Hkv, cap};
  if (bf16)
    return D == 128 ? launch_rope_append_t<__nv_bfloat16, 128>(a, int8_cache, stream)
                    : launch_rope_append_t<__nv_bfloat16, 64>(a, int8_cache, stream);
  return D == 128 ? launch_rope_append_t<__half, 128>(a, int8_cache, stream)
                  : launch_rope_append_t<__half, 64>(a, int8_cache, stream);
}

cudaError_t launch_quantize_into(bool int4, const void* X, void* codes, void* scales, int64_t groups, int64_t T,
                                 int D, int64_t cap, int64_t pos_host, const int* pos_dev, int sm_count,
                                 cudaStream_t stream) {
  const __half* x = static_cast<const __half*>(X);
  __half* sc = static_cast<__half*>(scales);
  const int64_t rows = groups * T;
  const QuantPlace pl{T, cap, pos_host, pos_dev};
  const unsigned blocks = unsigned(quant_blocks(rows, D, sm_count));
  if (D == 64) {
    if (int4) quantize_vec_kernel<true, 64, true><<<blocks, 256, 0, stream>>>(x, codes, sc, rows, pl);
    else quantize_vec_kernel<false, 64, true><<<blocks, 256, 0, stream>>>(x, codes, sc, rows, pl);
  } else {
    if (int4) quantize_vec_kernel<true, 128, true><<<blocks, 256, 0, stream>>>(x, codes, sc, rows, pl);
    else quantize_vec_kernel<false, 128, true><<<blocks, 256, 0, stream>>>(x, codes, sc, rows, pl);
  }
  return cudaGetLastError();
}

cudaError_t launch_quantize(bool int4, const void* X, void* codes, void* scales, int64_t rows, int D, int sm_count,
                            cudaStream_t stream) {
  return int4 ? launch_q<true>(X, codes, scales, rows, D, sm_count, stream)
              : launch_q<false>(X, codes, scales, rows, D, sm_count, stream);
}

}  // namespace fqkv
