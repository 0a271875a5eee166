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
// HBM-bound: a persistent grid whose CTAs stream 16 KiB tiles of tokens into
// a shared-memory ring with bulk copies (quantize_tma_kernel below).
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

// Staged quantizer (D in {64, 128, 256}, X 16-byte aligned).  A persistent grid;
// in every CTA one producer thread streams 16 KiB tiles of consecutive tokens
// (8192 / D of them) into a 4-stage shared-memory ring with 1-D bulk copies
// completing on mbarriers, and 8 consumer warps quantize each tile: D/16 lanes
// per token, 16 elements per lane (two 16-byte shared-memory reads), so the
// per-token amax reduction and scale are shared by 16 elements.  Codes leave by
// plain 8-byte (int8) / 4-byte (int4) streaming stores, scales by 2-byte
// stores.  The exact quotients use the packed fp32x2 multiply and FMAs of
// sm_100 (the same IEEE operations as the scalar ones, two lanes at a time).
constexpr int kQConsumerWarps = 8;
constexpr int kQThreads = 32 * (kQConsumerWarps + 1);
constexpr int kQStages = 4;
constexpr int kQTileBytes = 16384;
constexpr size_t kQSmemBytes = 128 + size_t(kQStages) * kQTileBytes + 2 * kQStages * sizeof(uint64_t);

__device__ __forceinline__ unsigned long long f32x2_pack(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f32x2_unpack(unsigned long long v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ unsigned long long f32x2_mul(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ unsigned long long f32x2_fma(unsigned long long a, unsigned long long b,
                                                        unsigned long long c) {
  unsigned long long r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

// Codes of the fp16 pair h for a normal fp16 scale s (ns2 = (-s, -s), y2 = (1/s~, 1/s~)):
// quot_fast on both lanes, then code_pair_bits.
__device__ __forceinline__ uint32_t code_pair_fast(__half2 h, unsigned long long ns2, unsigned long long y2) {
  const float2 f = __half22float2(h);
  const unsigned long long x2 = f32x2_pack(f.x, f.y);
  const unsigned long long q0 = f32x2_mul(x2, y2);
  const unsigned long long q1 = f32x2_fma(f32x2_fma(ns2, q0, x2), y2, q0);
  float lo, hi;
  f32x2_unpack(q1, lo, hi);
  return code_pair_bits(lo, hi);
}

template <bool kInt4, int D, bool kPlace>
__global__ void __launch_bounds__(kQThreads, 3)
    quantize_tma_kernel(const __half* __restrict__ X, void* __restrict__ codes, __half* __restrict__ scales,
                        int64_t rows, QuantPlace pl, WaitCtl wc, int debug_skip_loads) {
  constexpr int kTok = kQTileBytes / (2 * D);  // tokens per tile
  constexpr int kLPT = D / 16;                  // lanes per token
  constexpr int kTPW = 32 / kLPT;               // tokens per warp and pass
  constexpr int kPass = kTok / (kQConsumerWarps * kTPW);
  constexpr int Q = kInt4 ? 7 : 127;
  static_assert(kPass == 2, "two passes of the consumer warps per tile");
  extern __shared__ uint8_t qsmem_raw[];
  uint8_t* smem = qsmem_raw + ((uint32_t(128) - (smem_u32(qsmem_raw) & 127u)) & 127u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + size_t(kQStages) * kQTileBytes);
  uint64_t* empty = full + kQStages;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t ntiles = (rows + kTok - 1) / kTok;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kQStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kQConsumerWarps);
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  // ------------------------------------------------------------ producer
  if (warp == kQConsumerWarps) {
    if (lane != 0 || debug_skip_loads) return;
    int it = 0;
    bool ok = true;
    for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
      const int st = it % kQStages;
      if (it >= kQStages) {
        if (*reinterpret_cast<volatile int*>(&abort_flag) ||
            !mbar_wait(&empty[st], ((it / kQStages) - 1) & 1, wc, kDevTimeoutEmpty)) {
          ok = false;
          break;
        }
      }
      const int64_t t0 = t * kTok;
      const uint32_t bytes = uint32_t(rows - t0 < kTok ? rows - t0 : kTok) * (2 * D);
      mbar_arrive_expect_tx(&full[st], bytes);
      bulk_g2s(smem + size_t(st) * kQTileBytes, X + t0 * D, bytes, &full[st]);
    }
    if (!ok) {
      for (int j = (it > kQStages ? it - kQStages : 0); j < it; ++j)
        mbar_wait(&full[j % kQStages], (j / kQStages) & 1, wc, kDevTimeoutDrain);
    }
    return;
  }

  // ------------------------------------------------------------ consumers
  const int c = lane % kLPT;  // 16-element chunk of the token
  const int tl = lane / kLPT;  // token slot of the warp
  const int64_t pos0 = kPlace ? (pl.pos_dev ? int64_t(*pl.pos_dev) : pl.pos_host) : 0;
  int it = 0;
  for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
    const int st = it % kQStages;
    const bool ok = mbar_wait(&full[st], (it / kQStages) & 1, wc, kDevTimeoutFull) &&
                    !*reinterpret_cast<volatile int*>(&abort_flag);
    if (!__all_sync(0xffffffffu, ok)) {
      if (lane == 0) abort_flag = 1;
      break;
    }
    const uint8_t* tile = smem + size_t(st) * kQTileBytes;
    const int64_t t0 = t * kTok;
    const int nt = int(rows - t0 < kTok ? rows - t0 : kTok);
#pragma unroll
    for (int p = 0; p < kPass; ++p) {
      const int wtok = (p * kQConsumerWarps + warp) * kTPW;  // first token of this warp and pass
      if (wtok >= nt) break;                                  // warp-uniform
      const int tok = wtok + tl;
      // tokens past nt (the last tile's tail) read stale tile bytes: computed, never stored
      const uint4 ra = *reinterpret_cast<const uint4*>(tile + tok * (2 * D) + 32 * c);
      const uint4 rb = *reinterpret_cast<const uint4*>(tile + tok * (2 * D) + 32 * c + 16);
      __half2 h2[8];
      *reinterpret_cast<uint4*>(&h2[0]) = ra;
      *reinterpret_cast<uint4*>(&h2[4]) = rb;
      // amax in fp16 (exact), NaN-propagating like torch.amax, as packed pairs
      __half2 m2 = __habs2(h2[0]);
#pragma unroll
      for (int i = 1; i < 8; ++i) m2 = __hmax2_nan(m2, __habs2(h2[i]));
#pragma unroll
      for (int off = 1; off < kLPT; off <<= 1) m2 = __hmax2_nan(m2, __shfl_xor_sync(0xffffffffu, m2, off));
      m2 = __hmax2_nan(m2, __lowhigh2highlow(m2));
      const bool nan = __hisnan(__low2half(m2));
      const __half sh = quant_scale_fast<Q>(__low2float(m2), nan);
      const float sc = __half2float(sh);
      if (tok >= nt) continue;
      const int64_t row = t0 + tok;
      int64_t orow = row;
      if constexpr (kPlace) {  // append into a cache: group row / T, position pos0 + row % T
        const int64_t pos = pos0 + row % pl.T;
        if (pos < 0 || pos >= pl.cap) continue;
        orow = (row / pl.T) * pl.cap + pos;
      }
      if (c == 0) scales[orow] = sh;
      // cb[i]: codes of elements 2i (byte 0) and 2i + 1 (byte 2)
      uint32_t cb[8];
      if (normal_fp16_scale(sc)) {
        const float y = rcp_approx(sc);
        const unsigned long long y2 = f32x2_pack(y, y), ns2 = f32x2_pack(-sc, -sc);
#pragma unroll
        for (int i = 0; i < 8; ++i) cb[i] = code_pair_fast(h2[i], ns2, y2);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float2 f = __half22float2(h2[i]);
          cb[i] = (uint32_t(quant_code<Q>(f.x, sc)) & 0xFFu) | ((uint32_t(quant_code<Q>(f.y, sc)) & 0xFFu) << 16);
        }
      }
      uint32_t w[4];  // elements 4i .. 4i + 3, one byte each
#pragma unroll
      for (int i = 0; i < 4; ++i) w[i] = __byte_perm(cb[2 * i], cb[2 * i + 1], 0x6420u);
      if constexpr (kInt4) {
        // byte t = (code[2t] & 0xF) | (code[2t+1] << 4): even elements from bytes 0/2, odd from 1/3
        uint32_t pk[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const uint32_t ev = __byte_perm(w[2 * i], w[2 * i + 1], 0x6420u) & 0x0F0F0F0Fu;
          const uint32_t od = (__byte_perm(w[2 * i], w[2 * i + 1], 0x7531u) << 4) & 0xF0F0F0F0u;
          pk[i] = ev | od;
        }
        unsigned int* dst = reinterpret_cast<unsigned int*>(codes) + (orow * D) / 8 + 2 * c;
        __stcs(dst, pk[0]);
        __stcs(dst + 1, pk[1]);
      } else {
        uint2* dst = reinterpret_cast<uint2*>(codes) + (orow * D) / 8 + 2 * c;
        __stcs(dst, make_uint2(w[0], w[1]));
        __stcs(dst + 1, make_uint2(w[2], w[3]));
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
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

template <bool kInt4, int D, bool kPlace>
cudaError_t launch_qt(const __half* x, void* codes, __half* sc, int64_t rows, const QuantPlace& pl,
                      const QuantCtl& ctl, cudaStream_t stream) {
  const int64_t ntiles = (rows * 2 * D + kQTileBytes - 1) / kQTileBytes;
  const unsigned blocks = unsigned(std::max<int64_t>(1, std::min<int64_t>(ntiles, ctl.ctas)));
  const WaitCtl wc{ctl.status, ctl.timeout_ns};
  quantize_tma_kernel<kInt4, D, kPlace><<<blocks, kQThreads, kQSmemBytes, stream>>>(x, codes, sc, rows, pl, wc,
                                                                                    ctl.debug_skip_loads);
  return cudaGetLastError();
}

template <bool kInt4, bool kPlace>
cudaError_t launch_qt_d(const __half* x, void* codes, __half* sc, int64_t rows, int D, const QuantPlace& pl,
                        const QuantCtl& ctl, cudaStream_t stream) {
  if (D == 64) return launch_qt<kInt4, 64, kPlace>(x, codes, sc, rows, pl, ctl, stream);
  if (D == 128) return launch_qt<kInt4, 128, kPlace>(x, codes, sc, rows, pl, ctl, stream);
  return launch_qt<kInt4, 256, kPlace>(x, codes, sc, rows, pl, ctl, stream);
}

template <bool kInt4, int D, bool kPlace>
cudaError_t prepare_qt() {
  return cudaFuncSetAttribute(quantize_tma_kernel<kInt4, D, kPlace>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              int(kQSmemBytes));
}

template <bool kInt4>
cudaError_t launch_q(const void* X, void* codes, void* scales, int64_t rows, int D, const QuantCtl& ctl,
                     cudaStream_t stream) {
  const __half* x = static_cast<const __half*>(X);
  __half* sc = static_cast<__half*>(scales);
  const bool aligned = (reinterpret_cast<uintptr_t>(X) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(codes) % (kInt4 ? 4 : 8) == 0);
  if (aligned && (D == 64 || D == 128 || D == 256)) {
    const QuantPlace pl{rows, rows, 0, nullptr};
    return launch_qt_d<kInt4, false>(x, codes, sc, rows, D, pl, ctl, stream);
  }
  const int64_t blocks = (rows * 32 + 255) / 256;
  quantize_generic_kernel<kInt4><<<dim3(unsigned(blocks)), 256, 0, stream>>>(x, codes, sc, rows, D);
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

cudaError_t quantize_kernel_prepare(int* ctas_per_sm) {
  cudaError_t e = cudaSuccess;
  for (cudaError_t r : {prepare_qt<false, 64, false>(), prepare_qt<false, 128, false>(), prepare_qt<false, 256, false>(),
                        prepare_qt<true, 64, false>(), prepare_qt<true, 128, false>(), prepare_qt<true, 256, false>(),
                        prepare_qt<false, 64, true>(), prepare_qt<false, 128, true>(), prepare_qt<false, 256, true>(),
                        prepare_qt<true, 64, true>(), prepare_qt<true, 128, true>(), prepare_qt<true, 256, true>()})
    if (e == cudaSuccess) e = r;
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(ctas_per_sm, quantize_tma_kernel<false, 128, false>, kQThreads,
                                                       kQSmemBytes);
}

cudaError_t launch_quantize_into(bool int4, const void* X, void* codes, void* scales, int64_t groups, int64_t T,
                                 int D, int64_t cap, int64_t pos_host, const int* pos_dev, const QuantCtl& ctl,
                                 cudaStream_t stream) {
  const __half* x = static_cast<const __half*>(X);
  __half* sc = static_cast<__half*>(scales);
  const QuantPlace pl{T, cap, pos_host, pos_dev};
  return int4 ? launch_qt_d<true, true>(x, codes, sc, groups * T, D, pl, ctl, stream)
              : launch_qt_d<false, true>(x, codes, sc, groups * T, D, pl, ctl, stream);
}

cudaError_t launch_quantize(bool int4, const void* X, void* codes, void* scales, int64_t rows, int D,
                            const QuantCtl& ctl, cudaStream_t stream) {
  return int4 ? launch_q<true>(X, codes, scales, rows, D, ctl, stream)
              : launch_q<false>(X, codes, scales, rows, D, ctl, stream);
}

}  // namespace fqkv
