// Small fused kernels of the graph-captured Llama decode step around attention.
//
// A transformers decode step spends most of its non-GEMM time in the
// elementwise and reduction kernels of LlamaRMSNorm (cast to fp32, pow, mean,
// add eps, rsqrt, two multiplies, cast back) and of the SwiGLU MLP.  These
// kernels do the same arithmetic in one launch each:
//
//  * add_rmsnorm: h <- T(h + delta) (optional), y <- T(w * T(h32 * rsqrt(mean(h32^2) + eps)))
//    with T the model dtype (fp16 / bf16), exactly LlamaRMSNorm's sequence of
//    roundings; only the order of the fp32 sum of squares differs from torch's
//    reduction (the mean can differ in the last fp32 bit).
//  * silu_mul: y <- T(T(silu(g)) * u) on a fused [gate | up] projection, with
//    silu(x) = x / (1 + exp(-x)) in fp32 as torch evaluates it.
//
// One CTA per row for add_rmsnorm (hidden sizes up to 8192), a grid-stride
// loop for silu_mul.  Both are HBM-bound and tiny; the point is the launch
// count of a decode step.
#include <type_traits>
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

template <typename T>
__device__ __forceinline__ float ld(const T* p, int64_t i);
template <>
__device__ __forceinline__ float ld<__half>(const __half* p, int64_t i) { return __half2float(p[i]); }
template <>
__device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) { return __bfloat162float(p[i]); }
template <typename T>
__device__ __forceinline__ T cvt(float x);
template <>
__device__ __forceinline__ __half cvt<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 cvt<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <typename T>
__device__ __forceinline__ float rnd(float x);
template <>
__device__ __forceinline__ float rnd<__half>(float x) { return __half2float(__float2half_rn(x)); }
template <>
__device__ __forceinline__ float rnd<__nv_bfloat16>(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

constexpr int kNormThreads = 256;
constexpr int kMaxPerThread = 32;  // hidden size <= 8192

template <typename T>
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(T* __restrict__ h, const T* __restrict__ delta,
                                                                   const T* __restrict__ w, T* __restrict__ y, int H,
                                                                   float eps) {
  pdl_wait_primary();
  pdl_launch_dependents();
  const int64_t row = blockIdx.x;
  T* hr = h + row * H;
  const T* dr = delta ? delta + row * H : nullptr;
  float v[kMaxPerThread];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kMaxPerThread; ++k) {
    const int i = threadIdx.x + k * kNormThreads;
    if (i < H) {
      float x = ld<T>(hr, i);
      if (dr) {
        x = rnd<T>(x + ld<T>(dr, i));  // the residual add, rounded to the model dtype
        hr[i] = cvt<T>(x);
      }
      v[k] = x;
      ss = fmaf(x, x, ss);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  __shared__ float part[kNormThreads / 32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < kNormThreads / 32; ++k) tot += part[k];
  const float r = rsqrtf(tot * (1.f / float(H)) + eps);
  T* yr = y + row * H;
#pragma unroll
  for (int k = 0; k < kMaxPerThread; ++k) {
    const int i = threadIdx.x + k * kNormThreads;
    if (i < H) yr[i] = cvt<T>(ld<T>(w, i) * rnd<T>(v[k] * r));
  }
}

// Vectorised variant: H % 8 == 0, 16-byte aligned rows; every thread owns
// chunks of 8 consecutive elements and issues the loads of h, delta and the
// weight together, so a row costs one memory round trip before the reduction.
constexpr int kMaxChunks = 4;  // H <= 8 * 256 * 4 = 8192
template <typename T>
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_vec_kernel(T* __restrict__ h, const T* __restrict__ delta,
                                                                       const T* __restrict__ w, T* __restrict__ y,
                                                                       int H, float eps) {
  pdl_wait_primary();
  pdl_launch_dependents();
  const int64_t row = blockIdx.x;
  const int chunks = H / 8;
  uint4 hv[kMaxChunks], dv[kMaxChunks], wv[kMaxChunks];
#pragma unroll
  for (int k = 0; k < kMaxChunks; ++k) {
    const int c = threadIdx.x + k * kNormThreads;
    if (c < chunks) {
      hv[k] = reinterpret_cast<const uint4*>(h + row * H)[c];
      if (delta) dv[k] = reinterpret_cast<const uint4*>(delta + row * H)[c];
      wv[k] = reinterpret_cast<const uint4*>(w)[c];
    }
  }
  float v[kMaxChunks][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kMaxChunks; ++k) {
    const int c = threadIdx.x + k * kNormThreads;
    if (c < chunks) {
      const T* hp = reinterpret_cast<const T*>(&hv[k]);
      const T* dp = reinterpret_cast<const T*>(&dv[k]);
      uint4 out;
      T* op = reinterpret_cast<T*>(&out);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float x = ld<T>(hp, e);
        if (delta) {
          x = rnd<T>(x + ld<T>(dp, e));  // the residual add, rounded to the model dtype
          op[e] = cvt<T>(x);
        }
        v[k][e] = x;
        ss = fmaf(x, x, ss);
      }
      if (delta) reinterpret_cast<uint4*>(h + row * H)[c] = out;
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  __shared__ float part[kNormThreads / 32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < kNormThreads / 32; ++k) tot += part[k];
  const float r = rsqrtf(tot * (1.f / float(H)) + eps);
#pragma unroll
  for (int k = 0; k < kMaxChunks; ++k) {
    const int c = threadIdx.x + k * kNormThreads;
    if (c < chunks) {
      const T* wp = reinterpret_cast<const T*>(&wv[k]);
      uint4 out;
      T* op = reinterpret_cast<T*>(&out);
#pragma unroll
      for (int e = 0; e < 8; ++e) op[e] = cvt<T>(ld<T>(wp, e) * rnd<T>(v[k][e] * r));
      reinterpret_cast<uint4*>(y + row * H)[c] = out;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) silu_mul_kernel(const T* __restrict__ gu, T* __restrict__ y, int64_t rows,
                                                       int I, int64_t row_stride) {
  pdl_wait_primary();
  pdl_launch_dependents();
  const int64_t n = rows * I;
  for (int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < n;
       idx += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = idx / I;
    const int c = int(idx - r * I);
    const float g = ld<T>(gu, r * row_stride + c);
    const float u = ld<T>(gu, r * row_stride + I + c);
    const float s = rnd<T>(g / (1.f + expf(-g)));
    y[idx] = cvt<T>(s * u);
  }
}

// Same arithmetic, 8 elements per thread with 16-byte loads and stores
// (I % 8 == 0, row stride % 8 == 0, gu and y 16-byte aligned).
template <typename T>
__global__ void __launch_bounds__(256) silu_mul_vec_kernel(const T* __restrict__ gu, T* __restrict__ y,
                                                           int64_t rows, int I8, int64_t stride8) {
  pdl_wait_primary();
  pdl_launch_dependents();
  const int64_t n = rows * I8;
  const uint4* g4 = reinterpret_cast<const uint4*>(gu);
  for (int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < n;
       idx += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = idx / I8;
    const int c = int(idx - r * I8);
    const uint4 gv = g4[r * stride8 + c];
    const uint4 uv = g4[r * stride8 + I8 + c];
    const T* gp = reinterpret_cast<const T*>(&gv);
    const T* up = reinterpret_cast<const T*>(&uv);
    uint4 ov;
    T* op = reinterpret_cast<T*>(&ov);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float g = ld<T>(gp, e);
      const float s = rnd<T>(g / (1.f + expf(-g)));
      op[e] = cvt<T>(s * ld<T>(up, e));
    }
    reinterpret_cast<uint4*>(y)[idx] = ov;
  }
}

// Small-batch GEMV: y [B, N] = x [B, K] @ W[N, K]^T (+ bias), B <= 4, fp32
// accumulation, output rounded to the model dtype.  A batch-1..4 decode step's
// projections are weight-streaming GEMVs that cuBLAS's batch-1 kernels run far
// below HBM speed.  A row group of WPR warps owns RPW weight rows (two rows of
// one warp when K <= 2048; at batch 1 one row split into WPR K-slices of
// <= 2048 elements), and a lane issues a pass of 8 independent 16-byte loads
// per row, 256 elements apart (one pass per 2048 elements of its slice).  x is
// staged in shared memory; the WPR slice sums of a row are added in a fixed
// order.
// K % 256 == 0, rows 16-byte aligned.
// Epilogues (kEpi):
//  * kEpiSwiGLU (a concatenated [gate | up] projection, W [2N, K]): a warp owns
//    the gate row n and the up row N + n and writes y[b, n] = T(T(silu(g)) * u),
//    g and u the two projections rounded to T -- the same values as the GEMV of
//    both halves followed by the separate SwiGLU kernel, in one launch.
//  * kEpiRope (batch 1, the fused q/k/v projection of a decode step, N = (Hq +
//    2 Hkv) D rows): a warp owns rows i and i + D/2 of one head -- a rotate-half
//    pair -- and applies RoPE to q and k heads, casts to fp16 and writes q to
//    q_out and k / v into the fp16 cache at the step's position: the values of
//    the GEMV followed by rope_append_kernel (see quantize.cu), in one launch.
constexpr int kGemvWarps = 8;
constexpr int kEpiPlain = 0, kEpiSwiGLU = 1, kEpiRope = 2;
template <typename T, int B, int RPW, int WPR, int kEpi = kEpiPlain>
__global__ void __launch_bounds__(32 * kGemvWarps) gemv_kernel(const void* __restrict__ x, const T* __restrict__ W,
                                                               const T* __restrict__ bias, T* __restrict__ y, int N,
                                                               int K, bool x_f16, const GemvRope rp) {
  constexpr bool kSwi = kEpi == kEpiSwiGLU;
  constexpr bool kRope = kEpi == kEpiRope;
  static_assert(kEpi == kEpiPlain || (RPW == 2 && WPR == 1), "paired epilogues: two rows per warp");
  static_assert(!kRope || B == 1, "the RoPE epilogue serves batch 1");
  extern __shared__ uint4 xs[];  // [B][K/8] chunks
  __shared__ float red[kGemvWarps][RPW][B];
  constexpr int kGroups = kGemvWarps / WPR;  // row groups per CTA
  const int kc = K / 8;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  // first weight row of this warp; its rows are n0 + r, or n0 and N + n0 (SwiGLU), or n0 and n0 + D/2
  // (RoPE: head n0 / D, rotate-half pair i, i + D/2)
  const int gw = blockIdx.x * kGroups + warp / WPR;
  const int half = kRope ? rp.D / 2 : 0;
  const int n0 = kSwi ? gw : kRope ? (gw / half) * rp.D + gw % half : gw * RPW;
  const bool warp_live = kSwi ? n0 < N : kRope ? 2 * gw < N : n0 < N;
  const int kcw = kc / WPR;                  // chunks of this warp's K slice
  const int c_lo = (warp % WPR) * kcw, c_hi = c_lo + kcw;
  constexpr int U = 8;  // chunks per lane per pass: a 2048-element slice is one pass
  uint4 wv[RPW][U];
  // the first pass's weight loads are issued before x is staged, so the two
  // memory round trips overlap
  auto load_w = [&](int c) {
#pragma unroll
    for (int r = 0; r < RPW; ++r)
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int cc = c + 32 * u;
        const int wr = kSwi ? n0 + r * N : kRope ? n0 + r * half : n0 + r;
        const bool live = kEpi == kEpiPlain ? n0 + r < N : warp_live;
        if (cc < c_hi && live) wv[r][u] = reinterpret_cast<const uint4*>(W + int64_t(wr) * K)[cc];
        else wv[r][u] = make_uint4(0, 0, 0, 0);
      }
  };
  load_w(c_lo + lane);
  // Batch 1 is launched with programmatic dependent launch: the weights are
  // not written by the kernel this launch may overlap, only the activations
  // wait for it.  (The next kernel is released when this grid completes.)
  pdl_wait_primary();
  if (std::is_same<T, __half>::value || !x_f16) {
    for (int i = threadIdx.x; i < B * kc; i += blockDim.x) xs[i] = reinterpret_cast<const uint4*>(x)[i];
  } else {
    // fp16 activations for bf16 weights (the attention output): rounded to
    // bf16 here, as a separate cast would
    for (int i = threadIdx.x; i < B * kc; i += blockDim.x) {
      const uint4 hv = reinterpret_cast<const uint4*>(x)[i];
      const __half* hp = reinterpret_cast<const __half*>(&hv);
      uint4 bv;
      T* bp = reinterpret_cast<T*>(&bv);
#pragma unroll
      for (int e = 0; e < 8; ++e) bp[e] = cvt<T>(__half2float(hp[e]));
      xs[i] = bv;
    }
  }
  __syncthreads();
  float acc[RPW][B];
#pragma unroll
  for (int r = 0; r < RPW; ++r)
#pragma unroll
    for (int b = 0; b < B; ++b) acc[r][b] = 0.f;
  if (warp_live) {
    for (int c = c_lo + lane; c < c_hi; c += 32 * U) {
      if (c != c_lo + lane) load_w(c);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int cc = c + 32 * u;
        if (cc >= c_hi) continue;
#pragma unroll
        for (int b = 0; b < B; ++b) {
          const uint4 xv = xs[b * kc + cc];
          const T* xp = reinterpret_cast<const T*>(&xv);
#pragma unroll
          for (int r = 0; r < RPW; ++r) {
            const T* wp = reinterpret_cast<const T*>(&wv[r][u]);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[r][b] = fmaf(ld<T>(wp, e), ld<T>(xp, e), acc[r][b]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < RPW; ++r)
#pragma unroll
    for (int b = 0; b < B; ++b) {
      float v = acc[r][b];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      acc[r][b] = v;
    }
  if constexpr (kRope) {
    const int64_t pos = rp.pos_dev ? int64_t(*rp.pos_dev) : rp.pos_host;
    if (lane == 0 && warp_live && pos >= 0 && pos < rp.table_rows) {
      const int head = n0 / rp.D, i = n0 % rp.D;
      float lo = rnd<T>(acc[0][0] + (bias ? ld<T>(bias, n0) : 0.f));
      float hi = rnd<T>(acc[1][0] + (bias ? ld<T>(bias, n0 + half) : 0.f));
      if (head < rp.Hq + rp.Hkv) {  // q and k heads: out = T(T(x cos) + T(rotate_half(x) sin))
        const T* c = static_cast<const T*>(rp.cos_t) + pos * rp.D;
        const T* sn = static_cast<const T*>(rp.sin_t) + pos * rp.D;
        const float rl = rnd<T>(rnd<T>(lo * ld<T>(c, i)) + rnd<T>(-hi * ld<T>(sn, i)));
        const float rh = rnd<T>(rnd<T>(hi * ld<T>(c, i + half)) + rnd<T>(lo * ld<T>(sn, i + half)));
        lo = rl;
        hi = rh;
      }
      __half* dst = nullptr;
      if (head < rp.Hq) {
        dst = rp.q_out + int64_t(head) * rp.D;
      } else if (pos < rp.cap) {
        const bool is_v = head >= rp.Hq + rp.Hkv;
        const int kh = head - rp.Hq - (is_v ? rp.Hkv : 0);
        dst = (is_v ? rp.v_cache : rp.k_cache) + (int64_t(kh) * rp.cap + pos) * rp.D;
      }
      if (dst) {
        dst[i] = __float2half_rn(lo);  // x.to(float16)
        dst[i + half] = __float2half_rn(hi);
      }
    }
  } else if constexpr (kSwi) {
    if (lane == 0 && n0 < N) {
      const float bg = bias ? ld<T>(bias, n0) : 0.f, bu = bias ? ld<T>(bias, N + n0) : 0.f;
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const float g = rnd<T>(acc[0][b] + bg);
        const float s = rnd<T>(g / (1.f + expf(-g)));
        y[int64_t(b) * N + n0] = cvt<T>(s * rnd<T>(acc[1][b] + bu));
      }
    }
  } else if constexpr (WPR == 1) {
    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        if (n0 + r >= N) break;
        const float bv = bias ? ld<T>(bias, n0 + r) : 0.f;
#pragma unroll
        for (int b = 0; b < B; ++b) y[int64_t(b) * N + n0 + r] = cvt<T>(acc[r][b] + bv);
      }
    }
  } else {
    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < RPW; ++r)
#pragma unroll
        for (int b = 0; b < B; ++b) red[warp][r][b] = acc[r][b];
    }
    __syncthreads();
    const int t = threadIdx.x;
    if (t < kGroups * RPW * B) {
      const int g = t / (RPW * B), r = (t / B) % RPW, b = t % B;
      const int n = (blockIdx.x * kGroups + g) * RPW + r;
      if (n < N) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < WPR; ++w) v += red[g * WPR + w][r][b];
        const float bv = bias ? ld<T>(bias, n) : 0.f;
        y[int64_t(b) * N + n] = cvt<T>(v + bv);
      }
    }
  }
}

template <typename T, int B, int RPW, int WPR, int kEpi = kEpiPlain>
cudaError_t launch_gemv_k(const void* x, const void* W, const void* bias, void* y, int N, int K, bool x_f16,
                          cudaStream_t stream, const GemvRope& rp = GemvRope{}) {
  const size_t smem = size_t(B) * K * sizeof(T);
  // rows of N per CTA (SwiGLU: outputs, each two weight rows)
  constexpr int kRowsPerCta = kGemvWarps / WPR * (kEpi == kEpiSwiGLU ? 1 : RPW);
  const unsigned blocks = unsigned((N + kRowsPerCta - 1) / kRowsPerCta);
  auto fn = gemv_kernel<T, B, RPW, WPR, kEpi>;
  // dynamic + static (the slice sums) shared memory above the 48 KB default needs the opt-in
  if (smem + sizeof(float) * kGemvWarps * RPW * B > 48 * 1024)
    cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  // Dependent launch measured faster in the decode step at batch 1 only (Llama-1B
  // shapes on B200: 802 -> 772 us per step) and slower at batch 2 and 4 (886 ->
  // 976, 1000 -> 1108 us).
  if constexpr (B == 1)
    return launch_pdl(fn, dim3(blocks), dim3(32 * kGemvWarps), smem, stream, x, static_cast<const T*>(W),
                      static_cast<const T*>(bias), static_cast<T*>(y), N, K, x_f16, rp);
  fn<<<blocks, 32 * kGemvWarps, smem, stream>>>(x, static_cast<const T*>(W), static_cast<const T*>(bias),
                                               static_cast<T*>(y), N, K, x_f16, rp);
  return cudaGetLastError();
}

// K <= 2048: two rows per warp, one pass.  Longer rows at batch 1: the
// fewest warps per row (a power of two, <= 8) that cut it into K-slices of at
// most 2048 elements (down projection K = 8192: 9.35 -> 8.52 us on B200).  At
// batch 2..4 the x tile (B * K elements per CTA) limits the CTAs per SM and
// the slices measured slower (B = 4: 14.7 -> 17.7 us): one warp per row,
// several passes.
template <typename T, int B>
cudaError_t launch_gemv_t(const void* x, const void* W, const void* bias, void* y, int N, int K, bool x_f16,
                          cudaStream_t stream) {
  if (K <= 2048) return launch_gemv_k<T, B, 2, 1>(x, W, bias, y, N, K, x_f16, stream);
  if constexpr (B == 1) {
    if (K <= 4096) return launch_gemv_k<T, B, 1, 2>(x, W, bias, y, N, K, x_f16, stream);
    if (K <= 8192) return launch_gemv_k<T, B, 1, 4>(x, W, bias, y, N, K, x_f16, stream);
    return launch_gemv_k<T, B, 1, 8>(x, W, bias, y, N, K, x_f16, stream);
  }
  return launch_gemv_k<T, B, 1, 1>(x, W, bias, y, N, K, x_f16, stream);
}

template <typename T>
cudaError_t launch_gemv_b(const void* x, const void* W, const void* bias, void* y, int B, int N, int K, bool x_f16,
                          cudaStream_t stream) {
  switch (B) {
    case 1: return launch_gemv_t<T, 1>(x, W, bias, y, N, K, x_f16, stream);
    case 2: return launch_gemv_t<T, 2>(x, W, bias, y, N, K, x_f16, stream);
    case 3: return launch_gemv_t<T, 3>(x, W, bias, y, N, K, x_f16, stream);
    default: return launch_gemv_t<T, 4>(x, W, bias, y, N, K, x_f16, stream);
  }
}

template <typename T>
cudaError_t launch_gemv_swiglu_b(const void* x, const void* W, const void* bias, void* y, int B, int I, int K,
                                 cudaStream_t stream) {
  switch (B) {
    case 1: return launch_gemv_k<T, 1, 2, 1, kEpiSwiGLU>(x, W, bias, y, I, K, false, stream);
    case 2: return launch_gemv_k<T, 2, 2, 1, kEpiSwiGLU>(x, W, bias, y, I, K, false, stream);
    case 3: return launch_gemv_k<T, 3, 2, 1, kEpiSwiGLU>(x, W, bias, y, I, K, false, stream);
    default: return launch_gemv_k<T, 4, 2, 1, kEpiSwiGLU>(x, W, bias, y, I, K, false, stream);
  }
}

// Row-wise argmax of logits [rows, V] (model dtype) -> idx [rows] int64, as
// torch.argmax (first index of the maximum; NaN counts as the maximum).  A
// single-output torch reduction over a 128K vocabulary runs on one CTA; here
// `nblk` CTAs share a row (64 for one row, fewer as rows grow so the grid
// stays near 8 CTAs per SM), each writes its (value, index) partial, and the
// last CTA to arrive (counter per row, reset by that CTA, so the scratch stays
// reusable across calls and CUDA-graph replays) reduces the partials.
constexpr int kArgThreads = 256;
constexpr int kArgBlocks = 64;  // partial slots per row in the scratch

__device__ __forceinline__ bool arg_better(float v, int i, float bv, int bi) {
  // NaN is the largest value (torch.argmax); ties keep the lower index
  if (isnan(v)) return !isnan(bv) || i < bi;
  if (isnan(bv)) return false;
  return v > bv || (v == bv && i < bi);
}

template <typename T>
__global__ void __launch_bounds__(kArgThreads) argmax_kernel(const T* __restrict__ logits, int V, int per, bool vec,
                                                             float* __restrict__ part_v, int* __restrict__ part_i,
                                                             unsigned* __restrict__ counters,
                                                             int64_t* __restrict__ out) {
  pdl_wait_primary();
  pdl_launch_dependents();
  const int row = blockIdx.y, blk = blockIdx.x, nblk = gridDim.x;
  const T* lr = logits + int64_t(row) * V;
  const int lo = blk * per, hi = min(V, lo + per);
  float bv = -INFINITY;
  int bi = INT32_MAX;
  if (vec) {
    // `per` and the row start are multiples of 8 elements: 16-byte chunks,
    // then the row's ragged end element by element
    const int hi8 = lo + ((hi - lo) & ~7);
    for (int i = lo + 8 * threadIdx.x; i < hi8; i += 8 * kArgThreads) {
      const uint4 c = *reinterpret_cast<const uint4*>(lr + i);
      const T* cp = reinterpret_cast<const T*>(&c);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float v = ld<T>(cp, e);
        if (arg_better(v, i + e, bv, bi)) { bv = v; bi = i + e; }
      }
    }
    for (int i = hi8 + threadIdx.x; i < hi; i += kArgThreads) {
      const float v = ld<T>(lr, i);
      if (arg_better(v, i, bv, bi)) { bv = v; bi = i; }
    }
  } else {
    for (int i = lo + threadIdx.x; i < hi; i += kArgThreads) {
      const float v = ld<T>(lr, i);
      if (arg_better(v, i, bv, bi)) { bv = v; bi = i; }
    }
  }
  __shared__ float sv[kArgThreads / 32];
  __shared__ int si[kArgThreads / 32];
  __shared__ bool last;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
    if (arg_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
  }
  if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kArgThreads / 32; ++w)
      if (arg_better(sv[w], si[w], bv, bi)) { bv = sv[w]; bi = si[w]; }
    part_v[row * kArgBlocks + blk] = bv;
    part_i[row * kArgBlocks + blk] = bi;
    __threadfence();
    last = atomicAdd(&counters[row], 1u) == unsigned(nblk - 1);
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (threadIdx.x < 32) {
    float v = -INFINITY;
    int i = INT32_MAX;
    for (int b = threadIdx.x; b < nblk; b += 32) {
      const float pv = *reinterpret_cast<volatile float*>(&part_v[row * kArgBlocks + b]);
      const int pi = *reinterpret_cast<volatile int*>(&part_i[row * kArgBlocks + b]);
      if (arg_better(pv, pi, v, i)) { v = pv; i = pi; }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, off);
      const int oi = __shfl_xor_sync(0xffffffffu, i, off);
      if (arg_better(ov, oi, v, i)) { v = ov; i = oi; }
    }
    if (threadIdx.x == 0) {
      out[row] = int64_t(i);
      counters[row] = 0u;  // ready for the next call
    }
  }
}

}  // namespace

size_t argmax_scratch_bytes(int64_t rows) {
  return size_t(rows) * kArgBlocks * (sizeof(float) + sizeof(int)) + size_t(rows) * sizeof(unsigned);
}

cudaError_t launch_argmax(bool bf16, const void* logits, int64_t rows, int V, void* scratch, int64_t* out,
                          cudaStream_t stream) {
  float* pv = static_cast<float*>(scratch);
  int* pi = reinterpret_cast<int*>(pv + rows * kArgBlocks);
  unsigned* cnt = reinterpret_cast<unsigned*>(pi + rows * kArgBlocks);
  const int nblk = int(std::max<int64_t>(1, std::min<int64_t>(kArgBlocks, (148 * 8) / rows)));
  const bool vec = V % 8 == 0 && reinterpret_cast<uintptr_t>(logits) % 16 == 0;
  int per = (V + nblk - 1) / nblk;
  if (vec) per = (per + 7) & ~7;
  const dim3 grid{unsigned(nblk), unsigned(rows), 1u};
  if (bf16)
    return launch_pdl(argmax_kernel<__nv_bfloat16>, grid, dim3(kArgThreads), 0, stream,
                      static_cast<const __nv_bfloat16*>(logits), V, per, vec, pv, pi, cnt, out);
  return launch_pdl(argmax_kernel<__half>, grid, dim3(kArgThreads), 0, stream, static_cast<const __half*>(logits), V,
                    per, vec, pv, pi, cnt, out);
}

cudaError_t launch_gemv(bool bf16, bool x_f16, const void* x, const void* W, const void* bias, void* y, int B, int N,
                        int K, cudaStream_t stream) {
  return bf16 ? launch_gemv_b<__nv_bfloat16>(x, W, bias, y, B, N, K, x_f16, stream)
              : launch_gemv_b<__half>(x, W, bias, y, B, N, K, true, stream);
}

cudaError_t launch_gemv_swiglu(bool bf16, const void* x, const void* W, const void* bias, void* y, int B, int I, int K,
                               cudaStream_t stream) {
  return bf16 ? launch_gemv_swiglu_b<__nv_bfloat16>(x, W, bias, y, B, I, K, stream)
              : launch_gemv_swiglu_b<__half>(x, W, bias, y, B, I, K, stream);
}

cudaError_t launch_gemv_rope_append(bool bf16, const void* x, const void* W, const void* bias, int K,
                                    const GemvRope& rp, cudaStream_t stream) {
  const int N = (rp.Hq + 2 * rp.Hkv) * rp.D;
  return bf16 ? launch_gemv_k<__nv_bfloat16, 1, 2, 1, kEpiRope>(x, W, bias, nullptr, N, K, false, stream, rp)
              : launch_gemv_k<__half, 1, 2, 1, kEpiRope>(x, W, bias, nullptr, N, K, false, stream, rp);
}

cudaError_t launch_add_rmsnorm(bool bf16, void* h, const void* delta, const void* w, void* y, int64_t rows, int H,
                               float eps, cudaStream_t stream) {
  if (H > kNormThreads * kMaxPerThread) return cudaErrorInvalidValue;
  const auto al16 = [](const void* p) { return p == nullptr || reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  if (H % 8 == 0 && al16(h) && al16(delta) && al16(w) && al16(y)) {
    if (bf16)
      return launch_pdl(add_rmsnorm_vec_kernel<__nv_bfloat16>, dim3(unsigned(rows)), dim3(kNormThreads), 0, stream,
                        static_cast<__nv_bfloat16*>(h), static_cast<const __nv_bfloat16*>(delta),
                        static_cast<const __nv_bfloat16*>(w), static_cast<__nv_bfloat16*>(y), H, eps);
    return launch_pdl(add_rmsnorm_vec_kernel<__half>, dim3(unsigned(rows)), dim3(kNormThreads), 0, stream,
                      static_cast<__half*>(h), static_cast<const __half*>(delta), static_cast<const __half*>(w),
                      static_cast<__half*>(y), H, eps);
  }
  if (bf16)
    return launch_pdl(add_rmsnorm_kernel<__nv_bfloat16>, dim3(unsigned(rows)), dim3(kNormThreads), 0, stream,
                      static_cast<__nv_bfloat16*>(h), static_cast<const __nv_bfloat16*>(delta),
                      static_cast<const __nv_bfloat16*>(w), static_cast<__nv_bfloat16*>(y), H, eps);
  return launch_pdl(add_rmsnorm_kernel<__half>, dim3(unsigned(rows)), dim3(kNormThreads), 0, stream,
                    static_cast<__half*>(h), static_cast<const __half*>(delta), static_cast<const __half*>(w),
                    static_cast<__half*>(y), H, eps);
}

cudaError_t launch_silu_mul(bool bf16, const void* gu, void* y, int64_t rows, int I, int64_t row_stride,
                            cudaStream_t stream) {
  const auto al16 = [](const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  if (I % 8 == 0 && row_stride % 8 == 0 && al16(gu) && al16(y)) {
    const int64_t n8 = rows * (I / 8);
    const unsigned vblocks = unsigned(std::min<int64_t>((n8 + 255) / 256, 148 * 16));
    if (bf16)
      return launch_pdl(silu_mul_vec_kernel<__nv_bfloat16>, dim3(vblocks), dim3(256), 0, stream,
                        static_cast<const __nv_bfloat16*>(gu), static_cast<__nv_bfloat16*>(y), rows, I / 8,
                        row_stride / 8);
    return launch_pdl(silu_mul_vec_kernel<__half>, dim3(vblocks), dim3(256), 0, stream,
                      static_cast<const __half*>(gu), static_cast<__half*>(y), rows, I / 8, row_stride / 8);
  }
  const int64_t n = rows * I;
  const unsigned blocks = unsigned(std::min<int64_t>((n + 255) / 256, 148 * 16));
  if (bf16)
    return launch_pdl(silu_mul_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, stream,
                      static_cast<const __nv_bfloat16*>(gu), static_cast<__nv_bfloat16*>(y), rows, I, row_stride);
  return launch_pdl(silu_mul_kernel<__half>, dim3(blocks), dim3(256), 0, stream, static_cast<const __half*>(gu),
                    static_cast<__half*>(y), rows, I, row_stride);
}

}  // namespace fqkv
