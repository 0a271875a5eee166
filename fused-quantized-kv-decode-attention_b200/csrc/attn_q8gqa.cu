// int8-KV GQA decode attention (the int8 KV cache of a GQA model), sm_100a.
//
// The reference has int8 KV only for one query head per KV row
// (decode_attn_int8_mw, kernels/decode_attn_int8_mw.cu:6-51) and GQA only for
// fp16 (decode_attn_gqa, kernels/decode_attn_gqa.cu:8-55); a GQA model with an
// int8 cache needs both.  Layout: codes [B, Hkv, stride, D] int8, per-token
// scales [B, Hkv, stride] fp16 (the reference quantizer's output, e.g. written
// by fqkv_quantize_int8_into_cache), q/out [B, Hq, D] fp16.
//
//  * Same persistent, warp-specialised structure as the fp16 kernel: a unit is
//    (sequence, KV head, group of <= 8 query heads, split), warp 4 streams
//    64-key tiles of K and V codes plus their scale windows into a 4-stage ring
//    with 1-D bulk copies.
//  * Each consumer warp first turns its 16 keys of K and V codes into exact
//    fp16 integers in a private 128B-swizzled buffer (byte-permute into the
//    mantissa of 1024 + exact fp16 subtraction) and releases the stage, then
//    runs the tensor-core math of the fp16 kernel on that buffer: S = Q K^T
//    (ldmatrix + mma.sync f16 -> f32) scaled per key by its K scale, and
//    O += (P * V scale) V (ldmatrix.trans).  The softmax denominator sums the
//    unscaled P.  The KV bytes are read from HBM once for all heads of the
//    group.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "device_common.cuh"
#include "kernels.h"

namespace fqkv {
namespace {

constexpr int kConsumerWarps = 4;
constexpr int kThreads = 32 * (kConsumerWarps + 1);
constexpr int kTK = 64;
constexpr int kMergeHeads = 4;

template <int D>
struct Q8Cfg {
  static constexpr int kTileBytes = kTK * D;            // K (or V) codes of one tile
  static constexpr int kScaleBytes = 2 * kTK + 32;      // 16B-aligned scale window
  static constexpr int kStageBytes = 2 * kTileBytes + 2 * kScaleBytes;
  static constexpr int kStages = 4;
  static constexpr int kWarpBuf = 16 * D * 2;           // 16 keys x D fp16 (K or V)
  static constexpr size_t kRingBytes = size_t(kStages) * kStageBytes;
  static constexpr size_t kBufBytes = size_t(kConsumerWarps) * 2 * kWarpBuf;
  static constexpr size_t kBarBytes = 2 * kStages * sizeof(uint64_t);
  static constexpr size_t kMergeBytes = size_t(kConsumerWarps) * (2 * 8 + kMergeHeads * D) * sizeof(float);
  static constexpr size_t kSmemBytes = 1024 + kBufBytes + kRingBytes + kBarBytes + kMergeBytes;
};

struct UnitCoord {
  int b, kh, grp, s;
};

__device__ __forceinline__ UnitCoord decode_unit(const DecodeLaunch& a, int u) {
  UnitCoord c;
  c.grp = u % a.groups;
  u /= a.groups;
  c.s = u % a.S_eff;
  u /= a.S_eff;
  c.kh = u % a.Hkv;
  c.b = u / a.Hkv;
  return c;
}

// 16-byte chunk `chunk` (0 .. D/8-1) of row `row` (0..15) of a warp buffer made
// of D/64 blocks of [16 rows x 128 B], 128B-swizzled within each block.
__device__ __forceinline__ uint32_t swz16(int row, int chunk) {
  return uint32_t((chunk >> 3) * 2048 + row * 128 + (((chunk & 7) ^ (row & 7)) << 4));
}

__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// 16 int8 codes (one uint4) -> 16 exact fp16 values (two uint4, element order kept).
__device__ __forceinline__ void codes16_to_half(const uint4 w, uint4& lo, uint4& hi) {
  const uint32_t in[4] = {w.x, w.y, w.z, w.w};
  uint32_t out[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t x = in[i] ^ 0x80808080u;  // code + 128
    out[2 * i] = hsub2_u32(__byte_perm(x, 0x64646464u, 0x5140u), 0x64806480u);
    out[2 * i + 1] = hsub2_u32(__byte_perm(x, 0x64646464u, 0x7362u), 0x64806480u);
  }
  lo = make_uint4(out[0], out[1], out[2], out[3]);
  hi = make_uint4(out[4], out[5], out[6], out[7]);
}

template <int D>
__global__ void __launch_bounds__(kThreads, 2) decode_q8gqa_kernel(const __grid_constant__ DecodeLaunch a) {
  using C = Q8Cfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* bufs = smem;                                   // [warp][K|V][16 x D fp16], 1 KiB aligned
  uint8_t* ring = smem + C::kBufBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + C::kRingBytes);
  uint64_t* empty = full + C::kStages;
  float* sm_m = reinterpret_cast<float*>(empty + C::kStages);
  float* sm_l = sm_m + kConsumerWarps * 8;
  float* sm_o = sm_l + kConsumerWarps * 8;
  __shared__ int abort_flag;
  __shared__ int stage_off[C::kStages][2];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const WaitCtl wc{a.status, a.timeout_ns};
  const size_t row_stride = size_t(a.kv_stride) * D;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  pdl_launch_dependents();
  const int n_valid = a.n_dev ? min(a.N, *a.n_dev) : a.N;

  // ------------------------------------------------------------ producer
  if (warp == kConsumerWarps) {
    if (lane != 0 || a.debug_skip_loads) return;
    int it = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < a.units && ok; u += gridDim.x) {
      const UnitCoord uc = decode_unit(a, u);
      const int lo = uc.s * a.chunk;
      const int hi = min(n_valid, lo + a.chunk);
      const size_t r = size_t(uc.b) * a.Hkv + uc.kh;
      const uint8_t* Kr = static_cast<const uint8_t*>(a.K) + r * row_stride;
      const uint8_t* Vr = static_cast<const uint8_t*>(a.V) + r * row_stride;
      const __half* Ksr = static_cast<const __half*>(a.Ks) + r * a.kv_stride;
      const __half* Vsr = static_cast<const __half*>(a.Vs) + r * a.kv_stride;
      for (int k0 = lo; k0 < hi; k0 += kTK, ++it) {
        const int st = it % C::kStages;
        if (it >= C::kStages) {
          if (*reinterpret_cast<volatile int*>(&abort_flag) ||
              !mbar_wait(&empty[st], ((it / C::kStages) - 1) & 1, wc, kDevTimeoutEmpty)) {
            ok = false;
            break;
          }
        }
        const int nk = min(kTK, hi - k0);
        const uint32_t kv_bytes = uint32_t(nk) * D;
        const uintptr_t ka = reinterpret_cast<uintptr_t>(Ksr + k0);
        const uintptr_t va = reinterpret_cast<uintptr_t>(Vsr + k0);
        const uintptr_t ka0 = ka & ~uintptr_t(15), va0 = va & ~uintptr_t(15);
        const uint32_t kwin = uint32_t(((ka + 2u * nk + 15u) & ~uintptr_t(15)) - ka0);
        const uint32_t vwin = uint32_t(((va + 2u * nk + 15u) & ~uintptr_t(15)) - va0);
        stage_off[st][0] = int(ka - ka0) >> 1;
        stage_off[st][1] = int(va - va0) >> 1;
        uint8_t* base = ring + size_t(st) * C::kStageBytes;
        mbar_arrive_expect_tx(&full[st], 2 * kv_bytes + kwin + vwin);
        bulk_g2s(base, Kr + size_t(k0) * D, kv_bytes, &full[st]);
        bulk_g2s(base + C::kTileBytes, Vr + size_t(k0) * D, kv_bytes, &full[st]);
        bulk_g2s(base + 2 * C::kTileBytes, reinterpret_cast<const void*>(ka0), kwin, &full[st]);
        bulk_g2s(base + 2 * C::kTileBytes + C::kScaleBytes, reinterpret_cast<const void*>(va0), vwin, &full[st]);
      }
    }
    if (!ok) {
      for (int j = (it > C::kStages ? it - C::kStages : 0); j < it; ++j)
        mbar_wait(&full[j % C::kStages], (j / C::kStages) & 1, wc, kDevTimeoutDrain);
    }
    return;
  }

  // ------------------------------------------------------------ consumers
  const int g = lane >> 2;
  const int t = lane & 3;
  const int mi = lane >> 3;
  const int rr = lane & 7;
  const int r0 = warp * 16;
  uint8_t* kbuf = bufs + size_t(warp) * 2 * C::kWarpBuf;
  uint8_t* vbuf = kbuf + C::kWarpBuf;
  const uint32_t kbuf_u = smem_u32(kbuf), vbuf_u = smem_u32(vbuf);
  const float csc = a.sm_scale_log2;
  bool alive = true;
  int it = 0;

  for (int u = blockIdx.x; u < a.units; u += gridDim.x) {
    const UnitCoord uc = decode_unit(a, u);
    const int lo = uc.s * a.chunk;
    const int hi = min(n_valid, lo + a.chunk);
    const int h0 = uc.kh * a.G + uc.grp * a.GP;
    const int gvalid = min(a.GP, a.G - uc.grp * a.GP);

    uint32_t qa[D / 16][2];
    {
      const __half* qrow = static_cast<const __half*>(a.q) + (size_t(uc.b) * a.Hq + h0 + g) * D;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        if (g < gvalid) {
          qa[kk][0] = *reinterpret_cast<const uint32_t*>(qrow + 16 * kk + 2 * t);
          qa[kk][1] = *reinterpret_cast<const uint32_t*>(qrow + 16 * kk + 2 * t + 8);
        } else {
          qa[kk][0] = 0u;
          qa[kk][1] = 0u;
        }
      }
    }
    float o[D / 8][4];
#pragma unroll
    for (int j = 0; j < D / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m_run = -INFINITY, l_run = 0.f;

    for (int k0 = lo; k0 < hi; k0 += kTK, ++it) {
      const int st = it % C::kStages;
      if (alive) {
        const bool ok = mbar_wait(&full[st], (it / C::kStages) & 1, wc, kDevTimeoutFull) &&
                        !*reinterpret_cast<volatile int*>(&abort_flag);
        alive = __all_sync(0xffffffffu, ok);
        if (!alive && lane == 0) abort_flag = 1;
      }
      if (!alive) continue;
      const uint8_t* base = ring + size_t(st) * C::kStageBytes;

      // ---- this warp's 16 keys: codes -> exact fp16 in the private buffers
      {
        const uint8_t* kt = base + size_t(r0) * D;
        const uint8_t* vt = base + C::kTileBytes + size_t(r0) * D;
#pragma unroll 1
        for (int i = 0; i < D / 32; ++i) {     // 512-byte blocks of the warp's 16 x D codes
          const int off = 512 * i + 16 * lane;  // byte offset: row off / D, column off % D
          const int row = off / D, col = off % D;
          uint4 lo4, hi4;
          codes16_to_half(*reinterpret_cast<const uint4*>(kt + off), lo4, hi4);
          *reinterpret_cast<uint4*>(kbuf + swz16(row, col / 8)) = lo4;
          *reinterpret_cast<uint4*>(kbuf + swz16(row, col / 8 + 1)) = hi4;
          codes16_to_half(*reinterpret_cast<const uint4*>(vt + off), lo4, hi4);
          *reinterpret_cast<uint4*>(vbuf + swz16(row, col / 8)) = lo4;
          *reinterpret_cast<uint4*>(vbuf + swz16(row, col / 8 + 1)) = hi4;
        }
      }
      // per-key scales of the keys this thread's fragments cover
      const __half* kst = reinterpret_cast<const __half*>(base + 2 * C::kTileBytes) + stage_off[st][0];
      const __half* vst = reinterpret_cast<const __half*>(base + 2 * C::kTileBytes + C::kScaleBytes) + stage_off[st][1];
      float ks[2][2], vs[2][2];
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          ks[j][e] = __half2float(kst[r0 + 8 * j + 2 * t + e]);
          vs[j][e] = __half2float(vst[r0 + 8 * j + 2 * t + e]);
        }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);  // the stage is no longer read by this warp

      // ---- S = Q K^T
      float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const int row = ((mi >> 1) << 3) + rr;
        const int chunk = 2 * kk + (mi & 1);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(kbuf_u + swz16(row, chunk), b0, b1, b2, b3);
        mma_16816(sc[0], qa[kk][0], 0u, qa[kk][1], 0u, b0, b1);
        mma_16816(sc[1], qa[kk][0], 0u, qa[kk][1], 0u, b2, b3);
      }

      float mx = -INFINITY;
      bool valid[2][2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          valid[j][e] = (k0 + r0 + 8 * j + 2 * t + e) < hi;
          const float v = valid[j][e] ? sc[j][e] * ks[j][e] * csc : -INFINITY;
          sc[j][e] = v;
          mx = fmaxf(mx, v);
        }
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_run, mx);
      if (__any_sync(0xffffffffu, m_new > m_run)) {
        const float alpha = (m_new == -INFINITY) ? 1.f : ex2(m_run - m_new);
#pragma unroll
        for (int j = 0; j < D / 8; ++j) {
          o[j][0] *= alpha;
          o[j][1] *= alpha;
        }
        l_run *= alpha;
        m_run = m_new;
      }
      const float mu = (m_run == -INFINITY) ? 0.f : m_run;
      float p[2][2];
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) p[j][e] = ex2(sc[j][e] - mu);
      l_run += (p[0][0] + p[0][1]) + (p[1][0] + p[1][1]);
      const uint32_t pa0 = pack_half2(valid[0][0] ? p[0][0] * vs[0][0] : 0.f, valid[0][1] ? p[0][1] * vs[0][1] : 0.f);
      const uint32_t pa2 = pack_half2(valid[1][0] ? p[1][0] * vs[1][0] : 0.f, valid[1][1] ? p[1][1] * vs[1][1] : 0.f);

      // ---- O += (P * vscale) V
#pragma unroll
      for (int pp = 0; pp < D / 16; ++pp) {
        const int row = ((mi & 1) << 3) + rr;
        const int chunk = 2 * pp + (mi >> 1);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(vbuf_u + swz16(row, chunk), b0, b1, b2, b3);
        mma_16816(o[2 * pp], pa0, 0u, pa2, 0u, b0, b1);
        mma_16816(o[2 * pp + 1], pa0, 0u, pa2, 0u, b2, b3);
      }
      __syncwarp();  // the buffers are rewritten by the next tile
    }

    // ---- unit epilogue (as in the fp16 kernel)
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
    if (t == 0) {
      sm_m[warp * 8 + g] = m_run;
      sm_l[warp * 8 + g] = l_run;
    }
    const int ct = threadIdx.x;
    const size_t row_base = size_t(uc.b) * a.Hq + h0;
    for (int hp = 0; hp < gvalid; hp += kMergeHeads) {
      const int gl = g - hp;
      if (gl >= 0 && gl < kMergeHeads && g < gvalid) {
#pragma unroll
        for (int j = 0; j < D / 8; ++j)
          *reinterpret_cast<float2*>(&sm_o[(warp * kMergeHeads + gl) * D + 8 * j + 2 * t]) =
              make_float2(o[j][0], o[j][1]);
      }
      named_bar_sync(1, 32 * kConsumerWarps);
      const int nh = min(kMergeHeads, gvalid - hp);
      for (int idx = ct; idx < nh * D; idx += 32 * kConsumerWarps) {
        const int gl2 = idx / D, d = idx - gl2 * D;
        const int gg = hp + gl2;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, sm_m[w * 8 + gg]);
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) {
          const float mw = sm_m[w * 8 + gg];
          const float wt = (mw == -INFINITY) ? 0.f : ex2(mw - M);
          L += wt * sm_l[w * 8 + gg];
          O += wt * sm_o[(w * kMergeHeads + gl2) * D + d];
        }
        const size_t row = row_base + gg;
        if (a.S_eff == 1) {
          static_cast<__half*>(a.out)[row * D + d] = __float2half_rn(O / L);
        } else {
          const size_t slot = row * a.S + uc.s;
          if (d == 0) {
            a.part_m[slot] = M;
            a.part_l[slot] = L;
          }
          a.part_o[slot * D + d] = O;
        }
      }
      named_bar_sync(1, 32 * kConsumerWarps);
    }
  }
}

}  // namespace

cudaError_t decode_kernel_prepare_q8gqa(int D, int* ctas_per_sm) {
  const void* fn = D == 128 ? reinterpret_cast<const void*>(&decode_q8gqa_kernel<128>)
                            : reinterpret_cast<const void*>(&decode_q8gqa_kernel<64>);
  const size_t smem = D == 128 ? Q8Cfg<128>::kSmemBytes : Q8Cfg<64>::kSmemBytes;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(ctas_per_sm, fn, kThreads, smem);
}

cudaError_t launch_decode_q8gqa(const DecodeLaunch& a, cudaStream_t stream) {
  if (a.D == 128) decode_q8gqa_kernel<128><<<a.grid, kThreads, Q8Cfg<128>::kSmemBytes, stream>>>(a);
  else decode_q8gqa_kernel<64><<<a.grid, kThreads, Q8Cfg<64>::kSmemBytes, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace fqkv
