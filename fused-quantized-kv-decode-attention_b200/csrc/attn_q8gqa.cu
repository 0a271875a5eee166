// int8-KV GQA decode attention (the int8 KV cache of a GQA model), sm_100a.
//
// The reference has int8 KV only for one query head per KV row
// (decode_attn_int8_mw, kernels/decode_attn_int8_mw.cu:6-51) and GQA only for
// fp16 (decode_attn_gqa, kernels/decode_attn_gqa.cu:8-55); a GQA model with an
// int8 cache needs both.  Layout: codes [B, Hkv, stride, D] int8, per-token
// scales [B, Hkv, stride] fp16 (the reference quantizer's output, e.g. written
// by fqkv_quantize_int8_into_cache), q/out [B, Hq, D] fp16.
//
//  * Persistent, warp-specialised: a unit is (sequence, KV head, group of <= 8
//    query heads, split).  Warp 4 streams 64-key tiles of K and V codes with
//    3-D TMA tensor copies (128-byte swizzle for D = 128, 64-byte for D = 64,
//    keys past the end zero-filled) plus 16-byte-aligned windows of their
//    fp16 scales into a ring of stages; each consumer warp takes 16 keys of a
//    tile and reads every KV byte once for all heads of the group.
//  * S = Q K^T on the integer tensor cores (mma m16n8k32 s8 x s8 -> s32)
//    straight from the codes: q is held as a 2-plane fixed-point number per
//    head (q * Qs = hi * 256 + lo, |q * Qs| <= 32639, Qs = 32639 / max|q|);
//    rows 0-7 of the A operand carry the hi planes of the group's heads and
//    rows 8-15 the lo planes, so one MMA yields both partial sums of a score.
//    The head dimension is permuted (identically for q and K) so that each
//    thread reads one contiguous D/4-byte span of a key row.
//  * O^T += V^T (P * Vscale)^T on the fp16 tensor cores (m16n8k16): the A
//    operand pairs one dimension of two consecutive keys, built in registers
//    from the codes (byte permute, one three-input logic op giving the fp16
//    value 1152 + code, one exact fp16 subtraction); the B operand is the fp16
//    probabilities times the key's V scale, taken directly from the score
//    accumulators.  Rows of O^T are head dimensions, columns the group's
//    heads.  The softmax denominator sums the unscaled probabilities.
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
constexpr int kQMax = 32639;  // |q * Qs| bound: hi = (v + 128) >> 8 stays in [-127, 127]

template <int D>
struct Q8Cfg {
  static constexpr int kTileBytes = kTK * D;            // K (or V) codes of one tile
  static constexpr int kScaleBytes = 2 * kTK + 32;      // 16B-aligned scale window
  static constexpr int kStageRaw = 2 * kTileBytes + 2 * kScaleBytes;
  static constexpr int kStageBytes = (kStageRaw + 1023) & ~1023;  // tiles stay 1024-aligned (swizzle atom)
  static constexpr int kStages = D == 128 ? 3 : 4;
  static constexpr size_t kRingBytes = size_t(kStages) * kStageBytes;
  static constexpr size_t kBarBytes = 2 * kStages * sizeof(uint64_t);
  static constexpr size_t kMergeBytes = size_t(kConsumerWarps) * (2 * 8 + kMergeHeads * D) * sizeof(float);
  static constexpr size_t kSmemBytes = 1024 + kRingBytes + kBarBytes + kMergeBytes;
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

// Byte offset of 16-byte chunk `c` of key row `row` inside a tile written by
// the TMA copy (128-byte swizzle for 128-byte rows, 64-byte swizzle for
// 64-byte rows; the tile starts 1024-aligned).
template <int D>
__device__ __forceinline__ uint32_t tile_off(int row, int c) {
  if constexpr (D == 128) return uint32_t(row * 128 + ((c ^ (row & 7)) << 4));
  else return uint32_t(row * 64 + ((c ^ ((row >> 1) & 3)) << 4));
}

// D(16x8, s32) += A(16x32, s8, row) * B(32x8, s8, col).
__device__ __forceinline__ void mma_s8_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
      "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Exact fp16x2 {code of x's byte, code of y's byte} for the byte chosen by
// `sel` ({x.b, x.b, y.b, y.b}): the logic op forms 0x64 | (code ^ 0x80) in each
// half (the fp16 value 1152 + code), the subtraction removes 1152.
__device__ __forceinline__ uint32_t code_pair(uint32_t x, uint32_t y, uint32_t sel) {
  const uint32_t p = __byte_perm(x, y, sel);
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0x9c;" : "=r"(r) : "r"(p), "r"(0x64806480u), "r"(0xFF00FF00u));
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(r), "r"(0x64806480u));
  return r;
}

__device__ __forceinline__ uint32_t pack_s8x4(int a, int b, int c, int d) {
  return (uint32_t(a) & 0xFFu) | ((uint32_t(b) & 0xFFu) << 8) | ((uint32_t(c) & 0xFFu) << 16) |
         (uint32_t(d) << 24);
}

template <int D>
__global__ void __launch_bounds__(kThreads, 3) decode_q8gqa_kernel(const __grid_constant__ DecodeLaunch a) {
  using C = Q8Cfg<D>;
  constexpr int KS = D / 32;        // integer MMA k-steps over the head dimension
  constexpr int MT = D / 16;        // m-tiles of O^T (16 head dimensions each)
  constexpr int TW = D / 32;        // 32-bit words of this thread's V slice of one key
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
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

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kConsumerWarps && lane == 0) {
    prefetch_tensormap(&a.tmK);
    prefetch_tensormap(&a.tmV);
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
      const int z = uc.b * a.Hkv + uc.kh;
      const __half* Ksr = static_cast<const __half*>(a.Ks) + size_t(z) * a.kv_stride;
      const __half* Vsr = static_cast<const __half*>(a.Vs) + size_t(z) * a.kv_stride;
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
        const uintptr_t ka = reinterpret_cast<uintptr_t>(Ksr + k0);
        const uintptr_t va = reinterpret_cast<uintptr_t>(Vsr + k0);
        const uintptr_t ka0 = ka & ~uintptr_t(15), va0 = va & ~uintptr_t(15);
        const uint32_t kwin = uint32_t(((ka + 2u * nk + 15u) & ~uintptr_t(15)) - ka0);
        const uint32_t vwin = uint32_t(((va + 2u * nk + 15u) & ~uintptr_t(15)) - va0);
        stage_off[st][0] = int(ka - ka0) >> 1;
        stage_off[st][1] = int(va - va0) >> 1;
        uint8_t* base = ring + size_t(st) * C::kStageBytes;
        mbar_arrive_expect_tx(&full[st], 2 * C::kTileBytes + kwin + vwin);
        tma_load_3d(base, &a.tmK, 0, k0, z, &full[st]);
        tma_load_3d(base + C::kTileBytes, &a.tmV, 0, k0, z, &full[st]);
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
  const int r0 = warp * 16;
  const float csc = a.sm_scale_log2;
  bool alive = true;
  int it = 0;

  for (int u = blockIdx.x; u < a.units; u += gridDim.x) {
    const UnitCoord uc = decode_unit(a, u);
    const int lo = uc.s * a.chunk;
    const int hi = min(n_valid, lo + a.chunk);
    const int h0 = uc.kh * a.G + uc.grp * a.GP;
    const int gvalid = min(a.GP, a.G - uc.grp * a.GP);

    // ---- q of head g, dimensions [t*D/4, (t+1)*D/4), as two int8 planes
    uint32_t qa[KS][4];
    float hf;  // sm_scale_log2 / Qs of head g
    {
      float qf[D / 4];
      if (g < gvalid) {
        const uint32_t* qrow = reinterpret_cast<const uint32_t*>(
            static_cast<const __half*>(a.q) + (size_t(uc.b) * a.Hq + h0 + g) * D + t * (D / 4));
#pragma unroll
        for (int v = 0; v < D / 8; ++v) {
          const uint32_t w = qrow[v];
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w));
          qf[2 * v] = f.x;
          qf[2 * v + 1] = f.y;
        }
      } else {
#pragma unroll
        for (int i = 0; i < D / 4; ++i) qf[i] = 0.f;
      }
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < D / 4; ++i) amax = fmaxf(amax, fabsf(qf[i]));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      const float Qs = amax > 0.f ? float(kQMax) / amax : 0.f;
      hf = amax > 0.f ? csc * (amax / float(kQMax)) : 0.f;
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        int hv[8], lv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int v = __float2int_rn(qf[8 * kk + i] * Qs);
          hv[i] = (v + 128) >> 8;
          lv[i] = v - hv[i] * 256;
        }
        qa[kk][0] = pack_s8x4(hv[0], hv[1], hv[2], hv[3]);
        qa[kk][1] = pack_s8x4(lv[0], lv[1], lv[2], lv[3]);
        qa[kk][2] = pack_s8x4(hv[4], hv[5], hv[6], hv[7]);
        qa[kk][3] = pack_s8x4(lv[4], lv[5], lv[6], lv[7]);
      }
    }

    float o[MT][4];
#pragma unroll
    for (int i = 0; i < MT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
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
      const uint8_t* kt = ring + size_t(st) * C::kStageBytes;
      const uint8_t* vt = kt + C::kTileBytes;

      // ---- fragments of this warp's 16 keys (rows r0 .. r0 + 15 of the tile)
      uint32_t kb[2][2 * KS];  // key r0 + 8j + g: this thread's D/4 bytes
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int row = r0 + 8 * j + g;
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          const uint4 w = *reinterpret_cast<const uint4*>(kt + tile_off<D>(row, (D / 64) * t + c));
          kb[j][4 * c + 0] = w.x;
          kb[j][4 * c + 1] = w.y;
          kb[j][4 * c + 2] = w.z;
          kb[j][4 * c + 3] = w.w;
        }
      }
      uint32_t vw[4][TW];  // keys r0 + {2t, 2t+1, 2t+8, 2t+9}, dimensions [g*D/8, (g+1)*D/8)
#pragma unroll
      for (int kq = 0; kq < 4; ++kq) {
        const int row = r0 + 2 * t + (kq & 1) + 8 * (kq >> 1);
        if constexpr (D == 128) {
          const uint4 w = *reinterpret_cast<const uint4*>(vt + tile_off<D>(row, g));
          vw[kq][0] = w.x;
          vw[kq][1] = w.y;
          vw[kq][2] = w.z;
          vw[kq][3] = w.w;
        } else {
          const uint2 w = *reinterpret_cast<const uint2*>(vt + tile_off<D>(row, g >> 1) + 8 * (g & 1));
          vw[kq][0] = w.x;
          vw[kq][1] = w.y;
        }
      }
      const __half* kst = reinterpret_cast<const __half*>(kt + 2 * C::kTileBytes) + stage_off[st][0];
      const __half* vst = reinterpret_cast<const __half*>(kt + 2 * C::kTileBytes + C::kScaleBytes) +
                          stage_off[st][1];
      float ks[2][2], vs[2][2];
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          ks[j][e] = __half2float(kst[r0 + 8 * j + 2 * t + e]);
          vs[j][e] = __half2float(vst[r0 + 8 * j + 2 * t + e]);
        }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);  // everything this warp needs is in registers

      // ---- S = Q K^T in integers: hi plane of head g in c0/c1, lo plane in c2/c3
      int acc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
#pragma unroll
        for (int j = 0; j < 2; ++j)
          mma_s8_16832(acc[j], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], kb[j][2 * kk], kb[j][2 * kk + 1]);
      }

      float sc[2][2];
      float mx = -INFINITY;
      bool valid[2][2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          valid[j][e] = (k0 + r0 + 8 * j + 2 * t + e) < hi;
          const float s = float(acc[j][e] * 256 + acc[j][2 + e]) * (ks[j][e] * hf);
          sc[j][e] = valid[j][e] ? s : -INFINITY;
          mx = fmaxf(mx, sc[j][e]);
        }
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_run, mx);
      if (__any_sync(0xffffffffu, m_new > m_run)) {
        const float alpha = (m_new == -INFINITY) ? 1.f : ex2(m_run - m_new);
        l_run *= alpha;
        m_run = m_new;
        // O^T columns are heads 2t, 2t+1; their factors live with g = 2t, 2t+1
        const float a_lo = __shfl_sync(0xffffffffu, alpha, (2 * t) * 4);
        const float a_hi = __shfl_sync(0xffffffffu, alpha, (2 * t + 1) * 4);
#pragma unroll
        for (int i = 0; i < MT; ++i) {
          o[i][0] *= a_lo;
          o[i][1] *= a_hi;
          o[i][2] *= a_lo;
          o[i][3] *= a_hi;
        }
      }
      const float mu = (m_run == -INFINITY) ? 0.f : m_run;
      float p[2][2];
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) p[j][e] = valid[j][e] ? ex2(sc[j][e] - mu) : 0.f;
      l_run += (p[0][0] + p[0][1]) + (p[1][0] + p[1][1]);
      const uint32_t pb0 = pack_half2(valid[0][0] ? p[0][0] * vs[0][0] : 0.f, valid[0][1] ? p[0][1] * vs[0][1] : 0.f);
      const uint32_t pb1 = pack_half2(valid[1][0] ? p[1][0] * vs[1][0] : 0.f, valid[1][1] ? p[1][1] * vs[1][1] : 0.f);

      // ---- O^T += V^T P^T; m-tile i rows g / g+8 are dimensions g*D/8 + i / g*D/8 + D/16 + i
#pragma unroll
      for (int i = 0; i < MT; ++i) {
        const int w0 = i >> 2, w1 = (MT + i) >> 2;              // words holding bytes i and D/16 + i
        const uint32_t sel = uint32_t(i & 3) * 0x1111u + 0x4400u;  // {x.b, x.b, y.b, y.b}
        const uint32_t a0 = code_pair(vw[0][w0], vw[1][w0], sel);
        const uint32_t a1 = code_pair(vw[0][w1], vw[1][w1], sel);
        const uint32_t a2 = code_pair(vw[2][w0], vw[3][w0], sel);
        const uint32_t a3 = code_pair(vw[2][w1], vw[3][w1], sel);
        mma_16816(o[i], a0, a1, a2, a3, pb0, pb1);
      }
    }

    // ---- unit epilogue: merge the 4 warps' (m, l, O) per head
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
    if (t == 0) {
      sm_m[warp * 8 + g] = m_run;
      sm_l[warp * 8 + g] = l_run;
    }
    const int ct = threadIdx.x;
    const size_t row_base = size_t(uc.b) * a.Hq + h0;
    for (int hp = 0; hp < gvalid; hp += kMergeHeads) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int head = 2 * t + e;
        const int gl = head - hp;
        if (gl >= 0 && gl < kMergeHeads && head < gvalid) {
          float* dst = &sm_o[(warp * kMergeHeads + gl) * D + g * (D / 8)];
#pragma unroll
          for (int i = 0; i < MT; i += 4) {
            *reinterpret_cast<float4*>(dst + i) = make_float4(o[i][e], o[i + 1][e], o[i + 2][e], o[i + 3][e]);
            *reinterpret_cast<float4*>(dst + MT + i) =
                make_float4(o[i][2 + e], o[i + 1][2 + e], o[i + 2][2 + e], o[i + 3][2 + e]);
          }
        }
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
