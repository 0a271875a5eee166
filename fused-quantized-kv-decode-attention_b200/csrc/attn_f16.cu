// fp16-KV single-query decode attention (plain and GQA), sm_100a.
//
// Replaces the reference kernels decode_attn_fp16_mw_kernel
// (kernels/decode_attn_fp16_mw.cu:6-49), decode_attn_gqa_kernel
// (kernels/decode_attn_gqa.cu:8-55) and gqa_sk_partial_pa2
// (kernels/decode_attn_gqa_sk_fast.cu:6-54) with one persistent kernel:
//
//  * A work unit is (sequence b, KV head kh, group of <= 8 query heads that
//    share kh, split s).  Every K/V byte of the unit is read from HBM once and
//    used by all heads of the group (the reference re-reads KV once per query
//    head and relies on L2).
//  * Warp 4 is the producer: one lane streams 64-key tiles of K and V into a
//    STAGES-deep shared-memory ring with 3-D TMA tensor copies (128-byte
//    swizzle, rows past N zero-filled by the TMA unit), completing on
//    mbarriers.  It runs ahead across unit boundaries.
//  * Warps 0-3 are consumers; each owns 16 keys of every tile.  Scores and
//    P.V run on the tensor cores with mma.sync m16n8k16 (f16 in, f32
//    accumulate): rows = query heads of the group (<= 8 valid), columns =
//    keys for Q.K^T, and the probabilities are re-used from registers as the
//    A operand of P.V (V fragments via ldmatrix.trans).  Tensor cores here
//    remove the fp16->fp32 conversions and FMAs from the issue slots; the
//    kernel stays HBM-bound.
//  * Online softmax in the log2 domain (scores pre-multiplied by
//    log2(e)/sqrt(D)), rescale only when a row maximum grows.
//  * Unit epilogue: the 4 warps' (m, l, o) are merged through shared memory
//    and written either as the fp16 output (one split) or as an fp32 partial
//    (m in log2 units, l, unnormalised o) for the combine kernel.
//  * Cluster mode (split plans whose whole grid fits on the GPU at once, e.g.
//    batch 1): the S split CTAs of a unit form one thread-block cluster, one
//    CTA per SM with a deep ring.  Each CTA keeps its merged (m, l, o) in its
//    own shared memory; after a cluster barrier the CTAs merge them through
//    distributed shared memory (mapa + ld.shared::cluster), each CTA a slice
//    of the unit's outputs, and write fp16 -- one launch, no partials in
//    global memory, no combine kernel.
//  * Before waiting for the previous kernel on the stream (programmatic
//    dependent launch), the producer warms L2 with the CTA's first tiles, so
//    the first loads of a call overlap the tail of the previous kernel.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <type_traits>

#include "device_common.cuh"
#include "kernels.h"

namespace fqkv {
namespace {

constexpr int kGroupWarps = 4;     // consumer warps of one group: 16 keys of every tile each
constexpr int kTK = 64;            // keys per tile
constexpr int kHalfBytes = kTK * 128;
constexpr int kMergeHeads = 4;     // heads merged per epilogue pass

template <int D, bool kCl = false>
struct F16Cfg {
  static constexpr int kHalves = D / 64;                 // 128-byte column blocks per row
  static constexpr int kTileBytes = kHalves * kHalfBytes;  // K (or V) tile
  static constexpr int kStageBytes = 2 * kTileBytes;
  // D = 64: 3 stages keep shared memory at 55 KB so 4 CTAs fit per SM (one
  // wave for B*Hkv = 512 units; measured 20.5 -> 16.6 us at B=64, N=640 and
  // 329.6 -> 323.3 us at N=16K).  D = 128: 3 stages, 2 CTAs (registers).
  // Cluster mode: one CTA per SM streams alone, so it gets a 192 KB ring
  // (6 stages at D = 128, 12 at D = 64) to keep enough bytes in flight.
  static constexpr int kStages = kCl ? (192 * 1024) / kStageBytes : 3;
  static constexpr size_t kRingBytes = size_t(kStages) * kStageBytes;
  static constexpr size_t kBarBytes = 2 * kStages * sizeof(uint64_t);
  // Cluster mode runs one CTA per SM, so it gets two consumer groups taking
  // alternate tiles (two warps per scheduler to hide the MMA / ldmatrix /
  // exp latency chains); persistent mode has 2-4 CTAs per SM instead.
  static constexpr int kGroups = kCl ? 2 : 1;
  static constexpr int kCW = kGroupWarps * kGroups;  // consumer warps
  static constexpr int kThr = 32 * (kCW + 1);        // + the producer warp
  static constexpr size_t kMergeBytes = size_t(kCW) * (2 * 8 + kMergeHeads * D) * sizeof(float);
  // cluster mode: this CTA's merged (m, l) of up to 8 heads and o [8][D], read by the cluster
  static constexpr size_t kClusterBytes = kCl ? (2 * 8 + 8 * D) * sizeof(float) : 0;
  static constexpr size_t kSmemBytes = 1024 /*align slack*/ + kRingBytes + kBarBytes + kMergeBytes + kClusterBytes;
};
constexpr int kMaxCluster = 16;

struct UnitCoord {
  int b, kh, grp, s;
};

// Persistent mode: units ordered (b, kh, s, grp).  Cluster mode: (b, kh, grp, s),
// so the S_eff split CTAs of one unit are consecutive blocks -- one cluster.
template <bool kCl>
__device__ __forceinline__ UnitCoord decode_unit(const DecodeLaunch& a, int u) {
  UnitCoord c;
  if constexpr (kCl) {
    c.s = u % a.S_eff;
    u /= a.S_eff;
    c.grp = u % a.groups;
    u /= a.groups;
  } else {
    c.grp = u % a.groups;
    u /= a.groups;
    c.s = u % a.S_eff;
    u /= a.S_eff;
  }
  c.kh = u % a.Hkv;
  c.b = u / a.Hkv;
  return c;
}

// Byte offset of 16-byte chunk `chunk` (0 .. D/8-1) of tile row `row` in a
// 128B-swizzled tile made of D/64 column blocks of [kTK rows x 128 B].
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return uint32_t((chunk >> 3) * kHalfBytes + row * 128 + (((chunk & 7) ^ (row & 7)) << 4));
}

template <int D, bool kCl>
__global__ void __launch_bounds__(F16Cfg<D, kCl>::kThr) decode_f16_kernel(const __grid_constant__ DecodeLaunch a) {
  using C = F16Cfg<D, kCl>;
  extern __shared__ uint8_t smem_raw[];
  // aligned by an offset from the shared array, so that every access through `smem` stays a
  // shared-memory access (an integer round trip of the pointer would make them generic)
  uint8_t* smem = smem_raw + ((uint32_t(1024) - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kRingBytes);
  uint64_t* empty = full + C::kStages;
  float* sm_m = reinterpret_cast<float*>(empty + C::kStages);  // [warps][8]
  float* sm_l = sm_m + C::kCW * 8;                             // [warps][8]
  float* sm_o = sm_l + C::kCW * 8;                             // [warps][kMergeHeads][D]
  float* cl_m = sm_o + C::kCW * kMergeHeads * D;               // cluster mode: [8]
  float* cl_l = cl_m + 8;                                      // [8]
  float* cl_o = cl_l + 8;                                      // [8][D]
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const WaitCtl wc{a.status, a.timeout_ns};

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kGroupWarps);  // the 4 warps of the group that consumes the stage
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == C::kCW && lane == 0) {
    prefetch_tensormap(&a.tmK);
    prefetch_tensormap(&a.tmV);
    // warm L2 with this CTA's first tiles while the previous kernel finishes
    if (blockIdx.x < a.units && !a.debug_skip_loads) {
      const UnitCoord uc = decode_unit<kCl>(a, blockIdx.x);
      const int lo = uc.s * a.chunk;
      const int hi = min(a.N, lo + a.chunk);
      const int z = uc.b * a.Hkv + uc.kh;
      for (int k0 = lo, i = 0; k0 < hi && i < C::kStages; k0 += kTK, ++i) {
#pragma unroll
        for (int h = 0; h < C::kHalves; ++h) {
          tma_prefetch_l2_3d(&a.tmK, 64 * h, k0, z);
          tma_prefetch_l2_3d(&a.tmV, 64 * h, k0, z);
        }
      }
    }
  }
  __syncthreads();
  // Let the combine kernel (if any) get scheduled while this grid streams.
  pdl_launch_dependents();
  // Launched with programmatic serialization: wait for the previous kernel on
  // the stream (and its memory) before reading any input.
  pdl_wait_primary();
  // Valid keys: the launch's N, or the device-side length of a growing cache.
  const int n_valid = a.n_dev ? min(a.N, *a.n_dev) : a.N;

  // ------------------------------------------------------------ producer
  if (warp == C::kCW) {
    if (lane == 0 && !a.debug_skip_loads) {
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < a.units && ok; u += gridDim.x) {
        const UnitCoord uc = decode_unit<kCl>(a, u);
        const int lo = uc.s * a.chunk;
        const int hi = min(n_valid, lo + a.chunk);
        const int z = uc.b * a.Hkv + uc.kh;
        for (int k0 = lo; k0 < hi; k0 += kTK, ++it) {
          const int st = it % C::kStages;
          if (it >= C::kStages) {
            if (*reinterpret_cast<volatile int*>(&abort_flag) ||
                !mbar_wait(&empty[st], ((it / C::kStages) - 1) & 1, wc, kDevTimeoutEmpty)) {
              ok = false;
              break;
            }
          }
          mbar_arrive_expect_tx(&full[st], C::kStageBytes);
          uint8_t* sk = smem + size_t(st) * C::kStageBytes;
          uint8_t* sv = sk + C::kTileBytes;
#pragma unroll
          for (int h = 0; h < C::kHalves; ++h) tma_load_3d(sk + h * kHalfBytes, &a.tmK, 64 * h, k0, z, &full[st]);
#pragma unroll
          for (int h = 0; h < C::kHalves; ++h) tma_load_3d(sv + h * kHalfBytes, &a.tmV, 64 * h, k0, z, &full[st]);
        }
      }
      if (!ok) {
        // The consumers gave up: wait (bounded) for our own copies in flight so
        // no TMA write lands in shared memory after the CTA has exited.
        for (int j = (it > C::kStages ? it - C::kStages : 0); j < it; ++j)
          mbar_wait(&full[j % C::kStages], (j / C::kStages) & 1, wc, kDevTimeoutDrain);
      }
    }
    if constexpr (kCl) {
      // the whole warp takes part in the consumers' two cluster barriers (see the epilogue)
      __syncwarp();
      cluster_sync_all();
      cluster_sync_all();
    }
    return;
  }

  // ------------------------------------------------------------ consumers
  const int g = lane >> 2;   // mma row (query head within the group)
  const int t = lane & 3;
  const int mi = lane >> 3;  // ldmatrix matrix index supplied by this lane
  const int rr = lane & 7;   // ldmatrix row within that matrix
  const int grp = warp / kGroupWarps;         // consumer group: takes tiles it with it % kGroups == grp
  const int r0 = (warp % kGroupWarps) * 16;   // this warp's 16 keys within a tile
  const uint32_t ring = smem_u32(smem);
  const float csc = a.sm_scale_log2;
  bool alive = true;
  int it = 0;

  for (int u = blockIdx.x; u < a.units; u += gridDim.x) {
    const UnitCoord uc = decode_unit<kCl>(a, u);
    const int lo = uc.s * a.chunk;
    const int hi = min(n_valid, lo + a.chunk);
    const int h0 = uc.kh * a.G + uc.grp * a.GP;
    const int gvalid = min(a.GP, a.G - uc.grp * a.GP);

    // Q fragments (A operand rows = heads of the group; rows >= gvalid are 0).
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
      if (C::kGroups > 1 && it % C::kGroups != grp) continue;
      const int st = it % C::kStages;
      if (alive) {
        // warp-uniform decision: every lane waits, the warp proceeds only if all did
        const bool ok = mbar_wait(&full[st], (it / C::kStages) & 1, wc, kDevTimeoutFull) &&
                        !*reinterpret_cast<volatile int*>(&abort_flag);
        alive = __all_sync(0xffffffffu, ok);
        if (!alive && lane == 0) abort_flag = 1;
      }
      if (!alive) continue;
      const uint32_t sk = ring + uint32_t(st) * C::kStageBytes;
      const uint32_t sv = sk + C::kTileBytes;
      // One tile of this warp's 16 keys; kMask adds the per-key bound checks and V masks that only
      // the last (partial) tile of a unit needs.
      auto tile = [&](auto mask_tag) {
        constexpr bool kMask = decltype(mask_tag)::value;

        // ---- S = Q K^T for this warp's 16 keys (two n8 tiles)
        float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const int row = r0 + ((mi >> 1) << 3) + rr;
          const int chunk = 2 * kk + (mi & 1);
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4(sk + swz(row, chunk), b0, b1, b2, b3);
          mma_16816(sc[0], qa[kk][0], 0u, qa[kk][1], 0u, b0, b1);
          mma_16816(sc[1], qa[kk][0], 0u, qa[kk][1], 0u, b2, b3);
        }

        // ---- online softmax (log2 domain); row g, keys k0 + r0 + 8j + 2t + e
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int key = k0 + r0 + 8 * j + 2 * t + e;
            const float v = (!kMask || key < hi) ? sc[j][e] * csc : -INFINITY;
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
        const float p00 = ex2(sc[0][0] - mu), p01 = ex2(sc[0][1] - mu);
        const float p10 = ex2(sc[1][0] - mu), p11 = ex2(sc[1][1] - mu);
        l_run += (p00 + p01) + (p10 + p11);
        const uint32_t pa0 = pack_half2(p00, p01);
        const uint32_t pa2 = pack_half2(p10, p11);

        // ---- O += P V  (V^T fragments via ldmatrix.trans).  This lane's B registers
        // b0/b2 hold keys r0 + 2t, +1 and b1/b3 keys r0 + 8 + 2t, +9 (the columns of
        // its P registers).  Past the valid length a KV cache may hold anything
        // (a torch.empty tail): p = 0 there, but 0 * inf / NaN is NaN, so in the last
        // tile the V halves of keys past `hi` are masked to zero (one AND per B register).
        uint32_t vm0 = 0xffffffffu, vm1 = 0xffffffffu;
        if constexpr (kMask) {
          const int kb = k0 + r0 + 2 * t;
          vm0 = (kb < hi ? 0x0000ffffu : 0u) | (kb + 1 < hi ? 0xffff0000u : 0u);
          vm1 = (kb + 8 < hi ? 0x0000ffffu : 0u) | (kb + 9 < hi ? 0xffff0000u : 0u);
        }
#pragma unroll
        for (int pp = 0; pp < D / 16; ++pp) {
          const int row = r0 + ((mi & 1) << 3) + rr;
          const int chunk = 2 * pp + (mi >> 1);
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4_trans(sv + swz(row, chunk), b0, b1, b2, b3);
          if constexpr (kMask) {
            b0 &= vm0;
            b1 &= vm1;
            b2 &= vm0;
            b3 &= vm1;
          }
          mma_16816(o[2 * pp], pa0, 0u, pa2, 0u, b0, b1);
          mma_16816(o[2 * pp + 1], pa0, 0u, pa2, 0u, b2, b3);
        }
      };
      if (k0 + kTK <= hi) tile(std::false_type{});
      else tile(std::true_type{});
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }

    // ---- unit epilogue: merge the 4 warps, write output or partial
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
    if (t == 0) {
      sm_m[warp * 8 + g] = m_run;
      sm_l[warp * 8 + g] = l_run;
    }
    const int ct = threadIdx.x;  // 0 .. 127
    const size_t row_base = size_t(uc.b) * a.Hq + h0;
    for (int hp = 0; hp < gvalid; hp += kMergeHeads) {
      const int gl = g - hp;
      if (gl >= 0 && gl < kMergeHeads && g < gvalid) {
#pragma unroll
        for (int j = 0; j < D / 8; ++j) {
          float2 v2 = make_float2(o[j][0], o[j][1]);
          *reinterpret_cast<float2*>(&sm_o[(warp * kMergeHeads + gl) * D + 8 * j + 2 * t]) = v2;
        }
      }
      named_bar_sync(1, 32 * C::kCW);
      const int nh = min(kMergeHeads, gvalid - hp);
      for (int idx = ct; idx < nh * D; idx += 32 * C::kCW) {
        const int gl2 = idx / D, d = idx - gl2 * D;
        const int gg = hp + gl2;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < C::kCW; ++w) M = fmaxf(M, sm_m[w * 8 + gg]);
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < C::kCW; ++w) {
          const float mw = sm_m[w * 8 + gg];
          const float wt = (mw == -INFINITY) ? 0.f : ex2(mw - M);
          L += wt * sm_l[w * 8 + gg];
          O += wt * sm_o[(w * kMergeHeads + gl2) * D + d];
        }
        const size_t row = row_base + gg;
        if constexpr (kCl) {
          if (d == 0) {
            cl_m[gg] = M;
            cl_l[gg] = L;
          }
          cl_o[gg * D + d] = O;
        } else if (a.S_eff == 1) {
          store_out(a, row * D + d, O / L);
        } else {
          const size_t slot = row * a.S + uc.s;
          if (d == 0) {
            a.part_m[slot] = M;
            a.part_l[slot] = L;
          }
          a.part_o[slot * D + d] = O;
        }
      }
      named_bar_sync(1, 32 * C::kCW);
    }
    if constexpr (kCl) {
      // ---- cluster merge: every CTA's (m, l, o) is in its shared memory; CTA r
      // merges outputs r*128 + ct, r*128 + ct + S*128, ... of the unit's gvalid x D
      // (log-sum-exp weights, an empty split weighs 0) and writes them as fp16.
      // Every thread of every CTA (the producer warp too) passes both barriers.
      cluster_sync_all();
      const int S = a.S_eff;
      const uint32_t r = cluster_ctarank();
      for (int idx = int(r) * (32 * C::kCW) + ct; idx < gvalid * D; idx += S * 32 * C::kCW) {
        const int gg = idx / D, d = idx - gg * D;
        const uint32_t am = smem_u32(cl_m + gg), al = smem_u32(cl_l + gg), ao = smem_u32(cl_o + gg * D + d);
        float mj[kMaxCluster];
        float M = -INFINITY;
#pragma unroll
        for (int j = 0; j < kMaxCluster; ++j) {
          mj[j] = j < S ? ld_dsmem_f32(dsmem_addr(am, j)) : -INFINITY;
          M = fmaxf(M, mj[j]);
        }
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int j = 0; j < kMaxCluster; ++j) {
          if (j < S && mj[j] != -INFINITY) {
            const float wt = ex2(mj[j] - M);
            L = fmaf(wt, ld_dsmem_f32(dsmem_addr(al, j)), L);
            O = fmaf(wt, ld_dsmem_f32(dsmem_addr(ao, j)), O);
          }
        }
        store_out(a, (row_base + gg) * D + d, O / L);
      }
      // no CTA may exit (and release its shared memory) while others still read it
      cluster_sync_all();
    } else {
      if (a.S_eff == 1) signal_out(a, ct, 1, 32 * C::kCW);
    }
  }
}

}  // namespace

template <int D>
static cudaError_t launch_f16(const DecodeLaunch& a, cudaStream_t stream) {
  if (a.cluster == 0) {
    launch_pdl(decode_f16_kernel<D, false>, dim3(a.grid), dim3(F16Cfg<D>::kThr), F16Cfg<D>::kSmemBytes, stream, a);
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.grid);
  cfg.blockDim = dim3(F16Cfg<D, true>::kThr);
  cfg.dynamicSmemBytes = F16Cfg<D, true>::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = unsigned(a.cluster);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, decode_f16_kernel<D, true>, a);
}

KernelShape decode_kernel_shape_f16(int D) {
  return KernelShape{F16Cfg<64>::kThr, D == 128 ? F16Cfg<128>::kSmemBytes : F16Cfg<64>::kSmemBytes};
}

cudaError_t decode_kernel_prepare_f16(int D, int* ctas_per_sm) {
  const void* fn = D == 128 ? reinterpret_cast<const void*>(&decode_f16_kernel<128, false>)
                            : reinterpret_cast<const void*>(&decode_f16_kernel<64, false>);
  const size_t smem = decode_kernel_shape_f16(D).smem_bytes;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(ctas_per_sm, fn, F16Cfg<64>::kThr, smem);
}

template <int D>
static cudaError_t prepare_cluster(int (&max_clusters)[17]) {
  const void* fn = reinterpret_cast<const void*>(&decode_f16_kernel<D, true>);
  const size_t smem = F16Cfg<D, true>::kSmemBytes;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e == cudaSuccess) e = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e != cudaSuccess) return e;
  max_clusters[0] = max_clusters[1] = 0;
  for (int c = 2; c <= kMaxCluster; ++c) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(c);
    cfg.blockDim = dim3(F16Cfg<D, true>::kThr);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = unsigned(c);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess) {
      cudaGetLastError();  // an unsupported size is not an error of the library
      n = 0;
    }
    max_clusters[c] = n;
  }
  return cudaSuccess;
}

cudaError_t decode_kernel_prepare_f16_cluster(int D, int (&max_clusters)[17]) {
  return D == 128 ? prepare_cluster<128>(max_clusters) : prepare_cluster<64>(max_clusters);
}

cudaError_t launch_decode_f16(const DecodeLaunch& a, cudaStream_t stream) {
  return a.D == 128 ? launch_f16<128>(a, stream) : launch_f16<64>(a, stream);
}

}  // namespace fqkv
