// Quantized-KV decode attention on the tensor cores, sm_100a: int8 codes with
// several query heads per KV head (a GQA model's int8 cache) and int4 codes.
//
// The reference has int8 KV for one query head per KV row
// (decode_attn_int8_mw, kernels/decode_attn_int8_mw.cu:6-51), int4 KV for one
// query head per row and D = 64 (decode_attn_int4, kernels/decode_attn_int4.cu:
// 8-46) and GQA only for fp16 (decode_attn_gqa, kernels/decode_attn_gqa.cu:
// 8-55).  Layout: codes [B, Hkv, stride, RB] (RB = D bytes for int8, D/2 for
// int4: two signed nibbles per byte, element 2i in the low nibble, as the
// reference packs them, notebook lines 292-299), per-token scales
// [B, Hkv, stride] fp16, q/out [B, Hq, D] fp16.
//
//  * Persistent, warp-specialised: a unit is (sequence, KV head, group of <= 8
//    query heads, split).  Warp 4 streams tiles of 4*KPW keys of K and V codes
//    with 3-D TMA tensor copies (swizzled at the row width: 128, 64 or 32
//    bytes; keys past the end zero-filled) plus 16-byte-aligned windows of
//    their fp16 scales into a ring of stages; each consumer warp takes KPW keys
//    of a tile and reads every KV byte once for all heads of the group.
//  * S = Q K^T on the integer tensor cores (mma m16n8k32, s32 accumulate)
//    straight from the codes: q is a 2-plane fixed-point number per head
//    (q * Qs = hi * 256 + lo, |q * Qs| <= 32639, Qs = 32639 / max|q|); rows 0-7
//    of the A operand carry the hi planes of the group's heads and rows 8-15
//    the lo planes, so one MMA gives both partial sums of a score.  int8 codes
//    are the B operand as they are (s8).  int4 low nibbles enter as unsigned
//    bytes code + 8 (one logic op per 4 codes; the + 8 is removed once per
//    score with the head's 8 * sum(q) term), high nibbles as the signed bytes
//    16 * code they already are in place (one mask).  The head dimension is
//    permuted identically for q and K so that each thread reads one
//    contiguous D/4-dimension span of a key row.
//  * Several heads (int8): O^T += V^T (P * Vscale)^T on the fp16 tensor cores
//    (m16n8k16): the A operand pairs one dimension of two consecutive keys,
//    built in registers from the codes (a byte permute of the two keys' words,
//    one three-input logic op forming the exact fp16 1152 + code); the B
//    operand is the fp16 probabilities times the key's V scale, taken directly
//    from the score accumulators.  The 1152 offset leaves once per unit:
//    1152 times the per-head sum of the same B operand, which one extra MMA
//    of an all-ones A tile accumulates per 16 keys.
//    Rows of O^T are head dimensions, columns the group's heads.
//  * One head (int4): the same product on the integer tensor cores
//    (m16n8k32): V bytes arrive transposed by ldmatrix.trans plus two byte
//    permutes per register pair, P * Vscale is a three-plane 8-bit fixed-point
//    number in frames of one reference maximum and scale (see g1_key and
//    g1_flush below).  The softmax denominator sums the unscaled probabilities.
//  * Split plans of the several-heads variant merge either through fp32
//    partials and the PDL-chained combine kernel, or (kCl, small short calls)
//    inside one thread-block cluster: each CTA leaves its merged (m, l, O) of
//    the group's heads in shared memory and, after a cluster barrier that the
//    producer warp joins on every path, CTA r merges a slice of the outputs
//    through distributed shared memory -- one launch, no workspace.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <type_traits>

#include "device_common.cuh"
#include "kernels.h"

namespace fqkv {
namespace {

constexpr int kConsumerWarps = 4;  // consumer warps of one group: KPW keys of every tile each
constexpr int kQMax = 32639;  // |q * Qs| bound: hi = (v + 128) >> 8 stays in [-127, 127]

// kCl: 0 = persistent grid; 1 / 2 = the split CTAs of a unit merge inside one thread-block cluster,
// with one / two consumer groups per CTA.
template <int D, bool I4, bool G1, int kCl = 0>
struct QtcCfg {
  static constexpr int RB = I4 ? D / 2 : D;                   // bytes of one key row
  static constexpr int KPW = (!I4 && D == 128) ? 16 : 32;      // keys per consumer warp per tile
  static constexpr int TK = 4 * KPW;                           // keys per tile
  static constexpr int kTileBytes = TK * RB;                   // K (or V) codes of one tile
  static constexpr int kScaleBytes = 2 * TK + 32;              // 16B-aligned scale window
  static constexpr int kStageRaw = 2 * kTileBytes + 2 * kScaleBytes;
  static constexpr int kStageBytes = (kStageRaw + 1023) & ~1023;  // tiles stay 1024-aligned (swizzle atom)
  // Resident CTAs per SM and ring depth, measured on B200: the kernel is
  // issue-bound (consumers almost never wait for a tile), so the GQA variant
  // runs 4 CTAs (20 warps) with a 2-stage ring (332.6 -> 323.7 us at B=64,
  // N=16K, D=128); the one-head int4 variant keeps 3 CTAs and 4 stages.
  // The one-head int4 variant at D = 64 moves 4 KB tiles: 7 stages (3 CTAs still fit in 228 KB).
  // Cluster mode (int8 GQA): the cluster's CTAs each stream a split alone, so one CTA per SM with
  // an 8-stage ring (about 136 KB, which also keeps the hardware from packing a cluster onto few
  // SMs): measured 1.1-2.2x faster than the 4-CTA, 2-stage form in the same plans.
  static constexpr int kCtas = kCl ? 1 : (G1 ? 3 : 4);
  static constexpr int kStages = kCl ? 8 : (G1 ? (D == 64 ? 7 : 4) : 2);
  static constexpr int NSEG = RB / 16;                         // one head: 16-byte V row segments
  static constexpr int MH = G1 ? 1 : 4;                        // heads merged per epilogue pass
  static constexpr size_t kRingBytes = size_t(kStages) * kStageBytes;
  static constexpr size_t kBarBytes = 2 * kStages * sizeof(uint64_t);
  // Cluster mode runs one CTA per SM; its two-group form has two consumer groups taking alternate
  // tiles (twice the warps to issue the per-key work: batch 1, N = 16K, D = 128 18.8 -> 15.5 us),
  // the one-group form serves splits of one or two tiles, where a second group would sit idle
  // (N = 640: 5.3 -> 4.7 us); persistent mode has 3-4 CTAs per SM instead.
  static constexpr int kGroups = kCl == 2 ? 2 : 1;
  static constexpr int kCW = kConsumerWarps * kGroups;  // consumer warps
  static constexpr int kThr = 32 * (kCW + 1);           // + the producer warp
  static constexpr size_t kMergeBytes = size_t(kCW) * (2 * 8 + MH * D) * sizeof(float);
  // cluster mode (int8 GQA): this CTA's merged (m, l) of up to 8 heads and o [8][D], read by the cluster
  static constexpr size_t kClusterBytes = kCl ? (2 * 8 + 8 * D) * sizeof(float) : 0;
  static constexpr size_t kSmemBytes = 1024 + kRingBytes + kBarBytes + kMergeBytes + kClusterBytes;
  static_assert(TK == tile_keys(I4 ? KvFormat::I4Tc : KvFormat::I8Gqa, D), "planner tile size");
  static_assert(!G1 || KPW % 16 == 0, "one-head variant works in 16-key blocks");
};

constexpr int kMaxCluster = 16;

struct UnitCoord {
  int b, kh, grp, s;
};

// Persistent mode: units ordered (b, kh, s, grp).  Cluster mode: (b, kh, grp, s),
// so the S_eff split CTAs of one unit are consecutive blocks -- one cluster.
template <int kCl>
__device__ __forceinline__ UnitCoord decode_unit(const DecodeLaunch& a, int u) {
  UnitCoord c;
  if constexpr (kCl != 0) {
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

// Byte offset of byte `b` of key row `row` inside a tile written by the TMA
// copy with the swizzle of the row width (16-byte chunk index XOR the row's
// position in the 1024-byte swizzle atom; the tile starts 1024-aligned).
template <int RB>
__device__ __forceinline__ uint32_t tile_off(int row, int b) {
  const int c = b >> 4, w = b & 15;
  if constexpr (RB == 128) return uint32_t(row * 128 + ((c ^ (row & 7)) << 4) + w);
  else if constexpr (RB == 64) return uint32_t(row * 64 + ((c ^ ((row >> 1) & 3)) << 4) + w);
  else return uint32_t(row * 32 + ((c ^ ((row >> 2) & 1)) << 4) + w);
}

// Loads N bytes (4, 8 or 16; N-aligned) from shared memory into words w[0..N/4).
template <int N>
__device__ __forceinline__ void lds_words(const uint8_t* p, uint32_t* w) {
  if constexpr (N == 16) {
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  } else if constexpr (N == 8) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    w[0] = v.x; w[1] = v.y;
  } else {
    w[0] = *reinterpret_cast<const uint32_t*>(p);
  }
}

// D(16x8, s32) += A(16x32, s8 or u8, row) * B(32x8, s8 or u8, col).  A pure
// register operation (not volatile), so shared-memory loads may be scheduled around it.
template <bool kAUnsigned, bool kBUnsigned>
__device__ __forceinline__ void mma_i8_16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  static_assert(!(kAUnsigned && kBUnsigned), "unused combination");
  if constexpr (kBUnsigned) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else if constexpr (kAUnsigned) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// f(p) = B ? A : (p ^ A) bitwise: with p = {x.b, -, y.b, -} (byte b of the two keys' words) each
// half becomes an exact fp16 1024 + 128 + code (A holds 0x64 in the high byte of each half, the
// code byte's sign-flip bit in the low byte; B marks the bits taken from A).  The int8 GQA P.V
// multiplies these and removes 1152 * sum(P) once per unit -- sum(P) accumulated from the same
// fp16 B operand, four mixed-precision adds per 16 keys -- instead of one fp16 subtraction per
// code pair.
template <uint32_t A, uint32_t B>
__device__ __forceinline__ uint32_t code_pair_offset(uint32_t p) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0x9c;" : "=r"(r) : "r"(p), "r"(A), "r"(B));
  return r;
}
constexpr uint32_t kI8A = 0x64806480u, kI8B = 0xFF00FF00u;    // whole byte: int8 code
constexpr float kI8Offset = 1152.f;

// acc += both halves of an fp16 pair, exactly (mixed-precision FMAs by 1.0)
__device__ __forceinline__ void add_half2(float& acc, uint32_t h2) {
  asm("{\n\t.reg .f16 a, b, one;\n\tmov.b32 {a, b}, %1;\n\tmov.b16 one, 0x3C00;\n\t"
      "fma.rn.f32.f16 %0, a, one, %0;\n\tfma.rn.f32.f16 %0, b, one, %0;\n\t}"
      : "+f"(acc)
      : "r"(h2));
}

// The low nibble of every byte as the unsigned byte code + 8, in one logic op.
__device__ __forceinline__ uint32_t low_nibbles_offset(uint32_t x) { return xor_and<0x08080808u, 0x0F0F0F0Fu>(x); }

__device__ __forceinline__ uint32_t pack_s8x4(int a, int b, int c, int d) {
  return (uint32_t(a) & 0xFFu) | ((uint32_t(b) & 0xFFu) << 8) | ((uint32_t(c) & 0xFFu) << 16) |
         (uint32_t(d) << 24);
}

// Position (0 .. D/4-1, within this thread's span of the head dimension) of
// byte i (0..3) of operand half h (0: b0, 1: b1) of integer k-step kk.
template <int D, bool I4>
__device__ __forceinline__ constexpr int qk_dim(int kk, int h, int i) {
  if constexpr (!I4) {
    return 8 * kk + 4 * h + i;
  } else {
    constexpr int half = D / 64;  // low-nibble k-steps
    return kk < half ? 16 * kk + 8 * h + 2 * i : 16 * (kk - half) + 8 * h + 2 * i + 1;
  }
}

// ---- one-head int4 variant (G1): P.V on the integer tensor cores
//
// Key (0..31 within a warp's share of a tile) that lane group g holds as
// score i (0..3; i = 2 * m-tile + row half of S^T).  The P.V k-slot 4a + i
// carries key g1_key(a, i), so that the B operand of a thread's k-slots
// 4t..4t+3 (16+4t..) is the four scores of lane group t (t + 4), and the
// eight keys of every ldmatrix 8x8 matrix differ mod 8 (conflict-free with
// the 64-byte row swizzle).
__device__ __forceinline__ constexpr int g1_key(int g, int i) { return 8 * i + (g ^ (4 * (i & 1))); }

// P is fixed point in a frame (reference maximum m_run, scale Ps):
// v = rint(p * vs * Ps) with p = 2^(s - m_run) <= 2^kG1Headroom.  A frame
// starts when a tile's largest p * vs would exceed kG1VLim / Ps (Ps is then
// set to kG1VLim / (1.25 * that product)), so v <= kG1VLim < 2^23 - 32896
// and the largest products keep about 22 significant bits.  The float
// 2^23 + v + 32896 (one FMA with kG1Magic, rounding to nearest) holds
// u = v + 32896 = h * 65536 + (m + 128) * 256 + (l + 128) in its low 23
// bits: v = h * 65536 + m * 256 + l with the signed bytes m, l and h in
// [0, 127], the three planes of the B operand (columns 0, 1, 2).
constexpr float kG1Magic = 8421504.f;
constexpr float kG1Headroom = 3.f;
constexpr float kG1VLim = 8.0e6f;
// s32 accumulator bound: |code term| <= 128 and |plane| <= 128 per key, so a
// frame ends after at most 2048 tiles (65536 keys per warp, < 2^31 / 16384)
constexpr int kG1FrameTiles = 2048;

// Ends a frame: adds the integer accumulators times 1/Ps to the warp's fp32 O
// in shared memory and scales the sum by `rescale` (both are relative to the
// frame's maximum; rescale moves them to the next frame's), lane (g, 0)
// owning head dimensions 32s + 4g + 0..3 (s < NSEG = D/32); clears the
// accumulators.  oi[s] (s < NSEG) holds the low nibbles (code + 8, rows g /
// g + 8 = dimensions 32s + 4g / + 2), oi[NSEG + s] the high nibbles (16 *
// code, dimensions + 1); columns 0 / 1 are the h / m planes in lanes t = 0,
// column 2 the l plane in lanes t = 1.  bsum: the plane sums of this lane's
// keys (plane t), for the + 8 of the low nibbles.
template <int NSEG>
__device__ __forceinline__ void g1_flush(int (&oi)[8][4], int& bsum, float* so, float rescale, float inv_ps, int g,
                                         int t) {
  int bs = bsum;
  bs += __shfl_xor_sync(0xffffffffu, bs, 4);
  bs += __shfl_xor_sync(0xffffffffu, bs, 8);
  bs += __shfl_xor_sync(0xffffffffu, bs, 16);  // lane (g, c): sum of plane c over the frame
  const int b1 = __shfl_down_sync(0xffffffffu, bs, 1);
  const int b2 = __shfl_down_sync(0xffffffffu, bs, 2);
#pragma unroll
  for (int sg = 0; sg < NSEG; ++sg) {
    const int l0 = __shfl_down_sync(0xffffffffu, oi[sg][0], 1);
    const int l2 = __shfl_down_sync(0xffffffffu, oi[sg][2], 1);
    const int h0 = __shfl_down_sync(0xffffffffu, oi[NSEG + sg][0], 1);
    const int h2 = __shfl_down_sync(0xffffffffu, oi[NSEG + sg][2], 1);
    if (t == 0) {
      float4* dst = reinterpret_cast<float4*>(so + 32 * sg + 4 * g);
      float4 c = *dst;
      const float lg = float(oi[sg][0] - 8 * bs) * 65536.f + float(oi[sg][1] - 8 * b1) * 256.f + float(l0 - 8 * b2);
      const float hg = (float(oi[NSEG + sg][0]) * 65536.f + float(oi[NSEG + sg][1]) * 256.f + float(h0)) * 0.0625f;
      const float lg8 = float(oi[sg][2] - 8 * bs) * 65536.f + float(oi[sg][3] - 8 * b1) * 256.f + float(l2 - 8 * b2);
      const float hg8 =
          (float(oi[NSEG + sg][2]) * 65536.f + float(oi[NSEG + sg][3]) * 256.f + float(h2)) * 0.0625f;
      c.x = fmaf(lg, inv_ps, c.x) * rescale;
      c.y = fmaf(hg, inv_ps, c.y) * rescale;
      c.z = fmaf(lg8, inv_ps, c.z) * rescale;
      c.w = fmaf(hg8, inv_ps, c.w) * rescale;
      *dst = c;
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) oi[i][0] = oi[i][1] = oi[i][2] = oi[i][3] = 0;
  bsum = 0;
}

template <int D, bool I4, bool G1, int kCl = 0>
__global__ void __launch_bounds__(QtcCfg<D, I4, G1, kCl>::kThr, QtcCfg<D, I4, G1, kCl>::kCtas) decode_qtc_kernel(const __grid_constant__ DecodeLaunch a) {
  using C = QtcCfg<D, I4, G1, kCl>;
  static_assert(I4 == G1, "int4 runs the one-head variant, int8 the GQA one");
  static_assert(kCl == 0 || !G1, "the cluster merge serves the several-heads (int8 GQA) variant");
  constexpr int NSEG = C::NSEG;
  constexpr int MH = C::MH;
  constexpr int RB = C::RB;
  constexpr int KPW = C::KPW;
  constexpr int NJ = KPW / 8;          // score n-tiles (8 keys) per warp per tile
  constexpr int KP = KPW / 16;         // P.V k-steps (16 keys) per warp per tile
  constexpr int KS = D / 32;           // integer k-steps over the head dimension
  constexpr int MT = D / 16;           // m-tiles of O^T
  constexpr int KB = RB / 4;           // bytes of a K row this thread reads
  constexpr int VB = RB / 8;           // bytes of a V row this thread reads
  extern __shared__ uint8_t smem_raw[];
  // aligned by an offset from the shared array, so that every access through `smem` stays a
  // shared-memory access (an integer round trip of the pointer would make them generic)
  uint8_t* smem = smem_raw + ((uint32_t(1024) - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + C::kRingBytes);
  uint64_t* empty = full + C::kStages;
  float* sm_m = reinterpret_cast<float*>(empty + C::kStages);
  float* sm_l = sm_m + C::kCW * 8;
  float* sm_o = sm_l + C::kCW * 8;
  float* cl_m = sm_o + C::kCW * MH * D;  // cluster mode: [8]
  float* cl_l = cl_m + 8;                        // [8]
  float* cl_o = cl_l + 8;                        // [8][D]
  __shared__ int abort_flag;
  __shared__ int stage_off[C::kStages][2];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const WaitCtl wc{a.status, a.timeout_ns};

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);  // the warps of the group that consumes the stage
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == C::kCW && lane == 0) {
    prefetch_tensormap(&a.tmK);
    prefetch_tensormap(&a.tmV);
  }
  __syncthreads();
  pdl_launch_dependents();
  // Launched with programmatic serialization: wait for the previous kernel on
  // the stream (and its memory) before reading any input.
  pdl_wait_primary();
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
        const __half* Ksr = static_cast<const __half*>(a.Ks) + size_t(z) * a.kv_stride;
        const __half* Vsr = static_cast<const __half*>(a.Vs) + size_t(z) * a.kv_stride;
        for (int k0 = lo; k0 < hi; k0 += C::TK, ++it) {
          const int st = it % C::kStages;
          if (it >= C::kStages) {
            if (*reinterpret_cast<volatile int*>(&abort_flag) ||
                !mbar_wait(&empty[st], ((it / C::kStages) - 1) & 1, wc, kDevTimeoutEmpty)) {
              ok = false;
              break;
            }
          }
          const int nk = min(C::TK, hi - k0);
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
    }
    if constexpr (kCl != 0) {
      // the whole warp takes part in the consumers' two cluster barriers (see the epilogue)
      __syncwarp();
      cluster_sync_all();
      cluster_sync_all();
    }
    return;
  }

  // ------------------------------------------------------------ consumers
  const int g = lane >> 2;
  const int t = lane & 3;
  const int cgrp = warp / kConsumerWarps;       // consumer group: takes tiles it with it % kGroups == cgrp
  const int r0 = (warp % kConsumerWarps) * KPW;
  const float csc = a.sm_scale_log2;
  // V rows are read in a t-parity-dependent key order where that avoids bank
  // conflicts (rows of <= 64 bytes); the pair selector undoes the swap.
  constexpr bool kSwap = RB <= 64;
  const int vsw = kSwap ? (t & 1) : 0;
  const uint32_t sel_base = vsw ? 0x0044u : 0x4400u;
  // one head: this lane's ldmatrix row (matrix L/8 = k-slots {4t, 4t+1}, {4t+2, 4t+3} of groups
  // t < 4, then of groups t + 4; row L%8 = slot of group (L%8)/2) as a swizzled byte offset, and
  // the P plane this lane packs (t = 0 / 1 / 2: byte 2 / 1 / 0 of the magic float, 3: none)
  uint32_t v_row_off = 0, psel = 0, pxor = 0, pmask = 0;
  if constexpr (G1) {
    const int mi = lane >> 3, rr = lane & 7;
    const int row = r0 + g1_key((rr >> 1) + 4 * (mi >> 1), 2 * (mi & 1) + (rr & 1));
    v_row_off = tile_off<RB>(row, 0);  // chunk 0 of the swizzled row; segment sg: ^ (sg << 4)
    const uint32_t pb_ = t == 0 ? 2u : (t == 1 ? 1u : 0u);
    psel = pb_ | ((4u + pb_) << 4);
    pxor = (t == 1 || t == 2) ? 0x80808080u : 0u;
    pmask = t < 3 ? 0xFFFFFFFFu : 0u;
  }
  bool alive = true;
  int it = 0;

  for (int u = blockIdx.x; u < a.units; u += gridDim.x) {
    const UnitCoord uc = decode_unit<kCl>(a, u);
    const int lo = uc.s * a.chunk;
    const int hi = min(n_valid, lo + a.chunk);
    const int h0 = uc.kh * a.G + uc.grp * a.GP;
    const int gvalid = min(a.GP, a.G - uc.grp * a.GP);

    // ---- q of head g, dimensions [t*D/4, (t+1)*D/4), as two int8 planes
    uint32_t qa[KS][4];
    float hf;       // sm_scale_log2 / Qs of head g (int4: / 16 more)
    int qbias = 0;  // int4: 16 * 8 * sum of q * Qs over the low-nibble dimensions
    {
      float qf[D / 4];
      if (G1 || g < gvalid) {
        const uint32_t* qrow = reinterpret_cast<const uint32_t*>(
            static_cast<const __half*>(a.q) + (size_t(uc.b) * a.Hq + h0 + (G1 ? 0 : g)) * D + t * (D / 4));
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
      hf = amax > 0.f ? csc * (amax / float(kQMax)) * (I4 ? 0.0625f : 1.f) : 0.f;
      int qi[D / 4];
#pragma unroll
      for (int i = 0; i < D / 4; ++i) qi[i] = __float2int_rn(qf[i] * Qs);
      if constexpr (I4) {
#pragma unroll
        for (int i = 0; i < D / 4; i += 2) qbias += qi[i];
        qbias += __shfl_xor_sync(0xffffffffu, qbias, 1);
        qbias += __shfl_xor_sync(0xffffffffu, qbias, 2);
        qbias *= 128;
      }
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        int hv[8], lv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int v = qi[qk_dim<D, I4>(kk, i >> 2, i & 3)];
          hv[i] = (v + 128) >> 8;
          lv[i] = v - hv[i] * 256;
        }
        qa[kk][0] = pack_s8x4(hv[0], hv[1], hv[2], hv[3]);
        qa[kk][1] = pack_s8x4(lv[0], lv[1], lv[2], lv[3]);
        qa[kk][2] = pack_s8x4(hv[4], hv[5], hv[6], hv[7]);
        qa[kk][3] = pack_s8x4(lv[4], lv[5], lv[6], lv[7]);
        if constexpr (G1) {
          // one head: q is the B operand of S^T = K Q^T; columns 2c / 2c + 1 = hi / lo plane for
          // c = 0 .. 3, so the four lanes t of a group all hold the same scores (and lane t finishes
          // the score, probability and fixed-point word of the group's key t, see below)
          const uint32_t b0 = (g & 1) ? qa[kk][1] : qa[kk][0];
          const uint32_t b1 = (g & 1) ? qa[kk][3] : qa[kk][2];
          qa[kk][0] = b0;
          qa[kk][1] = b1;
        }
      }
    }

    float o[MT][4];   // several heads: O^T in fp32 (codes carried as 1152 + code)
    float pe = 0.f;   // several heads: this lane's sum of the fp16 B operand (head g)
    int oi[8][4];     // one head: the frame's integer O^T (see g1_flush)
    int bsum = 0, ftiles = 0;
    float ps = 0.f, inv_ps = 0.f;  // one head: the frame's fixed-point scale of P * vs and 1 / it
    float* so = sm_o + warp * D;  // one head: the warp's fp32 O
    if constexpr (G1) {
#pragma unroll
      for (int i = 0; i < 8; ++i) oi[i][0] = oi[i][1] = oi[i][2] = oi[i][3] = 0;
      if (lane < D / 4) reinterpret_cast<float4*>(so)[lane] = make_float4(0.f, 0.f, 0.f, 0.f);
      __syncwarp();
    } else {
#pragma unroll
      for (int i = 0; i < MT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    }
    float m_run = -INFINITY, l_run = 0.f;
    // several heads: the fp16 B operand p * vscale carries a warp-uniform power-of-two factor vsc,
    // lowered (O rescaled exactly) whenever a key's V scale times vsc would pass 2^14, so the operand
    // stays in fp16's normal range for any V magnitude (small V no longer rounds to subnormals,
    // which the fp16 MMA also runs slower on); O leaves the frame (/ vsc) in the epilogue.
    float vsc = 1099511627776.f, vk = 40.f;  // 2^40 = 2^vk; ex2(s - (m - vk)) = p * vsc, l sums the same

    for (int k0 = lo; k0 < hi; k0 += C::TK, ++it) {
      if (C::kGroups > 1 && it % C::kGroups != cgrp) continue;
      const int st = it % C::kStages;
      if (alive) {
        const bool ok = mbar_wait(&full[st], (it / C::kStages) & 1, wc, kDevTimeoutFull) &&
                        !*reinterpret_cast<volatile int*>(&abort_flag);
        alive = __all_sync(0xffffffffu, ok);
        if (!alive && lane == 0) abort_flag = 1;
      }
      if (!alive) continue;
      // the tile's body, compiled twice: full tiles (all but the last of a unit) without the
      // per-key bound checks
      auto tile = [&](auto mask_tag) {
        constexpr bool kMask = decltype(mask_tag)::value;
        const uint8_t* kt = ring + size_t(st) * C::kStageBytes;
        const uint8_t* vt = kt + C::kTileBytes;
        const __half* kst = reinterpret_cast<const __half*>(kt + 2 * C::kTileBytes) + stage_off[st][0];
        const __half* vst = reinterpret_cast<const __half*>(kt + 2 * C::kTileBytes + C::kScaleBytes) +
                            stage_off[st][1];

        // ---- scores of this warp's KPW keys (rows r0 ..) in integers.
        // Several heads: S = Q K^T, n-tile j holds keys 8j + 2t + e of head g.
        // One head (G1): S^T = K Q^T, m-tile mt holds (rows g / g + 8) keys
        // g1_key(g, 2mt + 0 / 1) in every lane t of group g (columns 2t / 2t + 1:
        // hi / lo plane); lane t keeps key g1_key(g, t) only (own_*).
        float sc[NJ][2];
        bool valid[NJ][2];
        float mx = -INFINITY;
        // one head: lane t of a group finishes the group's key t (k-slot 4g + t)
        int own_si = 0, own_key = 0;
        bool own_ok = false;
        float own_sc = -INFINITY;
        if constexpr (G1) {
          static_assert(!G1 || KP == 2, "one head: four keys per lane group and tile");
#pragma unroll
          for (int mt = 0; mt < KP; ++mt) {
            uint32_t kw[2][KB / 4];  // keys r0 + g1_key(g, 2mt) and r0 + g1_key(g, 2mt + 1)
#pragma unroll
            for (int e = 0; e < 2; ++e)
#pragma unroll
              for (int c = 0; c < KB; c += 16)
                lds_words<(KB < 16 ? KB : 16)>(kt + tile_off<RB>(r0 + g1_key(g, 2 * mt + e), t * KB + c), kw[e] + c / 4);
            int acc[4] = {0, 0, 0, 0};
            if constexpr (!I4) {
#pragma unroll
              for (int kk = 0; kk < KS; ++kk) {
                const uint32_t af[4] = {kw[0][2 * kk], kw[1][2 * kk], kw[0][2 * kk + 1], kw[1][2 * kk + 1]};
                mma_i8_16832<false, false>(acc, af, qa[kk][0], qa[kk][1]);
              }
            } else {
              int acch[4] = {0, 0, 0, 0};
#pragma unroll
              for (int kk = 0; kk < KS / 2; ++kk) {
                const uint32_t al[4] = {low_nibbles_offset(kw[0][2 * kk]), low_nibbles_offset(kw[1][2 * kk]),
                                        low_nibbles_offset(kw[0][2 * kk + 1]), low_nibbles_offset(kw[1][2 * kk + 1])};
                const uint32_t ah[4] = {kw[0][2 * kk] & 0xF0F0F0F0u, kw[1][2 * kk] & 0xF0F0F0F0u,
                                        kw[0][2 * kk + 1] & 0xF0F0F0F0u, kw[1][2 * kk + 1] & 0xF0F0F0F0u};
                mma_i8_16832<true, false>(acc, al, qa[kk][0], qa[kk][1]);
                mma_i8_16832<false, false>(acch, ah, qa[KS / 2 + kk][0], qa[KS / 2 + kk][1]);
              }
#pragma unroll
              for (int e = 0; e < 4; ++e) acc[e] = 16 * acc[e] + acch[e];
            }
            // the group's keys 2mt (rows g) and 2mt + 1 (rows g + 8): lane t keeps key t's sum
            const int si0 = acc[0] * 256 + acc[1] - (I4 ? qbias : 0);
            const int si1 = acc[2] * 256 + acc[3] - (I4 ? qbias : 0);
            if ((t >> 1) == mt) own_si = (t & 1) ? si1 : si0;
          }
          own_key = r0 + g1_key(g, t);
          own_ok = !kMask || (k0 + own_key) < hi;
          own_sc = own_ok ? float(own_si) * (__half2float(kst[own_key]) * hf) : -INFINITY;
          mx = own_sc;
        } else {
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
          uint32_t kw[KB / 4];  // key r0 + 8j + g, bytes [t*KB, (t+1)*KB)
#pragma unroll
          for (int c = 0; c < KB; c += 16)
            lds_words<(KB < 16 ? KB : 16)>(kt + tile_off<RB>(r0 + 8 * j + g, t * KB + c), kw + c / 4);
          int acc[4] = {0, 0, 0, 0};
          if constexpr (!I4) {
#pragma unroll
            for (int kk = 0; kk < KS; ++kk) mma_i8_16832<false, false>(acc, qa[kk], kw[2 * kk], kw[2 * kk + 1]);
          } else {
            int acch[4] = {0, 0, 0, 0};
#pragma unroll
            for (int kk = 0; kk < KS / 2; ++kk) {
              const uint32_t w0 = kw[2 * kk], w1 = kw[2 * kk + 1];
              mma_i8_16832<false, true>(acc, qa[kk], low_nibbles_offset(w0), low_nibbles_offset(w1));
              mma_i8_16832<false, false>(acch, qa[KS / 2 + kk], w0 & 0xF0F0F0F0u, w1 & 0xF0F0F0F0u);
            }
            // 16 * (low sum - 8 sum q) + high sum (a multiple of 16); hf carries the 1/16
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[e] = 16 * acc[e] + acch[e];
          }
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int key = r0 + 8 * j + 2 * t + e;
            valid[j][e] = !kMask || (k0 + key) < hi;
            const int si = I4 ? acc[e] * 256 + acc[2 + e] - qbias : acc[e] * 256 + acc[2 + e];
            const float s = float(si) * (__half2float(kst[key]) * hf);
            sc[j][e] = valid[j][e] ? s : -INFINITY;
            mx = fmaxf(mx, sc[j][e]);
          }
        }
        }
        if constexpr (G1) {
          // ---- V fragments: segment sg = bytes 16sg .. 16sg+15 of the 32 keys' rows; thread (g, t)
          // receives bytes 2g, 2g+1 of k-slots 4t+{0,1} (matrix 0), 4t+{2,3} (1), 16+4t+{0,1} (2), 16+4t+{2,3} (3)
          uint32_t vr[NSEG][4];
          const uint32_t vt_s = smem_u32(vt);
#pragma unroll
          for (int sg = 0; sg < NSEG; ++sg)
            ldmatrix_x4_trans(vt_s + (v_row_off ^ uint32_t(sg << 4)), vr[sg][0], vr[sg][1], vr[sg][2], vr[sg][3]);
          const float vs_own = __half2float(vst[own_key]);
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[st]);  // everything this warp needs is in registers

          // ---- frames: a key above m_run + headroom moves the reference maximum, a product
          // p * vs above the fixed-point range (or a full frame) the scale; either ends the frame
          // (lane-local tests and a vote; the warp-wide maxima only when a frame ends)
          if (__any_sync(0xffffffffu, mx > m_run + kG1Headroom)) {
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));  // lane t holds key t's score
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            const float rescale = (m_run == -INFINITY) ? 0.f : ex2(m_run - mx);
            g1_flush<NSEG>(oi, bsum, so, rescale, inv_ps, g, t);
            l_run *= rescale;
            m_run = mx;
            ftiles = 0;
          }
          // this lane's key only (l sums the four lanes per unit)
          const float pr = own_ok ? ex2(own_sc - m_run) : 0.f;
          l_run += pr;
          const float pv_own = own_ok ? pr * vs_own : 0.f;
          float pvm = pv_own;
          if (__any_sync(0xffffffffu, pvm * ps > kG1VLim || (ps == 0.f && pvm > 0.f)) || ftiles >= kG1FrameTiles) {
            pvm = fmaxf(pvm, __shfl_xor_sync(0xffffffffu, pvm, 1));
            pvm = fmaxf(pvm, __shfl_xor_sync(0xffffffffu, pvm, 2));
            pvm = fmaxf(pvm, __shfl_xor_sync(0xffffffffu, pvm, 4));
            pvm = fmaxf(pvm, __shfl_xor_sync(0xffffffffu, pvm, 8));
            pvm = fmaxf(pvm, __shfl_xor_sync(0xffffffffu, pvm, 16));
            g1_flush<NSEG>(oi, bsum, so, 1.f, inv_ps, g, t);
            if (pvm > 0.f) {
              const float pb_ = 1.25f * fmaxf(pvm, 1e-30f);
              ps = kG1VLim / pb_;
              inv_ps = pb_ / kG1VLim;
            }
            ftiles = 0;
          }
          ++ftiles;

          // ---- P in three planes; lane t < 3 packs plane t of its four keys (k-slots 4g + i)
          // and spreads them as the B operand (column c = plane c, c < 3)
          // each lane forms its key's fixed-point word, then every lane gathers the group's four
          const uint32_t fw_own = __float_as_uint(fmaf(pv_own, ps, kG1Magic));
          uint32_t fw[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) fw[i] = __shfl_sync(0xffffffffu, fw_own, (lane & ~3) | i);
          const uint32_t px = __byte_perm(fw[0], fw[1], psel);
          const uint32_t py = __byte_perm(fw[2], fw[3], psel);
          const uint32_t pw = (__byte_perm(px, py, 0x5410u) ^ pxor) & pmask;
          bsum = __dp4a(int(pw), 0x01010101, bsum);
          const uint32_t pb0 = __shfl_sync(0xffffffffu, pw, 4 * t + (g & 3));
          const uint32_t pb1 = __shfl_sync(0xffffffffu, pw, 16 + 4 * t + (g & 3));

          // ---- O^T += V^T P^T on the integer tensor cores: A rows g / g + 8 = bytes 2g / 2g + 1 of
          // the segment, four k-slots per register (byte transposes of the ldmatrix pairs)
#pragma unroll
          for (int sg = 0; sg < NSEG; ++sg) {
            const uint32_t w0 = __byte_perm(vr[sg][0], vr[sg][1], 0x6420u);
            const uint32_t w1 = __byte_perm(vr[sg][0], vr[sg][1], 0x7531u);
            const uint32_t w2 = __byte_perm(vr[sg][2], vr[sg][3], 0x6420u);
            const uint32_t w3 = __byte_perm(vr[sg][2], vr[sg][3], 0x7531u);
            const uint32_t al[4] = {low_nibbles_offset(w0), low_nibbles_offset(w1), low_nibbles_offset(w2),
                                    low_nibbles_offset(w3)};
            const uint32_t ah[4] = {w0 & 0xF0F0F0F0u, w1 & 0xF0F0F0F0u, w2 & 0xF0F0F0F0u, w3 & 0xF0F0F0F0u};
            mma_i8_16832<true, false>(oi[sg], al, pb0, pb1);
            mma_i8_16832<false, false>(oi[NSEG + sg], ah, pb0, pb1);
          }
        } else {
          // ---- V fragments and scales, then release the stage
          uint32_t vw[KP][4][VB / 4];  // per P.V k-step: keys {2t, 2t+1, 2t+8, 2t+9} (t-parity order)
#pragma unroll
          for (int kp = 0; kp < KP; ++kp)
#pragma unroll
            for (int kq = 0; kq < 4; ++kq) {
              const int row = r0 + 16 * kp + 2 * t + ((kq & 1) ^ vsw) + 8 * (kq >> 1);
              lds_words<VB>(vt + tile_off<RB>(row, g * VB), vw[kp][kq]);
            }
          float vs[NJ][2];
#pragma unroll
          for (int j = 0; j < NJ; ++j)
#pragma unroll
            for (int e = 0; e < 2; ++e) vs[j][e] = __half2float(vst[r0 + 8 * j + 2 * t + e]);
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[st]);  // everything this warp needs is in registers

          // ---- online softmax per head g over the KPW keys, and the V-scale frame: one rescale
          // block for both (a head's maximum grew; a key's V scale would push p * vs * vsc past 2^14)
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
          const float m_new = fmaxf(m_run, mx);
          float vmax = 0.f;
#pragma unroll
          for (int j = 0; j < NJ; ++j) {
            if (valid[j][0]) vmax = fmaxf(vmax, vs[j][0]);
            if (valid[j][1]) vmax = fmaxf(vmax, vs[j][1]);
          }
          if (__any_sync(0xffffffffu, m_new > m_run || vmax * vsc > 16384.f)) {
            vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 1));  // keys depend on t only
            vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 2));
            float nk = vk;
            const float nsc = vmax * vsc > 16384.f ? frame_for(vmax, nk) : vsc;  // warp-uniform
            const float ratio = nsc / vsc;  // a power of two: exact
            vsc = nsc;
            vk = nk;
            const float alpha = (m_new == -INFINITY) ? 1.f : ex2(m_run - m_new);
            l_run *= alpha * ratio;
            m_run = m_new;
            // O^T columns are heads 2t, 2t+1; their factors live with g = 2t, 2t+1
            const float a_lo = __shfl_sync(0xffffffffu, alpha, (2 * t) * 4) * ratio;
            const float a_hi = __shfl_sync(0xffffffffu, alpha, (2 * t + 1) * 4) * ratio;
#pragma unroll
            for (int i = 0; i < MT; ++i) {
              o[i][0] *= a_lo;
              o[i][1] *= a_hi;
              o[i][2] *= a_lo;
              o[i][3] *= a_hi;
            }
            pe *= alpha * ratio;  // this lane's head is g
          }
          const float mu = ((m_run == -INFINITY) ? 0.f : m_run) - vk;  // ex2(s - mu) = p * vsc
          uint32_t pb[NJ];
#pragma unroll
          for (int j = 0; j < NJ; ++j) {
            const float p0 = valid[j][0] ? ex2(sc[j][0] - mu) : 0.f;
            const float p1 = valid[j][1] ? ex2(sc[j][1] - mu) : 0.f;
            l_run += p0 + p1;
            pb[j] = pack_half2(valid[j][0] ? p0 * vs[j][0] : 0.f, valid[j][1] ? p1 * vs[j][1] : 0.f);
          }

          // ---- O^T += V^T P^T
#pragma unroll
          for (int kp = 0; kp < KP; ++kp) {
            // m-tile i rows g / g+8: dimensions g*D/8 + i / g*D/8 + MT + i (bytes i / MT + i)
#pragma unroll
            for (int i = 0; i < MT; ++i) {
              const int w0 = i >> 2, w1 = (MT + i) >> 2;
              const uint32_t s0 = uint32_t(i & 3) * 0x1111u + sel_base;
              const uint32_t s1 = uint32_t((MT + i) & 3) * 0x1111u + sel_base;
              const uint32_t a0 = code_pair_offset<kI8A, kI8B>(__byte_perm(vw[kp][0][w0], vw[kp][1][w0], s0));
              const uint32_t a1 = code_pair_offset<kI8A, kI8B>(__byte_perm(vw[kp][0][w1], vw[kp][1][w1], s1));
              const uint32_t a2 = code_pair_offset<kI8A, kI8B>(__byte_perm(vw[kp][2][w0], vw[kp][3][w0], s0));
              const uint32_t a3 = code_pair_offset<kI8A, kI8B>(__byte_perm(vw[kp][2][w1], vw[kp][3][w1], s1));
              mma_16816(o[i], a0, a1, a2, a3, pb[2 * kp], pb[2 * kp + 1]);
            }
            // B holds head g's keys 2t, 2t+1 (pb[2kp]) and 2t+8, 2t+9 (pb[2kp+1]) of the k-step
            add_half2(pe, pb[2 * kp]);
            add_half2(pe, pb[2 * kp + 1]);
          }
        }
      };
      if (k0 + C::TK <= hi) tile(std::false_type{});
      else tile(std::true_type{});
    }

    // ---- unit epilogue: merge the 4 warps' (m, l, O) per head
    if constexpr (G1) {
      // one head: the last frame joins the fp32 O; each lane summed the probabilities of its
      // group's key t, so l is the sum over all lanes
      g1_flush<NSEG>(oi, bsum, so, 1.f, inv_ps, g, t);
      l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);  // the four lanes of a group: one key each
      l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
      l_run += __shfl_xor_sync(0xffffffffu, l_run, 4);
      l_run += __shfl_xor_sync(0xffffffffu, l_run, 8);
      l_run += __shfl_xor_sync(0xffffffffu, l_run, 16);
    } else {
      l_run *= 1.f / vsc;  // leave the V-scale frame (a power of two: exact)
      l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
      l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
    }
    if (t == 0) {
      sm_m[warp * 8 + g] = m_run;
      sm_l[warp * 8 + g] = l_run;
    }
    const int ct = threadIdx.x;
    const size_t row_base = size_t(uc.b) * a.Hq + h0;
    // several heads: 1152 * sum(P) of the heads 2t, 2t + 1 whose columns this thread holds
    float off_lo = 0.f, off_hi = 0.f;
    if constexpr (!G1) {
      pe += __shfl_xor_sync(0xffffffffu, pe, 1);
      pe += __shfl_xor_sync(0xffffffffu, pe, 2);  // head g's sum over the warp's keys
      off_lo = kI8Offset * __shfl_sync(0xffffffffu, pe, (2 * t) * 4);
      off_hi = kI8Offset * __shfl_sync(0xffffffffu, pe, (2 * t + 1) * 4);
    }
    for (int hp = 0; hp < gvalid; hp += MH) {
      if constexpr (!G1) {  // one head: the warp's O is in shared memory already
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int head = 2 * t + e;
          const int gl = head - hp;
          if (gl >= 0 && gl < MH && head < gvalid) {
            // this thread's dimensions g*D/8 .. g*D/8 + D/8 - 1 of the head
            float val[D / 8];
            const float inv_vsc = 1.f / vsc;  // leave the V-scale frame (a power of two: exact)
#pragma unroll
            const float off = e ? off_hi : off_lo;  // the codes' 1152 offset times sum(P) of the head
#pragma unroll
            for (int i = 0; i < MT; ++i) {
              val[i] = (o[i][e] - off) * inv_vsc;
              val[MT + i] = (o[i][2 + e] - off) * inv_vsc;
            }
            float* dst = &sm_o[(warp * MH + gl) * D + g * (D / 8)];
#pragma unroll
            for (int i = 0; i < D / 8; i += 4)
              *reinterpret_cast<float4*>(dst + i) = make_float4(val[i], val[i + 1], val[i + 2], val[i + 3]);
          }
        }
      }
      named_bar_sync(1, 32 * C::kCW);
      const int nh = min(MH, gvalid - hp);
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
          O += wt * sm_o[(w * MH + gl2) * D + d];
        }
        const size_t row = row_base + gg;
        if constexpr (kCl != 0) {  // merged across the cluster below
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
    if constexpr (kCl != 0) {
      // ---- cluster merge: every CTA's (m, l, o) of the unit's heads is in its shared memory;
      // CTA r merges outputs r*128 + ct, r*128 + ct + S*128, ... of the unit's gvalid x D
      // (log-sum-exp weights, an empty split weighs 0) and writes them as fp16.  Every thread
      // of every CTA (the producer warp too) passes both barriers, on every path.
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

template <int D, bool I4, bool G1>
cudaError_t prepare_one(int* ctas_per_sm) {
  const void* fn = reinterpret_cast<const void*>(&decode_qtc_kernel<D, I4, G1>);
  const size_t smem = QtcCfg<D, I4, G1>::kSmemBytes;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(ctas_per_sm, fn, QtcCfg<D, I4, G1>::kThr, smem);
}

template <int D, bool I4, bool G1>
void launch_one(const DecodeLaunch& a, cudaStream_t stream) {
  launch_pdl(decode_qtc_kernel<D, I4, G1>, dim3(a.grid), dim3(QtcCfg<D, I4, G1>::kThr), QtcCfg<D, I4, G1>::kSmemBytes,
             stream, a);
}

// int8 GQA with the split CTAs of a unit merged inside one thread-block cluster.
template <int D, int kCl>
cudaError_t launch_cluster(const DecodeLaunch& a, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.grid);
  cfg.blockDim = dim3(QtcCfg<D, false, false, kCl>::kThr);
  cfg.dynamicSmemBytes = QtcCfg<D, false, false, kCl>::kSmemBytes;
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
  return cudaLaunchKernelEx(&cfg, decode_qtc_kernel<D, false, false, kCl>, a);
}

// Resident clusters of the cluster-merge int8 GQA kernel per cluster size (2..16); both forms run one
// CTA per SM, the two-group one (queried) with more threads and shared memory.
template <int D, int kCl>
cudaError_t prepare_cluster(int (&max_clusters)[17]) {
  const void* fn = reinterpret_cast<const void*>(&decode_qtc_kernel<D, false, false, kCl>);
  const size_t smem = QtcCfg<D, false, false, kCl>::kSmemBytes;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e == cudaSuccess) e = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e != cudaSuccess) return e;
  max_clusters[0] = max_clusters[1] = 0;
  for (int c = 2; c <= kMaxCluster; ++c) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(c);
    cfg.blockDim = dim3(QtcCfg<D, false, false, kCl>::kThr);
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

}  // namespace

// int8 codes reach this kernel only with several query heads per KV head
// (the planner's I8Gqa); int4 codes only with one (the C ABI requires
// Hq == Hkv for int4), which runs the one-head (S^T) variant.
cudaError_t decode_kernel_prepare_qtc(bool int4, int D, int* ctas_per_sm) {
  if (int4) return D == 128 ? prepare_one<128, true, true>(ctas_per_sm) : prepare_one<64, true, true>(ctas_per_sm);
  return D == 128 ? prepare_one<128, false, false>(ctas_per_sm) : prepare_one<64, false, false>(ctas_per_sm);
}

cudaError_t decode_kernel_prepare_qtc_cluster(int D, int (&max_clusters)[17]) {
  cudaError_t e = D == 128 ? prepare_cluster<128, 1>(max_clusters) : prepare_cluster<64, 1>(max_clusters);
  if (e != cudaSuccess) return e;  // the one-group form: attributes only (same residency per SM)
  return D == 128 ? prepare_cluster<128, 2>(max_clusters) : prepare_cluster<64, 2>(max_clusters);
}

cudaError_t launch_decode_qtc(const DecodeLaunch& a, cudaStream_t stream) {
  const bool i4 = a.fmt == KvFormat::I4Tc;
  if (i4 != (a.GP == 1)) return cudaErrorInvalidValue;
  if (a.cluster) {
    if (i4) return cudaErrorInvalidValue;  // only the several-heads variant merges in a cluster
    // one consumer group when each split is one or two tiles, two otherwise
    const bool two = a.chunk > 2 * (a.D == 128 ? QtcCfg<128, false, false, 2>::TK : QtcCfg<64, false, false, 2>::TK);
    if (a.D == 128) return two ? launch_cluster<128, 2>(a, stream) : launch_cluster<128, 1>(a, stream);
    return two ? launch_cluster<64, 2>(a, stream) : launch_cluster<64, 1>(a, stream);
  }
  if (i4) {
    if (a.D == 128) launch_one<128, true, true>(a, stream);
    else launch_one<64, true, true>(a, stream);
  } else {
    if (a.D == 128) launch_one<128, false, false>(a, stream);
    else launch_one<64, false, false>(a, stream);
  }
  return cudaGetLastError();
}

}  // namespace fqkv
