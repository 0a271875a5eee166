// int8-KV and int4-KV single-query decode attention, sm_100a.
//
// Replaces decode_attn_int8_mw_kernel (kernels/decode_attn_int8_mw.cu:6-51)
// and decode_attn_int4_kernel (kernels/decode_attn_int4.cu:8-46); int4 is
// generalised from the reference's D=64 to D in {64, 128}.
//
// Layout in HBM (exactly the reference's): codes [R, N, D] int8 or packed
// [R, N, D/2] uint8 (element 2t in the low nibble), scales [R, N] fp16.
//
//  * Persistent, warp-specialised: warp 4 streams 16 KiB (int4 at D = 64:
//    8 KiB) tiles of K and V codes plus the matching scale windows into a
//    3-stage (4-stage) ring with 1-D bulk copies (cp.async.bulk) completing
//    on mbarriers.  A scale window starts at
//    the 16-byte boundary at or below the tile's first scale, so it may read up
//    to 15 bytes on either side of the scale array -- always inside the
//    16-byte blocks that hold the first / last scale, never used.
//  * Each consumer warp owns a quarter of every tile.  A key row is split into
//    32-byte chunks, one per lane (L = row_bytes/32 lanes per key: 64 int4 or
//    32 int8 dims per lane, so the per-key work -- score reduction, softmax,
//    scale loads -- is shared by many elements; int4 at D = 64 uses 16-byte
//    chunks, two lanes per key, for occupancy), and every lane handles 4 keys
//    per tile.  Full tiles skip the per-key bounds masks.
//  * q . k on integer dot-product units: q is held as a 2-plane fixed-point
//    number (q * 2^e = hi * 256 + lo, hi signed byte, lo unsigned byte, 14
//    significant bits -- every fp16 q within 3 binades of max|q| is exact).
//    int8 codes enter dp4a directly; int4 nibbles enter as unsigned
//    (code + 8) bytes after one xor-and, and the +8 is removed once per unit.
//    The score is (integer dot) * k_scale * (log2(e) / sqrt(D)) / 2^e.
//  * p . v in fp32: codes become exact fp16 subnormal pairs in offset binary
//    ((code + 128) * 2^-24 for int8, s * (code + 8) * 2^-24 for int4 nibbles,
//    s = 1 or 16; one byte-permute or one logic op per pair) and are
//    accumulated with the mixed-precision f16 x f16 + f32 FMA, which takes
//    subnormal operands at full speed; the V scale is folded into p, and the
//    offset leaves once per unit through per-lane sums of the same fp16 p.
//  * Online softmax in the log2 domain, warp merge through shared memory,
//    output fp16 or an fp32 split partial like the fp16 kernel.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <type_traits>

#include "device_common.cuh"
#include "kernels.h"

namespace fqkv {
namespace {

constexpr int kConsumerWarps = 4;
constexpr int kThreads = 32 * (kConsumerWarps + 1);

template <bool kInt4, int D>
struct QCfg {
  static constexpr int kRowBytes = kInt4 ? D / 2 : D;
  // Bytes of a key row per lane: 32 (int8: 32 dims, int4 at D = 128: 64 dims).  int4 at
  // D = 64 splits its 32-byte rows over two lanes of 16 bytes (32 dims): half the
  // accumulators and q planes per lane, so four CTAs fit per SM instead of two (the
  // one-lane-per-key form was latency-bound: 0.84 eligible warps per scheduler).
  static constexpr int kLaneBytes = (kInt4 && D == 64) ? 16 : 32;
  static constexpr int kL = kRowBytes / kLaneBytes;        // lanes per key row
  static constexpr int kKPS = 32 / kL;                     // keys per warp step
  static constexpr int kTK = 4 * kConsumerWarps * kKPS;    // keys per tile: 4 per lane
  static constexpr int kTileBytes = kTK * kRowBytes;       // K (or V) codes of one tile (16 or 8 KiB)
  static constexpr int kDimsPerLane = kInt4 ? 2 * kLaneBytes : kLaneBytes;
  static constexpr int kWords = kLaneBytes / 4;            // 32-bit words per lane chunk
  // 16 KiB tiles: a 3-stage ring, 2 CTAs per SM.  8 KiB tiles (int4, D = 64): 3 stages and 4 CTAs
  // per SM (96 registers, no spills): the kernel is issue- and latency-bound, so 16 consumer warps
  // per SM beat 12 with a deeper ring (481 -> 466 us at R=8192, N=4096 on one box; 5 CTAs with
  // 2 stages spill 192 bytes and ran 526 us)
  static constexpr int kStages = 3;
  static constexpr int kMinBlocks = kTileBytes == 16384 ? 2 : 4;
  static constexpr int kScaleBytes = 2 * kTK + 32;         // scale window capacity
  static constexpr int kStageBytes = 2 * kTileBytes + 2 * kScaleBytes;
  static constexpr size_t kSmemBytes = 128 + size_t(kStages) * kStageBytes + 2 * kStages * sizeof(uint64_t) +
                                       size_t(kConsumerWarps) * (2 + D) * sizeof(float);
  static_assert(kTileBytes == 16384 || kTileBytes == 8192, "tile size");
};

// The kLaneBytes (16 or 32) bytes of a key row this lane handles, from shared memory.
template <int kLaneBytes>
__device__ __forceinline__ void lane_words(const uint8_t* p, uint32_t* w) {
  const uint4 a = *reinterpret_cast<const uint4*>(p);
  w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
  if constexpr (kLaneBytes == 32) {
    const uint4 b = *reinterpret_cast<const uint4*>(p + 16);
    w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
  }
}

// fp32 accumulate of p (fp16) times both halves of an fp16 pair:
// lo += p * v.lo, hi += p * v.hi, with the sm_100 mixed-precision FMA.
__device__ __forceinline__ void fma_pair(float& lo, float& hi, uint32_t v2, uint16_t p) {
  asm("{\n\t.reg .f16 a, b;\n\tmov.b32 {a, b}, %2;\n\t"
      "fma.rn.f32.f16 %0, %3, a, %0;\n\tfma.rn.f32.f16 %1, %3, b, %1;\n\t}"
      : "+f"(lo), "+f"(hi)
      : "r"(v2), "h"(p));
}

// acc += h (an fp16 value), one mixed-precision FMA by 1.0
__device__ __forceinline__ void add_half(float& acc, uint16_t h) {
  asm("{\n\t.reg .f16 one;\n\tmov.b16 one, 0x3C00;\n\tfma.rn.f32.f16 %0, %1, one, %0;\n\t}" : "+f"(acc) : "h"(h));
}

// dp4a with a signed-byte first operand and unsigned-byte second operand,
// and with both unsigned.
__device__ __forceinline__ int dp4a_su(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_uu(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

template <bool kInt4, int D>
__global__ void __launch_bounds__(kThreads, QCfg<kInt4, D>::kMinBlocks)
    decode_quant_kernel(const __grid_constant__ DecodeLaunch a) {
  using C = QCfg<kInt4, D>;
  constexpr int kStages = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  // aligned by an offset from the shared array, so that every access through `smem` stays a
  // shared-memory access (an integer round trip of the pointer would make them generic)
  uint8_t* smem = smem_raw + ((uint32_t(128) - (smem_u32(smem_raw) & 127u)) & 127u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + size_t(kStages) * C::kStageBytes);
  uint64_t* empty = full + kStages;
  float* sm_ml = reinterpret_cast<float*>(empty + kStages);  // [warps][2]
  float* sm_o = sm_ml + 2 * kConsumerWarps;                   // [warps][D]
  __shared__ int abort_flag;
  __shared__ int stage_off[kStages][2];                       // scale offsets (elements) in each window

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const WaitCtl wc{a.status, a.timeout_ns};
  const size_t row_stride = size_t(a.kv_stride) * C::kRowBytes;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  pdl_launch_dependents();
  // Valid keys: the launch's N, or the device-side length of a growing cache.
  // Launched with programmatic serialization: wait for the previous kernel on
  // the stream (and its memory) before reading any input.
  pdl_wait_primary();
  const int n_valid = a.n_dev ? min(a.N, *a.n_dev) : a.N;

  // ------------------------------------------------------------ producer
  if (warp == kConsumerWarps) {
    if (lane != 0 || a.debug_skip_loads) return;
    int it = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < a.units && ok; u += gridDim.x) {
      const int s = u % a.S_eff;
      const int r = u / a.S_eff;  // row = b * Hkv + kh (Hq == Hkv here)
      const int lo = s * a.chunk;
      const int hi = min(n_valid, lo + a.chunk);
      const uint8_t* Kr = static_cast<const uint8_t*>(a.K) + size_t(r) * row_stride;
      const uint8_t* Vr = static_cast<const uint8_t*>(a.V) + size_t(r) * row_stride;
      const __half* Ksr = static_cast<const __half*>(a.Ks) + size_t(r) * a.kv_stride;
      const __half* Vsr = static_cast<const __half*>(a.Vs) + size_t(r) * a.kv_stride;
      for (int k0 = lo; k0 < hi; k0 += C::kTK, ++it) {
        const int st = it % kStages;
        if (it >= kStages) {
          if (*reinterpret_cast<volatile int*>(&abort_flag) ||
              !mbar_wait(&empty[st], ((it / kStages) - 1) & 1, wc, kDevTimeoutEmpty)) {
            ok = false;
            break;
          }
        }
        const int nk = min(C::kTK, hi - k0);
        const uint32_t kv_bytes = uint32_t(nk) * C::kRowBytes;
        const uintptr_t ka = reinterpret_cast<uintptr_t>(Ksr + k0);
        const uintptr_t va = reinterpret_cast<uintptr_t>(Vsr + k0);
        const uintptr_t ka0 = ka & ~uintptr_t(15), va0 = va & ~uintptr_t(15);
        const uint32_t kwin = uint32_t(((ka + 2u * nk + 15u) & ~uintptr_t(15)) - ka0);
        const uint32_t vwin = uint32_t(((va + 2u * nk + 15u) & ~uintptr_t(15)) - va0);
        stage_off[st][0] = int(ka - ka0) >> 1;
        stage_off[st][1] = int(va - va0) >> 1;
        uint8_t* base = smem + size_t(st) * C::kStageBytes;
        // expect_tx has release semantics: the stage_off stores above are
        // visible to consumers that acquire the completed phase.
        mbar_arrive_expect_tx(&full[st], 2 * kv_bytes + kwin + vwin);
        bulk_g2s(base, Kr + size_t(k0) * C::kRowBytes, kv_bytes, &full[st]);
        bulk_g2s(base + C::kTileBytes, Vr + size_t(k0) * C::kRowBytes, kv_bytes, &full[st]);
        bulk_g2s(base + 2 * C::kTileBytes, reinterpret_cast<const void*>(ka0), kwin, &full[st]);
        bulk_g2s(base + 2 * C::kTileBytes + C::kScaleBytes, reinterpret_cast<const void*>(va0), vwin, &full[st]);
      }
    }
    if (!ok) {
      for (int j = (it > kStages ? it - kStages : 0); j < it; ++j)
        mbar_wait(&full[j % kStages], (j / kStages) & 1, wc, kDevTimeoutDrain);
    }
    return;
  }

  // ------------------------------------------------------------ consumers
  constexpr int kDPL = C::kDimsPerLane;
  constexpr bool kPairSplit = kInt4 && C::kL == 2;  // int4 at D = 64: two lanes per key row
  constexpr int kPW = kInt4 ? 2 * C::kWords : C::kWords;  // q plane words per lane
  const int c = lane % C::kL;          // 32-byte chunk of the key row
  const int j = lane / C::kL;          // key slot
  const int kw = warp * (C::kTK / kConsumerWarps);
  bool alive = true;
  int it = 0;

  for (int u = blockIdx.x; u < a.units; u += gridDim.x) {
    const int s = u % a.S_eff;
    const int r = u / a.S_eff;
    const int lo = s * a.chunk;
    const int hi = min(n_valid, lo + a.chunk);

    // ---- q as 2-plane fixed point for this lane's dims.  e is chosen from
    // max|q| over the whole row (the L lanes of one key slot cover all D dims)
    // so that |q| * 2^e < 2^14; the score factor undoes 2^e (and the 16 of the
    // int4 odd-nibble bytes).
    uint32_t qh[kPW], ql[kPW];
    float qscale_unit;
    int qbias = 0;
    {
      float qv[kDPL];
      const __half* qrow = static_cast<const __half*>(a.q) + size_t(r) * D + c * kDPL;
      float mq = 0.f;
#pragma unroll
      for (int d = 0; d < kDPL; ++d) {
        qv[d] = __half2float(qrow[d]);
        mq = fmaxf(mq, fabsf(qv[d]));
      }
#pragma unroll
      for (int off = 1; off < C::kL; off <<= 1) mq = fmaxf(mq, __shfl_xor_sync(0xffffffffu, mq, off));
      const int e = (mq > 0.f) ? 13 - ilogbf(mq) : 0;
      const float two_e = ldexpf(1.f, e);
#pragma unroll
      for (int d = 0; d < kDPL; ++d) qv[d] = rintf(qv[d] * two_e);  // |.| <= 16384
      qscale_unit = a.sm_scale_log2 * ldexpf(1.f, -e) * (kInt4 ? 0.0625f : 1.f);
      if (kInt4) {
        // int4 codes enter dp4a as unsigned (code + 8): remove 8 * 16 * sum(q)
#pragma unroll
        for (int d = 0; d < kDPL; ++d) qbias += int(qv[d]);
        qbias *= 128;
      }
      // planes: int8 -> word w covers dims 4w..4w+3; int4 -> word w covers
      // dims 8w..8w+7 split into even and odd dims (index 2w + parity).
#pragma unroll
      for (int w = 0; w < C::kWords; ++w) {
        if (kInt4) {
#pragma unroll
          for (int par = 0; par < 2; ++par) {
            uint32_t hw = 0, lw = 0;
#pragma unroll
            for (int bb = 0; bb < 4; ++bb) {
              const int qi = int(qv[8 * w + 2 * bb + par]);
              hw |= (uint32_t(qi >> 8) & 0xFFu) << (8 * bb);
              lw |= (uint32_t(qi) & 0xFFu) << (8 * bb);
            }
            qh[(2 * w + par) % kPW] = hw;
            ql[(2 * w + par) % kPW] = lw;
          }
        } else {
          uint32_t hw = 0, lw = 0;
#pragma unroll
          for (int bb = 0; bb < 4; ++bb) {
            const int qi = int(qv[(4 * w + bb) % kDPL]);
            hw |= (uint32_t(qi >> 8) & 0xFFu) << (8 * bb);
            lw |= (uint32_t(qi) & 0xFFu) << (8 * bb);
          }
          qh[w % kPW] = hw;
          ql[w % kPW] = lw;
        }
      }
    }

    float o[kDPL];
#pragma unroll
    for (int d = 0; d < kDPL; ++d) o[d] = 0.f;
    float m_run = -INFINITY, l_run = 0.f;
    // sums of the fp16 p (int8 codes, int4 low nibbles) and p / 16 (int4 high nibbles) this
    // lane multiplied, for the offset of the subnormal code fields (see the P.V step)
    float bias_lo = 0.f, bias_hi = 0.f;
    // p * vscale enters the fp16 FMA operand multiplied by vsc = 2^vk, a warp-uniform power of two
    // that keeps it in fp16's normal range: vsc is lowered (o, l and the bias sums rescaled
    // exactly) whenever a key's V scale passes vthr = 2^14 / vsc, so p * vscale * vsc <= 2^14
    // (p <= 1), and otherwise stays as large as the largest V scale so far allows -- a small V
    // (|V| ~ 1e-4) no longer rounds to fp16 subnormals.  The frame costs nothing per key: it is
    // folded into the exponent, ex2(s - (m - vk)) = p * vsc, and l sums the same scaled values;
    // the lane's o and l leave the frame (/ vsc) before the cross-lane reduction.
    float vsc = 1099511627776.f, vk = 40.f;  // 2^40: any nonzero fp16 V scale lowers it on its first tile
    float vthr = 1.4901161193847656e-8f;     // 2^14 / vsc = 2^-26

    // int4 at D = 64: the two lanes of a key row split the per-key scalar work -- lane c scales,
    // exponentiates and packs the probabilities of its keys sp = c and c + 2 of the four, and the
    // pair trades the partial dot products and the packed fp16 (p, p/16) by shuffles; l and the
    // offset sums then cover only a lane's own keys and are added across the pair per unit.
    auto tile_pair = [&](const uint8_t* base, int st, int k0, auto mask_tag) {
      constexpr bool kMask = decltype(mask_tag)::value;
      const uint8_t* kt = base;
      const uint8_t* vt = base + C::kTileBytes;
      const __half* kst = reinterpret_cast<const __half*>(base + 2 * C::kTileBytes) + stage_off[st][0];
      const __half* vst = reinterpret_cast<const __half*>(base + 2 * C::kTileBytes + C::kScaleBytes) + stage_off[st][1];
      float vso[2];  // V scales of this lane's own keys (sp = 2i + c)
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int kl = kw + j + C::kKPS * (2 * i + c);
        vso[i] = (!kMask || (k0 + kl) < hi) ? __half2float(vst[kl]) : 0.f;
      }
      float vmax = fmaxf(vso[0], vso[1]);
      int accp[4];  // this lane's half of every key's integer dot product
#pragma unroll
      for (int sp = 0; sp < 4; ++sp) {
        const int kl = kw + j + C::kKPS * sp;
        uint32_t kwd[C::kWords];
        lane_words<C::kLaneBytes>(kt + kl * C::kRowBytes + C::kLaneBytes * c, kwd);
        int ahe = 0, aho = 0, ale = 0, alo = 0;
#pragma unroll
        for (int w = 0; w < C::kWords; ++w) {
          const uint32_t ev = xor_and<0x88888888u, 0x0F0F0F0Fu>(kwd[w]);  // (code + 8) of even dims
          const uint32_t od = xor_and<0x88888888u, 0xF0F0F0F0u>(kwd[w]);  // 16 * (code + 8) of odd dims
          ahe = dp4a_su(qh[(2 * w) % kPW], ev, ahe);
          aho = dp4a_su(qh[(2 * w + 1) % kPW], od, aho);
          ale = dp4a_uu(ql[(2 * w) % kPW], ev, ale);
          alo = dp4a_uu(ql[(2 * w + 1) % kPW], od, alo);
        }
        accp[sp] = (ahe * 16 + aho) * 256 + (ale * 16 + alo) - qbias;
      }
      float sco[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        // one shuffle per two keys: each lane sends its half of the partner's own key
        const int recv = __shfl_xor_sync(0xffffffffu, c ? accp[2 * i] : accp[2 * i + 1], 1);
        const int acc = (c ? accp[2 * i + 1] : accp[2 * i]) + recv;
        const int kl = kw + j + C::kKPS * (2 * i + c);
        const float sv = float(acc) * (__half2float(kst[kl]) * qscale_unit);
        sco[i] = (!kMask || (k0 + kl) < hi) ? sv : -INFINITY;
      }
      float mx = fmaxf(sco[0], sco[1]);
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_new = fmaxf(m_run, mx);
      if (__any_sync(0xffffffffu, m_new > m_run || vmax > vthr)) {
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, off));
        const bool grow_v = vmax > vthr;  // rare: the V frame must move down
        const float alpha = m_new > m_run ? ex2(m_run - m_new) : 1.f;
        float nk = vk;
        const float nsc = grow_v ? frame_for(vmax, nk) : vsc;
        const float f = alpha * (nsc / vsc);  // the frame ratio is a power of two: exact
#pragma unroll
        for (int d = 0; d < kDPL; ++d) o[d] *= f;
        l_run *= f;
        bias_lo *= f;
        bias_hi *= f;
        m_run = m_new;
        vsc = nsc;
        vk = nk;
        vthr = 16384.f / nsc;  // a power of two: exact
      }
      const float mu = ((m_run == -INFINITY) ? 0.f : m_run) - vk;  // ex2(s - mu) = p * vsc
      uint32_t pw[2];  // own keys: fp16 p * vscale (low half) and p * vscale / 16 (high half)
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const float p = ex2(sco[i] - mu);
        l_run += p;
        const float pv = p * vso[i];
        const uint16_t ph = __half_as_ushort(__float2half_rn(pv));
        const uint16_t ph16 = __half_as_ushort(__float2half_rn(pv * 0.0625f));
        add_half(bias_lo, ph);
        add_half(bias_hi, ph16);
        pw[i] = uint32_t(ph) | (uint32_t(ph16) << 16);
      }
      const uint32_t pr[2] = {__shfl_xor_sync(0xffffffffu, pw[0], 1), __shfl_xor_sync(0xffffffffu, pw[1], 1)};
#pragma unroll
      for (int sp = 0; sp < 4; ++sp) {
        const int kl = kw + j + C::kKPS * sp;
        const int i = sp >> 1;
        const uint32_t pk = ((sp & 1) == c) ? pw[i] : pr[i];
        const uint16_t ph = uint16_t(pk & 0xFFFFu), ph16 = uint16_t(pk >> 16);
        uint32_t vwd[C::kWords];
        lane_words<C::kLaneBytes>(vt + kl * C::kRowBytes + C::kLaneBytes * c, vwd);
        // nibble fields as in the tile below: offset-binary fp16 subnormals, p/16 with the s = 16 halves
#pragma unroll
        for (int w = 0; w < C::kWords; ++w) {
          const uint32_t x = vwd[w];
          const uint32_t y = x >> 8;
          const uint32_t a04 = xor_and<0x00080008u, 0x000F000Fu>(x);
          const uint32_t a15 = xor_and<0x00800080u, 0x00F000F0u>(x);
          const uint32_t a26 = xor_and<0x00080008u, 0x000F000Fu>(y);
          const uint32_t a37 = xor_and<0x00800080u, 0x00F000F0u>(y);
          float* od = &o[(8 * w) % kDPL];
          fma_pair(od[0], od[4], a04, ph);
          fma_pair(od[1], od[5], a15, ph16);
          fma_pair(od[2], od[6], a26, ph);
          fma_pair(od[3], od[7], a37, ph16);
        }
      }
    };

    // One tile of this warp's keys; kMask adds the per-key bound checks that
    // only the last (partial) tile of a unit needs.
    auto tile = [&](const uint8_t* base, int st, int k0, auto mask_tag) {
      constexpr bool kMask = decltype(mask_tag)::value;
      const uint8_t* kt = base;
      const uint8_t* vt = base + C::kTileBytes;
      const __half* kst = reinterpret_cast<const __half*>(base + 2 * C::kTileBytes) + stage_off[st][0];
      const __half* vst = reinterpret_cast<const __half*>(base + 2 * C::kTileBytes + C::kScaleBytes) + stage_off[st][1];
      // the V scales of this lane's four keys first, so that the frame test below does not wait
      // for their loads
      float vs4[4];
#pragma unroll
      for (int sp = 0; sp < 4; ++sp) {
        const int kl = kw + j + C::kKPS * sp;
        vs4[sp] = (!kMask || (k0 + kl) < hi) ? __half2float(vst[kl]) : 0.f;
      }
      float vmax = fmaxf(fmaxf(vs4[0], vs4[1]), fmaxf(vs4[2], vs4[3]));
      float sco[4];
#pragma unroll
      for (int sp = 0; sp < 4; ++sp) {
        const int kl = kw + j + C::kKPS * sp;
        uint32_t kwd[C::kWords];
        lane_words<C::kLaneBytes>(kt + kl * C::kRowBytes + C::kLaneBytes * c, kwd);
        int acc;
        if (kInt4) {
          int ahe = 0, aho = 0, ale = 0, alo = 0;
#pragma unroll
          for (int w = 0; w < C::kWords; ++w) {
            const uint32_t ev = xor_and<0x88888888u, 0x0F0F0F0Fu>(kwd[w]);  // (code + 8) of even dims
            const uint32_t od = xor_and<0x88888888u, 0xF0F0F0F0u>(kwd[w]);  // 16 * (code + 8) of odd dims
            ahe = dp4a_su(qh[(2 * w) % kPW], ev, ahe);
            aho = dp4a_su(qh[(2 * w + 1) % kPW], od, aho);
            ale = dp4a_uu(ql[(2 * w) % kPW], ev, ale);
            alo = dp4a_uu(ql[(2 * w + 1) % kPW], od, alo);
          }
          acc = (ahe * 16 + aho) * 256 + (ale * 16 + alo) - qbias;
        } else {
          int ah = 0, al = 0;
#pragma unroll
          for (int w = 0; w < C::kWords; ++w) {
            ah = dp4a_ss(qh[w % kPW], kwd[w], ah);
            al = dp4a_us(ql[w % kPW], kwd[w], al);
          }
          acc = ah * 256 + al;
        }
#pragma unroll
        for (int off = 1; off < C::kL; off <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
        const float sv = float(acc) * (__half2float(kst[kl]) * qscale_unit);
        sco[sp] = (!kMask || (k0 + kl) < hi) ? sv : -INFINITY;
      }
      float mx = fmaxf(fmaxf(sco[0], sco[1]), fmaxf(sco[2], sco[3]));
#pragma unroll
      for (int off = C::kL; off < 32; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_new = fmaxf(m_run, mx);
      // one warp-uniform rescale block for both causes (a larger running maximum; a V scale above
      // the frame's threshold), so the loop carries one copy of the per-dimension multiply
      if (__any_sync(0xffffffffu, m_new > m_run || vmax > vthr)) {
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, off));
        const bool grow_v = vmax > vthr;  // rare: the V frame must move down
        const float alpha = m_new > m_run ? ex2(m_run - m_new) : 1.f;
        float nk = vk;
        const float nsc = grow_v ? frame_for(vmax, nk) : vsc;
        const float f = alpha * (nsc / vsc);  // the frame ratio is a power of two: exact
#pragma unroll
        for (int d = 0; d < kDPL; ++d) o[d] *= f;
        l_run *= f;
        bias_lo *= f;
        bias_hi *= f;
        m_run = m_new;
        vsc = nsc;
        vk = nk;
        vthr = 16384.f / nsc;  // a power of two: exact
      }
      const float mu = ((m_run == -INFINITY) ? 0.f : m_run) - vk;  // ex2(s - mu) = p * vsc
#pragma unroll
      for (int sp = 0; sp < 4; ++sp) {
        const int kl = kw + j + C::kKPS * sp;
        const float p = ex2(sco[sp] - mu);
        l_run += p;
        const float pv = p * vs4[sp];
        const uint16_t ph = __half_as_ushort(__float2half_rn(pv));
        uint32_t vwd[C::kWords];
        lane_words<C::kLaneBytes>(vt + kl * C::kRowBytes + C::kLaneBytes * c, vwd);
        if (kInt4) {
          // nibble n of word w is dim 8w + n.  One logic op leaves the nibble pair
          // (n, n+4) in offset binary as fp16 subnormals
          // s*(code+8) * 2^-24, s = 1 or 16 (exact; the FMA takes them as they are); p/16 pairs with the
          // s = 16 halves.  The offset, 8 * 2^-24 * sum(p) per dimension, leaves
          // once per unit through bias_lo / bias_hi.
          const uint16_t ph16 = __half_as_ushort(__float2half_rn(pv * 0.0625f));
          add_half(bias_lo, ph);
          add_half(bias_hi, ph16);
#pragma unroll
          for (int w = 0; w < C::kWords; ++w) {
            // each field to offset binary in one logic op (xor and mask with register constants)
            const uint32_t x = vwd[w];
            const uint32_t y = x >> 8;
            const uint32_t a04 = xor_and<0x00080008u, 0x000F000Fu>(x);
            const uint32_t a15 = xor_and<0x00800080u, 0x00F000F0u>(x);
            const uint32_t a26 = xor_and<0x00080008u, 0x000F000Fu>(y);
            const uint32_t a37 = xor_and<0x00800080u, 0x00F000F0u>(y);
            float* od = &o[(8 * w) % kDPL];
            fma_pair(od[0], od[4], a04, ph);
            fma_pair(od[1], od[5], a15, ph16);
            fma_pair(od[2], od[6], a26, ph);
            fma_pair(od[3], od[7], a37, ph16);
          }
        } else {
          // bytes (code + 128) become the fp16 subnormal pairs (code + 128) * 2^-24
          // with one byte-permute per pair (exact; the FMA takes them as they
          // are); the offset, 128 * 2^-24 * sum(p), leaves once per unit.
          add_half(bias_lo, ph);
#pragma unroll
          for (int w = 0; w < C::kWords; ++w) {
            const uint32_t x = vwd[w] ^ 0x80808080u;
            const uint32_t a01 = __byte_perm(x, 0u, 0x4140u);
            const uint32_t a23 = __byte_perm(x, 0u, 0x4342u);
            fma_pair(o[(4 * w) % kDPL], o[(4 * w + 1) % kDPL], a01, ph);
            fma_pair(o[(4 * w + 2) % kDPL], o[(4 * w + 3) % kDPL], a23, ph);
          }
        }
      }
    };

    for (int k0 = lo; k0 < hi; k0 += C::kTK, ++it) {
      const int st = it % kStages;
      if (alive) {
        bool ok = mbar_wait(&full[st], (it / kStages) & 1, wc, kDevTimeoutFull) &&
                  !*reinterpret_cast<volatile int*>(&abort_flag);
        alive = __all_sync(0xffffffffu, ok);
        if (!alive && lane == 0) abort_flag = 1;
      }
      if (!alive) continue;
      const uint8_t* base = smem + size_t(st) * C::kStageBytes;
      if constexpr (kPairSplit) {
        if (k0 + C::kTK <= hi) tile_pair(base, st, k0, std::false_type{});
        else tile_pair(base, st, k0, std::true_type{});
      } else {
        if (k0 + C::kTK <= hi) tile(base, st, k0, std::false_type{});
        else tile(base, st, k0, std::true_type{});
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }

    if constexpr (kPairSplit) {  // l and the offset sums covered this lane's own keys only
      l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
      bias_lo += __shfl_xor_sync(0xffffffffu, bias_lo, 1);
      bias_hi += __shfl_xor_sync(0xffffffffu, bias_hi, 1);
    }
    // scale the subnormal fields back, remove their offset (int4: + 8; int8: + 128) and leave
    // the lane's V-scale frame
    const float inv_vsc = 1.f / vsc;  // a power of two: exact
    l_run *= inv_vsc;
    if (kInt4) {
#pragma unroll
      for (int d = 0; d < kDPL; ++d)
        o[d] = fmaf(o[d], 16777216.f, -8.f * ((d & 1) ? 16.f * bias_hi : bias_lo)) * inv_vsc;
    } else {
#pragma unroll
      for (int d = 0; d < kDPL; ++d) o[d] = fmaf(o[d], 16777216.f, -128.f * bias_lo) * inv_vsc;
    }

    // ---- warp reduction over key slots, then merge the 4 warps
#pragma unroll
    for (int off = C::kL; off < 32; off <<= 1) {
      l_run += __shfl_xor_sync(0xffffffffu, l_run, off);
#pragma unroll
      for (int d = 0; d < kDPL; ++d) o[d] += __shfl_xor_sync(0xffffffffu, o[d], off);
    }
    if (lane == 0) {
      sm_ml[2 * warp] = m_run;
      sm_ml[2 * warp + 1] = l_run;
    }
    if (j == 0) {
#pragma unroll
      for (int d = 0; d < kDPL; d += 4)
        *reinterpret_cast<float4*>(&sm_o[warp * D + c * kDPL + d]) = make_float4(o[d], o[d + 1], o[d + 2], o[d + 3]);
    }
    named_bar_sync(1, 32 * kConsumerWarps);
    const int ct = threadIdx.x;
    if (ct < D) {
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, sm_ml[2 * w]);
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        const float mw = sm_ml[2 * w];
        const float wt = (mw == -INFINITY) ? 0.f : ex2(mw - M);
        L += wt * sm_ml[2 * w + 1];
        O += wt * sm_o[w * D + ct];
      }
      if (a.S_eff == 1) {
        store_out(a, size_t(r) * D + ct, O / L);
      } else {
        const size_t slot = size_t(r) * a.S + s;
        if (ct == 0) {
          a.part_m[slot] = M;
          a.part_l[slot] = L;
        }
        a.part_o[slot * D + ct] = O;
      }
    }
    named_bar_sync(1, 32 * kConsumerWarps);
    if (a.S_eff == 1) signal_out(a, ct, 1, 32 * kConsumerWarps);
  }
}

template <bool kInt4, int D>
const void* qfn() {
  return reinterpret_cast<const void*>(&decode_quant_kernel<kInt4, D>);
}

const void* quant_fn(bool int4, int D) {
  if (int4) return D == 128 ? qfn<true, 128>() : qfn<true, 64>();
  return D == 128 ? qfn<false, 128>() : qfn<false, 64>();
}

size_t quant_smem(bool int4, int D) {
  if (int4) return D == 128 ? QCfg<true, 128>::kSmemBytes : QCfg<true, 64>::kSmemBytes;
  return D == 128 ? QCfg<false, 128>::kSmemBytes : QCfg<false, 64>::kSmemBytes;
}

}  // namespace

KernelShape decode_kernel_shape_quant(bool int4, int D) { return KernelShape{kThreads, quant_smem(int4, D)}; }

cudaError_t decode_kernel_prepare_quant(bool int4, int D, int* ctas_per_sm) {
  const void* fn = quant_fn(int4, D);
  const size_t smem = quant_smem(int4, D);
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(ctas_per_sm, fn, kThreads, smem);
}

cudaError_t launch_decode_quant(const DecodeLaunch& a, cudaStream_t stream) {
  const bool int4 = a.fmt == KvFormat::I4;
  const size_t smem = quant_smem(int4, a.D);
  if (int4) {
    if (a.D == 128) launch_pdl(decode_quant_kernel<true, 128>, dim3(a.grid), dim3(kThreads), smem, stream, a);
    else launch_pdl(decode_quant_kernel<true, 64>, dim3(a.grid), dim3(kThreads), smem, stream, a);
  } else {
    if (a.D == 128) launch_pdl(decode_quant_kernel<false, 128>, dim3(a.grid), dim3(kThreads), smem, stream, a);
    else launch_pdl(decode_quant_kernel<false, 64>, dim3(a.grid), dim3(kThreads), smem, stream, a);
  }
  return cudaGetLastError();
}

}  // namespace fqkv
