// Internal interface between the C-ABI layer (capi.cu) and the kernel
// translation units.  Host-only types: plain pointers, sizes and a stream.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace fqkv {

// I8Gqa / I4Tc: int8 codes with more than one query head per KV head, and
// int4 codes, on the tensor-core quantized kernel (attn_qtc.cu); chosen by the
// planner, never passed in by callers.
enum class KvFormat : int { F16 = 0, I8 = 1, I4 = 2, I8Gqa = 3, I4Tc = 4 };

// Bytes of one key row of K (or V) in HBM.
constexpr int64_t kv_row_bytes(KvFormat f, int64_t D) {
  return f == KvFormat::F16 ? 2 * D : ((f == KvFormat::I8 || f == KvFormat::I8Gqa) ? D : D / 2);
}

// Keys per pipeline stage (one tile).  The fp16 kernel uses 64-key tiles of
// 128-byte swizzled rows; the tensor-core quantized kernel 64 (int8, D = 128)
// or 128 keys (16 or 32 per consumer warp); the CUDA-core quantized kernel
// 16 KiB tiles of K (and V).
constexpr int tile_keys(KvFormat f, int64_t D) {
  return f == KvFormat::F16     ? 64
         : f == KvFormat::I8Gqa ? (D == 128 ? 64 : 128)
         : f == KvFormat::I4Tc  ? 128
                                : static_cast<int>(16384 / kv_row_bytes(f, D));
}

// Tensor-parallel output: instead of `out`, the final fp16 output is stored at
// dst[p] + dst_off (+ the row offset) for every rank p < world, and each unit
// of output counts one arrival on cnt[p][rank].  world == 0: plain output.
constexpr int kTpMaxRanks = 8;
struct TpOut {
  int world;
  int rank;
  long long dst_off;
  __half_raw* dst[kTpMaxRanks];
  unsigned long long* cnt[kTpMaxRanks];
};

// One decode-attention launch, in the library's canonical form:
//   q [B, Hq, D] fp16, K/V [B, Hkv, N, *], (scales [B, Hkv, N] fp16),
//   out [B, Hq, D] fp16.  Query head h reads KV head h / G, G = Hq / Hkv.
// A work unit is (b, kv head, head group, split); heads of one group share
// every K/V byte the unit reads.
struct DecodeLaunch {
  KvFormat fmt;
  const void* q;
  const void* K;
  const void* V;
  const void* Ks;     // fp16 per-token scales (quantized formats)
  const void* Vs;
  void* out;
  float* part_m;      // [B*Hq, S] (S > 1 only)
  float* part_l;
  float* part_o;      // [B*Hq, S, D]
  int B, Hq, Hkv, N, D;
  int kv_stride;      // keys between consecutive (b, kv head) rows in memory (>= N)
  const int* n_dev;   // optional device-side valid length (<= N), read at kernel start
  int G;              // Hq / Hkv
  int GP;             // query heads handled by one unit (<= 8)
  int groups;         // ceil(G / GP)
  int S;              // splits (partial slots per row)
  int S_eff;          // non-empty splits actually launched (<= S)
  int chunk;          // keys per split, a multiple of the tile
  int units;          // B * Hkv * groups * S_eff
  int grid;           // persistent CTAs (cluster mode: one CTA per unit)
  int cluster;        // fp16 only: 0, or S_eff when the S_eff split CTAs of a unit form a thread-block
                      // cluster and merge through distributed shared memory (no partials, no combine)
  float sm_scale_log2;                 // (1/sqrt(D)) * log2(e)
  int* status;                         // device status word
  unsigned long long timeout_ns;
  int debug_skip_loads;                // test hook: producer issues nothing
  CUtensorMap tmK, tmV;                // tiled K/V maps (fp16, and int8 GQA)
  TpOut tp;                            // tensor-parallel output (tp.world == 0: write `out`)
  bool out_bf16;                       // `out` is bf16 (local output only; the default is fp16)
};

#ifdef __CUDACC__
// Final output element `idx` (row * D + d) of a launch: fp16, or bf16 when
// the caller asked for it (rounded once from fp32 either way).
__device__ __forceinline__ void store_out(const DecodeLaunch& a, size_t idx, float v) {
  if (a.out_bf16) {
    static_cast<__nv_bfloat16*>(a.out)[idx] = __float2bfloat16_rn(v);
    return;
  }
  const __half_raw h = __half_raw(__float2half_rn(v));
  if (a.tp.world == 0) {
    static_cast<__half_raw*>(a.out)[idx] = h;
  } else {
    for (int p = 0; p < a.tp.world; ++p) a.tp.dst[p][a.tp.dst_off + idx] = h;
  }
}

// After the `nthreads` threads of named barrier `bar` have stored one unit of
// final output: with tensor-parallel output, make the stores visible to the
// other GPUs, then count the unit on every rank.
__device__ __forceinline__ void signal_out(const DecodeLaunch& a, int tid, int bar, int nthreads) {
  if (a.tp.world == 0) return;
  __threadfence_system();
  asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(nthreads) : "memory");
  if (tid == 0) {
    for (int p = 0; p < a.tp.world; ++p) atomicAdd_system(a.tp.cnt[p] + a.tp.rank, 1ull);
  }
}
#endif

// Kernel resource queries and launches, per KV format (attn_f16.cu,
// attn_quant.cu).  *_prepare sets the dynamic shared-memory opt-in for the
// current device and returns how many CTAs of the kernel fit on one SM.
struct KernelShape {
  int threads;
  size_t smem_bytes;
};
KernelShape decode_kernel_shape_f16(int D);
cudaError_t decode_kernel_prepare_f16(int D, int* ctas_per_sm);
// Cluster variant of the fp16 kernel: sets its attributes on the current device and
// returns, for cluster sizes 0..16, how many such clusters can be resident at once.
cudaError_t decode_kernel_prepare_f16_cluster(int D, int (&max_clusters)[17]);
cudaError_t launch_decode_f16(const DecodeLaunch& a, cudaStream_t stream);
KernelShape decode_kernel_shape_quant(bool int4, int D);
cudaError_t decode_kernel_prepare_quant(bool int4, int D, int* ctas_per_sm);
cudaError_t launch_decode_quant(const DecodeLaunch& a, cudaStream_t stream);
cudaError_t decode_kernel_prepare_qtc(bool int4, int D, int* ctas_per_sm);
// Resident thread-block clusters (sizes 2..16) of the int8 GQA tensor-core kernel's cluster-merge form.
cudaError_t decode_kernel_prepare_qtc_cluster(int D, int (&max_clusters)[17]);
cudaError_t launch_decode_qtc(const DecodeLaunch& a, cudaStream_t stream);
// Fused RoPE + q cast + KV append (quantize.cu).
cudaError_t launch_rope_append(bool bf16, bool int8_cache, const void* qkv, int64_t qkv_stride, const void* cos_t,
                               const void* sin_t, int64_t table_rows, int64_t pos_host, const int* pos_dev,
                               void* q_out, void* k_cache, void* v_cache, void* k_scales, void* v_scales, int B,
                               int Hq, int Hkv, int D, int cap, cudaStream_t stream);
// Decode-step model kernels (model_ops.cu).
cudaError_t launch_add_rmsnorm(bool bf16, void* h, const void* delta, const void* w, void* y, int64_t rows, int H,
                               float eps, cudaStream_t stream);
cudaError_t launch_silu_mul(bool bf16, const void* gu, void* y, int64_t rows, int I, int64_t row_stride,
                            cudaStream_t stream);
cudaError_t launch_gemv(bool bf16, bool x_f16, const void* x, const void* W, const void* bias, void* y, int B, int N,
                        int K, cudaStream_t stream);
// The batch-1 fused q/k/v projection with RoPE, the fp16 cast of q and the append of k / v to an
// fp16 cache [Hkv, cap, D] at position *pos_dev (or pos_host) in its epilogue (model_ops.cu).
struct GemvRope {
  const void* cos_t = nullptr;  // [table_rows, D] in the model dtype
  const void* sin_t = nullptr;
  int64_t table_rows = 0;
  int64_t pos_host = 0;
  const int* pos_dev = nullptr;
  __half* q_out = nullptr;      // [Hq, D]
  __half* k_cache = nullptr;    // [Hkv, cap, D]
  __half* v_cache = nullptr;
  int Hq = 0, Hkv = 0, D = 0, cap = 0;
};
cudaError_t launch_gemv_rope_append(bool bf16, const void* x, const void* W, const void* bias, int K,
                                    const GemvRope& rp, cudaStream_t stream);
// SwiGLU of a concatenated [gate | up] projection W [2I, K] (bias [2I] or null): y [B, I].
cudaError_t launch_gemv_swiglu(bool bf16, const void* x, const void* W, const void* bias, void* y, int B, int I, int K,
                               cudaStream_t stream);
size_t argmax_scratch_bytes(int64_t rows);
cudaError_t launch_argmax(bool bf16, const void* logits, int64_t rows, int V, void* scratch, int64_t* out,
                          cudaStream_t stream);
// Tensor-parallel arrival wait (tp.cu).
cudaError_t launch_tp_wait(const unsigned long long* counters, int world, unsigned long long per_call,
                           unsigned long long* sequence, int* status, unsigned long long timeout_ns,
                           cudaStream_t stream);

// Log-sum-exp merge of the S_eff partials of every row into out (fp16),
// chained to the preceding launch by programmatic dependent launch.
cudaError_t launch_combine(const DecodeLaunch& a, cudaStream_t stream);

// Per-token quantizers (quantize.cu).  ctas: the persistent grid's size limit
// (resident CTAs of the staged kernel); status / timeout_ns: the bounded waits
// of its shared-memory ring; debug_skip_loads: the failure-path test hook.  quantize_kernel_prepare sets the staged kernel's
// dynamic shared-memory opt-in on the current device and returns its CTAs per SM.
struct QuantCtl {
  int ctas;
  int* status;
  unsigned long long timeout_ns;
  int debug_skip_loads;  // test hook: the producer issues nothing
};
cudaError_t quantize_kernel_prepare(int* ctas_per_sm);
cudaError_t launch_quantize(bool int4, const void* X, void* codes, void* scales, int64_t rows, int D,
                            const QuantCtl& ctl, cudaStream_t stream);
// Quantize groups x T tokens [groups, T, D] into a cache [groups, cap, D]
// (int4: [groups, cap, D/2]) at positions pos .. pos+T-1 of every group, pos =
// *pos_dev if given else pos_host; D in {64, 128}; X 16-byte aligned.
cudaError_t launch_quantize_into(bool int4, const void* X, void* codes, void* scales, int64_t groups, int64_t T,
                                 int D, int64_t cap, int64_t pos_host, const int* pos_dev, const QuantCtl& ctl,
                                 cudaStream_t stream);

}  // namespace fqkv
