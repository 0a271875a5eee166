/*
 * fqkv_b200.h -- C ABI of the B200 (sm_100a) fused single-query decode-attention
 * library (libfqkv_b200.so).
 *
 * Every entry point takes raw device pointers, sizes and a CUDA stream, returns
 * an fqkv_status_t, never allocates device memory (the fqkv_ipc_* setup
 * functions of the tensor-parallel exchange are the only exception), and
 * launches asynchronously on `stream` (pass NULL for the legacy default stream).  All launches are
 * stream-ordered; the entry points whose buffers all come from the caller are
 * capturable in a CUDA graph.  On failure,
 * fqkv_last_error() returns a message for the calling thread.
 *
 * Tensor layouts are the reference's (emirabayer/Fused-Quantized-KV-Decode-
 * Attention); each entry point names the reference function it replaces as
 * `reference: file:line`.  Element types:
 *   f16  = IEEE binary16, i8 = int8 codes, u8 = packed int4 (two signed
 *   nibbles per byte, element 2t in the low nibble), f32 = binary32.
 * Softmax scale is 1/sqrt(D) in every attention entry point (as in the
 * reference).  Accumulation is fp32; outputs are rounded once to f16.
 *
 * Alignment: K/V code or f16 tensors must start on a 16-byte boundary; q and
 * out on a 4-byte boundary; scale arrays need only natural (2-byte)
 * alignment.  The int8/int4 kernels read scales in 16-byte blocks and may
 * touch up to 15 bytes before the first and after the last scale of an
 * array, always inside the 16-byte blocks that hold those scales.
 */
#ifndef FQKV_B200_H_
#define FQKV_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same type as cudaStream_t / CUstream. */
typedef struct CUstream_st* fqkv_stream_t;

typedef enum fqkv_status_t {
  FQKV_OK = 0,
  FQKV_ERR_INVALID_ARGUMENT = 1, /* bad size, head_dim, W / CW / S, or null pointer */
  FQKV_ERR_MISALIGNED = 2,       /* a pointer violates the alignment rules above */
  FQKV_ERR_CUDA = 3,             /* CUDA runtime / launch error (see fqkv_last_error) */
  FQKV_ERR_UNSUPPORTED_DEVICE = 4, /* current device is not sm_100 */
  FQKV_ERR_DEVICE_TIMEOUT = 5,   /* a bounded in-kernel wait gave up (see fqkv_device_status) */
  FQKV_ERR_PEER = 6              /* tensor-parallel exchange: IPC mapping of a peer's buffer failed */
} fqkv_status_t;

/* KV storage formats for the workspace query. */
typedef enum fqkv_kv_format_t { FQKV_KV_F16 = 0, FQKV_KV_INT8 = 1, FQKV_KV_INT4 = 2 } fqkv_kv_format_t;

/* Message of the last failing call on this thread ("" if none). */
const char* fqkv_last_error(void);

/* Library version string. */
const char* fqkv_version(void);

/* Reads (and, if clear != 0, resets) the in-kernel status word of the current
 * device: 0 = healthy, otherwise the code of the first bounded wait that gave
 * up (61 tile never arrived, 62 stage never freed, 63 copy drain failed,
 * 64 a tensor-parallel peer's attention outputs never arrived).
 * Synchronizes with the device. */
int fqkv_device_status(int* status_out, int clear);

/* Overrides the wall-clock limit of every in-kernel wait (milliseconds,
 * default 2000).  Intended for tests of the failure path. */
void fqkv_set_wait_timeout_ms(uint32_t ms);

/* Test hook for the failure path: while enabled, decode launches and the
 * staged quantizers (D = 64, 128, 256) issue no tile loads, so every in-kernel
 * wait for a tile runs out after the wait limit; the kernel then unwinds (no
 * load is in flight), records status 61 in the device status word and
 * returns, leaving the context usable.  Outputs of such launches are
 * undefined.  Never enable it outside tests. */
void fqkv_debug_skip_loads(int enable);

/* How split plans of the fp16 and the int8 GQA kernels merge their splits
 * (process-wide).  FQKV_SPLIT_AUTO (default): the library decides per call.
 * For small grids (batch-1 decode, short contexts) the split CTAs of each
 * unit form a thread-block cluster that merges through distributed shared
 * memory in the same launch (no workspace used); otherwise splits write fp32
 * partials to the workspace and a second, PDL-chained kernel merges them.  FQKV_SPLIT_COMBINE: always the partials + combine kernel.
 * FQKV_SPLIT_CLUSTER: the cluster merge whenever the grid fits on the GPU.
 * Results agree to fp32 rounding.  For tuning and tests; no counterpart in
 * the reference (which always launches its partial + combine kernel pair). */
enum { FQKV_SPLIT_AUTO = 0, FQKV_SPLIT_COMBINE = 1, FQKV_SPLIT_CLUSTER = 2 };
int fqkv_set_split_mode(int mode);

/* Bytes of optional workspace (split-K partials) that makes the single-block
 * entry points below run with their preferred split count on the current
 * device.  Passing less (or NULL) is valid: the split count is reduced to what
 * fits, down to 1 (no workspace).  Rows are B*Hq (Hq = Hkv = 1 for the
 * non-GQA entry points with B = R). */
size_t fqkv_decode_workspace_bytes(int kv_format, int64_t B, int64_t Hq, int64_t Hkv, int64_t N, int64_t D);

/* What the library found on the current device (for tuning records): info[0]
 * = SMs, info[1] / info[2] = resident CTAs per SM of the fp16 decode kernel at
 * D = 128 / 64, info[3 + c - 2] (c = 2..16) = thread-block clusters of size c
 * of the fp16 cluster-merge kernel that can be resident at once at D = 128,
 * info[18 + c - 2] the same at D = 64.  Writes min(n, FQKV_DEVICE_INFO_LEN)
 * values.  No counterpart in the reference. */
#define FQKV_DEVICE_INFO_LEN 33
int fqkv_device_info(int32_t* info, int32_t n);

/* The launch plan a decode call with these sizes and this much workspace gets
 * on the current device (for tuning, tests and benchmark records):
 * plan_out[0] = splits per (sequence, KV head) work unit (1 = unsplit),
 * plan_out[1] = cluster size when the splits merge through a thread-block
 * cluster (0 = they do not), plan_out[2] = CTAs launched, plan_out[3] = keys
 * per split, plan_out[4] = kernel family (0 fp16, 1 int8 CUDA-core, 2 int4
 * CUDA-core, 3 int8 tensor-core GQA, 4 int4 tensor-core).  Rows as in
 * fqkv_decode_workspace_bytes.  No counterpart in the reference. */
int fqkv_decode_plan(int kv_format, int64_t B, int64_t Hq, int64_t Hkv, int64_t N, int64_t D, size_t workspace_bytes,
                     int32_t* plan_out);

/* fp16 KV.  q [R,D] f16, K/V [R,N,D] f16 -> o [R,D] f16.  D in {64,128};
 * W in {2,4,8} is accepted for compatibility (the kernel picks its own
 * launch shape).
 * reference: kernels/decode_attn_fp16_mw.cu:50 decode_attn_fp16_mw(q,K,V,W) */
int fqkv_decode_attn_fp16_mw(const void* q, const void* K, const void* V, void* o, int64_t R, int64_t N,
                             int64_t D, int64_t W, void* workspace, size_t workspace_bytes,
                             fqkv_stream_t stream);

/* int8 KV.  q [R,D] f16, Kq/Vq [R,N,D] i8, Ks/Vs [R,N] f16 -> o [R,D] f16.
 * reference: kernels/decode_attn_int8_mw.cu:52 decode_attn_int8_mw(q,K,V,Ks,Vs,W) */
int fqkv_decode_attn_int8_mw(const void* q, const void* Kq, const void* Vq, const void* Ks, const void* Vs,
                             void* o, int64_t R, int64_t N, int64_t D, int64_t W, void* workspace,
                             size_t workspace_bytes, fqkv_stream_t stream);

/* int4 KV.  q [R,D] f16, Kp/Vp [R,N,D/2] u8, Ks/Vs [R,N] f16 -> o [R,D] f16.
 * D in {64,128} (the reference supports D = 64 only).
 * reference: kernels/decode_attn_int4.cu:47 decode_attn_int4(q,K,V,Ks,Vs,W) */
int fqkv_decode_attn_int4(const void* q, const void* Kp, const void* Vp, const void* Ks, const void* Vs,
                          void* o, int64_t R, int64_t N, int64_t D, int64_t W, void* workspace,
                          size_t workspace_bytes, fqkv_stream_t stream);

/* GQA fp16 KV.  q [B,Hq,D] f16, K/V [B,Hkv,N,D] f16 -> o [B,Hq,D] f16; query
 * head h reads KV head h / (Hq/Hkv).  Hq must be a multiple of Hkv.
 * reference: kernels/decode_attn_gqa.cu:56 decode_attn_gqa(q,K,V,W) */
int fqkv_decode_attn_gqa(const void* q, const void* K, const void* V, void* o, int64_t B, int64_t Hq,
                         int64_t Hkv, int64_t N, int64_t D, int64_t W, void* workspace,
                         size_t workspace_bytes, fqkv_stream_t stream);

/* GQA fp16 decode over a preallocated KV cache (the decode step of a model).
 * q [B,Hq,D] f16; K/V [B,Hkv,max_len,D] f16 of which positions [0, n) are
 * valid; out [B,Hq,D] f16.  n = *seq_len_dev when seq_len_dev != NULL (int32,
 * read on the device, clamped to max_len -- so one launch, e.g. replayed from
 * a CUDA graph, follows a growing cache), otherwise n = n_host.  Positions
 * [n, max_len) may hold anything (e.g. an unwritten torch.empty tail, NaN or
 * inf): they never reach the output.  Workspace:
 * fqkv_decode_workspace_bytes(FQKV_KV_F16, B, Hq, Hkv, N, D) with N = max_len
 * when seq_len_dev is used, else n_host.
 * Extends decode_attn_gqa (reference: kernels/decode_attn_gqa.cu:56) to the
 * static-cache layout used by the reference's live-model hook (nb:1043-1061). */
int fqkv_decode_attn_gqa_kvcache(const void* q, const void* K, const void* V, void* o, int64_t B, int64_t Hq,
                                 int64_t Hkv, int64_t max_len, int64_t D, int64_t n_host,
                                 const int32_t* seq_len_dev, void* workspace, size_t workspace_bytes,
                                 fqkv_stream_t stream);

/* GQA int8 KV.  q [B,Hq,D] f16, Kq/Vq [B,Hkv,N,D] i8, Ks/Vs [B,Hkv,N] f16 ->
 * o [B,Hq,D] f16; query head h reads KV head h / (Hq/Hkv).  With Hq > Hkv the
 * codes go through a tensor-core kernel that reads each KV head once for all
 * its query heads; Hq == Hkv is fqkv_decode_attn_int8_mw.
 * Combines decode_attn_int8_mw (reference: kernels/decode_attn_int8_mw.cu:52)
 * with the head mapping of decode_attn_gqa (kernels/decode_attn_gqa.cu:56). */
int fqkv_decode_attn_gqa_int8(const void* q, const void* Kq, const void* Vq, const void* Ks, const void* Vs,
                              void* o, int64_t B, int64_t Hq, int64_t Hkv, int64_t N, int64_t D, void* workspace,
                              size_t workspace_bytes, fqkv_stream_t stream);

/* GQA int8 decode over a preallocated int8 KV cache: codes [B,Hkv,max_len,D]
 * i8, scales [B,Hkv,max_len] f16, positions [0, n) valid with n as in
 * fqkv_decode_attn_gqa_kvcache (device-side or host length); codes and
 * scales past n may hold anything (NaN / inf scales included).  Workspace:
 * fqkv_decode_workspace_bytes(FQKV_KV_INT8, B, Hq, Hkv, N, D) with the same N. */
int fqkv_decode_attn_gqa_int8_kvcache(const void* q, const void* Kq, const void* Vq, const void* Ks,
                                      const void* Vs, void* o, int64_t B, int64_t Hq, int64_t Hkv,
                                      int64_t max_len, int64_t D, int64_t n_host, const int32_t* seq_len_dev,
                                      void* workspace, size_t workspace_bytes, fqkv_stream_t stream);

/* GQA split-K (batch 1).  q [Hq,D] f16, K/V [Hkv,N,D] f16; caller-owned
 * scratch m_part/l_part [Hq,S] f32, o_part [Hq,S,D] f32; out [Hq,D] f16.
 * At most S splits are used: the library picks the count (<= S, whole
 * 64-key tiles per split) that fills the GPU; the scratch contents after the
 * call are unspecified.  W in {2,4,8}, CW in {4,8}
 * are accepted for compatibility.
 * reference: kernels/decode_attn_gqa_sk_fast.cu:95 gqa_sk_fast(q,K,V,m_part,l_part,o_part,o,S,W,CW) */
int fqkv_gqa_sk_fast(const void* q, const void* K, const void* V, float* m_part, float* l_part, float* o_part,
                     void* out, int64_t Hq, int64_t Hkv, int64_t N, int64_t D, int64_t S, int64_t W, int64_t CW,
                     fqkv_stream_t stream);

/* Split-K GQA decode that allocates nothing: same inputs, output and result as
 * fqkv_gqa_sk_fast, but the per-split partials live in a 4 MiB array that the
 * library keeps in device memory (one per GPU, held until exit) instead of in
 * caller scratch.  For callers that may not allocate device memory at the
 * call site (a serving runtime's enqueue/plugin hook that owns all device
 * memory, a decode loop that must not stall on cudaMalloc, a C host with no
 * allocator).  Limit: 2*pad256(4*Hq*S) + 4*Hq*S*D bytes must fit in 4 MiB
 * (e.g. Hq=32, D=128 allows S <= 252), else FQKV_ERR_INVALID_ARGUMENT and
 * nothing is launched.  The first call on a device (with it current) looks up
 * the array's device address and caches it; make it before any stream
 * capture.  A failed lookup returns FQKV_ERR_CUDA and is retried on the next
 * call.  All calls share the array: calls that overlap on the GPU race on it.
 * No counterpart in the reference. */
int fqkv_gqa_sk_fast_static_scratch(const void* q, const void* K, const void* V, void* out, int64_t Hq,
                                    int64_t Hkv, int64_t N, int64_t D, int64_t S, int64_t W, int64_t CW,
                                    fqkv_stream_t stream);

/* Per-token symmetric int8 quantizer, bit-exact with the reference's torch
 * code.  X [rows,D] f16 -> codes [rows,D] i8, scales [rows] f16 (any D >= 1).
 * reference: notebooks/integration_and_benchmarks.ipynb:236-238 qpt(X),
 *            tests/test_kernels.py:32-34 */
int fqkv_quantize_int8_per_token(const void* X, void* codes, void* scales, int64_t rows, int64_t D,
                                 fqkv_stream_t stream);

/* Per-token symmetric int4 quantizer + nibble packer, bit-exact.
 * X [rows,D] f16 (D even) -> packed [rows,D/2] u8, scales [rows] f16.
 * reference: notebooks/integration_and_benchmarks.ipynb:292-299 quant_int4_per_token(X) */
int fqkv_quantize_int4_per_token(const void* X, void* packed, void* scales, int64_t rows, int64_t D,
                                 fqkv_stream_t stream);

/* Quantize-on-append: X [groups,T,D] f16 (D in {64,128}, 16-byte aligned) is
 * quantized exactly like fqkv_quantize_int8_per_token and written into a
 * cache codes [groups,cap,D] i8 / scales [groups,cap] f16 at positions
 * pos .. pos+T-1 of every group, pos = *pos_dev (device int32, for a decode
 * step replayed from a CUDA graph) if non-NULL else pos_host.  Tokens that
 * would land at or past cap are not written.
 * reference: quantizer of notebooks/integration_and_benchmarks.ipynb:236-238,
 * applied per appended token instead of to the whole cache. */
int fqkv_quantize_int8_into_cache(const void* X, void* codes, void* scales, int64_t groups, int64_t T, int64_t D,
                                  int64_t cap, int64_t pos_host, const int32_t* pos_dev, fqkv_stream_t stream);

/* Same for the int4 cache: packed [groups,cap,D/2] u8, scales [groups,cap] f16.
 * reference: notebooks/integration_and_benchmarks.ipynb:292-299 */
int fqkv_quantize_int4_into_cache(const void* X, void* packed, void* scales, int64_t groups, int64_t T,
                                  int64_t D, int64_t cap, int64_t pos_host, const int32_t* pos_dev,
                                  fqkv_stream_t stream);

/* Fused decode-step prologue of a Llama-style attention block: rotary
 * embedding of q and k, the fp16 cast of q, and the append of k and v to the
 * KV cache, in one launch.  qkv [B, qkv_row_stride] in the model dtype
 * (model_dtype 0 = f16, 1 = bf16) holds each sequence's fused projection
 * output [q heads | k heads | v heads], D elements per head; cos_table /
 * sin_table [table_rows, D] (model dtype) are the model's rotary tables.  At
 * position pos = *pos_dev (device int32) if non-NULL else pos_host:
 *   q_out [B,Hq,D] f16      <- fp16(rope(q))
 *   K cache [B,Hkv,cap,D]   <- fp16(rope(k)) at pos (kv_format FQKV_KV_F16), or
 *                              its int8 codes + f16 scale [B,Hkv,cap]
 *                              (FQKV_KV_INT8, bit-exact with the reference
 *                              quantizer), and V likewise from fp16(v).
 * rope(x)_i = T(T(x_i*cos_i) + T(r_i*sin_i)), r = cat(-x[D/2:], x[:D/2]),
 * T = rounding to the model dtype: bit-exact with transformers'
 * apply_rotary_pos_emb followed by .to(float16).  Positions at or past cap (or
 * the table) write nothing to the cache.  D in {64, 128}.
 * reference: the live-model hook's per-step cache update
 * (notebooks/integration_and_benchmarks.ipynb:1043-1061) with the quantizer of
 * lines 236-238 applied to the new token only. */
int fqkv_rope_qkv_append(int32_t kv_format, int32_t model_dtype, const void* qkv, int64_t qkv_row_stride,
                         const void* cos_table, const void* sin_table, int64_t table_rows, int64_t pos_host,
                         const int32_t* pos_dev, void* q_out, void* k_cache, void* v_cache, void* k_scales,
                         void* v_scales, int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t cap,
                         fqkv_stream_t stream);

/* Decode-step helpers of the graph-captured Llama decoder (no counterpart in
 * the reference, whose end-to-end path runs transformers' eager modules;
 * they cut the launches of a step).  model_dtype 0 = f16, 1 = bf16.
 * Residual add + RMSNorm of rows [rows, H] (H <= 8192):
 *   if delta: h <- T(h + delta)   (in place)
 *   y <- T(w * T(h * rsqrt(mean(h^2) + eps)))     (fp32 inside, T = model dtype)
 * -- transformers' LlamaRMSNorm arithmetic (the fp32 sum of squares may be
 * summed in a different order). */
int fqkv_add_rmsnorm(int32_t model_dtype, void* h, const void* delta, const void* weight, void* y, int64_t rows,
                     int64_t H, float eps, fqkv_stream_t stream);

/* SwiGLU: y [rows, I] <- T(T(silu(g)) * u) with g = gu[:, :I], u = gu[:, I:2I]
 * (row stride gu_row_stride elements), silu(x) = x / (1 + exp(-x)) in fp32. */
int fqkv_silu_mul(int32_t model_dtype, const void* gu, void* y, int64_t rows, int64_t I, int64_t gu_row_stride,
                  fqkv_stream_t stream);

/* Small-batch projection of a decode step: y [B,N] = x [B,K] W^T (+ bias [N])
 * with W [N,K] row-major, W / bias / y in the model dtype, fp32
 * accumulation, B in 1..4, K a multiple of 256, x / W / y 16-byte aligned.
 * x_dtype is the model dtype, or 0 (fp16) with bf16 weights: x is then
 * rounded to bf16 as it is read (the fp16 attention output feeding a bf16
 * output projection, with no separate cast).  At B = 1 the kernel is
 * launched with programmatic dependent launch and issues its first weight
 * loads before it waits for the previous kernel on the stream, so W and bias
 * must not be written by a kernel that may still be running (model weights
 * never are); x is read after the wait. */
int fqkv_gemv(int32_t model_dtype, int32_t x_dtype, const void* x, const void* W, const void* bias, void* y, int64_t B,
              int64_t N, int64_t K, fqkv_stream_t stream);

/* The gate/up projection of a SwiGLU MLP and the SwiGLU in one launch: W
 * [2I, K] is the concatenation [gate_proj.weight; up_proj.weight] (bias [2I]
 * the concatenated biases, or null), y [B, I] = T(T(silu(g)) * u) with g, u
 * the two projections of x [B, K] rounded to the model dtype T -- the values
 * of fqkv_gemv on W followed by fqkv_silu_mul, without the [B, 2I]
 * intermediate or the second launch.  Same sizes, alignment and launch
 * behaviour as fqkv_gemv (x in the model dtype).  No counterpart in the
 * reference (it replaces the Llama MLP's gate/up linear and act_fn * up in
 * the decode step, transformers LlamaMLP.forward). */
int fqkv_gemv_swiglu(int32_t model_dtype, const void* x, const void* W, const void* bias, void* y, int64_t B,
                     int64_t I, int64_t K, fqkv_stream_t stream);

/* Batch-1 decode-step attention prologue in one launch: the fused q/k/v
 * projection y = x W^T (+ bias) of one token (x [K], W [(Hq + 2 Hkv) D, K] =
 * [q_proj; k_proj; v_proj] weights, model dtype), then in its epilogue what
 * fqkv_rope_qkv_append does for an fp16 cache: RoPE of the q and k heads from
 * the model's rotary tables [table_rows, D] at position pos (*pos_dev when
 * given, else pos_host), the cast to fp16, q into q_out [Hq, D] and k / v
 * into the caches [Hkv, cap, D] at row pos (not written when pos >= cap).
 * The values equal fqkv_gemv followed by fqkv_rope_qkv_append.  D is 64 or
 * 128, K a multiple of 256 in [256, 16384]; x and W 16-byte aligned.
 * Launched with programmatic dependent launch like fqkv_gemv at B = 1 (W and
 * bias must not be written by a kernel that may still be running).  No
 * counterpart in the reference (it replaces the q/k/v linears,
 * apply_rotary_pos_emb and the cache update of the decode step). */
int fqkv_gemv_rope_append(int32_t model_dtype, const void* x, const void* W, const void* bias, int64_t K,
                          const void* cos_table, const void* sin_table, int64_t table_rows, int64_t pos_host,
                          const int32_t* pos_dev, void* q_out, void* k_cache, void* v_cache, int64_t Hq, int64_t Hkv,
                          int64_t D, int64_t cap, fqkv_stream_t stream);

/* Greedy token choice: idx [rows] int64 = argmax over each row of logits
 * [rows, V] (model dtype), first index of the maximum, NaN largest (as
 * torch.argmax).  `scratch` holds fqkv_argmax_scratch_bytes(rows) bytes,
 * zero-filled before its first use; the call leaves it reusable. */
size_t fqkv_argmax_scratch_bytes(int64_t rows);
int fqkv_argmax(int32_t model_dtype, const void* logits, int64_t rows, int64_t V, void* scratch, int64_t* idx,
                fqkv_stream_t stream);

/* ------------------------------------------------------------------------
 * Tensor-parallel decode: attention fused with the all-gather of its outputs.
 * No counterpart in the reference: its tensor-parallel end-to-end config
 * all-gathers the attention outputs of every layer with NCCL.  Here the decode
 * kernel that produces a rank's attention output (or the split-K combine, when
 * the plan splits) stores it straight into every rank's receive buffer over
 * NVLink and then counts one arrival per output unit on every rank's counter
 * slot for this rank (system-scope atomic after a system fence);
 * fqkv_tp_wait, enqueued before the consumer of the gathered outputs, waits
 * (bounded) until every rank's arrivals for this call are in.  Counters only
 * grow, so a whole decode step, collectives included, replays from one CUDA
 * graph.  Receive buffers and counters live in memory from fqkv_ipc_alloc,
 * mapped on the other ranks with fqkv_ipc_open. */
#define FQKV_TP_MAX_RANKS 8

typedef struct fqkv_tp_out {
  int32_t world;       /* number of ranks (2 .. FQKV_TP_MAX_RANKS) */
  int32_t rank;        /* this rank: its slice of every receive buffer, its counter slot */
  int64_t dst_offset;  /* f16 elements from each dst[] to this rank's [B, Hq_local, D] slice */
  void* dst[FQKV_TP_MAX_RANKS];                      /* receive buffers of ranks 0..world-1, mapped here */
  unsigned long long* counters[FQKV_TP_MAX_RANKS];   /* arrival counters [world] of ranks 0..world-1, mapped here */
} fqkv_tp_out_t;

/* fqkv_decode_attn_gqa_kvcache (kv_format FQKV_KV_F16: Ks = Vs = NULL) or
 * fqkv_decode_attn_gqa_int8_kvcache (FQKV_KV_INT8) with the output o [B, Hq,
 * D] in out_dtype 0 (fp16, as those entries) or 1 (bf16, for a bf16 model's
 * output projection; each element is rounded once from the fp32 result).
 * No counterpart in the reference. */
int fqkv_decode_attn_kvcache_out(int32_t kv_format, int32_t out_dtype, const void* q, const void* K, const void* V,
                                 const void* Ks, const void* Vs, void* o, int64_t B, int64_t Hq, int64_t Hkv,
                                 int64_t max_len, int64_t D, int64_t n_host, const int32_t* seq_len_dev,
                                 void* workspace, size_t workspace_bytes, fqkv_stream_t stream);

/* fqkv_decode_attn_gqa_kvcache (kv_format FQKV_KV_F16: Ks = Vs = NULL) or
 * fqkv_decode_attn_gqa_int8_kvcache (FQKV_KV_INT8) for this rank's heads, with
 * the output sent to every rank as described above instead of to an `o`
 * tensor.  Each receive buffer must hold dst_offset + B*Hq*D f16 (16-byte
 * aligned); every rank must make the same calls with the same sizes. */
int fqkv_decode_attn_kvcache_tp(int32_t kv_format, const void* q, const void* K, const void* V, const void* Ks,
                                const void* Vs, int64_t B, int64_t Hq, int64_t Hkv, int64_t max_len, int64_t D,
                                int64_t n_host, const int32_t* seq_len_dev, void* workspace, size_t workspace_bytes,
                                const fqkv_tp_out_t* tp, fqkv_stream_t stream);

/* Arrivals one call of fqkv_decode_attn_kvcache_tp with these sizes (and the
 * same workspace size) counts on each counter slot; the waiter's per_call.
 * Returns -1 (message in fqkv_last_error) on bad arguments. */
int64_t fqkv_tp_arrivals(int32_t kv_format, int64_t B, int64_t Hq, int64_t Hkv, int64_t max_len, int64_t D,
                         size_t workspace_bytes);

/* Waits on `stream` until counters[r] >= (*sequence + 1) * per_call for every
 * rank r < world (counters and sequence: this rank's own device memory), then
 * increments *sequence.  Bounded: after the wait limit it records status 64 in
 * the device status word and returns (the call still completes).  While the
 * device status word is non-zero (a bounded wait gave up and nobody has read
 * and cleared it with fqkv_device_status) the wait returns at once. */
int fqkv_tp_wait(const unsigned long long* counters, int32_t world, uint64_t per_call,
                 unsigned long long* sequence, fqkv_stream_t stream);

/* Exchange memory: `bytes` of zero-filled device memory on the current device
 * and its 64-byte IPC handle (to send to the other ranks of the node). */
int fqkv_ipc_alloc(size_t bytes, void** dev_ptr, void* ipc_handle);
/* Maps another rank's exchange memory (its 64-byte handle) on the current device. */
int fqkv_ipc_open(const void* ipc_handle, void** dev_ptr);
/* Unmaps memory from fqkv_ipc_open. */
int fqkv_ipc_close(void* dev_ptr);
/* Frees memory from fqkv_ipc_alloc (after every rank has closed its mapping). */
int fqkv_ipc_free(void* dev_ptr);

#ifdef __cplusplus
}
#endif

#endif /* FQKV_B200_H_ */
