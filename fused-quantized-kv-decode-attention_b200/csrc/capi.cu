// extern "C" entry points of libfqkv_b200.so (declared in include/fqkv_b200.h).
//
// Responsibilities: argument validation with the reference's error conditions
// (before any CUDA call, so a bad call fails the same way with or without a
// GPU), per-device one-time set-up (SM count, shared-memory opt-in, occupancy,
// status-word address), TMA tensor-map encoding, the split-K plan, and the
// launches.  No device memory is allocated here: split-K partials live in the
// caller's workspace (or the caller's m/l/o scratch for gqa_sk_fast).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <functional>
#include <mutex>

#include "../../include/fqkv_b200.h"
#include "kernels.h"

// In-kernel status word (one per device image): written by a bounded wait that
// gives up, read by fqkv_device_status().
__device__ int g_fqkv_device_status;

namespace {

using fqkv::DecodeLaunch;
using fqkv::KvFormat;

thread_local char t_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err, sizeof(t_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(FQKV_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

std::atomic<unsigned long long> g_timeout_ns{2000ull * 1000ull * 1000ull};
std::atomic<int> g_debug_skip_loads{0};
std::atomic<int> g_split_mode{FQKV_SPLIT_AUTO};

// ------------------------------------------------------------------ device state
constexpr int kMaxDevices = 64;

struct DeviceState {
  std::once_flag once;
  int err_code = FQKV_OK;
  char err_msg[256] = "";
  int sm_count = 0;
  int* status = nullptr;
  int occ_f16[2] = {0, 0};      // D = 64, 128
  int occ_q[2][2] = {{0, 0}, {0, 0}};  // [int4][D==128]
  int occ_qtc[2][2] = {{0, 0}, {0, 0}};  // tensor-core quantized kernel [int4][D==128]
  int max_clusters_f16[2][17] = {};      // fp16 cluster mode: resident clusters per cluster size [D==128][size]
  int max_clusters_qtc[2][17] = {};      // int8 GQA cluster mode: the same for the tensor-core kernel
  int occ_quantize = 0;                  // staged quantizer CTAs per SM
};
DeviceState g_dev[kMaxDevices];

void init_device(DeviceState& ds, int dev) {
  auto bad = [&](int code, const char* msg) {
    ds.err_code = code;
    snprintf(ds.err_msg, sizeof(ds.err_msg), "%s", msg);
  };
  int major = 0, minor = 0;
  cudaError_t e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&ds.sm_count, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return bad(FQKV_ERR_CUDA, cudaGetErrorString(e));
  if (major != 10 || minor != 0) {
    char m[128];
    snprintf(m, sizeof(m), "device %d is sm_%d%d; this library is built for sm_100a (B200)", dev, major, minor);
    return bad(FQKV_ERR_UNSUPPORTED_DEVICE, m);
  }
  e = cudaGetSymbolAddress(reinterpret_cast<void**>(&ds.status), g_fqkv_device_status);
  if (e != cudaSuccess) return bad(FQKV_ERR_CUDA, cudaGetErrorString(e));
  for (int i = 0; i < 2 && e == cudaSuccess; ++i) e = fqkv::decode_kernel_prepare_f16(i ? 128 : 64, &ds.occ_f16[i]);
  for (int i = 0; i < 2 && e == cudaSuccess; ++i)
    e = fqkv::decode_kernel_prepare_f16_cluster(i ? 128 : 64, ds.max_clusters_f16[i]);
  for (int i = 0; i < 2 && e == cudaSuccess; ++i)
    e = fqkv::decode_kernel_prepare_qtc_cluster(i ? 128 : 64, ds.max_clusters_qtc[i]);
  for (int q = 0; q < 2 && e == cudaSuccess; ++q)
    for (int i = 0; i < 2 && e == cudaSuccess; ++i)
      e = fqkv::decode_kernel_prepare_quant(q == 1, i ? 128 : 64, &ds.occ_q[q][i]);
  for (int i = 0; i < 2 && e == cudaSuccess; ++i) e = fqkv::decode_kernel_prepare_qtc(false, i ? 128 : 64, &ds.occ_qtc[0][i]);
  for (int i = 0; i < 2 && e == cudaSuccess; ++i) e = fqkv::decode_kernel_prepare_qtc(true, i ? 128 : 64, &ds.occ_qtc[1][i]);
  if (e == cudaSuccess) e = fqkv::quantize_kernel_prepare(&ds.occ_quantize);
  if (e != cudaSuccess) return bad(FQKV_ERR_CUDA, cudaGetErrorString(e));
}

int device_state(DeviceState** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(FQKV_ERR_CUDA, "device index %d out of range", dev);
  DeviceState& ds = g_dev[dev];
  std::call_once(ds.once, init_device, std::ref(ds), dev);
  if (ds.err_code != FQKV_OK) return fail(ds.err_code, "device init: %s", ds.err_msg);
  *out = &ds;
  return FQKV_OK;
}

// ------------------------------------------------------------------ per-thread caches
// A decode call's host work is dominated by the split plan (a search over split
// counts) and two TMA descriptor encodings; both are pure functions of their
// inputs, so the last few results are kept per thread and reused when the same
// sizes (and, for descriptors, the same pointers) come again -- the usual case
// in a decode loop.
template <typename Key, typename Val, int kN>
struct SmallCache {
  Key keys[kN];
  Val vals[kN];
  bool used[kN] = {};
  int next = 0;
  const Val* find(const Key& k) const {
    for (int i = 0; i < kN; ++i)
      if (used[i] && std::memcmp(&keys[i], &k, sizeof(Key)) == 0) return &vals[i];
    return nullptr;
  }
  void put(const Key& k, const Val& v) {
    keys[next] = k;
    vals[next] = v;
    used[next] = true;
    next = (next + 1) % kN;
  }
};

struct MapKey {
  const void* base;
  int64_t BH, N, inner, stride;
  int tile, kind;  // kind 0: fp16 rows of `inner` dims; 1: code rows of `inner` bytes
};

// ------------------------------------------------------------------ tensor maps
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// K or V viewed as [B*Hkv][N][D] fp16 with `stride` keys between consecutive
// (b, kv head) rows, box = 64 dims x 64 keys x 1, 128B swizzle.
int make_kv_map(CUtensorMap* map, const void* base, int64_t BH, int64_t N, int64_t D, int64_t stride) {
  thread_local SmallCache<MapKey, CUtensorMap, 8> cache;
  MapKey key;
  std::memset(&key, 0, sizeof(key));
  key.base = base; key.BH = BH; key.N = N; key.inner = D; key.stride = stride; key.tile = 64; key.kind = 0;
  if (const CUtensorMap* hit = cache.find(key)) {
    *map = *hit;
    return FQKV_OK;
  }
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(FQKV_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  const cuuint64_t dims[3] = {cuuint64_t(D), cuuint64_t(N), cuuint64_t(BH)};
  const cuuint64_t strides[2] = {cuuint64_t(D) * 2, cuuint64_t(stride) * cuuint64_t(D) * 2};
  const cuuint32_t box[3] = {64, 64, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FQKV_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", int(r));
  cache.put(key, *map);
  return FQKV_OK;
}

// Quantized codes viewed as [B*Hkv][N][rb] bytes (rb = 128, 64 or 32 bytes
// per key row) with `stride` keys between consecutive (b, kv head) rows; box =
// one tile of `tile` whole rows, swizzled at the row width.
int make_kv_map_codes(CUtensorMap* map, const void* base, int64_t BH, int64_t N, int64_t rb, int64_t stride,
                      int tile) {
  thread_local SmallCache<MapKey, CUtensorMap, 8> cache;
  MapKey key;
  std::memset(&key, 0, sizeof(key));
  key.base = base; key.BH = BH; key.N = N; key.inner = rb; key.stride = stride; key.tile = tile; key.kind = 1;
  if (const CUtensorMap* hit = cache.find(key)) {
    *map = *hit;
    return FQKV_OK;
  }
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(FQKV_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  const cuuint64_t dims[3] = {cuuint64_t(rb), cuuint64_t(N), cuuint64_t(BH)};
  const cuuint64_t strides[2] = {cuuint64_t(rb), cuuint64_t(stride) * cuuint64_t(rb)};
  const cuuint32_t box[3] = {cuuint32_t(rb), cuuint32_t(tile), 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapSwizzle sw = rb == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                : rb == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                           : CU_TENSOR_MAP_SWIZZLE_32B;
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FQKV_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", int(r));
  cache.put(key, *map);
  return FQKV_OK;
}

// ------------------------------------------------------------------ planning
size_t partial_bytes(int64_t rows, int64_t S, int64_t D) {
  const size_t ml = size_t(rows) * size_t(S) * sizeof(float);
  const size_t ml_al = (ml + 255) & ~size_t(255);
  return 2 * ml_al + size_t(rows) * size_t(S) * size_t(D) * sizeof(float);
}

void carve_partials(DecodeLaunch& a, void* ws, int64_t rows) {
  const size_t ml = size_t(rows) * size_t(a.S) * sizeof(float);
  const size_t ml_al = (ml + 255) & ~size_t(255);
  uint8_t* p = static_cast<uint8_t*>(ws);
  a.part_m = reinterpret_cast<float*>(p);
  a.part_l = reinterpret_cast<float*>(p + ml_al);
  a.part_o = reinterpret_cast<float*>(p + 2 * ml_al);
}

int ctas_per_sm(const DeviceState& ds, KvFormat f, int D) {
  const int i = D == 128 ? 1 : 0;
  if (f == KvFormat::F16) return std::max(1, ds.occ_f16[i]);
  if (f == KvFormat::I8Gqa || f == KvFormat::I4Tc) return std::max(1, ds.occ_qtc[f == KvFormat::I4Tc ? 1 : 0][i]);
  return std::max(1, ds.occ_q[f == KvFormat::I4 ? 1 : 0][i]);
}

// Fills the geometry of `a` (fmt, B, Hq, Hkv, N, D set by the caller).
// S_fixed > 0: use at most S_fixed splits (gqa_sk_fast).  Otherwise pick the
// split count that minimises the modelled time, limited to what `ws_bytes`
// can hold when `limit_ws`.
struct PlanKey {
  const DeviceState* ds;
  int fmt, B, Hq, Hkv, N, D, tp, mode;
  int64_t S_fixed;
  size_t ws_bytes;
  int limit_ws;
};
struct PlanVal {
  int fmt, G, GP, groups, cluster, S, S_eff, chunk, units, grid;
};

void plan_geometry(DecodeLaunch& a, const DeviceState& ds, int64_t S_fixed, size_t ws_bytes, bool limit_ws);

// Fills the plan of `a` (fmt, B, Hq, Hkv, N, D and tp set by the caller), from the
// per-thread cache when the same sizes were planned before.
void plan(DecodeLaunch& a, const DeviceState& ds, int64_t S_fixed, size_t ws_bytes, bool limit_ws) {
  thread_local SmallCache<PlanKey, PlanVal, 8> cache;
  PlanKey key;
  std::memset(&key, 0, sizeof(key));
  key.ds = &ds; key.fmt = int(a.fmt); key.B = a.B; key.Hq = a.Hq; key.Hkv = a.Hkv; key.N = a.N; key.D = a.D;
  key.tp = a.tp.world != 0; key.mode = g_split_mode.load(); key.S_fixed = S_fixed;
  key.ws_bytes = limit_ws ? ws_bytes : 0; key.limit_ws = limit_ws;
  if (const PlanVal* v = cache.find(key)) {
    a.fmt = KvFormat(v->fmt); a.G = v->G; a.GP = v->GP; a.groups = v->groups; a.cluster = v->cluster;
    a.S = v->S; a.S_eff = v->S_eff; a.chunk = v->chunk; a.units = v->units; a.grid = v->grid;
  } else {
    plan_geometry(a, ds, S_fixed, ws_bytes, limit_ws);
    cache.put(key, PlanVal{int(a.fmt), a.G, a.GP, a.groups, a.cluster, a.S, a.S_eff, a.chunk, a.units, a.grid});
  }
  a.sm_scale_log2 = float(1.4426950408889634 / std::sqrt(double(a.D)));
  a.status = ds.status;
  a.timeout_ns = g_timeout_ns.load();
  a.debug_skip_loads = g_debug_skip_loads.load();
}

void plan_geometry(DecodeLaunch& a, const DeviceState& ds, int64_t S_fixed, size_t ws_bytes, bool limit_ws) {
  // int8 codes shared by several query heads go to the tensor-core GQA kernel.
  // int8 codes shared by several query heads, and int4 codes with D = 128, go
  // to the tensor-core quantized kernel (measured on B200: int4 D = 128 817 vs
  // 871 us on the CUDA-core kernel at config 3; at D = 64 the CUDA-core kernel
  // is faster, 463 vs 578 us, its per-key softmax work being shared by fewer
  // dimensions on the tensor-core path).
  if (a.fmt == KvFormat::I8 && a.Hq != a.Hkv) a.fmt = KvFormat::I8Gqa;
  if (a.fmt == KvFormat::I4 && a.D == 128) a.fmt = KvFormat::I4Tc;
  a.G = a.Hq / a.Hkv;
  a.GP = std::min(a.G, 8);
  a.groups = (a.G + a.GP - 1) / a.GP;
  const int TK = fqkv::tile_keys(a.fmt, a.D);
  const int64_t tiles = (int64_t(a.N) + TK - 1) / TK;
  const int64_t units0 = int64_t(a.B) * a.Hkv * a.groups;
  const int64_t C = int64_t(ds.sm_count) * ctas_per_sm(ds, a.fmt, a.D);
  const int64_t rows = int64_t(a.B) * a.Hq;

  auto geometry = [&](int64_t S, int64_t* chunk_tiles, int64_t* S_eff) {
    *chunk_tiles = (tiles + S - 1) / S;
    *S_eff = (tiles + *chunk_tiles - 1) / *chunk_tiles;
  };
  // Modelled time: every round of the persistent grid costs
  // max(active CTAs, 3/5 of the grid) x tiles per unit -- with fewer CTAs than
  // that the machine stops being HBM-bound -- and splitting adds about one
  // tile of epilogue work per unit.  S_fixed > 0 (gqa_sk_fast) caps the split
  // count at the caller's scratch capacity; otherwise the caller's workspace
  // bytes cap it when `limit_ws`.  The floor and the combine terms below were
  // fitted on B200 to forced-split sweeps of the fp16 GQA kernel (Hq=32,
  // Hkv=8, D in {64, 128}, B in {1, 2, 4, 8}, N from 2K to 64K): mean loss
  // against the best measured split 3.7 % -> 1.4 %; planned calls over
  // B <= 64, N >= 640 1.6 % faster in sum (B=1, N=2048, D=128: 8.9 -> 7.8 us;
  // N=16K: 18.4 -> 17.7 us).
  const int64_t floor_ctas = (3 * C) / 5;
  const int64_t maxS = S_fixed > 0 ? std::min<int64_t>(tiles, S_fixed) : std::min<int64_t>(tiles, 256);
  auto best_split = [&](bool respect_ws) {
    double best = 1e300;
    int64_t best_S = 1;
    for (int64_t S = 1; S <= maxS; ++S) {
      int64_t ct, se;
      geometry(S, &ct, &se);
      if (se != S) continue;
      if (respect_ws && se > 1 && partial_bytes(rows, se, a.D) > ws_bytes) continue;
      const int64_t U = units0 * se;
      double cost = 0;
      for (int64_t done = 0; done < U; done += C) {
        const int64_t active = std::min(C, U - done);
        cost += double(std::max<int64_t>(active, floor_ctas)) * double(ct + (se > 1 ? 1 : 0));
      }
      // The combine kernel (its wait for the partial grid, the partials' round
      // trip through L2) costs about three tile-rounds of the whole grid (B=64,
      // Hkv=8, N=640, D=64 runs 20.4 us unsplit against 25.7 us in two splits),
      // plus 0.07 of a round per split (its loop over the partials: config 4
      // at 16K measured 3.1 us of combine at 24 splits, 5.6 us at 37).
      if (se > 1) cost += (3.0 + 0.07 * double(se)) * double(C);
      if (cost < best * 0.999) {
        best = cost;
        best_S = se;
      }
    }
    return best_S;
  };
  // The cluster merge below needs no workspace, so whether to split is decided
  // first without the workspace limit; the limit applies to the combine plan.
  const bool ws_limited = S_fixed <= 0 && limit_ws;
  int64_t ct, se;
  geometry(best_split(false), &ct, &se);
  a.cluster = 0;
  // Cluster mode (fp16 and int8 GQA, local output): when the grid is too small to fill the GPU
  // without splitting, the S split CTAs of each unit form one thread-block cluster (S <= 16) and
  // merge through distributed shared memory -- one launch, no partials, no combine.  The fp16
  // kernel's cluster form runs one CTA per SM with a deep ring and two consumer groups.
  // The cluster is the largest size whose clusters are all resident at once (batch 1 with 8 KV
  // heads would need 8 resident clusters of 16 and B200 holds 7 -- one GPC has fewer than 16 SMs
  // free -- so it gets 10).  Automatic choice, from forced-mode sweeps on B200 (us per call,
  // partials + combine -> cluster merge; Hkv = 8):
  //  * short contexts, D = 64 and 128: dropping the combine's fixed cost wins even with few SMs
  //    streaming and even where the split search alone would not split (D = 64, N = 512 / 640 /
  //    1024 / 2048: batch 1 4.76 -> 3.68, 5.42 -> 3.99, 5.68 -> 3.88, 6.38 -> 4.56; batch 4 5.56
  //    -> 4.21, 5.65 -> 4.65, 6.34 -> 4.90, 8.08 -> 7.25; batch 8 (unsplit plan) 7.82 -> 4.80,
  //    6.90 -> 5.39, 8.10 -> 7.07, 10.16 -> 10.26), so it is taken up to N = 4096 at D = 64, and
  //    up to N = 8192 for a grid of at most 8 units (batch 1 with Hkv = 8: N = 8192 9.49 -> 8.60;
  //    N = 16K 11.74 -> 12.58; batch 2 and 4 at N = 16K 15.7 -> 18.2 and 24.5 -> 25.7);
  //  * D = 128 up to N = 32K (batch 1, N = 2K / 16K / 32K / 64K: 7.21 -> 5.36, 16.99 -> 15.56,
  //    27.2 -> 26.4, 46.0 -> 47.4; batch 2: 8.75 -> 7.18, 25.8 -> 24.3, 44.8 -> 44.4, 83.0 -> 84.0;
  //    batch 3: 9.33 -> 8.77, 34.9 -> 33.0, 63.4 -> 61.3, 120.4 -> 116.8), and at any length when
  //    the grid-filling cluster is resident and keeps at least half the SMs streaming (B=4:
  //    N=4K 16.5 -> 14.0, 16K 43.8 -> 43.1, 64K 159.9 -> 156.8; B=8: 26.1 -> 23.8, 84.0 -> 82.0,
  //    325.6 -> 323.3);
  //  * D = 64 longer contexts keep the combine: one CTA per SM streams too slowly there (batch 1,
  //    N=16K: 11.8 -> 12.6 us; B=4, N=64K: 83 -> 97 us).
  const int mode = g_split_mode.load();
  const int64_t short_n = a.D == 128 ? 32768 : (units0 <= 8 ? 8192 : 4096);
  const bool f16 = a.fmt == KvFormat::F16;
  // int8 GQA (tensor-core kernel; its cluster form runs one CTA per SM with an 8-stage ring and one
  // or two consumer groups): the cluster merge up to N = 16K (N = 4096 from 64 units on), where it
  // measured faster than partials + combine (us per call, combine -> cluster; Hkv = 8): D = 64,
  // N = 640 / 4096 / 16384: batch 1 5.76 -> 3.99, 7.85 -> 5.52, 11.58 -> 9.89; batch 4 6.79 ->
  // 4.64, 9.30 -> 7.44, 21.10 -> 17.72; batch 8 9.02 -> 5.24, 10.71 -> 10.89; D = 128: batch 1
  // 8.47 -> 4.69, 11.93 -> 7.88, 17.28 -> 15.47; batch 4 8.65 -> 5.85, 14.98 -> 11.40, 32.46 ->
  // 31.00; batch 8 10.04 -> 6.87, 21.10 -> 17.70.  At N = 64K partials + combine stay faster
  // (batch 1, D = 128: 37.2 against 47.3).
  const bool i8_small = !f16 && a.N <= 16384 && (units0 < 64 || a.N <= 4096);
  const bool auto_ok = f16 ? (a.N <= short_n ? true : (a.D == 128 && se > 1)) : i8_small;
  if ((f16 || a.fmt == KvFormat::I8Gqa) && a.tp.world == 0 && mode != FQKV_SPLIT_COMBINE &&
      (mode == FQKV_SPLIT_CLUSTER || auto_ok) && units0 < ds.sm_count) {
    int64_t sc = std::min<int64_t>({16, tiles, std::max<int64_t>(1, ds.sm_count / units0)});
    if (S_fixed > 0) sc = std::min<int64_t>(sc, S_fixed);
    const int di = a.D == 128 ? 1 : 0;
    const int(&max_cl)[17] = f16 ? ds.max_clusters_f16[di] : ds.max_clusters_qtc[di];
    // the largest cluster size (<= sc) whose clusters are all resident at once
    int64_t cct = 0, cse = 0;
    const int64_t sc0 = sc;
    for (; sc >= 2; --sc) {
      geometry(sc, &cct, &cse);
      if (cse >= 2 && units0 <= max_cl[cse]) break;
    }
    const bool reduced = sc < sc0;
    const bool f16_ok = f16 && (a.N <= short_n || (!reduced && 2 * units0 * cse >= ds.sm_count));
    if (sc >= 2 && cse >= 2 && units0 <= max_cl[cse] && (mode == FQKV_SPLIT_CLUSTER || f16_ok || i8_small)) {
      ct = cct;
      se = cse;
      a.cluster = int(cse);
    }
  }
  if (!a.cluster && ws_limited && se > 1 && partial_bytes(rows, se, a.D) > ws_bytes) geometry(best_split(true), &ct, &se);
  a.S = S_fixed > 0 ? int(S_fixed) : int(se);   // partial-slot stride per row
  a.S_eff = int(se);
  a.chunk = int(ct * TK);
  const int64_t units = units0 * a.S_eff;
  a.units = int(units);
  a.grid = a.cluster ? int(units) : int(std::min<int64_t>(units, C));
}

bool aligned(const void* p, uintptr_t n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; }

int check_W(int64_t W) {
  if (W != 2 && W != 4 && W != 8) return fail(FQKV_ERR_INVALID_ARGUMENT, "W: must be 2, 4 or 8 (got %lld)", (long long)W);
  return FQKV_OK;
}
int check_D(int64_t D) {
  if (D != 64 && D != 128) return fail(FQKV_ERR_INVALID_ARGUMENT, "D: head_dim must be 64 or 128 (got %lld)", (long long)D);
  return FQKV_OK;
}

int launch(DecodeLaunch& a, cudaStream_t stream) {
  cudaError_t e = a.fmt == KvFormat::F16     ? fqkv::launch_decode_f16(a, stream)
                  : (a.fmt == KvFormat::I8Gqa || a.fmt == KvFormat::I4Tc) ? fqkv::launch_decode_qtc(a, stream)
                                             : fqkv::launch_decode_quant(a, stream);
  if (e != cudaSuccess) return cuda_fail(e, "launch");
  if (a.S_eff > 1 && !a.cluster) {
    e = fqkv::launch_combine(a, stream);
    if (e != cudaSuccess) return cuda_fail(e, "combine launch");
  }
  return FQKV_OK;
}

// Shared body of the four decode entry points (canonical GQA form).
// kv_stride: keys between consecutive (b, kv head) rows (N for dense tensors,
// the cache capacity for a KV cache); n_dev: optional device-side valid length.
int run_decode(KvFormat fmt, const void* q, const void* K, const void* V, const void* Ks, const void* Vs, void* o,
               int64_t B, int64_t Hq, int64_t Hkv, int64_t N, int64_t D, void* ws, size_t ws_bytes,
               fqkv_stream_t stream, int64_t kv_stride = -1, const int* n_dev = nullptr,
               const fqkv_tp_out_t* tp = nullptr, bool out_bf16 = false) {
  if (kv_stride < 0) kv_stride = N;
  if (int rc = check_D(D)) return rc;
  if (B < 0 || Hq < 1 || Hkv < 1 || N < 0) return fail(FQKV_ERR_INVALID_ARGUMENT, "negative or zero size");
  if (Hq % Hkv != 0) return fail(FQKV_ERR_INVALID_ARGUMENT, "Hq (%lld) must be a multiple of Hkv (%lld)", (long long)Hq, (long long)Hkv);
  if (fmt == KvFormat::I4 && Hq != Hkv)
    return fail(FQKV_ERR_INVALID_ARGUMENT, "int4 KV supports one query head per KV head (Hq == Hkv)");
  if (B == 0) return FQKV_OK;
  if (N == 0) return fail(FQKV_ERR_INVALID_ARGUMENT, "N: the KV cache is empty (softmax over zero keys)");
  if (!q || !K || !V || (!o && !tp) || (fmt != KvFormat::F16 && (!Ks || !Vs)))
    return fail(FQKV_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (B * Hkv > INT32_MAX || N > INT32_MAX || B * Hq > INT32_MAX)
    return fail(FQKV_ERR_INVALID_ARGUMENT, "sizes exceed the 32-bit index range");
  if (!aligned(K, 16) || !aligned(V, 16)) return fail(FQKV_ERR_MISALIGNED, "K/V must be 16-byte aligned");
  if (!aligned(q, 4) || !aligned(o, 4)) return fail(FQKV_ERR_MISALIGNED, "q/out must be 4-byte aligned");
  if ((Ks && !aligned(Ks, 2)) || (Vs && !aligned(Vs, 2))) return fail(FQKV_ERR_MISALIGNED, "scales must be 2-byte aligned");

  DeviceState* ds = nullptr;
  if (int rc = device_state(&ds)) return rc;
  DecodeLaunch a{};
  a.fmt = fmt;
  a.q = q; a.K = K; a.V = V; a.Ks = Ks; a.Vs = Vs; a.out = o;
  a.B = int(B); a.Hq = int(Hq); a.Hkv = int(Hkv); a.N = int(N); a.D = int(D);
  a.kv_stride = int(kv_stride);
  a.n_dev = n_dev;
  a.out_bf16 = out_bf16;
  if (tp) {
    a.tp.world = tp->world;
    a.tp.rank = tp->rank;
    a.tp.dst_off = tp->dst_offset;
    for (int p = 0; p < tp->world; ++p) {
      a.tp.dst[p] = static_cast<__half_raw*>(tp->dst[p]);
      a.tp.cnt[p] = tp->counters[p];
    }
  }
  plan(a, *ds, 0, ws ? ws_bytes : 0, true);
  if (int64_t(a.B) * a.Hkv * a.groups * a.S_eff > INT32_MAX) return fail(FQKV_ERR_INVALID_ARGUMENT, "too many work units");
  if (a.S_eff > 1 && !a.cluster) {
    if (!aligned(ws, 16)) return fail(FQKV_ERR_MISALIGNED, "workspace must be 16-byte aligned");
    carve_partials(a, ws, int64_t(a.B) * a.Hq);
  }
  if (a.fmt == KvFormat::F16) {
    if (int rc = make_kv_map(&a.tmK, K, B * Hkv, N, D, kv_stride)) return rc;
    if (int rc = make_kv_map(&a.tmV, V, B * Hkv, N, D, kv_stride)) return rc;
  } else if (a.fmt == KvFormat::I8Gqa || a.fmt == KvFormat::I4Tc) {
    const int64_t rb = fqkv::kv_row_bytes(a.fmt, D);
    const int tk = fqkv::tile_keys(a.fmt, D);
    if (int rc = make_kv_map_codes(&a.tmK, K, B * Hkv, N, rb, kv_stride, tk)) return rc;
    if (int rc = make_kv_map_codes(&a.tmV, V, B * Hkv, N, rb, kv_stride, tk)) return rc;
  }
  return launch(a, reinterpret_cast<cudaStream_t>(stream));
}

}  // namespace

namespace fqkv {
// Records `msg` as the calling thread's fqkv_last_error() text; returns `code`.
int record_error(int code, const char* msg) { return fail(code, "%s", msg); }
}  // namespace fqkv

extern "C" {

const char* fqkv_last_error(void) { return t_err; }

const char* fqkv_version(void) { return "fqkv_b200 0.1.0 (sm_100a)"; }

void fqkv_set_wait_timeout_ms(uint32_t ms) { g_timeout_ns.store(uint64_t(ms) * 1000000ull); }

void fqkv_debug_skip_loads(int enable) { g_debug_skip_loads.store(enable ? 1 : 0); }

int fqkv_set_split_mode(int mode) {
  if (mode != FQKV_SPLIT_AUTO && mode != FQKV_SPLIT_COMBINE && mode != FQKV_SPLIT_CLUSTER)
    return fail(FQKV_ERR_INVALID_ARGUMENT, "split mode: FQKV_SPLIT_AUTO, _COMBINE or _CLUSTER (got %d)", mode);
  g_split_mode.store(mode);
  return FQKV_OK;
}

int fqkv_device_status(int* status_out, int clear) {
  if (!status_out) return fail(FQKV_ERR_INVALID_ARGUMENT, "status_out is null");
  DeviceState* ds = nullptr;
  if (int rc = device_state(&ds)) return rc;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  e = cudaMemcpy(status_out, ds->status, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "read status");
  if (clear) {
    e = cudaMemset(ds->status, 0, sizeof(int));
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "clear status");
  }
  return FQKV_OK;
}

size_t fqkv_decode_workspace_bytes(int kv_format, int64_t B, int64_t Hq, int64_t Hkv, int64_t N, int64_t D) {
  if (kv_format < 0 || kv_format > 2 || B <= 0 || Hq < 1 || Hkv < 1 || N < 1 || (D != 64 && D != 128) ||
      Hq % Hkv != 0)
    return 0;
  DeviceState* ds = nullptr;
  if (device_state(&ds) != FQKV_OK) return 0;
  DecodeLaunch a{};
  a.fmt = static_cast<KvFormat>(kv_format);
  a.B = int(B); a.Hq = int(Hq); a.Hkv = int(Hkv); a.N = int(N); a.D = int(D);
  plan(a, *ds, 0, 0, false);
  return (a.S_eff > 1 && !a.cluster) ? partial_bytes(B * Hq, a.S_eff, D) : 0;
}

int fqkv_device_info(int32_t* info, int32_t n) {
  if (!info || n < 1) return fail(FQKV_ERR_INVALID_ARGUMENT, "device_info: need an output array");
  DeviceState* ds = nullptr;
  if (int rc = device_state(&ds)) return rc;
  int32_t v[FQKV_DEVICE_INFO_LEN];
  v[0] = ds->sm_count;
  v[1] = ds->occ_f16[1];
  v[2] = ds->occ_f16[0];
  for (int c = 2; c <= 16; ++c) {
    v[3 + (c - 2)] = ds->max_clusters_f16[1][c];
    v[18 + (c - 2)] = ds->max_clusters_f16[0][c];
  }
  for (int i = 0; i < n && i < FQKV_DEVICE_INFO_LEN; ++i) info[i] = v[i];
  return FQKV_OK;
}

int fqkv_decode_plan(int kv_format, int64_t B, int64_t Hq, int64_t Hkv, int64_t N, int64_t D, size_t workspace_bytes,
                     int32_t* plan_out) {
  if (!plan_out) return fail(FQKV_ERR_INVALID_ARGUMENT, "plan_out is null");
  if (kv_format < 0 || kv_format > 2 || B <= 0 || Hq < 1 || Hkv < 1 || N < 1 || (D != 64 && D != 128) ||
      Hq % Hkv != 0 || (kv_format == FQKV_KV_INT4 && Hq != Hkv) || B * Hkv > INT32_MAX || N > INT32_MAX)
    return fail(FQKV_ERR_INVALID_ARGUMENT, "decode_plan: bad kv_format or sizes");
  DeviceState* ds = nullptr;
  if (int rc = device_state(&ds)) return rc;
  DecodeLaunch a{};
  a.fmt = static_cast<KvFormat>(kv_format);
  a.B = int(B); a.Hq = int(Hq); a.Hkv = int(Hkv); a.N = int(N); a.D = int(D);
  plan(a, *ds, 0, workspace_bytes, true);
  plan_out[0] = a.S_eff;
  plan_out[1] = a.cluster;
  plan_out[2] = a.grid;
  plan_out[3] = a.chunk;
  plan_out[4] = static_cast<int32_t>(a.fmt);
  return FQKV_OK;
}

int fqkv_decode_attn_fp16_mw(const void* q, const void* K, const void* V, void* o, int64_t R, int64_t N,
                             int64_t D, int64_t W, void* workspace, size_t workspace_bytes, fqkv_stream_t stream) {
  if (int rc = check_W(W)) return rc;
  return run_decode(KvFormat::F16, q, K, V, nullptr, nullptr, o, R, 1, 1, N, D, workspace, workspace_bytes, stream);
}

int fqkv_decode_attn_int8_mw(const void* q, const void* Kq, const void* Vq, const void* Ks, const void* Vs, void* o,
                             int64_t R, int64_t N, int64_t D, int64_t W, void* workspace, size_t workspace_bytes,
                             fqkv_stream_t stream) {
  if (int rc = check_W(W)) return rc;
  return run_decode(KvFormat::I8, q, Kq, Vq, Ks, Vs, o, R, 1, 1, N, D, workspace, workspace_bytes, stream);
}

int fqkv_decode_attn_int4(const void* q, const void* Kp, const void* Vp, const void* Ks, const void* Vs, void* o,
                          int64_t R, int64_t N, int64_t D, int64_t W, void* workspace, size_t workspace_bytes,
                          fqkv_stream_t stream) {
  if (int rc = check_W(W)) return rc;
  return run_decode(KvFormat::I4, q, Kp, Vp, Ks, Vs, o, R, 1, 1, N, D, workspace, workspace_bytes, stream);
}

int fqkv_decode_attn_gqa(const void* q, const void* K, const void* V, void* o, int64_t B, int64_t Hq, int64_t Hkv,
                         int64_t N, int64_t D, int64_t W, void* workspace, size_t workspace_bytes,
                         fqkv_stream_t stream) {
  if (int rc = check_W(W)) return rc;
  return run_decode(KvFormat::F16, q, K, V, nullptr, nullptr, o, B, Hq, Hkv, N, D, workspace, workspace_bytes,
                    stream);
}

int fqkv_decode_attn_gqa_kvcache(const void* q, const void* K, const void* V, void* o, int64_t B, int64_t Hq,
                                 int64_t Hkv, int64_t max_len, int64_t D, int64_t n_host, const int32_t* seq_len_dev,
                                 void* workspace, size_t workspace_bytes, fqkv_stream_t stream) {
  if (max_len < 1) return fail(FQKV_ERR_INVALID_ARGUMENT, "max_len must be >= 1");
  if (!seq_len_dev && (n_host < 1 || n_host > max_len))
    return fail(FQKV_ERR_INVALID_ARGUMENT, "n: valid length %lld outside [1, max_len=%lld]", (long long)n_host,
                (long long)max_len);
  if (max_len > INT32_MAX) return fail(FQKV_ERR_INVALID_ARGUMENT, "sizes exceed the 32-bit index range");
  if (seq_len_dev && !aligned(seq_len_dev, 4)) return fail(FQKV_ERR_MISALIGNED, "seq_len must be 4-byte aligned");
  // Host length: plan for exactly n keys.  Device length: plan for max_len and
  // let the kernel stop at the length it reads.
  const int64_t N = seq_len_dev ? max_len : n_host;
  return run_decode(KvFormat::F16, q, K, V, nullptr, nullptr, o, B, Hq, Hkv, N, D, workspace, workspace_bytes,
                    stream, max_len, reinterpret_cast<const int*>(seq_len_dev));
}

int fqkv_decode_attn_gqa_int8(const void* q, const void* Kq, const void* Vq, const void* Ks, const void* Vs, void* o,
                              int64_t B, int64_t Hq, int64_t Hkv, int64_t N, int64_t D, void* workspace,
                              size_t workspace_bytes, fqkv_stream_t stream) {
  return run_decode(KvFormat::I8, q, Kq, Vq, Ks, Vs, o, B, Hq, Hkv, N, D, workspace, workspace_bytes, stream);
}

int fqkv_decode_attn_gqa_int8_kvcache(const void* q, const void* Kq, const void* Vq, const void* Ks, const void* Vs,
                                      void* o, int64_t B, int64_t Hq, int64_t Hkv, int64_t max_len, int64_t D,
                                      int64_t n_host, const int32_t* seq_len_dev, void* workspace,
                                      size_t workspace_bytes, fqkv_stream_t stream) {
  if (max_len < 1) return fail(FQKV_ERR_INVALID_ARGUMENT, "max_len must be >= 1");
  if (!seq_len_dev && (n_host < 1 || n_host > max_len))
    return fail(FQKV_ERR_INVALID_ARGUMENT, "n: valid length %lld outside [1, max_len=%lld]", (long long)n_host,
                (long long)max_len);
  if (max_len > INT32_MAX) return fail(FQKV_ERR_INVALID_ARGUMENT, "sizes exceed the 32-bit index range");
  if (seq_len_dev && !aligned(seq_len_dev, 4)) return fail(FQKV_ERR_MISALIGNED, "seq_len must be 4-byte aligned");
  const int64_t N = seq_len_dev ? max_len : n_host;
  return run_decode(KvFormat::I8, q, Kq, Vq, Ks, Vs, o, B, Hq, Hkv, N, D, workspace, workspace_bytes, stream,
                    max_len, reinterpret_cast<const int*>(seq_len_dev));
}

static fqkv::QuantCtl quant_ctl(const DeviceState& ds) {
  return fqkv::QuantCtl{ds.sm_count * std::max(1, ds.occ_quantize), ds.status, g_timeout_ns.load(),
                        g_debug_skip_loads.load()};
}

static int run_quantize_into(bool int4, const void* X, void* codes, void* scales, int64_t groups, int64_t T,
                             int64_t D, int64_t cap, int64_t pos_host, const int32_t* pos_dev,
                             fqkv_stream_t stream) {
  if (D != 64 && D != 128) return fail(FQKV_ERR_INVALID_ARGUMENT, "D: head_dim must be 64 or 128 (got %lld)", (long long)D);
  if (groups < 0 || T < 0 || cap < 1) return fail(FQKV_ERR_INVALID_ARGUMENT, "negative size or empty cache");
  if (!pos_dev && (pos_host < 0 || pos_host + T > cap))
    return fail(FQKV_ERR_INVALID_ARGUMENT, "pos: tokens [%lld, %lld) outside the cache capacity %lld",
                (long long)pos_host, (long long)(pos_host + T), (long long)cap);
  if (groups == 0 || T == 0) return FQKV_OK;
  if (!X || !codes || !scales) return fail(FQKV_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (!aligned(X, 16)) return fail(FQKV_ERR_MISALIGNED, "X must be 16-byte aligned");
  if (!aligned(codes, int4 ? 4 : 8) || !aligned(scales, 2)) return fail(FQKV_ERR_MISALIGNED, "cache misaligned");
  if (pos_dev && !aligned(pos_dev, 4)) return fail(FQKV_ERR_MISALIGNED, "pos must be 4-byte aligned");
  if (groups * T > (int64_t(1) << 40)) return fail(FQKV_ERR_INVALID_ARGUMENT, "too many tokens");
  DeviceState* ds = nullptr;
  if (int rc = device_state(&ds)) return rc;
  cudaError_t e = fqkv::launch_quantize_into(int4, X, codes, scales, groups, T, int(D), cap, pos_host,
                                             reinterpret_cast<const int*>(pos_dev), quant_ctl(*ds),
                                             reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "quantize launch");
  return FQKV_OK;
}

int fqkv_quantize_int8_into_cache(const void* X, void* codes, void* scales, int64_t groups, int64_t T, int64_t D,
                                  int64_t cap, int64_t pos_host, const int32_t* pos_dev, fqkv_stream_t stream) {
  return run_quantize_into(false, X, codes, scales, groups, T, D, cap, pos_host, pos_dev, stream);
}

int fqkv_quantize_int4_into_cache(const void* X, void* packed, void* scales, int64_t groups, int64_t T, int64_t D,
                                  int64_t cap, int64_t pos_host, const int32_t* pos_dev, fqkv_stream_t stream) {
  return run_quantize_into(true, X, packed, scales, groups, T, D, cap, pos_host, pos_dev, stream);
}

int fqkv_gqa_sk_fast(const void* q, const void* K, const void* V, float* m_part, float* l_part, float* o_part,
                     void* out, int64_t Hq, int64_t Hkv, int64_t N, int64_t D, int64_t S, int64_t W, int64_t CW,
                     fqkv_stream_t stream) {
  if (int rc = check_W(W)) return rc;
  if (CW != 4 && CW != 8) return fail(FQKV_ERR_INVALID_ARGUMENT, "CW: must be 4 or 8 (got %lld)", (long long)CW);
  if (S < 1 || S > (1 << 20)) return fail(FQKV_ERR_INVALID_ARGUMENT, "S: split count must be in [1, 2^20] (got %lld)", (long long)S);
  if (int rc = check_D(D)) return rc;
  if (Hq < 1 || Hkv < 1 || N < 0) return fail(FQKV_ERR_INVALID_ARGUMENT, "negative or zero size");
  if (Hq % Hkv != 0) return fail(FQKV_ERR_INVALID_ARGUMENT, "Hq (%lld) must be a multiple of Hkv (%lld)", (long long)Hq, (long long)Hkv);
  if (N == 0) return fail(FQKV_ERR_INVALID_ARGUMENT, "N: the KV cache is empty (softmax over zero keys)");
  if (!q || !K || !V || !out || !m_part || !l_part || !o_part) return fail(FQKV_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (N > INT32_MAX) return fail(FQKV_ERR_INVALID_ARGUMENT, "sizes exceed the 32-bit index range");
  if (!aligned(K, 16) || !aligned(V, 16)) return fail(FQKV_ERR_MISALIGNED, "K/V must be 16-byte aligned");
  if (!aligned(q, 4) || !aligned(out, 4)) return fail(FQKV_ERR_MISALIGNED, "q/out must be 4-byte aligned");
  if (!aligned(m_part, 4) || !aligned(l_part, 4) || !aligned(o_part, 4)) return fail(FQKV_ERR_MISALIGNED, "partials must be 4-byte aligned");

  DeviceState* ds = nullptr;
  if (int rc = device_state(&ds)) return rc;
  DecodeLaunch a{};
  a.fmt = KvFormat::F16;
  a.q = q; a.K = K; a.V = V; a.out = out;
  a.B = 1; a.Hq = int(Hq); a.Hkv = int(Hkv); a.N = int(N); a.D = int(D);
  a.kv_stride = int(N);
  a.n_dev = nullptr;
  plan(a, *ds, S, 0, false);
  a.part_m = m_part; a.part_l = l_part; a.part_o = o_part;
  if (int rc = make_kv_map(&a.tmK, K, Hkv, N, D, N)) return rc;
  if (int rc = make_kv_map(&a.tmV, V, Hkv, N, D, N)) return rc;
  return launch(a, reinterpret_cast<cudaStream_t>(stream));
}

static int run_quantize(bool int4, const void* X, void* codes, void* scales, int64_t rows, int64_t D,
                        fqkv_stream_t stream) {
  if (rows < 0 || D < 1) return fail(FQKV_ERR_INVALID_ARGUMENT, "rows must be >= 0 and D >= 1");
  if (int4 && (D % 2)) return fail(FQKV_ERR_INVALID_ARGUMENT, "D: int4 packing needs an even head_dim (got %lld)", (long long)D);
  if (D > (1 << 20)) return fail(FQKV_ERR_INVALID_ARGUMENT, "D too large");
  if (rows == 0) return FQKV_OK;
  if (!X || !codes || !scales) return fail(FQKV_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (!aligned(X, 2) || !aligned(scales, 2)) return fail(FQKV_ERR_MISALIGNED, "X/scales must be 2-byte aligned");
  if (rows > (int64_t(1) << 40)) return fail(FQKV_ERR_INVALID_ARGUMENT, "too many rows");
  DeviceState* ds = nullptr;
  if (int rc = device_state(&ds)) return rc;
  cudaError_t e =
      fqkv::launch_quantize(int4, X, codes, scales, rows, int(D), quant_ctl(*ds), reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "quantize launch");
  return FQKV_OK;
}

int fqkv_quantize_int8_per_token(const void* X, void* codes, void* scales, int64_t rows, int64_t D,
                                 fqkv_stream_t stream) {
  return run_quantize(false, X, codes, scales, rows, D, stream);
}

int fqkv_quantize_int4_per_token(const void* X, void* packed, void* scales, int64_t rows, int64_t D,
                                 fqkv_stream_t stream) {
  return run_quantize(true, X, packed, scales, rows, D, stream);
}


// ------------------------------------------------------------------ fused RoPE + append
int fqkv_rope_qkv_append(int32_t kv_format, int32_t model_dtype, const void* qkv, int64_t qkv_row_stride,
                         const void* cos_table, const void* sin_table, int64_t table_rows, int64_t pos_host,
                         const int32_t* pos_dev, void* q_out, void* k_cache, void* v_cache, void* k_scales,
                         void* v_scales, int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t cap,
                         fqkv_stream_t stream) {
  if (kv_format != FQKV_KV_F16 && kv_format != FQKV_KV_INT8)
    return fail(FQKV_ERR_INVALID_ARGUMENT, "kv_format: FQKV_KV_F16 or FQKV_KV_INT8");
  if (model_dtype != 0 && model_dtype != 1) return fail(FQKV_ERR_INVALID_ARGUMENT, "model_dtype: 0 (f16) or 1 (bf16)");
  if (int rc = check_D(D)) return rc;
  if (B < 0 || Hq < 1 || Hkv < 1 || cap < 1 || table_rows < 1 || Hq % Hkv != 0)
    return fail(FQKV_ERR_INVALID_ARGUMENT, "bad sizes (B=%lld Hq=%lld Hkv=%lld cap=%lld table_rows=%lld)",
                (long long)B, (long long)Hq, (long long)Hkv, (long long)cap, (long long)table_rows);
  if (qkv_row_stride < (Hq + 2 * Hkv) * D)
    return fail(FQKV_ERR_INVALID_ARGUMENT, "qkv_row_stride %lld < (Hq + 2 Hkv) D", (long long)qkv_row_stride);
  if (!pos_dev && (pos_host < 0 || pos_host >= table_rows))
    return fail(FQKV_ERR_INVALID_ARGUMENT, "pos %lld outside the rotary table (%lld rows)", (long long)pos_host,
                (long long)table_rows);
  if (B == 0) return FQKV_OK;
  if (!qkv || !cos_table || !sin_table || !q_out || !k_cache || !v_cache ||
      (kv_format == FQKV_KV_INT8 && (!k_scales || !v_scales)))
    return fail(FQKV_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (!aligned(qkv, 2) || !aligned(q_out, 2) || !aligned(k_cache, 2) || !aligned(v_cache, 2) ||
      !aligned(cos_table, 2) || !aligned(sin_table, 2) || (pos_dev && !aligned(pos_dev, 4)))
    return fail(FQKV_ERR_MISALIGNED, "rope_qkv_append: misaligned pointer");
  if (B * (Hq + 2 * Hkv) > INT32_MAX / 32 || B * Hkv * cap > INT32_MAX * int64_t(64))
    return fail(FQKV_ERR_INVALID_ARGUMENT, "sizes exceed the index range");
  cudaError_t e = fqkv::launch_rope_append(model_dtype == 1, kv_format == FQKV_KV_INT8, qkv, qkv_row_stride, cos_table,
                                           sin_table, table_rows, pos_host, reinterpret_cast<const int*>(pos_dev), q_out,
                                           k_cache, v_cache, k_scales, v_scales, int(B), int(Hq), int(Hkv), int(D),
                                           int(cap), reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "rope_qkv_append launch");
  return FQKV_OK;
}

// ------------------------------------------------------------------ decode-step model helpers
int fqkv_add_rmsnorm(int32_t model_dtype, void* h, const void* delta, const void* weight, void* y, int64_t rows,
                     int64_t H, float eps, fqkv_stream_t stream) {
  if (model_dtype != 0 && model_dtype != 1) return fail(FQKV_ERR_INVALID_ARGUMENT, "model_dtype: 0 (f16) or 1 (bf16)");
  if (rows < 0 || H < 1 || H > 8192) return fail(FQKV_ERR_INVALID_ARGUMENT, "rows/H: need rows >= 0, 1 <= H <= 8192");
  if (rows > INT32_MAX) return fail(FQKV_ERR_INVALID_ARGUMENT, "rows exceed the grid range");
  if (rows == 0) return FQKV_OK;
  if (!h || !weight || !y) return fail(FQKV_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (!aligned(h, 2) || !aligned(weight, 2) || !aligned(y, 2) || (delta && !aligned(delta, 2)))
    return fail(FQKV_ERR_MISALIGNED, "add_rmsnorm: misaligned pointer");
  cudaError_t e = fqkv::launch_add_rmsnorm(model_dtype == 1, h, delta, weight, y, rows, int(H), eps,
                                           reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "add_rmsnorm launch");
  return FQKV_OK;
}

int fqkv_silu_mul(int32_t model_dtype, const void* gu, void* y, int64_t rows, int64_t I, int64_t gu_row_stride,
                  fqkv_stream_t stream) {
  if (model_dtype != 0 && model_dtype != 1) return fail(FQKV_ERR_INVALID_ARGUMENT, "model_dtype: 0 (f16) or 1 (bf16)");
  if (rows < 0 || I < 1 || I > INT32_MAX || gu_row_stride < 2 * I)
    return fail(FQKV_ERR_INVALID_ARGUMENT, "silu_mul: bad sizes (rows %lld, I %lld, stride %lld)", (long long)rows,
                (long long)I, (long long)gu_row_stride);
  if (rows == 0) return FQKV_OK;
  if (!gu || !y) return fail(FQKV_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (!aligned(gu, 2) || !aligned(y, 2)) return fail(FQKV_ERR_MISALIGNED, "silu_mul: misaligned pointer");
  cudaError_t e = fqkv::launch_silu_mul(model_dtype == 1, gu, y, rows, int(I), gu_row_stride,
                                        reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "silu_mul launch");
  return FQKV_OK;
}

int fqkv_gemv(int32_t model_dtype, int32_t x_dtype, const void* x, const void* W, const void* bias, void* y, int64_t B,
              int64_t N, int64_t K, fqkv_stream_t stream) {
  if (model_dtype != 0 && model_dtype != 1) return fail(FQKV_ERR_INVALID_ARGUMENT, "model_dtype: 0 (f16) or 1 (bf16)");
  if (x_dtype != 0 && x_dtype != model_dtype)
    return fail(FQKV_ERR_INVALID_ARGUMENT, "gemv: x_dtype is the model dtype or 0 (f16)");
  if (B < 1 || B > 4 || N < 1 || N > INT32_MAX / 2 || K < 256 || K % 256 != 0 || K > 16384)
    return fail(FQKV_ERR_INVALID_ARGUMENT, "gemv: need 1 <= B <= 4, N >= 1, K a multiple of 256 in [256, 16384]");
  if (!x || !W || !y) return fail(FQKV_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (!aligned(x, 16) || !aligned(W, 16) || !aligned(y, 2) || (bias && !aligned(bias, 2)))
    return fail(FQKV_ERR_MISALIGNED, "gemv: x and W must be 16-byte aligned");
  cudaError_t e = fqkv::launch_gemv(model_dtype == 1, x_dtype == 0, x, W, bias, y, int(B), int(N), int(K),
                                    reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "gemv launch");
  return FQKV_OK;
}

int fqkv_gemv_swiglu(int32_t model_dtype, const void* x, const void* W, const void* bias, void* y, int64_t B,
                     int64_t I, int64_t K, fqkv_stream_t stream) {
  if (model_dtype != 0 && model_dtype != 1) return fail(FQKV_ERR_INVALID_ARGUMENT, "model_dtype: 0 (f16) or 1 (bf16)");
  if (B < 1 || B > 4 || I < 1 || I > INT32_MAX / 4 || K < 256 || K % 256 != 0 || K > 16384)
    return fail(FQKV_ERR_INVALID_ARGUMENT, "gemv_swiglu: need 1 <= B <= 4, I >= 1, K a multiple of 256 in [256, 16384]");
  if (!x || !W || !y) return fail(FQKV_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (!aligned(x, 16) || !aligned(W, 16) || !aligned(y, 2) || (bias && !aligned(bias, 2)))
    return fail(FQKV_ERR_MISALIGNED, "gemv_swiglu: x and W must be 16-byte aligned");
  cudaError_t e = fqkv::launch_gemv_swiglu(model_dtype == 1, x, W, bias, y, int(B), int(I), int(K),
                                           reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "gemv_swiglu launch");
  return FQKV_OK;
}

int fqkv_gemv_rope_append(int32_t model_dtype, const void* x, const void* W, const void* bias, int64_t K,
                          const void* cos_table, const void* sin_table, int64_t table_rows, int64_t pos_host,
                          const int32_t* pos_dev, void* q_out, void* k_cache, void* v_cache, int64_t Hq, int64_t Hkv,
                          int64_t D, int64_t cap, fqkv_stream_t stream) {
  if (model_dtype != 0 && model_dtype != 1) return fail(FQKV_ERR_INVALID_ARGUMENT, "model_dtype: 0 (f16) or 1 (bf16)");
  if (int rc = check_D(D)) return rc;
  if (K < 256 || K % 256 != 0 || K > 16384)
    return fail(FQKV_ERR_INVALID_ARGUMENT, "gemv_rope_append: K must be a multiple of 256 in [256, 16384]");
  if (Hq < 1 || Hkv < 1 || Hq % Hkv != 0 || Hq + 2 * Hkv > 4096 || cap < 1 || cap > INT32_MAX || table_rows < 1)
    return fail(FQKV_ERR_INVALID_ARGUMENT, "gemv_rope_append: bad sizes (Hq=%lld Hkv=%lld cap=%lld table_rows=%lld)",
                (long long)Hq, (long long)Hkv, (long long)cap, (long long)table_rows);
  if (!pos_dev && (pos_host < 0 || pos_host >= table_rows))
    return fail(FQKV_ERR_INVALID_ARGUMENT, "pos %lld outside the rotary table (%lld rows)", (long long)pos_host,
                (long long)table_rows);
  if (!x || !W || !cos_table || !sin_table || !q_out || !k_cache || !v_cache)
    return fail(FQKV_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (!aligned(x, 16) || !aligned(W, 16) || (bias && !aligned(bias, 2)) || !aligned(cos_table, 2) ||
      !aligned(sin_table, 2) || !aligned(q_out, 2) || !aligned(k_cache, 2) || !aligned(v_cache, 2) ||
      (pos_dev && !aligned(pos_dev, 4)))
    return fail(FQKV_ERR_MISALIGNED, "gemv_rope_append: x and W must be 16-byte aligned");
  fqkv::GemvRope rp;
  rp.cos_t = cos_table;
  rp.sin_t = sin_table;
  rp.table_rows = table_rows;
  rp.pos_host = pos_host;
  rp.pos_dev = reinterpret_cast<const int*>(pos_dev);
  rp.q_out = static_cast<__half*>(q_out);
  rp.k_cache = static_cast<__half*>(k_cache);
  rp.v_cache = static_cast<__half*>(v_cache);
  rp.Hq = int(Hq);
  rp.Hkv = int(Hkv);
  rp.D = int(D);
  rp.cap = int(cap);
  cudaError_t e = fqkv::launch_gemv_rope_append(model_dtype == 1, x, W, bias, int(K), rp,
                                                reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "gemv_rope_append launch");
  return FQKV_OK;
}

size_t fqkv_argmax_scratch_bytes(int64_t rows) { return rows > 0 ? fqkv::argmax_scratch_bytes(rows) : 0; }

int fqkv_argmax(int32_t model_dtype, const void* logits, int64_t rows, int64_t V, void* scratch, int64_t* idx,
                fqkv_stream_t stream) {
  if (model_dtype != 0 && model_dtype != 1) return fail(FQKV_ERR_INVALID_ARGUMENT, "model_dtype: 0 (f16) or 1 (bf16)");
  if (rows < 0 || rows > 65535 || V < 1 || V > INT32_MAX) return fail(FQKV_ERR_INVALID_ARGUMENT, "argmax: bad sizes");
  if (rows == 0) return FQKV_OK;
  if (!logits || !scratch || !idx) return fail(FQKV_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (!aligned(logits, 2) || !aligned(scratch, 4) || !aligned(idx, 8))
    return fail(FQKV_ERR_MISALIGNED, "argmax: misaligned pointer");
  cudaError_t e = fqkv::launch_argmax(model_dtype == 1, logits, rows, int(V), scratch, idx,
                                      reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "argmax launch");
  return FQKV_OK;
}

// ------------------------------------------------------------------ tensor-parallel decode
int fqkv_decode_attn_kvcache_out(int32_t kv_format, int32_t out_dtype, const void* q, const void* K, const void* V,
                                 const void* Ks, const void* Vs, void* o, int64_t B, int64_t Hq, int64_t Hkv,
                                 int64_t max_len, int64_t D, int64_t n_host, const int32_t* seq_len_dev,
                                 void* workspace, size_t workspace_bytes, fqkv_stream_t stream) {
  if (kv_format != FQKV_KV_F16 && kv_format != FQKV_KV_INT8)
    return fail(FQKV_ERR_INVALID_ARGUMENT, "kv_format: FQKV_KV_F16 or FQKV_KV_INT8");
  if (out_dtype != 0 && out_dtype != 1) return fail(FQKV_ERR_INVALID_ARGUMENT, "out_dtype: 0 (f16) or 1 (bf16)");
  if (max_len < 1) return fail(FQKV_ERR_INVALID_ARGUMENT, "max_len must be >= 1");
  if (!seq_len_dev && (n_host < 1 || n_host > max_len))
    return fail(FQKV_ERR_INVALID_ARGUMENT, "n: valid length %lld outside [1, max_len=%lld]", (long long)n_host,
                (long long)max_len);
  if (max_len > INT32_MAX) return fail(FQKV_ERR_INVALID_ARGUMENT, "sizes exceed the 32-bit index range");
  if (seq_len_dev && !aligned(seq_len_dev, 4)) return fail(FQKV_ERR_MISALIGNED, "seq_len must be 4-byte aligned");
  const int64_t N = seq_len_dev ? max_len : n_host;
  return run_decode(kv_format == FQKV_KV_INT8 ? KvFormat::I8 : KvFormat::F16, q, K, V, Ks, Vs, o, B, Hq, Hkv, N, D,
                    workspace, workspace_bytes, stream, max_len, reinterpret_cast<const int*>(seq_len_dev), nullptr,
                    out_dtype == 1);
}

int fqkv_decode_attn_kvcache_tp(int32_t kv_format, const void* q, const void* K, const void* V, const void* Ks,
                                const void* Vs, int64_t B, int64_t Hq, int64_t Hkv, int64_t max_len, int64_t D,
                                int64_t n_host, const int32_t* seq_len_dev, void* workspace, size_t workspace_bytes,
                                const fqkv_tp_out_t* tp, fqkv_stream_t stream) {
  if (kv_format != FQKV_KV_F16 && kv_format != FQKV_KV_INT8)
    return fail(FQKV_ERR_INVALID_ARGUMENT, "kv_format: tensor-parallel decode takes FQKV_KV_F16 or FQKV_KV_INT8");
  if (!tp) return fail(FQKV_ERR_INVALID_ARGUMENT, "tp: null tensor-parallel output descriptor");
  if (tp->world < 2 || tp->world > FQKV_TP_MAX_RANKS || tp->rank < 0 || tp->rank >= tp->world)
    return fail(FQKV_ERR_INVALID_ARGUMENT, "tp: world %d / rank %d outside 2..%d", int(tp->world), int(tp->rank),
                FQKV_TP_MAX_RANKS);
  if (tp->dst_offset < 0) return fail(FQKV_ERR_INVALID_ARGUMENT, "tp: negative dst_offset");
  for (int p = 0; p < tp->world; ++p) {
    if (!tp->dst[p] || !tp->counters[p]) return fail(FQKV_ERR_INVALID_ARGUMENT, "tp: null buffer of rank %d", p);
    if (!aligned(tp->dst[p], 16) || !aligned(tp->counters[p], 8))
      return fail(FQKV_ERR_MISALIGNED, "tp: buffer of rank %d misaligned (dst 16 B, counters 8 B)", p);
  }
  if (max_len < 1) return fail(FQKV_ERR_INVALID_ARGUMENT, "max_len must be >= 1");
  if (!seq_len_dev && (n_host < 1 || n_host > max_len))
    return fail(FQKV_ERR_INVALID_ARGUMENT, "n: valid length %lld outside [1, max_len=%lld]", (long long)n_host,
                (long long)max_len);
  if (max_len > INT32_MAX) return fail(FQKV_ERR_INVALID_ARGUMENT, "sizes exceed the 32-bit index range");
  if (seq_len_dev && !aligned(seq_len_dev, 4)) return fail(FQKV_ERR_MISALIGNED, "seq_len must be 4-byte aligned");
  const int64_t N = seq_len_dev ? max_len : n_host;
  const KvFormat fmt = kv_format == FQKV_KV_F16 ? KvFormat::F16 : KvFormat::I8;
  return run_decode(fmt, q, K, V, Ks, Vs, nullptr, B, Hq, Hkv, N, D, workspace, workspace_bytes, stream, max_len,
                    reinterpret_cast<const int*>(seq_len_dev), tp);
}

int64_t fqkv_tp_arrivals(int32_t kv_format, int64_t B, int64_t Hq, int64_t Hkv, int64_t max_len, int64_t D,
                         size_t workspace_bytes) {
  if ((kv_format != FQKV_KV_F16 && kv_format != FQKV_KV_INT8) || B < 1 || Hq < 1 || Hkv < 1 || max_len < 1 ||
      (D != 64 && D != 128) || Hq % Hkv != 0) {
    fail(FQKV_ERR_INVALID_ARGUMENT, "tp_arrivals: bad kv_format or sizes");
    return -1;
  }
  DeviceState* ds = nullptr;
  if (device_state(&ds) != FQKV_OK) return -1;  // device_state recorded the message
  DecodeLaunch a{};
  a.fmt = kv_format == FQKV_KV_F16 ? KvFormat::F16 : KvFormat::I8;
  a.B = int(B); a.Hq = int(Hq); a.Hkv = int(Hkv); a.N = int(max_len); a.D = int(D);
  a.tp.world = 2;  // tensor-parallel output: planned as fqkv_decode_attn_kvcache_tp plans it (no cluster mode)
  plan(a, *ds, 0, workspace_bytes, true);
  // unsplit: one arrival per unit (decode kernel epilogue); split: one per row (combine)
  return a.S_eff == 1 ? int64_t(a.units) : B * Hq;
}

int fqkv_tp_wait(const unsigned long long* counters, int32_t world, uint64_t per_call, unsigned long long* sequence,
                 fqkv_stream_t stream) {
  if (!counters || !sequence) return fail(FQKV_ERR_INVALID_ARGUMENT, "null counters / sequence");
  if (world < 1 || world > FQKV_TP_MAX_RANKS)
    return fail(FQKV_ERR_INVALID_ARGUMENT, "world %d outside 1..%d", int(world), FQKV_TP_MAX_RANKS);
  if (!aligned(counters, 8) || !aligned(sequence, 8)) return fail(FQKV_ERR_MISALIGNED, "counters / sequence: 8 B");
  DeviceState* ds = nullptr;
  if (int rc = device_state(&ds)) return rc;
  cudaError_t e = fqkv::launch_tp_wait(counters, int(world), per_call, sequence, ds->status, g_timeout_ns.load(),
                                       reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "tp wait launch");
  return FQKV_OK;
}

int fqkv_ipc_alloc(size_t bytes, void** dev_ptr, void* ipc_handle) {
  if (!dev_ptr || !ipc_handle || bytes == 0) return fail(FQKV_ERR_INVALID_ARGUMENT, "ipc_alloc: bad argument");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "ipc_alloc: cudaMalloc");
  e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "ipc_alloc: zero fill / handle");
  }
  std::memcpy(ipc_handle, &h, sizeof(h));
  *dev_ptr = p;
  return FQKV_OK;
}

int fqkv_ipc_open(const void* ipc_handle, void** dev_ptr) {
  if (!dev_ptr || !ipc_handle) return fail(FQKV_ERR_INVALID_ARGUMENT, "ipc_open: bad argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(FQKV_ERR_PEER, "ipc_open: %s", cudaGetErrorString(e));
  }
  *dev_ptr = p;
  return FQKV_OK;
}

int fqkv_ipc_close(void* dev_ptr) {
  if (!dev_ptr) return fail(FQKV_ERR_INVALID_ARGUMENT, "ipc_close: null pointer");
  cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
  if (e != cudaSuccess) return cuda_fail(e, "ipc_close");
  return FQKV_OK;
}

int fqkv_ipc_free(void* dev_ptr) {
  if (!dev_ptr) return fail(FQKV_ERR_INVALID_ARGUMENT, "ipc_free: null pointer");
  cudaError_t e = cudaFree(dev_ptr);
  if (e != cudaSuccess) return cuda_fail(e, "ipc_free");
  return FQKV_OK;
}

}  // extern "C"
