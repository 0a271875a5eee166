// fqkv_gqa_sk_fast_static_scratch: the split-K GQA decode for callers that
// cannot allocate device memory.
//
// Who needs it: code that runs where device allocation is not allowed or not
// affordable -- an op called from a serving runtime's enqueue / plugin hook
// whose host framework owns every byte of device memory and forbids
// allocating inside the op, a decode loop that must not stall (cudaMalloc can
// synchronise the device), or a plain C host with no allocator to manage a
// workspace's lifetime.  gqa_sk_fast asks its caller for three fp32 scratch
// tensors; this variant takes none and instead uses one fixed array that the
// library itself places in device memory.
//
// The scratch: g_sk_static_scratch, kStaticScratchBytes (4 MiB) per GPU that
// loads the library, held until the process exits.  It stores the per-split
// partials m [Hq,S], l [Hq,S] (each padded to 256 bytes) and o [Hq,S,D] fp32,
// so a call needs 2*pad256(4*Hq*S) + 4*Hq*S*D bytes; larger requests are
// rejected with FQKV_ERR_INVALID_ARGUMENT and nothing is launched.  Nothing in
// it has to start at zero: every partial the combine reads is written earlier
// in the same call.  All calls on a device share the array and it keeps the
// last call's contents, so calls whose kernels overlap on the GPU (different
// streams with no ordering between them) race on it; calls on one stream are
// ordered and safe.
//
// Set-up: host code cannot use the array's name as a device address (in host
// code it is only a stand-in symbol).  The first call on each device, with
// that device current, resolves the real address with cudaGetSymbolAddress
// and caches it; make that first call before any stream capture begins on the
// device.  Only a successful lookup is cached: if it fails (e.g. the first
// call came during a capture, or the context was not ready), the call
// returns FQKV_ERR_CUDA and the next call on that device tries again.  A
// device reset (cudaDeviceReset) is not supported: the cached address would
// belong to the destroyed context.  No cudaMalloc, cudaFree or allocating library
// routine is called here or in the launch path it reuses (fqkv_gqa_sk_fast).
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <mutex>

#include "../../include/fqkv_b200.h"

namespace fqkv {
int record_error(int code, const char* msg);  // capi.cu
}

namespace {

constexpr size_t kStaticScratchBytes = size_t(4) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_sk_static_scratch[kStaticScratchBytes];

// Device address of g_sk_static_scratch per device, set once a lookup succeeds.
std::mutex g_addr_mu;
void* g_addr[kMaxDevices] = {};

// Cached address of the array on device `dev` (current), looked up on first use;
// a failed lookup is not cached, so a later call retries it.
cudaError_t scratch_address(int dev, void** out) {
  std::lock_guard<std::mutex> lock(g_addr_mu);
  if (g_addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_sk_static_scratch);
    if (e != cudaSuccess || p == nullptr) return e != cudaSuccess ? e : cudaErrorInvalidSymbol;
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return cudaSuccess;
}

size_t pad256(size_t n) { return (n + 255) & ~size_t(255); }

}  // namespace

extern "C" int fqkv_gqa_sk_fast_static_scratch(const void* q, const void* K, const void* V, void* out, int64_t Hq,
                                               int64_t Hkv, int64_t N, int64_t D, int64_t S, int64_t W, int64_t CW,
                                               fqkv_stream_t stream) {
  char msg[320];
  if (Hq < 1 || S < 1 || (D != 64 && D != 128)) {
    snprintf(msg, sizeof(msg),
             "static-scratch split-K: need Hq >= 1, S >= 1 and D in {64,128} (got Hq=%lld S=%lld D=%lld)",
             (long long)Hq, (long long)S, (long long)D);
    return fqkv::record_error(FQKV_ERR_INVALID_ARGUMENT, msg);
  }
  if (Hq > (int64_t(1) << 20) || S > (int64_t(1) << 20))
    return fqkv::record_error(FQKV_ERR_INVALID_ARGUMENT, "static-scratch split-K: Hq or S too large");
  const size_t ml = pad256(size_t(Hq) * size_t(S) * sizeof(float));
  const size_t need = 2 * ml + size_t(Hq) * size_t(S) * size_t(D) * sizeof(float);
  if (need > kStaticScratchBytes) {
    snprintf(msg, sizeof(msg),
             "static-scratch split-K: Hq=%lld x S=%lld x D=%lld needs %zu bytes of split scratch, more than the "
             "%zu-byte static array; lower S or use fqkv_gqa_sk_fast with caller scratch",
             (long long)Hq, (long long)S, (long long)D, need, kStaticScratchBytes);
    return fqkv::record_error(FQKV_ERR_INVALID_ARGUMENT, msg);
  }
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    snprintf(msg, sizeof(msg), "static-scratch split-K: cudaGetDevice: %s", cudaGetErrorString(e));
    return fqkv::record_error(FQKV_ERR_CUDA, msg);
  }
  void* addr = nullptr;
  e = scratch_address(dev, &addr);
  if (e != cudaSuccess) {
    snprintf(msg, sizeof(msg), "static-scratch split-K: cudaGetSymbolAddress failed: %s (retried on the next call)",
             cudaGetErrorString(e));
    return fqkv::record_error(FQKV_ERR_CUDA, msg);
  }
  unsigned char* base = static_cast<unsigned char*>(addr);
  float* m_part = reinterpret_cast<float*>(base);
  float* l_part = reinterpret_cast<float*>(base + ml);
  float* o_part = reinterpret_cast<float*>(base + 2 * ml);
  return fqkv_gqa_sk_fast(q, K, V, m_part, l_part, o_part, out, Hq, Hkv, N, D, S, W, CW, stream);
}
