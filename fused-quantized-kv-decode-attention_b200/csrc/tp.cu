// Tensor-parallel decode: the wait that closes the fused all-gather.
//
// Each rank's decode kernel stores its attention output into every rank's
// receive buffer over NVLink and then adds one arrival per output unit to the
// counter slot for its rank on every rank (system fence, system-scope atomic;
// see store_out / signal_out in kernels.h).  This kernel, enqueued before the
// consumer of the gathered outputs, waits until each slot has reached
// (sequence + 1) * per_call, then advances the rank-local sequence number.
// Counters only grow, so no reset is ever needed and the whole decode step
// replays from one CUDA graph.  The wait is bounded: after the limit it
// records status 64 and lets the step complete.  Once any bounded wait on the
// device has given up (the status word is non-zero), later waits return at
// once: a peer that stopped never catches up, and waiting out the limit again
// in every layer of every remaining step would stall the host for minutes
// before it can read the status and raise.
//
// Kernels on different GPUs wait on one another here, never two kernels on one
// GPU: the producers are the other ranks' decode kernels.
#include <cuda_runtime.h>

#include <cstdint>

#include "device_common.cuh"
#include "kernels.h"

namespace fqkv {
namespace {

constexpr int kDevTimeoutPeer = 64;  // a peer's arrivals never came

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__global__ void tp_wait_kernel(const unsigned long long* __restrict__ counters, int world, unsigned long long per_call,
                               unsigned long long* __restrict__ sequence, int* status, unsigned long long timeout_ns) {
  const unsigned long long target = (*sequence + 1ull) * per_call;
  bool ok = true;
  // a wait on this device already gave up: the outputs of this step are void anyway
  const bool failed = *reinterpret_cast<volatile int*>(status) != kDevOk;
  if (!failed && int(threadIdx.x) < world) {
    const unsigned long long* c = counters + threadIdx.x;
    if (ld_acquire_sys(c) < target) {
      const unsigned long long t0 = globaltimer_ns();
      ok = false;
      for (uint32_t it = 1; it < (1u << 30); ++it) {
        if (ld_acquire_sys(c) >= target) {
          ok = true;
          break;
        }
        if ((it & 63u) == 0u && globaltimer_ns() - t0 > timeout_ns) break;
        __nanosleep(32);
      }
    }
  }
  ok = __syncthreads_and(ok);
  if (threadIdx.x == 0) {
    *sequence = *sequence + 1ull;
    if (!ok) atomicCAS(status, kDevOk, kDevTimeoutPeer);
  }
}

}  // namespace

cudaError_t launch_tp_wait(const unsigned long long* counters, int world, unsigned long long per_call,
                           unsigned long long* sequence, int* status, unsigned long long timeout_ns,
                           cudaStream_t stream) {
  tp_wait_kernel<<<1, 32, 0, stream>>>(counters, world, per_call, sequence, status, timeout_ns);
  return cudaGetLastError();
}

}  // namespace fqkv
