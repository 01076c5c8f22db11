// pdl.cuh — programmatic dependent launch and last-CTA helpers.
//
// Every decode kernel is launched with programmatic stream serialization, so
// it can be resident while its predecessor runs. Its code is split in two:
// before pdl_wait() it may only touch data that existed before the
// predecessor started (weights, older KV-cache rows, and outputs of kernels
// two or more launches back, read through L2 with __ldcg); after pdl_wait()
// the predecessor has completed and its writes are visible. Each kernel calls
// pdl_trigger() right after its own pdl_wait(), so when its successor starts,
// every kernel before this one has completed.
#pragma once

#include <cuda_runtime.h>

#include <utility>

#include "common.cuh"

namespace chalot {

CHALOT_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
CHALOT_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// True in exactly one CTA of the grid (or of the n CTAs sharing `counter`):
// the last one to get here. The other CTAs' global writes made before their
// call are visible to it (read them with __ldcg). Resets the counter for the
// next launch.
// The CTA barrier orders the CTA's writes before thread 0's device-scope
// fence and ticket (the pattern of a cooperative grid barrier).
__device__ __forceinline__ bool last_cta(unsigned* counter, unsigned n = 0) {
  __shared__ bool is_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (n == 0) n = gridDim.x * gridDim.y * gridDim.z;
    const unsigned t = atomicAdd(counter, 1u);
    is_last = (t == n - 1);
    if (is_last) {
      atomicExch(counter, 0u);
      __threadfence();
    }
  }
  __syncthreads();
  return is_last;
}

// Phase trace (compile with -DCHALOT_PHASE_TRACE): thread 0 of every CTA
// stores %globaltimer at the phase boundaries of a decode kernel into
// g_phase_trace[slot][cta][phase] (slot = layer*8 + kernel kind). Normal
// builds compile the macro away.
constexpr int kTraceCtas = 1024, kTracePhases = 8, kTraceSlots = 8 * 64;
#ifdef CHALOT_PHASE_TRACE
// One copy per kernel file (no relocatable device code); each file exports
// readers through CHALOT_TRACE_EXPORT and the engine merges them.
static __device__ unsigned long long g_phase_trace[kTraceSlots * kTraceCtas * kTracePhases];
#define CHALOT_TRACE_EXPORT(name)                                                          \
  cudaError_t name(unsigned long long* dst, size_t n) {                                    \
    return cudaMemcpyFromSymbol(dst, g_phase_trace, n * sizeof(unsigned long long));       \
  }                                                                                        \
  cudaError_t name##_clear() {                                                             \
    void* p = nullptr;                                                                     \
    cudaError_t r = cudaGetSymbolAddress(&p, g_phase_trace);                               \
    return r == cudaSuccess ? cudaMemset(p, 0, sizeof(g_phase_trace)) : r;                 \
  }
#define CHALOT_TRACE(slot, phase)                                                         \
  do {                                                                                    \
    if (threadIdx.x == 0) {                                                               \
      unsigned long long t_;                                                              \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                              \
      const int cta_ = blockIdx.x + blockIdx.y * gridDim.x;                               \
      if ((slot) < kTraceSlots && cta_ < kTraceCtas)                                      \
        g_phase_trace[((size_t)(slot) * kTraceCtas + cta_) * kTracePhases + (phase)] = t_; \
    }                                                                                     \
  } while (0)
#else
#define CHALOT_TRACE(slot, phase) \
  do {                            \
  } while (0)
#endif

// Launches `k` with programmatic stream serialization when `pdl` is set.
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                     bool pdl, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k, std::forward<Args>(args)...);
}

}  // namespace chalot
