// k_peak.cu — measured peak of the int8 tensor cores (tcgen05.mma kind::i8),
// the denominator of the MoE prefill's tensor roofline.
//
// One CTA per SM keeps one M128 x N256 x K32 MMA stream going out of shared
// memory (no memory traffic): one thread issues `iters` x 4 MMAs into a
// 256-column TMEM accumulator, commits to an mbarrier and waits (bounded).
// The operands are a fixed byte pattern, not zeros, so the tensor pipes draw
// their usual power.
#include <cuda_runtime.h>

#include <string>

#include "capi_internal.h"
#include "tc.cuh"
#include "tma.cuh"

namespace chalot {
namespace {

constexpr int kPeakM = 128, kPeakN = 256, kPeakK = 32;
constexpr uint32_t kPeakIdesc = tc_idesc_i8(kPeakM, kPeakN);
// A and B tiles of 128-byte rows (1 KB aligned), padded so one CTA fits per SM
constexpr int kPeakSmem = 120 * 1024;
static_assert((kPeakM + kPeakN) * 128 + 1024 <= kPeakSmem, "operand tiles fit");

__global__ void __launch_bounds__(128, 1) k_mma_i8_peak(int iters, unsigned* err) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t done;
  __shared__ uint32_t tmem_slot;
  unsigned char* A = reinterpret_cast<unsigned char*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  unsigned char* B = A + kPeakM * 128;
  const int warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < (kPeakM + kPeakN) * 128; i += blockDim.x) A[i] = (unsigned char)(i * 37 + 11);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic stores -> tensor-core reads
  if (threadIdx.x == 0) {
    mbar_init_n(&done, 1);
    mbar_fence_init();
  }
  if (warp == 0) tc_alloc(&tmem_slot, kPeakN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  if (threadIdx.x == 0) {
    const uint32_t a0 = smem_u32(A), b0 = smem_u32(B);
    for (int i = 0; i < iters; ++i)
#pragma unroll
      for (int k = 0; k < 128 / kPeakK; ++k)
        tc_mma_i8(tmem, tc_desc_sw128(a0 + k * kPeakK), tc_desc_sw128(b0 + k * kPeakK), kPeakIdesc,
                  (i | k) != 0);
    tc_commit(&done);
    mbar_wait(&done, 0, err);  // bounded; a timeout leaves *err set
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tc_dealloc(tmem, kPeakN);
  }
}

// Self-check of libm::div_rn (the fast exact division) against the
// compiler's division: n pseudo-random pairs (splitmix64 from seed) with
// exponents in [-40, 40], both signs, plus pairs in the ranges the decode path
// divides (x / 127, x / 30, 1 / x, x / dim); counts bitwise mismatches.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
__global__ void k_div_check(uint64_t n, uint64_t seed, unsigned long long* bad, float* example) {
  unsigned long long local = 0;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t r = mix64(seed + 0x9E3779B97F4A7C15ull * (i + 1));
    const uint32_t ea = 127 - 40 + (uint32_t)((r >> 8) % 81), eb = 127 - 40 + (uint32_t)((r >> 16) % 81);
    float a = __uint_as_float((uint32_t)(r >> 63) << 31 | ea << 23 | ((uint32_t)(r >> 24) & 0x7fffff));
    float b = __uint_as_float((uint32_t)((r >> 62) & 1) << 31 | eb << 23 | ((uint32_t)(r >> 40) & 0x7fffff));
    switch (r & 7) {  // divisors of the decode path
      case 0: b = 127.0f; break;
      case 1: b = 30.0f; break;
      case 2: a = 1.0f; break;
      case 3: b = 896.0f; break;
      default: break;
    }
    const float q = libm::div_rn(a, b), ref = __fdiv_rn(a, b);
    if (__float_as_uint(q) != __float_as_uint(ref)) {
      ++local;
      example[0] = a;
      example[1] = b;
    }
  }
  if (local) atomicAdd(bad, local);
}

}  // namespace
}  // namespace chalot

extern "C" {

__attribute__((visibility("default"))) int chalot_selftest_division(uint64_t n, uint64_t seed, uint64_t* mismatches,
                                                                    float* example) {
  using namespace chalot;
  if (!mismatches) return set_error(CHALOT_ERR_ARG, "selftest_division: null argument");
  unsigned long long* bad = nullptr;
  float* ex = nullptr;
  cudaError_t r = cudaMalloc(&bad, sizeof(unsigned long long));
  if (r == cudaSuccess) r = cudaMalloc(&ex, 2 * sizeof(float));
  if (r == cudaSuccess) r = cudaMemset(bad, 0, sizeof(unsigned long long));
  if (r == cudaSuccess) r = cudaMemset(ex, 0, 2 * sizeof(float));
  if (r == cudaSuccess) {
    k_div_check<<<1184, 256>>>(n, seed, bad, ex);
    r = cudaDeviceSynchronize();
  }
  unsigned long long h = 0;
  float he[2] = {0, 0};
  if (r == cudaSuccess) r = cudaMemcpy(&h, bad, sizeof h, cudaMemcpyDeviceToHost);
  if (r == cudaSuccess) r = cudaMemcpy(he, ex, sizeof he, cudaMemcpyDeviceToHost);
  if (bad) cudaFree(bad);
  if (ex) cudaFree(ex);
  if (r != cudaSuccess) return set_error(CHALOT_ERR_CUDA, std::string("selftest_division: ") + cudaGetErrorString(r));
  *mismatches = h;
  if (example) {
    example[0] = he[0];
    example[1] = he[1];
  }
  return CHALOT_OK;
}


__attribute__((visibility("default"))) int chalot_probe_int8_mma(int iters, double* tops, double* ms) {
  using namespace chalot;
  if (iters < 1 || iters > (1 << 20) || !tops || !ms) return set_error(CHALOT_ERR_ARG, "probe_int8_mma: bad argument");
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  unsigned* err = nullptr;
  cudaEvent_t a = nullptr, b = nullptr;
  cudaError_t r = cudaMalloc(&err, sizeof(unsigned));
  if (r == cudaSuccess) r = cudaMemset(err, 0, sizeof(unsigned));
  if (r == cudaSuccess) r = cudaFuncSetAttribute(k_mma_i8_peak, cudaFuncAttributeMaxDynamicSharedMemorySize, kPeakSmem);
  if (r == cudaSuccess) r = cudaEventCreate(&a);
  if (r == cudaSuccess) r = cudaEventCreate(&b);
  float t = 0.0f;
  if (r == cudaSuccess) {
    k_mma_i8_peak<<<sms, 128, kPeakSmem>>>(iters / 8 + 1, err);  // warm-up
    cudaEventRecord(a);
    k_mma_i8_peak<<<sms, 128, kPeakSmem>>>(iters, err);
    cudaEventRecord(b);
    r = cudaEventSynchronize(b);
    if (r == cudaSuccess) r = cudaGetLastError();
    if (r == cudaSuccess) r = cudaEventElapsedTime(&t, a, b);
  }
  unsigned h = 0;
  if (r == cudaSuccess) r = cudaMemcpy(&h, err, sizeof(unsigned), cudaMemcpyDeviceToHost);
  if (a) cudaEventDestroy(a);
  if (b) cudaEventDestroy(b);
  if (err) cudaFree(err);
  if (r != cudaSuccess) return set_error(CHALOT_ERR_CUDA, std::string("probe_int8_mma: ") + cudaGetErrorString(r));
  if (h) return set_error(CHALOT_ERR_TIMEOUT, "probe_int8_mma: the MMA completion wait ran out");
  *ms = t;
  const double ops = 2.0 * kPeakM * kPeakN * 128.0 * (double)iters * (double)sms;
  *tops = ops / (t * 1e-3) / 1e12;
  return CHALOT_OK;
}

}  // extern "C"
