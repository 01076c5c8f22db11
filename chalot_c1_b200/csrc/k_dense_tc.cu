// k_dense_tc.cu — the int8 GEMMs of batched decode (QKV, O and the output
// projection for up to 256 tokens) on the tensor cores.
//
// out[t][r] (=|+=) ((float)dot(W[r], xq[t]) * ws[r]) * xs[t] is the
// reference's matmul_int8 row (src/tensor/matmul.rs:183-298): an exact int32
// dot over the whole row, then two f32 products (and the residual add of
// engine.rs:312-322 for O). An int32 sum is exact in any order, so the dot
// accumulates in TMEM across K, and the f32 arithmetic runs once per output.
//
// One CTA per 128-row tile of W: kind::i8 MMAs of M=128 (weight rows, operand
// A) x N (tokens, operand B; N = B rounded up to 16) x K=32, fed by a TMA ring
// of 128-column chunks of both operands with the 128-byte swizzle; TMA fills
// rows past R or B with zeros. Warp 0 issues TMA, warp 1 owns TMEM and issues
// the MMAs, warps 2..5 are the epilogue (warp w reads TMEM lanes 32*(w%4)..,
// lane = weight row, column = token), whose stores of one token's 32 rows
// are 128 contiguous bytes. Every wait is bounded and records a failure in the
// device's check word instead of hanging.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "batch.h"
#include "common.cuh"
#include "devstat.h"
#include "tc.cuh"
#include "tmap.h"

namespace chalot {
namespace {

constexpr int kDtThreads = 192;
constexpr int kDtMaxStages = 8;
constexpr int kDtATile = 128 * 128;  // one 128-row x 128-column int8 chunk of W

struct DtSmem {
  uint64_t full[kDtMaxStages], empty[kDtMaxStages], done;
  uint32_t tmem;
  int abort;
};

__host__ __device__ constexpr int dt_stage_bytes(int n) { return kDtATile + n * 128; }

__device__ __forceinline__ bool dt_aborted(DtSmem* sm) {
  return *reinterpret_cast<volatile int*>(&sm->abort) != 0;
}
__device__ __forceinline__ bool dt_wait(uint64_t* bar, uint32_t parity, unsigned* err, DtSmem* sm) {
  if (mbar_wait(bar, parity, err)) return true;
  atomicExch(&sm->abort, 1);
  return false;
}

template <bool ADD>
__global__ void __launch_bounds__(kDtThreads, 1)
    k_dense_tc(const __grid_constant__ CUtensorMap tW, const __grid_constant__ CUtensorMap tX, int B, int R, int C,
               int N, int stages, uint32_t ncols, const float* __restrict__ ws, const float* __restrict__ xs,
               float* out, int ldo, unsigned* err) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  unsigned char* ring = smem_raw + (base - smem_u32(smem_raw));
  const int sb = dt_stage_bytes(N);
  DtSmem* sm = reinterpret_cast<DtSmem*>(ring + (size_t)stages * sb);
  const int r0 = blockIdx.x * 128;
  const int nch = C >> 7;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    for (int i = 0; i < stages; ++i) {
      mbar_init_n(&sm->full[i], 1);
      mbar_init_n(&sm->empty[i], 1);
    }
    mbar_init_n(&sm->done, 1);
    sm->abort = 0;
    mbar_fence_init();
  }
  if (warp == 1) tc_alloc(&sm->tmem, ncols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm->tmem;
  const uint32_t idesc = tc_idesc_i8(128, N);

  if (warp == 0) {
    if (lane == 0) {  // TMA producer
      int c = 0;
      for (; c < nch && !dt_aborted(sm); ++c) {
        const int st = c % stages, n = c / stages;
        if (n > 0 && !dt_wait(&sm->empty[st], (n - 1) & 1, err, sm)) break;
        unsigned char* a = ring + (size_t)st * sb;
        mbar_expect_tx(&sm->full[st], (uint32_t)sb);
        tma_load_2d(a, &tW, c * 128, r0, &sm->full[st]);
        tma_load_2d(a + kDtATile, &tX, c * 128, 0, &sm->full[st]);
      }
      // copies still in flight land before the CTA exits
      for (int k = max(0, c - stages); k < c; ++k) mbar_wait(&sm->full[k % stages], (k / stages) & 1, err);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      for (int c = 0; c < nch; ++c) {
        const int st = c % stages;
        if (!dt_wait(&sm->full[st], (c / stages) & 1, err, sm)) break;
        tc_fence_after();
        const uint32_t a0 = base + (uint32_t)(st * sb), b0 = a0 + kDtATile;
#pragma unroll
        for (int j = 0; j < 4; ++j)
          tc_mma_i8(tmem, tc_desc_sw128(a0 + j * 32), tc_desc_sw128(b0 + j * 32), idesc, (c | j) != 0);
        tc_commit(&sm->empty[st]);
      }
      tc_commit(&sm->done);  // every MMA issued has completed
    }
  } else {  // epilogue
    const int q = warp & 3;
    const int row = r0 + 32 * q + lane;
    const bool live = row < R;
    const float wsr = live ? ws[row] : 0.0f;
    // the next 16 tokens' scales (and residual values) are loaded ahead: the
    // first 16 while the MMAs run, the others while the previous 16 are stored
    float nx_s[16], nx_o[16];
    auto fetch = [&](int cb) {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int t = cb + j;
        nx_s[j] = t < B ? __ldg(xs + t) : 0.0f;
        if (ADD) nx_o[j] = live && t < B ? out[(size_t)t * ldo + row] : 0.0f;
      }
    };
    fetch(0);
    const bool ok = dt_wait(&sm->done, 0, err, sm);
    tc_fence_after();
    if (ok) {
      const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16);
      for (int cb = 0; cb < N; cb += 16) {
        uint32_t r[16];
        tc_ld16(taddr + cb, r);
        float cs[16], co[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          cs[j] = nx_s[j];
          co[j] = ADD ? nx_o[j] : 0.0f;
        }
        if (cb + 16 < N) fetch(cb + 16);
        tc_wait_ld();
        if (live) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int t = cb + j;
            if (t < B) {
              const float v = __fmul_rn(__fmul_rn(__int2float_rn((int)r[j]), wsr), cs[j]);
              out[(size_t)t * ldo + row] = ADD ? __fadd_rn(co[j], v) : v;
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tc_dealloc(tmem, ncols);
  }
}

// Tensor maps of the engine's weights and activation buffers, built once per
// (address, shape): the map encodes only those, so a later buffer at the same
// address with the same shape maps the same way.
struct MapKey {
  const void* p;
  uint64_t cols, rows;
  uint32_t box_r;
  bool operator<(const MapKey& o) const {
    return std::tie(p, cols, rows, box_r) < std::tie(o.p, o.cols, o.rows, o.box_r);
  }
};

bool cached_map(CUtensorMap* m, const void* p, uint64_t cols, uint64_t rows, uint32_t box_r) {
  static std::mutex mu;
  static std::map<MapKey, CUtensorMap> cache;
  const MapKey k{p, cols, rows, box_r};
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(k);
  if (it != cache.end()) {
    *m = it->second;
    return true;
  }
  if (!make_map(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, p, cols, rows, 128, box_r, true)) return false;
  if (cache.size() > 4096) cache.clear();
  cache.emplace(k, *m);
  return true;
}

int g_sms = 0;

}  // namespace

// The tensor-core path takes B <= 256 tokens, C a multiple of 128 and
// 16-byte aligned operands; CHALOT_DENSE_PATH=simt turns it off.
bool b_gemm_tc_eligible(int B, int C, const int8_t* W, const int8_t* xq) {
  static const bool off = [] {
    const char* e = std::getenv("CHALOT_DENSE_PATH");
    return e && !std::strcmp(e, "simt");
  }();
  if (off || B < 1 || B > 256 || C % 128 || C <= 0) return false;
  return ((reinterpret_cast<uintptr_t>(W) | reinterpret_cast<uintptr_t>(xq)) & 15) == 0;
}

cudaError_t b_gemm_tc(int B, int R, int C, const int8_t* W, const float* ws, const int8_t* xq, const float* xs,
                      float* out, int ldo, bool add, cudaStream_t s) {
  const int N = std::max(16, (B + 15) & ~15);
  CUtensorMap mW, mX;
  if (!cached_map(&mW, W, (uint64_t)C, (uint64_t)R, 128) || !cached_map(&mX, xq, (uint64_t)C, (uint64_t)B, N))
    return cudaErrorInvalidValue;
  if (!g_sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_sms <= 0) g_sms = 148;
  }
  const int tiles = (R + 127) / 128;
  const int sb = dt_stage_bytes(N);
  // deep rings when each SM gets one tile, two CTAs per SM when there are more tiles than SMs
  const int budget = tiles <= g_sms ? 200 * 1024 : 100 * 1024;
  const int stages = std::max(2, std::min(kDtMaxStages, budget / sb));
  const uint32_t ncols = N <= 32 ? 32u : N <= 64 ? 64u : N <= 128 ? 128u : 256u;
  const size_t smem = 1024 + (size_t)stages * sb + sizeof(DtSmem);
  auto k = add ? k_dense_tc<true> : k_dense_tc<false>;
  cudaError_t r = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (r != cudaSuccess) return r;
  k<<<tiles, kDtThreads, smem, s>>>(mW, mX, B, R, C, N, stages, ncols, ws, xs, out, ldo, devstat_word());
  return cudaGetLastError();
}

}  // namespace chalot
