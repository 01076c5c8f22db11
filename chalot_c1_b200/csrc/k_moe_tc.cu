// k_moe_tc.cu — tensor-core (tcgen05 kind::i8) expert products of the
// batched MoE layer, for prefill-sized batches.
//
// The reference's matmul_int4 (src/tensor/matmul.rs:452-654) computes, per
// output row and per group g of 32 columns, an exact int32 group dot and then
// t = t + ((float)gdot_g * s_g) * x_scale in group order. Here the group dots
// come from the tensor cores: one M=128 x N=128 x K=32 MMA per group writes
// the int32 dots of a 128-slot x 128-row tile into TMEM (overwrite, not
// accumulate), and eight epilogue warps read them back and run the f32 group
// epilogue in registers, in group order. The MMA for group g+1 (second TMEM
// buffer) overlaps the epilogue of group g; the epilogue is the bound.
//
// Operands are int8 in HBM, K-major, loaded by 2-D TMA with the 128-byte
// swizzle into a 4-stage ring (128 columns = 4 groups per stage):
//   A: the expert-sorted activation rows (gathered int8 x, or int8 h)
//   B: the expert weights, unpacked from int4 once per call (k_tc_unpack);
//      gate/up rows are interleaved per 64 hidden units (64 gate rows, then
//      the 64 up rows of the same units) so one tile yields both SwiGLU inputs
//   S: the group scales, transposed to [group][row] so a 4-group x 128-row
//      box lands as four 512-byte scale rows.
// Warp roles: warp 0 issues TMA, warp 1 owns TMEM and issues the MMAs,
// warps 2..9 are the epilogue (warp w reads TMEM lanes 32*(w%4).., columns
// split in halves by (w-2)/4). Every wait is bounded and records a failure in
// the error word instead of hanging.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "blockops.cuh"
#include "common.cuh"
#include "moe_layer.h"
#include "tc.cuh"

namespace chalot {
namespace {

constexpr int kTcThreads = 320;
constexpr int kStages = 4;        // A/B ring depth (128 columns each)
constexpr int kSRing = 4;         // scale ring depth
constexpr int kTileBytes = 128 * 128;
constexpr uint32_t kTmemCols = 256;  // two 128-column int32 buffers
constexpr uint32_t kIdesc = tc_idesc_i8(128, 128);

struct TcSmem {
  uint64_t full[kStages], empty[kStages], s_full[kSRing], s_empty[kSRing], t_full[2], t_empty[2], done;
  uint32_t tmem;
  int abort;
};

size_t tc_smem_bytes() {
  return 1024 + (size_t)kStages * 2 * kTileBytes + (size_t)kSRing * 4 * 128 * 4 + sizeof(TcSmem);
}

// (float)v for |v| < 2^22, exactly (v placed in the mantissa of 1.5*2^23).
__device__ __forceinline__ float i2f_exact(int v) {
  return __fsub_rn(__int_as_float(v + 0x4B400000), 12582912.0f);
}

__device__ __forceinline__ void unpack32(uint4 p, uint4* dst) {
  const uint32_t in[4] = {p.x, p.y, p.z, p.w};
  uint32_t o[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t lo = in[i] & 0x0F0F0F0Fu, hi = (in[i] >> 4) & 0x0F0F0F0Fu;
    o[2 * i] = (__byte_perm(lo, hi, 0x5140) + 0x78787878u) ^ 0x80808080u;
    o[2 * i + 1] = (__byte_perm(lo, hi, 0x7362) + 0x78787878u) ^ 0x80808080u;
  }
  dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
  dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
}

// One warp per destination row: int4 (file layout) -> int8, scales transposed.
__global__ void __launch_bounds__(256) k_tc_unpack(MlDims d, const uint8_t* __restrict__ experts,
                                                   size_t ex_bytes, MlTcWork t) {
  const int lane = threadIdx.x & 31;
  const long row = (long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const long gu_rows = (long)d.E * 2 * d.H, dn_rows = (long)d.E * d.dim;
  const int ngd = d.dim / d.group, ngh = d.H / d.group;
  const size_t gu_bytes = (size_t)2 * d.H * (d.dim / 2), gu_sc = (size_t)2 * d.H * ngd * 4;
  if (row < gu_rows) {
    const int e = (int)(row / (2 * d.H)), r = (int)(row % (2 * d.H));
    const int hb = r >> 7, rr = r & 127;
    const int src = rr < 64 ? hb * 64 + rr : d.H + hb * 64 + (rr - 64);
    const uint8_t* eb = experts + (size_t)e * ex_bytes;
    const uint8_t* s = eb + (size_t)src * (d.dim / 2);
    int8_t* dst = t.w8gu + (size_t)row * d.dim;
    for (int j = lane; j < d.dim / 32; j += 32)
      unpack32(__ldg(reinterpret_cast<const uint4*>(s + j * 16)), reinterpret_cast<uint4*>(dst + j * 32));
    const float* sc = reinterpret_cast<const float*>(eb + gu_bytes) + (size_t)src * ngd;
    for (int g = lane; g < ngd; g += 32) t.sgu[((size_t)e * ngd + g) * 2 * d.H + r] = __ldg(sc + g);
  } else if (row < gu_rows + dn_rows) {
    const long rr = row - gu_rows;
    const int e = (int)(rr / d.dim), i = (int)(rr % d.dim);
    const uint8_t* eb = experts + (size_t)e * ex_bytes + gu_bytes + gu_sc;
    const uint8_t* s = eb + (size_t)i * (d.H / 2);
    int8_t* dst = t.w8dn + (size_t)rr * d.H;
    for (int j = lane; j < d.H / 32; j += 32)
      unpack32(__ldg(reinterpret_cast<const uint4*>(s + j * 16)), reinterpret_cast<uint4*>(dst + j * 32));
    const float* sc = reinterpret_cast<const float*>(eb + (size_t)d.dim * (d.H / 2)) + (size_t)i * ngh;
    for (int g = lane; g < ngh; g += 32) t.sdn[((size_t)e * ngh + g) * d.dim + i] = __ldg(sc + g);
  }
}

// One warp per slot: its token's int8 row and scale, in expert-sorted order.
__global__ void __launch_bounds__(256) k_tc_gather(MlDims d, MlWork w, MlTcWork t) {
  const int lane = threadIdx.x & 31;
  const long p = (long)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (p >= (long)d.T * d.K) return;
  const int tok = w.perm[p] / d.K;
  const uint4* s = reinterpret_cast<const uint4*>(w.xq + (size_t)tok * d.dim);
  uint4* o = reinterpret_cast<uint4*>(t.xp + (size_t)p * d.dim);
  for (int j = lane; j < d.dim / 16; j += 32) o[j] = __ldg(s + j);
  if (lane == 0) t.xsp[p] = w.xs[tok];
}

__device__ __forceinline__ bool aborted(TcSmem* sm) { return *reinterpret_cast<volatile int*>(&sm->abort) != 0; }

// Bounded wait; on failure records it and raises the CTA's abort flag.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, unsigned* err, TcSmem* sm) {
  if (mbar_wait(bar, parity, err)) return true;
  atomicExch(&sm->abort, 1);
  return false;
}

template <bool GU>
__global__ void __launch_bounds__(kTcThreads, 1)
    k_tc_gemm(const __grid_constant__ CUtensorMap tA, const __grid_constant__ CUtensorMap tB,
              const __grid_constant__ CUtensorMap tS, MlDims d, MlWork w, MlTcWork t) {
  extern __shared__ unsigned char smem_raw[];
  const int mb = blockIdx.y;
  if (mb >= *w.n_mb) return;
  const int e = w.mb_e[mb], p0 = w.mb_p0[mb], cnt = w.mb_n[mb];
  const int nb = blockIdx.x;
  const int K = GU ? d.dim : d.H;
  const int nchunks = K >> 7, ngroups = K >> 5;
  const int ng = K / d.group;
  const int brow0 = GU ? e * 2 * d.H + nb * 128 : e * d.dim + nb * 128;
  const int srow0 = e * ng;

  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  unsigned char* sbase = smem_raw + (base - smem_u32(smem_raw));
  unsigned char* A = sbase;
  unsigned char* B = A + kStages * kTileBytes;
  float* S = reinterpret_cast<float*>(B + kStages * kTileBytes);
  TcSmem* sm = reinterpret_cast<TcSmem*>(S + kSRing * 4 * 128);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init_n(&sm->full[i], 1);
      mbar_init_n(&sm->empty[i], 1);
    }
    for (int i = 0; i < kSRing; ++i) {
      mbar_init_n(&sm->s_full[i], 1);
      mbar_init_n(&sm->s_empty[i], 8);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init_n(&sm->t_full[i], 1);
      mbar_init_n(&sm->t_empty[i], 8);
    }
    mbar_init_n(&sm->done, 1);
    sm->abort = 0;
    mbar_fence_init();
  }
  if (warp == 1) tc_alloc(&sm->tmem, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm->tmem;

  if (warp == 0) {
    if (lane == 0) {  // TMA producer
      int issued = 0, s_issued = 0;
      for (int c = 0; c < nchunks && !aborted(sm); ++c) {
        const int st = c % kStages, n = c / kStages;
        if (n > 0 && !wait_or_abort(&sm->empty[st], (n - 1) & 1, t.err, sm)) break;
        mbar_expect_tx(&sm->full[st], 2 * kTileBytes);
        tma_load_2d(A + st * kTileBytes, &tA, c * 128, p0, &sm->full[st]);
        tma_load_2d(B + st * kTileBytes, &tB, c * 128, brow0, &sm->full[st]);
        issued = c + 1;
        const int ss = c % kSRing, m = c / kSRing;
        if (m > 0 && !wait_or_abort(&sm->s_empty[ss], (m - 1) & 1, t.err, sm)) break;
        mbar_expect_tx(&sm->s_full[ss], 4 * 128 * 4);
        tma_load_2d(S + ss * 4 * 128, &tS, nb * 128, srow0 + c * 4, &sm->s_full[ss]);
        s_issued = c + 1;
      }
      // copies still in flight land before the CTA exits
      for (int c = max(0, issued - kStages); c < issued; ++c)
        mbar_wait(&sm->full[c % kStages], (c / kStages) & 1, t.err);
      for (int c = max(0, s_issued - kSRing); c < s_issued; ++c)
        mbar_wait(&sm->s_full[c % kSRing], (c / kSRing) & 1, t.err);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      for (int c = 0; c < nchunks && !aborted(sm); ++c) {
        const int st = c % kStages;
        if (!wait_or_abort(&sm->full[st], (c / kStages) & 1, t.err, sm)) break;
        tc_fence_after();
        const uint32_t a0 = smem_u32(A + st * kTileBytes), b0 = smem_u32(B + st * kTileBytes);
        bool ok = true;
        for (int j = 0; j < 4; ++j) {
          const int g = c * 4 + j, buf = g & 1, u = g >> 1;
          if (u > 0) {
            if (!wait_or_abort(&sm->t_empty[buf], (u - 1) & 1, t.err, sm)) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
          tc_mma_i8(tmem + buf * 128, tc_desc_sw128(a0 + j * 32), tc_desc_sw128(b0 + j * 32), kIdesc, 0);
          tc_commit(&sm->t_full[buf]);
        }
        if (!ok) break;
        tc_commit(&sm->empty[st]);
      }
      tc_commit(&sm->done);  // every MMA issued has completed before TMEM is freed
      mbar_wait(&sm->done, 0, t.err);
    }
  } else {  // epilogue
    const int ew = warp - 2, q = warp & 3, half = ew >> 2;
    const int row = 32 * q + lane;
    const bool live = row < cnt;
    const float xs = live ? (GU ? t.xsp[p0 + row] : w.hs[p0 + row]) : 0.0f;
    const int col_a = GU ? 32 * half : 64 * half;
    const int col_b = GU ? 64 + 32 * half : 64 * half + 32;
    float acc0[32], acc1[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) acc0[j] = acc1[j] = 0.0f;
    const uint32_t lane_addr = tmem + ((uint32_t)(32 * q) << 16);
    for (int g = 0; g < ngroups; ++g) {
      const int buf = g & 1, c = g >> 2, gl = g & 3, ss = c % kSRing;
      if (!wait_or_abort(&sm->t_full[buf], (g >> 1) & 1, t.err, sm)) break;
      tc_fence_after();
      if (gl == 0 && !wait_or_abort(&sm->s_full[ss], (c / kSRing) & 1, t.err, sm)) break;
      uint32_t r0[32], r1[32];
      tc_ld32(lane_addr + buf * 128 + col_a, r0);
      tc_ld32(lane_addr + buf * 128 + col_b, r1);
      tc_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm->t_empty[buf]);
      const float4* sa = reinterpret_cast<const float4*>(S + (ss * 4 + gl) * 128 + col_a);
      const float4* sb = reinterpret_cast<const float4*>(S + (ss * 4 + gl) * 128 + col_b);
#pragma unroll
      for (int j4 = 0; j4 < 8; ++j4) {
        const float4 va = sa[j4], vb = sb[j4];
        const float fa[4] = {va.x, va.y, va.z, va.w}, fb[4] = {vb.x, vb.y, vb.z, vb.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int j = j4 * 4 + u;
          acc0[j] = __fadd_rn(acc0[j], __fmul_rn(__fmul_rn(i2f_exact((int)r0[j]), fa[u]), xs));
          acc1[j] = __fadd_rn(acc1[j], __fmul_rn(__fmul_rn(i2f_exact((int)r1[j]), fb[u]), xs));
        }
      }
      if (gl == 3) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm->s_empty[ss]);
      }
    }
    if (live && !aborted(sm)) {
      const size_t p = (size_t)(p0 + row);
      if (GU) {
        const int hu0 = nb * 64 + 32 * half;
        float4* o = reinterpret_cast<float4*>(w.h + p * d.H + hu0);
#pragma unroll
        for (int j4 = 0; j4 < 8; ++j4) {
          float v[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int j = j4 * 4 + u;
            v[u] = swiglu_elem(acc0[j], acc1[j], hu0 + j, d.H);
          }
          o[j4] = make_float4(v[0], v[1], v[2], v[3]);
        }
      } else {
        float4* o = reinterpret_cast<float4*>(w.y + p * d.dim + nb * 128 + col_a);
#pragma unroll
        for (int j4 = 0; j4 < 8; ++j4)
          o[j4] = make_float4(acc0[4 * j4], acc0[4 * j4 + 1], acc0[4 * j4 + 2], acc0[4 * j4 + 3]);
        o += 8;
#pragma unroll
        for (int j4 = 0; j4 < 8; ++j4)
          o[j4] = make_float4(acc1[4 * j4], acc1[4 * j4 + 1], acc1[4 * j4 + 2], acc1[4 * j4 + 3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tc_dealloc(tmem, kTmemCols);
  }
}

// ---- host: tensor maps -------------------------------------------------------

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                 CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                 CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  });
  return fn;
}

// 2-D map over a row-major [rows][cols] matrix (cols contiguous).
bool make_map(CUtensorMap* m, CUtensorMapDataType dt, size_t esize, const void* ptr, uint64_t cols,
              uint64_t rows, uint32_t box_c, uint32_t box_r, bool swizzle) {
  EncodeTiled enc = encoder();
  if (!enc) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * esize};
  const cuuint32_t box[2] = {box_c, box_r};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool ml_tc_eligible(const MlDims& d) {
  return d.group == 32 && d.dim % 128 == 0 && d.H % 128 == 0 && d.dim <= 16384 && d.H <= 16384;
}

size_t ml_tc_layout(const MlDims& d, size_t off, void* base, MlTcWork* t) {
  const size_t N = (size_t)d.T * d.K;
  const int ngd = d.dim / d.group, ngh = d.H / d.group;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) & ~size_t(255);
    return base ? static_cast<unsigned char*>(base) + o : nullptr;
  };
  MlTcWork w{};
  w.xp = reinterpret_cast<int8_t*>(take(N * d.dim));
  w.xsp = reinterpret_cast<float*>(take(N * 4));
  w.w8gu = reinterpret_cast<int8_t*>(take((size_t)d.E * 2 * d.H * d.dim));
  w.sgu = reinterpret_cast<float*>(take((size_t)d.E * ngd * 2 * d.H * 4));
  w.w8dn = reinterpret_cast<int8_t*>(take((size_t)d.E * d.dim * d.H));
  w.sdn = reinterpret_cast<float*>(take((size_t)d.E * ngh * d.dim * 4));
  w.err = reinterpret_cast<unsigned*>(take(16));
  if (t) *t = w;
  return off;
}

cudaError_t ml_tc_prepare(const MlDims& d, const uint8_t* experts, const MlWork& w, const MlTcWork& t,
                          cudaStream_t s) {
  const long rows = (long)d.E * 2 * d.H + (long)d.E * d.dim;
  k_tc_unpack<<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(d, experts, ml_expert_bytes(d), t);
  const long N = (long)d.T * d.K;
  k_tc_gather<<<(unsigned)((N + 7) / 8), 256, 0, s>>>(d, w, t);
  return cudaGetLastError();
}

cudaError_t ml_tc_gemm(const MlDims& d, bool gate_up, const MlWork& w, const MlTcWork& t, unsigned n_mblocks,
                       cudaStream_t s) {
  const size_t N = (size_t)d.T * d.K;
  CUtensorMap mA, mB, mS;
  bool ok;
  if (gate_up) {
    ok = make_map(&mA, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, t.xp, d.dim, N, 128, 128, true) &&
         make_map(&mB, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, t.w8gu, d.dim, (uint64_t)d.E * 2 * d.H, 128, 128,
                  true) &&
         make_map(&mS, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, t.sgu, 2 * d.H,
                  (uint64_t)d.E * (d.dim / d.group), 128, 4, false);
  } else {
    ok = make_map(&mA, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w.hq, d.H, N, 128, 128, true) &&
         make_map(&mB, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, t.w8dn, d.H, (uint64_t)d.E * d.dim, 128, 128, true) &&
         make_map(&mS, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, t.sdn, d.dim, (uint64_t)d.E * (d.H / d.group), 128,
                  4, false);
  }
  if (!ok) return cudaErrorInvalidValue;
  const size_t smem = tc_smem_bytes();
  auto k = gate_up ? k_tc_gemm<true> : k_tc_gemm<false>;
  cudaError_t r = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (r != cudaSuccess) return r;
  const unsigned ntiles = gate_up ? (unsigned)(d.H / 64) : (unsigned)(d.dim / 128);
  k<<<dim3(ntiles, n_mblocks), kTcThreads, smem, s>>>(mA, mB, mS, d, w, t);
  return cudaGetLastError();
}

}  // namespace chalot
