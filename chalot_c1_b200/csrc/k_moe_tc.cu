// k_moe_tc.cu — tensor-core (tcgen05 kind::i8) expert products of the
// batched MoE layer, for prefill-sized batches.
//
// The reference's matmul_int4 (src/tensor/matmul.rs:452-654) computes, per
// output row and per group g of 32 columns, an exact int32 group dot and then
// t = t + ((float)gdot_g * s_g) * x_scale in group order. Here the group dots
// come from the tensor cores: one M=128 x N=128 x K=32 MMA per group writes
// the int32 dots of a 128-slot x 128-row tile into TMEM (overwrite, not
// accumulate), and sixteen epilogue warps read them back and run the f32 group
// epilogue in registers, in group order. Four TMEM buffers let the MMAs run
// up to three groups ahead of the epilogue, which is the bound.
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
// warps 2..17 are the epilogue (warp w reads TMEM lanes 32*(w%4).., columns
// split in quarters by (w-2)/4, 16 warps). Every wait is bounded and records
// a failure in the error word instead of hanging.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "blockops.cuh"
#include "common.cuh"
#include "devstat.h"
#include "moe_layer.h"
#include "tc.cuh"
#include "tmap.h"
#include "unpack.cuh"

namespace chalot {
namespace {

constexpr int kEpiWarps = 16;                 // epilogue warps: 4 per TMEM lane quadrant
constexpr int kTcThreads = 64 + 32 * kEpiWarps;
constexpr int kStages = 4;        // A/B ring depth (128 columns each)
constexpr int kSRing = 4;         // scale ring depth
constexpr int kTileBytes = 128 * 128;
constexpr int kTBufs = 4;            // TMEM accumulator buffers (128 columns each)
constexpr uint32_t kTmemCols = 128 * kTBufs;
constexpr uint32_t kIdesc = tc_idesc_i8(128, 128);

struct TcSmem {
  uint64_t full[kStages], empty[kStages], s_full[kSRing], s_empty[kSRing], t_full[kTBufs], t_empty[kTBufs], done;
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

// One warp per destination row: int4 -> int8, scales transposed.
__global__ void __launch_bounds__(256) k_tc_unpack(MlDims d, const MlExperts X, MlTcWork t) {
  if (reinterpret_cast<volatile int*>(t.key)[8] == 0) return;  // the workspace holds these experts already
  const int lane = threadIdx.x & 31;
  const long row = (long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const long gu_rows = (long)d.E * 2 * d.H, dn_rows = (long)d.E * d.dim;
  const int ngd = d.dim / d.group, ngh = d.H / d.group;
  const bool rp = X.repacked != 0;
  if (row < gu_rows) {
    const int e = (int)(row / (2 * d.H)), r = (int)(row % (2 * d.H));
    const int hb = r >> 7, rr = r & 127;
    const int src = rr < 64 ? hb * 64 + rr : d.H + hb * 64 + (rr - 64);
    const uint8_t* s = X.ex[e].gu + (size_t)src * (d.dim / 2);
    int8_t* dst = t.w8gu + (size_t)row * d.dim;
    for (int j = lane; j < d.dim / 32; j += 32)
      unpack32_any(__ldg(reinterpret_cast<const uint4*>(s + j * 16)), reinterpret_cast<uint4*>(dst + j * 32), rp);
    const float* sc = X.ex[e].gus + (size_t)src * ngd;
    for (int g = lane; g < ngd; g += 32) t.sgu[((size_t)e * ngd + g) * 2 * d.H + r] = __ldg(sc + g);
  } else if (row < gu_rows + dn_rows) {
    const long rr = row - gu_rows;
    const int e = (int)(rr / d.dim), i = (int)(rr % d.dim);
    const uint8_t* s = X.ex[e].dn + (size_t)i * (d.H / 2);
    int8_t* dst = t.w8dn + (size_t)rr * d.H;
    for (int j = lane; j < d.H / 32; j += 32)
      unpack32_any(__ldg(reinterpret_cast<const uint4*>(s + j * 16)), reinterpret_cast<uint4*>(dst + j * 32), rp);
    const float* sc = X.ex[e].dns + (size_t)i * ngh;
    for (int g = lane; g < ngh; g += 32) t.sdn[((size_t)e * ngh + g) * d.dim + i] = __ldg(sc + g);
  }
}

// The int8 copy of the experts in the workspace is kept between calls: a
// 4-word key (the experts' addresses, the shape and layout) records what it
// holds. Before an unpack the key is compared and, if it differs, cleared
// (so an interrupted unpack is never taken for a complete one); after it the
// new key is written. Changing the expert weights in place at the same
// address requires a fresh (or cleared) workspace.
__global__ void k_tc_key_check(MlTcWork t, unsigned long long k0, unsigned long long k1, unsigned long long k2,
                               unsigned long long k3) {
  if (threadIdx.x != 0) return;
  const bool same = t.key[0] == k0 && t.key[1] == k1 && t.key[2] == k2 && t.key[3] == k3;
  reinterpret_cast<int*>(t.key)[8] = same ? 0 : 1;
  if (!same) t.key[0] = t.key[1] = t.key[2] = t.key[3] = 0ull;
}
__global__ void k_tc_key_write(MlTcWork t, unsigned long long k0, unsigned long long k1, unsigned long long k2,
                               unsigned long long k3) {
  if (threadIdx.x != 0 || reinterpret_cast<int*>(t.key)[8] == 0) return;
  t.key[0] = k0;
  t.key[1] = k1;
  t.key[2] = k2;
  t.key[3] = k3;
}

// One warp per slot: its token's int8 row and scale, in expert-sorted order.
__global__ void __launch_bounds__(256) k_tc_gather(MlDims d, MlWork w, MlTcWork t) {
  const int lane = threadIdx.x & 31;
  const long p = (long)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (p >= (long)d.T * d.K) return;
  const int tok = w.perm[p] / d.K;
  if (tok < 0 || tok >= d.T) return;  // a position no valid slot filled
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

constexpr uint32_t kMagic = 0x4B400000u;  // bits of 1.5 * 2^23

// Persistent kernel: CTA b takes tiles b, b + gridDim.x, ... of the
// (128-slot block, 128-row tile) grid, row tiles fastest. The TMA ring, the
// scale ring and the TMEM buffers run continuously across tiles, so the
// next tile's loads and first MMAs overlap this tile's last groups and its
// stores. Each group's MMA overwrites its TMEM buffer with the int32 dots;
// the epilogue adds the bits of 1.5*2^23 to each word as an integer, so the
// word reads as the float 12582912 + gdot (exact, |gdot| < 2^22) and one
// packed subtraction gives (float)gdot.
template <bool GU>
__global__ void __launch_bounds__(kTcThreads, 1)
    k_tc_gemm(const __grid_constant__ CUtensorMap tA, const __grid_constant__ CUtensorMap tB,
              const __grid_constant__ CUtensorMap tS, MlDims d, MlWork w, MlTcWork t, int ntn) {
  extern __shared__ unsigned char smem_raw[];
  const int total = *w.n_mb * ntn;
  if ((int)blockIdx.x >= total) return;
  const int K = GU ? d.dim : d.H;
  const int nchunks = K >> 7, ngroups = K >> 5;
  const int ng = K / d.group;

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
      mbar_init_n(&sm->s_empty[i], kEpiWarps);
    }
    for (int i = 0; i < kTBufs; ++i) {
      mbar_init_n(&sm->t_full[i], 1);
      mbar_init_n(&sm->t_empty[i], kEpiWarps);
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
      int it = 0, s_issued = 0;
      for (int tile = blockIdx.x; tile < total && !aborted(sm); tile += gridDim.x) {
        const int mb = tile / ntn, nb = tile - mb * ntn;
        const int e = w.mb_e[mb], p0 = w.mb_p0[mb];
        const int brow0 = GU ? e * 2 * d.H + nb * 128 : e * d.dim + nb * 128;
        bool ok = true;
        for (int c = 0; c < nchunks; ++c, ++it) {
          const int st = it % kStages, n = it / kStages;
          if (n > 0 && !wait_or_abort(&sm->empty[st], (n - 1) & 1, t.err, sm)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&sm->full[st], 2 * kTileBytes);
          tma_load_2d(A + st * kTileBytes, &tA, c * 128, p0, &sm->full[st]);
          tma_load_2d(B + st * kTileBytes, &tB, c * 128, brow0, &sm->full[st]);
          const int m = it / kSRing, ss = it % kSRing;
          if (m > 0 && !wait_or_abort(&sm->s_empty[ss], (m - 1) & 1, t.err, sm)) {
            ok = false;
            ++it;
            break;
          }
          mbar_expect_tx(&sm->s_full[ss], 4 * 128 * 4);
          tma_load_2d(S + ss * 4 * 128, &tS, nb * 128, e * ng + c * 4, &sm->s_full[ss]);
          ++s_issued;
        }
        if (!ok) break;
      }
      // copies still in flight land before the CTA exits
      for (int c = max(0, it - kStages); c < it; ++c)
        mbar_wait(&sm->full[c % kStages], (c / kStages) & 1, t.err);
      for (int c = max(0, s_issued - kSRing); c < s_issued; ++c)
        mbar_wait(&sm->s_full[c % kSRing], (c / kSRing) & 1, t.err);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      int it = 0, gall = 0;
      for (int tile = blockIdx.x; tile < total && !aborted(sm); tile += gridDim.x) {
        bool ok = true;
        for (int c = 0; c < nchunks && ok; ++c, ++it) {
          const int st = it % kStages;
          if (!wait_or_abort(&sm->full[st], (it / kStages) & 1, t.err, sm)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(A + st * kTileBytes), b0 = smem_u32(B + st * kTileBytes);
          for (int j = 0; j < 4; ++j, ++gall) {
            const int buf = gall % kTBufs;
            if (!wait_or_abort(&sm->t_empty[buf], (gall / kTBufs) & 1, t.err, sm)) {
              ok = false;
              break;
            }
            tc_fence_after();
            tc_mma_i8(tmem + buf * 128, tc_desc_sw128(a0 + j * 32), tc_desc_sw128(b0 + j * 32), kIdesc, 0);
            tc_commit(&sm->t_full[buf]);
          }
          if (ok) tc_commit(&sm->empty[st]);
        }
        if (!ok) break;
      }
      tc_commit(&sm->done);  // every MMA issued has completed before TMEM is freed
      mbar_wait(&sm->done, 0, t.err);
    }
  } else {  // epilogue: warp w reads TMEM lanes 32*(w%4).., columns by quarter (w-2)/4
    const int ew = warp - 2, q = warp & 3, quarter = ew >> 2;
    // gate/up tiles: gate units 16*quarter.. (columns) and their up units 64 + 16*quarter..;
    // down tiles: columns 32*quarter..
    const int col_a = GU ? 16 * quarter : 32 * quarter;
    const int col_b = GU ? 64 + 16 * quarter : 32 * quarter + 16;
    const uint32_t lane_addr = tmem + ((uint32_t)(32 * q) << 16);
    // every buffer starts free
    tc_fence_before();
    __syncwarp();
    if (lane == 0)
      for (int b = 0; b < kTBufs; ++b) mbar_arrive(&sm->t_empty[b]);
    const f32x2 bias = f2_pack(12582912.0f, 12582912.0f);
    int it = 0, gall = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
      const int mb = tile / ntn, nb = tile - mb * ntn;
      const int p0 = w.mb_p0[mb], cnt = w.mb_n[mb];
      const int row = 32 * q + lane;
      const bool live = row < cnt;
      const float xs1 = live ? (GU ? t.xsp[p0 + row] : w.hs[p0 + row]) : 0.0f;
      const f32x2 xs = f2_pack(xs1, xs1);
      f32x2 acc0[8], acc1[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc0[j] = acc1[j] = 0ull;
      for (int g = 0; g < ngroups; ++g, ++gall) {
        const int buf = gall % kTBufs, gl = g & 3, ss = it % kSRing;
        if (!wait_or_abort(&sm->t_full[buf], (gall / kTBufs) & 1, t.err, sm)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (gl == 0 && !wait_or_abort(&sm->s_full[ss], (it / kSRing) & 1, t.err, sm)) {
          ok = false;
          break;
        }
        const uint32_t ta = lane_addr + buf * 128;
        const f32x2* sa = reinterpret_cast<const f32x2*>(S + (ss * 4 + gl) * 128 + col_a);
        const f32x2* sb = reinterpret_cast<const f32x2*>(S + (ss * 4 + gl) * 128 + col_b);
        uint32_t r[16];
        tc_ld16(ta + col_a, r);
        tc_wait_ld();
        // acc = acc + ((float)gdot * s) * xs, lane-wise in f32
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const f32x2 ga = f2_sub(f2_pack_bits(r[2 * j] + kMagic, r[2 * j + 1] + kMagic), bias);
          acc0[j] = f2_add_nc(acc0[j], f2_mul(f2_mul(ga, sa[j]), xs));
        }
        tc_ld16(ta + col_b, r);
        tc_wait_ld();
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const f32x2 gb = f2_sub(f2_pack_bits(r[2 * j] + kMagic, r[2 * j + 1] + kMagic), bias);
          acc1[j] = f2_add_nc(acc1[j], f2_mul(f2_mul(gb, sb[j]), xs));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm->t_empty[buf]);
        if (gl == 3) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm->s_empty[ss]);
          ++it;
        }
      }
      if (!ok || aborted(sm)) break;
      if (live) {
        const size_t p = (size_t)(p0 + row);
        if (GU) {
          const int hu0 = nb * 64 + 16 * quarter;
          float4* o = reinterpret_cast<float4*>(w.h + p * d.H + hu0);
          float amax = 0.0f;
#pragma unroll
          for (int j = 0; j < 8; j += 2) {
            float g0, g1, g2, g3, u0, u1, u2, u3;
            f2_unpack(acc0[j], g0, g1);
            f2_unpack(acc0[j + 1], g2, g3);
            f2_unpack(acc1[j], u0, u1);
            f2_unpack(acc1[j + 1], u2, u3);
            const int k = hu0 + 2 * j;
            const float4 v = make_float4(swiglu_elem(g0, u0, k, d.H), swiglu_elem(g1, u1, k + 1, d.H),
                                         swiglu_elem(g2, u2, k + 2, d.H), swiglu_elem(g3, u3, k + 3, d.H));
            amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
            o[j >> 1] = v;
          }
          atomicMax(t.amax + p, __float_as_uint(amax));  // non-negative floats order as their bits
        } else {
          f32x2* o = reinterpret_cast<f32x2*>(w.y + p * d.dim + nb * 128 + col_a);
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = acc0[j];
#pragma unroll
          for (int j = 0; j < 8; ++j) o[8 + j] = acc1[j];
        }
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

// quantize_f32_to_i8 of each h row with its absmax already reduced by the
// gate/up epilogue: 16 elements per thread, one 16-byte store.
__global__ void __launch_bounds__(256) k_tc_quant(MlDims d, MlWork w, MlTcWork t) {
  const int per_row = d.H >> 4;
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)d.T * d.K * per_row) return;
  const long p = i / per_row;
  const int c = (int)(i - p * per_row);
  float scale, inv;
  quant_scale(__uint_as_float(t.amax[p]), &scale, &inv);
  const float4* src = reinterpret_cast<const float4*>(w.h + p * d.H + c * 16);
  uint32_t o[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float4 v = src[k];
    o[k] = (uint32_t)(uint8_t)quant_elem(v.x, inv) | ((uint32_t)(uint8_t)quant_elem(v.y, inv) << 8) |
           ((uint32_t)(uint8_t)quant_elem(v.z, inv) << 16) | ((uint32_t)(uint8_t)quant_elem(v.w, inv) << 24);
  }
  *reinterpret_cast<uint4*>(w.hq + p * d.H + c * 16) = make_uint4(o[0], o[1], o[2], o[3]);
  if (c == 0) w.hs[p] = scale;
}

}  // namespace

// ---- host: tensor maps -------------------------------------------------------

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                 CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                 CUtensorMapFloatOOBfill);

static EncodeTiled encoder() {
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
  w.key = reinterpret_cast<unsigned long long*>(take(256));
  w.w8gu = reinterpret_cast<int8_t*>(take((size_t)d.E * 2 * d.H * d.dim));
  w.sgu = reinterpret_cast<float*>(take((size_t)d.E * ngd * 2 * d.H * 4));
  w.w8dn = reinterpret_cast<int8_t*>(take((size_t)d.E * d.dim * d.H));
  w.sdn = reinterpret_cast<float*>(take((size_t)d.E * ngh * d.dim * 4));
  w.amax = reinterpret_cast<unsigned*>(take(N * 4));
  (void)take(16);  // former per-call error word (layout kept)
  w.err = base ? devstat_word() : nullptr;  // the device's sticky check word (devstat.h)
  if (t) *t = w;
  return off;
}

cudaError_t ml_tc_prepare(const MlDims& d, const MlExperts& X, const MlWork& w, const MlTcWork& t,
                          cudaStream_t s) {
  const long rows = (long)d.E * 2 * d.H + (long)d.E * d.dim;
  const unsigned long long k0 = reinterpret_cast<uintptr_t>(X.ex[0].gu) | 1ull;  // never 0
  const unsigned long long k1 = reinterpret_cast<uintptr_t>(X.ex[d.E - 1].dn);
  const unsigned long long k2 = (unsigned long long)d.E | ((unsigned long long)d.dim << 16) |
                                ((unsigned long long)d.H << 40);
  const unsigned long long k3 = (unsigned long long)d.group | ((unsigned long long)X.repacked << 32);
  k_tc_key_check<<<1, 32, 0, s>>>(t, k0, k1, k2, k3);
  k_tc_unpack<<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(d, X, t);
  k_tc_key_write<<<1, 32, 0, s>>>(t, k0, k1, k2, k3);
  const long N = (long)d.T * d.K;
  k_tc_gather<<<(unsigned)((N + 7) / 8), 256, 0, s>>>(d, w, t);
  return cudaGetLastError();
}

cudaError_t ml_tc_gather_rows(const MlDims& d, const MlWork& w, const MlTcWork& t, cudaStream_t s) {
  const long N = (long)d.T * d.K;
  if (N == 0) return cudaSuccess;
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
  const int ntn = gate_up ? d.H / 64 : d.dim / 128;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const unsigned grid = (unsigned)std::min<size_t>((size_t)n_mblocks * ntn, (size_t)sms);
  k<<<grid, kTcThreads, smem, s>>>(mA, mB, mS, d, w, t, ntn);
  return cudaGetLastError();
}

cudaError_t ml_tc_quant(const MlDims& d, const MlWork& w, const MlTcWork& t, cudaStream_t s) {
  const long n = (long)d.T * d.K * (d.H / 16);
  k_tc_quant<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(d, w, t);
  return cudaGetLastError();
}

}  // namespace chalot
