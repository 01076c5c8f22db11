// k_moe_layer.cu — one MoE FFN layer for a batch of T tokens (the operator
// behind chalot_moe_layer): router, top-k gating, dispatch by expert, int4
// SwiGLU expert products and the gated combine.
//
// Per token this is the expert block of Engine::forward
// (src/model/engine.rs:334-401) applied to an already normalised input row:
//   logits = b + dot_f32(Wr[e], x)      softmax_top_k(logits, k)
//   for each selected (e, w): gate/up = matmul_int4(x), h = swiglu(gate, up),
//   y = matmul_int4(down, h); out = 0 + w_0*y_0 + w_1*y_1 ... in selection order.
// The batch is processed expert by expert: the T*k (token, choice) slots are
// sorted by expert with a stable counting sort (histogram, prefix sum,
// scatter), so each expert's weights are read once per tile of 32 slots.
//
// Kernels (all on one stream):
//   k_ml_route     one CTA per token: router logits, top-k, quantize x
//   k_ml_dispatch  one CTA: per-expert histogram, prefix sums, slot order,
//                  and the table of slot blocks (expert, first slot, count):
//                  32 slots for the tile GEMMs below, 128 for the tensor-core
//                  path (k_moe_tc.cu), which replaces k_ml_gemm for large T
//   k_ml_gemm<GU>  tiles of 32 slots x 128 weight rows: exact int32 group dots
//                  (dp4a on unpacked int4), the f32 group epilogue in group
//                  order; GU=true writes swiglu(gate, up), else y
//   k_ml_quant     one CTA per slot: quantize h (quantize_f32_to_i8)
//   k_ml_combine   one CTA per token: gated sum in selection order
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <string>

#include "blockops.cuh"
#include "capi_internal.h"
#include "common.cuh"
#include "devstat.h"
#include "moe_layer.h"
#include "tc.cuh"
#include "unpack.cuh"

namespace chalot {
namespace {

constexpr int kThreads = 256;
constexpr int kBM = 32;    // slots per tile
constexpr int kBN = 128;   // weight rows per tile (gate/up: 64 gate rows + the 64 matching up rows)
constexpr int kKC = 256;   // columns staged per chunk
constexpr int kWS = kKC + 16;  // shared row stride of unpacked weights (16-B aligned, 4 banks apart)
constexpr int kSS = kKC / 32 + 1;  // shared row stride of group scales

// (float)v for |v| < 2^22: the integer is placed in the mantissa of 1.5*2^23
// and that bias is subtracted; both steps are exact.
__device__ __forceinline__ float i2f_exact(int v) {
  return __fsub_rn(__int_as_float(v + 0x4B400000), 12582912.0f);
}

__global__ void __launch_bounds__(kThreads) k_ml_route(MlDims d, const float* __restrict__ x,
                                                       const float* __restrict__ rw,
                                                       const float* __restrict__ rb, MlWork w) {
  extern __shared__ __align__(16) unsigned char smem[];
  float* xb = reinterpret_cast<float*>(smem);
  float* lanes = xb + d.dim;
  float* logit = lanes + 16 * d.E;
  float* red = logit + 32;
  const int t = blockIdx.x;
  const float* xt = x + (size_t)t * d.dim;
  for (int i = threadIdx.x; i < d.dim; i += blockDim.x) xb[i] = xt[i];
  __syncthreads();
  router_logits(rw, rb, xb, d.dim, d.E, lanes, logit);
  if (threadIdx.x < 32) topk_warp(logit, d.E, d.K, w.sel + (size_t)t * d.K, w.selw + (size_t)t * d.K);
  const float s = quantize_smem(xb, d.dim, w.xq + (size_t)t * d.dim, red);
  if (threadIdx.x == 0) w.xs[t] = s;
}

// k_ml_route on the un-normalised residual rows: rmsnorm_avx2 with the FFN
// norm weights first (the batched decode's k_b_rmsnorm, engine.rs:325-331),
// then the router, top-k and quantization of the normalised row.
__global__ void __launch_bounds__(kThreads) k_ml_route_norm(MlDims d, const float* __restrict__ x,
                                                            const float* __restrict__ norm_w,
                                                            const float* __restrict__ rw,
                                                            const float* __restrict__ rb, MlWork w) {
  extern __shared__ __align__(16) unsigned char smem[];
  float* xb = reinterpret_cast<float*>(smem);
  float* wbuf = xb + d.dim;
  float* lanes = wbuf + d.dim;
  float* logit = lanes + 16 * d.E;
  float* red = logit + 32;
  const int t = blockIdx.x;
  rmsnorm_smem(x + (size_t)t * d.dim, norm_w, d.dim, xb, wbuf, red, true);
  router_logits(rw, rb, xb, d.dim, d.E, lanes, logit);
  if (threadIdx.x < 32) topk_warp(logit, d.E, d.K, w.sel + (size_t)t * d.K, w.selw + (size_t)t * d.K);
  const float s = quantize_smem(xb, d.dim, w.xq + (size_t)t * d.dim, red);
  if (threadIdx.x == 0) w.xs[t] = s;
}

// Stable counting sort of the N = T*k slots by expert. Warp v walks slots
// [v*chunk, (v+1)*chunk) in order; lanes holding the same expert are grouped
// with __match_any_sync, so positions follow slot order within each expert.
// With n_ranks > 1 the sort key of expert e is (e % n_ranks) * (E / n_ranks) +
// e / n_ranks: slots come out grouped by the rank that holds their expert
// (expert e lives on rank e % n_ranks), then by that rank's local expert.
// Expert ids outside [0, E) get no position (key -1) and their slot's inv is -1.
__device__ __forceinline__ int dispatch_key(int e, int E, int n_ranks) {
  if (e < 0 || e >= E) return -1;
  return n_ranks > 1 ? (e % n_ranks) * (E / n_ranks) + e / n_ranks : e;
}

__global__ void __launch_bounds__(1024) k_ml_dispatch(MlDims d, MlWork w, int bm, int n_ranks, int32_t* offs_out) {
  __shared__ int cnt[32][33];
  __shared__ int off[33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int N = d.T * d.K;
  const int chunk = ((N + 1023) / 1024) * 32;
  const int beg = warp * chunk, end = min(N, beg + chunk);
  for (int i = threadIdx.x; i < 32 * 33; i += blockDim.x) (&cnt[0][0])[i] = 0;
  if (w.amax)  // the h absmax the few-slot gate/up kernel raises
    for (int i = threadIdx.x; i < N; i += blockDim.x) w.amax[i] = 0u;
  __syncthreads();
  for (int i0 = beg; i0 < end; i0 += 32) {
    const int i = i0 + lane;
    const int e = i < end ? dispatch_key(w.sel[i], d.E, n_ranks) : -1;
    const unsigned m = __match_any_sync(0xffffffffu, e);
    if (e >= 0 && lane == __ffs(m) - 1) cnt[warp][e] += __popc(m);
    __syncwarp();
  }
  __syncthreads();
  if (threadIdx.x < d.E) {  // exclusive prefix over warps, per expert
    const int e = threadIdx.x;
    int run = 0;
    for (int v = 0; v < 32; ++v) {
      const int c = cnt[v][e];
      cnt[v][e] = run;
      run += c;
    }
    off[e + 1] = run;  // totals, turned into offsets below
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    off[0] = 0;
    for (int e = 0; e < d.E; ++e) off[e + 1] += off[e];
    if (offs_out)
      for (int e = 0; e <= d.E; ++e) offs_out[e] = off[e];
    if (w.mb_e) {
      int n = 0;
      for (int e = 0; e < d.E; ++e)
        for (int p = off[e]; p < off[e + 1]; p += bm) {
          w.mb_e[n] = e;
          w.mb_p0[n] = p;
          w.mb_n[n] = min(bm, off[e + 1] - p);
          ++n;
        }
      *w.n_mb = n;
    }
  }
  __syncthreads();
  for (int i0 = beg; i0 < end; i0 += 32) {
    const int i = i0 + lane;
    const int e = i < end ? dispatch_key(w.sel[i], d.E, n_ranks) : -1;
    const unsigned m = __match_any_sync(0xffffffffu, e);
    if (e >= 0) {
      const int pos = off[e] + cnt[warp][e] + __popc(m & ((1u << lane) - 1u));
      w.perm[pos] = i;
      w.inv[i] = pos;
    } else if (i < end) {
      w.inv[i] = -1;
    }
    __syncwarp();
    if (e >= 0 && lane == __ffs(m) - 1) cnt[warp][e] += __popc(m);
    __syncwarp();
  }
}

// One tile: slots [p0, p0+cnt) of expert e against 128 weight rows.
// Thread (warp v, lane l) owns slots SPW*v..SPW*v+SPW-1 (tiles of 8*SPW slots:
// 32 for prefill, 8 when an expert gets few slots) and tile rows l, l+32, l+64,
// l+96. For gate/up, tile rows 0..63 are gate rows r0.. and 64..127 are the
// up rows of the same hidden units, so a thread holds gate and up of the
// hidden units r0+l and r0+l+32 for its four slots.
template <bool GU, int SPW>
__global__ void __launch_bounds__(kThreads) k_ml_gemm(MlDims d, const MlExperts XP, MlWork w) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int mb = blockIdx.y;
  if (mb >= *w.n_mb) return;
  const int e = w.mb_e[mb], p0 = w.mb_p0[mb], cnt = w.mb_n[mb];
  const int in_dim = GU ? d.dim : d.H;
  const int out_rows = GU ? d.H : d.dim;
  const int ng = in_dim / d.group;
  const int r0 = blockIdx.x * (GU ? kBN / 2 : kBN);
  const uint8_t* wmat = GU ? XP.ex[e].gu : XP.ex[e].dn;
  const float* smat = GU ? XP.ex[e].gus : XP.ex[e].dns;
  const int8_t* amat = GU ? w.xq : w.hq;
  const float* ascale = GU ? w.xs : w.hs;

  int8_t* X = reinterpret_cast<int8_t*>(smem);              // [kBM][kKC]
  int8_t* W = X + kBM * kKC;                                 // [kBN][kWS]
  float* S = reinterpret_cast<float*>(W + kBN * kWS);        // [kBN][kSS]
  const uint8_t** wrow = reinterpret_cast<const uint8_t**>(S + kBN * kSS);  // [kBN]
  const float** srow = reinterpret_cast<const float**>(wrow + kBN);          // [kBN]
  const int8_t** arow = reinterpret_cast<const int8_t**>(srow + kBN);        // [kBM]

  constexpr int BM = 8 * SPW;  // slots per tile: SPW per warp
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid < kBN) {  // weight row of tile row tid, or null past the matrix
    const int hr = GU ? r0 + (tid & 63) : r0 + tid;
    const int mrow = GU ? (tid < 64 ? hr : d.H + hr) : hr;
    const bool ok = hr < out_rows;
    wrow[tid] = ok ? wmat + (size_t)mrow * (in_dim / 2) : nullptr;
    srow[tid] = ok ? smat + (size_t)mrow * ng : nullptr;
  } else if (tid < kBN + BM) {
    const int s = tid - kBN;
    const int p = p0 + s;
    arow[s] = s < cnt ? (GU ? amat + (size_t)(w.perm[p] / d.K) * in_dim : amat + (size_t)p * in_dim)
                      : nullptr;
  }
  float xsv[SPW];
#pragma unroll
  for (int s = 0; s < SPW; ++s) {
    const int sl = warp * SPW + s;
    xsv[s] = sl < cnt ? (GU ? ascale[w.perm[p0 + sl] / d.K] : ascale[p0 + sl]) : 0.0f;
  }
  float acc[SPW][4];
#pragma unroll
  for (int s = 0; s < SPW; ++s)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[s][i] = 0.0f;

  const int gw = d.group >> 2;  // 32-bit words per group
  for (int k0 = 0; k0 < in_dim; k0 += kKC) {
    const int kc = min(kKC, in_dim - k0);  // a multiple of group
    __syncthreads();
    // activations: kBM rows of kc int8
    const int xch = kc >> 4;
    for (int c = tid; c < BM * xch; c += kThreads) {
      const int s = c / xch, j = c - s * xch;
      const int8_t* a = arow[s];
      *reinterpret_cast<uint4*>(X + s * kKC + j * 16) =
          a ? __ldg(reinterpret_cast<const uint4*>(a + k0 + j * 16)) : make_uint4(0, 0, 0, 0);
    }
    // weights: kBN rows of kc/2 packed bytes, unpacked to int8
    const int wch = kc >> 5;
    for (int c = tid; c < kBN * wch; c += kThreads) {
      const int r = c / wch, j = c - r * wch;
      const uint8_t* wr = wrow[r];
      uint4* dst = reinterpret_cast<uint4*>(W + r * kWS + j * 32);
      if (wr) {
        unpack32_any(ldg_stream(wr + (k0 >> 1) + j * 16), dst, XP.repacked != 0);
      } else {
        dst[0] = make_uint4(0, 0, 0, 0);
        dst[1] = make_uint4(0, 0, 0, 0);
      }
    }
    const int gpc = kc / d.group;
    for (int c = tid; c < kBN * gpc; c += kThreads) {
      const int r = c / gpc, g = c - r * gpc;
      S[r * kSS + g] = srow[r] ? __ldg(srow[r] + k0 / d.group + g) : 0.0f;
    }
    __syncthreads();
    for (int g = 0; g < gpc; ++g) {
      int dots[SPW][4];
#pragma unroll
      for (int s = 0; s < SPW; ++s)
#pragma unroll
        for (int i = 0; i < 4; ++i) dots[s][i] = 0;
      for (int q = 0; q < gw; q += 4) {
        const int col = g * d.group + q * 4;
        uint4 xv[SPW], wv[4];
#pragma unroll
        for (int s = 0; s < SPW; ++s) xv[s] = lds16(X + (warp * SPW + s) * kKC + col);
#pragma unroll
        for (int i = 0; i < 4; ++i) wv[i] = lds16(W + (lane + 32 * i) * kWS + col);
#pragma unroll
        for (int s = 0; s < SPW; ++s)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            int t = dots[s][i];
            t = __dp4a((int)wv[i].x, (int)xv[s].x, t);
            t = __dp4a((int)wv[i].y, (int)xv[s].y, t);
            t = __dp4a((int)wv[i].z, (int)xv[s].z, t);
            t = __dp4a((int)wv[i].w, (int)xv[s].w, t);
            dots[s][i] = t;
          }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float sc = S[(lane + 32 * i) * kSS + g];
#pragma unroll
        for (int s = 0; s < SPW; ++s)
          acc[s][i] = __fadd_rn(acc[s][i], __fmul_rn(__fmul_rn(i2f_exact(dots[s][i]), sc), xsv[s]));
      }
    }
  }
#pragma unroll
  for (int s = 0; s < SPW; ++s) {
    const int sl = warp * SPW + s;
    if (sl >= cnt) continue;
    const size_t p = (size_t)(p0 + sl);
    if (GU) {
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int hr = r0 + lane + 32 * i;
        if (hr < d.H) w.h[p * d.H + hr] = swiglu_elem(acc[s][i], acc[s][i + 2], hr, d.H);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = r0 + lane + 32 * i;
        if (r < d.dim) w.y[p * d.dim + r] = acc[s][i];
      }
    }
  }
}

// Few-slot expert products (batched decode: a handful of slots per expert).
// Expert weights stream once per expert through a cp.async ring in their
// packed form, coalesced; the group dots run on the tensor cores as
// mma.sync m16n8k32 (s8 x s8 -> s32) straight from registers: a warp owns 16
// weight rows and takes, per group of 32 columns, one MMA per 8 slots. Its A
// fragment is unpacked from the staged int4 bytes (lane (g, t) holds packed
// word t of rows g and g+8: low nibbles as k 4t..4t+3, high nibbles as
// 16+4t.., each as 16 x its value; the activations' B fragment pairs the same
// columns), its accumulator input is the bits of 1.5*2^23, so every D element
// reads back as 12582912 + 16 gdot, exact, and one subtraction gives
// (float)(16 gdot), which the group scale / 16 turns into gdot * s exactly. The f32
// group epilogue t = t + ((float)gdot * s_g) * xs then runs on the D fragment
// in registers, in group order, as in matmul_int4 (src/tensor/matmul.rs:
// 452-654). Gate/up warps hold 8 gate rows (units u..u+7) and the 8 up rows
// of the same units, so lane (g, t) ends with gate and up of unit u+g for its
// slots and applies SwiGLU itself. Only as many MMAs (and epilogues) as 8-slot
// tiles hold slots run. Group 32 only; dims multiples of kFewKc.
//
// A dp4a formulation of the same products spends 8 dp4a per (row, slot,
// group) on top of the 4-operation epilogue; here the MMA covers 16 rows x 8
// slots x 32 columns in one instruction and the epilogue is what remains.
constexpr int kFewSlots = 16;     // slots per block (the dispatch's tile size): two 8-slot MMA tiles
constexpr int kFewKc = 128;       // columns per stage: 4 groups of 32
constexpr int kFewStages = 4;
constexpr int kFewWarps = 8;      // 16 weight rows per warp: 128 rows per block
constexpr int kFewThreads = 32 * kFewWarps;
constexpr int kFewRows = 16 * kFewWarps;
constexpr int kFewWStride = kFewKc / 2 + 16;  // packed row stride (80 B: A-fragment loads conflict-free)
constexpr int kFewXStride = kFewKc + 32;      // activation row stride (160 B: B-fragment loads conflict-free)
// stage: packed rows [kFewRows][kFewWStride], scales [kFewRows][4] f32, activations [kFewSlots][kFewXStride]
constexpr size_t kFewStageBytes = (size_t)kFewRows * (kFewWStride + 16) + (size_t)kFewSlots * kFewXStride;
constexpr size_t kFewSmem = kFewStageBytes * kFewStages;

CHALOT_DEV void few_cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src)
               : "memory");
}
CHALOT_DEV void few_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
CHALOT_DEV void few_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// One packed int4 word (8 columns) -> int8 words of 16 x its low and high
// nibbles: a two's complement nibble moved to the top of a byte reads as the
// signed byte 16 * value (in [-128, 112]), so no sign extension is needed.
// Repacked layout: low nibbles are columns 8j..8j+3, high ones 8j+4..8j+7,
// two's complement. File layout: byte k holds columns 2k (low) and 2k+1
// (high) as value + 8 (flipping a nibble's top bit makes it two's
// complement), so low nibbles are the even columns.
template <bool RP>
CHALOT_DEV void few_nibbles16(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t v = RP ? w : w ^ 0x88888888u;
  lo = (v << 4) & 0xF0F0F0F0u;
  hi = v & 0xF0F0F0F0u;
}

// D = A * B + C, m16n8k32, A row-major s8, B column-major s8, s32 accumulators.
CHALOT_DEV void mma_s8_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                             uint32_t b1, int c) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%10, %10, %10, %10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c));
}

template <bool GU, bool RP>
__global__ void __launch_bounds__(kFewThreads) k_ml_few(MlDims d, const MlExperts XP, MlWork w) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int mb = blockIdx.y;
  if (mb >= *w.n_mb) return;
  const int e = w.mb_e[mb], p0 = w.mb_p0[mb], cnt = w.mb_n[mb];
  const int in_dim = GU ? d.dim : d.H;
  const int out_rows = GU ? d.H : d.dim;
  const int ng = in_dim >> 5;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  // block rows: gate/up: units u0 + 8*warp + i (i < 8: gate row, i >= 8: up row of unit i-8); down: r0 + row
  const int r0 = blockIdx.x * (GU ? kFewRows / 2 : kFewRows);
  const uint8_t* wmat = GU ? XP.ex[e].gu : XP.ex[e].dn;
  const float* smat = GU ? XP.ex[e].gus : XP.ex[e].dns;
  const int ntiles = cnt > 8 ? 2 : 1;

  // this lane's slots: nt*8 + 2t and nt*8 + 2t + 1 of each 8-slot tile
  float xs[2][2];
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int s = nt * 8 + 2 * t + j;
      xs[nt][j] = s < cnt ? (GU ? w.xs[w.perm[p0 + s] / d.K] : w.hs[p0 + s]) : 0.0f;
    }

  auto unit_of = [&](int lr) { return GU ? r0 + (lr >> 4) * 8 + (lr & 7) : r0 + lr; };
  auto mrow_of = [&](int lr, int unit) { return GU ? ((lr & 8) ? d.H + unit : unit) : unit; };

  static_assert(kFewSlots * (kFewKc / 16) <= kFewThreads, "one activation chunk per thread at most");
  // this thread's copies of every stage (the same rows and chunks each
  // stage, 128 columns further): up to three 16-byte pieces of packed
  // weights or scales and one activation chunk
  constexpr int kPieces = (kFewRows * 5 + kFewThreads - 1) / kFewThreads;
  const unsigned char* src[kPieces];
  int dst[kPieces], step[kPieces];
#pragma unroll
  for (int i = 0; i < kPieces; ++i) {
    const int c = tid + i * kFewThreads;
    src[i] = nullptr;
    dst[i] = step[i] = 0;
    if (c < kFewRows * 5) {  // per row: 4 x 16 B of packed weights, 16 B of scales
      const int lr = c / 5, j = c - lr * 5;
      const int unit = unit_of(lr);
      if (unit < out_rows) {
        const int mrow = mrow_of(lr, unit);
        if (j < 4) {
          src[i] = wmat + (size_t)mrow * (in_dim >> 1) + j * 16;
          dst[i] = lr * kFewWStride + j * 16;
          step[i] = kFewKc / 2;
        } else {
          src[i] = reinterpret_cast<const unsigned char*>(smat + (size_t)mrow * ng);
          dst[i] = kFewRows * kFewWStride + lr * 16;
          step[i] = kFewKc / 32 * 4;
        }
      }
    }
  }
  const int8_t* xsrc = nullptr;
  int xdst = 0;
  if (tid < cnt * (kFewKc / 16)) {  // cnt <= kFewSlots: at most one activation chunk per thread
    const int s = tid / (kFewKc / 16), j = tid % (kFewKc / 16);
    xsrc = (GU ? w.xq + (size_t)(w.perm[p0 + s] / d.K) * in_dim : w.hq + (size_t)(p0 + s) * in_dim) + j * 16;
    xdst = kFewRows * (kFewWStride + 16) + s * kFewXStride + j * 16;
  }
  const int nk = in_dim / kFewKc;
  auto load = [&](int k) {
    unsigned char* base = smem + (size_t)(k % kFewStages) * kFewStageBytes;
#pragma unroll
    for (int i = 0; i < kPieces; ++i)
      if (src[i]) few_cp16(base + dst[i], src[i] + (size_t)k * step[i]);
    if (xsrc) few_cp16(base + xdst, xsrc + (size_t)k * kFewKc);
  };

  float acc[2][4];
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[nt][i] = 0.0f;

#pragma unroll
  for (int k = 0; k < kFewStages - 1; ++k) {
    if (k < nk) load(k);
    few_commit();
  }
  const int la = warp * 16 + g, lb = la + 8;  // this lane's two rows in the block
  for (int k = 0; k < nk; ++k) {
    few_wait<kFewStages - 2>();
    __syncthreads();  // stage k landed for every thread; stage k-1 is free
    if (k + kFewStages - 1 < nk) load(k + kFewStages - 1);
    few_commit();
    const unsigned char* W = smem + (size_t)(k % kFewStages) * kFewStageBytes;
    const float* S = reinterpret_cast<const float*>(W + kFewRows * kFewWStride);
    const int8_t* X = reinterpret_cast<const int8_t*>(S + kFewRows * 4);
    const float4 sa = *reinterpret_cast<const float4*>(S + la * 4), sb = *reinterpret_cast<const float4*>(S + lb * 4);
#pragma unroll
    for (int q = 0; q < 4; ++q) {  // the stage's groups, in order
      uint32_t a0, a1, a2, a3;
      few_nibbles16<RP>(*reinterpret_cast<const uint32_t*>(W + la * kFewWStride + q * 16 + 4 * t), a0, a2);
      few_nibbles16<RP>(*reinterpret_cast<const uint32_t*>(W + lb * kFewWStride + q * 16 + 4 * t), a1, a3);
      // the MMA sums 16 x the group dot (exact, |16 gdot| < 2^22); s / 16 is
      // exact for every normal scale (s >= 2^-122), and then (16 gdot) * (s / 16)
      // rounds as gdot * s
      const float wa = __fmul_rn(q == 0 ? sa.x : q == 1 ? sa.y : q == 2 ? sa.z : sa.w, 0.0625f);
      const float wb = __fmul_rn(q == 0 ? sb.x : q == 1 ? sb.y : q == 2 ? sb.z : sb.w, 0.0625f);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        if (nt < ntiles) {
          // B fragment: columns 8t..8t+7 of the group for slot nt*8 + g (even/odd split in the file layout)
          const uint2 xv = *reinterpret_cast<const uint2*>(X + (nt * 8 + g) * kFewXStride + q * 32 + 8 * t);
          const uint32_t b0 = RP ? xv.x : __byte_perm(xv.x, xv.y, 0x6420);
          const uint32_t b1 = RP ? xv.y : __byte_perm(xv.x, xv.y, 0x7531);
          int dd[4];
          mma_s8_16832(dd, a0, a1, a2, a3, b0, b1, 0x4B400000);
          // ((float)gdot * s) * xs for the slot pair of each row as packed f32x2
          // (each lane rounded as the scalar instruction), then scalar adds,
          // which the assembler never fuses with the multiplies
          const f32x2 bias = f2_pack(12582912.0f, 12582912.0f), x01 = f2_pack(xs[nt][0], xs[nt][1]);
          const f32x2 pa = f2_mul(f2_mul(f2_sub(f2_pack_bits(dd[0], dd[1]), bias), f2_pack(wa, wa)), x01);
          const f32x2 pb = f2_mul(f2_mul(f2_sub(f2_pack_bits(dd[2], dd[3]), bias), f2_pack(wb, wb)), x01);
          float v0, v1, v2, v3;
          f2_unpack(pa, v0, v1);
          f2_unpack(pb, v2, v3);
          acc[nt][0] = __fadd_rn(acc[nt][0], v0);
          acc[nt][1] = __fadd_rn(acc[nt][1], v1);
          acc[nt][2] = __fadd_rn(acc[nt][2], v2);
          acc[nt][3] = __fadd_rn(acc[nt][3], v3);
        }
      }
    }
  }
  // D fragment: acc[nt][0..1] = row la, slots nt*8+2t+{0,1}; acc[nt][2..3] = row lb, same slots
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    if (nt >= ntiles) break;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int s = nt * 8 + 2 * t + j;
      const bool ok = s < cnt;
      const size_t p = (size_t)(p0 + s);
      if (GU) {
        // gate (row la) and up (row lb) of unit u: h, and its absmax over the
        // row for the quantization (non-negative floats order as their bits)
        const int u = unit_of(la);
        const bool live = ok && u < out_rows;
        const float h = live ? swiglu_elem(acc[nt][j], acc[nt][2 + j], u, d.H) : 0.0f;
        if (live) w.h[p * d.H + u] = h;
        float m = fabsf(h);
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
        if (g == 0 && ok) atomicMax(w.amax + p, __float_as_uint(m));
      } else if (ok) {
        const int ua = unit_of(la), ub = unit_of(lb);
        if (ua < out_rows) w.y[p * d.dim + ua] = acc[nt][j];
        if (ub < out_rows) w.y[p * d.dim + ub] = acc[nt][2 + j];
      }
    }
  }
}

// quantize_f32_to_i8 of each h row with its absmax reduced by the few-slot
// gate/up kernel: 16 elements per thread, one 16-byte store (H % 16 == 0, so
// every element takes the vector path of the quantizer).
__global__ void __launch_bounds__(256) k_ml_quant_amax(MlDims d, MlWork w) {
  const int per_row = d.H >> 4;
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)d.T * d.K * per_row) return;
  const long p = i / per_row;
  const int c = (int)(i - p * per_row);
  float scale, inv;
  quant_scale(__uint_as_float(w.amax[p]), &scale, &inv);
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

__global__ void __launch_bounds__(kThreads) k_ml_quant(MlDims d, MlWork w) {
  extern __shared__ __align__(16) unsigned char smem[];
  float* v = reinterpret_cast<float*>(smem);
  float* red = v + d.H;
  const size_t p = blockIdx.x;
  const float* h = w.h + p * d.H;
  for (int i = threadIdx.x; i < d.H; i += blockDim.x) v[i] = h[i];
  __syncthreads();
  const float s = quantize_smem(v, d.H, w.hq + p * d.H, red);
  if (threadIdx.x == 0) w.hs[p] = s;
}

__global__ void __launch_bounds__(kThreads) k_ml_combine(MlDims d, MlWork w, float* __restrict__ out) {
  const int t = blockIdx.x;
  for (int i = threadIdx.x; i < d.dim; i += blockDim.x) {
    float acc = 0.0f;
    for (int j = 0; j < d.K; ++j) {
      const int slot = t * d.K + j;
      const int p = w.inv[slot];
      if (p >= 0) acc = __fadd_rn(acc, __fmul_rn(w.selw[slot], w.y[(size_t)p * d.dim + i]));
    }
    out[(size_t)t * d.dim + i] = acc;
  }
}

// The gated combine of k_ml_combine added to the residual rows (x += expert
// out, engine.rs:401), then rmsnorm + quantize of the new row with the next
// norm weights (the batched decode's k_b_add and k_b_norm_quant), per token.
__global__ void __launch_bounds__(kThreads) k_ml_combine_norm(MlDims d, MlWork w, float* __restrict__ x,
                                                              const float* __restrict__ norm_w, int8_t* xq,
                                                              float* xs) {
  extern __shared__ __align__(16) float cnsm[];  // [dim] norm weights, [dim] scratch
  __shared__ float red[40];
  const int t = blockIdx.x;
  float* xr = x + (size_t)t * d.dim;
  load_f32(cnsm, norm_w, d.dim);
  for (int i = threadIdx.x; i < d.dim; i += blockDim.x) {
    float acc = 0.0f;
    for (int j = 0; j < d.K; ++j) {
      const int slot = t * d.K + j;
      const int p = w.inv[slot];
      if (p >= 0) acc = __fadd_rn(acc, __fmul_rn(w.selw[slot], w.y[(size_t)p * d.dim + i]));
    }
    xr[i] = __fadd_rn(xr[i], acc);
  }
  __syncthreads();  // the block's new residual row is visible to all its threads
  norm_quant_tail(xr, cnsm, d.dim, xq + (size_t)t * d.dim, xs + t, cnsm + d.dim, red);
}

size_t gemm_smem() {
  return (size_t)kBM * kKC + (size_t)kBN * kWS + (size_t)kBN * kSS * 4 + (2 * kBN + kBM) * sizeof(void*);
}

}  // namespace

MlExperts ml_experts_from_blob(const MlDims& d, const uint8_t* blob) {
  MlExperts X{};
  const size_t ng_d = d.dim / d.group, ng_h = d.H / d.group, ex = ml_expert_bytes(d);
  const size_t gu_bytes = (size_t)2 * d.H * (d.dim / 2), gu_sc = (size_t)2 * d.H * ng_d * 4;
  const size_t dn_bytes = (size_t)d.dim * (d.H / 2);
  for (int e = 0; e < d.E && e < 32; ++e) {
    const uint8_t* eb = blob + (size_t)e * ex;
    X.ex[e] = MlExpert{eb, reinterpret_cast<const float*>(eb + gu_bytes), eb + gu_bytes + gu_sc,
                       reinterpret_cast<const float*>(eb + gu_bytes + gu_sc + dn_bytes)};
  }
  (void)ng_h;
  X.repacked = 0;
  return X;
}

size_t ml_expert_bytes(const MlDims& d) {
  const size_t ng_d = d.dim / d.group, ng_h = d.H / d.group;
  return (size_t)2 * d.H * (d.dim / 2) + (size_t)2 * d.H * ng_d * 4 + (size_t)d.dim * (d.H / 2) +
         (size_t)d.dim * ng_h * 4;
}

// Workspace regions, each 256-byte aligned; with base == nullptr only the
// total size is computed.
size_t ml_layout(const MlDims& d, void* base, MlWork* w) {
  const size_t N = (size_t)d.T * d.K, nmb = N / 8 + d.E + 1;  // blocks of 8 slots at the smallest
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) & ~size_t(255);
    return base ? static_cast<unsigned char*>(base) + o : nullptr;
  };
  MlWork t{};
  t.sel = reinterpret_cast<int32_t*>(take(N * 4));
  t.selw = reinterpret_cast<float*>(take(N * 4));
  t.xq = reinterpret_cast<int8_t*>(take((size_t)d.T * d.dim));
  t.xs = reinterpret_cast<float*>(take((size_t)d.T * 4));
  t.perm = reinterpret_cast<int32_t*>(take(N * 4));
  t.inv = reinterpret_cast<int32_t*>(take(N * 4));
  t.mb_e = reinterpret_cast<int32_t*>(take(nmb * 4));
  t.mb_p0 = reinterpret_cast<int32_t*>(take(nmb * 4));
  t.mb_n = reinterpret_cast<int32_t*>(take(nmb * 4));
  t.n_mb = reinterpret_cast<int32_t*>(take(4));
  t.h = reinterpret_cast<float*>(take(N * d.H * 4));
  t.hq = reinterpret_cast<int8_t*>(take(N * d.H));
  t.hs = reinterpret_cast<float*>(take(N * 4));
  t.y = reinterpret_cast<float*>(take(N * d.dim * 4));
  t.amax = reinterpret_cast<unsigned*>(take(N * 4));
  if (w) *w = t;
  return off;
}

const char* ml_check(const MlDims& d) {
  if (d.dim <= 0 || d.H <= 0) return "dim and hidden_dim must be positive";
  if (d.dim % 32 || d.H % 32) return "dim and hidden_dim must be multiples of 32";
  if (d.group < 32 || d.group > 256 || (d.group & (d.group - 1)))
    return "group must be a power of two in [32, 256]";
  if (d.dim % d.group || d.H % d.group) return "group must divide dim and hidden_dim";
  if (d.E < 2 || d.E > 32) return "n_experts must be in [2, 32]";
  if (d.K < 1 || d.K > d.E) return "top_k must be in [1, n_experts]";
  if (d.dim > 16384 || d.H > 16384) return "dim and hidden_dim must be at most 16384";
  return nullptr;
}

static void route_and_dispatch(const MlDims& d, const float* x, const float* rw, const float* rb,
                               const MlWork& w, int bm, cudaStream_t s) {
  const size_t rsm = ((size_t)d.dim + 16 * d.E + 32 + 40) * 4;
  cudaFuncSetAttribute(k_ml_route, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rsm);
  k_ml_route<<<d.T, kThreads, rsm, s>>>(d, x, rw, rb, w);
  k_ml_dispatch<<<1, 1024, 0, s>>>(d, w, bm, 1, nullptr);
}

static void quantize_h(const MlDims& d, const MlWork& w, cudaStream_t s) {
  const size_t qsm = ((size_t)d.H + 40) * 4;
  cudaFuncSetAttribute(k_ml_quant, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)qsm);
  k_ml_quant<<<(unsigned)((size_t)d.T * d.K), kThreads, qsm, s>>>(d, w);
}

static void quantize_h_amax(const MlDims& d, const MlWork& w, cudaStream_t s) {
  const long n = (long)d.T * d.K * (d.H / 16);
  k_ml_quant_amax<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(d, w);
}

// The few-slot kernels need group 32, dims that are multiples of kFewKc and
// 16-byte aligned expert tensors (their cp.async copies are 16 bytes).
static bool few_eligible(const MlDims& d, const MlExperts& X) {
  if (d.group != 32 || d.dim % kFewKc || d.H % kFewKc) return false;
  for (int e = 0; e < d.E && e < 32; ++e) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(X.ex[e].gu) | reinterpret_cast<uintptr_t>(X.ex[e].gus) |
                        reinterpret_cast<uintptr_t>(X.ex[e].dn) | reinterpret_cast<uintptr_t>(X.ex[e].dns);
    if (a & 15) return false;
  }
  return true;
}

// Slots per tile: when the experts get few slots each (batched decode), the
// few-slot kernels (kFewSlots) or, for shapes they do not take, 8-slot tile
// GEMMs; else 32-slot tile GEMMs.
static int tile_slots(const MlDims& d, const MlExperts& X) {
  if ((size_t)d.T * d.K / d.E >= 24) return kBM;
  return few_eligible(d, X) ? kFewSlots : 8;
}

// gate/up tile GEMM, quantize h, down tile GEMM, with tiles of bm slots.
static void tile_gemms(const MlDims& d, const MlExperts& X, const MlWork& w, int bm, cudaStream_t s) {
  const size_t N = (size_t)d.T * d.K;
  const size_t gsm = gemm_smem();
  const unsigned nmb = (unsigned)std::min(N, N / bm + d.E);
  const dim3 ggu((d.H + kBN / 2 - 1) / (kBN / 2), nmb), gdn((d.dim + kBN - 1) / kBN, nmb);
  if (bm == kFewSlots) {
    const dim3 fgu((d.H + kFewRows / 2 - 1) / (kFewRows / 2), nmb), fdn((d.dim + kFewRows - 1) / kFewRows, nmb);
    auto gu = X.repacked ? k_ml_few<true, true> : k_ml_few<true, false>;
    auto dn = X.repacked ? k_ml_few<false, true> : k_ml_few<false, false>;
    cudaFuncSetAttribute(gu, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kFewSmem);
    cudaFuncSetAttribute(dn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kFewSmem);
    gu<<<fgu, kFewThreads, kFewSmem, s>>>(d, X, w);
    quantize_h_amax(d, w, s);
    dn<<<fdn, kFewThreads, kFewSmem, s>>>(d, X, w);
  } else if (bm == 8) {
    cudaFuncSetAttribute(k_ml_gemm<true, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gsm);
    cudaFuncSetAttribute(k_ml_gemm<false, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gsm);
    k_ml_gemm<true, 1><<<ggu, kThreads, gsm, s>>>(d, X, w);
    quantize_h(d, w, s);
    k_ml_gemm<false, 1><<<gdn, kThreads, gsm, s>>>(d, X, w);
  } else {
    cudaFuncSetAttribute(k_ml_gemm<true, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gsm);
    cudaFuncSetAttribute(k_ml_gemm<false, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gsm);
    k_ml_gemm<true, 4><<<ggu, kThreads, gsm, s>>>(d, X, w);
    quantize_h(d, w, s);
    k_ml_gemm<false, 4><<<gdn, kThreads, gsm, s>>>(d, X, w);
  }
}

cudaError_t ml_run(const MlDims& d, const float* x, const float* rw, const float* rb,
                   const MlExperts& X, const MlWork& w, float* out, cudaStream_t s) {
  if (d.T == 0) return cudaSuccess;
  const size_t N = (size_t)d.T * d.K;
  const int bm = tile_slots(d, X);
  route_and_dispatch(d, x, rw, rb, w, bm, s);
  tile_gemms(d, X, w, bm, s);
  (void)N;
  k_ml_combine<<<d.T, kThreads, 0, s>>>(d, w, out);
  return cudaGetLastError();
}

// The batched decode's MoE block with its ends fused: the FFN rmsnorm runs in
// the router kernel, and the gated combine, the residual add and the next
// rmsnorm + quantization run in one kernel. x holds the residual rows (read
// by the router, updated by the combine); xq/xs receive the next layer's
// quantized input. The expert products between are ml_run's (t: tensor-core path).
cudaError_t ml_run_decode(const MlDims& d, float* x, const float* norm_ffn, const float* rw, const float* rb,
                          const MlExperts& X, const MlWork& w, const MlTcWork* t, const float* norm_next,
                          int8_t* xq, float* xs, cudaStream_t s) {
  if (d.T == 0) return cudaSuccess;
  const size_t N = (size_t)d.T * d.K;
  cudaError_t r = cudaSuccess;
  if (t && (r = t->err ? cudaMemsetAsync(t->amax, 0, N * 4, s) : cudaErrorInvalidValue) != cudaSuccess) return r;
  const size_t rsm = ((size_t)2 * d.dim + 16 * d.E + 32 + 40) * 4;
  cudaFuncSetAttribute(k_ml_route_norm, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rsm);
  k_ml_route_norm<<<d.T, kThreads, rsm, s>>>(d, x, norm_ffn, rw, rb, w);
  if (t) {
    k_ml_dispatch<<<1, 1024, 0, s>>>(d, w, 128, 1, nullptr);
    if ((r = ml_tc_prepare(d, X, w, *t, s)) != cudaSuccess) return r;
    const unsigned nmb = (unsigned)std::min(N, N / 128 + d.E);
    if ((r = ml_tc_gemm(d, true, w, *t, nmb, s)) != cudaSuccess) return r;
    if ((r = ml_tc_quant(d, w, *t, s)) != cudaSuccess) return r;
    if ((r = ml_tc_gemm(d, false, w, *t, nmb, s)) != cudaSuccess) return r;
  } else {
    const int bm = tile_slots(d, X);
    k_ml_dispatch<<<1, 1024, 0, s>>>(d, w, bm, 1, nullptr);
    tile_gemms(d, X, w, bm, s);
  }
  const size_t csm = (size_t)2 * d.dim * 4;
  cudaFuncSetAttribute(k_ml_combine_norm, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)csm);
  k_ml_combine_norm<<<d.T, kThreads, csm, s>>>(d, w, x, norm_next, xq, xs);
  return cudaGetLastError();
}

// The same layer with the expert products on the tensor cores.
cudaError_t ml_run_tc(const MlDims& d, const float* x, const float* rw, const float* rb,
                      const MlExperts& X, const MlWork& w, const MlTcWork& t, float* out,
                      cudaStream_t s) {
  if (d.T == 0) return cudaSuccess;
  const size_t N = (size_t)d.T * d.K;
  cudaError_t r = t.err ? cudaMemsetAsync(t.amax, 0, N * 4, s) : cudaErrorInvalidValue;
  if (r != cudaSuccess) return r;
  route_and_dispatch(d, x, rw, rb, w, 128, s);
  if ((r = ml_tc_prepare(d, X, w, t, s)) != cudaSuccess) return r;
  const unsigned nmb = (unsigned)std::min(N, N / 128 + d.E);
  if ((r = ml_tc_gemm(d, true, w, t, nmb, s)) != cudaSuccess) return r;
  if ((r = ml_tc_quant(d, w, t, s)) != cudaSuccess) return r;
  if ((r = ml_tc_gemm(d, false, w, t, nmb, s)) != cudaSuccess) return r;
  k_ml_combine<<<d.T, kThreads, 0, s>>>(d, w, out);
  return cudaGetLastError();
}

__global__ void k_fill_f32(float* p, size_t n, float v) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    p[i] = v;
}

void ml_launch_route(const MlDims& d, const float* x, const float* rw, const float* rb, const MlWork& w,
                     cudaStream_t s) {
  const size_t rsm = ((size_t)d.dim + 16 * d.E + 32 + 40) * 4;
  cudaFuncSetAttribute(k_ml_route, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rsm);
  k_ml_route<<<d.T, kThreads, rsm, s>>>(d, x, rw, rb, w);
}

void ml_launch_plan(const MlDims& d, const MlWork& w, int n_ranks, int32_t* offs, cudaStream_t s) {
  k_ml_dispatch<<<1, 1024, 0, s>>>(d, w, kBM, n_ranks, offs);
}

void ml_launch_combine(const MlDims& d, const MlWork& w, float* out, cudaStream_t s) {
  k_ml_combine<<<d.T, kThreads, 0, s>>>(d, w, out);
}

// Expert products of rows whose input is already quantized: w.sel holds each
// row's (local) expert, w.xq / w.xs the rows; d.K == 1. y[row] (the expert
// output) is written in row order through the combine with weight 1.0, which
// reproduces y exactly (0 + 1*y).
cudaError_t ml_run_rows(const MlDims& d, const MlExperts& X, const MlWork& w, const MlTcWork* t, float* y,
                        cudaStream_t s, int est_rows) {
  if (d.T == 0) return cudaSuccess;
  const size_t N = (size_t)d.T;
  k_fill_f32<<<(unsigned)std::min<size_t>((N + 255) / 256, 1024), 256, 0, s>>>(w.selw, N, 1.0f);
  if (t) {
    cudaError_t r = t->err ? cudaMemsetAsync(t->amax, 0, N * 4, s) : cudaErrorInvalidValue;
    if (r != cudaSuccess) return r;
    k_ml_dispatch<<<1, 1024, 0, s>>>(d, w, 128, 1, nullptr);
    if ((r = ml_tc_prepare(d, X, w, *t, s)) != cudaSuccess) return r;
    const unsigned nmb = (unsigned)std::min(N, N / 128 + d.E);
    if ((r = ml_tc_gemm(d, true, w, *t, nmb, s)) != cudaSuccess) return r;
    if ((r = ml_tc_quant(d, w, *t, s)) != cudaSuccess) return r;
    if ((r = ml_tc_gemm(d, false, w, *t, nmb, s)) != cudaSuccess) return r;
  } else {
    MlDims de = d;  // the slot tiles from the live rows when the caller knows them
    if (est_rows >= 0) de.T = std::max(1, std::min(est_rows, d.T));
    const int bm = tile_slots(de, X);
    k_ml_dispatch<<<1, 1024, 0, s>>>(d, w, bm, 1, nullptr);
    tile_gemms(d, X, w, bm, s);
  }
  k_ml_combine<<<d.T, kThreads, 0, s>>>(d, w, y);
  return cudaGetLastError();
}

bool ml_use_tc(const MlDims& d) {
  const char* env = std::getenv("CHALOT_MOE_PATH");
  if (env && !std::strcmp(env, "simt")) return false;
  if (!ml_tc_eligible(d)) return false;
  if (env && !std::strcmp(env, "tc")) return true;
  return (size_t)d.T * d.K >= 1024;
}

}  // namespace chalot

using namespace chalot;

static int ml_prepare(const chalot_moe_desc* desc, size_t n_tok, MlDims* d) {
  if (!desc) return set_error(CHALOT_ERR_ARG, "null descriptor");
  if (n_tok * std::max<uint32_t>(desc->top_k, 1) > (size_t)(1 << 20))
    return set_error(CHALOT_ERR_ARG, "moe_layer: n_tok * top_k above 2^20");
  *d = MlDims{(int)n_tok, (int)desc->dim, (int)desc->hidden_dim, (int)desc->n_experts,
              (int)desc->top_k, (int)(desc->group ? desc->group : 32)};
  if (const char* m = ml_check(*d)) return set_error(CHALOT_ERR_ARG, std::string("moe_layer: ") + m);
  if (!desc->router_w || !desc->router_b || !desc->experts)
    return set_error(CHALOT_ERR_ARG, "moe_layer: null weight pointer");
  if (reinterpret_cast<uintptr_t>(desc->experts) & 15)
    return set_error(CHALOT_ERR_ARG, "moe_layer: experts must be 16-byte aligned");
  return CHALOT_OK;
}

// Tensor-core expert products from 1024 (token, choice) slots on, when the
// shape allows them (group 32, dim and hidden_dim multiples of 128);
// CHALOT_MOE_PATH=simt|tc overrides the choice (tests use it to cover both).
static bool use_tc(const MlDims& d) { return ml_use_tc(d); }

extern "C" {

__attribute__((visibility("default"))) size_t chalot_moe_workspace_size(const chalot_moe_desc* desc,
                                                                         size_t n_tok) {
  MlDims d;
  if (ml_prepare(desc, n_tok, &d) != CHALOT_OK) return 0;
  const size_t simt = ml_layout(d, nullptr, nullptr);
  return use_tc(d) ? ml_tc_layout(d, simt, nullptr, nullptr) : simt;
}

__attribute__((visibility("default"))) int chalot_moe_layer(const chalot_moe_desc* desc, const float* x,
                                                            size_t n_tok, float* out, int32_t* sel_out,
                                                            float* selw_out, void* workspace,
                                                            size_t workspace_bytes, void* stream) {
  MlDims d;
  if (int rc = ml_prepare(desc, n_tok, &d)) return rc;
  if (n_tok == 0) return CHALOT_OK;
  if (!x || !out) return set_error(CHALOT_ERR_ARG, "moe_layer: null x or out");
  // a tensor-core wait of earlier work that gave up (devstat.h)
  if (int rc = devstat_poll("moe_layer", static_cast<cudaStream_t>(stream))) return rc;
  const bool tc = use_tc(d);
  const size_t simt = ml_layout(d, nullptr, nullptr);
  const size_t need = tc ? ml_tc_layout(d, simt, nullptr, nullptr) : simt;
  if (!workspace || workspace_bytes < need)
    return set_error(CHALOT_ERR_ARG, "moe_layer: workspace too small (need " + std::to_string(need) +
                                         " bytes)");
  if (reinterpret_cast<uintptr_t>(workspace) & 255)
    return set_error(CHALOT_ERR_ARG, "moe_layer: workspace must be 256-byte aligned");
  MlWork w;
  ml_layout(d, workspace, &w);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  MlTcWork t{};
  if (tc) ml_tc_layout(d, simt, workspace, &t);
  const MlExperts X = ml_experts_from_blob(d, desc->experts);
  cudaError_t r = tc ? ml_run_tc(d, x, desc->router_w, desc->router_b, X, w, t, out, s)
                     : ml_run(d, x, desc->router_w, desc->router_b, X, w, out, s);
  const size_t N = n_tok * d.K;
  if (r == cudaSuccess && sel_out) r = cudaMemcpyAsync(sel_out, w.sel, N * 4, cudaMemcpyDeviceToDevice, s);
  if (r == cudaSuccess && selw_out) r = cudaMemcpyAsync(selw_out, w.selw, N * 4, cudaMemcpyDeviceToDevice, s);
  if (r != cudaSuccess) return set_error(CHALOT_ERR_CUDA, std::string("moe_layer: ") + cudaGetErrorString(r));
  return CHALOT_OK;
}

}  // extern "C"
