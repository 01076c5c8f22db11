// k_moe.cu — router and int4 expert kernels of the decode step, and the int4
// matmul / router operators.
//
// matmul_int4 (src/tensor/matmul.rs:363-401, AVX2 452-654): per row and per
// group g of `group` columns, gdot_g = sum((nibble-8) * x_q) is an exact int32
// and the row result is t = ((t + ((float)gdot_0*s_0)*xs) + ...) in group order.
// The kernels keep that order: the lanes of a warp stream a row 16 bytes (one
// 32-column chunk) at a time and compute exact group dots with dp4a; each group
// leader writes p_g = ((float)gdot*s_g)*xs to shared memory, and one thread per
// row then adds p_0, p_1, ... sequentially.
//   k_gateup  rmsnorm(x) -> quantize -> router logits -> softmax top-k
//             (engine.rs:325-344), then gate and up rows of the selected
//             experts -> SwiGLU -> h and absmax(h) (engine.rs:366-377)
//   k_down    quantize(h) -> down rows of every selected expert -> gated sum in
//             selection order -> x += (engine.rs:380-401)
#include <cuda_runtime.h>

#include <algorithm>

#include "blockops.cuh"
#include "kernels.cuh"
#include "pdl.cuh"
#include "tma.cuh"

namespace chalot {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

// One row of a batched int4 GEMV: its packed weights, its group scales and
// which quantized input vector (index into xp/csum/xs) it is dotted with.
struct RowJob {
  const uint8_t* w;
  const float* s;
  int x;
};

// Group products p_g = ((float)gdot_g * s_g) * xs of rows[0..nrows) into
// P[row][g] (row stride ps); in_dim % 32 == 0, group % 32 == 0. Warp w takes
// rows w*R.. (R at a time) and loads IT 32-lane strides of each row before
// computing, so R*IT 16-byte loads per lane are in flight.
template <int R, int IT>
__device__ __forceinline__ void group_products(const RowJob* rows, int nrows, int in_dim, int group,
                                               const int8_t* xp, const int* csum, const float* xs,
                                               float* P, int ps) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int chunks = in_dim >> 5, cpg = group >> 5;
  const int gsh = __ffs(cpg) - 1;  // group % 32 == 0 and a power of two: c / cpg == c >> gsh
  for (int r0 = warp * R; r0 < nrows; r0 += kWarps * R) {
    for (int cb = 0; cb < chunks; cb += 32 * IT) {
      uint4 w[R][IT];
      float sc[R][IT];
#pragma unroll
      for (int i = 0; i < R; ++i)
#pragma unroll
        for (int it = 0; it < IT; ++it) {
          const int c = cb + it * 32 + lane;
          const bool ok = c < chunks && r0 + i < nrows;
          w[i][it] = ok ? ldg_stream(rows[r0 + i].w + (size_t)c * 16) : make_uint4(0, 0, 0, 0);
          sc[i][it] = ok ? __ldg(rows[r0 + i].s + (c >> gsh)) : 0.0f;  // this chunk's group scale
        }
#pragma unroll
      for (int it = 0; it < IT; ++it) {
        const int c = cb + it * 32 + lane;
        if (cb + it * 32 >= chunks) break;  // warp-uniform
#pragma unroll
        for (int i = 0; i < R; ++i) {
          const bool live = r0 + i < nrows;
          const int xsel = live ? rows[r0 + i].x : 0;
          const int8_t* xv = xp + (size_t)xsel * in_dim;
          int dv = 0;
          if (c < chunks) {
            const uint4 xe = lds16(xv + (size_t)c * 32), xo = lds16(xv + (size_t)c * 32 + 16);
            dv = dot32_u4(w[i][it], xe, xo, 0) - 8 * csum[xsel * chunks + c];
          }
          // the chunks of one group sit in consecutive lanes: reduce them exactly
          for (int o = 1; o < cpg; o <<= 1) dv += __shfl_xor_sync(0xffffffffu, dv, o);
          if (live && c < chunks && (c & (cpg - 1)) == 0)
            P[(r0 + i) * ps + (c >> gsh)] = __fmul_rn(__fmul_rn((float)dv, sc[i][it]), xs[xsel]);
        }
      }
    }
  }
}

__device__ __forceinline__ void group_products_any(const RowJob* rows, int nrows, int in_dim,
                                                   int group, const int8_t* xp, const int* csum,
                                                   const float* xs, float* P, int ps) {
  const int chunks = in_dim >> 5;
  if (chunks <= 32)
    group_products<8, 1>(rows, nrows, in_dim, group, xp, csum, xs, P, ps);
  else if (chunks <= 64)
    group_products<4, 2>(rows, nrows, in_dim, group, xp, csum, xs, P, ps);
  else
    group_products<1, 8>(rows, nrows, in_dim, group, xp, csum, xs, P, ps);
}

// In-place conversion of packed int4 rows from the file layout to the
// engine's repacked layout (repack_word), once at load.
__global__ void k_repack_i4(uint32_t* p, size_t n_words) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_words;
       i += (size_t)gridDim.x * blockDim.x)
    p[i] = repack_word(p[i]);
}

// Ordered group sum of one row: t = t + p_g for g = 0..ng-1 (matmul.rs:576-577).
__device__ __forceinline__ float ordered_sum(const float* p, int ng) {
  float t = 0.0f;
  int g = 0;
  for (; g + 8 <= ng; g += 8) {  // 8 independent loads, then 8 dependent adds
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = p[g + u];
#pragma unroll
    for (int u = 0; u < 8; ++u) t = __fadd_rn(t, v[u]);
  }
  for (; g < ng; ++g) t = __fadd_rn(t, p[g]);
  return t;
}

// Sums of every 32-byte chunk of xp (n bytes): 8 dp4a per chunk.
__device__ __forceinline__ void chunk_sums(const int8_t* xp, int n, int* csum) {
  const int* w = reinterpret_cast<const int*>(xp);
  for (int c = threadIdx.x; c < (n >> 5); c += blockDim.x) {
    int s = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) s = __dp4a(w[c * 8 + k], 0x01010101, s);
    csum[c] = s;
  }
}

// ---------------------------------------------------------------------------
// Decode expert kernels (one token). Both stream every weight byte once and
// keep the exact group arithmetic of matmul_int4: per group g an exact int32
// dot, p_g = ((float)gdot_g * s_g) * xs, and the row result t = t + p_g in
// group order (matmul.rs:576-577).

constexpr int kMaxGroups = 64;  // dim / group (checked at load)

// quantize_f32_to_i8 of h_j (quantization.rs:56-104) by one CTA, with the
// absmax the expert's gate/up CTAs left: the scale and up to kHq float4 of h
// per thread are requested together, so one pass costs one L2 round trip.
// hidden % 8 == 0, so every element takes the vector rounding.
constexpr int kHq = 8;
__device__ __forceinline__ void quantize_h(const DecodeBufs& b, int j, int H) {
  __shared__ float inv_s;
  if (threadIdx.x == 0) {
    float sc, inv;
    quant_scale(__uint_as_float(__ldcg(b.amax + j)), &sc, &inv);
    b.xs_h[j] = sc;
    inv_s = inv;
  }
  const int n4 = H >> 2;
  const float4* hv = reinterpret_cast<const float4*>(b.h + (size_t)j * H);
  uint32_t* xw = reinterpret_cast<uint32_t*>(b.xq_h + (size_t)j * H);
  for (int base = 0; base < n4; base += kHq * (int)blockDim.x) {
    float4 v[kHq];
#pragma unroll
    for (int u = 0; u < kHq; ++u) {
      const int i = base + u * (int)blockDim.x + (int)threadIdx.x;
      if (i < n4) v[u] = __ldcg(hv + i);
    }
    if (base == 0) __syncthreads();  // the scale
    const float inv = inv_s;
#pragma unroll
    for (int u = 0; u < kHq; ++u) {
      const int i = base + u * (int)blockDim.x + (int)threadIdx.x;
      if (i < n4) {
        const uint32_t q0 = (uint8_t)quant_elem(v[u].x, inv), q1 = (uint8_t)quant_elem(v[u].y, inv);
        const uint32_t q2 = (uint8_t)quant_elem(v[u].z, inv), q3 = (uint8_t)quant_elem(v[u].w, inv);
        xw[i] = q0 | (q1 << 8) | (q2 << 16) | (q3 << 24);
      }
    }
  }
}

// Gate and up rows of routed expert sel[blockIdx.y] (engine.rs:366-374), then
// SwiGLU (activations.rs:59-87) into h and |h| into the expert's absmax slot.
// Warp w owns PPW = 4/IT row pairs (gate rows i and up rows H+i); lane l holds
// the 32-column chunks l, l+32, ... (IT of them) of each of its rows in
// registers, loaded straight from HBM with streaming loads, and the matching
// chunks of the quantized input. A chunk is one group when group == 32 (else
// the group's chunks, on consecutive lanes, are reduced exactly by shuffles).
// The group products go to shared memory and one lane per row adds them in
// group order. The last CTA of each expert quantizes that expert's h.
template <int IT>
__global__ void __launch_bounds__(kThreads, 4) k_gateup(Dims d, LayerPtrs L, int layer, DecodeBufs b) {
  constexpr int RW = 8 / IT, PPW = RW / 2, PPC = kWarps * PPW, PS = kMaxGroups + 1;
  __shared__ float P[kWarps * RW * PS];
  __shared__ float wmax[kWarps];
  __shared__ __align__(16) int8_t xsm[32 * 32 * IT];  // the quantized FFN input (dim <= 1024 * IT)
  __shared__ int e_s;
  __shared__ float xs_s;
  [[maybe_unused]] const int slot = layer * 8 + 4;
  CHALOT_TRACE(slot, 0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = d.hidden, chunks = d.dim >> 5, cpg = d.group >> 5, gsh = __ffs(cpg) - 1;
  const int ng = d.dim / d.group, prow = d.dim >> 1, j = blockIdx.y;
  const int i0 = blockIdx.x * PPC + warp * PPW;  // first pair of this warp
  pdl_wait();  // the routing and the quantized FFN input come from the O-projection's last CTA
  pdl_trigger();
  CHALOT_TRACE(slot, 2);
  // the routing and the input once per CTA (one request per line and CTA)
  if (threadIdx.x == 0) e_s = __ldcg(b.sel + j);
  if (threadIdx.x == 1) xs_s = __ldcg(b.xs_ffn);
  copy16(reinterpret_cast<uint4*>(xsm), reinterpret_cast<const uint4*>(b.xq_ffn), d.dim >> 4, true);
  __syncthreads();
  const int e = e_s;
  const float xs = xs_s;
  uint4 xa[IT], xb[IT];
#pragma unroll
  for (int it = 0; it < IT; ++it) {
    const int c = min(lane + 32 * it, chunks - 1);
    xa[it] = lds16(xsm + c * 32);
    xb[it] = lds16(xsm + c * 32 + 16);
  }
  const ExpertPtrs X = expert_ptrs(L, d.n_experts, e);
  uint4 w[RW][IT];
  float s[RW][IT];
#pragma unroll
  for (int r = 0; r < RW; ++r) {
    const int pair = i0 + (r % PPW);
    const size_t row = (size_t)(r < PPW ? 0 : H) + pair;
#pragma unroll
    for (int it = 0; it < IT; ++it) {
      const int c = lane + 32 * it;
      const bool ok = pair < H && c < chunks;
      w[r][it] = ok ? ldg_stream(X.gu + row * prow + (size_t)c * 16) : make_uint4(0, 0, 0, 0);
      s[r][it] = (ok && (c & (cpg - 1)) == 0) ? __ldcs(X.gu_s + row * ng + (c >> gsh)) : 0.0f;
    }
  }
  CHALOT_TRACE(slot, 3);
#pragma unroll
  for (int r = 0; r < RW; ++r)
#pragma unroll
    for (int it = 0; it < IT; ++it) {
      const int c = lane + 32 * it;
      int dv = dot32_rp(w[r][it], xa[it], xb[it]);
      for (int o = 1; o < cpg; o <<= 1) dv += __shfl_xor_sync(0xffffffffu, dv, o);
      if (c < chunks && (c & (cpg - 1)) == 0)
        P[(warp * RW + r) * PS + (c >> gsh)] = __fmul_rn(__fmul_rn((float)dv, s[r][it]), xs);
    }
  __syncwarp();
  float tot = 0.0f;
  if (lane < RW) {  // row `lane` of this warp: t = t + p_g in group order
    const float* p = P + (warp * RW + lane) * PS;
    int g = 0;
    for (; g + 8 <= ng; g += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = p[g + u];
#pragma unroll
      for (int u = 0; u < 8; ++u) tot = __fadd_rn(tot, v[u]);
    }
    for (; g < ng; ++g) tot = __fadd_rn(tot, p[g]);
  }
  CHALOT_TRACE(slot, 4);
  const float up = __shfl_sync(0xffffffffu, tot, (lane + PPW) & 31);  // lane p: up row of pair p
  float m = 0.0f;
  if (lane < PPW && i0 + lane < H) {
    const int pair = i0 + lane;
    const float hv = swiglu_elem(tot, up, pair, H);
    b.h[(size_t)j * H + pair] = hv;
    m = fabsf(hv);
  }
  m = warp_max(m);
  if (lane == 0) wmax[warp] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float mm = wmax[0];
#pragma unroll
    for (int i = 1; i < kWarps; ++i) mm = fmaxf(mm, wmax[i]);
    atomicMax(&b.amax[j], __float_as_uint(mm));  // one update per CTA
  }
  const bool tail = last_cta(b.counters + 8 + j, gridDim.x);  // the last CTA of expert j
  CHALOT_TRACE(slot, 5);
  if (!tail) return;
  quantize_h(b, j, H);  // once, for every down CTA
  if (threadIdx.x == 0) b.amax[j] = 0u;  // read by this thread only: clear for the next layer
  CHALOT_TRACE(slot, 6);
}

// Output rows r0..r0+rpc-1 for every routed expert, one row per warp
// (engine.rs:380-401). The routing is two launches old, so before waiting for
// the gate/up kernel the CTA requests its rows and their scales (one bulk
// copy per expert: the rpc rows are contiguous), the x values it will update
// and the final norm's weights after the last layer. After the wait it copies
// the quantized h of every routed expert into shared memory. The warps of an
// expert split its 32-column chunks, each x chunk serving all rpc rows; lane 0
// of warp r adds row r's group products in order, and x[r] += sum_j w_j *
// y_j[r] in selection order. After the last layer (next_norm = the final
// norm, else null) the last CTA computes the lm_head's quantized input.
__global__ void __launch_bounds__(kThreads, 4) k_down(Dims d, LayerPtrs L, int layer,
                                                   const float* next_norm, DecodeBufs b, int dense,
                                                   int rpc) {
  extern __shared__ __align__(16) unsigned char smem[];
  [[maybe_unused]] const int slot = layer * 8 + 5;
  CHALOT_TRACE(slot, 0);
  const int H = d.hidden, K = d.top_k, ng = H / d.group, cpg = d.group >> 5, gsh = __ffs(cpg) - 1;
  const int prow = H >> 1, chunks = H >> 5;
  const int nrow = K * rpc;  // <= kWarps
  uint8_t* W = smem;                                          // [nrow][prow]
  float* S = reinterpret_cast<float*>(W + kWarps * prow);     // [nrow][ng]
  int8_t* xq = reinterpret_cast<int8_t*>(S + kWarps * ng);    // [K][H]
  float* P = reinterpret_cast<float*>(xq + (size_t)K * H);    // [nrow][ng] (ng % 4 == 0)
  float* wn = P + kWarps * ng;                                // [dim] next norm weights
  float* xbuf = wn + d.dim;                                   // [dim] tail scratch
  __shared__ __align__(8) uint64_t bar;
  __shared__ float xs_j[8];
  __shared__ float selw_s[8];
  __shared__ float y[kWarps];
  __shared__ float red[40];
  __shared__ int ok_s;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = blockIdx.x * rpc;
  const int nr = min(rpc, d.dim - r0);
  if (threadIdx.x == 0) {
    mbar_init(&bar);
    // per expert rpc rows and rpc scale rows, each block contiguous and at a
    // 16-byte aligned offset (prow % 16 == 0, ng % 4 == 0, dim % rpc == 0)
    mbar_expect_tx(&bar, (uint32_t)(K * rpc * (prow + ng * 4)));
  }
  __syncthreads();
  if (threadIdx.x < K) {
    const int jx = threadIdx.x;
    const ExpertPtrs E = expert_ptrs(L, d.n_experts, __ldcg(b.sel + jx));
    const uint64_t pol = l2_evict_first();
    tma_load_hint(W + (size_t)jx * rpc * prow, E.dn + (size_t)r0 * prow, (uint32_t)(rpc * prow), &bar, pol);
    tma_load_hint(S + (size_t)jx * rpc * ng, E.dn_s + (size_t)r0 * ng, (uint32_t)(rpc * ng * 4), &bar, pol);
    selw_s[jx] = __ldcg(b.selw + jx);
  }
  // x[r] was last written by the O-projection, two launches back
  const float xold = threadIdx.x < nr ? __ldcg(b.x + r0 + threadIdx.x) : 0.0f;
  if (next_norm) load_f32(wn, next_norm, d.dim);
  CHALOT_TRACE(slot, 1);
  pdl_wait();
  pdl_trigger();
  CHALOT_TRACE(slot, 2);
  // the quantized h of every routed expert (the gate/up kernel's last CTA)
  if (threadIdx.x < K) xs_j[threadIdx.x] = __ldcg(b.xs_h + threadIdx.x);
  copy16(reinterpret_cast<uint4*>(xq), reinterpret_cast<const uint4*>(b.xq_h), (K * H) >> 4, true);
  if (threadIdx.x == 0) ok_s = mbar_wait(&bar, 0, b.err) ? 1 : 0;
  __syncthreads();
  CHALOT_TRACE(slot, 3);
  if (!ok_s) return;
  // group products: the warps of expert j split its chunks, and each x chunk
  // (read from shared memory once per CTA) serves the expert's rpc rows
  const int wpe = kWarps / K;  // warps per expert (K <= 8)
  if (warp < K * wpe) {
    const int jx = warp / wpe, wq = warp % wpe;
    const int8_t* xj = xq + (size_t)jx * H;
    const float xs = xs_j[jx];
    for (int c0 = wq * 32; c0 < chunks; c0 += 32 * wpe) {  // warp-uniform
      const int c = c0 + lane, cc = min(c, chunks - 1), g = cc >> gsh;
      const bool lead = c < chunks && (c & (cpg - 1)) == 0;
      const uint4 x0 = lds16(xj + (size_t)cc * 32), x1 = lds16(xj + (size_t)cc * 32 + 16);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (i < rpc) {  // CTA-uniform
          const int row = jx * rpc + i;
          int dv = dot32_rp(lds16(W + (size_t)row * prow + (size_t)cc * 16), x0, x1);
          for (int o = 1; o < cpg; o <<= 1) dv += __shfl_xor_sync(0xffffffffu, dv, o);
          if (lead) P[row * ng + g] = __fmul_rn(__fmul_rn((float)dv, S[row * ng + g]), xs);
        }
      }
    }
  }
  __syncthreads();
  if (warp < nrow && lane == 0) {  // row `warp`: t = t + p_g in group order, four groups per load
    const float* prow_p = P + (size_t)warp * ng;
    float t = 0.0f;
    int g4 = 0;
    for (; g4 + 4 <= (ng >> 2); g4 += 4) {
      float4 a[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) a[u] = lds16f(prow_p + 4 * (g4 + u));
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        t = __fadd_rn(t, a[u].x);
        t = __fadd_rn(t, a[u].y);
        t = __fadd_rn(t, a[u].z);
        t = __fadd_rn(t, a[u].w);
      }
    }
    for (; g4 < (ng >> 2); ++g4) {
      const float4 a = lds16f(prow_p + 4 * g4);
      t = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(t, a.x), a.y), a.z), a.w);
    }
    y[warp] = t;
  }
  __syncthreads();
  CHALOT_TRACE(slot, 4);
  if (threadIdx.x < nr) {
    float add;
    if (dense) {
      add = y[threadIdx.x];  // engine.rs:436-440
    } else {
      add = 0.0f;  // expert_out = sum_k w_k * y_k in selection order (engine.rs:390-396)
      for (int jx = 0; jx < K; ++jx) add = __fadd_rn(add, __fmul_rn(selw_s[jx], y[jx * rpc + threadIdx.x]));
    }
    b.x[r0 + threadIdx.x] = __fadd_rn(xold, add);
  }
  if (!next_norm) return;
  const bool tail = last_cta(b.counters + 2);
  CHALOT_TRACE(slot, 5);
  if (!tail) return;
  norm_quant_tail(b.x, wn, d.dim, b.xq_attn, b.xs_attn, xbuf, red);
  CHALOT_TRACE(slot, 6);
}

// ---- operators ---------------------------------------------------------------

// matmul_int4 over caller-owned memory, vector path (in_dim % 32 == 0,
// group % 32 == 0, 16-byte aligned rows).
constexpr int kOpRows = 16;
__global__ void __launch_bounds__(kThreads) k_matmul_i4_op(float* __restrict__ out,
                                                           const uint8_t* __restrict__ W,
                                                           const float* __restrict__ S,
                                                           const float* __restrict__ x, int out_dim,
                                                           int in_dim, int group) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int ng = in_dim / group, ps = ng + 1;
  int8_t* xp = reinterpret_cast<int8_t*>(smem);
  int* csum = reinterpret_cast<int*>(smem + in_dim);
  float* P = reinterpret_cast<float*>(smem + in_dim + (in_dim >> 5) * 4);
  __shared__ RowJob rows[kOpRows];
  __shared__ float red[40];
  __shared__ float xs_s[1];
  float m = 0.0f;
  for (int i = threadIdx.x; i < in_dim; i += blockDim.x) m = fmaxf(m, fabsf(x[i]));
  m = block_max(m, red);
  float scale, inv;
  quant_scale(m, &scale, &inv);
  for (int i = threadIdx.x; i < in_dim; i += blockDim.x) xp[perm32(i)] = quant_any(x[i], inv, i, in_dim);
  if (threadIdx.x == 0) xs_s[0] = scale;
  __syncthreads();
  chunk_sums(xp, in_dim, csum);
  __syncthreads();
  const int prow = in_dim >> 1;
  for (int rb = blockIdx.x * kOpRows; rb < out_dim; rb += gridDim.x * kOpRows) {
    if (threadIdx.x < kOpRows) {
      const int r = min(rb + (int)threadIdx.x, out_dim - 1);
      rows[threadIdx.x] = RowJob{W + (size_t)r * prow, S + (size_t)r * ng, 0};
    }
    __syncthreads();
    group_products_any(rows, kOpRows, in_dim, group, xp, csum, xs_s, P, ps);
    __syncthreads();
    if (threadIdx.x < kOpRows && rb + threadIdx.x < out_dim)
      out[rb + threadIdx.x] = ordered_sum(P + threadIdx.x * ps, ng);
    __syncthreads();
  }
}

// Generic matmul_int4 for shapes off the vector path: one thread per row,
// the same exact group dots and ordered sum.
__global__ void k_matmul_i4_generic(float* __restrict__ out, const uint8_t* __restrict__ W,
                                    const float* __restrict__ S, const float* __restrict__ x,
                                    int out_dim, int in_dim, int group) {
  extern __shared__ __align__(16) unsigned char smem[];
  int8_t* xq = reinterpret_cast<int8_t*>(smem);
  __shared__ float red[40];
  float m = 0.0f;
  for (int i = threadIdx.x; i < in_dim; i += blockDim.x) m = fmaxf(m, fabsf(x[i]));
  m = block_max(m, red);
  float scale, inv;
  quant_scale(m, &scale, &inv);
  for (int i = threadIdx.x; i < in_dim; i += blockDim.x) xq[i] = quant_any(x[i], inv, i, in_dim);
  __syncthreads();
  const int ng = (in_dim + group - 1) / group, prow = (in_dim + 1) / 2;
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < out_dim; r += gridDim.x * blockDim.x) {
    const uint8_t* row = W + (size_t)r * prow;
    float t = 0.0f;
    for (int g = 0; g < ng; ++g) {
      const int s = g * group, e = min(s + group, in_dim);
      int acc = 0;
      for (int k = s; k < e; ++k) {
        const uint8_t by = row[k >> 1];
        const int nb = (k & 1) ? (by >> 4) : (by & 0x0F);
        acc += (nb - 8) * (int)xq[k];
      }
      t = __fadd_rn(t, __fmul_rn(__fmul_rn((float)acc, S[(size_t)r * ng + g]), scale));
    }
    out[r] = t;
  }
}

__global__ void __launch_bounds__(kThreads) k_router_op(int32_t* idx, float* w,
                                                        const float* __restrict__ x,
                                                        const float* __restrict__ rw,
                                                        const float* __restrict__ rb, int dim,
                                                        int E, int k) {
  extern __shared__ __align__(16) unsigned char smem[];
  float* xb = reinterpret_cast<float*>(smem);
  float* lanes = xb + dim;
  float* logit = lanes + 16 * E;
  const float* xt = x + (size_t)blockIdx.x * dim;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) xb[i] = xt[i];
  __syncthreads();
  router_logits(rw, rb, xb, dim, E, lanes, logit);
  if (threadIdx.x < 32) topk_warp(logit, E, k, idx + (size_t)blockIdx.x * k, w + (size_t)blockIdx.x * k);
}

}  // namespace

static size_t down_smem(const Dims& d) {
  const size_t H = d.hidden, K = d.top_k, ng = H / d.group, prow = H / 2;
  return kWarps * prow + kWarps * ng * 4 + K * H + kWarps * ng * 4 + (size_t)d.dim * 8;
}

void launch_gateup(const Dims& d, const LayerPtrs& L, int layer, const DecodeBufs& b, cudaStream_t s,
                   bool pdl) {
  const int lc = (d.dim / 32 + 31) / 32;  // chunks per lane and row: dim <= 4096 gives 1..4
  const int it = lc <= 1 ? 1 : lc <= 2 ? 2 : 4;
  const int ppc = kWarps * (8 / it) / 2;
  dim3 grid((d.hidden + ppc - 1) / ppc, d.top_k);
  if (it == 1)
    launch_k(k_gateup<1>, grid, dim3(kThreads), 0, s, pdl, d, L, layer, b);
  else if (it == 2)
    launch_k(k_gateup<2>, grid, dim3(kThreads), 0, s, pdl, d, L, layer, b);
  else
    launch_k(k_gateup<4>, grid, dim3(kThreads), 0, s, pdl, d, L, layer, b);
}

void launch_down(const Dims& d, const LayerPtrs& L, int layer, const float* next_norm,
                 const DecodeBufs& b, cudaStream_t s, bool pdl) {
  const int rpc = std::max(1, kWarps / d.top_k);  // rows per CTA: the CTA's warps over all experts
  const int grid = (d.dim + rpc - 1) / rpc;
  const int dense = d.n_experts < 2 ? 1 : 0;
  const size_t smem = down_smem(d);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(k_down, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  launch_k(k_down, dim3(grid), dim3(kThreads), smem, s, pdl, d, L, layer, next_norm, b, dense, rpc);
}

cudaError_t repack_int4(uint8_t* p, size_t bytes, cudaStream_t s) {
  const size_t words = bytes / 4;
  if (words == 0) return cudaSuccess;
  const int grid = (int)std::min<size_t>((words + 255) / 256, 4096);
  k_repack_i4<<<grid, 256, 0, s>>>(reinterpret_cast<uint32_t*>(p), words);
  return cudaGetLastError();
}

cudaError_t op_matmul_i4(float* out, const uint8_t* wp, const float* ws, const float* x,
                         size_t out_dim, size_t in_dim, size_t group, int num_sms, cudaStream_t s) {
  const bool vec = in_dim % 32 == 0 && group % 32 == 0 && group <= 1024 && (group & (group - 1)) == 0 &&
                   ((reinterpret_cast<uintptr_t>(wp) & 15) == 0);
  if (vec) {
    const size_t ng = in_dim / group;
    const size_t smem = in_dim + (in_dim >> 5) * 4 + (size_t)kOpRows * (ng + 1) * 4;
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    cudaFuncSetAttribute(k_matmul_i4_op, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    const int grid = (int)std::min<size_t>((out_dim + kOpRows - 1) / kOpRows, (size_t)num_sms * 4);
    k_matmul_i4_op<<<std::max(grid, 1), kThreads, smem, s>>>(out, wp, ws, x, (int)out_dim,
                                                              (int)in_dim, (int)group);
  } else {
    const size_t smem = (in_dim + 15) & ~size_t(15);
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    cudaFuncSetAttribute(k_matmul_i4_generic, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    const int grid = (int)std::min<size_t>((out_dim + 255) / 256, (size_t)num_sms * 4);
    k_matmul_i4_generic<<<std::max(grid, 1), 256, smem, s>>>(out, wp, ws, x, (int)out_dim,
                                                            (int)in_dim, (int)group);
  }
  return cudaGetLastError();
}

cudaError_t op_router_topk(int32_t* idx, float* w, const float* x, const float* rw,
                           const float* rb, size_t n_tok, size_t dim, size_t n_experts,
                           size_t top_k, cudaStream_t s) {
  if (n_experts > 32 || top_k > n_experts || top_k == 0) return cudaErrorInvalidValue;
  const size_t smem = (dim + 17 * n_experts) * 4;
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  cudaFuncSetAttribute(k_router_op, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  k_router_op<<<(unsigned)n_tok, kThreads, smem, s>>>(idx, w, x, rw, rb, (int)dim, (int)n_experts,
                                                       (int)top_k);
  return cudaGetLastError();
}

#ifdef CHALOT_PHASE_TRACE
CHALOT_TRACE_EXPORT(trace_moe)
#endif

}  // namespace chalot
