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
          const uint4* xv = reinterpret_cast<const uint4*>(xp + (size_t)xsel * in_dim);
          int dv = 0;
          if (c < chunks) dv = dot32_u4(w[i][it], xv[2 * c], xv[2 * c + 1], 0) - 8 * csum[xsel * chunks + c];
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

constexpr int kGuPairs = 32;  // gate/up row pairs per CTA
constexpr int kSegs = 4;      // threads per gate/up row (the ordered sum is handed along)
constexpr int kMaxSegGroups = 16;  // groups per thread: dim / group <= 64

// Group dot of column group g of a repacked int4 row in shared memory with the
// natural-order x_q in shared memory (cpg 32-column chunks per group).
__device__ __forceinline__ int group_dot_smem(const uint8_t* wrow, const int8_t* xq, int g, int cpg) {
  int dv = 0;
  for (int cc = 0; cc < cpg; ++cc) {
    const int c = g * cpg + cc;
    const uint4 wv = *reinterpret_cast<const uint4*>(wrow + (size_t)c * 16);
    const uint4* xv = reinterpret_cast<const uint4*>(xq + (size_t)c * 32);
    dv += dot32_rp(wv, xv[0], xv[1]);
  }
  return dv;
}

// Gate rows base..base+31 and the matching up rows of routed expert
// sel[blockIdx.y] (engine.rs:366-374), then SwiGLU (activations.rs:59-87): h
// goes to global memory and |h| into the expert's absmax slot. The 64 rows
// arrive in shared memory by TMA bulk copies (one per row, row stride padded
// by 16 bytes); 4 threads share a row, each computing the exact products of a
// quarter of its groups, and the running sum is handed from quarter to
// quarter so the groups are added in order (matmul.rs:576-577). The last CTA
// quantizes every expert's finished h once for the down kernel.
__global__ void __launch_bounds__(kThreads) k_gateup(Dims d, LayerPtrs L, int layer, DecodeBufs b) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int slot = layer * 8 + 4;
  CHALOT_TRACE(slot, 0);
  const int ng = d.dim / d.group, cpg = d.group >> 5, prow = d.dim >> 1, wst = prow + 16;
  uint8_t* W = smem;                                                 // [64][wst]
  float* S = reinterpret_cast<float*>(smem + 2 * kGuPairs * wst);    // [64][ng]
  int8_t* xq = reinterpret_cast<int8_t*>(S + 2 * kGuPairs * ng);     // [dim]
  __shared__ __align__(8) uint64_t bar;
  __shared__ float xs_s;
  __shared__ float tots[2 * kGuPairs];
  __shared__ const uint8_t* gsrc[2];
  __shared__ const float* ssrc[2];

  const int H = d.hidden, j = blockIdx.y, base = blockIdx.x * kGuPairs;
  const int npairs = min(kGuPairs, H - base);
  if (threadIdx.x == 0) mbar_init(&bar);
  pdl_wait();  // the routing comes from the O-projection's last CTA
  pdl_trigger();
  CHALOT_TRACE(slot, 2);
  if (threadIdx.x == 0) {
    const ExpertPtrs X = expert_ptrs(L, d.n_experts, __ldcg(b.sel + j));
    gsrc[0] = X.gu + (size_t)base * prow;        // gate rows
    gsrc[1] = X.gu + (size_t)(H + base) * prow;  // up rows
    ssrc[0] = X.gu_s + (size_t)base * ng;
    ssrc[1] = X.gu_s + (size_t)(H + base) * ng;
    // rows and scales: npairs == 32 (hidden % 32 == 0), the scale blocks are
    // 32*ng floats (a multiple of 16 bytes) at 16-byte aligned offsets
    mbar_expect_tx(&bar, (uint32_t)(2 * npairs * prow + 2 * npairs * ng * 4));
  }
  __syncthreads();
  if (threadIdx.x < 2 * kGuPairs) {  // one bulk copy per row
    const int half = threadIdx.x / kGuPairs, i = threadIdx.x % kGuPairs;
    if (i < npairs) tma_load(W + threadIdx.x * wst, gsrc[half] + (size_t)i * prow, prow, &bar);
  } else if (threadIdx.x < 2 * kGuPairs + 2) {  // the two scale blocks
    const int half = threadIdx.x - 2 * kGuPairs;
    tma_load(S + half * kGuPairs * ng, ssrc[half], (uint32_t)(npairs * ng * 4), &bar);
  }
  copy16(reinterpret_cast<uint4*>(xq), reinterpret_cast<const uint4*>(b.xq_ffn), d.dim >> 4, true);
  if (threadIdx.x == 0) xs_s = __ldcg(b.xs_ffn);
  __syncthreads();
  CHALOT_TRACE(slot, 3);
  if (!mbar_wait(&bar, 0, b.err)) return;
  CHALOT_TRACE(layer * 8 + 7, 1);
  // row r = t/4, quarter q = t%4 over groups [q*ng/4, (q+1)*ng/4)
  const int r = threadIdx.x >> 2, q = threadIdx.x & 3;
  const int g0 = q * ng / kSegs, g1 = (q + 1) * ng / kSegs;
  const bool live = (r % kGuPairs) < npairs;
  const float xs = xs_s;
  float p[kMaxSegGroups];
#pragma unroll
  for (int i = 0; i < kMaxSegGroups; ++i) {
    const int g = g0 + i;
    p[i] = 0.0f;
    if (live && g < g1)
      p[i] = __fmul_rn(__fmul_rn((float)group_dot_smem(W + r * wst, xq, g, cpg), S[r * ng + g]), xs);
  }
  float acc = 0.0f;
  const int lane = threadIdx.x & 31, lead = lane & ~3;
#pragma unroll
  for (int st = 0; st < kSegs; ++st) {
    if (q == st)
#pragma unroll
      for (int i = 0; i < kMaxSegGroups; ++i)
        if (g0 + i < g1) acc = __fadd_rn(acc, p[i]);
    acc = __shfl_sync(0xffffffffu, acc, lead + st);
  }
  if (q == 0) tots[r] = acc;
  __syncthreads();
  CHALOT_TRACE(slot, 4);
  float m = 0.0f;
  if (threadIdx.x < npairs) {
    const int rr = base + threadIdx.x;
    const float hv = swiglu_elem(tots[threadIdx.x], tots[kGuPairs + threadIdx.x], rr, H);
    b.h[(size_t)j * H + rr] = hv;
    m = fabsf(hv);
  }
  m = warp_max(m);  // npairs <= 32: only warp 0 holds values
  if (threadIdx.x == 0) atomicMax(&b.amax[j], __float_as_uint(m));
  const bool tail = last_cta(b.counters + 3);
  CHALOT_TRACE(slot, 5);
  if (!tail) return;
  const int h4 = H >> 2;
  for (int jj = 0; jj < d.top_k; ++jj) {
    float scale, inv;
    quant_scale(__uint_as_float(__ldcg(b.amax + jj)), &scale, &inv);
    if (threadIdx.x == 0) b.xs_h[jj] = scale;
    quant_store_words(reinterpret_cast<uint32_t*>(b.xq_h) + (size_t)jj * h4,
                      reinterpret_cast<const float4*>(b.h) + (size_t)jj * h4, h4, inv, H);
  }
  CHALOT_TRACE(slot, 6);
}

// Output rows r0..r0+rpc-1 for every routed expert (one row per warp). The
// routing is two launches old, so the rows are requested by TMA bulk copies
// (and the scales and the next norm's weights staged) before waiting for the
// gate/up kernel; then each warp forms the exact group products against the
// quantized h and one thread per row adds them in group order; x[r] +=
// sum_j w_j * y_j[r] in selection order (engine.rs:380-401). The last CTA
// computes the next layer's quantized attention input from the finished x.
__global__ void __launch_bounds__(kThreads) k_down(Dims d, LayerPtrs L, int layer,
                                                   const float* next_norm, DecodeBufs b, int dense,
                                                   int rpc) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int slot = layer * 8 + 5;
  CHALOT_TRACE(slot, 0);
  const int H = d.hidden, K = d.top_k, ng = H / d.group, ps = ng + 1, cpg = d.group >> 5;
  const int prow = H >> 1, wst = prow + 16;
  const int nrow = K * rpc;  // <= kWarps
  uint8_t* W = smem;                                          // [nrow][wst]
  float* S = reinterpret_cast<float*>(W + kWarps * wst);      // [nrow][ng]
  int8_t* xq = reinterpret_cast<int8_t*>(S + kWarps * ng);    // [K][H]
  float* P = reinterpret_cast<float*>(xq + (size_t)K * H);    // [nrow][ng+1]
  float* wn = P + kWarps * ps;                                // [dim] next norm weights
  float* xb = wn + d.dim;                                     // [dim] tail scratch
  __shared__ __align__(8) uint64_t bar;
  __shared__ const uint8_t* rsrc[kWarps];
  __shared__ const float* ssrc[kWarps];
  __shared__ float xs_j[8];
  __shared__ float selw_s[8];
  __shared__ float y[kWarps];
  __shared__ float red[40];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = blockIdx.x * rpc;
  const int nr = min(rpc, d.dim - r0);
  if (threadIdx.x == 0) {
    mbar_init(&bar);
    // rows, and per expert one block of rpc scale rows (rpc*ng floats at a
    // 16-byte aligned offset: dim % rpc == 0, rpc*ng*4 % 16 == 0)
    mbar_expect_tx(&bar, (uint32_t)(nrow * prow + K * rpc * ng * 4));
  }
  if (threadIdx.x < nrow) {
    const int jx = threadIdx.x / rpc, i = threadIdx.x % rpc;
    const ExpertPtrs E = expert_ptrs(L, d.n_experts, __ldcg(b.sel + jx));
    const int r = r0 + i;  // dim % rpc == 0: every CTA has rpc whole rows
    rsrc[threadIdx.x] = E.dn + (size_t)r * prow;
    ssrc[threadIdx.x] = E.dn_s + (size_t)r * ng;
  }
  if (threadIdx.x < K) selw_s[threadIdx.x] = __ldcg(b.selw + threadIdx.x);
  __syncthreads();
  if (threadIdx.x < nrow) {
    tma_load(W + threadIdx.x * wst, rsrc[threadIdx.x], prow, &bar);
    if (threadIdx.x % rpc == 0)  // first row of each expert's block: its rpc scale rows
      tma_load(S + threadIdx.x * ng, ssrc[threadIdx.x], (uint32_t)(rpc * ng * 4), &bar);
  }
  load_f32(wn, next_norm, d.dim);
  CHALOT_TRACE(slot, 1);
  pdl_wait();
  pdl_trigger();
  CHALOT_TRACE(slot, 2);
  // the quantized h of every routed expert (the gate/up kernel's last CTA)
  copy16(reinterpret_cast<uint4*>(xq), reinterpret_cast<const uint4*>(b.xq_h), (K * H) >> 4, true);
  if (threadIdx.x < K) xs_j[threadIdx.x] = __ldcg(b.xs_h + threadIdx.x);
  __syncthreads();
  CHALOT_TRACE(slot, 3);
  if (!mbar_wait(&bar, 0, b.err)) return;
#ifdef CHALOT_PHASE_TRACE
  long long c0_ = clock64();
#endif
  if (warp < nrow) {
    const int jx = warp / rpc;
    const int8_t* xj = xq + (size_t)jx * H;
    const uint8_t* wrow = W + warp * wst;
    const float xs = xs_j[jx];
    for (int g = lane; g < ng; g += 32)
      P[warp * ps + g] = __fmul_rn(__fmul_rn((float)group_dot_smem(wrow, xj, g, cpg), S[warp * ng + g]), xs);
  }
  __syncthreads();
  if (threadIdx.x < nrow) y[threadIdx.x] = ordered_sum(P + threadIdx.x * ps, ng);
  __syncthreads();
  CHALOT_TRACE(slot, 4);
#ifdef CHALOT_PHASE_TRACE
  if (threadIdx.x == 0 && blockIdx.x == 0)  // SM cycles of the compute, next to its ns (phases 3..4)
    g_phase_trace[((size_t)(layer * 8 + 7) * kTraceCtas + 1000) * kTracePhases] = clock64() - c0_;
#endif
  if (threadIdx.x < nr) {
    const int r = r0 + threadIdx.x;
    float add;
    if (dense) {
      add = y[threadIdx.x];  // engine.rs:436-440
    } else {
      add = 0.0f;  // expert_out = sum_k w_k * y_k in selection order (engine.rs:390-396)
      for (int j = 0; j < K; ++j) add = __fadd_rn(add, __fmul_rn(selw_s[j], y[j * rpc + threadIdx.x]));
    }
    b.x[r] = __fadd_rn(__ldcg(b.x + r), add);
  }
  const bool tail = last_cta(b.counters + 2);
  CHALOT_TRACE(slot, 5);
  if (!tail) return;
  norm_quant_tail(b.x, wn, d.dim, b.xq_attn, b.xs_attn, xb, red);
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

static size_t gateup_smem(const Dims& d) {
  const size_t ng = d.dim / d.group, wst = d.dim / 2 + 16;
  return 2 * kGuPairs * wst + 2 * kGuPairs * ng * 4 + d.dim;
}
static size_t down_smem(const Dims& d) {
  const size_t H = d.hidden, K = d.top_k, ng = H / d.group, wst = H / 2 + 16;
  return kWarps * wst + kWarps * ng * 4 + K * H + kWarps * (ng + 1) * 4 + (size_t)d.dim * 8;
}

void launch_gateup(const Dims& d, const LayerPtrs& L, int layer, const DecodeBufs& b, cudaStream_t s,
                   bool pdl) {
  const size_t smem = gateup_smem(d);
  if (smem > 48 * 1024) cudaFuncSetAttribute(k_gateup, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid((d.hidden + kGuPairs - 1) / kGuPairs, d.top_k);
  launch_k(k_gateup, grid, dim3(kThreads), smem, s, pdl, d, L, layer, b);
}

void launch_down(const Dims& d, const LayerPtrs& L, int layer, const float* next_norm,
                 const DecodeBufs& b, cudaStream_t s, bool pdl) {
  const int rpc = std::max(1, kWarps / d.top_k);  // rows per CTA: one row per warp over all experts
  const size_t smem = down_smem(d);
  const int grid = (d.dim + rpc - 1) / rpc;
  const int dense = d.n_experts < 2 ? 1 : 0;
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
