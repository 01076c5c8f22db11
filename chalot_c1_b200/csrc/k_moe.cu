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
//   k_router  rmsnorm(x) -> quantize -> router logits -> softmax top-k
//             (engine.rs:325-344)
//   k_gateup  gate and up rows of the selected experts -> SwiGLU -> h and
//             absmax(h) (engine.rs:366-377)
//   k_down    quantize(h) -> down rows of every selected expert -> gated sum in
//             selection order -> x += (engine.rs:380-401)
#include <cuda_runtime.h>

#include <algorithm>

#include "blockops.cuh"
#include "kernels.cuh"

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
  for (int r0 = warp * R; r0 < nrows; r0 += kWarps * R) {
    for (int cb = 0; cb < chunks; cb += 32 * IT) {
      uint4 w[R][IT];
#pragma unroll
      for (int i = 0; i < R; ++i)
#pragma unroll
        for (int it = 0; it < IT; ++it) {
          const int c = cb + it * 32 + lane;
          w[i][it] = (c < chunks && r0 + i < nrows) ? ldg_stream(rows[r0 + i].w + (size_t)c * 16)
                                                    : make_uint4(0, 0, 0, 0);
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
          if (live && c < chunks && (c % cpg) == 0) {
            const int g = c / cpg;
            P[(r0 + i) * ps + g] = __fmul_rn(__fmul_rn((float)dv, rows[r0 + i].s[g]), xs[xsel]);
          }
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

// Ordered group sum of one row: t = t + p_g for g = 0..ng-1 (matmul.rs:576-577).
__device__ __forceinline__ float ordered_sum(const float* p, int ng) {
  float t = 0.0f;
  for (int g = 0; g < ng; ++g) t = __fadd_rn(t, p[g]);
  return t;
}

// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(kThreads) k_router(Dims d, LayerPtrs L, int layer, DecodeBufs b) {
  extern __shared__ __align__(16) unsigned char smem[];
  float* xb = reinterpret_cast<float*>(smem);
  float* lanes = xb + d.dim;                 // [16*E]
  float* logit = lanes + 16 * d.n_experts;  // [E]
  __shared__ float red[40];
  rmsnorm_smem(b.x, L.rms_ffn, d.dim, xb, red);  // engine.rs:325-329
  const float xs = quantize_smem(xb, d.dim, b.xq_ffn, red);
  if (threadIdx.x < d.top_k) b.amax[threadIdx.x] = 0u;
  if (threadIdx.x == 0) *b.xs_ffn = xs;
  if (d.n_experts >= 2) {
    router_logits(L.router_w, L.router_b, xb, d.dim, d.n_experts, lanes, logit);
    if (threadIdx.x == 0) {
      if (b.router_trace)
        for (int e = 0; e < d.n_experts; ++e) b.router_trace[layer * d.n_experts + e] = logit[e];
      topk_serial(logit, d.n_experts, d.top_k, b.sel, b.selw);
    }
  } else if (threadIdx.x == 0) {
    b.sel[0] = 0;
    b.selw[0] = 1.0f;
  }
}

constexpr int kGuPairs = 32;  // gate/up row pairs per CTA

__global__ void __launch_bounds__(kThreads) k_gateup(Dims d, LayerPtrs L, DecodeBufs b) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int ng = d.dim / d.group, ps = ng + 1;
  int8_t* xp = reinterpret_cast<int8_t*>(smem);
  int* csum = reinterpret_cast<int*>(smem + d.dim);
  float* P = reinterpret_cast<float*>(smem + d.dim + (d.dim >> 5) * 4);
  __shared__ RowJob rows[2 * kGuPairs];
  __shared__ float xs_s[1];
  __shared__ float tots[2 * kGuPairs];

  const int j = blockIdx.y;
  const ExpertPtrs E = L.experts[b.sel[j]];
  const int H = d.hidden, prow = d.dim >> 1;
  const int base = blockIdx.x * kGuPairs;
  const int npairs = min(kGuPairs, H - base);
  if (threadIdx.x < 2 * kGuPairs) {
    const int i = threadIdx.x, k = i % kGuPairs;
    const int r = (i < kGuPairs ? base : H + base) + min(k, npairs - 1);  // gate rows, then up rows
    rows[i] = RowJob{E.gu + (size_t)r * prow, E.gu_s + (size_t)r * ng, 0};
  }
  // the quantized FFN input (xb of the router) in permuted order
  for (int i = threadIdx.x; i < d.dim; i += blockDim.x) xp[perm32(i)] = b.xq_ffn[i];
  if (threadIdx.x == 0) xs_s[0] = *b.xs_ffn;
  __syncthreads();
  for (int c = threadIdx.x; c < (d.dim >> 5); c += blockDim.x) {
    int s = 0;
    for (int i = 0; i < 32; ++i) s += xp[c * 32 + i];
    csum[c] = s;
  }
  __syncthreads();
  group_products_any(rows, 2 * kGuPairs, d.dim, d.group, xp, csum, xs_s, P, ps);
  __syncthreads();
  if (threadIdx.x < 2 * kGuPairs) tots[threadIdx.x] = ordered_sum(P + threadIdx.x * ps, ng);
  __syncthreads();
  float m = 0.0f;
  if (threadIdx.x < npairs) {
    const int r = base + threadIdx.x;
    const float hv = swiglu_elem(tots[threadIdx.x], tots[kGuPairs + threadIdx.x], r, H);
    b.h[(size_t)j * H + r] = hv;
    m = fabsf(hv);
  }
  m = warp_max(m);  // npairs <= 32: only warp 0 holds values
  if (threadIdx.x == 0) atomicMax(&b.amax[j], __float_as_uint(m));
}

constexpr int kDnRows = 4;  // output rows per CTA (for every selected expert)

__global__ void __launch_bounds__(kThreads) k_down(Dims d, LayerPtrs L, DecodeBufs b, int dense) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int H = d.hidden, K = d.top_k, ng = H / d.group, ps = ng + 1;
  int8_t* xp = reinterpret_cast<int8_t*>(smem);                        // [K][H]
  int* csum = reinterpret_cast<int*>(smem + (size_t)K * H);             // [K][H/32]
  float* P = reinterpret_cast<float*>(smem + (size_t)K * H + (size_t)K * (H >> 5) * 4);
  __shared__ RowJob rows[8 * kDnRows];
  __shared__ float xs_j[8];
  __shared__ float y[8 * kDnRows];

  const int r0 = blockIdx.x * kDnRows;
  const int nr = min(kDnRows, d.dim - r0);
  const int prow = H >> 1;
  if (threadIdx.x < K * kDnRows) {
    const int j = threadIdx.x / kDnRows, i = threadIdx.x % kDnRows;
    const ExpertPtrs E = L.experts[b.sel[j]];
    const int r = r0 + min(i, nr - 1);
    rows[threadIdx.x] = RowJob{E.dn + (size_t)r * prow, E.dn_s + (size_t)r * ng, j};
  }
  // quantize h of every selected expert with the absmax the gate/up kernel
  // accumulated (quantize_f32_to_i8 of the down projection's input, engine.rs:383-384)
  for (int j = 0; j < K; ++j) {
    float scale, inv;
    quant_scale(__uint_as_float(b.amax[j]), &scale, &inv);
    const float* hj = b.h + (size_t)j * H;
    int8_t* xj = xp + (size_t)j * H;
    for (int i = threadIdx.x; i < H; i += blockDim.x) xj[perm32(i)] = quant_any(hj[i], inv, i, H);
    if (threadIdx.x == 0) xs_j[j] = scale;
  }
  __syncthreads();
  for (int c = threadIdx.x; c < K * (H >> 5); c += blockDim.x) {
    const int8_t* p = xp + (size_t)c * 32;
    int s = 0;
    for (int i = 0; i < 32; ++i) s += p[i];
    csum[c] = s;
  }
  __syncthreads();
  group_products_any(rows, K * kDnRows, H, d.group, xp, csum, xs_j, P, ps);
  __syncthreads();
  if (threadIdx.x < K * kDnRows) y[threadIdx.x] = ordered_sum(P + threadIdx.x * ps, ng);
  __syncthreads();
  if (threadIdx.x < nr) {
    const int r = r0 + threadIdx.x;
    float add;
    if (dense) {
      add = y[threadIdx.x];  // engine.rs:436-440
    } else {
      add = 0.0f;  // expert_out = sum_k w_k * y_k in selection order (engine.rs:390-396)
      for (int j = 0; j < K; ++j) add = __fadd_rn(add, __fmul_rn(b.selw[j], y[j * kDnRows + threadIdx.x]));
    }
    b.x[r] = __fadd_rn(b.x[r], add);
  }
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
  for (int c = threadIdx.x; c < (in_dim >> 5); c += blockDim.x) {
    int s = 0;
    for (int i = 0; i < 32; ++i) s += xp[c * 32 + i];
    csum[c] = s;
  }
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
  if (threadIdx.x == 0) topk_serial(logit, E, k, idx + (size_t)blockIdx.x * k, w + (size_t)blockIdx.x * k);
}

}  // namespace

void launch_router(const Dims& d, const LayerPtrs& L, int layer, const DecodeBufs& b, cudaStream_t s) {
  const size_t smem = ((size_t)d.dim + 17 * (size_t)d.n_experts) * 4;
  k_router<<<1, kThreads, smem, s>>>(d, L, layer, b);
}

static size_t gateup_smem(const Dims& d) {
  const int ng = d.dim / d.group;
  return (size_t)d.dim + (size_t)(d.dim >> 5) * 4 + (size_t)2 * kGuPairs * (ng + 1) * 4;
}
static size_t down_smem(const Dims& d) {
  const size_t H = d.hidden, K = d.top_k, ng = H / d.group;
  return K * H + K * (H >> 5) * 4 + K * kDnRows * (ng + 1) * 4;
}

void launch_gateup(const Dims& d, const LayerPtrs& L, const DecodeBufs& b, cudaStream_t s) {
  const size_t smem = gateup_smem(d);
  static unsigned long long done_mask = 0;  // devices whose attributes are set
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !(done_mask & (1ull << dev))) {
    cudaFuncSetAttribute(k_gateup, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    cudaFuncSetAttribute(k_down, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    __atomic_fetch_or(&done_mask, 1ull << dev, __ATOMIC_RELAXED);
  }
  dim3 grid((d.hidden + kGuPairs - 1) / kGuPairs, d.top_k);
  k_gateup<<<grid, kThreads, smem, s>>>(d, L, b);
}

void launch_down(const Dims& d, const LayerPtrs& L, const DecodeBufs& b, cudaStream_t s) {
  k_down<<<(d.dim + kDnRows - 1) / kDnRows, kThreads, down_smem(d), s>>>(d, L, b,
                                                                        d.n_experts < 2 ? 1 : 0);
}

cudaError_t op_matmul_i4(float* out, const uint8_t* wp, const float* ws, const float* x,
                         size_t out_dim, size_t in_dim, size_t group, int num_sms, cudaStream_t s) {
  const bool vec = in_dim % 32 == 0 && group % 32 == 0 && ((reinterpret_cast<uintptr_t>(wp) & 15) == 0);
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
  if (n_experts > 64 || top_k > n_experts || top_k == 0) return cudaErrorInvalidValue;
  const size_t smem = (dim + 17 * n_experts) * 4;
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  cudaFuncSetAttribute(k_router_op, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  k_router_op<<<(unsigned)n_tok, kThreads, smem, s>>>(idx, w, x, rw, rb, (int)dim, (int)n_experts,
                                                       (int)top_k);
  return cudaGetLastError();
}

}  // namespace chalot
