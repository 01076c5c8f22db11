// k_attn.cu — decode attention over the f32 KV cache in the reference's
// rounding order (src/model/engine.rs:283-309).
//
//   k_attn_scores  s[h][t] = 30 * tanh((dot_f32(q_h, K[t]_h) * (1/sqrt(hd))) / 30)
//                  for t <= pos; one thread per (head, t), the dot in the
//                  two-accumulator 8-lane order of dot_f32_avx2
//                  (src/tensor/attention_helpers.rs:41-80) and the cap of
//                  logit_soft_cap (src/tensor/activations.rs:133-135) with the
//                  host libm's tanhf restated in libm_f32.h.
//   k_attn_pv      softmax_avx2 over s[h][0..pos] (normalization.rs:106-160),
//                  then out[d] = sum_t p_t * V[t][d] added in t order
//                  (engine.rs:302-308). The add chain of a column is serial by
//                  definition, so each CTA owns 8 columns of one head: its 256
//                  threads stage V[0..pos][8 columns] in shared memory with
//                  wide loads (spreading the KV read over heads*hd/8 CTAs),
//                  transposed so each column is contiguous, and 8 threads then
//                  run the chains out of shared memory, loading the next 16
//                  products while adding the current ones.
// The cache layout is the reference's: [layer][max_seq][dim], head h at
// columns h*hd .. h*hd+hd-1.
#include <cuda_runtime.h>

#include "blockops.cuh"
#include "kernels.cuh"
#include "pdl.cuh"

namespace chalot {
namespace {

constexpr int kScoreThreads = 128;

// K row of (layer, t, head h): 16 floats per c16 step, loaded as float4.
template <int C16>
__device__ __forceinline__ void load_k_row(const float* k, float4 (&kr)[C16 * 4]) {
#pragma unroll
  for (int i = 0; i < C16 * 4; ++i) kr[i] = reinterpret_cast<const float4*>(k)[i];
}

template <int C16>  // head_dim / 16
__global__ void __launch_bounds__(kScoreThreads) k_attn_scores(Dims d, int layer, DecodeBufs b) {
  __shared__ __align__(16) float qh[256];
  [[maybe_unused]] const int slot = layer * 8 + 1;
  CHALOT_TRACE(slot, 0);
  const int h = blockIdx.y, hd = d.head_dim;
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t pos = b.st->pos;
  const float* k = b.kc + ((size_t)layer * d.max_seq + t) * d.dim + (size_t)h * hd;
  float4 kr[C16 * 4];
  // rows before pos were written by earlier forwards: load them before waiting
  if ((uint32_t)t < pos) load_k_row<C16>(k, kr);
  CHALOT_TRACE(slot, 1);
  pdl_wait();
  pdl_trigger();
  CHALOT_TRACE(slot, 2);
  if (blockIdx.x * blockDim.x > pos) return;  // whole CTA beyond the causal range
  for (int i = threadIdx.x; i < hd; i += blockDim.x) qh[i] = __ldcg(b.q + h * hd + i);
  __syncthreads();
  if ((uint32_t)t > pos) return;
  if ((uint32_t)t == pos) {  // this forward's key, written by the QKV kernel
#pragma unroll
    for (int i = 0; i < C16 * 4; ++i) kr[i] = __ldcg(reinterpret_cast<const float4*>(k) + i);
  }
  const float* kk = reinterpret_cast<const float*>(kr);
  float a0[8], a1[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) a0[j] = a1[j] = 0.0f;
#pragma unroll
  for (int c = 0; c < C16; ++c)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      a0[j] = __fadd_rn(a0[j], __fmul_rn(qh[c * 16 + j], kk[c * 16 + j]));
      a1[j] = __fadd_rn(a1[j], __fmul_rn(qh[c * 16 + 8 + j], kk[c * 16 + 8 + j]));
    }
  const int rem = C16 * 16;
  const bool extra = rem + 8 <= hd;  // head_dim % 16 == 8: one more 8-chunk into a0
  if (extra)
#pragma unroll
    for (int j = 0; j < 8; ++j) a0[j] = __fadd_rn(a0[j], __fmul_rn(qh[rem + j], __ldcg(k + rem + j)));
  float cmb[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) cmb[j] = __fadd_rn(a0[j], a1[j]);
  const float dot = hsum8(cmb);
  const float inv_sqrt = div_rn(1.0f, __fsqrt_rn((float)hd));
  const float x = __fmul_rn(dot, inv_sqrt);
  b.scores[(size_t)h * d.max_seq + t] = __fmul_rn(30.0f, libm::tanh_f32(div_rn(x, 30.0f)));
}

constexpr int kPvThreads = 256;
constexpr int kPvCols = 8;     // output columns per CTA: V loads spread over heads*hd/8 CTAs
constexpr int kPvTile = 1024;  // V rows staged in shared memory at a time
constexpr int kPvLd = kPvTile + 4;  // row stride of the staged columns (16-byte aligned, bank spread)

// Stages V[t0 .. t0+rows)[8 columns] transposed into vt[col][t - t0 + off]:
// each column contiguous, so a chain thread reads its column four t at a time.
__device__ __forceinline__ void stage_v(float* vt, const float* vbase, int dim, int t0, int rows, int off,
                                        bool coherent) {
  constexpr int U = 8;
  const int n = rows * (kPvCols / 4);
  for (int base = 0; base < n; base += U * kPvThreads) {
    float4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * kPvThreads + (int)threadIdx.x;
      if (i < n) {
        const int r = i / (kPvCols / 4), q = i % (kPvCols / 4);
        const float4* src = reinterpret_cast<const float4*>(vbase + (size_t)(t0 + r) * dim + q * 4);
        v[u] = coherent ? __ldcg(src) : __ldg(src);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * kPvThreads + (int)threadIdx.x;
      if (i < n) {
        const int r = i / (kPvCols / 4), q = i % (kPvCols / 4);
        float* d = vt + (q * 4) * kPvLd + off + r;
        d[0] = v[u].x;
        d[kPvLd] = v[u].y;
        d[2 * kPvLd] = v[u].z;
        d[3 * kPvLd] = v[u].w;
      }
    }
  }
}

__global__ void __launch_bounds__(kPvThreads) k_attn_pv(Dims d, int layer, DecodeBufs b) {
  extern __shared__ __align__(16) float sm[];
  [[maybe_unused]] const int slot = layer * 8 + 2;
  CHALOT_TRACE(slot, 0);
  float* p = sm;                            // [max_seq] probabilities
  float* vt = sm + ((d.max_seq + 3) & ~3);  // [kPvCols][kPvLd] staged V columns (16-B aligned)
  __shared__ float red[40];
  __shared__ float inv_s;
  const int h = blockIdx.x, hd = d.head_dim, c0 = blockIdx.y * kPvCols;
  const int n = (int)b.st->pos + 1;
  const float* vbase = b.vc + (size_t)layer * d.max_seq * d.dim + (size_t)h * hd + c0;
  // V rows 0..n-2 of the first tile were written by earlier forwards
  stage_v(vt, vbase, d.dim, 0, min(n - 1, kPvTile), 0, false);
  CHALOT_TRACE(slot, 1);
  pdl_wait();
  pdl_trigger();
  CHALOT_TRACE(slot, 2);
  if (n - 1 < kPvTile) stage_v(vt, vbase, d.dim, n - 1, 1, n - 1, true);
  const float* s = b.scores + (size_t)h * d.max_seq;
  // softmax_avx2 over the n scores of this head (normalization.rs:106-160)
  float mx = -INFINITY;
  for (int base = 0; base < n; base += 8 * kPvThreads) {  // 8 loads in flight per thread
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = base + u * kPvThreads + (int)threadIdx.x;
      v[u] = i < n ? __ldcg(s + i) : -INFINITY;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = base + u * kPvThreads + (int)threadIdx.x;
      if (i < n) p[i] = v[u];
      mx = fmaxf(mx, v[u]);
    }
  }
  mx = block_max(mx, red);
  const int full = n & ~7;
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    if (i < full)
      p[i] = fast_exp(__fsub_rn(p[i], mx));
    else
      p[i] = expf_cr(__fsub_rn(p[i], mx));
  __syncthreads();
  if (threadIdx.x < 8) {  // lane j sums elements 8c+j in c order
    float acc = 0.0f;
    int c = 0;
    const int nc = full >> 3;
    for (; c + 8 <= nc; c += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = p[(c + u) * 8 + threadIdx.x];
#pragma unroll
      for (int u = 0; u < 8; ++u) acc = __fadd_rn(acc, v[u]);
    }
    for (; c < nc; ++c) acc = __fadd_rn(acc, p[c * 8 + threadIdx.x]);
    red[threadIdx.x] = acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float l8[8];
    for (int j = 0; j < 8; ++j) l8[j] = red[j];
    float sum = hsum8(l8);
    for (int i = full; i < n; ++i) sum = __fadd_rn(sum, p[i]);
    inv_s = div_rn(1.0f, sum);
  }
  __syncthreads();
  const float inv = inv_s;
  for (int i = threadIdx.x; i < n; i += blockDim.x) p[i] = __fmul_rn(p[i], inv);
  __syncthreads();
  CHALOT_TRACE(slot, 3);
  // out[c] = sum_t p_t * V[t][c], added in t order (engine.rs:302-308): the
  // products of the next 16 t are loaded while this block's adds run
  float acc = 0.0f;
  for (int t0 = 0; t0 < n; t0 += kPvTile) {
    const int rows = min(kPvTile, n - t0);
    if (t0 > 0) {  // later tiles: stage now
      __syncthreads();
      stage_v(vt, vbase, d.dim, t0, rows, 0, true);
      __syncthreads();
    }
    if (threadIdx.x < kPvCols) {
      const float* pv = p + t0;  // t0 % 4 == 0: 16-byte aligned
      const float* vc = vt + threadIdx.x * kPvLd;
      int t = 0;
      if (rows >= 16) {
        float4 pa[4], va[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          pa[u] = lds16f(pv + 4 * u);
          va[u] = lds16f(vc + 4 * u);
        }
        for (; t + 16 <= rows; t += 16) {
          float4 pb[4], vb[4];
          const bool more = t + 32 <= rows;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            pb[u] = more ? lds16f(pv + t + 16 + 4 * u) : pa[u];
            vb[u] = more ? lds16f(vc + t + 16 + 4 * u) : va[u];
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            acc = __fadd_rn(acc, __fmul_rn(pa[u].x, va[u].x));
            acc = __fadd_rn(acc, __fmul_rn(pa[u].y, va[u].y));
            acc = __fadd_rn(acc, __fmul_rn(pa[u].z, va[u].z));
            acc = __fadd_rn(acc, __fmul_rn(pa[u].w, va[u].w));
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            pa[u] = pb[u];
            va[u] = vb[u];
          }
        }
      }
      for (; t < rows; ++t) acc = __fadd_rn(acc, __fmul_rn(pv[t], vc[t]));
    }
  }
  if (threadIdx.x < kPvCols) b.att_out[h * hd + c0 + threadIdx.x] = acc;
  CHALOT_TRACE(slot, 4);
}

}  // namespace

void launch_scores(const Dims& d, int layer, const DecodeBufs& b, cudaStream_t s, bool pdl) {
  dim3 g1((d.max_seq + kScoreThreads - 1) / kScoreThreads, d.n_heads);
  switch (d.head_dim / 16) {  // 16 <= head_dim <= 256, head_dim % 8 == 0
    case 1: launch_k(k_attn_scores<1>, g1, dim3(kScoreThreads), 0, s, pdl, d, layer, b); break;
    case 2: launch_k(k_attn_scores<2>, g1, dim3(kScoreThreads), 0, s, pdl, d, layer, b); break;
    case 3: launch_k(k_attn_scores<3>, g1, dim3(kScoreThreads), 0, s, pdl, d, layer, b); break;
    case 4: launch_k(k_attn_scores<4>, g1, dim3(kScoreThreads), 0, s, pdl, d, layer, b); break;
    case 5: launch_k(k_attn_scores<5>, g1, dim3(kScoreThreads), 0, s, pdl, d, layer, b); break;
    case 6: launch_k(k_attn_scores<6>, g1, dim3(kScoreThreads), 0, s, pdl, d, layer, b); break;
    case 7: launch_k(k_attn_scores<7>, g1, dim3(kScoreThreads), 0, s, pdl, d, layer, b); break;
    case 8: launch_k(k_attn_scores<8>, g1, dim3(kScoreThreads), 0, s, pdl, d, layer, b); break;
    case 9: launch_k(k_attn_scores<9>, g1, dim3(kScoreThreads), 0, s, pdl, d, layer, b); break;
    case 10: launch_k(k_attn_scores<10>, g1, dim3(kScoreThreads), 0, s, pdl, d, layer, b); break;
    case 11: launch_k(k_attn_scores<11>, g1, dim3(kScoreThreads), 0, s, pdl, d, layer, b); break;
    case 12: launch_k(k_attn_scores<12>, g1, dim3(kScoreThreads), 0, s, pdl, d, layer, b); break;
    case 13: launch_k(k_attn_scores<13>, g1, dim3(kScoreThreads), 0, s, pdl, d, layer, b); break;
    case 14: launch_k(k_attn_scores<14>, g1, dim3(kScoreThreads), 0, s, pdl, d, layer, b); break;
    case 15: launch_k(k_attn_scores<15>, g1, dim3(kScoreThreads), 0, s, pdl, d, layer, b); break;
    default: launch_k(k_attn_scores<16>, g1, dim3(kScoreThreads), 0, s, pdl, d, layer, b); break;
  }
}

void launch_pv(const Dims& d, int layer, const DecodeBufs& b, cudaStream_t s, bool pdl) {
  dim3 g2(d.n_heads, d.head_dim / kPvCols);
  const size_t smem = ((((size_t)d.max_seq + 3) & ~size_t(3)) + (size_t)kPvLd * kPvCols) * 4;
  if (smem > 48 * 1024) cudaFuncSetAttribute(k_attn_pv, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  launch_k(k_attn_pv, g2, dim3(kPvThreads), smem, s, pdl, d, layer, b);
}

void launch_attention(const Dims& d, int layer, const DecodeBufs& b, cudaStream_t s, bool pdl) {
  launch_scores(d, layer, b, s, pdl);
  launch_pv(d, layer, b, s, pdl);
}

#ifdef CHALOT_PHASE_TRACE
CHALOT_TRACE_EXPORT(trace_attn)
#endif

}  // namespace chalot
