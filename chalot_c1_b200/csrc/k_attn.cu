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
//                  wide loads (spreading the KV read over heads*hd/8 CTAs) and
//                  8 threads then run the chains out of shared memory.
// The cache layout is the reference's: [layer][max_seq][dim], head h at
// columns h*hd .. h*hd+hd-1.
#include <cuda_runtime.h>

#include "blockops.cuh"
#include "kernels.cuh"

namespace chalot {
namespace {

constexpr int kScoreThreads = 128;

__global__ void __launch_bounds__(kScoreThreads) k_attn_scores(Dims d, int layer, DecodeBufs b) {
  __shared__ __align__(16) float qh[256];
  const int h = blockIdx.y, hd = d.head_dim;
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t pos = b.st->pos;
  if (blockIdx.x * blockDim.x > pos) return;  // whole CTA beyond the causal range
  for (int i = threadIdx.x; i < hd; i += blockDim.x) qh[i] = b.q[h * hd + i];
  __syncthreads();
  if ((uint32_t)t > pos) return;
  const float* k = b.kc + ((size_t)layer * d.max_seq + t) * d.dim + (size_t)h * hd;
  float a0[8], a1[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) a0[j] = a1[j] = 0.0f;
  const int c16 = hd >> 4, rem = c16 * 16;
  for (int c = 0; c < c16; ++c) {
    const float4* kv = reinterpret_cast<const float4*>(k + c * 16);
    const float4 k0 = kv[0], k1 = kv[1], k2 = kv[2], k3 = kv[3];
    const float kk[16] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w,
                          k2.x, k2.y, k2.z, k2.w, k3.x, k3.y, k3.z, k3.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      a0[j] = __fadd_rn(a0[j], __fmul_rn(qh[c * 16 + j], kk[j]));
      a1[j] = __fadd_rn(a1[j], __fmul_rn(qh[c * 16 + 8 + j], kk[8 + j]));
    }
  }
  const bool extra = rem + 8 <= hd;
  if (extra)
#pragma unroll
    for (int j = 0; j < 8; ++j) a0[j] = __fadd_rn(a0[j], __fmul_rn(qh[rem + j], k[rem + j]));
  float cmb[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) cmb[j] = __fadd_rn(a0[j], a1[j]);
  float dot = hsum8(cmb);
  for (int i = extra ? rem + 8 : rem; i < hd; ++i) dot = __fadd_rn(dot, __fmul_rn(qh[i], k[i]));
  const float inv_sqrt = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));
  const float x = __fmul_rn(dot, inv_sqrt);
  b.scores[(size_t)h * d.max_seq + t] = __fmul_rn(30.0f, libm::tanh_f32(__fdiv_rn(x, 30.0f)));
}

constexpr int kPvThreads = 256;
constexpr int kPvCols = 8;     // output columns per CTA: V loads spread over heads*hd/8 CTAs
constexpr int kPvTile = 1024;  // V rows staged in shared memory at a time

__global__ void __launch_bounds__(kPvThreads) k_attn_pv(Dims d, int layer, DecodeBufs b) {
  extern __shared__ __align__(16) float sm[];
  float* p = sm;                      // [max_seq] probabilities
  float* vt = sm + ((d.max_seq + 3) & ~3);  // [kPvTile][kPvCols] staged V (16-B aligned)
  __shared__ float red[40];
  __shared__ float inv_s;
  const int h = blockIdx.x, hd = d.head_dim, c0 = blockIdx.y * kPvCols;
  const int n = (int)b.st->pos + 1;
  const float* s = b.scores + (size_t)h * d.max_seq;
  // softmax_avx2 over the n scores of this head (normalization.rs:106-160)
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = s[i];
    p[i] = v;
    mx = fmaxf(mx, v);
  }
  mx = block_max(mx, red);
  const int full = n & ~7;
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    p[i] = (i < full) ? fast_exp(__fsub_rn(p[i], mx)) : expf_cr(__fsub_rn(p[i], mx));
  __syncthreads();
  if (threadIdx.x < 8) {  // lane j sums elements 8c+j in c order
    float acc = 0.0f;
    for (int c = 0; c < (full >> 3); ++c) acc = __fadd_rn(acc, p[c * 8 + threadIdx.x]);
    red[threadIdx.x] = acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float l8[8];
    for (int j = 0; j < 8; ++j) l8[j] = red[j];
    float sum = hsum8(l8);
    for (int i = full; i < n; ++i) sum = __fadd_rn(sum, p[i]);
    inv_s = __fdiv_rn(1.0f, sum);
  }
  __syncthreads();
  const float inv = inv_s;
  for (int i = threadIdx.x; i < n; i += blockDim.x) p[i] = __fmul_rn(p[i], inv);
  // out[c] = sum_t p_t * V[t][c], added in t order; V staged tile by tile
  const float* vbase = b.vc + (size_t)layer * d.max_seq * d.dim + (size_t)h * hd + c0;
  float acc = 0.0f;
  for (int t0 = 0; t0 < n; t0 += kPvTile) {
    const int rows = min(kPvTile, n - t0);
    __syncthreads();
    for (int i = threadIdx.x; i < rows * (kPvCols / 4); i += blockDim.x) {
      const int r = i / (kPvCols / 4), q = i % (kPvCols / 4);
      reinterpret_cast<float4*>(vt)[i] =
          *reinterpret_cast<const float4*>(vbase + (size_t)(t0 + r) * d.dim + q * 4);
    }
    __syncthreads();
    if (threadIdx.x < kPvCols) {
      const float* pv = p + t0;
#pragma unroll 8
      for (int t = 0; t < rows; ++t) acc = __fadd_rn(acc, __fmul_rn(pv[t], vt[t * kPvCols + threadIdx.x]));
    }
  }
  if (threadIdx.x < kPvCols) b.att_out[h * hd + c0 + threadIdx.x] = acc;
}

}  // namespace

void launch_attention(const Dims& d, int layer, const DecodeBufs& b, cudaStream_t s) {
  dim3 g1((d.max_seq + kScoreThreads - 1) / kScoreThreads, d.n_heads);
  k_attn_scores<<<g1, kScoreThreads, 0, s>>>(d, layer, b);
  dim3 g2(d.n_heads, d.head_dim / kPvCols);
  const size_t smem = ((((size_t)d.max_seq + 3) & ~size_t(3)) + (size_t)kPvTile * kPvCols) * 4;
  if (smem > 48 * 1024) cudaFuncSetAttribute(k_attn_pv, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  k_attn_pv<<<g2, kPvThreads, smem, s>>>(d, layer, b);
}

}  // namespace chalot
