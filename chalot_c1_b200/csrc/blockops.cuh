// blockops.cuh — CTA-level building blocks reproducing the reference's
// vector routines with their exact rounding order.
#pragma once

#include "common.cuh"

namespace chalot {

// Copies n floats (n % 4 == 0, 16-byte aligned) from global to shared memory
// with every load of a thread issued before any store.
__device__ __forceinline__ void load_f32(float* dst, const float* __restrict__ src, int n) {
  const float4* s4 = reinterpret_cast<const float4*>(src);
  float4* d4 = reinterpret_cast<float4*>(dst);
  const int n4 = n >> 2;
#pragma unroll 4
  for (int i = threadIdx.x; i < n4; i += blockDim.x) d4[i] = s4[i];
}

// Same, reading through L2 only (__ldcg): for data other CTAs of the running
// grid wrote, which the L1 of this SM may hold stale.
__device__ __forceinline__ void load_f32_cg(float* dst, const float* src, int n) {
  const float4* s4 = reinterpret_cast<const float4*>(src);
  float4* d4 = reinterpret_cast<float4*>(dst);
  const int n4 = n >> 2;
#pragma unroll 4
  for (int i = threadIdx.x; i < n4; i += blockDim.x) d4[i] = __ldcg(s4 + i);
}

// rmsnorm_avx2 (src/tensor/normalization.rs:35-67) of x into xb (shared):
// lane j of 8 accumulates x[8c+j]^2 over c, the lanes are combined by hsum8,
// the tail is added in order, inv = 1/sqrt(ss/dim + 1e-5), xb = (x*inv)*w.
// dim % 32 == 0. `wbuf` is shared scratch of dim floats for the weights.
__device__ __forceinline__ void rmsnorm_smem(const float* x, const float* __restrict__ w, int dim,
                                             float* xb, float* wbuf, float* red,
                                             bool x_coherent = false) {
  if (x_coherent)
    load_f32_cg(xb, x, dim);
  else
    load_f32(xb, x, dim);
  load_f32(wbuf, w, dim);
  __syncthreads();
  const int chunks = dim >> 3;
  if (threadIdx.x < 8) {
    float s = 0.0f;
#pragma unroll 8
    for (int c = 0; c < chunks; ++c) {
      float v = xb[c * 8 + threadIdx.x];
      s = __fadd_rn(s, __fmul_rn(v, v));
    }
    red[threadIdx.x] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float lanes[8];
    for (int j = 0; j < 8; ++j) lanes[j] = red[j];
    float ss = hsum8(lanes);
    for (int i = chunks * 8; i < dim; ++i) ss = __fadd_rn(ss, __fmul_rn(xb[i], xb[i]));
    red[8] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)dim), 1e-5f)));
  }
  __syncthreads();
  const float inv = red[8];
  for (int i = threadIdx.x; i < dim; i += blockDim.x)
    xb[i] = __fmul_rn(__fmul_rn(xb[i], inv), wbuf[i]);
  __syncthreads();
}

// Absolute maximum of v[0..n) over the CTA.
__device__ __forceinline__ float absmax_smem(const float* v, int n, float* red) {
  float m = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, fabsf(v[i]));
  return block_max(m, red);
}

// rmsnorm then quantize_f32_to_i8 of a vector other CTAs just finished
// writing, into q_out/s_out (global). `xb`, `wbuf`: shared scratch of dim
// floats each.
__device__ __forceinline__ void norm_quant_tail(const float* x, const float* __restrict__ w, int dim,
                                                int8_t* q_out, float* s_out, float* xb, float* wbuf,
                                                float* red) {
  rmsnorm_smem(x, w, dim, xb, wbuf, red, true);
  float scale, inv;
  quant_scale(absmax_smem(xb, dim, red), &scale, &inv);
  for (int i = threadIdx.x; i < dim; i += blockDim.x) q_out[i] = quant_any(xb[i], inv, i, dim);
  if (threadIdx.x == 0) *s_out = scale;
}

// quantize_f32_to_i8 of v[0..n) into q (shared or global); returns the scale.
__device__ __forceinline__ float quantize_smem(const float* v, int n, int8_t* q, float* red) {
  float scale, inv;
  quant_scale(absmax_smem(v, n, red), &scale, &inv);
  for (int i = threadIdx.x; i < n; i += blockDim.x) q[i] = quant_any(v[i], inv, i, n);
  __syncthreads();
  return scale;
}

// Position of column i in the int4-friendly permuted layout: within each
// 8-column block, even columns first then odd ones, blocks of a 32-column
// chunk grouped as [4 words of evens][4 words of odds] (see dot32_u4).
__device__ __forceinline__ int perm32(int i) {
  const int chunk = i >> 5, k = i & 31, j = k >> 3, t = k & 7;
  return chunk * 32 + ((t & 1) ? 16 : 0) + j * 4 + (t >> 1);
}

// softmax_avx2 over s[0..n) in place, serial (n is small):
// fast_exp on the whole 8-chunks, libm exp on the tail, 8-lane sums + hsum8
// (src/tensor/normalization.rs:106-160).
__device__ __forceinline__ void softmax_serial(float* s, int n) {
  if (n <= 0) return;
  float mx = -INFINITY;
  for (int i = 0; i < n; ++i) mx = fmaxf(mx, s[i]);
  const int full = n & ~7;
  float lanes[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int i = 0; i < full; ++i) {
    const float e = fast_exp(__fsub_rn(s[i], mx));
    s[i] = e;
    lanes[i & 7] = __fadd_rn(lanes[i & 7], e);
  }
  float sum = hsum8(lanes);
  for (int i = full; i < n; ++i) {
    const float e = expf_cr(__fsub_rn(s[i], mx));
    s[i] = e;
    sum = __fadd_rn(sum, e);
  }
  const float inv = __fdiv_rn(1.0f, sum);
  for (int i = 0; i < n; ++i) s[i] = __fmul_rn(s[i], inv);
}

// softmax_top_k (src/tensor/normalization.rs:203-216) by one thread: the k
// largest probabilities in descending order, lower index first among equal
// values (what the insertion sort behind sort_unstable_by does for <= 20
// elements), renormalised by their sum when it exceeds 1e-12.
__device__ __forceinline__ void topk_serial(float* s, int n, int k, int32_t* idx, float* w) {
  softmax_serial(s, n);
  uint64_t taken = 0;  // n <= 64
  float sum = -0.0f;
  for (int j = 0; j < k; ++j) {
    int best = -1;
    for (int i = 0; i < n; ++i) {
      if (taken & (1ull << i)) continue;
      if (best < 0 || s[i] > s[best]) best = i;
    }
    taken |= 1ull << best;
    idx[j] = best;
    w[j] = s[best];
    sum = __fadd_rn(sum, s[best]);
  }
  if (sum > 1e-12f)
    for (int j = 0; j < k; ++j) w[j] = __fdiv_rn(w[j], sum);
}

// Router logits of one token: logit[e] = b[e] + dot_f32(W[e], xb) with the
// two-accumulator 8-lane order of dot_f32_avx2
// (src/tensor/attention_helpers.rs:41-80). `lanes` is shared scratch of
// 16*E floats; the result lands in logit[0..E) (shared).
__device__ __forceinline__ void router_logits(const float* __restrict__ W,
                                              const float* __restrict__ bias, const float* xb,
                                              int dim, int E, float* lanes, float* logit) {
  const int c16 = dim >> 4;
  const int rem = c16 * 16;
  const bool extra = rem + 8 <= dim;
  for (int t = threadIdx.x; t < 16 * E; t += blockDim.x) {
    const int e = t >> 4, l = t & 15, half = l >> 3, j = l & 7;
    const float* w = W + (size_t)e * dim;
    float s = 0.0f;
#pragma unroll 8
    for (int c = 0; c < c16; ++c) {
      const int k = c * 16 + half * 8 + j;
      s = __fadd_rn(s, __fmul_rn(w[k], xb[k]));
    }
    if (half == 0 && extra) s = __fadd_rn(s, __fmul_rn(w[rem + j], xb[rem + j]));
    lanes[t] = s;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    float c[8];
    for (int j = 0; j < 8; ++j) c[j] = __fadd_rn(lanes[e * 16 + j], lanes[e * 16 + 8 + j]);
    float r = hsum8(c);
    const float* w = W + (size_t)e * dim;
    for (int i = extra ? rem + 8 : rem; i < dim; ++i) r = __fadd_rn(r, __fmul_rn(w[i], xb[i]));
    logit[e] = __fadd_rn(bias[e], r);
  }
  __syncthreads();
}

}  // namespace chalot
