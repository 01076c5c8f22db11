// blockops.cuh — CTA-level building blocks reproducing the reference's
// vector routines with their exact rounding order.
#pragma once

#include "common.cuh"

namespace chalot {

// Copies n 16-byte elements from global memory to shared memory: each
// thread issues up to 8 loads before its stores, so a copy costs about one
// memory latency per 8*blockDim elements (through L2 only when `coherent`:
// for data other CTAs of the running grid wrote).
template <typename V>
__device__ __forceinline__ void copy16(V* __restrict__ dst, const V* __restrict__ src, int n,
                                       bool coherent) {
  constexpr int U = 8;
  for (int base = 0; base < n; base += U * (int)blockDim.x) {
    V v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * (int)blockDim.x + (int)threadIdx.x;
      if (i < n) v[u] = coherent ? __ldcg(src + i) : __ldg(src + i);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * (int)blockDim.x + (int)threadIdx.x;
      if (i < n) dst[i] = v[u];
    }
  }
}

// n floats (n % 4 == 0, 16-byte aligned) from global to shared memory.
__device__ __forceinline__ void load_f32(float* dst, const float* __restrict__ src, int n) {
  copy16(reinterpret_cast<float4*>(dst), reinterpret_cast<const float4*>(src), n >> 2, false);
}
__device__ __forceinline__ void load_f32_cg(float* dst, const float* src, int n) {
  copy16(reinterpret_cast<float4*>(dst), reinterpret_cast<const float4*>(src), n >> 2, true);
}

// Quantizes n floats (n % 4 == 0) that other CTAs just wrote with a known
// scale reciprocal into natural-order int8 words in global memory; loads are
// batched 8 float4 per thread before the stores.
__device__ __forceinline__ void quant_store_words(uint32_t* __restrict__ dst, const float4* src, int n4,
                                                  float inv, int n) {
  constexpr int U = 8;
  for (int base = 0; base < n4; base += U * (int)blockDim.x) {
    float4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * (int)blockDim.x + (int)threadIdx.x;
      if (i < n4) v[u] = __ldcg(src + i);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i4 = base + u * (int)blockDim.x + (int)threadIdx.x;
      if (i4 < n4) {
        const int i = i4 * 4;
        const uint32_t q0 = (uint8_t)quant_any(v[u].x, inv, i, n), q1 = (uint8_t)quant_any(v[u].y, inv, i + 1, n);
        const uint32_t q2 = (uint8_t)quant_any(v[u].z, inv, i + 2, n), q3 = (uint8_t)quant_any(v[u].w, inv, i + 3, n);
        dst[i4] = q0 | (q1 << 8) | (q2 << 16) | (q3 << 24);
      }
    }
  }
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
    int c = 0;
    for (; c + 8 <= chunks; c += 8) {  // 8 independent loads, then 8 dependent adds
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = xb[(c + u) * 8 + threadIdx.x];
#pragma unroll
      for (int u = 0; u < 8; ++u) s = __fadd_rn(s, __fmul_rn(v[u], v[u]));
    }
    for (; c < chunks; ++c) {
      const float v = xb[c * 8 + threadIdx.x];
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
    red[8] = div_rn(1.0f, __fsqrt_rn(__fadd_rn(div_rn(ss, (float)dim), 1e-5f)));
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

// rmsnorm then quantize_f32_to_i8 of a vector x other CTAs just finished
// writing, into q_out/s_out (global). `wsm` holds the norm weights already in
// shared memory (staged before the dependency wait); `xb`: shared scratch of
// dim floats that ends up holding rmsnorm(x).
__device__ __forceinline__ void norm_quant_tail(const float* x, const float* wsm, int dim,
                                                int8_t* q_out, float* s_out, float* xb, float* red) {
  load_f32_cg(xb, x, dim);
  __syncthreads();
  const int chunks = dim >> 3;
  if (threadIdx.x < 8) {  // lane j accumulates x[8c+j]^2 over c in order
    float s = 0.0f;
    int c = 0;
    for (; c + 16 <= chunks; c += 16) {  // 16 loads issued together, then the chain
      float v[16];
#pragma unroll
      for (int u = 0; u < 16; ++u) v[u] = xb[(c + u) * 8 + threadIdx.x];
#pragma unroll
      for (int u = 0; u < 16; ++u) s = __fadd_rn(s, __fmul_rn(v[u], v[u]));
    }
    for (; c < chunks; ++c) {
      const float v = xb[c * 8 + threadIdx.x];
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
    red[8] = div_rn(1.0f, __fsqrt_rn(__fadd_rn(div_rn(ss, (float)dim), 1e-5f)));
  }
  __syncthreads();
  const float inv = red[8];
  float m = 0.0f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const float v = __fmul_rn(__fmul_rn(xb[i], inv), wsm[i]);
    xb[i] = v;
    m = fmaxf(m, fabsf(v));
  }
  float scale, qinv;
  quant_scale(block_max(m, red), &scale, &qinv);
  for (int i = threadIdx.x; i < dim; i += blockDim.x) q_out[i] = quant_any(xb[i], qinv, i, dim);
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

// softmax_top_k (src/tensor/normalization.rs:203-216) of s[0..n) (n <= 32)
// by one warp, in the reference's arithmetic order: softmax_avx2 with
// fast_exp on whole 8-chunks and libm exp on the tail, 8-lane sums combined
// by hsum8 (normalization.rs:106-160); then the k largest probabilities in
// descending order, lower index first among equal values (the insertion sort
// behind sort_unstable_by for <= 20 elements), renormalised by their sum when
// it exceeds 1e-12. Called by all 32 lanes of one warp.
__device__ __forceinline__ void topk_warp(const float* s, int n, int k, int32_t* idx, float* w) {
  const int lane = threadIdx.x & 31;
  const float v = lane < n ? s[lane] : -INFINITY;
  const float mx = warp_max(v);
  const int full = n & ~7;
  float e = 0.0f;
  if (lane < full)
    e = fast_exp(__fsub_rn(v, mx));
  else if (lane < n)
    e = expf_cr(__fsub_rn(v, mx));
  // lane j < 8 accumulates e[8c + j] over c in order
  float acc = 0.0f;
  for (int c = 0; c < (full >> 3); ++c) {
    const float t = __shfl_sync(0xffffffffu, e, c * 8 + (lane & 7));
    acc = __fadd_rn(acc, t);
  }
  float l8[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) l8[j] = __shfl_sync(0xffffffffu, acc, j);
  float sum = hsum8(l8);
  for (int i = full; i < n; ++i) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, e, i));
  const float p = __fmul_rn(e, div_rn(1.0f, sum));
  // the k rounds of (max probability, lowest index) as ranks: rank r is the
  // pick of round r
  int rank = 0;
  for (int o = 0; o < n; ++o) {
    const float q = __shfl_sync(0xffffffffu, p, o);
    rank += (q > p || (q == p && o < lane)) ? 1 : 0;
  }
  const bool live = lane < n;
  float tot = -0.0f;  // the picks' sum in round order
  for (int r = 0; r < k; ++r) {
    const unsigned m = __ballot_sync(0xffffffffu, live && rank == r);
    const float pr = __shfl_sync(0xffffffffu, p, m ? __ffs(m) - 1 : 0);
    tot = __fadd_rn(tot, pr);
  }
  if (live && rank < k) {
    idx[rank] = lane;
    w[rank] = (tot > 1e-12f) ? div_rn(p, tot) : p;
  }
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
    int c = 0;
    for (; c + 32 <= c16; c += 32) {  // 32 weight loads in flight, then the ordered sum
      float wv[32];
#pragma unroll
      for (int u = 0; u < 32; ++u) wv[u] = w[(c + u) * 16 + half * 8 + j];  // W may be in shared memory
#pragma unroll
      for (int u = 0; u < 32; ++u) s = __fadd_rn(s, __fmul_rn(wv[u], xb[(c + u) * 16 + half * 8 + j]));
    }
#pragma unroll 8
    for (; c < c16; ++c) {
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
