// k_persist.cu — the whole batch-1 decode step (Engine::forward,
// src/model/engine.rs:173-494) as ONE persistent kernel: one CTA per SM,
// co-resident by cooperative launch, the phases of a layer separated by
// bounded grid-wide and head-group barriers instead of kernel boundaries and
// last-CTA tickets.
//
// Per layer (every float operation in the reference's order, as the
// multi-kernel path in k_dense.cu / k_attn.cu / k_moe.cu):
//   A  every CTA: rmsnorm(x, rms_attn) and quantize_f32_to_i8 in shared
//      memory; the CTAs of head group h compute head h's Q, K and V row pairs
//      (weights requested before the barrier), RoPE, the K/V cache rows.
//      -> head-group barrier
//   B1 group h: scores of head h for a slice of positions (dot_f32 order,
//      soft-cap with the restated tanhf). -> head-group barrier
//   B2 group h: every CTA runs softmax_avx2 over all scores of the head, then
//      the t-ordered sums of its slice of the head's output columns.
//      -> grid barrier
//   C  every CTA quantizes att_out; CTA c computes its O rows and updates the
//      x rows it owns (rows [c*dim/N, (c+1)*dim/N), also its down rows).
//      -> grid barrier
//   D  every CTA: rmsnorm(x, rms_ffn), quantize, router logits and
//      softmax_top_k (the same bits in every CTA), then bulk-copies its share
//      of the selected experts' gate/up rows and its down rows into shared
//      memory.
//   E  gate/up group products, ordered group sums, SwiGLU -> h; absmax(h).
//      -> grid barrier
//   F  every CTA quantizes h of each selected expert; CTA c's down rows,
//      ordered sums, gated combine in selection order, x rows += .
//      -> grid barrier (the next layer's A)
// After the last layer every CTA computes the final norm and quantization and
// streams its slice of the lm_head rows; the argmax (ties to the last index)
// is a 64-bit atomicMax.
//
// Every wait is bounded (globaltimer, 200 ms): a CTA that gives up sets the
// engine's error word (the host reports CHALOT_ERR_TIMEOUT) and every other
// waiter leaves as soon as it sees that word. The barrier counters start at
// zero (k_persist_reset runs after each step).
#include <cuda_runtime.h>

#include <algorithm>

#include "blockops.cuh"
#include "kernels.cuh"
#include "persist.h"
#include "tma.cuh"

namespace chalot {
namespace {

constexpr int kT = kPersistThreads;
constexpr int kW = kT / 32;
constexpr unsigned long long kWaitNs = 200ull * 1000 * 1000;

CHALOT_DEV unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
CHALOT_DEV unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
CHALOT_DEV void red_release(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Barrier over the CTAs sharing `ctr` (n of them, `k`-th use in this launch):
// the CTA's writes before it are visible to every member after it. Returns
// false (error word set) when the wait ran out or another CTA gave up.
__device__ __noinline__ bool cta_barrier(unsigned* ctr, unsigned target, unsigned* err, int* fail_s) {
  __syncthreads();
  if (threadIdx.x == 0) {
    red_release(ctr, 1u);
    if (ld_acquire(ctr) < target) {
      const unsigned long long t0 = gtimer();
      for (int k = 1;; ++k) {
        if (ld_acquire(ctr) >= target) break;
        if ((k & 31) == 0) {
          if (*(volatile unsigned*)err) {
            *fail_s = 1;
            break;
          }
          if (gtimer() - t0 > kWaitNs) {
            atomicOr(err, 1u);
            *fail_s = 1;
            break;
          }
        }
      }
    }
  }
  __syncthreads();
  return *(volatile int*)fail_s == 0;
}

// mbarrier wait bounded by time; false when it ran out (error word set).
CHALOT_DEV bool mbar_wait_t(uint64_t* bar, uint32_t parity, unsigned* err) {
  const uint32_t a = smem_u32(bar);
  unsigned long long t0 = 0;
  for (int k = 0;; ++k) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(a), "r"(parity)
        : "memory");
    if (ok) return true;
    if (k == 0) t0 = gtimer();
    if ((k & 15) == 15 && gtimer() - t0 > kWaitNs) {
      atomicOr(err, 1u);
      return false;
    }
  }
}

// Loads IT 16-byte chunks (lane, lane+32, ...) of an int8 row of `n` bytes.
template <int IT>
CHALOT_DEV void row_load(const int8_t* row, int n, uint4 (&w)[IT]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int it = 0; it < IT; ++it) {
    const int c = lane + 32 * it;
    w[it] = (row && c < (n >> 4)) ? ldg_stream(row + (size_t)c * 16) : make_uint4(0, 0, 0, 0);
  }
}
template <int IT>
CHALOT_DEV int row_dot(const uint4 (&w)[IT], const int8_t* xq, int n) {
  const int lane = threadIdx.x & 31;
  int acc = 0;
#pragma unroll
  for (int it = 0; it < IT; ++it) {
    const int c = lane + 32 * it;
    if (c < (n >> 4)) acc = dot16_i8(w[it], lds16(xq + c * 16), acc);
  }
  return warp_sum_i(acc);
}

// rmsnorm_avx2 (normalization.rs:35-67) of xs (shared, dim floats) with
// weights w (global) into xb (shared), then quantize_f32_to_i8
// (quantization.rs:56-104) into xq (shared); returns the scale.
CHALOT_DEV float norm_quant_smem(const float* xs, const float* __restrict__ w, int dim, float* xb,
                                 int8_t* xq, float* red) {
  float wr[4];  // this thread's weights (dim <= 4 * kT), requested before the sum of squares
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int i = threadIdx.x + u * kT;
    wr[u] = i < dim ? __ldg(w + i) : 0.0f;
  }
  const int chunks = dim >> 3;
  if (threadIdx.x < 8) {
    float s = 0.0f;
    int c = 0;
    for (; c + 16 <= chunks; c += 16) {
      float v[16];
#pragma unroll
      for (int u = 0; u < 16; ++u) v[u] = xs[(c + u) * 8 + threadIdx.x];
#pragma unroll
      for (int u = 0; u < 16; ++u) s = __fadd_rn(s, __fmul_rn(v[u], v[u]));
    }
    for (; c < chunks; ++c) {
      const float v = xs[c * 8 + threadIdx.x];
      s = __fadd_rn(s, __fmul_rn(v, v));
    }
    red[threadIdx.x] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float l8[8];
    for (int j = 0; j < 8; ++j) l8[j] = red[j];
    float ss = hsum8(l8);
    for (int i = chunks * 8; i < dim; ++i) ss = __fadd_rn(ss, __fmul_rn(xs[i], xs[i]));
    red[8] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)dim), 1e-5f)));
  }
  __syncthreads();
  const float inv = red[8];
  float m = 0.0f;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int i = threadIdx.x + u * kT;
    if (i < dim) {
      const float v = __fmul_rn(__fmul_rn(xs[i], inv), wr[u]);
      xb[i] = v;
      m = fmaxf(m, fabsf(v));
    }
  }
  float scale, qinv;
  quant_scale(block_max(m, red), &scale, &qinv);
  for (int i = threadIdx.x; i < dim; i += kT) xq[i] = quant_any(xb[i], qinv, i, dim);
  __syncthreads();
  return scale;
}

CHALOT_DEV const ExpertPtrs& layer_expert(const LayerPtrs& L, int E, int e) {
  return E <= 16 ? L.ex[e] : L.experts[e];
}

template <int IT, int HD>
__global__ void __launch_bounds__(kT, 1) k_persist(PersistArgs a) {
  extern __shared__ __align__(128) unsigned char sm[];
  const Dims& d = a.d;
  const DecodeBufs& b = a.b;
  const PersistPlan& pl = a.plan;
  const int c = blockIdx.x, NC = gridDim.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int dim = d.dim, H = d.hidden, K = d.top_k, E = d.n_experts;
  const int ngd = dim >> 5, ngh = H >> 5;
  int8_t* xq = reinterpret_cast<int8_t*>(sm + pl.o_xq);     // [dim] quantized vector of the phase
  float* xf = reinterpret_cast<float*>(sm + pl.o_xf);       // [dim] x (or att_out)
  float* xb = reinterpret_cast<float*>(sm + pl.o_xb);       // [dim] normalised vector
  float* own = reinterpret_cast<float*>(sm + pl.o_own);     // [rows_max] this CTA's x rows
  float* red = reinterpret_cast<float*>(sm + pl.o_red);     // [64] + routing
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + pl.o_bars);  // [3] gate/up, down, router copies
  float* P = reinterpret_cast<float*>(sm + pl.o_P);         // group products
  float* Tt = reinterpret_cast<float*>(sm + pl.o_T);        // row totals
  int8_t* xh = reinterpret_cast<int8_t*>(sm + pl.o_xh);     // [K][H] quantized h
  unsigned char* stg = sm + pl.o_stage;                     // expert rows / V columns / scores
  __shared__ int fail_s;
  __shared__ int sel_s[8];
  __shared__ float selw_s[8];
  __shared__ float xs_s;
  if (tid == 0) {
    fail_s = 0;
    mbar_init(&bars[0]);
    mbar_init(&bars[1]);
    mbar_init(&bars[2]);
  }
  unsigned n_grid = 0;   // grid barriers passed in this launch
  unsigned n_group = 0;  // head-group barriers passed
  const uint32_t pos = b.st->pos, tok = b.st->token;
  const int n = (int)pos + 1;
  // head group of this CTA and its place in it
  const int h = (int)(((long)c * d.n_heads) / NC);
  const int g0 = (int)(((long)h * NC + d.n_heads - 1) / d.n_heads);
  const int g1 = (int)(((long)(h + 1) * NC + d.n_heads - 1) / d.n_heads);
  const int gs = g1 - g0, gj = c - g0;
  // rows of x (O rows, down rows) owned by this CTA
  const int r0 = (int)(((long)c * dim) / NC), r1 = (int)(((long)(c + 1) * dim) / NC), nr = r1 - r0;
  unsigned* gbar = a.bar;                  // grid barrier counter
  unsigned* hbar = a.bar + 32 * (1 + h);   // head-group counter (own 128-byte line)
  unsigned long long* tr = (a.trace && c == 0 && tid == 0) ? a.trace : nullptr;
  auto mark = [&](int slot) {
    if (tr) tr[slot] = gtimer();
  };
  mark(16 * d.n_layers + 0);
  // ---- embedding (engine.rs:201-210): every CTA builds x itself ----
  {
    const float s = __ldg(a.emb_s + tok);
    const int8_t* row = a.emb + (size_t)tok * dim;
    for (int i = tid; i < dim; i += kT) xf[i] = __fmul_rn((float)row[i], s);
    if (c == 0 && tid == 0) b.st->argmax_key = 0ull;
    __syncthreads();
    for (int i = tid; i < nr; i += kT) {
      own[i] = xf[r0 + i];
      __stcg(b.x + r0 + i, own[i]);
    }
  }
  const int np_h = 3 * HD / 2;  // Q, K, V row pairs of one head
  const int pq0 = (gj * np_h) / gs, pq1 = ((gj + 1) * np_h) / gs;
  const int half = HD >> 1;
  for (int l = 0; l < d.n_layers; ++l) {
    const LayerPtrs& L = a.layers[l];
    mark(l * 16 + 0);
    // ---- A: QKV of head h ----
    // this warp's first row pair, requested before the barrier
    uint4 w0[IT], w1[IT];
    {
      const int p = pq0 + warp;
      const int sec = p / half, i = p % half;
      const int8_t* row = p < pq1 ? L.qkv + ((size_t)sec * dim + h * HD + 2 * i) * dim : nullptr;
      row_load<IT>(row, dim, w0);
      row_load<IT>(row ? row + dim : nullptr, dim, w1);
    }
    if (l > 0) {
      if (!cta_barrier(gbar, (++n_grid) * NC, a.err, &fail_s)) return;
      for (int i = tid; i < dim; i += kT) xf[i] = __ldcg(b.x + i);
      __syncthreads();
    }
    mark(l * 16 + 1);
    {
      const float s = norm_quant_smem(xf, L.rms_attn, dim, xb, xq, red);
      for (int p = pq0 + warp; p < pq1; p += kW) {
        const int sec = p / half, i = p % half;
        const size_t row = (size_t)sec * dim + h * HD + 2 * i;
        if (p != pq0 + warp) {
          row_load<IT>(L.qkv + row * dim, dim, w0);
          row_load<IT>(L.qkv + (row + 1) * dim, dim, w1);
        }
        const int dot0 = row_dot<IT>(w0, xq, dim), dot1 = row_dot<IT>(w1, xq, dim);
        if (lane == 0) {
          float v0 = __fmul_rn(__fmul_rn((float)dot0, __ldg(L.qkv_s + row)), s);
          float v1 = __fmul_rn(__fmul_rn((float)dot1, __ldg(L.qkv_s + row + 1)), s);
          if (sec < 2) {  // RoPE on the interleaved pair (engine.rs:252-271)
            const float cs = __ldg(b.rope_cos + (size_t)pos * half + i), sn = __ldg(b.rope_sin + (size_t)pos * half + i);
            const float x0 = __fsub_rn(__fmul_rn(v0, cs), __fmul_rn(v1, sn));
            const float x1 = __fadd_rn(__fmul_rn(v0, sn), __fmul_rn(v1, cs));
            v0 = x0;
            v1 = x1;
          }
          const int col = h * HD + 2 * i;
          if (sec == 0) {
            __stcg(b.q + col, v0);
            __stcg(b.q + col + 1, v1);
          } else {  // engine.rs:274-280
            float* cache = sec == 1 ? b.kc : b.vc;
            const size_t off = ((size_t)l * d.max_seq + pos) * dim + col;
            __stcg(cache + off, v0);
            __stcg(cache + off + 1, v1);
          }
        }
      }
    }
    mark(l * 16 + 2);
    if (!cta_barrier(hbar, (++n_group) * gs, a.err, &fail_s)) return;
    mark(l * 16 + 3);
    // ---- B1: scores of head h for positions [t0, t1) ----
    {
      float* qh = xb;  // [HD]
      for (int i = tid; i < HD; i += kT) qh[i] = __ldcg(b.q + h * HD + i);
      __syncthreads();
      const int t0 = (gj * n) / gs, t1 = ((gj + 1) * n) / gs;
      const float inv_sqrt = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
      for (int t = t0 + tid; t < t1; t += kT) {
        const float4* kr = reinterpret_cast<const float4*>(b.kc + ((size_t)l * d.max_seq + t) * dim + h * HD);
        float a0[8], a1[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) a0[j] = a1[j] = 0.0f;
        const bool cur = t == (int)pos;
#pragma unroll
        for (int cb = 0; cb < HD / 32; ++cb) {  // 32 values (two 16-strides) per load batch
          float4 kv[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) kv[u] = cur ? __ldcg(kr + cb * 8 + u) : __ldg(kr + cb * 8 + u);
          const float* kk = reinterpret_cast<const float*>(kv);
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2)
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const int col = cb * 32 + h2 * 16;
              a0[j] = __fadd_rn(a0[j], __fmul_rn(qh[col + j], kk[h2 * 16 + j]));
              a1[j] = __fadd_rn(a1[j], __fmul_rn(qh[col + 8 + j], kk[h2 * 16 + 8 + j]));
            }
        }
        float cmb[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) cmb[j] = __fadd_rn(a0[j], a1[j]);
        const float x = __fmul_rn(hsum8(cmb), inv_sqrt);
        __stcg(b.scores + (size_t)h * d.max_seq + t, __fmul_rn(30.0f, libm::tanh_f32(__fdiv_rn(x, 30.0f))));
      }
    }
    mark(l * 16 + 4);
    if (!cta_barrier(hbar, (++n_group) * gs, a.err, &fail_s)) return;
    mark(l * 16 + 5);
    // ---- B2: softmax over the head's n scores, t-ordered sums of columns [k0, k1) ----
    {
      float* p = reinterpret_cast<float*>(stg);   // [max_seq]
      float* vt = p + ((d.max_seq + 3) & ~3);     // [ncol][kPvTile + 4]
      const float* s = b.scores + (size_t)h * d.max_seq;
      float mx = -INFINITY;
      for (int i = tid; i < n; i += kT) {
        const float v = __ldcg(s + i);
        p[i] = v;
        mx = fmaxf(mx, v);
      }
      mx = block_max(mx, red);
      const int full = n & ~7;
      for (int i = tid; i < n; i += kT)
        p[i] = (i < full) ? fast_exp(__fsub_rn(p[i], mx)) : expf_cr(__fsub_rn(p[i], mx));
      __syncthreads();
      if (tid < 8) {
        float acc = 0.0f;
        const int nc8 = full >> 3;
        int cc = 0;
        for (; cc + 8 <= nc8; cc += 8) {
          float v[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) v[u] = p[(cc + u) * 8 + tid];
#pragma unroll
          for (int u = 0; u < 8; ++u) acc = __fadd_rn(acc, v[u]);
        }
        for (; cc < nc8; ++cc) acc = __fadd_rn(acc, p[cc * 8 + tid]);
        red[tid] = acc;
      }
      __syncthreads();
      if (tid == 0) {
        float l8[8];
        for (int j = 0; j < 8; ++j) l8[j] = red[j];
        float sum = hsum8(l8);
        for (int i = full; i < n; ++i) sum = __fadd_rn(sum, p[i]);
        red[9] = __fdiv_rn(1.0f, sum);
      }
      __syncthreads();
      const float inv = red[9];
      for (int i = tid; i < n; i += kT) p[i] = __fmul_rn(p[i], inv);
      const int k0 = (gj * HD) / gs, k1 = ((gj + 1) * HD) / gs, ncol = k1 - k0;
      const float* vbase = b.vc + (size_t)l * d.max_seq * dim + h * HD + k0;
      float acc = 0.0f;
      for (int tt = 0; tt < n; tt += kPvTile) {
        const int rows = min(kPvTile, n - tt);
        __syncthreads();
        // products p_t * V[t][col] of this tile, column-major (each chain reads its column)
        for (int i = tid; i < rows * ncol; i += kT) {
          const int r = i / ncol, cc = i - r * ncol, t = tt + r;
          const float* src = vbase + (size_t)t * dim + cc;
          const float v = (t == (int)pos) ? __ldcg(src) : __ldg(src);
          vt[cc * (kPvTile + 4) + r] = __fmul_rn(p[t], v);
        }
        __syncthreads();
        if (tid < ncol) {  // out[c] = sum_t p_t v_t[c], added in t order (engine.rs:302-308)
          const float* pc = vt + tid * (kPvTile + 4);
          int r = 0;
          for (; r + 16 <= rows; r += 16) {
            float4 q4[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) q4[u] = lds16f(pc + r + 4 * u);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              acc = __fadd_rn(acc, q4[u].x);
              acc = __fadd_rn(acc, q4[u].y);
              acc = __fadd_rn(acc, q4[u].z);
              acc = __fadd_rn(acc, q4[u].w);
            }
          }
          for (; r < rows; ++r) acc = __fadd_rn(acc, pc[r]);
        }
      }
      if (tid < ncol) __stcg(b.att_out + h * HD + k0 + tid, acc);
    }
    mark(l * 16 + 6);
    // ---- C: O rows r0..r1 + residual (engine.rs:312-322) ----
    uint4 ow[IT];
    row_load<IT>(warp < nr ? L.o + (size_t)(r0 + warp) * dim : nullptr, dim, ow);
    if (!cta_barrier(gbar, (++n_grid) * NC, a.err, &fail_s)) return;
    mark(l * 16 + 7);
    float* rw_s = reinterpret_cast<float*>(stg);  // [E][dim] router weights for D
    if (tid == 0) {  // the attention's staging is free: fetch the router weights
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_expect_tx(&bars[2], (uint32_t)(E * dim * 4));
      tma_load(rw_s, L.router_w, (uint32_t)(E * dim * 4), &bars[2]);
    }
    {
      float m = 0.0f;
      for (int i = tid; i < dim; i += kT) {
        const float v = __ldcg(b.att_out + i);
        xf[i] = v;
        m = fmaxf(m, fabsf(v));
      }
      float scale, qinv;
      quant_scale(block_max(m, red), &scale, &qinv);
      for (int i = tid; i < dim; i += kT) xq[i] = quant_any(xf[i], qinv, i, dim);
      __syncthreads();
      for (int w = warp; w < nr; w += kW) {
        if (w != warp) row_load<IT>(L.o + (size_t)(r0 + w) * dim, dim, ow);
        const int dot = row_dot<IT>(ow, xq, dim);
        if (lane == 0) {
          const float v = __fmul_rn(__fmul_rn((float)dot, __ldg(L.o_s + r0 + w)), scale);
          own[w] = __fadd_rn(own[w], v);
          __stcg(b.x + r0 + w, own[w]);
        }
      }
    }
    mark(l * 16 + 8);
    if (!cta_barrier(gbar, (++n_grid) * NC, a.err, &fail_s)) {
      if (tid == 0) mbar_wait_t(&bars[2], l & 1, a.err);  // no copy may land after the CTA left
      return;
    }
    mark(l * 16 + 9);
    // ---- D: FFN norm, quantize, routing (engine.rs:325-344) ----
    for (int i = tid; i < dim; i += kT) xf[i] = __ldcg(b.x + i);
    __syncthreads();
    {
      const float s = norm_quant_smem(xf, L.rms_ffn, dim, xb, xq, red);
      float* lanes = rw_s + (size_t)E * dim;  // [16E]
      float* logit = lanes + 16 * E;
      if (tid == 0 && !mbar_wait_t(&bars[2], l & 1, a.err)) fail_s = 1;
      __syncthreads();
      if (fail_s) return;
      router_logits(rw_s, L.router_b, xb, dim, E, lanes, logit);
      if (warp == 0) topk_warp(logit, E, K, sel_s, selw_s);
      if (tid == 0) xs_s = s;
      if (c == 0 && b.router_trace)
        for (int e = tid; e < E; e += kT) b.router_trace[l * E + e] = logit[e];
      __syncthreads();
    }
    // bulk copies of this CTA's gate/up pairs [q0, q1) over the K*H (choice,
    // unit) pairs and of its down rows of every selected expert
    const int q0 = (int)(((long)c * K * H) / NC), q1 = (int)(((long)(c + 1) * K * H) / NC);
    const int npair = q1 - q0;
    const int prow = dim >> 1, hrow = H >> 1;
    unsigned char* gu_w = stg;                                   // [2*npair][prow]
    float* gu_s = reinterpret_cast<float*>(gu_w + (size_t)pl.max_pairs * 2 * prow);  // [2*npair][ngd]
    unsigned char* dn_w = reinterpret_cast<unsigned char*>(gu_s + (size_t)pl.max_pairs * 2 * ngd);  // [K*nr][hrow]
    float* dn_s = reinterpret_cast<float*>(dn_w + (size_t)K * pl.max_rows * hrow);             // [K*nr][ngh]
    // segment j of the pair range: choice j, units [u0, u1), local rows from lb
    if (tid == 0) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      uint32_t bytes_gu = (uint32_t)npair * 2 * (prow + ngd * 4);
      mbar_expect_tx(&bars[0], bytes_gu);
      const uint64_t pol = l2_evict_first();
      int lb = 0;
      for (int q = q0; q < q1;) {
        const int j = q / H, u0 = q % H, u1 = min(H, u0 + (q1 - q));
        const int m = u1 - u0;
        const ExpertPtrs& X = layer_expert(L, E, sel_s[j]);
        if (m <= 0) break;
        tma_load_hint(gu_w + (size_t)lb * prow, X.gu + (size_t)u0 * prow, (uint32_t)(m * prow), &bars[0], pol);
        tma_load_hint(gu_w + (size_t)(lb + m) * prow, X.gu + (size_t)(H + u0) * prow, (uint32_t)(m * prow), &bars[0], pol);
        tma_load_hint(gu_s + (size_t)lb * ngd, X.gu_s + (size_t)u0 * ngd, (uint32_t)(m * ngd * 4), &bars[0], pol);
        tma_load_hint(gu_s + (size_t)(lb + m) * ngd, X.gu_s + (size_t)(H + u0) * ngd, (uint32_t)(m * ngd * 4), &bars[0], pol);
        lb += 2 * m;
        q += m;
      }
      mbar_expect_tx(&bars[1], (uint32_t)(K * nr * (hrow + ngh * 4)));
      for (int j = 0; j < K && nr > 0; ++j) {
        const ExpertPtrs& X = layer_expert(L, E, sel_s[j]);
        tma_load_hint(dn_w + (size_t)j * nr * hrow, X.dn + (size_t)r0 * hrow, (uint32_t)(nr * hrow), &bars[1], pol);
        tma_load_hint(dn_s + (size_t)j * nr * ngh, X.dn_s + (size_t)r0 * ngh, (uint32_t)(nr * ngh * 4), &bars[1], pol);
      }
    }
    // reset the absmax slots the next layer uses (read two barriers ago at the latest)
    if (c == 0 && tid < K) a.amax[((l + 1) & 1) * 8 + tid] = 0u;
    mark(l * 16 + 10);
    // ---- E: gate/up (engine.rs:366-377) ----
    {
      const float xs = xs_s;
      if (tid == 0 && !mbar_wait_t(&bars[0], l & 1, a.err)) fail_s = 1;
      __syncthreads();
      if (fail_s) {
        if (tid == 0) mbar_wait_t(&bars[1], l & 1, a.err);
        return;
      }
      const int nrow = 2 * npair, PS = ngd + 1;
      for (int it = tid; it < nrow * ngd; it += kT) {
        const int row = it / ngd, g = it - row * ngd;
        const uint4 w = lds16(gu_w + (size_t)row * prow + g * 16);
        const int dv = dot32_rp(w, lds16(xq + g * 32), lds16(xq + g * 32 + 16));
        P[row * PS + g] = __fmul_rn(__fmul_rn((float)dv, gu_s[(size_t)row * ngd + g]), xs);
      }
      __syncthreads();
      for (int row = tid; row < nrow; row += kT) {  // t = t + p_g in group order (matmul.rs:576-577)
        const float* pr = P + row * PS;
        float t = 0.0f;
        for (int g = 0; g < ngd; ++g) t = __fadd_rn(t, pr[g]);
        Tt[row] = t;
      }
      __syncthreads();
      // pair k of segment (lb, m): gate row lb + k, up row lb + m + k
      float mloc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) mloc[j] = 0.0f;
      {
        int lb = 0;
        for (int q = q0; q < q1;) {
          const int j = q / H, u0 = q % H, m = min(H, u0 + (q1 - q)) - u0;
          for (int k = tid; k < m; k += kT) {
            const float hv = swiglu_elem(Tt[lb + k], Tt[lb + m + k], u0 + k, H);
            __stcg(b.h + (size_t)j * H + u0 + k, hv);
#pragma unroll
            for (int jj = 0; jj < 8; ++jj)
              if (jj == j) mloc[jj] = fmaxf(mloc[jj], fabsf(hv));
          }
          lb += 2 * m;
          q += m;
        }
      }
      for (int j = 0; j < K; ++j) {
        const float m = block_max(mloc[j], red);
        if (tid == 0 && m > 0.0f) atomicMax(a.amax + (l & 1) * 8 + j, __float_as_uint(m));
      }
    }
    mark(l * 16 + 11);
    if (!cta_barrier(gbar, (++n_grid) * NC, a.err, &fail_s)) {
      if (tid == 0) mbar_wait_t(&bars[1], l & 1, a.err);
      return;
    }
    mark(l * 16 + 12);
    // ---- F: quantize h, down rows, gated combine, residual (engine.rs:380-401) ----
    {
      float* xsh = red + 16;  // [K] scales of h
      float* invh = red + 24;
      if (tid < K) {
        float sc, inv;
        quant_scale(__uint_as_float(__ldcg(a.amax + (l & 1) * 8 + tid)), &sc, &inv);
        xsh[tid] = sc;
        invh[tid] = inv;
      }
      __syncthreads();
      const int n4 = (K * H) >> 2;
      const float4* hv = reinterpret_cast<const float4*>(b.h);
      uint32_t* xw = reinterpret_cast<uint32_t*>(xh);
      for (int i = tid; i < n4; i += kT) {
        const float4 v = __ldcg(hv + i);
        const float inv = invh[(i * 4) / H];
        const uint32_t b0 = (uint8_t)quant_elem(v.x, inv), b1 = (uint8_t)quant_elem(v.y, inv);
        const uint32_t b2 = (uint8_t)quant_elem(v.z, inv), b3 = (uint8_t)quant_elem(v.w, inv);
        xw[i] = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
      }
      if (tid == 0 && !mbar_wait_t(&bars[1], l & 1, a.err)) fail_s = 1;
      __syncthreads();
      if (fail_s) return;
      const int nrow = K * nr, PS = ngh + 1;
      for (int it = tid; it < nrow * ngh; it += kT) {
        const int row = it / ngh, g = it - row * ngh, j = row / nr;
        const uint4 w = lds16(dn_w + (size_t)row * hrow + g * 16);
        const int8_t* xj = xh + (size_t)j * H + g * 32;
        const int dv = dot32_rp(w, lds16(xj), lds16(xj + 16));
        P[row * PS + g] = __fmul_rn(__fmul_rn((float)dv, dn_s[(size_t)row * ngh + g]), xsh[j]);
      }
      __syncthreads();
      for (int row = tid; row < nrow; row += kT) {
        const float* pr = P + row * PS;
        float t = 0.0f;
        for (int g = 0; g < ngh; ++g) t = __fadd_rn(t, pr[g]);
        Tt[row] = t;
      }
      __syncthreads();
      if (tid < nr) {
        float add = 0.0f;  // expert_out = sum_k w_k * y_k in selection order (engine.rs:390-396)
        for (int j = 0; j < K; ++j) add = __fadd_rn(add, __fmul_rn(selw_s[j], Tt[j * nr + tid]));
        own[tid] = __fadd_rn(own[tid], add);
        __stcg(b.x + r0 + tid, own[tid]);
      }
    }
    mark(l * 16 + 13);
  }
  // ---- final norm, lm_head, argmax (engine.rs:470-493, sampling.rs:34-41) ----
  constexpr int kLmRows = 4;
  const int v0 = (int)(((long)c * d.vocab) / NC), v1 = (int)(((long)(c + 1) * d.vocab) / NC);
  uint4 lw[kLmRows][IT];
  int rb = v0 + warp * kLmRows;
#pragma unroll
  for (int i = 0; i < kLmRows; ++i) row_load<IT>(rb + i < v1 ? a.out_w + (size_t)(rb + i) * dim : nullptr, dim, lw[i]);
  if (!cta_barrier(gbar, (++n_grid) * NC, a.err, &fail_s)) return;
  mark(16 * d.n_layers + 1);
  for (int i = tid; i < dim; i += kT) xf[i] = __ldcg(b.x + i);
  __syncthreads();
  const float xs = norm_quant_smem(xf, a.final_norm, dim, xb, xq, red);
  unsigned long long best = 0ull;
  for (; rb < v1; rb += kW * kLmRows) {
    int acc[kLmRows];
#pragma unroll
    for (int i = 0; i < kLmRows; ++i) acc[i] = row_dot<IT>(lw[i], xq, dim);
    const int nb = rb + kW * kLmRows;
#pragma unroll
    for (int i = 0; i < kLmRows; ++i) row_load<IT>(nb + i < v1 ? a.out_w + (size_t)(nb + i) * dim : nullptr, dim, lw[i]);
#pragma unroll
    for (int i = 0; i < kLmRows; ++i) {
      const int r = rb + i;
      if (lane == i && r < v1) {
        const float v = __fmul_rn(__fmul_rn((float)acc[i], __ldg(a.out_s + r)), xs);
        b.logits[r] = v;
        const unsigned long long key = ((unsigned long long)ordered_key(v) << 32) | (unsigned)r;
        best = key > best ? key : best;
      }
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  if (lane == 0 && best) atomicMax(&b.st->argmax_key, best);
  mark(16 * d.n_layers + 2);
}

// Resets the barrier counters and absmax slots after a step (stream order:
// after k_persist), then optionally advances the step state as k_advance does.
__global__ void k_persist_reset(unsigned* bar, int n_words, unsigned* amax) {
  for (int i = threadIdx.x; i < n_words; i += blockDim.x) bar[i] = 0u;
  if (threadIdx.x < 16) amax[threadIdx.x] = 0u;
}

}  // namespace

bool persist_plan(const Dims& d, int num_sms, PersistPlan* pl, std::string* why) {
  auto no = [&](const char* m) {
    if (why) *why = m;
    return false;
  };
  if (d.n_experts < 2 || d.top_k < 1 || d.top_k > 8) return no("needs a MoE model with top_k <= 8");
  if (d.group != 32) return no("needs int4 group 32");
  if (d.dim % 128 || d.hidden % 128 || d.dim > 2048) return no("needs dim, hidden multiples of 128, dim <= 2048");
  if (d.head_dim != 64 && d.head_dim != 128) return no("needs head_dim 64 or 128");
  if (d.n_heads * d.head_dim != d.dim) return no("needs n_heads * head_dim == dim");
  const int NC = num_sms;
  if (NC < 2 * d.n_heads) return no("needs two CTAs per head");
  const int K = d.top_k, H = d.hidden, dim = d.dim, ngd = dim / 32, ngh = H / 32;
  const int max_pairs = (int)(((long)K * H + NC - 1) / NC) + 1;
  const int max_rows = (dim + NC - 1) / NC + 1;
  const int min_gs = NC / d.n_heads;
  const int max_cols = (d.head_dim + min_gs - 1) / min_gs;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 127) & ~size_t(127);
    return (int)o;
  };
  pl->o_xq = take(dim);
  pl->o_xf = take((size_t)dim * 4);
  pl->o_xb = take((size_t)dim * 4);
  pl->o_own = take((size_t)max_rows * 4);
  pl->o_red = take(64 * 4);
  pl->o_bars = take(24);
  const size_t p_gu = (size_t)2 * max_pairs * (ngd + 1), p_dn = (size_t)K * max_rows * (ngh + 1);
  pl->o_P = take(std::max(p_gu, p_dn) * 4);
  pl->o_T = take((size_t)std::max(2 * max_pairs, K * max_rows) * 4);
  pl->o_xh = take((size_t)K * H);
  const size_t st_exp = (size_t)max_pairs * 2 * (dim / 2 + ngd * 4) + (size_t)K * max_rows * (H / 2 + ngh * 4);
  const size_t st_att = (size_t)(((d.max_seq + 3) & ~3) + max_cols * (kPvTile + 4)) * 4;
  const size_t st_rt = ((size_t)d.n_experts * (dim + 16) + 32) * 4;  // router W, lanes, logits
  pl->o_stage = take(std::max(std::max(st_exp, st_att), st_rt));
  pl->smem = off;
  pl->max_pairs = max_pairs;
  pl->max_rows = max_rows;
  if (off > 227 * 1024) return no("shared memory plan above 227 KB");
  return true;
}

cudaError_t launch_persist(const PersistArgs& a, int num_sms, cudaStream_t s) {
  const Dims& d = a.d;
  const int it = (d.dim / 16 + 31) / 32;
  void (*k)(PersistArgs) = nullptr;
  if (d.head_dim == 64)
    k = it <= 1 ? k_persist<1, 64> : it == 2 ? k_persist<2, 64> : it == 3 ? k_persist<3, 64> : k_persist<4, 64>;
  else
    k = it <= 1 ? k_persist<1, 128> : it == 2 ? k_persist<2, 128> : it == 3 ? k_persist<3, 128> : k_persist<4, 128>;
  cudaError_t r = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)a.plan.smem);
  if (r != cudaSuccess) return r;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_sms);
  cfg.blockDim = dim3(kT);
  cfg.dynamicSmemBytes = a.plan.smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, a);
}

cudaError_t launch_persist_reset(unsigned* bar, unsigned* amax, cudaStream_t s) {
  k_persist_reset<<<1, 256, 0, s>>>(bar, kPersistBarWords, amax);
  return cudaGetLastError();
}

}  // namespace chalot
