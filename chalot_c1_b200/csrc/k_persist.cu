// k_persist.cu — the whole batch-1 decode step (Engine::forward,
// src/model/engine.rs:173-494) as ONE persistent kernel: one CTA per SM,
// co-resident by cooperative launch, with no grid barrier at all.
//
// Every value one CTA passes to another travels in a 64-bit word that holds
// the f32 value and a 32-bit tag (step epoch, layer, phase): the producer
// writes the word with one 64-bit store, the consumer spins on the word
// itself until its tag is the expected one. A 64-bit aligned access is
// single-copy atomic, so the tag and the value arrive together, and each
// dependency costs one L2 round trip instead of a barrier followed by a load.
//
// Per layer (every float operation in the reference's order, as the
// multi-kernel path in k_dense.cu / k_attn.cu / k_moe.cu):
//   A  every CTA: x (the previous layer's rows, tagged), rmsnorm(x, rms_attn)
//      and quantize_f32_to_i8 in shared memory; the CTAs of head group h
//      compute head h's Q, K and V row pairs (weights requested earlier),
//      RoPE; K and V go to the cache and, with q, to tagged words.
//   B1 group h: scores of head h for a slice of positions (K rows of earlier
//      steps prefetched into shared memory; dot_f32 order; soft-cap with the
//      restated tanhf) -> tagged words.
//   B2 group h: every CTA of the group runs softmax_avx2 over all scores of
//      the head, then the t-ordered sums of its slice of output columns (V
//      rows of earlier steps prefetched) -> tagged att_out words.
//   C  every CTA quantizes att_out; CTA c computes its O rows and updates the
//      x rows it owns (rows [c*dim/N, (c+1)*dim/N), also its down rows).
//   D  every CTA: rmsnorm(x, rms_ffn), quantize, router logits and
//      softmax_top_k (the same bits in every CTA), then bulk-copies its share
//      of the selected experts' gate/up rows and its down rows into shared
//      memory.
//   E  gate/up group products, ordered group sums, SwiGLU -> tagged h words.
//   F  every CTA reads all of h, takes its absmax per expert, quantizes it;
//      CTA c's down rows, ordered sums, gated combine in selection order,
//      x rows += -> tagged x words.
// After the last layer every CTA computes the final norm and quantization and
// streams its slice of the lm_head rows through a ring of bulk copies; the
// argmax (ties to the last index) is a 64-bit atomicMax.
//
// Every wait is bounded (globaltimer, 200 ms): a CTA that gives up sets the
// engine's error word (the host reports CHALOT_ERR_TIMEOUT) and every other
// waiter leaves as soon as it sees that word. The step epoch advances after
// each launch (k_persist_epoch), so no word of an earlier step can match.
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

// phases of the tagged words
enum : uint32_t { kTagQkv = 1, kTagScore = 2, kTagAtt = 3, kTagXc = 4, kTagH = 5, kTagXf = 6 };

CHALOT_DEV unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

CHALOT_DEV void ll_store(uint64_t* p, float v, uint32_t tag) {
  const uint64_t w = ((uint64_t)tag << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
CHALOT_DEV uint64_t ll_load(const uint64_t* p) {
  uint64_t w;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}

// Announces that this CTA wrote its part of a broadcast: one relaxed add on
// each of the kCntLines counter lines of `cnt` (the tagged words themselves
// still validate every value).
constexpr int kCntLines = 8;
CHALOT_DEV void ll_announce(unsigned* cnt) {
  __syncthreads();
  if (threadIdx.x < kCntLines)
    asm volatile("red.relaxed.gpu.global.add.u32 [%0], 1;" ::"l"(cnt + 32 * threadIdx.x) : "memory");
}

// Waits (one thread, bounded, with a short back-off) until counter line
// c % kCntLines of `cnt` reaches `target`: every producer of the broadcast
// has announced, so the following gather finds its words written. Only a
// few CTAs poll each line.
__device__ __noinline__ bool ll_wait_count(const unsigned* cnt, unsigned target, unsigned* err, int* fail_s) {
  if (threadIdx.x == 0) {
    const unsigned* p = cnt + 32 * (blockIdx.x % kCntLines);
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    if (v < target) {
      const unsigned long long t0 = gtimer();
      for (int k = 1;; ++k) {
        __nanosleep(32);
        asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
        if (v >= target) break;
        if ((k & 63) == 0 && (*(volatile unsigned*)err || gtimer() - t0 > kWaitNs)) {
          atomicOr(err, 1u);
          *(volatile int*)fail_s = 1;
          break;
        }
      }
    }
  }
  __syncthreads();
  return *(volatile int*)fail_s == 0;
}

// dst[i] = value of p[i] for i < n, each word waited for until it carries
// `tag`. Every thread of the CTA calls it; the values are in shared memory
// after the barrier at the end. False (the error word set, or seen set) when
// a wait ran out.
__device__ __noinline__ bool ll_gather(const uint64_t* p, int n, uint32_t tag, float* dst, unsigned* err,
                                       int* fail_s) {
  constexpr int U = 10;
  bool ok = true;
  for (int base = 0; base < n && ok; base += U * kT) {
    uint64_t w[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * kT + (int)threadIdx.x;
      w[u] = i < n ? ll_load(p + i) : ((uint64_t)tag << 32);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * kT + (int)threadIdx.x;
      if ((uint32_t)(w[u] >> 32) != tag) {
        const unsigned long long t0 = gtimer();
        for (int k = 1;; ++k) {
          w[u] = ll_load(p + i);
          if ((uint32_t)(w[u] >> 32) == tag) break;
          if ((k & 63) == 0 && (*(volatile unsigned*)err || gtimer() - t0 > kWaitNs)) {
            atomicOr(err, 1u);
            ok = false;
            break;
          }
        }
        if (!ok) break;
      }
      if (i < n) dst[i] = __uint_as_float((uint32_t)w[u]);
    }
  }
  if (!ok) *(volatile int*)fail_s = 1;
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

// 16-byte asynchronous copy global -> shared (L2 only), completed by
// cp_async_wait_all in the issuing thread.
CHALOT_DEV void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
CHALOT_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

CHALOT_DEV void mbar_init_count(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
CHALOT_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
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
// The same for a row in shared memory.
template <int IT>
CHALOT_DEV int row_dot_smem(const int8_t* row, const int8_t* xq, int n) {
  const int lane = threadIdx.x & 31;
  int acc = 0;
#pragma unroll
  for (int it = 0; it < IT; ++it) {
    const int c = lane + 32 * it;
    if (c < (n >> 4)) acc = dot16_i8(lds16(row + c * 16), lds16(xq + c * 16), acc);
  }
  return warp_sum_i(acc);
}

// t = t + p[g] for g = 0..ng-1 in order (matmul.rs:576-577), p 16-byte
// aligned in shared memory: the next 16 values are loaded while the current
// 16 are added, so the chain runs at the add latency.
CHALOT_DEV float ordered_sum16(const float* p, int ng) {
  float t = 0.0f;
  int g = 0;
  if (ng >= 16) {
    float4 a[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) a[u] = lds16f(p + 4 * u);
    for (; g + 16 <= ng; g += 16) {
      float4 nx[4];
      const bool more = g + 32 <= ng;
#pragma unroll
      for (int u = 0; u < 4; ++u) nx[u] = more ? lds16f(p + g + 16 + 4 * u) : a[u];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        t = __fadd_rn(t, a[u].x);
        t = __fadd_rn(t, a[u].y);
        t = __fadd_rn(t, a[u].z);
        t = __fadd_rn(t, a[u].w);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) a[u] = nx[u];
    }
  }
  for (; g < ng; ++g) t = __fadd_rn(t, p[g]);
  return t;
}

// This thread's elements i = threadIdx.x + u*kT (dim <= 4*kT) of a global
// vector, requested before a barrier.
CHALOT_DEV void load4(const float* __restrict__ w, int dim, float (&wr)[4]) {
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int i = threadIdx.x + u * kT;
    wr[u] = i < dim ? __ldg(w + i) : 0.0f;
  }
}

// Block-wide maximum of non-negative values with one barrier; every thread
// gets it. `part` (kW floats, 16-byte aligned) must not be in use by a
// concurrent call.
CHALOT_DEV float block_max1(float v, float* part) {
  v = warp_max(v);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = v;
  __syncthreads();
  float m = 0.0f;
#pragma unroll
  for (int w = 0; w < kW; w += 4) {
    const float4 q = lds16f(part + w);
    m = fmaxf(fmaxf(m, q.x), fmaxf(fmaxf(q.y, q.z), q.w));
  }
  return m;
}

// rmsnorm_avx2 (normalization.rs:35-67) of xs (shared, dim floats, dim % 8
// == 0) with the weights wr (load4) into xb (shared), then
// quantize_f32_to_i8 (quantization.rs:56-104) into xq (shared); returns the
// scale. Lane j of 8 adds x[8c+j]^2 over c in order: the squares are first
// written column by column (sq: 8 rows of `sqs` floats) so each lane's chain
// reads them with vector loads; the 8 lane sums are combined as hsum8 with
// shuffles.
CHALOT_DEV float norm_quant_smem(const float* xs, const float (&wr)[4], int dim, float* xb, int8_t* xq,
                                 float* red, float* sq, int sqs) {
  const int nc = dim >> 3;
  for (int i = threadIdx.x; i < dim; i += kT) sq[(i & 7) * sqs + (i >> 3)] = __fmul_rn(xs[i], xs[i]);
  __syncthreads();
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    const float sj = lane < 8 ? ordered_sum16(sq + lane * sqs, nc) : 0.0f;
    const float t = __fadd_rn(sj, __shfl_down_sync(0xffffffffu, sj, 4));  // t_j = s_j + s_{j+4}
    const float u = __fadd_rn(t, __shfl_down_sync(0xffffffffu, t, 2));    // t0 + t2, t1 + t3
    const float ss = __fadd_rn(u, __shfl_down_sync(0xffffffffu, u, 1));
    if (lane == 0) red[8] = div_rn(1.0f, __fsqrt_rn(__fadd_rn(div_rn(ss, (float)dim), 1e-5f)));
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
  quant_scale(block_max1(m, red + 32), &scale, &qinv);
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int i = threadIdx.x + u * kT;
    if (i < dim) xq[i] = quant_any(xb[i], qinv, i, dim);
  }
  __syncthreads();
  return scale;
}

CHALOT_DEV ExpertPtrs layer_expert(const LayerPtrs& L, int E, int e) {
  return E <= 16 ? L.ex[e] : L.experts[e];
}

// Requests the K rows [t0, min(t1, pos)) and the V columns [k0, k0+ncol)
// of rows [0, pos) of head h of layer l (rows written by earlier steps) into
// shared memory: ks [t1-t0][HD], vs [n][ncol].
template <int HD>
CHALOT_DEV void prefetch_kv(const DecodeBufs& b, const Dims& d, int l, int h, int pos, int t0, int t1, int k0,
                            int ncol, float* ks, float* vs) {
  const size_t lb = (size_t)l * d.max_seq;
  const int te = min(t1, pos);
  const int nk = max(te - t0, 0) * (HD / 4);
  for (int i = threadIdx.x; i < nk; i += kT) {
    const int r = i / (HD / 4), u = i - r * (HD / 4);
    cp_async16(ks + r * HD + 4 * u, b.kc + (lb + t0 + r) * d.dim + h * HD + 4 * u);
  }
  const int q = ncol >> 2, nv = pos * q;
  for (int i = threadIdx.x; i < nv; i += kT) {
    const int t = i / q, u = i - t * q;
    cp_async16(vs + t * ncol + 4 * u, b.vc + (lb + t) * d.dim + h * HD + k0 + 4 * u);
  }
}

template <int IT, int HD>
__global__ void __launch_bounds__(kT, 1) k_persist(PersistArgs a) {
  extern __shared__ __align__(128) unsigned char sm[];
  const Dims& d = a.d;
  const DecodeBufs& b = a.b;
  const PersistPlan& pl = a.plan;
  const PersistLL& ll = a.ll;
  const int c = blockIdx.x, NC = gridDim.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int dim = d.dim, H = d.hidden, K = d.top_k, E = d.n_experts;
  const int ngd = dim >> 5, ngh = H >> 5;
  int8_t* xq = reinterpret_cast<int8_t*>(sm + pl.o_xq);     // [dim] quantized vector of the phase
  float* xf = reinterpret_cast<float*>(sm + pl.o_xf);       // [dim] x (or att_out)
  float* xb = reinterpret_cast<float*>(sm + pl.o_xb);       // [dim] normalised vector
  float* own = reinterpret_cast<float*>(sm + pl.o_own);     // [rows_max] this CTA's x rows
  float* red = reinterpret_cast<float*>(sm + pl.o_red);     // [64] reductions, scales
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + pl.o_bars);  // gate/up, down, router, lm_head ring
  float* P = reinterpret_cast<float*>(sm + pl.o_P);         // group products
  float* Tt = reinterpret_cast<float*>(sm + pl.o_T);        // row totals
  int8_t* xh = reinterpret_cast<int8_t*>(sm + pl.o_xh);     // [K][H] quantized h
  ExpertPtrs* xp_s = reinterpret_cast<ExpertPtrs*>(sm + pl.o_xp);  // [E] this layer's experts
  float* sq = reinterpret_cast<float*>(sm + pl.o_sq);        // [8][sqs] squares of the norm
  unsigned char* stg = sm + pl.o_stage;                     // K/V, router weights, expert rows, lm_head rows
  __shared__ int fail_s;
  __shared__ int sel_s[8];
  __shared__ float selw_s[8];
  __shared__ float xs_s;
  __shared__ float rb_s[64];
  if (tid == 0) {
    fail_s = 0;
    for (int i = 0; i < 3 + kLmStages; ++i) mbar_init(&bars[i]);
  }
  const uint32_t pos = b.st->pos, tok = b.st->token;
  const int n = (int)pos + 1;
  const uint32_t tag0 = *a.epoch * (uint32_t)(8 * d.n_layers + 8);
  auto tag = [&](int l, uint32_t ph) { return tag0 + (uint32_t)(8 * l) + ph; };
  // head group of this CTA and its place in it
  const int h = (int)(((long)c * d.n_heads) / NC);
  const int g0 = (int)(((long)h * NC + d.n_heads - 1) / d.n_heads);
  const int g1 = (int)(((long)(h + 1) * NC + d.n_heads - 1) / d.n_heads);
  const int gs = g1 - g0, gj = c - g0;
  // positions [t0, t1) of this CTA's scores; output columns [k0, k0+ncol) (4-aligned)
  const int t0 = (gj * n) / gs, t1 = ((gj + 1) * n) / gs;
  const int k0 = 4 * ((gj * (HD / 4)) / gs), ncol = 4 * (((gj + 1) * (HD / 4)) / gs) - k0;
  float* ks = reinterpret_cast<float*>(stg);                            // [t1-t0][HD]
  float* vs = reinterpret_cast<float*>(stg + pl.o_vs);                  // [n][ncol]
  float* pp = reinterpret_cast<float*>(stg + pl.o_pp);                  // [max_seq] probabilities
  float* vt = reinterpret_cast<float*>(stg + pl.o_vt);                  // [ncol][kPvTile + 4] products
  // rows of x (O rows, down rows) owned by this CTA
  const int r0 = (int)(((long)c * dim) / NC), r1 = (int)(((long)(c + 1) * dim) / NC), nr = r1 - r0;
  unsigned long long* tr = (a.trace && c == 0 && tid == 0) ? a.trace : nullptr;
  // with a.trace_max: the latest time any CTA reached each mark
  unsigned long long* trm = (a.trace_max && tid == 0) ? a.trace_max : nullptr;
  auto mark = [&](int slot) {
    if (tr) tr[slot] = gtimer();
    if (trm) asm volatile("red.relaxed.gpu.global.max.u64 [%0], %1;" ::"l"(trm + slot), "l"(gtimer()) : "memory");
  };
  auto mark_clk = [&](int slot) {  // SM clock cycles (with the ns marks: the clock rate)
    if (tr) tr[slot] = clock64();
  };
  mark(32 * d.n_layers + 0);
  prefetch_kv<HD>(b, d, 0, h, (int)pos, t0, t1, k0, ncol, ks, vs);
  // ---- embedding (engine.rs:201-210): every CTA builds x itself ----
  {
    const float s = __ldg(a.emb_s + tok);
    const int8_t* row = a.emb + (size_t)tok * dim;
    for (int i = tid; i < dim; i += kT) xf[i] = __fmul_rn((float)row[i], s);
    if (c == 0 && tid == 0) b.st->argmax_key = 0ull;
    __syncthreads();
    for (int i = tid; i < nr; i += kT) own[i] = xf[r0 + i];
  }
  const int np_h = 3 * HD / 2;  // Q, K, V row pairs of one head
  const int pq0 = (gj * np_h) / gs, pq1 = ((gj + 1) * np_h) / gs;
  const int half = HD >> 1;
  const float inv_sqrt = div_rn(1.0f, __fsqrt_rn((float)HD));
  float wn[4];  // norm weights of the next normalisation, requested before its wait
  for (int l = 0; l < d.n_layers; ++l) {
    const LayerPtrs& L = a.layers[l];
    mark(l * 32 + 0);
    mark_clk(l * 32 + 30);
    // ---- A: QKV of head h ----
    // before the wait: this warp's first row pair, its scales and rotation,
    // the norm weights
    uint4 w0[IT], w1[IT];
    float sc0 = 0.0f, sc1 = 0.0f, cs = 1.0f, sn = 0.0f;
    {
      const int p = pq0 + warp;
      const int sec = p / half, i = p % half;
      const size_t row = (size_t)sec * dim + h * HD + 2 * i;
      row_load<IT>(p < pq1 ? L.qkv + row * dim : nullptr, dim, w0);
      row_load<IT>(p < pq1 ? L.qkv + (row + 1) * dim : nullptr, dim, w1);
      if (p < pq1 && lane == 0) {
        sc0 = __ldg(L.qkv_s + row);
        sc1 = __ldg(L.qkv_s + row + 1);
        if (sec < 2) {
          cs = __ldg(b.rope_cos + (size_t)pos * half + i);
          sn = __ldg(b.rope_sin + (size_t)pos * half + i);
        }
      }
      load4(L.rms_attn, dim, wn);
    }
    if (l > 0 && !(ll_wait_count(ll.cnt + kCntXf, (unsigned)(NC * l), a.err, &fail_s) &&
                   ll_gather(ll.x + dim, dim, tag(l - 1, kTagXf), xf, a.err, &fail_s)))
      break;
    mark(l * 32 + 1);
    {
      const float s = norm_quant_smem(xf, wn, dim, xb, xq, red, sq, pl.sqs);
      mark(l * 32 + 16);
      for (int p = pq0 + warp; p < pq1; p += kW) {
        const int sec = p / half, i = p % half;
        const size_t row = (size_t)sec * dim + h * HD + 2 * i;
        if (p != pq0 + warp) {
          row_load<IT>(L.qkv + row * dim, dim, w0);
          row_load<IT>(L.qkv + (row + 1) * dim, dim, w1);
          if (lane == 0) {
            sc0 = __ldg(L.qkv_s + row);
            sc1 = __ldg(L.qkv_s + row + 1);
            cs = sec < 2 ? __ldg(b.rope_cos + (size_t)pos * half + i) : 1.0f;
            sn = sec < 2 ? __ldg(b.rope_sin + (size_t)pos * half + i) : 0.0f;
          }
        }
        const int dot0 = row_dot<IT>(w0, xq, dim), dot1 = row_dot<IT>(w1, xq, dim);
        if (lane == 0) {
          float v0 = __fmul_rn(__fmul_rn((float)dot0, sc0), s);
          float v1 = __fmul_rn(__fmul_rn((float)dot1, sc1), s);
          if (sec < 2) {  // RoPE on the interleaved pair (engine.rs:252-271)
            const float x0 = __fsub_rn(__fmul_rn(v0, cs), __fmul_rn(v1, sn));
            const float x1 = __fadd_rn(__fmul_rn(v0, sn), __fmul_rn(v1, cs));
            v0 = x0;
            v1 = x1;
          }
          const int col = h * HD + 2 * i;
          if (sec > 0) {  // engine.rs:274-280: the cache row, for later steps
            float* cache = sec == 1 ? b.kc : b.vc;
            const size_t off = ((size_t)l * d.max_seq + pos) * dim + col;
            cache[off] = v0;
            cache[off + 1] = v1;
          }
          uint64_t* dst = ll.q + (size_t)sec * dim + col;  // q, k, v of this step, tagged
          ll_store(dst, v0, tag(l, kTagQkv));
          ll_store(dst + 1, v1, tag(l, kTagQkv));
        }
      }
    }
    mark(l * 32 + 2);
    // ---- B1: scores of head h for positions [t0, t1) ----
    {
      float* qh = xb;  // [HD], then this step's key [HD] when pos is in the slice
      const bool has_pos = (int)pos >= t0 && (int)pos < t1;
      // q (and k at pos) of head h from the group's tagged words; V at pos for B2
      if (!ll_gather(ll.q + h * HD, HD, tag(l, kTagQkv), qh, a.err, &fail_s)) break;
      if (has_pos && !ll_gather(ll.q + dim + h * HD, HD, tag(l, kTagQkv), ks + ((int)pos - t0) * HD, a.err, &fail_s))
        break;
      mark(l * 32 + 3);
      cp_async_wait_all();
      __syncthreads();
      for (int t = t0 + tid; t < t1; t += kT) {
        const float* kk = ks + (t - t0) * HD;
        float a0[8], a1[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) a0[j] = a1[j] = 0.0f;
#pragma unroll
        for (int cc = 0; cc < HD / 16; ++cc) {
          const float4 k4[4] = {lds16f(kk + cc * 16), lds16f(kk + cc * 16 + 4), lds16f(kk + cc * 16 + 8),
                                lds16f(kk + cc * 16 + 12)};
          const float* kv = reinterpret_cast<const float*>(k4);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            a0[j] = __fadd_rn(a0[j], __fmul_rn(qh[cc * 16 + j], kv[j]));
            a1[j] = __fadd_rn(a1[j], __fmul_rn(qh[cc * 16 + 8 + j], kv[8 + j]));
          }
        }
        float cmb[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) cmb[j] = __fadd_rn(a0[j], a1[j]);
        const float x = __fmul_rn(hsum8(cmb), inv_sqrt);
        ll_store(ll.score + (size_t)h * d.max_seq + t, __fmul_rn(30.0f, libm::tanh_f32(div_rn(x, 30.0f))),
                 tag(l, kTagScore));
      }
    }
    mark(l * 32 + 4);
    // ---- B2: softmax over the head's n scores, t-ordered sums of columns [k0, k0+ncol) ----
    if (ncol > 0) {
      if (!ll_gather(ll.score + (size_t)h * d.max_seq, n, tag(l, kTagScore), pp, a.err, &fail_s)) break;
      if (!ll_gather(ll.q + 2 * dim + h * HD + k0, ncol, tag(l, kTagQkv), vs + (size_t)pos * ncol, a.err, &fail_s))
        break;
      mark(l * 32 + 5);
      // softmax_avx2 (normalization.rs:106-160): max; e = fast_exp(s - max) on
      // whole 8-chunks, libm exp on the tail; lane j of 8 adds e[8c+j] over c
      // in order (the e of the chunks also written column by column, eT, for
      // vector loads), hsum8, then the tail in order; inv = 1/sum.
      float mx = -INFINITY;
      for (int i = tid; i < n; i += kT) mx = fmaxf(mx, pp[i]);
      {  // block max (scores may be negative)
        mx = warp_max(mx);
        if (lane == 0) red[32 + warp] = mx;
        __syncthreads();
        mx = red[32];
#pragma unroll
        for (int w = 1; w < kW; ++w) mx = fmaxf(mx, red[32 + w]);
      }
      const int full = n & ~7, nc8 = full >> 3, es = pl.ets;
      float* eT = vt;  // [8][es]: the chunk part of e by lane (the products come later)
      for (int i = tid; i < n; i += kT) {
        float e;
        if (i < full)
          e = fast_exp(__fsub_rn(pp[i], mx));
        else
          e = expf_cr(__fsub_rn(pp[i], mx));
        pp[i] = e;
        if (i < full) eT[(i & 7) * es + (i >> 3)] = e;
      }
      __syncthreads();
      if (warp == 0) {
        const float sj = lane < 8 ? ordered_sum16(eT + lane * es, nc8) : 0.0f;
        const float t = __fadd_rn(sj, __shfl_down_sync(0xffffffffu, sj, 4));
        const float u = __fadd_rn(t, __shfl_down_sync(0xffffffffu, t, 2));
        float sum = __fadd_rn(u, __shfl_down_sync(0xffffffffu, u, 1));
        if (lane == 0) {
          for (int i = full; i < n; ++i) sum = __fadd_rn(sum, pp[i]);
          red[9] = div_rn(1.0f, sum);
        }
      }
      __syncthreads();
      mark(l * 32 + 17);
      const float inv = red[9];
      float acc = 0.0f;
      for (int tt = 0; tt < n; tt += kPvTile) {
        const int rows = min(kPvTile, n - tt);
        if (tt > 0) __syncthreads();
        // products p_t * V[t][col] of this tile, column-major (each chain reads its column)
        for (int i = tid; i < rows * ncol; i += kT) {
          const int r = i / ncol, cc = i - r * ncol, t = tt + r;
          vt[cc * (kPvTile + 4) + r] = __fmul_rn(__fmul_rn(pp[t], inv), vs[t * ncol + cc]);
        }
        __syncthreads();
        mark(l * 32 + 18);
        if (tid < ncol) {  // out[c] = sum_t p_t v_t[c], added in t order (engine.rs:302-308)
          const float* pc = vt + tid * (kPvTile + 4);
          int r = 0;
          if (rows >= 16) {
            float4 q4[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) q4[u] = lds16f(pc + 4 * u);
            for (; r + 16 <= rows; r += 16) {
              float4 nx[4];
              const bool more = r + 32 <= rows;
#pragma unroll
              for (int u = 0; u < 4; ++u) nx[u] = more ? lds16f(pc + r + 16 + 4 * u) : q4[u];
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                acc = __fadd_rn(acc, q4[u].x);
                acc = __fadd_rn(acc, q4[u].y);
                acc = __fadd_rn(acc, q4[u].z);
                acc = __fadd_rn(acc, q4[u].w);
              }
#pragma unroll
              for (int u = 0; u < 4; ++u) q4[u] = nx[u];
            }
          }
          for (; r < rows; ++r) acc = __fadd_rn(acc, pc[r]);
        }
      }
      if (tid < ncol) ll_store(ll.att + h * HD + k0 + tid, acc, tag(l, kTagAtt));
    }
    mark(l * 32 + 6);
    // ---- C: O rows r0..r1 + residual (engine.rs:312-322) ----
    uint4 ow[IT];
    float os = 0.0f;
    row_load<IT>(warp < nr ? L.o + (size_t)(r0 + warp) * dim : nullptr, dim, ow);
    if (warp < nr && lane == 0) os = __ldg(L.o_s + r0 + warp);
    __syncthreads();  // the attention's staging area is free
    float* rw_s = reinterpret_cast<float*>(stg);  // [E][dim] router weights for D
    if (tid == 0) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_expect_tx(&bars[2], (uint32_t)(E * dim * 4));
      tma_load(rw_s, L.router_w, (uint32_t)(E * dim * 4), &bars[2]);
    }
    if (!ll_gather(ll.att, dim, tag(l, kTagAtt), xf, a.err, &fail_s)) {
      if (tid == 0) mbar_wait_t(&bars[2], l & 1, a.err);  // no copy may land after the CTA left
      break;
    }
    mark(l * 32 + 7);
    {
      float m = 0.0f;
      for (int i = tid; i < dim; i += kT) m = fmaxf(m, fabsf(xf[i]));
      float scale, qinv;
      quant_scale(block_max(m, red), &scale, &qinv);
      for (int i = tid; i < dim; i += kT) xq[i] = quant_any(xf[i], qinv, i, dim);
      __syncthreads();
      for (int w = warp; w < nr; w += kW) {
        if (w != warp) {
          row_load<IT>(L.o + (size_t)(r0 + w) * dim, dim, ow);
          if (lane == 0) os = __ldg(L.o_s + r0 + w);
        }
        const int dot = row_dot<IT>(ow, xq, dim);
        if (lane == 0) {
          const float v = __fmul_rn(__fmul_rn((float)dot, os), scale);
          own[w] = __fadd_rn(own[w], v);
          ll_store(ll.x + r0 + w, own[w], tag(l, kTagXc));
        }
      }
      ll_announce(ll.cnt + kCntXc);
    }
    mark(l * 32 + 8);
    // before the wait: FFN norm weights, router bias, this layer's expert pointers
    load4(L.rms_ffn, dim, wn);
    if (tid < E) {
      rb_s[tid] = __ldg(L.router_b + tid);
      xp_s[tid] = layer_expert(L, E, tid);
    }
    if (!(ll_wait_count(ll.cnt + kCntXc, (unsigned)(NC * (l + 1)), a.err, &fail_s) &&
          ll_gather(ll.x, dim, tag(l, kTagXc), xf, a.err, &fail_s))) {
      if (tid == 0) mbar_wait_t(&bars[2], l & 1, a.err);
      break;
    }
    mark(l * 32 + 9);
    // ---- D: FFN norm, quantize, routing (engine.rs:325-344) ----
    {
      const float s = norm_quant_smem(xf, wn, dim, xb, xq, red, sq, pl.sqs);
      mark(l * 32 + 19);
      float* lanes = rw_s + (size_t)E * dim;  // [16E]
      float* logit = lanes + 16 * E;
      if (tid == 0 && !mbar_wait_t(&bars[2], l & 1, a.err)) fail_s = 1;
      __syncthreads();
      if (fail_s) break;
      mark(l * 32 + 20);
      router_logits(rw_s, rb_s, xb, dim, E, lanes, logit);
      mark(l * 32 + 21);
      if (warp == 0) topk_warp(logit, E, K, sel_s, selw_s);
      if (tid == 0) xs_s = s;
      mark(l * 32 + 14);
      if (c == 0 && b.router_trace)
        for (int e = tid; e < E; e += kT) b.router_trace[l * E + e] = logit[e];
      __syncthreads();
      mark(l * 32 + 15);
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
    if (warp == 0) {  // the copies, one per lane of warp 0
      if (lane == 0) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_expect_tx(&bars[0], (uint32_t)npair * 2 * (prow + ngd * 4));
        mbar_expect_tx(&bars[1], (uint32_t)(K * nr * (hrow + ngh * 4)));
      }
      __syncwarp();
      const uint64_t pol = l2_evict_first();
      // segments of the pair range: choice j, units [u0, u0+m), local rows from lb;
      // copy k of segment sg: 0 gate rows, 1 up rows, 2 gate scales, 3 up scales
      int lb = 0, sg = 0;
      for (int q = q0; q < q1; ++sg) {
        const int j = q / H, u0 = q % H, m = min(H, u0 + (q1 - q)) - u0;
        if (m <= 0) break;
        if (lane >= 4 * sg && lane < 4 * sg + 4) {
          const ExpertPtrs& X = xp_s[sel_s[j]];
          const int k = lane - 4 * sg, up = k & 1;
          if (k < 2)
            tma_load_hint(gu_w + (size_t)(lb + up * m) * prow, X.gu + (size_t)(up * H + u0) * prow,
                          (uint32_t)(m * prow), &bars[0], pol);
          else
            tma_load_hint(gu_s + (size_t)(lb + up * m) * ngd, X.gu_s + (size_t)(up * H + u0) * ngd,
                          (uint32_t)(m * ngd * 4), &bars[0], pol);
        }
        lb += 2 * m;
        q += m;
      }
      // down rows and scales of choice j: lanes 16 + 2j (rows), 17 + 2j (scales)
      if (lane >= 16 && lane < 16 + 2 * K && nr > 0) {
        const int j = (lane - 16) >> 1;
        const ExpertPtrs& X = xp_s[sel_s[j]];
        if (((lane - 16) & 1) == 0)
          tma_load_hint(dn_w + (size_t)j * nr * hrow, X.dn + (size_t)r0 * hrow, (uint32_t)(nr * hrow), &bars[1], pol);
        else
          tma_load_hint(dn_s + (size_t)j * nr * ngh, X.dn_s + (size_t)r0 * ngh, (uint32_t)(nr * ngh * 4), &bars[1],
                        pol);
      }
    }
    mark(l * 32 + 10);
    // ---- E: gate/up (engine.rs:366-377) ----
    {
      const float xs = xs_s;
      if (tid == 0 && !mbar_wait_t(&bars[0], l & 1, a.err)) fail_s = 1;
      __syncthreads();
      if (fail_s) {
        if (tid == 0) mbar_wait_t(&bars[1], l & 1, a.err);
        break;
      }
      mark(l * 32 + 22);
      const int nrow = 2 * npair, PS = pl.ps_gu;
      // warp w: rows w, w + kW, ...; lane g: groups g, g + 32, ... (x chunks in registers)
      for (int g0 = 0; g0 < ngd; g0 += 32) {
        const int g = g0 + lane;
        const bool gl = g < ngd;
        const uint4 x0 = gl ? lds16(xq + g * 32) : make_uint4(0, 0, 0, 0);
        const uint4 x1 = gl ? lds16(xq + g * 32 + 16) : make_uint4(0, 0, 0, 0);
        if (gl)
          for (int row = warp; row < nrow; row += kW) {
            const int dv = dot32_rp(lds16(gu_w + (size_t)row * prow + g * 16), x0, x1);
            P[row * PS + g] = __fmul_rn(__fmul_rn((float)dv, gu_s[(size_t)row * ngd + g]), xs);
          }
      }
      __syncthreads();
      mark(l * 32 + 23);
      for (int row = tid; row < nrow; row += kT) Tt[row] = ordered_sum16(P + row * PS, ngd);
      __syncthreads();
      mark(l * 32 + 24);
      // pair k of segment (lb, m): gate row lb + k, up row lb + m + k
      int lb = 0;
      for (int q = q0; q < q1;) {
        const int j = q / H, u0 = q % H, m = min(H, u0 + (q1 - q)) - u0;
        for (int k = tid; k < m; k += kT)
          ll_store(ll.h + (size_t)j * H + u0 + k, swiglu_elem(Tt[lb + k], Tt[lb + m + k], u0 + k, H), tag(l, kTagH));
        lb += 2 * m;
        q += m;
      }
      ll_announce(ll.cnt + kCntH);
    }
    mark(l * 32 + 11);
    // ---- F: quantize h, down rows, gated combine, residual (engine.rs:380-401) ----
    {
      float* hf = reinterpret_cast<float*>(stg + pl.o_hf);  // [K][H] f32 h (the gate/up rows are consumed)
      if (!(ll_wait_count(ll.cnt + kCntH, (unsigned)(NC * (l + 1)), a.err, &fail_s) &&
            ll_gather(ll.h, K * H, tag(l, kTagH), hf, a.err, &fail_s))) {
        if (tid == 0) mbar_wait_t(&bars[1], l & 1, a.err);
        break;
      }
      mark(l * 32 + 12);
      float* xsh = red + 16;  // [K] scales of h
      {  // quantize_f32_to_i8 of each h_j (quantization.rs:56-104): absmax, then RNE
        const int n4 = (K * H) >> 2, h4 = H >> 2;
        float mj[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) mj[j] = 0.0f;
        for (int i = tid; i < n4; i += kT) {
          const float4 v = lds16f(hf + 4 * i);
          const float m4 = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
          const int j = i / h4;
#pragma unroll
          for (int jj = 0; jj < 8; ++jj)
            if (jj == j) mj[jj] = fmaxf(mj[jj], m4);
        }
        float* part = P;  // [K][kW] warp maxima (the products come later)
        for (int j = 0; j < K; ++j) {
          const float m = warp_max(mj[j]);
          if (lane == 0) part[j * kW + warp] = m;
        }
        __syncthreads();
        for (int j = 0; j < K; ++j) {
          float m = 0.0f;
#pragma unroll
          for (int w = 0; w < kW; w += 4) {
            const float4 q = lds16f(part + j * kW + w);
            m = fmaxf(fmaxf(m, q.x), fmaxf(fmaxf(q.y, q.z), q.w));
          }
          float sc, inv;
          quant_scale(m, &sc, &inv);
          mj[j] = inv;
          if (tid == 0) xsh[j] = sc;
        }
        mark(l * 32 + 25);
        uint32_t* xw = reinterpret_cast<uint32_t*>(xh);
        for (int i = tid; i < n4; i += kT) {
          const float4 v = lds16f(hf + 4 * i);
          const int j = i / h4;
          float inv = mj[0];
#pragma unroll
          for (int jj = 1; jj < 8; ++jj)
            if (jj == j) inv = mj[jj];
          const uint32_t b0 = (uint8_t)quant_elem(v.x, inv), b1 = (uint8_t)quant_elem(v.y, inv);
          const uint32_t b2 = (uint8_t)quant_elem(v.z, inv), b3 = (uint8_t)quant_elem(v.w, inv);
          xw[i] = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
        }
      }
      if (tid == 0 && !mbar_wait_t(&bars[1], l & 1, a.err)) fail_s = 1;
      __syncthreads();
      if (fail_s) break;
      mark(l * 32 + 26);
      const int nrow = K * nr, PS = pl.ps_dn;
      for (int row = warp; row < nrow; row += kW) {  // warp per row, lanes over the groups
        const int j = row / nr;
        const int8_t* xj = xh + (size_t)j * H;
        const unsigned char* wr = dn_w + (size_t)row * hrow;
        const float* sr = dn_s + (size_t)row * ngh;
        const float xsj = xsh[j];
        for (int g = lane; g < ngh; g += 32) {
          const int dv = dot32_rp(lds16(wr + g * 16), lds16(xj + g * 32), lds16(xj + g * 32 + 16));
          P[row * PS + g] = __fmul_rn(__fmul_rn((float)dv, sr[g]), xsj);
        }
      }
      __syncthreads();
      mark(l * 32 + 27);
      for (int row = tid; row < nrow; row += kT) Tt[row] = ordered_sum16(P + row * PS, ngh);
      __syncthreads();
      mark(l * 32 + 28);
      if (tid < nr) {
        float add = 0.0f;  // expert_out = sum_k w_k * y_k in selection order (engine.rs:390-396)
        for (int j = 0; j < K; ++j) add = __fadd_rn(add, __fmul_rn(selw_s[j], Tt[j * nr + tid]));
        own[tid] = __fadd_rn(own[tid], add);
        ll_store(ll.x + dim + r0 + tid, own[tid], tag(l, kTagXf));
      }
      ll_announce(ll.cnt + kCntXf);  // (its barrier also frees the staging area)
    }
    mark(l * 32 + 13);
    mark_clk(l * 32 + 31);
    if (l + 1 < d.n_layers) prefetch_kv<HD>(b, d, l + 1, h, (int)pos, t0, t1, k0, ncol, ks, vs);
  }
  if (fail_s) {
    cp_async_wait_all();
    return;
  }
  // ---- final norm, lm_head, argmax (engine.rs:470-493, sampling.rs:34-41) ----
  // CTA c streams rows [v0, v1) through a ring of kLmStages chunks of kLmChunk
  // rows (bulk copies issued by warp kW-1, consumed by the other warps, two
  // rows each per chunk); the first chunks are requested before the wait.
  const int v0 = (int)(((long)c * d.vocab) / NC), v1 = (int)(((long)(c + 1) * d.vocab) / NC);
  const int nchunk = (v1 - v0 + kLmChunk - 1) / kLmChunk;
  const size_t chunk_bytes = (size_t)kLmChunk * dim;
  uint64_t* full = bars + 3;
  uint64_t* empty = bars + 3 + kLmStages;
  int8_t* ring = reinterpret_cast<int8_t*>(stg);
  if (tid == 0) {
    for (int i = 0; i < kLmStages; ++i) mbar_init_count(&empty[i], kW - 1);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    for (int k = 0; k < min(kLmStages, nchunk); ++k) {
      const int rows = min(kLmChunk, v1 - v0 - k * kLmChunk);
      mbar_expect_tx(&full[k], (uint32_t)(rows * dim));
      tma_load(ring + k * chunk_bytes, a.out_w + (size_t)(v0 + k * kLmChunk) * dim, (uint32_t)(rows * dim), &full[k]);
    }
  }
  load4(a.final_norm, dim, wn);
  const bool ok = ll_wait_count(ll.cnt + kCntXf, (unsigned)(NC * d.n_layers), a.err, &fail_s) &&
                  ll_gather(ll.x + dim, dim, tag(d.n_layers - 1, kTagXf), xf, a.err, &fail_s);
  mark(32 * d.n_layers + 1);
  float xs = 0.0f;
  if (ok) xs = norm_quant_smem(xf, wn, dim, xb, xq, red, sq, pl.sqs);
  mark(32 * d.n_layers + 3);
  if (warp == kW - 1) {  // producer: refill stage k % S once its rows were consumed
    if (lane == 0)
      for (int k = kLmStages; k < nchunk; ++k) {
        const int st = k % kLmStages;
        if (!mbar_wait_t(&empty[st], ((k / kLmStages) - 1) & 1, a.err)) break;
        const int rows = min(kLmChunk, v1 - v0 - k * kLmChunk);
        mbar_expect_tx(&full[st], (uint32_t)(rows * dim));
        tma_load(ring + st * chunk_bytes, a.out_w + (size_t)(v0 + k * kLmChunk) * dim, (uint32_t)(rows * dim),
                 &full[st]);
      }
  } else {
    unsigned long long best = 0ull;
    for (int k = 0; k < nchunk; ++k) {
      const int st = k % kLmStages;
      if (!mbar_wait_t(&full[st], (k / kLmStages) & 1, a.err)) break;
      const int rbase = v0 + k * kLmChunk, rows = min(kLmChunk, v1 - rbase);
      const int8_t* cb = ring + st * chunk_bytes;
      int acc[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int rr = warp * 2 + i;
        acc[i] = rr < rows ? row_dot_smem<IT>(cb + (size_t)rr * dim, xq, dim) : 0;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
      if (ok && lane < 2) {
        const int rr = warp * 2 + lane;
        if (rr < rows) {
          const int r = rbase + rr;
          const float v = __fmul_rn(__fmul_rn((float)(lane ? acc[1] : acc[0]), __ldg(a.out_s + r)), xs);
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
    if (ok && lane == 0 && best) atomicMax(&b.st->argmax_key, best);
  }
  mark(32 * d.n_layers + 2);
}

// Advances the step epoch after a launch of k_persist (stream order), so the
// tagged words of this step never match the next step's tags.
__global__ void k_persist_epoch(unsigned* epoch, unsigned* cnt) {
  if (threadIdx.x == 0) *epoch += 1u;
  for (int i = threadIdx.x; i < kPersistCntWords; i += blockDim.x) cnt[i] = 0u;
}

}  // namespace

bool persist_plan(const Dims& d, int num_sms, PersistPlan* pl, std::string* why) {
  auto no = [&](const char* m) {
    if (why) *why = m;
    return false;
  };
  if (d.n_experts < 2 || d.n_experts > 64 || d.top_k < 1 || d.top_k > 8)
    return no("needs a MoE model with at most 64 experts and top_k <= 8");
  if (d.group != 32) return no("needs int4 group 32");
  if (d.dim % 128 || d.hidden % 128 || d.dim > 2048) return no("needs dim, hidden multiples of 128, dim <= 2048");
  if (d.head_dim != 64 && d.head_dim != 128) return no("needs head_dim 64 or 128");
  if (d.n_heads * d.head_dim != d.dim) return no("needs n_heads * head_dim == dim");
  const int NC = num_sms;
  if (NC < 2 * d.n_heads || d.n_heads > 70) return no("needs two CTAs per head");
  const int K = d.top_k, H = d.hidden, dim = d.dim, ngd = dim / 32, ngh = H / 32;
  const int max_pairs = (int)(((long)K * H + NC - 1) / NC) + 1;
  const int max_rows = (dim + NC - 1) / NC + 1;
  const int min_gs = NC / d.n_heads;
  const int max_cols = 4 * ((d.head_dim / 4 + min_gs - 1) / min_gs);
  const int max_trows = (d.max_seq + min_gs - 1) / min_gs + 1;
  auto r128 = [](size_t b) { return (b + 127) & ~size_t(127); };
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += r128(bytes);
    return (int)o;
  };
  pl->ps_gu = ((ngd + 31) / 32) * 32 + 4;
  pl->ps_dn = ((ngh + 31) / 32) * 32 + 4;
  pl->o_xq = take(dim);
  pl->o_xf = take((size_t)dim * 4);
  pl->o_xb = take((size_t)dim * 4);
  pl->o_own = take((size_t)max_rows * 4);
  pl->o_red = take(64 * 4);
  pl->o_bars = take((3 + 2 * kLmStages) * 8);
  pl->o_xp = take((size_t)d.n_experts * sizeof(ExpertPtrs));
  const size_t p_gu = (size_t)2 * max_pairs * pl->ps_gu, p_dn = (size_t)K * max_rows * pl->ps_dn;
  pl->o_P = take(std::max(p_gu, p_dn) * 4);
  pl->o_T = take((size_t)std::max(2 * max_pairs, K * max_rows) * 4);
  pl->o_xh = take((size_t)K * H);
  pl->sqs = ((dim / 8 + 3) & ~3) + 4;
  pl->o_sq = take((size_t)8 * pl->sqs * 4);
  // the staging area, by phase: K/V slices, probabilities and products
  // (attention); router weights (routing); expert rows; lm_head ring
  pl->o_vs = (int)r128((size_t)max_trows * d.head_dim * 4);
  pl->o_pp = pl->o_vs + (int)r128((size_t)d.max_seq * max_cols * 4);
  pl->o_vt = pl->o_pp + (int)r128((size_t)d.max_seq * 4);
  pl->ets = ((d.max_seq / 8 + 3) & ~3) + 4;
  const size_t st_att = (size_t)pl->o_vt + std::max((size_t)max_cols * (kPvTile + 4), (size_t)8 * pl->ets) * 4;
  const size_t gu_bytes = (size_t)max_pairs * 2 * (dim / 2 + ngd * 4);
  const size_t dn_end = gu_bytes + (size_t)K * max_rows * (H / 2 + ngh * 4);
  const size_t hf_bytes = (size_t)K * H * 4;  // f32 h in F: over the consumed gate/up rows if they fit
  pl->o_hf = hf_bytes <= gu_bytes ? 0 : (int)r128(dn_end);
  const size_t st_exp = std::max(dn_end, (size_t)pl->o_hf + hf_bytes);
  const size_t st_rt = ((size_t)d.n_experts * (dim + 16) + 32) * 4;
  const size_t st_lm = (size_t)kLmStages * kLmChunk * dim;
  pl->o_stage = take(std::max(std::max(st_exp, st_att), std::max(st_rt, st_lm)));
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

cudaError_t launch_persist_epoch(unsigned* epoch, unsigned* cnt, cudaStream_t s) {
  k_persist_epoch<<<1, 256, 0, s>>>(epoch, cnt);
  return cudaGetLastError();
}

}  // namespace chalot
