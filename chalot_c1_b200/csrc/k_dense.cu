// k_dense.cu — int8 GEMV kernels of the decode step and the int8 operator.
//
// matmul_int8 (src/tensor/matmul.rs:47-97, 183-298): the input vector is
// quantized per call (quantize_f32_to_i8, quantization.rs:56-104), every row
// dot is an exact int32, and the row result is ((float)dot * w_scale) * x_scale.
// The decode kernels fuse the producer and consumer of that GEMV:
//   k_qkv    rmsnorm(x) -> quantize (every CTA) -> Q/K/V rows -> RoPE -> KV-cache write
//            (engine.rs:235-280)
//   k_oproj  quantize(att_out) (every CTA) -> O rows -> x += out (engine.rs:312-322)
//   k_lmhead rmsnorm(x) -> quantize -> vocab rows -> logits + argmax
//            (engine.rs:470-493, sampling.rs:34-41)
// Rows are streamed with 16-byte non-allocating loads; each warp owns a few
// rows and its lanes stride the row in 16-byte chunks (coalesced 512 B per warp
// instruction), dotting them with dp4a against the quantized vector in shared
// memory.
#include <cuda_runtime.h>

#include <algorithm>

#include "blockops.cuh"
#include "kernels.cuh"
#include "pdl.cuh"

namespace chalot {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

// Loads the 16-byte chunks lane, lane+32, ... (IT of them) of R consecutive
// int8 rows into registers (rows past n_rows or chunks past the row load 0).
template <int R, int IT>
__device__ __forceinline__ void rows_load_i8(const int8_t* __restrict__ W, int in_dim, int row0,
                                             int n_rows, uint4 (&w)[R][IT]) {
  const int lane = threadIdx.x & 31, chunks = in_dim >> 4;
#pragma unroll
  for (int i = 0; i < R; ++i)
#pragma unroll
    for (int it = 0; it < IT; ++it) {
      const int c = lane + 32 * it;
      w[i][it] = (row0 + i < n_rows && c < chunks)
                     ? ldg_stream(W + (size_t)(row0 + i) * in_dim + (size_t)c * 16)
                     : make_uint4(0, 0, 0, 0);
    }
}

// Exact int32 dots of the loaded rows with xq (shared, 16-aligned); every
// lane returns the full sums. in_dim % 16 == 0 and in_dim <= 512 * IT.
template <int R, int IT>
__device__ __forceinline__ void rows_dot_i8(const uint4 (&w)[R][IT], int in_dim, const int8_t* xq,
                                            int acc[R]) {
  const int lane = threadIdx.x & 31, chunks = in_dim >> 4;
  const uint4* xv = reinterpret_cast<const uint4*>(xq);
#pragma unroll
  for (int i = 0; i < R; ++i) acc[i] = 0;
#pragma unroll
  for (int it = 0; it < IT; ++it) {
    const int c = lane + 32 * it;
    const uint4 x = (c < chunks) ? xv[c] : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int i = 0; i < R; ++i) acc[i] = dot16_i8(w[i][it], x, acc[i]);
  }
#pragma unroll
  for (int i = 0; i < R; ++i) acc[i] = warp_sum_i(acc[i]);
}

// R consecutive rows dotted with xq for any in_dim % 16 == 0 (operator path).
template <int R>
__device__ __forceinline__ void rows_dot_i8_loop(const int8_t* __restrict__ W, int in_dim, int row0,
                                                 int n_rows, const int8_t* xq, int acc[R]) {
  const int lane = threadIdx.x & 31, chunks = in_dim >> 4;
  const uint4* xv = reinterpret_cast<const uint4*>(xq);
#pragma unroll
  for (int i = 0; i < R; ++i) acc[i] = 0;
#pragma unroll 2
  for (int c = lane; c < chunks; c += 32) {
    uint4 w[R];
#pragma unroll
    for (int i = 0; i < R; ++i)
      w[i] = (row0 + i < n_rows) ? ldg_stream(W + (size_t)(row0 + i) * in_dim + (size_t)c * 16)
                                 : make_uint4(0, 0, 0, 0);
    const uint4 x = xv[c];
#pragma unroll
    for (int i = 0; i < R; ++i) acc[i] = dot16_i8(w[i], x, acc[i]);
  }
#pragma unroll
  for (int i = 0; i < R; ++i) acc[i] = warp_sum_i(acc[i]);
}

// Copies a quantized vector (n bytes, n % 16 == 0) and its scale, produced by
// another grid, into shared memory through L2: one request per line and CTA
// (every warp reading the same lines would queue thousands of requests on a
// few L2 slices).
__device__ __forceinline__ void load_q(int8_t* dst, const int8_t* src, int n, float* xs_dst,
                                       const float* xs_src) {
  if (threadIdx.x == blockDim.x - 1) *xs_dst = __ldcg(xs_src);
  copy16(reinterpret_cast<uint4*>(dst), reinterpret_cast<const uint4*>(src), n >> 4, true);
}

// ---------------------------------------------------------------------------

// x = embedding row (engine.rs:201-210), one CTA.
__global__ void __launch_bounds__(kThreads) k_embed(Dims d, const int8_t* __restrict__ emb,
                                                    const float* __restrict__ emb_s, DecodeBufs b) {
  const uint32_t tok = b.st->token;
  const float s = emb_s[tok];
  const int8_t* row = emb + (size_t)tok * d.dim;
  for (int i = threadIdx.x; i < d.dim; i += blockDim.x) b.x[i] = __fmul_rn((float)row[i], s);
  if (threadIdx.x == 0) b.st->argmax_key = 0ull;
}

constexpr int kQkvRows = 2;  // rows per warp: one RoPE pair

template <int IT>
__global__ void __launch_bounds__(kThreads) k_qkv(Dims d, LayerPtrs L, int layer, DecodeBufs b) {
  extern __shared__ __align__(16) float qsm[];  // [dim] attention norm weights, [dim] scratch
  __shared__ __align__(16) int8_t xq[512 * IT];
  __shared__ float red[40];
  __shared__ float xs_s;
  [[maybe_unused]] const int slot = layer * 8 + 0;
  CHALOT_TRACE(slot, 0);
  const int warp = threadIdx.x >> 5;
  const int r0 = (blockIdx.x * kWarps + warp) * kQkvRows;
  const int n_rows = 3 * d.dim;
  uint4 w[kQkvRows][IT];
  rows_load_i8<kQkvRows, IT>(L.qkv, d.dim, r0, n_rows, w);  // weights do not depend on the token
  // scales, position and rotation of this row pair: known before the token's x
  const int sec = r0 / d.dim, rr = r0 - sec * d.dim;
  const uint32_t pos = b.st->pos;
  float s0 = 0.0f, s1 = 0.0f, c = 1.0f, sn = 0.0f;
  if (r0 < n_rows && (threadIdx.x & 31) == 0) {
    s0 = L.qkv_s[r0];
    s1 = L.qkv_s[r0 + 1];
    if (sec < 2) {
      const int half = d.head_dim >> 1, i = (rr % d.head_dim) >> 1;
      c = b.rope_cos[pos * half + i];
      sn = b.rope_sin[pos * half + i];
    }
  }
  load_f32(qsm, L.rms_attn, d.dim);
  CHALOT_TRACE(slot, 1);
  pdl_wait();
  pdl_trigger();
  CHALOT_TRACE(slot, 2);
  // rmsnorm(x, rms_attn) then quantize_f32_to_i8 (engine.rs:230-236), by every
  // CTA from the x the previous layer's down kernel left in L2
  norm_quant_tail(b.x, qsm, d.dim, xq, &xs_s, qsm + d.dim, red);
  __syncthreads();
  CHALOT_TRACE(slot, 3);
  if (r0 >= n_rows) return;
  const float xs = xs_s;
  int acc[kQkvRows];
  rows_dot_i8<kQkvRows, IT>(w, d.dim, xq, acc);
  if ((threadIdx.x & 31) != 0) return;
  float v0 = __fmul_rn(__fmul_rn((float)acc[0], s0), xs);
  float v1 = __fmul_rn(__fmul_rn((float)acc[1], s1), xs);
  if (sec < 2) {  // RoPE on the interleaved pair (engine.rs:252-271)
    const float s = sn;
    const float a = __fsub_rn(__fmul_rn(v0, c), __fmul_rn(v1, s));
    const float e = __fadd_rn(__fmul_rn(v0, s), __fmul_rn(v1, c));
    v0 = a;
    v1 = e;
  }
  if (sec == 0) {
    b.q[rr] = v0;
    b.q[rr + 1] = v1;
  } else {
    float* cache = (sec == 1) ? b.kc : b.vc;  // engine.rs:274-280
    const size_t off = ((size_t)layer * d.max_seq + pos) * d.dim + rr;
    cache[off] = v0;
    cache[off + 1] = v1;
  }
}

constexpr int kORows = 2;

// O rows + residual; the last CTA then runs the FFN prologue of the layer
// once for every later kernel: xb = rmsnorm(x, rms_ffn), xq_ffn/xs_ffn =
// quantize(xb), router logits and softmax_top_k -> sel/selw (engine.rs:325-344).
template <int IT>
__global__ void __launch_bounds__(kThreads) k_oproj(Dims d, LayerPtrs L, int layer, DecodeBufs b) {
  extern __shared__ __align__(16) float osm[];  // tail scratch: xb, wbuf [dim] each, lanes [16E], logit [E]
  __shared__ __align__(16) int8_t xq[512 * IT];
  __shared__ float red[40];
  [[maybe_unused]] const int slot = layer * 8 + 3;
  CHALOT_TRACE(slot, 0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = (blockIdx.x * kWarps + warp) * kORows;
  const int E = d.n_experts;
  float* xb = osm;
  float* wbuf = osm + d.dim;
  float* lanes = wbuf + d.dim;
  float* logit = lanes + 16 * E;
  float* rbias = logit + 32;
  float* rw = rbias + 32;  // [E][dim] router weights
  uint4 w[kORows][IT];
  rows_load_i8<kORows, IT>(L.o, d.dim, r0, d.dim, w);
  // whichever CTA finishes last runs the FFN prologue: every CTA stages its
  // static inputs (norm weights, router weights and bias) before waiting
  load_f32(wbuf, L.rms_ffn, d.dim);
  if (E >= 2) {
    load_f32(rw, L.router_w, E * d.dim);
    if (threadIdx.x < E) rbias[threadIdx.x] = L.router_b[threadIdx.x];
  }
  CHALOT_TRACE(slot, 1);
  pdl_wait();
  pdl_trigger();
  CHALOT_TRACE(slot, 2);
  // quantize_f32_to_i8 of the attention output (engine.rs:312-314), by every
  // CTA from the f32 values the attention kernel left in L2
  __shared__ float xs_s;
  load_f32_cg(xb, b.att_out, d.dim);
  __syncthreads();
  {
    float scale, qinv;
    quant_scale(absmax_smem(xb, d.dim, red), &scale, &qinv);
    for (int i = threadIdx.x; i < d.dim; i += blockDim.x) xq[i] = quant_any(xb[i], qinv, i, d.dim);
    if (threadIdx.x == 0) xs_s = scale;
  }
  __syncthreads();
  CHALOT_TRACE(slot, 3);
  if (r0 < d.dim) {
    const float xs = xs_s;
    int acc[kORows];
    rows_dot_i8<kORows, IT>(w, d.dim, xq, acc);
    if (lane < kORows && r0 + lane < d.dim) {
      const int r = r0 + lane;
      int dot = acc[0];
#pragma unroll
      for (int i = 1; i < kORows; ++i) dot = (lane == i) ? acc[i] : dot;
      const float v = __fmul_rn(__fmul_rn((float)dot, L.o_s[r]), xs);
      b.x[r] = __fadd_rn(__ldcg(b.x + r), v);  // residual (engine.rs:320-322)
    }
  }
  CHALOT_TRACE(slot, 4);
  const bool tail = last_cta(b.counters + 1);
  CHALOT_TRACE(slot, 5);
  if (!tail) return;
  [[maybe_unused]] const int tslot = layer * 8 + 6;
  CHALOT_TRACE(tslot, 0);
  norm_quant_tail(b.x, wbuf, d.dim, b.xq_ffn, b.xs_ffn, xb, red);
  CHALOT_TRACE(tslot, 2);
  if (E >= 2) {
    router_logits(rw, rbias, xb, d.dim, E, lanes, logit);
    CHALOT_TRACE(tslot, 3);
    if (threadIdx.x < 32) topk_warp(logit, E, d.top_k, b.sel, b.selw);
    CHALOT_TRACE(tslot, 4);
    if (b.router_trace)
      for (int e = threadIdx.x; e < E; e += blockDim.x) b.router_trace[layer * E + e] = logit[e];
  } else if (threadIdx.x == 0) {
    b.sel[0] = 0;
    b.selw[0] = 1.0f;
  }
  CHALOT_TRACE(slot, 6);
}

constexpr int kLmRows = 4;

template <int IT>
__global__ void __launch_bounds__(kThreads) k_lmhead(Dims d, const int8_t* __restrict__ W,
                                                     const float* __restrict__ ws, DecodeBufs b) {
  __shared__ __align__(16) int8_t xq[512 * IT];
  __shared__ unsigned long long best_w[kWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int step = gridDim.x * kWarps * kLmRows;
  int r0 = (blockIdx.x * kWarps + warp) * kLmRows;
  uint4 w[kLmRows][IT];
  rows_load_i8<kLmRows, IT>(W, d.dim, r0, d.vocab, w);
  pdl_wait();
  pdl_trigger();
  __shared__ float xs_s;
  load_q(xq, b.xq_attn, d.dim, &xs_s, b.xs_attn);  // rmsnorm(x, final_norm) quantized by the last down kernel
  __syncthreads();
  const float xs = xs_s;
  unsigned long long best = 0ull;
  for (; r0 < d.vocab; r0 += step) {
    int acc[kLmRows];
    rows_dot_i8<kLmRows, IT>(w, d.dim, xq, acc);
    if (r0 + step < d.vocab) rows_load_i8<kLmRows, IT>(W, d.dim, r0 + step, d.vocab, w);
#pragma unroll
    for (int i = 0; i < kLmRows; ++i) {
      const int r = r0 + i;
      if (lane == i && r < d.vocab) {
        const float v = __fmul_rn(__fmul_rn((float)acc[i], ws[r]), xs);
        b.logits[r] = v;
        const unsigned long long key = ((unsigned long long)ordered_key(v) << 32) | (unsigned)r;
        best = key > best ? key : best;
      }
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  if (lane == 0) best_w[warp] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long m = 0ull;
    for (int i = 0; i < kWarps; ++i) m = best_w[i] > m ? best_w[i] : m;
    atomicMax(&b.st->argmax_key, m);
  }
}

// Records the forward's argmax and picks the next token (engine.rs:509-545):
// during prefill the next prompt token clamped to vocab-1, then the argmax.
__global__ void k_advance(Dims d, DecodeBufs b) {
  pdl_wait();
  StepState* st = b.st;
  const uint32_t idx = (uint32_t)(st->argmax_key & 0xffffffffull);
  const uint32_t step = st->step;
  b.out_tokens[step] = idx;
  const uint32_t next_pos = st->pos + 1;
  uint32_t next = idx;
  if (next_pos < st->n_prefill) next = min(b.prompt[next_pos], (uint32_t)(d.vocab - 1));
  st->pos = next_pos;
  st->token = next;
  st->step = step + 1;
}

// apply_repetition_penalty (src/tensor/sampling.rs:168-178) over hist[0..n),
// sequentially so that repeated tokens are penalised repeatedly.
__global__ void k_penalty(Dims d, DecodeBufs b, const uint32_t* __restrict__ hist, int n,
                          float p) {
  if (threadIdx.x == 0) {
    for (int i = 0; i < n; ++i) {
      const uint32_t t = hist[i];
      if (t < (uint32_t)d.vocab) {
        const float v = b.logits[t];
        b.logits[t] = (v > 0.0f) ? div_rn(v, p) : __fmul_rn(v, p);
      }
    }
    b.st->argmax_key = 0ull;
  }
}

__global__ void __launch_bounds__(kThreads) k_argmax(const float* __restrict__ v, int n,
                                                     unsigned long long* key_out) {
  __shared__ unsigned long long best_w[kWarps];
  unsigned long long best = 0ull;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const unsigned long long k = ((unsigned long long)ordered_key(v[i]) << 32) | (unsigned)i;
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  if ((threadIdx.x & 31) == 0) best_w[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long m = 0ull;
    for (int i = 0; i < kWarps; ++i) m = best_w[i] > m ? best_w[i] : m;
    atomicMax(key_out, m);
  }
}

// ---- operator: matmul_int8 over caller-owned device memory ---------------------
// Each CTA quantizes x into shared memory itself (the quantization depends only
// on x), then streams rows. Rows with in_dim % 16 != 0 or unaligned weights
// take a byte-wise path with the same exact int32 result.
__global__ void __launch_bounds__(kThreads) k_matmul_i8_op(float* __restrict__ out,
                                                           const int8_t* __restrict__ W,
                                                           const float* __restrict__ ws,
                                                           const float* __restrict__ x,
                                                           int out_dim, int in_dim, int vec) {
  extern __shared__ __align__(16) unsigned char smem[];
  int8_t* xq = reinterpret_cast<int8_t*>(smem);
  __shared__ float red[40];
  float m = 0.0f;
  for (int i = threadIdx.x; i < in_dim; i += blockDim.x) m = fmaxf(m, fabsf(x[i]));
  m = block_max(m, red);
  float xs, inv;
  quant_scale(m, &xs, &inv);
  for (int i = threadIdx.x; i < in_dim; i += blockDim.x) xq[i] = quant_any(x[i], inv, i, in_dim);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int step = gridDim.x * kWarps * 2;
  for (int r0 = (blockIdx.x * kWarps + warp) * 2; r0 < out_dim; r0 += step) {
    int acc[2];
    if (vec) {
      rows_dot_i8_loop<2>(W, in_dim, r0, out_dim, xq, acc);
    } else {
      for (int i = 0; i < 2; ++i) {
        int a = 0;
        if (r0 + i < out_dim)
          for (int k = lane; k < in_dim; k += 32) a += (int)W[(size_t)(r0 + i) * in_dim + k] * (int)xq[k];
        acc[i] = warp_sum_i(a);
      }
    }
    if (lane < 2 && r0 + lane < out_dim) {
      const int r = r0 + lane;
      out[r] = __fmul_rn(__fmul_rn((float)(lane ? acc[1] : acc[0]), ws[r]), xs);
    }
  }
}

__global__ void __launch_bounds__(kThreads) k_quantize_op(int8_t* __restrict__ q, float* scale,
                                                          const float* __restrict__ x, int n) {
  __shared__ float red[40];
  const float* v = x + (size_t)blockIdx.x * n;
  float m = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, fabsf(v[i]));
  m = block_max(m, red);
  float s, inv;
  quant_scale(m, &s, &inv);
  for (int i = threadIdx.x; i < n; i += blockDim.x) q[(size_t)blockIdx.x * n + i] = quant_any(v[i], inv, i, n);
  if (threadIdx.x == 0) scale[blockIdx.x] = s;
}

}  // namespace

// in_dim of the dense projections is at most 4096: 16-byte chunks per lane
static int dense_it(int dim) { return (dim + 511) / 512; }

void launch_embed(const Dims& d, const int8_t* emb, const float* emb_s, const DecodeBufs& b,
                  cudaStream_t s) {
  launch_k(k_embed, dim3(1), dim3(kThreads), 0, s, false, d, emb, emb_s, b);
}

#define CHALOT_IT_SWITCH(it, CALL) \
  switch (it) {                    \
    case 1: CALL(1); break;        \
    case 2: CALL(2); break;        \
    case 3: CALL(3); break;        \
    case 4: CALL(4); break;        \
    case 5: CALL(5); break;        \
    case 6: CALL(6); break;        \
    case 7: CALL(7); break;        \
    default: CALL(8); break;       \
  }

void launch_qkv(const Dims& d, const LayerPtrs& L, int layer, const DecodeBufs& b, cudaStream_t s,
                bool pdl) {
  const int rows_per_block = kWarps * kQkvRows;
  const int grid = (3 * d.dim + rows_per_block - 1) / rows_per_block;
#define QKV_CALL(IT) \
  launch_k(k_qkv<IT>, dim3(grid), dim3(kThreads), (size_t)d.dim * 8, s, pdl, d, L, layer, b)
  CHALOT_IT_SWITCH(dense_it(d.dim), QKV_CALL)
#undef QKV_CALL
}

void launch_oproj(const Dims& d, const LayerPtrs& L, int layer, const DecodeBufs& b,
                  cudaStream_t s, bool pdl) {
  const int rows_per_block = kWarps * kORows;
  const int grid = (d.dim + rows_per_block - 1) / rows_per_block;
  const size_t E = d.n_experts;
  const size_t smem = ((size_t)d.dim * 2 + 16 * E + 64 + E * d.dim) * 4;
#define O_CALL(IT)                                                                           \
  do {                                                                                      \
    if (smem > 48 * 1024)                                                                   \
      cudaFuncSetAttribute(k_oproj<IT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    launch_k(k_oproj<IT>, dim3(grid), dim3(kThreads), smem, s, pdl, d, L, layer, b);        \
  } while (0)
  CHALOT_IT_SWITCH(dense_it(d.dim), O_CALL)
#undef O_CALL
}

void launch_lmhead(const Dims& d, const int8_t* w, const float* ws, const DecodeBufs& b,
                   int num_sms, cudaStream_t s, bool pdl) {
  const int rows_per_block = kWarps * kLmRows;
  const int grid = std::min((d.vocab + rows_per_block - 1) / rows_per_block, num_sms * 4);
#define LM_CALL(IT) launch_k(k_lmhead<IT>, dim3(grid), dim3(kThreads), 0, s, pdl, d, w, ws, b)
  CHALOT_IT_SWITCH(dense_it(d.dim), LM_CALL)
#undef LM_CALL
}

void launch_advance(const Dims& d, const DecodeBufs& b, cudaStream_t s, bool pdl) {
  launch_k(k_advance, dim3(1), dim3(1), 0, s, pdl, d, b);
}

void launch_penalty_argmax(const Dims& d, const DecodeBufs& b, const uint32_t* hist, int n_hist,
                           float penalty, cudaStream_t s) {
  k_penalty<<<1, 32, 0, s>>>(d, b, hist, n_hist, penalty);
  k_argmax<<<std::min(148, (d.vocab + kThreads - 1) / kThreads), kThreads, 0, s>>>(
      b.logits, d.vocab, &b.st->argmax_key);
}

cudaError_t launch_argmax_op(const float* logits, int V, unsigned long long* out, cudaStream_t s) {
  k_argmax<<<std::min(148, (V + kThreads - 1) / kThreads), kThreads, 0, s>>>(logits, V, out);
  return cudaGetLastError();
}

cudaError_t op_matmul_i8(float* out, const int8_t* w, const float* ws, const float* x,
                         size_t out_dim, size_t in_dim, int num_sms, cudaStream_t s) {
  const int vec = (in_dim % 16 == 0) && ((reinterpret_cast<uintptr_t>(w) & 15) == 0);
  const size_t smem = (in_dim + 15) & ~size_t(15);
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(k_matmul_i8_op, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int rows_per_block = kWarps * 2;
  const int grid = (int)std::min<size_t>((out_dim + rows_per_block - 1) / rows_per_block,
                                         (size_t)num_sms * 4);
  k_matmul_i8_op<<<std::max(grid, 1), kThreads, smem, s>>>(out, w, ws, x, (int)out_dim,
                                                            (int)in_dim, vec);
  return cudaGetLastError();
}

cudaError_t op_quantize_i8(int8_t* q, float* scale, const float* x, size_t n_vec, size_t n,
                           cudaStream_t s) {
  k_quantize_op<<<(unsigned)n_vec, kThreads, 0, s>>>(q, scale, x, (int)n);
  return cudaGetLastError();
}

#ifdef CHALOT_PHASE_TRACE
CHALOT_TRACE_EXPORT(trace_dense)
#endif

}  // namespace chalot
