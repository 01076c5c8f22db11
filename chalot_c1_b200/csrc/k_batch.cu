// k_batch.cu — batched decode: one forward of B sequences at once, each at
// its own position with its own f32 KV cache slot. Per token the arithmetic is
// Engine::forward's (src/model/engine.rs:173-494) in the reference's rounding
// order, so every sequence decodes exactly as it would alone:
//   k_b_embed       embedding row * scale, rmsnorm, quantize (engine.rs:201-210)
//   k_b_norm_quant  rmsnorm + quantize of each token's residual
//   k_b_gemm_i8     int8 GEMM for B tokens: exact int32 dots (dp4a over shared
//                   tiles of 32 tokens x 32 or 128 rows), then (dot*ws)*xs; stores,
//                   or adds to the residual (matmul.rs:183-298, engine.rs:320-322)
//   k_b_rope_kv     RoPE on q and k, K/V rows into the sequence's cache slot
//   k_b_scores      s[b][h][t] = 30*tanh((dot_f32(q, k_t)/sqrt(hd))/30)
//   k_b_pv          softmax in the AVX2 order, then sum_t p_t v_t in t order
//   k_b_rmsnorm     the FFN input rows (the MoE layer quantizes them itself)
//   k_b_add         x += expert_out
//   k_b_argmax      argmax of each token's logits, ties to the last index
// The MoE block between k_b_rmsnorm and k_b_add is the batched MoE layer
// (k_moe_layer.cu / k_moe_tc.cu) on the engine's repacked expert weights.
// KV cache: [slot][layer][max_seq][dim] f32.
#include <cuda_runtime.h>

#include "batch.h"
#include "blockops.cuh"

namespace chalot {
namespace {

constexpr int kT = 256;

// Offset (in floats) of the K or V row of position t of a slot in layer `layer`.
__device__ __forceinline__ size_t kv_off(const BatchDims& d, int slot, int layer, int t) {
  if (!d.ptab) return (((size_t)slot * d.n_layers + layer) * d.max_seq + t) * d.dim;
  const size_t page = (size_t)d.ptab[(size_t)slot * d.maxp + (t >> d.pt_shift)];
  return (((page * d.n_layers + layer) << d.pt_shift) + (size_t)(t & ((1 << d.pt_shift) - 1))) * d.dim;
}

__global__ void __launch_bounds__(kT) k_b_embed(int dim, const uint32_t* toks, const int8_t* __restrict__ emb,
                                                const float* __restrict__ emb_s, const float* __restrict__ rms0,
                                                float* x, int8_t* xq, float* xs) {
  extern __shared__ __align__(16) float esm[];  // [dim] norm weights, [dim] scratch
  __shared__ float red[40];
  const int b = blockIdx.x;
  load_f32(esm, rms0, dim);
  const uint32_t tok = toks[b];
  const float s = emb_s[tok];
  const int8_t* row = emb + (size_t)tok * dim;
  float* xr = x + (size_t)b * dim;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) xr[i] = __fmul_rn((float)row[i], s);
  __syncthreads();
  norm_quant_tail(xr, esm, dim, xq + (size_t)b * dim, xs + b, esm + dim, red);
}

__global__ void __launch_bounds__(kT) k_b_norm_quant(int dim, const float* x, const float* __restrict__ w, int8_t* xq,
                                                     float* xs) {
  extern __shared__ __align__(16) float esm[];
  __shared__ float red[40];
  const int b = blockIdx.x;
  load_f32(esm, w, dim);
  __syncthreads();
  norm_quant_tail(x + (size_t)b * dim, esm, dim, xq + (size_t)b * dim, xs + b, esm + dim, red);
}

constexpr int kGT = 32, kGK = 256, kGWS = kGK + 16;

// out[t][r] (=|+=) ((float)dot(W[r], xq[t]) * ws[r]) * xs[t] for t < B, r < R.
// Tiles of 32 tokens x 32*RPL rows; thread (warp v, lane l): tokens 4v..4v+3,
// rows l, l+32, ... (RPL of them).
template <bool ADD, int RPL>
__global__ void __launch_bounds__(kT) k_b_gemm_i8(int B, int R, int C, const int8_t* __restrict__ W,
                                                  const float* __restrict__ ws, const int8_t* __restrict__ xq,
                                                  const float* __restrict__ xs, float* out, int ldo) {
  constexpr int GR = 32 * RPL;
  __shared__ __align__(16) int8_t X[kGT * kGK];
  __shared__ __align__(16) int8_t Wt[GR * kGWS];
  const int r0 = blockIdx.x * GR, t0 = blockIdx.y * kGT;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int acc[4][RPL];
#pragma unroll
  for (int s = 0; s < 4; ++s)
#pragma unroll
    for (int i = 0; i < RPL; ++i) acc[s][i] = 0;
  for (int k0 = 0; k0 < C; k0 += kGK) {
    const int kc = min(kGK, C - k0), ch = kc >> 4;
    __syncthreads();
    for (int c = tid; c < kGT * ch; c += kT) {
      const int s = c / ch, j = c - s * ch;
      *reinterpret_cast<uint4*>(X + s * kGK + j * 16) =
          t0 + s < B ? __ldg(reinterpret_cast<const uint4*>(xq + (size_t)(t0 + s) * C + k0 + j * 16))
                     : make_uint4(0, 0, 0, 0);
    }
    for (int c = tid; c < GR * ch; c += kT) {
      const int r = c / ch, j = c - r * ch;
      *reinterpret_cast<uint4*>(Wt + r * kGWS + j * 16) =
          r0 + r < R ? ldg_stream(W + (size_t)(r0 + r) * C + k0 + j * 16) : make_uint4(0, 0, 0, 0);
    }
    __syncthreads();
    for (int q = 0; q < ch; ++q) {
      uint4 xv[4], wv[RPL];
#pragma unroll
      for (int s = 0; s < 4; ++s) xv[s] = lds16(X + (warp * 4 + s) * kGK + q * 16);
#pragma unroll
      for (int i = 0; i < RPL; ++i) wv[i] = lds16(Wt + (lane + 32 * i) * kGWS + q * 16);
#pragma unroll
      for (int s = 0; s < 4; ++s)
#pragma unroll
        for (int i = 0; i < RPL; ++i) {
          int t = acc[s][i];
          t = __dp4a((int)wv[i].x, (int)xv[s].x, t);
          t = __dp4a((int)wv[i].y, (int)xv[s].y, t);
          t = __dp4a((int)wv[i].z, (int)xv[s].z, t);
          t = __dp4a((int)wv[i].w, (int)xv[s].w, t);
          acc[s][i] = t;
        }
    }
  }
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    const int tok = t0 + warp * 4 + s;
    if (tok >= B) continue;
    const float xsc = xs[tok];
#pragma unroll
    for (int i = 0; i < RPL; ++i) {
      const int r = r0 + lane + 32 * i;
      if (r >= R) continue;
      const float v = __fmul_rn(__fmul_rn(__int2float_rn(acc[s][i]), ws[r]), xsc);
      float* o = out + (size_t)tok * ldo + r;
      *o = ADD ? __fadd_rn(*o, v) : v;
    }
  }
}

// One thread per (token, row pair) of the QKV output: RoPE on the interleaved
// pairs of q and k (engine.rs:252-271), then q to `q`, k and v into the cache.
__global__ void k_b_rope_kv(BatchDims d, int layer, int B, const int32_t* pos, const int32_t* slot,
                            const float* __restrict__ qkv, float* q, float* kc, float* vc,
                            const float* __restrict__ rcos, const float* __restrict__ rsin) {
  const int pairs = 3 * d.dim / 2;
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)B * pairs) return;
  const int b = (int)(idx / pairs), r = 2 * (int)(idx % pairs);
  const int sec = r / d.dim, rr = r - sec * d.dim;
  const int p = pos[b];
  float v0 = qkv[(size_t)b * 3 * d.dim + r], v1 = qkv[(size_t)b * 3 * d.dim + r + 1];
  if (sec < 2) {
    const int half = d.head_dim >> 1, i = (rr % d.head_dim) >> 1;
    const float c = rcos[(size_t)p * half + i], s = rsin[(size_t)p * half + i];
    const float a = __fsub_rn(__fmul_rn(v0, c), __fmul_rn(v1, s));
    const float e = __fadd_rn(__fmul_rn(v0, s), __fmul_rn(v1, c));
    v0 = a;
    v1 = e;
  }
  if (sec == 0) {
    q[(size_t)b * d.dim + rr] = v0;
    q[(size_t)b * d.dim + rr + 1] = v1;
  } else {
    float* cache = sec == 1 ? kc : vc;
    const size_t off = kv_off(d, slot[b], layer, p) + rr;
    cache[off] = v0;
    cache[off + 1] = v1;
  }
}

constexpr int kScoreT = 128;

template <int C16>
__global__ void __launch_bounds__(kScoreT) k_b_scores(BatchDims d, int layer, const int32_t* pos,
                                                      const int32_t* slot, const float* q, const float* kc,
                                                      float* scores) {
  __shared__ __align__(16) float qh[256];
  const int b = blockIdx.z, h = blockIdx.y, hd = d.head_dim;
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  const int P = pos[b];
  if ((int)(blockIdx.x * blockDim.x) > P) return;
  for (int i = threadIdx.x; i < hd; i += blockDim.x) qh[i] = q[(size_t)b * d.dim + h * hd + i];
  __syncthreads();
  if (t > P) return;
  const float* k = kc + kv_off(d, slot[b], layer, t) + (size_t)h * hd;
  float a0[8], a1[8];  // dot_f32_avx2: two 8-lane accumulators over 16-element strides
#pragma unroll
  for (int j = 0; j < 8; ++j) a0[j] = a1[j] = 0.0f;
#pragma unroll
  for (int c = 0; c < C16; ++c) {
    const float4* kk = reinterpret_cast<const float4*>(k + c * 16);
    const float4 k0 = kk[0], k1 = kk[1], k2 = kk[2], k3 = kk[3];
    const float kv[16] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w,
                          k2.x, k2.y, k2.z, k2.w, k3.x, k3.y, k3.z, k3.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      a0[j] = __fadd_rn(a0[j], __fmul_rn(qh[c * 16 + j], kv[j]));
      a1[j] = __fadd_rn(a1[j], __fmul_rn(qh[c * 16 + 8 + j], kv[8 + j]));
    }
  }
  const int rem = C16 * 16;
  if (rem + 8 <= hd)  // head_dim % 16 == 8: one more 8-chunk into acc0
#pragma unroll
    for (int j = 0; j < 8; ++j) a0[j] = __fadd_rn(a0[j], __fmul_rn(qh[rem + j], k[rem + j]));
  float cmb[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) cmb[j] = __fadd_rn(a0[j], a1[j]);
  const float dot = hsum8(cmb);
  const float x = __fmul_rn(dot, div_rn(1.0f, __fsqrt_rn((float)hd)));
  scores[((size_t)b * d.n_heads + h) * d.max_seq + t] = __fmul_rn(30.0f, libm::tanh_f32(div_rn(x, 30.0f)));
}

constexpr int kPvCols = 8, kPvTile = 1024;

__device__ __forceinline__ void b_stage_v(float* vt, const float* vc, const BatchDims& d, int slot, int layer,
                                          int col0, int t0, int rows) {
  const int n = rows * (kPvCols / 4);
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int r = i / (kPvCols / 4), qq = i % (kPvCols / 4);
    reinterpret_cast<float4*>(vt)[i] =
        *reinterpret_cast<const float4*>(vc + kv_off(d, slot, layer, t0 + r) + col0 + qq * 4);
  }
}

// CTA (head, 8 columns, token): softmax_avx2 over s[0..pos] then the t-ordered sums.
__global__ void __launch_bounds__(kT) k_b_pv(BatchDims d, int layer, const int32_t* pos, const int32_t* slot,
                                             const float* scores, const float* vc, float* att) {
  extern __shared__ __align__(16) float sm[];
  float* p = sm;
  float* vt = sm + ((d.max_seq + 3) & ~3);
  __shared__ float red[40];
  __shared__ float inv_s;
  const int h = blockIdx.x, hd = d.head_dim, c0 = blockIdx.y * kPvCols, b = blockIdx.z;
  const int n = pos[b] + 1;
  const float* s = scores + ((size_t)b * d.n_heads + h) * d.max_seq;
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = s[i];
    p[i] = v;
    mx = fmaxf(mx, v);
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
    for (int c = 0; c < (full >> 3); ++c) acc = __fadd_rn(acc, p[c * 8 + threadIdx.x]);
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
  float acc = 0.0f;
  for (int t0 = 0; t0 < n; t0 += kPvTile) {
    const int rows = min(kPvTile, n - t0);
    __syncthreads();
    b_stage_v(vt, vc, d, slot[b], layer, h * hd + c0, t0, rows);
    __syncthreads();
    if (threadIdx.x < kPvCols)
      for (int t = 0; t < rows; ++t) acc = __fadd_rn(acc, __fmul_rn(p[t0 + t], vt[t * kPvCols + threadIdx.x]));
  }
  if (threadIdx.x < kPvCols) att[(size_t)b * d.dim + h * hd + c0 + threadIdx.x] = acc;
}

constexpr int kAttT = 128;  // threads of the fused attention CTA (head_dim <= 128)
constexpr int kAttU = 16;   // V rows in flight per thread

// CTA (head h, token b): the scores of positions 0..pos (four lanes per
// position: dot_f32_avx2 order, then 30*tanh(x/30)), softmax_avx2 over them
// in shared memory, then o[c] = sum_t p_t v_t[c] in t order (thread c), with
// kAttU V rows loaded ahead. One pass over this head's K and V, and the
// softmax once per head instead of once per 8 output columns.
template <int C16>
__global__ void __launch_bounds__(kAttT, 4) k_b_attn(BatchDims d, int layer, const int32_t* pos, const int32_t* slot,
                                                  const float* q, const float* kc, const float* vc, float* att) {
  extern __shared__ __align__(16) float p[];  // [max_seq] scores, then probabilities
  __shared__ __align__(16) float qh[256];
  __shared__ float red[40];
  __shared__ float inv_s;
  const int h = blockIdx.x, b = blockIdx.y, hd = d.head_dim;
  const int n = pos[b] + 1;
  const int sl = slot[b];
  for (int i = threadIdx.x; i < hd; i += blockDim.x) qh[i] = q[(size_t)b * d.dim + h * hd + i];
  __syncthreads();
  const float rs = div_rn(1.0f, __fsqrt_rn((float)hd));
  // scores: four lanes per position, lane l4 owning elements 4*l4..4*l4+3 of
  // every 16-element chunk, i.e. the dot_f32_avx2 accumulators a0[0..3]
  // (l4 = 0), a0[4..7] (1), a1[0..3] (2), a1[4..7] (3), each summed in chunk
  // order; the lanes then combine them as the reference does (a0 + a1, then
  // hsum8). A quad reads 64 contiguous bytes of its K row per chunk.
  const int lane = threadIdx.x & 31, quad = lane >> 2, l4 = lane & 3;
  const int warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  float qv[C16][4];
#pragma unroll
  for (int c = 0; c < C16; ++c)
#pragma unroll
    for (int u = 0; u < 4; ++u) qv[c][u] = qh[16 * c + 4 * l4 + u];
  float mx = -INFINITY;
  for (int t0 = warp * 8; t0 < n; t0 += nwarps * 8) {
    const int t = t0 + quad;
    float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (t < n) {
      const float* k = kc + kv_off(d, sl, layer, t) + (size_t)h * hd + 4 * l4;
      float4 kv[C16];
#pragma unroll
      for (int c = 0; c < C16; ++c) kv[c] = *reinterpret_cast<const float4*>(k + 16 * c);
#pragma unroll
      for (int c = 0; c < C16; ++c) {
        a[0] = __fadd_rn(a[0], __fmul_rn(qv[c][0], kv[c].x));
        a[1] = __fadd_rn(a[1], __fmul_rn(qv[c][1], kv[c].y));
        a[2] = __fadd_rn(a[2], __fmul_rn(qv[c][2], kv[c].z));
        a[3] = __fadd_rn(a[3], __fmul_rn(qv[c][3], kv[c].w));
      }
    }
    float cmb[4], hi[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) cmb[u] = __fadd_rn(a[u], __shfl_xor_sync(0xffffffffu, a[u], 2));  // a0 + a1
#pragma unroll
    for (int u = 0; u < 4; ++u) hi[u] = __shfl_xor_sync(0xffffffffu, cmb[u], 1);  // cmb[4..7] to l4 = 0
    if (l4 == 0 && t < n) {
      const float t0s = __fadd_rn(cmb[0], hi[0]), t1s = __fadd_rn(cmb[1], hi[1]);
      const float t2s = __fadd_rn(cmb[2], hi[2]), t3s = __fadd_rn(cmb[3], hi[3]);
      const float x = __fmul_rn(__fadd_rn(__fadd_rn(t0s, t2s), __fadd_rn(t1s, t3s)), rs);
      const float sc = __fmul_rn(30.0f, libm::tanh_f32(div_rn(x, 30.0f)));
      p[t] = sc;
      mx = fmaxf(mx, sc);
    }
  }
  mx = block_max(mx, red);  // its barriers also publish p[]
  const int full = n & ~7;
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    p[i] = i < full ? fast_exp(__fsub_rn(p[i], mx)) : expf_cr(__fsub_rn(p[i], mx));
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
    inv_s = div_rn(1.0f, sum);
  }
  __syncthreads();
  const float inv = inv_s;
  for (int i = threadIdx.x; i < n; i += blockDim.x) p[i] = __fmul_rn(p[i], inv);
  __syncthreads();
  if (threadIdx.x >= hd) return;
  const float* v = vc + (size_t)h * hd + threadIdx.x;
  // the rows of positions u..u+kAttU-1 (u a multiple of kAttU) are consecutive:
  // in the flat cache, and in one page (pages hold a multiple of kAttU positions)
  auto vblk = [&](int u) { return v + kv_off(d, sl, layer, u); };
  const size_t ld = d.dim;
  float acc = 0.0f, cur[kAttU], nxt[kAttU];
  const int nb = n / kAttU;
  if (nb > 0) {
    const float* vb = vblk(0);
#pragma unroll
    for (int u = 0; u < kAttU; ++u) cur[u] = vb[(size_t)u * ld];
  }
  for (int i = 0; i < nb; ++i) {
    const int t = i * kAttU;
    if (i + 1 < nb) {
      const float* vb = vblk(t + kAttU);
#pragma unroll
      for (int u = 0; u < kAttU; ++u) nxt[u] = vb[(size_t)u * ld];
    }
#pragma unroll
    for (int u = 0; u < kAttU; ++u) acc = __fadd_rn(acc, __fmul_rn(p[t + u], cur[u]));
#pragma unroll
    for (int u = 0; u < kAttU; ++u) cur[u] = nxt[u];
  }
  for (int t = nb * kAttU; t < n; ++t) acc = __fadd_rn(acc, __fmul_rn(p[t], v[kv_off(d, sl, layer, t)]));
  att[(size_t)b * d.dim + h * hd + threadIdx.x] = acc;
}

__global__ void __launch_bounds__(kT) k_b_rmsnorm(int dim, const float* x, const float* __restrict__ w, float* xb) {
  extern __shared__ __align__(16) float esm[];  // xb [dim], wbuf [dim]
  __shared__ float red[40];
  const int b = blockIdx.x;
  rmsnorm_smem(x + (size_t)b * dim, w, dim, esm, esm + dim, red, true);
  for (int i = threadIdx.x; i < dim; i += blockDim.x) xb[(size_t)b * dim + i] = esm[i];
}

__global__ void k_b_add(long n, float* x, const float* y) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    x[i] = __fadd_rn(x[i], y[i]);
}

// argmax of each token's logits; ties go to the last index (sampling.rs:34-41).
__global__ void __launch_bounds__(kT) k_b_argmax(int V, const float* logits, uint32_t* out) {
  __shared__ unsigned long long best[kT / 32];
  const int b = blockIdx.x;
  const float* l = logits + (size_t)b * V;
  unsigned long long m = 0;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const unsigned long long k = ((unsigned long long)ordered_key(l[i]) << 32) | (unsigned)i;
    m = k > m ? k : m;
  }
  for (int o = 16; o; o >>= 1) {
    const unsigned long long v = __shfl_xor_sync(0xffffffffu, m, o);
    m = v > m ? v : m;
  }
  if ((threadIdx.x & 31) == 0) best[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long r = 0;
    for (int w = 0; w < kT / 32; ++w) r = best[w] > r ? best[w] : r;
    out[b] = (uint32_t)(r & 0xffffffffu);
  }
}

}  // namespace

void b_embed(const BatchDims& d, int B, const uint32_t* toks, const int8_t* emb, const float* emb_s,
             const float* rms0, float* x, int8_t* xq, float* xs, cudaStream_t s) {
  k_b_embed<<<B, kT, (size_t)d.dim * 8, s>>>(d.dim, toks, emb, emb_s, rms0, x, xq, xs);
}

void b_norm_quant(const BatchDims& d, int B, const float* x, const float* w, int8_t* xq, float* xs,
                  cudaStream_t s) {
  k_b_norm_quant<<<B, kT, (size_t)d.dim * 8, s>>>(d.dim, x, w, xq, xs);
}

void b_gemm_i8(int B, int R, int C, const int8_t* W, const float* ws, const int8_t* xq, const float* xs,
               float* out, int ldo, bool add, cudaStream_t s) {
  if (b_gemm_tc_eligible(B, C, W, xq) && b_gemm_tc(B, R, C, W, ws, xq, xs, out, ldo, add, s) == cudaSuccess)
    return;
  const int tt = (B + kGT - 1) / kGT;
  // 128-row tiles while they give two waves of CTAs, else 32-row tiles
  const bool wide = (long)((R + 127) / 128) * tt >= 296;
  const dim3 grid(wide ? (R + 127) / 128 : (R + 31) / 32, tt);
  if (wide) {
    if (add) k_b_gemm_i8<true, 4><<<grid, kT, 0, s>>>(B, R, C, W, ws, xq, xs, out, ldo);
    else k_b_gemm_i8<false, 4><<<grid, kT, 0, s>>>(B, R, C, W, ws, xq, xs, out, ldo);
  } else {
    if (add) k_b_gemm_i8<true, 1><<<grid, kT, 0, s>>>(B, R, C, W, ws, xq, xs, out, ldo);
    else k_b_gemm_i8<false, 1><<<grid, kT, 0, s>>>(B, R, C, W, ws, xq, xs, out, ldo);
  }
}

void b_rope_kv(const BatchDims& d, int layer, int B, const int32_t* pos, const int32_t* slot, const float* qkv,
               float* q, float* kc, float* vc, const float* rcos, const float* rsin, cudaStream_t s) {
  const long n = (long)B * 3 * d.dim / 2;
  k_b_rope_kv<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(d, layer, B, pos, slot, qkv, q, kc, vc, rcos, rsin);
}

void b_attention(const BatchDims& d, int layer, int B, const int32_t* pos, const int32_t* slot, const float* q,
                 const float* kc, const float* vc, float* scores, float* att, cudaStream_t s) {
  if (d.head_dim <= kAttT && d.head_dim % 16 == 0) {  // one fused CTA per (head, token)
    const size_t psm = (size_t)d.max_seq * 4;
    const dim3 g(d.n_heads, B);
    switch (d.head_dim / 16) {  // 16 <= head_dim <= 128, head_dim % 16 == 0
#define CHALOT_B_ATTN(C)                                                                             \
  case C:                                                                                            \
    cudaFuncSetAttribute(k_b_attn<C>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)psm);        \
    k_b_attn<C><<<g, kAttT, psm, s>>>(d, layer, pos, slot, q, kc, vc, att);                          \
    break;
      CHALOT_B_ATTN(1) CHALOT_B_ATTN(2) CHALOT_B_ATTN(3) CHALOT_B_ATTN(4)
      CHALOT_B_ATTN(5) CHALOT_B_ATTN(6) CHALOT_B_ATTN(7) default: CHALOT_B_ATTN(8)
#undef CHALOT_B_ATTN
    }
    return;
  }
  dim3 g1((d.max_seq + kScoreT - 1) / kScoreT, d.n_heads, B);
  switch (d.head_dim / 16) {  // 16 <= head_dim <= 256, head_dim % 8 == 0
#define CHALOT_B_SCORES(C) \
  case C: k_b_scores<C><<<g1, kScoreT, 0, s>>>(d, layer, pos, slot, q, kc, scores); break;
    CHALOT_B_SCORES(1) CHALOT_B_SCORES(2) CHALOT_B_SCORES(3) CHALOT_B_SCORES(4) CHALOT_B_SCORES(5)
    CHALOT_B_SCORES(6) CHALOT_B_SCORES(7) CHALOT_B_SCORES(8) CHALOT_B_SCORES(9) CHALOT_B_SCORES(10)
    CHALOT_B_SCORES(11) CHALOT_B_SCORES(12) CHALOT_B_SCORES(13) CHALOT_B_SCORES(14) CHALOT_B_SCORES(15)
    default: k_b_scores<16><<<g1, kScoreT, 0, s>>>(d, layer, pos, slot, q, kc, scores); break;
#undef CHALOT_B_SCORES
  }
  const size_t smem = ((size_t)((d.max_seq + 3) & ~3) + (size_t)kPvTile * kPvCols) * 4;
  cudaFuncSetAttribute(k_b_pv, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  k_b_pv<<<dim3(d.n_heads, d.head_dim / kPvCols, B), kT, smem, s>>>(d, layer, pos, slot, scores, vc, att);
}

void b_rmsnorm(const BatchDims& d, int B, const float* x, const float* w, float* xb, cudaStream_t s) {
  k_b_rmsnorm<<<B, kT, (size_t)d.dim * 8, s>>>(d.dim, x, w, xb);
}

void b_add(long n, float* x, const float* y, cudaStream_t s) {
  k_b_add<<<(unsigned)std::min<long>((n + 255) / 256, 4096), 256, 0, s>>>(n, x, y);
}

void b_argmax(int B, int V, const float* logits, uint32_t* out, cudaStream_t s) {
  k_b_argmax<<<B, kT, 0, s>>>(V, logits, out);
}

}  // namespace chalot
