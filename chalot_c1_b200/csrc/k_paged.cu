// k_paged.cu — paged int8 KV cache for long-context decode: the page store
// (quantize f32 K/V into pages) and decode-step attention over the pages.
//
// Format (a new one; the reference's own PagedKVCache, src/model/memory.rs,
// keeps 256-token pages with one scale per token row): pages of P tokens. In
// each page the K block and the V block of every head (P x head_dim values,
// token-major) are int8 with one f32 scale per block, quantized with
// quantize_f32_to_i8's rule (absmax/127, round to nearest even,
// src/tensor/quantization.rs:56-104).
//   data   [page][K|V][head][P][head_dim] int8   (one page is contiguous)
//   scales [page][K|V][head] f32
//
// Attention per (sequence, head) is the attention of Engine::forward
// (src/model/engine.rs:283-309) over the dequantized rows: s_t =
// 30*tanh((q.k_t / sqrt(hd)) / 30), softmax, o = sum_t p_t v_t. It runs as
// split-page flash decoding: CTA (split, seq) streams its share of the
// sequence's pages through shared memory with 1-D bulk copies (one copy per
// page, a multi-stage ring), warp h computes head h with an online softmax,
// and k_paged_combine merges the splits. The kernel is bound by HBM reads of
// the pages; the softmax reorders the reference's sums (float tolerance).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <string>

#include "blockops.cuh"
#include "capi_internal.h"
#include "common.cuh"
#include "tc.cuh"

namespace chalot {
namespace {

constexpr int kMaxStages = 8;
constexpr size_t kMaxSmem = 227 * 1024;

// Set by k_paged_store when a page id is out of range (that page is skipped).
__device__ unsigned g_store_err;

struct PagedDims {
  int P, H, hd, n_pages, n_seq, max_pages, n_split, stages;
};

// One CTA per (page i, K|V x head): quantize its P x hd block.
__global__ void __launch_bounds__(256) k_paged_store(PagedDims d, int8_t* data, float* scales,
                                                     const int32_t* __restrict__ page_ids,
                                                     const float* __restrict__ k, const float* __restrict__ v,
                                                     unsigned* err) {
  extern __shared__ __align__(16) float blk[];
  __shared__ float red[40];
  const int i = blockIdx.x, kv = blockIdx.y / d.H, h = blockIdx.y % d.H;
  const float* src = kv ? v : k;
  const int n = d.P * d.hd;
  int page = page_ids[i];
  if (page < 0 || page >= d.n_pages) {  // a bad id is reported, never written through
    if (threadIdx.x == 0) atomicExch(err, 1u);
    return;
  }
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    const int t = j / d.hd, c = j - t * d.hd;
    blk[j] = src[((size_t)(i * d.P + t) * d.H + h) * d.hd + c];
  }
  __syncthreads();
  const size_t b = ((size_t)page * 2 + kv) * d.H + h;
  const float s = quantize_smem(blk, n, data + b * n, red);
  if (threadIdx.x == 0) scales[b] = s;
}

// int8 x 4 (one word) to floats, exactly: bytes biased to unsigned are placed
// in the mantissa of 2^23 and the bias 2^23 + 128 is subtracted.
__device__ __forceinline__ void i8x4_to_f32(uint32_t w, float* f) {
  const uint32_t u = w ^ 0x80808080u;
  f[0] = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)), 8388736.0f);
  f[1] = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541)), 8388736.0f);
  f[2] = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)), 8388736.0f);
  f[3] = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543)), 8388736.0f);
}

struct PagedBars {
  uint64_t full[kMaxStages], empty[kMaxStages];
};

__device__ __forceinline__ int checked_page(const PagedDims& d, int page, unsigned* err) {
  if (page < 0 || page >= d.n_pages) {
    atomicExch(err, 1u);
    return 0;  // read an in-bounds page; the call reports the error
  }
  return page;
}

// CTA (split, seq): warps 0..H-1 compute heads, warp H issues the page copies.
// Partial results (running max m, sum l, unnormalised o) go to `part`.
template <int HD, int P>
__global__ void __launch_bounds__(1024, 1) k_paged_attn(PagedDims d, const int8_t* __restrict__ data,
                                                     const float* __restrict__ scales,
                                                     const int32_t* __restrict__ page_table,
                                                     const int32_t* __restrict__ lens,
                                                     const float* __restrict__ q, float* part,
                                                     unsigned* err) {
  constexpr int LPT = 32 / P;    // lanes per token
  constexpr int DPL = HD / LPT;  // q.k dims per lane
  constexpr int DPO = HD / 32;   // output dims per lane
  extern __shared__ unsigned char smem_raw[];
  const size_t PB = (size_t)2 * d.H * P * HD;
  unsigned char* stage0 = reinterpret_cast<unsigned char*>(((uintptr_t)smem_raw + 127) & ~(uintptr_t)127);
  PagedBars* bars = reinterpret_cast<PagedBars*>(stage0 + d.stages * PB);

  const int s = blockIdx.y, split = blockIdx.x;
  const int L = lens[s];
  const int npages = min((max(L, 0) + P - 1) / P, d.max_pages);
  const int pps = (d.max_pages + d.n_split - 1) / d.n_split;
  const int pb = split * pps, pe = min(npages, pb + pps);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int32_t* pt = page_table + (size_t)s * d.max_pages;

  if (threadIdx.x == 0) {
    for (int i = 0; i < d.stages; ++i) {
      mbar_init_n(&bars->full[i], 1);
      mbar_init_n(&bars->empty[i], d.H);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == d.H) {
    if (lane == 0) {  // producer
      int issued = 0;
      for (int i = pb; i < pe; ++i, ++issued) {
        const int st = issued % d.stages, n = issued / d.stages;
        if (n > 0 && !mbar_wait(&bars->empty[st], (n - 1) & 1, err)) break;
        const int page = checked_page(d, pt[i], err);
        mbar_expect_tx(&bars->full[st], (uint32_t)PB);
        tma_load(stage0 + st * PB, data + (size_t)page * PB, (uint32_t)PB, &bars->full[st]);
      }
      for (int c = max(0, issued - d.stages); c < issued; ++c)  // copies in flight land first
        mbar_wait(&bars->full[c % d.stages], (c / d.stages) & 1, err);
    }
    return;
  }

  // consumer: head h = warp
  const int h = warp;
  const int t = lane / LPT, lp = lane % LPT;
  // this head's query in shared memory (lanes of a token part read the same words)
  float* qsm = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(bars) + sizeof(PagedBars)) + h * HD;
  for (int j = lane; j < HD; j += 32) qsm[j] = q[((size_t)s * d.H + h) * HD + j];
  __syncwarp();
  const float4* qv4 = reinterpret_cast<const float4*>(qsm + lp * DPL);
  const float inv_sqrt = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
  float m = -INFINITY, l = 0.0f, o[DPO];
#pragma unroll
  for (int j = 0; j < DPO; ++j) o[j] = 0.0f;
  int used = 0;
  for (int i = pb; i < pe; ++i, ++used) {
    const int st = used % d.stages;
    if (!mbar_wait(&bars->full[st], (used / d.stages) & 1, err)) break;
    const int page = checked_page(d, pt[i], err);
    const float sk = __ldg(scales + ((size_t)page * 2) * d.H + h);
    const float sv = __ldg(scales + ((size_t)page * 2 + 1) * d.H + h);
    const unsigned char* kb = stage0 + st * PB + (size_t)h * P * HD;
    const unsigned char* vb = stage0 + st * PB + (size_t)(d.H + h) * P * HD;
    // q . k8 for this lane's token and dims
    float dot = 0.0f;
    const uint4* kr = reinterpret_cast<const uint4*>(kb + t * HD + lp * DPL);
#pragma unroll
    for (int c = 0; c < DPL / 16; ++c) {
      const uint4 w = kr[c];
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        float f[4];
        i8x4_to_f32(ws[u], f);
        const float4 qq = qv4[c * 4 + u];
        dot = __fadd_rn(dot, __fmul_rn(qq.x, f[0]));
        dot = __fadd_rn(dot, __fmul_rn(qq.y, f[1]));
        dot = __fadd_rn(dot, __fmul_rn(qq.z, f[2]));
        dot = __fadd_rn(dot, __fmul_rn(qq.w, f[3]));
      }
    }
#pragma unroll
    for (int off = 1; off < LPT; off <<= 1) dot = __fadd_rn(dot, __shfl_xor_sync(0xffffffffu, dot, off));
    const bool valid = i * P + t < L;
    float sc = -INFINITY;
    if (valid) {
      const float x = __fmul_rn(__fmul_rn(dot, sk), inv_sqrt);
      sc = __fmul_rn(30.0f, libm::tanh_f32(__fdiv_rn(x, 30.0f)));
    }
    const float m_new = fmaxf(m, warp_max(sc));
    const float c = (m == -INFINITY) ? 0.0f : fast_exp(__fsub_rn(m, m_new));
    const float p = valid ? fast_exp(__fsub_rn(sc, m_new)) : 0.0f;
    float ps = (lp == 0) ? p : 0.0f;
#pragma unroll
    for (int off = 16; off; off >>= 1) ps = __fadd_rn(ps, __shfl_xor_sync(0xffffffffu, ps, off));
    l = __fadd_rn(__fmul_rn(l, c), ps);
    float acc[DPO];
#pragma unroll
    for (int j = 0; j < DPO; ++j) acc[j] = 0.0f;
#pragma unroll
    for (int tt = 0; tt < P; ++tt) {
      const float ptt = __shfl_sync(0xffffffffu, p, tt * LPT);
      const unsigned char* vr = vb + tt * HD + lane * DPO;
      if (DPO == 4) {
        float f[4];
        i8x4_to_f32(*reinterpret_cast<const uint32_t*>(vr), f);
#pragma unroll
        for (int j = 0; j < DPO; ++j) acc[j] = __fadd_rn(acc[j], __fmul_rn(ptt, f[j]));
      } else {
        const uint32_t w2 = *reinterpret_cast<const uint16_t*>(vr);
        float f[4];
        i8x4_to_f32(w2, f);
#pragma unroll
        for (int j = 0; j < DPO; ++j) acc[j] = __fadd_rn(acc[j], __fmul_rn(ptt, f[j]));
      }
    }
#pragma unroll
    for (int j = 0; j < DPO; ++j) o[j] = __fadd_rn(__fmul_rn(o[j], c), __fmul_rn(acc[j], sv));
    m = m_new;
    __syncwarp();
    if (lane == 0) mbar_arrive(&bars->empty[st]);
  }
  float* pp = part + (((size_t)s * d.H + h) * d.n_split + split) * (HD + 2);
  if (lane == 0) {
    pp[0] = m;
    pp[1] = l;
  }
#pragma unroll
  for (int j = 0; j < DPO; ++j) pp[2 + lane * DPO + j] = o[j];
}

// Merges the splits of each (sequence, head): o = sum_i o_i e^(m_i - M) / sum_i l_i e^(m_i - M).
__global__ void k_paged_combine(PagedDims d, const float* __restrict__ part, float* out) {
  const int s = blockIdx.x / d.H, h = blockIdx.x % d.H;
  const float* pp = part + ((size_t)s * d.H + h) * d.n_split * (d.hd + 2);
  float M = -INFINITY;
  for (int i = 0; i < d.n_split; ++i) M = fmaxf(M, pp[i * (d.hd + 2)]);
  for (int j = threadIdx.x; j < d.hd; j += blockDim.x) {
    float L = 0.0f, O = 0.0f;
    for (int i = 0; i < d.n_split; ++i) {
      const float* pi = pp + i * (d.hd + 2);
      if (pi[0] == -INFINITY) continue;
      const float w = fast_exp(__fsub_rn(pi[0], M));
      L = __fadd_rn(L, __fmul_rn(pi[1], w));
      O = __fadd_rn(O, __fmul_rn(pi[2 + j], w));
    }
    out[((size_t)s * d.H + h) * d.hd + j] = L > 0.0f ? __fdiv_rn(O, L) : 0.0f;
  }
}

int sm_count() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    sms = 148;
  return sms;
}

const char* paged_check(const chalot_paged_kv* kv) {
  if (!kv || !kv->data || !kv->scales) return "null cache";
  if (kv->page_tokens != 8 && kv->page_tokens != 16 && kv->page_tokens != 32) return "page_tokens must be 8, 16 or 32";
  if (kv->head_dim != 64 && kv->head_dim != 128) return "head_dim must be 64 or 128";
  if (kv->n_heads < 1 || kv->n_heads > 31) return "n_heads must be in [1, 31]";
  if (kv->n_pages < 1) return "n_pages must be positive";
  if (reinterpret_cast<uintptr_t>(kv->data) & 15) return "data must be 16-byte aligned";
  if (2 * ((size_t)2 * kv->n_heads * kv->page_tokens * kv->head_dim) + 128 + 2 * kMaxStages * 8 +
          (size_t)kv->n_heads * kv->head_dim * 4 > kMaxSmem)
    return "two pages do not fit in shared memory (n_heads * page_tokens * head_dim too large)";
  return nullptr;
}

PagedDims paged_dims(const chalot_paged_kv* kv, size_t n_seq, size_t max_pages) {
  PagedDims d{};
  d.P = (int)kv->page_tokens;
  d.H = (int)kv->n_heads;
  d.hd = (int)kv->head_dim;
  d.n_pages = (int)kv->n_pages;
  d.n_seq = (int)n_seq;
  d.max_pages = (int)max_pages;
  const int want = (4 * sm_count() + (int)std::max<size_t>(n_seq, 1) - 1) / (int)std::max<size_t>(n_seq, 1);
  d.n_split = std::max(1, std::min(want, (int)std::max<size_t>(max_pages, 1)));
  const size_t pb = (size_t)2 * d.H * d.P * d.hd;
  d.stages = (int)std::max<size_t>(2, std::min<size_t>(kMaxStages, (size_t)(192 * 1024) / pb));
  return d;
}

size_t part_bytes(const PagedDims& d) { return (size_t)d.n_seq * d.H * d.n_split * (d.hd + 2) * 4; }

template <int HD, int P>
cudaError_t launch_attn(const PagedDims& d, const chalot_paged_kv* kv, const int32_t* pt, const int32_t* lens,
                        const float* q, float* part, unsigned* err, cudaStream_t s) {
  const size_t smem = 128 + (size_t)d.stages * 2 * d.H * P * HD + sizeof(PagedBars) + (size_t)d.H * HD * 4;
  cudaError_t r = cudaFuncSetAttribute(k_paged_attn<HD, P>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (r != cudaSuccess) return r;
  k_paged_attn<HD, P><<<dim3(d.n_split, d.n_seq), (d.H + 1) * 32, smem, s>>>(d, kv->data, kv->scales, pt, lens, q,
                                                                             part, err);
  return cudaGetLastError();
}

}  // namespace
}  // namespace chalot

using namespace chalot;

extern "C" {

__attribute__((visibility("default"))) int chalot_paged_kv_store(const chalot_paged_kv* kv, const int32_t* page_ids,
                                                                 size_t n, const float* k, const float* v,
                                                                 void* stream) {
  if (const char* m = paged_check(kv)) return set_error(CHALOT_ERR_ARG, std::string("paged_kv_store: ") + m);
  if (n == 0) return CHALOT_OK;
  if (!page_ids || !k || !v) return set_error(CHALOT_ERR_ARG, "paged_kv_store: null pointer");
  PagedDims d = paged_dims(kv, 0, 0);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned* err = nullptr;
  cudaError_t r = cudaGetSymbolAddress(reinterpret_cast<void**>(&err), g_store_err);
  const size_t smem = (size_t)d.P * d.hd * 4;
  if (r == cudaSuccess && smem > 48 * 1024)
    r = cudaFuncSetAttribute(k_paged_store, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (r == cudaSuccess) r = cudaMemsetAsync(err, 0, 4, s);
  if (r == cudaSuccess) {
    k_paged_store<<<dim3((unsigned)n, 2 * d.H), 256, smem, s>>>(d, kv->data, kv->scales, page_ids, k, v, err);
    r = cudaGetLastError();
  }
  unsigned herr = 0;  // the store is synchronous, as KVPage::write_token is
  if (r == cudaSuccess) r = cudaMemcpyAsync(&herr, err, 4, cudaMemcpyDeviceToHost, s);
  if (r == cudaSuccess) r = cudaStreamSynchronize(s);
  if (r != cudaSuccess) return set_error(CHALOT_ERR_CUDA, std::string("paged_kv_store: ") + cudaGetErrorString(r));
  if (herr) return set_error(CHALOT_ERR_ARG, "paged_kv_store: a page id is outside [0, n_pages); those pages were skipped");
  return CHALOT_OK;
}

__attribute__((visibility("default"))) size_t chalot_paged_attention_workspace_size(const chalot_paged_kv* kv,
                                                                                    size_t n_seq,
                                                                                    size_t max_pages) {
  if (const char* m = paged_check(kv)) {
    set_error(CHALOT_ERR_ARG, std::string("paged_attention: ") + m);
    return 0;
  }
  PagedDims d = paged_dims(kv, n_seq, max_pages);
  return ((part_bytes(d) + 255) & ~size_t(255)) + 256;
}

__attribute__((visibility("default"))) int chalot_paged_attention(const chalot_paged_kv* kv, const float* q,
                                                                  size_t n_seq, const int32_t* page_table,
                                                                  size_t max_pages, const int32_t* seq_lens,
                                                                  float* out, void* workspace,
                                                                  size_t workspace_bytes, void* stream) {
  if (const char* m = paged_check(kv)) return set_error(CHALOT_ERR_ARG, std::string("paged_attention: ") + m);
  if (n_seq == 0) return CHALOT_OK;
  if (!q || !page_table || !seq_lens || !out) return set_error(CHALOT_ERR_ARG, "paged_attention: null pointer");
  if (max_pages == 0 || max_pages > (1u << 24) || n_seq > 65535)
    return set_error(CHALOT_ERR_ARG, "paged_attention: max_pages must be in [1, 2^24], n_seq at most 65535");
  const size_t need = chalot_paged_attention_workspace_size(kv, n_seq, max_pages);
  if (!workspace || workspace_bytes < need)
    return set_error(CHALOT_ERR_ARG, "paged_attention: workspace too small (need " + std::to_string(need) + " bytes)");
  PagedDims d = paged_dims(kv, n_seq, max_pages);
  float* part = static_cast<float*>(workspace);
  unsigned* err = reinterpret_cast<unsigned*>(static_cast<unsigned char*>(workspace) + ((part_bytes(d) + 255) & ~size_t(255)));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t r = cudaMemsetAsync(err, 0, 4, s);
  if (r == cudaSuccess) {
    if (d.hd == 64 && d.P == 16) r = launch_attn<64, 16>(d, kv, page_table, seq_lens, q, part, err, s);
    else if (d.hd == 64 && d.P == 8) r = launch_attn<64, 8>(d, kv, page_table, seq_lens, q, part, err, s);
    else if (d.hd == 64 && d.P == 32) r = launch_attn<64, 32>(d, kv, page_table, seq_lens, q, part, err, s);
    else if (d.hd == 128 && d.P == 16) r = launch_attn<128, 16>(d, kv, page_table, seq_lens, q, part, err, s);
    else if (d.hd == 128 && d.P == 8) r = launch_attn<128, 8>(d, kv, page_table, seq_lens, q, part, err, s);
    else r = launch_attn<128, 32>(d, kv, page_table, seq_lens, q, part, err, s);
  }
  if (r == cudaSuccess) {
    k_paged_combine<<<(unsigned)(n_seq * d.H), 128, 0, s>>>(d, part, out);
    r = cudaGetLastError();
  }
  if (r != cudaSuccess) return set_error(CHALOT_ERR_CUDA, std::string("paged_attention: ") + cudaGetErrorString(r));
  if (std::getenv("CHALOT_PAGED_SYNC_CHECK")) {  // tests: surface a bad page id or a wait that ran out
    unsigned herr = 0;
    r = cudaMemcpyAsync(&herr, err, 4, cudaMemcpyDeviceToHost, s);
    if (r == cudaSuccess) r = cudaStreamSynchronize(s);
    if (r != cudaSuccess) return set_error(CHALOT_ERR_CUDA, std::string("paged_attention: ") + cudaGetErrorString(r));
    if (herr) return set_error(CHALOT_ERR_ARG, "paged_attention: a page id was outside [0, n_pages) or a copy timed out");
  }
  return CHALOT_OK;
}

}  // extern "C"
