// k_paged.cu — paged int8 KV cache for long-context decode: the page store
// (quantize f32 K/V into pages) and decode-step attention over the pages.
//
// Format (a new one; the reference's own PagedKVCache, src/model/memory.rs,
// keeps 256-token pages with one scale per token row): pages of P tokens. In
// each page the K block and the V block of every head (P x head_dim values,
// token-major) are int8 with one f32 scale per block, quantized with
// quantize_f32_to_i8's rule (absmax/127, round to nearest even,
// src/tensor/quantization.rs:56-104).
//   data   [page][K|V][head][P x head_dim] int8 (one page is contiguous); K
//          blocks token-major [P][head_dim], V blocks dim-major [head_dim][P]
//   scales [page][K|V][head] f32
//
// Attention per (sequence, head) is the attention of Engine::forward
// (src/model/engine.rs:283-309) over the dequantized rows: s_t =
// 30*tanh((q.k_t / sqrt(hd)) / 30), softmax, o = sum_t p_t v_t. It runs as
// split-page flash decoding in one persistent kernel: each CTA takes
// (sequence, split) items in turn and streams their pages through shared
// memory with 1-D bulk copies (one copy per page, a multi-stage ring running
// across items), warp h computes head h with an online softmax, and
// k_paged_merge combines the splits of each (sequence, head). The dot products
// run on dp4a: the query is split into two int8 planes (q ~ s1*q1 + s2*q2,
// s2 = s1/254, error below max|q|*1.6e-5 per element) against the int8 K rows, and the softmax
// weights p in [0, 1] into two planes (p ~ (p1 + p2/254)/127) against the
// dim-major int8 V rows, so the kernel stays bound by HBM reads of the pages.
// The sums are reordered and the planes round q and p slightly: agreement with
// the reference's f32 arithmetic is to float tolerance, not bits.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <string>

#include "blockops.cuh"
#include "capi_internal.h"
#include "common.cuh"
#include "devstat.h"
#include "tc.cuh"

namespace chalot {
namespace {

constexpr int kMaxStages = 8;
constexpr size_t kMaxSmem = 227 * 1024;

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
    if (threadIdx.x == 0) *(volatile unsigned*)(err + 1) = 1u;  // devstat word 1: a bad page id
    return;
  }
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    const int t = j / d.hd, c = j - t * d.hd;
    blk[j] = src[((size_t)(i * d.P + t) * d.H + h) * d.hd + c];
  }
  __syncthreads();
  const size_t b = ((size_t)page * 2 + kv) * d.H + h;
  float scale, inv;
  quant_scale(absmax_smem(blk, n, red), &scale, &inv);
  int8_t* dst = data + b * n;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    const int t = j / d.hd, c = j - t * d.hd;
    dst[kv ? c * d.P + t : j] = quant_any(blk[j], inv, j, n);  // V blocks dim-major
  }
  if (threadIdx.x == 0) scales[b] = scale;
}

struct PagedBars {
  uint64_t full[kMaxStages], empty[kMaxStages];
};

__device__ __forceinline__ int checked_page(const PagedDims& d, int page, unsigned* err) {
  if (page < 0 || page >= d.n_pages) {
    *(volatile unsigned*)(err + 1) = 1u;  // devstat word 1: a bad page id
    return 0;  // read an in-bounds page; the call reports the error
  }
  return page;
}

// Persistent CTA (two per SM): warps 0..H-1 compute heads, warp H issues the
// page copies. Work items are (sequence, split) pairs, item w -> sequence
// w / n_split, split w % n_split, taken in the order blockIdx.x, + gridDim.x,
// ...; the page ring (and the ring of page scales beside it, written by the
// producer before it arms each stage) runs across items, so the next item's
// pages stream in while this one finishes. Each item leaves its partial
// (running max m, sum l, unnormalised o) in `part` for k_paged_merge.
template <int HD, int P>
__global__ void __launch_bounds__(1024, 1) k_paged_attn(PagedDims d, const int8_t* __restrict__ data,
                                                        const float* __restrict__ scales,
                                                        const int32_t* __restrict__ page_table,
                                                        const int32_t* __restrict__ lens,
                                                        const float* __restrict__ q, float* part,
                                                        unsigned* err) {
  constexpr int PPI = 32 / P;    // pages per step: one token per lane
  constexpr int DPO = HD / 32;   // output dims per lane (lane + 32 j)
  extern __shared__ unsigned char smem_raw[];
  const size_t PB = (size_t)2 * d.H * P * HD;
  unsigned char* stage0 = reinterpret_cast<unsigned char*>(((uintptr_t)smem_raw + 127) & ~(uintptr_t)127);
  PagedBars* bars = reinterpret_cast<PagedBars*>(stage0 + d.stages * PB);
  unsigned char* after = reinterpret_cast<unsigned char*>(bars) + sizeof(PagedBars);
  float* sring = reinterpret_cast<float*>(after + (size_t)d.H * (2 * HD + 64));  // [stages][K|V][head]
  const int n_items = d.n_seq * d.n_split;
  const int pps = (d.max_pages + d.n_split - 1) / d.n_split;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < d.stages; ++i) {
      mbar_init_n(&bars->full[i], 1);
      mbar_init_n(&bars->empty[i], d.H);
    }
    mbar_fence_init();
  }
  __syncthreads();
  auto item_pages = [&](int it, int& s, int& split, int& L, int& pb, int& pe) {
    s = it / d.n_split;
    split = it - s * d.n_split;
    L = lens[s];
    const int npages = min((max(L, 0) + P - 1) / P, d.max_pages);
    pb = split * pps;
    pe = min(npages, pb + pps);
  };

  if (warp == d.H) {  // producer warp: lane 0 arms the stages and issues the copies
    int* pids = reinterpret_cast<int*>(sring + d.stages * 2 * d.H);  // the item's page ids
    int issued = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
      int s, split, L, pb, pe;
      item_pages(it, s, split, L, pb, pe);
      const int32_t* pt = page_table + (size_t)s * d.max_pages;
      for (int j = lane; j < pe - pb; j += 32) pids[j] = checked_page(d, pt[pb + j], err);
      __syncwarp();
      // the scales of the next page, one page ahead: lane j holds entries j and j + 32
      float n0 = 0.0f, n1 = 0.0f;
      auto fetch = [&](int i) {
        const float* sp = scales + (size_t)pids[i - pb] * 2 * d.H;
        n0 = lane < 2 * d.H ? __ldg(sp + lane) : 0.0f;
        n1 = lane + 32 < 2 * d.H ? __ldg(sp + lane + 32) : 0.0f;
      };
      if (pb < pe) fetch(pb);
      for (int i = pb; i < pe; ++i, ++issued) {
        const int st = issued % d.stages, n = issued / d.stages;
        const float c0 = n0, c1 = n1;
        const int page = pids[i - pb];
        if (i + 1 < pe) fetch(i + 1);
        bool free_ok = true;
        if (lane == 0 && n > 0) free_ok = mbar_wait(&bars->empty[st], (n - 1) & 1, err);
        if (!__shfl_sync(0xffffffffu, free_ok, 0)) {
          ok = false;
          break;
        }
        if (lane < 2 * d.H) sring[st * 2 * d.H + lane] = c0;
        if (lane + 32 < 2 * d.H) sring[st * 2 * d.H + lane + 32] = c1;
        __syncwarp();  // the scales are written before lane 0's release of the stage
        if (lane == 0) {
          mbar_expect_tx(&bars->full[st], (uint32_t)PB);
          tma_load(stage0 + st * PB, data + (size_t)page * PB, (uint32_t)PB, &bars->full[st]);
        }
      }
      __syncwarp();  // pids is rewritten by the next item
    }
    if (lane == 0)
      for (int c = max(0, issued - d.stages); c < issued; ++c)  // copies in flight land first
        mbar_wait(&bars->full[c % d.stages], (c / d.stages) & 1, err);
    return;
  }

  // consumer: head h = warp; lane = (page j of the step, token t)
  const int h = warp;
  const int jp = lane / P, t = lane % P;
  // per-warp shared scratch: query planes q1, q2 (HD bytes each), weight planes p1, p2 (32 bytes each)
  int8_t* wsm = reinterpret_cast<int8_t*>(after) + h * (2 * HD + 64);
  int8_t *q1 = wsm, *q2 = wsm + HD, *p1 = wsm + 2 * HD, *p2 = wsm + 2 * HD + 32;
  const uint4* q1w = reinterpret_cast<const uint4*>(q1);
  const uint4* q2w = reinterpret_cast<const uint4*>(q2);
  const float kscale = 1.0f / (sqrtf((float)HD) * 30.0f);  // q.k / sqrt(hd) / 30
  int u = 0;  // ring uses so far
  float qn[DPO];  // the query of the next item, loaded one item ahead
  auto load_q = [&](int it) {
#pragma unroll
    for (int j = 0; j < DPO; ++j)
      qn[j] = it < n_items ? q[((size_t)(it / d.n_split) * d.H + h) * HD + lane + 32 * j] : 0.0f;
  };
  load_q(blockIdx.x);
  for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
    int s, split, L, pb, pe;
    item_pages(it, s, split, L, pb, pe);
    float s1, s2;
    {
      float qv[DPO], amax = 0.0f;
#pragma unroll
      for (int j = 0; j < DPO; ++j) {
        qv[j] = qn[j];
        amax = fmaxf(amax, fabsf(qv[j]));
      }
      load_q(it + gridDim.x);
      amax = warp_max(amax);
      s1 = amax > 0.0f ? amax / 127.0f : 1.0f;
      s2 = s1 / 254.0f;
      __syncwarp();  // the previous item's reads of the planes are done
#pragma unroll
      for (int j = 0; j < DPO; ++j) {
        const float a = fminf(fmaxf(rintf(qv[j] / s1), -127.0f), 127.0f);
        const float r = qv[j] - a * s1;
        q1[lane + 32 * j] = (int8_t)a;
        q2[lane + 32 * j] = (int8_t)fminf(fmaxf(rintf(r / s2), -127.0f), 127.0f);
      }
      __syncwarp();
    }
    float m = -INFINITY, l = 0.0f, o[DPO];
#pragma unroll
    for (int j = 0; j < DPO; ++j) o[j] = 0.0f;
    bool ok = true;
    for (int i0 = pb; i0 < pe; i0 += PPI) {
      const int np = min(PPI, pe - i0);  // pages in this step
      for (int j = 0; j < np; ++j) ok = ok && mbar_wait(&bars->full[(u + j) % d.stages], ((u + j) / d.stages) & 1, err);
      if (!ok) break;
      const int i = i0 + jp;
      const bool have = jp < np;
      const bool valid = have && i * P + t < L;
      float sc = -INFINITY;
      if (valid) {
        const int st = (u + jp) % d.stages;
        const unsigned char* kb = stage0 + st * PB + (size_t)h * P * HD;
        const uint4* kr = reinterpret_cast<const uint4*>(kb + t * HD);
        int i1 = 0, i2 = 0;  // q.k_t as two exact int32 dot products
#pragma unroll
        for (int c0 = 0; c0 < HD / 16; ++c0) {
          const int c = (c0 + t) & (HD / 16 - 1);  // rotated so neighbouring rows hit different banks
          const uint4 w = lds16(kr + c), a = lds16(q1w + c), b2 = lds16(q2w + c);
          i1 = __dp4a((int)w.x, (int)a.x, i1);
          i1 = __dp4a((int)w.y, (int)a.y, i1);
          i1 = __dp4a((int)w.z, (int)a.z, i1);
          i1 = __dp4a((int)w.w, (int)a.w, i1);
          i2 = __dp4a((int)w.x, (int)b2.x, i2);
          i2 = __dp4a((int)w.y, (int)b2.y, i2);
          i2 = __dp4a((int)w.z, (int)b2.z, i2);
          i2 = __dp4a((int)w.w, (int)b2.w, i2);
        }
        const float dot = fmaf(s1, (float)i1, s2 * (float)i2);
        sc = 30.0f * tanhf(dot * sring[st * 2 * d.H + h] * kscale);
      }
      const float m_new = fmaxf(m, warp_max(sc));
      const float c = (m == -INFINITY) ? 0.0f : __expf(m - m_new);
      const float p = valid ? __expf(sc - m_new) : 0.0f;
      float ps = p;
#pragma unroll
      for (int off = 16; off; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
      l = fmaf(l, c, ps);
      {  // p in [0, 1] as two int8 planes
        const float a = rintf(p * 127.0f);
        p1[lane] = (int8_t)a;
        p2[lane] = (int8_t)fminf(fmaxf(rintf((p * 127.0f - a) * 254.0f), -127.0f), 127.0f);
      }
      __syncwarp();
      float acc[DPO];
#pragma unroll
      for (int j = 0; j < DPO; ++j) acc[j] = 0.0f;
      for (int jj = 0; jj < np; ++jj) {
        const int st = (u + jj) % d.stages;
        const unsigned char* vb = stage0 + st * PB + (size_t)(d.H + h) * P * HD;
        const float sv = sring[st * 2 * d.H + d.H + h];
#pragma unroll
        for (int j = 0; j < DPO; ++j) {
          int vw[P / 4];  // the dim's row of P int8 in one shared load
          const unsigned char* vr = vb + (size_t)(lane + 32 * j) * P;
          if (P == 8) {
            const uint2 x = *reinterpret_cast<const uint2*>(vr);
            vw[0] = (int)x.x;
            vw[1 % (P / 4)] = (int)x.y;
          } else {
#pragma unroll
            for (int w4 = 0; w4 < P / 16; ++w4) {
              const uint4 x = reinterpret_cast<const uint4*>(vr)[w4];
              vw[(4 * w4) % (P / 4)] = (int)x.x;
              vw[(4 * w4 + 1) % (P / 4)] = (int)x.y;
              vw[(4 * w4 + 2) % (P / 4)] = (int)x.z;
              vw[(4 * w4 + 3) % (P / 4)] = (int)x.w;
            }
          }
          int a1 = 0, a2 = 0;
#pragma unroll
          for (int w = 0; w < P / 4; ++w) {
            a1 = __dp4a(vw[w], *reinterpret_cast<const int*>(p1 + jj * P + 4 * w), a1);
            a2 = __dp4a(vw[w], *reinterpret_cast<const int*>(p2 + jj * P + 4 * w), a2);
          }
          acc[j] = fmaf(fmaf((float)a1, 1.0f / 127.0f, (float)a2 * (1.0f / (127.0f * 254.0f))), sv, acc[j]);
        }
      }
#pragma unroll
      for (int j = 0; j < DPO; ++j) o[j] = fmaf(o[j], c, acc[j]);
      m = m_new;
      __syncwarp();
      if (lane == 0)
        for (int j = 0; j < np; ++j) mbar_arrive(&bars->empty[(u + j) % d.stages]);
      u += np;
    }
    if (!ok) return;  // a copy never landed: recorded in err; this warp stops
    float* pp = part + (((size_t)s * d.H + h) * d.n_split + split) * (HD + 2);
    if (lane == 0) {
      pp[0] = m;
      pp[1] = l;
    }
#pragma unroll
    for (int j = 0; j < DPO; ++j) pp[2 + lane + 32 * j] = o[j];
  }
}

// Merges the splits of each (sequence, head), one warp per pair: o = sum_i
// o_i e^(m_i - M) / sum_i l_i e^(m_i - M), eight splits' partials loaded at
// a time.
template <int HD>
__global__ void __launch_bounds__(128) k_paged_merge(PagedDims d, const float* __restrict__ part, float* out) {
  constexpr int DPO = HD / 32;
  const int pair = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (pair >= d.n_seq * d.H) return;
  const float* base = part + (size_t)pair * d.n_split * (HD + 2);
  float M = -INFINITY;
  for (int i = lane; i < d.n_split; i += 32) M = fmaxf(M, base[(size_t)i * (HD + 2)]);
  M = warp_max(M);
  float Ls = 0.0f, O[DPO];
#pragma unroll
  for (int j = 0; j < DPO; ++j) O[j] = 0.0f;
  for (int i0 = 0; i0 < d.n_split; i0 += 8) {  // eight splits' loads in flight, then their sums in order
    float mi[8], li[8], oi[8][DPO];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const bool in = i0 + k < d.n_split;
      const float* pi = base + (size_t)(in ? i0 + k : 0) * (HD + 2);
      mi[k] = in ? pi[0] : -INFINITY;
      li[k] = pi[1];
#pragma unroll
      for (int j = 0; j < DPO; ++j) oi[k][j] = pi[2 + lane + 32 * j];
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (mi[k] == -INFINITY) continue;  // an empty split
      const float wgt = __expf(mi[k] - M);
      Ls = __fadd_rn(Ls, __fmul_rn(li[k], wgt));
#pragma unroll
      for (int j = 0; j < DPO; ++j) O[j] = __fadd_rn(O[j], __fmul_rn(oi[k][j], wgt));
    }
  }
#pragma unroll
  for (int j = 0; j < DPO; ++j) out[(size_t)pair * HD + lane + 32 * j] = Ls > 0.0f ? div_rn(O[j], Ls) : 0.0f;
}

int sm_count() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    sms = 148;
  return sms;
}

constexpr int kMaxItemPages = 64;  // pages of one (sequence, split) item; sets the least split count

size_t attn_smem(int H, int P, int HD, int stages) {
  return 128 + (size_t)stages * 2 * H * P * HD + sizeof(PagedBars) + (size_t)H * (2 * HD + 64) +
         (size_t)stages * 2 * H * 4 + kMaxItemPages * 4;
}

const char* paged_check(const chalot_paged_kv* kv) {
  if (!kv || !kv->data || !kv->scales) return "null cache";
  if (kv->page_tokens != 8 && kv->page_tokens != 16 && kv->page_tokens != 32) return "page_tokens must be 8, 16 or 32";
  if (kv->head_dim != 64 && kv->head_dim != 128) return "head_dim must be 64 or 128";
  if (kv->n_heads < 1 || kv->n_heads > 31) return "n_heads must be in [1, 31]";
  if (kv->n_pages < 1) return "n_pages must be positive";
  if (reinterpret_cast<uintptr_t>(kv->data) & 15) return "data must be 16-byte aligned";
  if (attn_smem((int)kv->n_heads, (int)kv->page_tokens, (int)kv->head_dim, 2) > kMaxSmem)
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
  // splits: about eight (sequence, split) items per SM for the persistent
  // CTAs (two per SM, three page stages each) to share out evenly
  const int want = (8 * sm_count() + (int)std::max<size_t>(n_seq, 1) - 1) / (int)std::max<size_t>(n_seq, 1);
  d.n_split = std::max(1, std::min(want, (int)std::max<size_t>(max_pages, 1)));
  d.n_split = std::max(d.n_split, (int)((max_pages + kMaxItemPages - 1) / kMaxItemPages));
  const size_t pb = (size_t)2 * d.H * d.P * d.hd;
  d.stages = (int)std::max<size_t>(2, std::min<size_t>(kMaxStages, (size_t)(96 * 1024) / pb));
  return d;
}

size_t part_bytes(const PagedDims& d) { return (size_t)d.n_seq * d.H * d.n_split * (d.hd + 2) * 4; }

template <int HD, int P>
cudaError_t launch_attn(const PagedDims& d, const chalot_paged_kv* kv, const int32_t* pt, const int32_t* lens,
                        const float* q, float* part, float* out, unsigned* err, cudaStream_t s) {
  const size_t smem = attn_smem(d.H, P, HD, d.stages);
  cudaError_t r = cudaFuncSetAttribute(k_paged_attn<HD, P>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (r != cudaSuccess) return r;
  const int items = d.n_seq * d.n_split;
  const int grid = std::max(1, std::min(items, 2 * sm_count()));
  k_paged_attn<HD, P><<<grid, (d.H + 1) * 32, smem, s>>>(d, kv->data, kv->scales, pt, lens, q, part, err);
  k_paged_merge<HD><<<(d.n_seq * d.H + 3) / 4, 128, 0, s>>>(d, part, out);
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
  // asynchronous: a page id outside the pool is skipped on the device and
  // reported by the next operator call or chalot_device_status (devstat.h)
  if (int rc = devstat_poll("paged_kv_store", s)) return rc;
  unsigned* err = devstat_word();
  if (!err) return set_error(CHALOT_ERR_CUDA, "paged_kv_store: device status word unavailable");
  const size_t smem = (size_t)d.P * d.hd * 4;
  cudaError_t r = cudaSuccess;
  if (smem > 48 * 1024)
    r = cudaFuncSetAttribute(k_paged_store, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (r == cudaSuccess) {
    k_paged_store<<<dim3((unsigned)n, 2 * d.H), 256, smem, s>>>(d, kv->data, kv->scales, page_ids, k, v, err);
    r = cudaGetLastError();
  }
  if (r != cudaSuccess) return set_error(CHALOT_ERR_CUDA, std::string("paged_kv_store: ") + cudaGetErrorString(r));
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
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (int rc = devstat_poll("paged_attention", s)) return rc;
  unsigned* err = devstat_word();  // bad page ids and timed-out waits (devstat.h)
  if (!err) return set_error(CHALOT_ERR_CUDA, "paged_attention: device status word unavailable");
  cudaError_t r;
  if (d.hd == 64 && d.P == 16) r = launch_attn<64, 16>(d, kv, page_table, seq_lens, q, part, out, err, s);
  else if (d.hd == 64 && d.P == 8) r = launch_attn<64, 8>(d, kv, page_table, seq_lens, q, part, out, err, s);
  else if (d.hd == 64 && d.P == 32) r = launch_attn<64, 32>(d, kv, page_table, seq_lens, q, part, out, err, s);
  else if (d.hd == 128 && d.P == 16) r = launch_attn<128, 16>(d, kv, page_table, seq_lens, q, part, out, err, s);
  else if (d.hd == 128 && d.P == 8) r = launch_attn<128, 8>(d, kv, page_table, seq_lens, q, part, out, err, s);
  else r = launch_attn<128, 32>(d, kv, page_table, seq_lens, q, part, out, err, s);
  if (r != cudaSuccess) return set_error(CHALOT_ERR_CUDA, std::string("paged_attention: ") + cudaGetErrorString(r));
  return CHALOT_OK;
}

}  // extern "C"
