// k_sample.cu — the reference's sampling strategies on device logits
// (src/tensor/sampling.rs:45-165, chosen by Engine::sample_from_logits,
// src/model/engine.rs:551-569), for a given uniform draw r in [0, 1).
//
//   top-k  logits * (1/T) when T > 0; the k largest; p = exp(l - max) / sum;
//          the first token in descending order whose running sum exceeds r
//   top-p  logits * (1/T) when T > 0 and T != 1; softmax; the shortest
//          descending prefix whose mass exceeds top_p; renormalised; the
//          first token of that prefix whose running sum exceeds r
//   min-p  as top-p's scaling and softmax; the tokens with p >= max_p * min_p
//          in index order; renormalised; the first whose running sum exceeds r
//
// One CTA of 1024 threads, with no sort of the vocabulary. The descending
// orders come from radix selection over 32-bit keys: four 8-bit passes of
// shared-memory histograms, counting tokens for the top-k threshold and
// summing probability mass to find where a running sum crosses a target.
// Ties at a threshold are taken lowest index first (the reference's unstable
// sort leaves their order unspecified). Thread t owns the contiguous index
// range [t*C, (t+1)*C), so "index order" is a prefix over threads. Mass sums
// are added in a different order than the reference's sequential sums, so a
// draw within rounding of a boundary may pick the neighbouring token: parity
// of the sampler is distributional (the reference draws r from the clock).
#include <cuda_runtime.h>

#include "common.cuh"

namespace chalot {
namespace {

constexpr int kST = 1024;

struct SampleSm {
  int hist_c[256];
  float hist_m[256];
  float red[32];
  int redi[32];
  int scan[kST];
  float scanf_[kST];
  unsigned prefix, mask;
  float target, acc_before;
  int remaining;
  int result;
};

__device__ __forceinline__ float block_sum_f(float v, SampleSm* sm) {
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sm->red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = 0.0f;
  if (threadIdx.x == 0) {
    for (int w = 0; w < kST / 32; ++w) r += sm->red[w];
    sm->red[0] = r;
  }
  __syncthreads();
  r = sm->red[0];
  __syncthreads();
  return r;
}

__device__ __forceinline__ float block_max_f(float v, SampleSm* sm) {
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sm->red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    float r = -INFINITY;
    for (int w = 0; w < kST / 32; ++w) r = fmaxf(r, sm->red[w]);
    sm->red[0] = r;
  }
  __syncthreads();
  const float r = sm->red[0];
  __syncthreads();
  return r;
}

// Exclusive prefix over threads of `v` (counts); returns this thread's offset.
__device__ __forceinline__ int block_excl_scan_i(int v, SampleSm* sm, int* total) {
  sm->scan[threadIdx.x] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int i = 0; i < kST; ++i) {
      const int c = sm->scan[i];
      sm->scan[i] = run;
      run += c;
    }
    sm->redi[0] = run;
  }
  __syncthreads();
  const int r = sm->scan[threadIdx.x];
  *total = sm->redi[0];
  __syncthreads();
  return r;
}

__device__ __forceinline__ float block_excl_scan_f(float v, SampleSm* sm) {
  sm->scanf_[threadIdx.x] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    float run = 0.0f;
    for (int i = 0; i < kST; ++i) {
      const float c = sm->scanf_[i];
      sm->scanf_[i] = run;
      run += c;
    }
  }
  __syncthreads();
  const float r = sm->scanf_[threadIdx.x];
  __syncthreads();
  return r;
}

// Sampling context: per index a key (descending order), a mass and a filter.
struct Ctx {
  const float* logits;
  int V, c0, c1;
  float scale;  // logits * scale
  int mode;     // 0: key = ordered logit, mass = exp(l - mx); 1: key = bits of mass, mass = p
  float mx, inv_sum;
  // kept-set restriction: key > kmin, or key == kmin and index <= kidx (none when kall)
  bool kall;
  unsigned kmin;
  int kidx;
};

__device__ __forceinline__ float scaled(const Ctx& c, int i) { return __fmul_rn(c.logits[i], c.scale); }

__device__ __forceinline__ void key_mass(const Ctx& c, int i, unsigned* key, float* mass) {
  const float l = scaled(c, i);
  if (c.mode == 0) {
    *key = ordered_key(l);
    *mass = expf(__fsub_rn(l, c.mx));
  } else {
    const float p = __fmul_rn(fast_exp(__fsub_rn(l, c.mx)), c.inv_sum);
    *key = __float_as_uint(p);
    *mass = p;
  }
}

__device__ __forceinline__ bool kept(const Ctx& c, unsigned key, int i) {
  return c.kall || key > c.kmin || (key == c.kmin && i <= c.kidx);
}

// Index of the j-th (0-based) kept element with key == k in index order.
__device__ int nth_tie(const Ctx& c, unsigned k, int j, SampleSm* sm) {
  int n = 0;
  for (int i = c.c0; i < c.c1; ++i) {
    unsigned key;
    float m;
    key_mass(c, i, &key, &m);
    n += (key == k && kept(c, key, i)) ? 1 : 0;
  }
  int total;
  const int off = block_excl_scan_i(n, sm, &total);
  if (threadIdx.x == 0) sm->result = -1;
  __syncthreads();
  j = min(j, total - 1);
  if (j >= off && j < off + n) {
    int seen = off;
    for (int i = c.c0; i < c.c1; ++i) {
      unsigned key;
      float m;
      key_mass(c, i, &key, &m);
      if (key == k && kept(c, key, i)) {
        if (seen == j) {
          sm->result = i;
          break;
        }
        ++seen;
      }
    }
  }
  __syncthreads();
  const int r = sm->result;
  __syncthreads();
  return r;
}

// Descending radix select over kept elements. count mode: the element of rank
// `rank` (1-based); mass mode: the first element whose running mass exceeds
// `target`. Returns the index; *key_out its key, *before the mass (or count)
// of the kept elements strictly before it in descending order.
__device__ int select_desc(const Ctx& c, bool by_mass, int rank, float target, unsigned* key_out, float* before,
                           SampleSm* sm) {
  if (threadIdx.x == 0) {
    sm->prefix = 0;
    sm->mask = 0;
    sm->target = target;
    sm->remaining = rank;
  }
  __syncthreads();
  float acc_total = 0.0f;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int b = threadIdx.x; b < 256; b += kST) {
      sm->hist_c[b] = 0;
      sm->hist_m[b] = 0.0f;
    }
    __syncthreads();
    const unsigned prefix = sm->prefix, mask = sm->mask;
    for (int i = c.c0; i < c.c1; ++i) {
      unsigned key;
      float m;
      key_mass(c, i, &key, &m);
      if ((key & mask) != prefix || !kept(c, key, i)) continue;
      const int b = (key >> shift) & 255;
      if (by_mass)
        atomicAdd(&sm->hist_m[b], m);
      else
        atomicAdd(&sm->hist_c[b], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int sel = -1, last = -1;
      if (by_mass) {
        float acc = 0.0f;
        for (int b = 255; b >= 0; --b) {
          if (sm->hist_m[b] <= 0.0f) continue;
          last = b;
          if (acc + sm->hist_m[b] > sm->target) {
            sel = b;
            break;
          }
          acc += sm->hist_m[b];
        }
        if (sel < 0) {  // rounding: no bucket crossed; take the smallest one
          sel = last < 0 ? 0 : last;
          acc -= last < 0 ? 0.0f : sm->hist_m[last];
        }
        sm->target -= acc;
        acc_total += acc;
      } else {
        int acc = 0;
        for (int b = 255; b >= 0; --b) {
          if (sm->hist_c[b] == 0) continue;
          last = b;
          if (acc + sm->hist_c[b] >= sm->remaining) {
            sel = b;
            break;
          }
          acc += sm->hist_c[b];
        }
        if (sel < 0) {
          sel = last < 0 ? 0 : last;
          acc -= last < 0 ? 0 : sm->hist_c[last];
        }
        sm->remaining -= acc;
        acc_total += (float)acc;
      }
      sm->prefix = prefix | ((unsigned)sel << shift);
      sm->mask = mask | (255u << shift);
      sm->acc_before = acc_total;
    }
    __syncthreads();
  }
  const unsigned k = sm->prefix;
  float tie_mass = 0.0f;
  if (by_mass) {  // all ties share one mass: which of them crosses
    for (int i = c.c0; i < c.c1; ++i) {
      unsigned key;
      float m;
      key_mass(c, i, &key, &m);
      if (key == k && kept(c, key, i)) tie_mass = m;
    }
    tie_mass = block_max_f(tie_mass, sm);
  }
  const int j = by_mass ? (tie_mass > 0.0f ? (int)floorf(sm->target / tie_mass) : 0) : sm->remaining - 1;
  const float acc_before = sm->acc_before;
  __syncthreads();
  const int idx = nth_tie(c, k, max(j, 0), sm);
  *key_out = k;
  *before = acc_before + (by_mass ? (float)max(j, 0) * tie_mass : (float)max(j, 0));
  return idx;
}

__global__ void __launch_bounds__(kST) k_sample(const float* __restrict__ logits, int V, int strategy,
                                                float temperature, int top_k, float top_p, float min_p, float r,
                                                unsigned long long* out) {
  __shared__ SampleSm sm;
  Ctx c;
  c.logits = logits;
  c.V = V;
  const int C = (V + kST - 1) / kST;
  c.c0 = min(V, (int)threadIdx.x * C);
  c.c1 = min(V, c.c0 + C);
  c.kall = true;
  c.kmin = 0;
  c.kidx = -1;
  const bool scale_t = strategy == 1 ? temperature > 0.0f : (temperature > 0.0f && temperature != 1.0f);
  c.scale = scale_t ? div_rn(1.0f, temperature) : 1.0f;
  float mx = -INFINITY;
  for (int i = c.c0; i < c.c1; ++i) mx = fmaxf(mx, scaled(c, i));
  c.mx = block_max_f(mx, &sm);
  int token = 0;
  if (strategy == 1) {  // top-k
    c.mode = 0;
    const int k = max(1, min(top_k, V));
    unsigned kk;
    float before;
    const int kth = select_desc(c, false, k, 0.0f, &kk, &before, &sm);
    c.kall = false;
    c.kmin = kk;
    c.kidx = kth;
    float s = 0.0f;
    for (int i = c.c0; i < c.c1; ++i) {
      unsigned key;
      float m;
      key_mass(c, i, &key, &m);
      if (kept(c, key, i)) s += m;
    }
    s = block_sum_f(s, &sm);
    token = select_desc(c, true, 0, __fmul_rn(r, s), &kk, &before, &sm);
  } else {  // top-p (2) and min-p (3): softmax of the scaled logits
    c.mode = 1;
    float s = 0.0f;
    for (int i = c.c0; i < c.c1; ++i) s += fast_exp(__fsub_rn(scaled(c, i), c.mx));
    c.inv_sum = div_rn(1.0f, block_sum_f(s, &sm));
    if (strategy == 2) {
      unsigned kc;
      float before;
      const int cut = select_desc(c, true, 0, top_p, &kc, &before, &sm);
      c.kall = false;
      c.kmin = kc;
      c.kidx = cut;
      float m = 0.0f;
      for (int i = c.c0; i < c.c1; ++i) {
        unsigned key;
        float p;
        key_mass(c, i, &key, &p);
        if (kept(c, key, i)) m += p;
      }
      m = block_sum_f(m, &sm);
      token = select_desc(c, true, 0, __fmul_rn(r, m), &kc, &before, &sm);
    } else {  // min-p, index order
      float pmax = 0.0f;
      for (int i = c.c0; i < c.c1; ++i) {
        unsigned key;
        float p;
        key_mass(c, i, &key, &p);
        pmax = fmaxf(pmax, p);
      }
      const float thr = __fmul_rn(block_max_f(pmax, &sm), min_p);
      float m = 0.0f;
      for (int i = c.c0; i < c.c1; ++i) {
        unsigned key;
        float p;
        key_mass(c, i, &key, &p);
        if (p >= thr) m += p;
      }
      const float mine = m;
      const float total = block_sum_f(m, &sm);
      const float off = block_excl_scan_f(mine, &sm);
      const float target = __fmul_rn(r, total);
      if (threadIdx.x == 0) sm.result = -1;
      __syncthreads();
      if (off <= target && target < off + mine) {
        float cum = off;
        for (int i = c.c0; i < c.c1; ++i) {
          unsigned key;
          float p;
          key_mass(c, i, &key, &p);
          if (p < thr) continue;
          cum += p;
          if (cum > target) {
            sm.result = i;
            break;
          }
        }
      }
      __syncthreads();
      token = sm.result;
      if (token < 0) {  // rounding past the end: the last kept index
        int last = -1;
        for (int i = c.c0; i < c.c1; ++i) {
          unsigned key;
          float p;
          key_mass(c, i, &key, &p);
          if (p >= thr) last = i;
        }
        for (int o = 16; o; o >>= 1) last = max(last, __shfl_xor_sync(0xffffffffu, last, o));
        if ((threadIdx.x & 31) == 0) sm.redi[threadIdx.x >> 5] = last;
        __syncthreads();
        if (threadIdx.x == 0) {
          int b = -1;
          for (int w = 0; w < kST / 32; ++w) b = max(b, sm.redi[w]);
          sm.result = b;
        }
        __syncthreads();
        token = max(sm.result, 0);
      }
    }
  }
  if (threadIdx.x == 0) *out = (unsigned long long)(unsigned)max(token, 0);
}

}  // namespace

cudaError_t launch_sample(const float* logits, int V, int strategy, float temperature, int top_k, float top_p,
                          float min_p, float r, unsigned long long* out, cudaStream_t s) {
  k_sample<<<1, kST, 0, s>>>(logits, V, strategy, temperature, top_k, top_p, min_p, r, out);
  return cudaGetLastError();
}

}  // namespace chalot
