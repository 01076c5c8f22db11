// oracle.cpp — CPU restatement of chalot_C1's inference hot path.
//
// TEST INFRASTRUCTURE ONLY. This library is the parity checker for the CUDA
// implementation and the timed CPU baseline; nothing in the product links,
// loads or calls it.
//
// The reference (chalot28/chalot_C1) is Rust and cannot be built here, so this
// file restates, function by function, the code path the reference takes on an
// x86-64 host with AVX2 (every `is_x86_feature_detected!("avx2")` branch):
//   quantize_f32_to_i8_avx2   src/tensor/quantization.rs:56-104
//   unpack/pack_int4          src/tensor/quantization.rs:114-126
//   quantize_f32_to_i4        src/tensor/quantization.rs:131-162
//   matmul_int8_avx2          src/tensor/matmul.rs:47-97, 183-298
//   matmul_int4_avx2          src/tensor/matmul.rs:363-401, 452-654
//   rmsnorm_avx2              src/tensor/normalization.rs:35-67
//   softmax_avx2, fast_exp    src/tensor/normalization.rs:106-200
//   softmax_top_k             src/tensor/normalization.rs:203-216
//   swiglu_fused_avx2         src/tensor/activations.rs:59-127
//   logit_soft_cap            src/tensor/activations.rs:133-135
//   dot_f32_avx2              src/tensor/attention_helpers.rs:41-80
//   sample_argmax             src/tensor/sampling.rs:34-41
//   apply_repetition_penalty  src/tensor/sampling.rs:168-178
//   InferenceState::new RoPE  src/model/state.rs:41-60
//   Engine::forward           src/model/engine.rs:173-494
//   expert block, T tokens    src/model/engine.rs:334-401 (orc_moe_forward)
//   paged int8 KV attention   engine.rs:283-309 over memory.rs:69-74 dequantized rows
//   PagedKVCache              src/model/memory.rs:26-201 (orc_kvc_*)
//   sampling strategies       src/tensor/sampling.rs:45-165 (orc_sample, given the draw)
//   Engine::generate          src/model/engine.rs:497-548
//   sample_from_logits        src/model/engine.rs:551-569
//   header/config/index       src/model/header.rs:40-133, config.rs:40-69,
//                             weight_index.rs:85-263
// Float reductions are written as explicit 8-lane arrays in the order the AVX2
// code adds them; compiled without contraction (-ffp-contract=off) and without
// -ffast-math each lane operation rounds exactly as the SIMD instruction does.
// Transcendentals call glibc (expf, tanhf, powf, cosf, sinf), the libm Rust's
// std links on Linux. Integer dot products are exact in any order.
//
// Pinning: the operators are pinned by the reference's own known-answer tests
// (src/tensor/tests.rs, src/model/memory.rs tests; tests/test_oracle.py) and by
// an independent numpy restatement; the reference holds no end-to-end outputs
// and cannot be run here, so whole-model decode parity is unpinned beyond this
// restatement.
#include <fcntl.h>
#include <immintrin.h>
#include <omp.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <deque>
#include <map>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#define ORC_API extern "C" __attribute__((visibility("default")))

namespace {

thread_local std::string g_err;

// ---------------------------------------------------------------------------
// Lane helpers
// ---------------------------------------------------------------------------

// Horizontal sum of an 8-lane f32 accumulator in the reference's order:
// extract hi/lo halves and add (lane j + lane j+4), then movehl (+2), then
// shuffle (+1): ((t0 + t2) + (t1 + t3)).
inline float hsum8(const float s[8]) {
  float t0 = s[0] + s[4], t1 = s[1] + s[5], t2 = s[2] + s[6], t3 = s[3] + s[7];
  float u0 = t0 + t2, u1 = t1 + t3;
  return u0 + u1;
}

inline float bits_to_float(uint32_t b) {
  float f;
  std::memcpy(&f, &b, 4);
  return f;
}

// _mm256_cvtps_epi32 under the default rounding mode: nearest-even, and the
// "integer indefinite" 0x80000000 for NaN or out-of-range inputs.
inline int32_t cvt_rne_i32(float x) {
  if (!(x >= -2147483648.0f && x < 2147483648.0f)) return INT32_MIN;
  return int32_t(std::nearbyint(x));
}

// fast_exp_avx2, one lane (normalization.rs:165-200; the copy in
// activations.rs:92-127 is identical).
inline float fast_exp(float x) {
  const float ln2 = 0.693147180559945309f;
  const float inv_ln2 = 1.442695040888963407f;
  const float c0 = 1.0f, c1 = 1.0f, c2 = 0.5f, c3 = 0.166666666666f,
              c4 = 0.041666666666f, c5 = 0.008333333333f;
  float n = std::floor(x * inv_ln2);
  float r = x - n * ln2;
  float p = c5;
  p = p * r + c4;
  p = p * r + c3;
  p = p * r + c2;
  p = p * r + c1;
  p = p * r + c0;
  uint32_t e = (uint32_t(cvt_rne_i32(n)) + 127u) << 23;
  return p * bits_to_float(e);
}

// Rust's f32::round: half away from zero.
inline float round_half_away(float x) { return std::round(x); }

// Rust's `as i8` from f32: saturating, NaN -> 0.
inline int8_t sat_i8(float x) {
  if (x != x) return 0;
  if (x >= 127.0f) return 127;
  if (x <= -128.0f) return -128;
  return int8_t(x);
}

// ---------------------------------------------------------------------------
// Quantization (quantization.rs:56-104)
// ---------------------------------------------------------------------------
float quantize_i8(const float* x, int8_t* q, size_t n) {
  const size_t chunks = n / 8;
  float m[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (size_t c = 0; c < chunks; ++c)
    for (int j = 0; j < 8; ++j) {
      float a = std::fabs(x[c * 8 + j]);
      m[j] = (m[j] > a) ? m[j] : a;  // _mm256_max_ps(max_vec, abs_v)
    }
  // hi/lo max, movehl, shuffle: max is order-free for non-NaN inputs.
  float amax = m[0];
  for (int j = 1; j < 8; ++j) amax = std::max(amax, m[j]);
  for (size_t i = chunks * 8; i < n; ++i) amax = std::max(amax, std::fabs(x[i]));
  amax = std::max(amax, 1e-12f);
  const float scale = amax / 127.0f;
  const float inv = 1.0f / scale;
  for (size_t i = 0; i < chunks * 8; ++i) {
    float s = x[i] * inv;
    s = (s < 127.0f) ? s : 127.0f;    // _mm256_min_ps(scaled, 127)
    s = (s > -127.0f) ? s : -127.0f;  // _mm256_max_ps(., -127)
    q[i] = int8_t(cvt_rne_i32(s));    // in range after the clamp
  }
  for (size_t i = chunks * 8; i < n; ++i) {  // scalar tail: .round().clamp() as i8
    float s = round_half_away(x[i] * inv);
    s = std::min(std::max(s, -127.0f), 127.0f);
    q[i] = sat_i8(s);
  }
  return scale;
}

// ---------------------------------------------------------------------------
// Integer dot products (exact)
// ---------------------------------------------------------------------------
int32_t dot_i8(const int8_t* w, const int8_t* x, size_t n) {
  __m256i acc = _mm256_setzero_si256();
  size_t k = 0;
  for (; k + 32 <= n; k += 32) {
    __m256i vw = _mm256_loadu_si256((const __m256i*)(w + k));
    __m256i vx = _mm256_loadu_si256((const __m256i*)(x + k));
    __m256i wl = _mm256_cvtepi8_epi16(_mm256_castsi256_si128(vw));
    __m256i wh = _mm256_cvtepi8_epi16(_mm256_extracti128_si256(vw, 1));
    __m256i xl = _mm256_cvtepi8_epi16(_mm256_castsi256_si128(vx));
    __m256i xh = _mm256_cvtepi8_epi16(_mm256_extracti128_si256(vx, 1));
    acc = _mm256_add_epi32(acc, _mm256_add_epi32(_mm256_madd_epi16(wl, xl), _mm256_madd_epi16(wh, xh)));
  }
  alignas(32) int32_t lanes[8];
  _mm256_store_si256((__m256i*)lanes, acc);
  int32_t s = 0;
  for (int j = 0; j < 8; ++j) s += lanes[j];
  for (; k < n; ++k) s += int32_t(w[k]) * int32_t(x[k]);
  return s;
}

// Signed value of column k of a packed int4 row (low nibble = even column).
inline int32_t nib(const uint8_t* row, size_t k) {
  uint8_t b = row[k >> 1];
  return int32_t((k & 1) ? (b >> 4) : (b & 0x0F)) - 8;
}

// Dot of columns [s, e) of a packed int4 row with x_q; s is even.
int32_t dot_i4(const uint8_t* row, const int8_t* x, size_t s, size_t e) {
  int32_t acc = 0;
  size_t k = s;
  if (e - s >= 32) {
    const __m128i m = _mm_set1_epi8(0x0F), eight = _mm_set1_epi8(8);
    __m256i v = _mm256_setzero_si256();
    for (; k + 32 <= e; k += 32) {
      __m128i p = _mm_loadu_si128((const __m128i*)(row + (k >> 1)));
      __m128i lo = _mm_sub_epi8(_mm_and_si128(p, m), eight);
      __m128i hi = _mm_sub_epi8(_mm_and_si128(_mm_srli_epi16(p, 4), m), eight);
      __m128i a = _mm_unpacklo_epi8(lo, hi), b = _mm_unpackhi_epi8(lo, hi);
      __m256i vx = _mm256_loadu_si256((const __m256i*)(x + k));
      __m256i xa = _mm256_cvtepi8_epi16(_mm256_castsi256_si128(vx));
      __m256i xb = _mm256_cvtepi8_epi16(_mm256_extracti128_si256(vx, 1));
      v = _mm256_add_epi32(v, _mm256_add_epi32(_mm256_madd_epi16(_mm256_cvtepi8_epi16(a), xa),
                                               _mm256_madd_epi16(_mm256_cvtepi8_epi16(b), xb)));
    }
    alignas(32) int32_t lanes[8];
    _mm256_store_si256((__m256i*)lanes, v);
    for (int j = 0; j < 8; ++j) acc += lanes[j];
  }
  for (; k < e; ++k) acc += nib(row, k) * int32_t(x[k]);
  return acc;
}

// matmul_int8: out[r] = ((float)dot * w_scale[r]) * x_scale (matmul.rs:260-261, 296)
void matmul_i8_q(float* out, int32_t* dots, const int8_t* w, const float* ws, const int8_t* xq,
                 float xs, size_t out_dim, size_t in_dim, int threads) {
#pragma omp parallel for schedule(static) num_threads(threads) if (threads > 1 && out_dim >= 256)
  for (long r = 0; r < long(out_dim); ++r) {
    int32_t d = dot_i8(w + size_t(r) * in_dim, xq, in_dim);
    if (dots) dots[r] = d;
    out[r] = (float(d) * ws[r]) * xs;
  }
}

void matmul_i8(float* out, const int8_t* w, const float* ws, const float* x, size_t out_dim,
               size_t in_dim, int threads) {
  std::vector<int8_t> xq(in_dim);
  float xs = quantize_i8(x, xq.data(), in_dim);
  matmul_i8_q(out, nullptr, w, ws, xq.data(), xs, out_dim, in_dim, threads);
}

// matmul_int4: total += ((float)gdot * gs) * xs, sequentially over groups
// (matmul.rs:576-577, 649).
void matmul_i4_q(float* out, int32_t* gdots, const uint8_t* wp, const float* ws, const int8_t* xq,
                 float xs, size_t out_dim, size_t in_dim, size_t group, int threads) {
  const size_t ng = (in_dim + group - 1) / group, prow = (in_dim + 1) / 2;
#pragma omp parallel for schedule(static) num_threads(threads) if (threads > 1 && out_dim >= 256)
  for (long r = 0; r < long(out_dim); ++r) {
    const uint8_t* row = wp + size_t(r) * prow;
    float total = 0.0f;
    for (size_t g = 0; g < ng; ++g) {
      size_t s = g * group, e = std::min(s + group, in_dim);
      int32_t d = dot_i4(row, xq, s, e);
      if (gdots) gdots[size_t(r) * ng + g] = d;
      total += (float(d) * ws[size_t(r) * ng + g]) * xs;
    }
    out[r] = total;
  }
}

void matmul_i4(float* out, const uint8_t* wp, const float* ws, const float* x, size_t out_dim,
               size_t in_dim, size_t group, int threads) {
  std::vector<int8_t> xq(in_dim);
  float xs = quantize_i8(x, xq.data(), in_dim);
  matmul_i4_q(out, nullptr, wp, ws, xq.data(), xs, out_dim, in_dim, group, threads);
}

// ---------------------------------------------------------------------------
// Norm, softmax, activations, dot (normalization.rs, activations.rs,
// attention_helpers.rs)
// ---------------------------------------------------------------------------
void rmsnorm(float* out, const float* x, const float* w, size_t dim) {
  const size_t chunks = dim / 8;
  float s[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (size_t c = 0; c < chunks; ++c)
    for (int j = 0; j < 8; ++j) {
      float v = x[c * 8 + j];
      float sq = v * v;
      s[j] = s[j] + sq;
    }
  float ss = hsum8(s);
  for (size_t i = chunks * 8; i < dim; ++i) {
    float sq = x[i] * x[i];
    ss += sq;
  }
  float inv = 1.0f / std::sqrt(ss / float(dim) + 1e-5f);
  for (size_t i = 0; i < dim; ++i) {
    float a = x[i] * inv;
    out[i] = a * w[i];
  }
}

void softmax(float* x, size_t n) {
  if (n == 0) return;
  const size_t chunks = n / 8;
  float m[8];
  for (int j = 0; j < 8; ++j) m[j] = -INFINITY;
  for (size_t c = 0; c < chunks; ++c)
    for (int j = 0; j < 8; ++j) {
      float v = x[c * 8 + j];
      m[j] = (m[j] > v) ? m[j] : v;  // _mm256_max_ps(max_v, v)
    }
  // hi/lo, movehl, shuffle max tree
  float t0 = (m[0] > m[4]) ? m[0] : m[4], t1 = (m[1] > m[5]) ? m[1] : m[5];
  float t2 = (m[2] > m[6]) ? m[2] : m[6], t3 = (m[3] > m[7]) ? m[3] : m[7];
  float u0 = (t0 > t2) ? t0 : t2, u1 = (t1 > t3) ? t1 : t3;
  float mx = (u0 > u1) ? u0 : u1;
  for (size_t i = chunks * 8; i < n; ++i) mx = std::max(mx, x[i]);  // f32::max
  float s[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (size_t c = 0; c < chunks; ++c)
    for (int j = 0; j < 8; ++j) {
      float e = fast_exp(x[c * 8 + j] - mx);
      x[c * 8 + j] = e;
      s[j] = s[j] + e;
    }
  float sum = hsum8(s);
  for (size_t i = chunks * 8; i < n; ++i) {
    float e = std::exp(x[i] - mx);
    x[i] = e;
    sum += e;
  }
  const float inv = 1.0f / sum;
  for (size_t i = 0; i < n; ++i) x[i] = x[i] * inv;
}

float dot_f32(const float* a, const float* b, size_t len) {
  const size_t c16 = len / 16;
  float a0[8] = {0, 0, 0, 0, 0, 0, 0, 0}, a1[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (size_t c = 0; c < c16; ++c)
    for (int j = 0; j < 8; ++j) {
      float p0 = a[c * 16 + j] * b[c * 16 + j];
      a0[j] = a0[j] + p0;
      float p1 = a[c * 16 + 8 + j] * b[c * 16 + 8 + j];
      a1[j] = a1[j] + p1;
    }
  const size_t rem = c16 * 16;
  if (rem + 8 <= len)
    for (int j = 0; j < 8; ++j) {
      float p = a[rem + j] * b[rem + j];
      a0[j] = a0[j] + p;
    }
  float c[8];
  for (int j = 0; j < 8; ++j) c[j] = a0[j] + a1[j];
  float r = hsum8(c);
  for (size_t i = (rem + 8 <= len) ? rem + 8 : rem; i < len; ++i) {
    float p = a[i] * b[i];
    r += p;
  }
  return r;
}

void swiglu(float* g, const float* u, size_t n) {
  const size_t chunks = n / 8;
  for (size_t i = 0; i < chunks * 8; ++i) {
    float ng = 0.0f - g[i];
    float den = 1.0f + fast_exp(ng);
    float si = g[i] / den;
    g[i] = si * u[i];
  }
  for (size_t i = chunks * 8; i < n; ++i) {
    float den = 1.0f + std::exp(-g[i]);
    float si = g[i] / den;
    g[i] = si * u[i];
  }
}

inline float soft_cap(float x, float cap) { return cap * std::tanh(x / cap); }

// softmax_top_k: softmax, stable descending order (the insertion sort Rust's
// sort_unstable_by uses below 20 elements keeps equal keys in index order),
// truncate, renormalise when the sum exceeds 1e-12.
size_t softmax_top_k(float* scores, size_t n, size_t k, int32_t* idx, float* w) {
  softmax(scores, n);
  std::vector<int32_t> order(n);
  for (size_t i = 0; i < n; ++i) order[i] = int32_t(i);
  std::stable_sort(order.begin(), order.end(),
                   [&](int32_t a, int32_t b) { return scores[a] > scores[b]; });
  k = std::min(k, n);
  float sum = -0.0f;
  for (size_t i = 0; i < k; ++i) sum += scores[order[i]];
  for (size_t i = 0; i < k; ++i) {
    idx[i] = order[i];
    w[i] = (sum > 1e-12f) ? scores[order[i]] / sum : scores[order[i]];
  }
  return k;
}

// sample_argmax: Iterator::max_by keeps the LAST of equal maxima.
long argmax(const float* x, size_t n) {
  if (n == 0) return 0;
  size_t best = 0;
  for (size_t i = 0; i < n; ++i) {
    if (x[i] != x[i]) return -1;  // the reference panics on NaN
    if (x[i] >= x[best]) best = i;
  }
  return long(best);
}

void repetition_penalty(float* logits, size_t n, const uint32_t* hist, size_t nh, float p) {
  for (size_t i = 0; i < nh; ++i) {
    uint32_t t = hist[i];
    if (t < n) {
      if (logits[t] > 0.0f)
        logits[t] /= p;
      else
        logits[t] *= p;
    }
  }
}

// ---------------------------------------------------------------------------
// .myai parsing (header.rs, config.rs, weight_index.rs)
// ---------------------------------------------------------------------------
inline uint32_t rd32(const uint8_t* p) {
  return uint32_t(p[0]) | (uint32_t(p[1]) << 8) | (uint32_t(p[2]) << 16) | (uint32_t(p[3]) << 24);
}

struct Expert {
  size_t gu, gu_s, dn, dn_s, gu_bytes, gu_count;
};
struct Layer {
  size_t rms_attn, qkv, qkv_s, o, o_s, rms_ffn, rw, rb;
  std::vector<Expert> ex;
};
struct Config {
  size_t dim, hidden, layers, heads, hd, vocab, max_seq, experts, top_k, group, depth_layer;
  float theta;
};

struct Index {
  size_t emb, emb_s, final_norm, out, out_s, total;
  std::vector<Layer> L;
};

bool parse(const uint8_t* d, size_t len, Config* c, Index* ix) {
  if (len < 128) {
    g_err = "File too small for header";
    return false;
  }
  uint32_t magic = rd32(d), version = rd32(d + 4);
  if (magic != 0x4D594149u) {
    g_err = "Bad magic";
    return false;
  }
  if (version == 0 || version > 2) {
    g_err = "Unsupported version";
    return false;
  }
  uint32_t ne = 0, tk = 0, gs = 0, dr = 0, ms = 0, th = 0;
  if (version >= 2 && len >= 256) {
    ne = rd32(d + 128), tk = rd32(d + 132), gs = rd32(d + 136), dr = rd32(d + 140),
    ms = rd32(d + 144), th = rd32(d + 148);
  }
  c->dim = rd32(d + 8);
  c->hidden = rd32(d + 12);
  c->layers = rd32(d + 16);
  c->heads = rd32(d + 20);
  c->vocab = rd32(d + 24);
  if (!c->heads || !c->dim) {
    g_err = "zero dim or heads";
    return false;
  }
  c->hd = c->dim / c->heads;
  c->experts = ne >= 2 ? ne : 1;
  size_t k = tk >= 1 ? tk : std::min<size_t>(c->experts, 2);
  c->top_k = std::min(k, c->experts);
  c->group = gs > 0 ? gs : 64;
  c->max_seq = ms > 0 ? ms : 512;
  c->depth_layer = dr;
  c->theta = th == 0 ? 10000.0f : float(th) / 100.0f;

  const size_t dim = c->dim, H = c->hidden, V = c->vocab, G = c->group;
  size_t cur = (c->experts >= 2 || G > 0) ? 256 : 128;
  ix->emb = cur;
  cur += V * dim;
  ix->emb_s = cur;
  cur += V * 4;
  ix->L.resize(c->layers);
  for (auto& l : ix->L) {
    l.rms_attn = cur;
    cur += dim * 4;
    l.qkv = cur;
    cur += 3 * dim * dim;
    l.qkv_s = cur;
    cur += 3 * dim * 4;
    l.o = cur;
    cur += dim * dim;
    l.o_s = cur;
    cur += dim * 4;
    l.rms_ffn = cur;
    cur += dim * 4;
    l.rw = l.rb = 0;
    if (c->experts >= 2) {
      l.rw = cur;
      cur += c->experts * dim * 4;
      l.rb = cur;
      cur += c->experts * 4;
    }
    l.ex.resize(c->experts);
    for (auto& e : l.ex) {
      e.gu = cur;
      e.gu_bytes = 2 * H * ((dim + 1) / 2);
      cur += e.gu_bytes;
      e.gu_s = cur;
      e.gu_count = 2 * H * ((dim + G - 1) / G);
      cur += e.gu_count * 4;
      e.dn = cur;
      cur += dim * ((H + 1) / 2);
      e.dn_s = cur;
      cur += dim * ((H + G - 1) / G) * 4;
    }
  }
  if (c->depth_layer > 0) cur += dim * 32 * 4 + 32 * 4 + 32 * 4 + 4;
  ix->final_norm = cur;
  cur += dim * 4;
  ix->out = cur;
  cur += V * dim;
  ix->out_s = cur;
  cur += V * 4;
  ix->total = cur;
  return true;
}

}  // namespace

// ---------------------------------------------------------------------------
// Engine (engine.rs:94-569)
// ---------------------------------------------------------------------------
struct orc_engine {
  uint8_t* map = nullptr;
  size_t map_len = 0;
  Config c{};
  Index ix{};
  int threads = 0;  // 0: one thread + one thread per selected expert
  std::vector<float> x, xb, q, k, v, att_out, att_scores, logits, kc, vc, cosv, sinv, scores, eout;
  // per-layer trace of the last forward
  bool trace = false;
  std::vector<float> tr_x_attn, tr_x_moe, tr_router, tr_w;
  std::vector<int32_t> tr_sel;

  const int8_t* i8(size_t off) const { return reinterpret_cast<const int8_t*>(map + off); }
  const float* f32(size_t off) const { return reinterpret_cast<const float*>(map + off); }
  const uint8_t* u8(size_t off) const { return map + off; }
};

ORC_API const char* orc_error(void) { return g_err.c_str(); }

ORC_API orc_engine* orc_load(const char* path, int threads) {
  int fd = ::open(path, O_RDONLY);
  if (fd < 0) {
    g_err = std::string("open: ") + path;
    return nullptr;
  }
  struct stat st;
  if (fstat(fd, &st) != 0) {
    ::close(fd);
    g_err = "stat";
    return nullptr;
  }
  size_t len = size_t(st.st_size);
  void* p = mmap(nullptr, len, PROT_READ, MAP_PRIVATE | MAP_POPULATE, fd, 0);
  ::close(fd);
  if (p == MAP_FAILED) {
    g_err = "mmap";
    return nullptr;
  }
  auto* e = new orc_engine();
  e->map = static_cast<uint8_t*>(p);
  e->map_len = len;
  if (!parse(e->map, len, &e->c, &e->ix)) {
    munmap(p, len);
    delete e;
    return nullptr;
  }
  if (len < e->ix.total) {
    g_err = "file smaller than its header implies";
    munmap(p, len);
    delete e;
    return nullptr;
  }
  e->threads = threads;
  const Config& c = e->c;
  const size_t dim = c.dim;
  e->x.assign(dim, 0);
  e->xb.assign(dim, 0);
  e->q.assign(dim, 0);
  e->k.assign(dim, 0);
  e->v.assign(dim, 0);
  e->att_out.assign(dim, 0);
  e->att_scores.assign(c.max_seq, 0);
  e->logits.assign(c.vocab, 0);
  e->kc.assign(c.layers * c.max_seq * dim, 0);
  e->vc.assign(c.layers * c.max_seq * dim, 0);
  e->scores.assign(c.experts, 0);
  e->eout.assign(dim, 0);
  const size_t half = c.hd / 2;
  e->cosv.assign(c.max_seq * half, 0);
  e->sinv.assign(c.max_seq * half, 0);
  for (size_t pos = 0; pos < c.max_seq; ++pos)  // state.rs:53-60
    for (size_t i = 0; i < half; ++i) {
      float freq = 1.0f / std::pow(c.theta, float(2 * i) / float(c.hd));
      float th = float(pos) * freq;
      e->cosv[pos * half + i] = std::cos(th);
      e->sinv[pos * half + i] = std::sin(th);
    }
  return e;
}

ORC_API void orc_free(orc_engine* e) {
  if (!e) return;
  munmap(e->map, e->map_len);
  delete e;
}

ORC_API void orc_set_trace(orc_engine* e, int on) {
  e->trace = on != 0;
  const size_t L = e->c.layers, d = e->c.dim;
  e->tr_x_attn.assign(on ? L * d : 0, 0);
  e->tr_x_moe.assign(on ? L * d : 0, 0);
  e->tr_router.assign(on ? L * e->c.experts : 0, 0);
  e->tr_sel.assign(on ? L * e->c.top_k : 0, -1);
  e->tr_w.assign(on ? L * e->c.top_k : 0, 0);
}

// Copies a trace array of the last forward: 0 x after attention [L][dim],
// 1 x after the FFN [L][dim], 2 router logits [L][E], 3 selected experts
// [L][k] (as float), 4 selected weights [L][k].
ORC_API size_t orc_get_trace(orc_engine* e, int which, float* dst, size_t n) {
  const std::vector<float>* src = nullptr;
  switch (which) {
    case 0: src = &e->tr_x_attn; break;
    case 1: src = &e->tr_x_moe; break;
    case 2: src = &e->tr_router; break;
    case 4: src = &e->tr_w; break;
    case 3: {
      size_t m = std::min(n, e->tr_sel.size());
      for (size_t i = 0; i < m; ++i) dst[i] = float(e->tr_sel[i]);
      return m;
    }
    default: return 0;
  }
  size_t m = std::min(n, src->size());
  std::memcpy(dst, src->data(), m * 4);
  return m;
}

namespace {

// Runs one expert's SwiGLU block on `xin` (engine.rs:353-386).
void run_expert(const orc_engine* e, const Expert& ew, const float* xin, float* out, int threads) {
  const Config& c = e->c;
  const size_t H = c.hidden, dim = c.dim;
  std::vector<float> hb(H), hb2(H);
  const size_t half_bytes = ew.gu_bytes / 2, half_count = ew.gu_count / 2;
  matmul_i4(hb.data(), e->u8(ew.gu), e->f32(ew.gu_s), xin, H, dim, c.group, threads);
  matmul_i4(hb2.data(), e->u8(ew.gu + half_bytes), e->f32(ew.gu_s) + half_count, xin, H, dim,
            c.group, threads);
  swiglu(hb.data(), hb2.data(), H);
  matmul_i4(out, e->u8(ew.dn), e->f32(ew.dn_s), hb.data(), dim, H, c.group, threads);
}

}  // namespace

ORC_API long orc_forward(orc_engine* e, uint32_t token, uint32_t pos) {
  const Config& c = e->c;
  const size_t dim = c.dim, hd = c.hd, half = hd / 2, heads = c.heads;
  if (token >= c.vocab || pos >= c.max_seq) {
    g_err = "token or position out of range";
    return -1;
  }
  const int mt = e->threads > 0 ? e->threads : 1;
  float* x = e->x.data();
  float* xb = e->xb.data();
  // 1. embedding (engine.rs:201-210)
  {
    const int8_t* row = e->i8(e->ix.emb) + size_t(token) * dim;
    float s = e->f32(e->ix.emb_s)[token];
    for (size_t i = 0; i < dim; ++i) x[i] = float(row[i]) * s;
  }
  std::vector<float> tmp(std::max(dim, c.hidden));
  std::vector<int8_t> xq(dim);
  for (size_t l = 0; l < c.layers; ++l) {
    const Layer& L = e->ix.L[l];
    rmsnorm(xb, x, e->f32(L.rms_attn), dim);
    // QKV: three matmul_int8 calls on the same xb quantize identically
    {
      float xs = quantize_i8(xb, xq.data(), dim);
      const int8_t* w = e->i8(L.qkv);
      const float* s = e->f32(L.qkv_s);
      matmul_i8_q(e->q.data(), nullptr, w, s, xq.data(), xs, dim, dim, mt);
      matmul_i8_q(e->k.data(), nullptr, w + dim * dim, s + dim, xq.data(), xs, dim, dim, mt);
      matmul_i8_q(e->v.data(), nullptr, w + 2 * dim * dim, s + 2 * dim, xq.data(), xs, dim, dim, mt);
    }
    // RoPE on interleaved pairs (engine.rs:252-271)
    for (size_t h = 0; h < heads; ++h)
      for (size_t i = 0; i < half; ++i) {
        float ct = e->cosv[pos * half + i], st = e->sinv[pos * half + i];
        size_t b = h * hd + 2 * i;
        float q0 = e->q[b], q1 = e->q[b + 1];
        float a = q0 * ct, bb = q1 * st, cc = q0 * st, dd = q1 * ct;
        e->q[b] = a - bb;
        e->q[b + 1] = cc + dd;
        float k0 = e->k[b], k1 = e->k[b + 1];
        a = k0 * ct, bb = k1 * st, cc = k0 * st, dd = k1 * ct;
        e->k[b] = a - bb;
        e->k[b + 1] = cc + dd;
      }
    const size_t lbase = l * c.max_seq * dim;
    std::memcpy(&e->kc[lbase + pos * dim], e->k.data(), dim * 4);
    std::memcpy(&e->vc[lbase + pos * dim], e->v.data(), dim * 4);
    // attention (engine.rs:283-309)
    std::fill(e->att_out.begin(), e->att_out.end(), 0.0f);
    const float inv_sqrt = 1.0f / std::sqrt(float(hd));
    for (size_t h = 0; h < heads; ++h) {
      const size_t qo = h * hd;
      for (size_t t = 0; t <= pos; ++t) {
        float d = dot_f32(&e->q[qo], &e->kc[lbase + t * dim + qo], hd);
        e->att_scores[t] = soft_cap(d * inv_sqrt, 30.0f);
      }
      softmax(e->att_scores.data(), pos + 1);
      for (size_t t = 0; t <= pos; ++t) {
        const float w = e->att_scores[t];
        const float* vr = &e->vc[lbase + t * dim + qo];
        for (size_t dd = 0; dd < hd; ++dd) {
          float p = w * vr[dd];
          e->att_out[qo + dd] += p;
        }
      }
    }
    // O projection + residual (engine.rs:312-322)
    matmul_i8(xb, e->i8(L.o), e->f32(L.o_s), e->att_out.data(), dim, dim, mt);
    for (size_t i = 0; i < dim; ++i) x[i] += xb[i];
    if (e->trace) std::memcpy(&e->tr_x_attn[l * dim], x, dim * 4);
    // FFN (engine.rs:325-442)
    rmsnorm(xb, x, e->f32(L.rms_ffn), dim);
    if (c.experts >= 2) {
      const float* rw = e->f32(L.rw);
      const float* rb = e->f32(L.rb);
      for (size_t ex = 0; ex < c.experts; ++ex) e->scores[ex] = rb[ex] + dot_f32(rw + ex * dim, xb, dim);
      if (e->trace) std::memcpy(&e->tr_router[l * c.experts], e->scores.data(), c.experts * 4);
      std::vector<int32_t> sel(c.top_k);
      std::vector<float> sw(c.top_k);
      size_t k = softmax_top_k(e->scores.data(), c.experts, c.top_k, sel.data(), sw.data());
      std::vector<std::vector<float>> res(k, std::vector<float>(dim));
      if (e->threads == 0 && k > 1) {
        // rayon par_iter over the selected experts: one thread each
#pragma omp parallel for num_threads(int(k)) schedule(static, 1)
        for (long i = 0; i < long(k); ++i) run_expert(e, L.ex[sel[i]], xb, res[i].data(), 1);
      } else {
        for (size_t i = 0; i < k; ++i) run_expert(e, L.ex[sel[i]], xb, res[i].data(), mt);
      }
      for (size_t i = 0; i < dim; ++i) e->eout[i] = 0.0f;
      for (size_t j = 0; j < k; ++j)
        for (size_t i = 0; i < dim; ++i) {
          float p = sw[j] * res[j][i];
          e->eout[i] += p;
        }
      for (size_t i = 0; i < dim; ++i) x[i] += e->eout[i];
      if (e->trace)
        for (size_t j = 0; j < k; ++j) {
          e->tr_sel[l * c.top_k + j] = sel[j];
          e->tr_w[l * c.top_k + j] = sw[j];
        }
    } else if (!L.ex.empty()) {
      std::vector<float> out(dim);
      run_expert(e, L.ex[0], xb, out.data(), mt);
      for (size_t i = 0; i < dim; ++i) x[i] += out[i];
    }
    if (e->trace) std::memcpy(&e->tr_x_moe[l * dim], x, dim * 4);
  }
  // final norm + logits + argmax (engine.rs:470-493)
  std::memcpy(tmp.data(), x, dim * 4);
  rmsnorm(x, tmp.data(), e->f32(e->ix.final_norm), dim);
  matmul_i8(e->logits.data(), e->i8(e->ix.out), e->f32(e->ix.out_s), x, c.vocab, dim, mt);
  long r = argmax(e->logits.data(), c.vocab);
  if (r < 0) g_err = "NaN in logits";
  return r;
}

// sample_from_logits with the Greedy strategy (engine.rs:551-569).
ORC_API long orc_sample_greedy(orc_engine* e, const uint32_t* hist, size_t nh, float penalty,
                               uint32_t window) {
  if (penalty > 1.0f && nh > 0) {
    size_t w = std::min<size_t>(nh, window);
    repetition_penalty(e->logits.data(), e->logits.size(), hist + (nh - w), w, penalty);
  }
  return argmax(e->logits.data(), e->logits.size());
}

// Engine::generate with the Greedy strategy (engine.rs:497-548).
ORC_API int orc_generate(orc_engine* e, const uint32_t* prompt, size_t n, size_t max_new,
                         float penalty, uint32_t window, const uint32_t* stop, size_t nstop,
                         uint32_t* out, size_t* n_out) {
  const Config& c = e->c;
  std::vector<uint32_t> hist(prompt, prompt + n);
  size_t room = c.max_seq > max_new ? c.max_seq - max_new : 0;
  size_t n_prefill = std::min(n, std::max<size_t>(room, 1));
  for (size_t p = 0; p < n_prefill; ++p) {
    uint32_t t = std::min<uint32_t>(prompt[p], uint32_t(c.vocab - 1));
    if (orc_forward(e, t, uint32_t(p)) < 0) return -1;
  }
  long next = 1;
  if (n_prefill > 0) next = orc_sample_greedy(e, hist.data(), hist.size(), penalty, window);
  if (next < 0) return -1;
  size_t cnt = 0;
  for (size_t step = 0; step < max_new; ++step) {
    size_t pos = n_prefill + step;
    if (pos >= c.max_seq) break;
    bool is_stop = false;
    for (size_t i = 0; i < nstop; ++i) is_stop |= (stop[i] == uint32_t(next));
    if (is_stop) break;
    out[cnt++] = uint32_t(next);
    hist.push_back(uint32_t(next));
    if (orc_forward(e, uint32_t(next), uint32_t(pos)) < 0) return -1;
    next = orc_sample_greedy(e, hist.data(), hist.size(), penalty, window);
    if (next < 0) return -1;
  }
  *n_out = cnt;
  return 0;
}

// Fills KV-cache positions [0, n) of every layer with seeded values so a
// timing sample can run forwards at realistic positions without paying for a
// full prefill. Timing use only: the values are not a model state.
ORC_API void orc_fill_kv_random(orc_engine* e, size_t n, uint64_t seed) {
  const Config& c = e->c;
  n = std::min(n, c.max_seq);
  uint64_t s = seed * 0x9E3779B97F4A7C15ull + 1;
  for (size_t l = 0; l < c.layers; ++l)
    for (size_t p = 0; p < n; ++p)
      for (size_t i = 0; i < c.dim; ++i) {
        s ^= s << 13, s ^= s >> 7, s ^= s << 17;
        float v = float(int64_t(s >> 40) - (1 << 23)) * (1.0f / float(1 << 23));
        e->kc[(l * c.max_seq + p) * c.dim + i] = v;
        e->vc[(l * c.max_seq + p) * c.dim + i] = -v;
      }
}

ORC_API size_t orc_get_logits(orc_engine* e, float* dst, size_t n) {
  size_t m = std::min(n, e->logits.size());
  std::memcpy(dst, e->logits.data(), m * 4);
  return m;
}

// Reads the config: [dim, hidden, layers, heads, head_dim, vocab, max_seq,
// experts, top_k, group, total_bytes].
ORC_API void orc_config(orc_engine* e, uint64_t* out11) {
  const Config& c = e->c;
  uint64_t v[11] = {c.dim, c.hidden, c.layers, c.heads, c.hd, c.vocab, c.max_seq,
                    c.experts, c.top_k, c.group, e->ix.total};
  std::memcpy(out11, v, sizeof v);
}

// ---------------------------------------------------------------------------
// Operator-level entry points (for known-answer and differential tests)
// ---------------------------------------------------------------------------
ORC_API float orc_quantize_i8(const float* x, int8_t* q, size_t n) { return quantize_i8(x, q, n); }

ORC_API void orc_matmul_i8(float* out, const int8_t* w, const float* ws, const float* x,
                           size_t out_dim, size_t in_dim) {
  matmul_i8(out, w, ws, x, out_dim, in_dim, 1);
}

// Integer row dots of matmul_int8 for a given x_q (no float epilogue).
ORC_API void orc_matmul_i8_dots(int32_t* dots, const int8_t* w, const int8_t* xq, size_t out_dim,
                                size_t in_dim) {
  for (size_t r = 0; r < out_dim; ++r) dots[r] = dot_i8(w + r * in_dim, xq, in_dim);
}

ORC_API void orc_matmul_i4(float* out, const uint8_t* wp, const float* ws, const float* x,
                           size_t out_dim, size_t in_dim, size_t group) {
  matmul_i4(out, wp, ws, x, out_dim, in_dim, group ? group : 64, 1);
}

// Per-group integer dots of matmul_int4: gdots[r][g].
ORC_API void orc_matmul_i4_gdots(int32_t* gdots, const uint8_t* wp, const int8_t* xq,
                                 size_t out_dim, size_t in_dim, size_t group) {
  const size_t ng = (in_dim + group - 1) / group, prow = (in_dim + 1) / 2;
  for (size_t r = 0; r < out_dim; ++r)
    for (size_t g = 0; g < ng; ++g)
      gdots[r * ng + g] = dot_i4(wp + r * prow, xq, g * group, std::min((g + 1) * group, in_dim));
}

ORC_API void orc_rmsnorm(float* out, const float* x, const float* w, size_t n) { rmsnorm(out, x, w, n); }
ORC_API void orc_softmax(float* x, size_t n) { softmax(x, n); }
ORC_API float orc_fast_exp(float x) { return fast_exp(x); }
ORC_API float orc_dot_f32(const float* a, const float* b, size_t n) { return dot_f32(a, b, n); }
ORC_API void orc_swiglu(float* g, const float* u, size_t n) { swiglu(g, u, n); }
ORC_API float orc_soft_cap(float x, float cap) { return soft_cap(x, cap); }
ORC_API long orc_argmax(const float* x, size_t n) { return argmax(x, n); }
ORC_API void orc_repetition_penalty(float* l, size_t n, const uint32_t* h, size_t nh, float p) {
  repetition_penalty(l, n, h, nh, p);
}
ORC_API size_t orc_softmax_top_k(float* scores, size_t n, size_t k, int32_t* idx, float* w) {
  return softmax_top_k(scores, n, k, idx, w);
}
ORC_API uint8_t orc_pack_int4(int8_t lo, int8_t hi) {
  return uint8_t((uint8_t(lo + 8) & 0x0F) | ((uint8_t(hi + 8) & 0x0F) << 4));
}
ORC_API void orc_unpack_int4(uint8_t b, int8_t* lo, int8_t* hi) {
  *lo = int8_t(int(b & 0x0F) - 8);
  *hi = int8_t(int((b >> 4) & 0x0F) - 8);
}

// quantize_f32_to_i4 with the fixed group of 64 (quantization.rs:131-162).
ORC_API void orc_quantize_i4(const float* x, size_t n, uint8_t* out, float* scales) {
  const size_t G = 64, ng = (n + G - 1) / G;
  for (size_t g = 0; g < ng; ++g) {
    size_t s = g * G, e = std::min(s + G, n);
    float amax = 0.0f;
    for (size_t j = s; j < e; ++j) amax = std::max(amax, std::fabs(x[j]));
    amax = std::max(amax, 1e-12f);
    float sc = amax / 7.0f;
    scales[g] = sc;
    float inv = 1.0f / sc;
    for (size_t j = s; j < e; j += 2) {
      float a = std::min(std::max(round_half_away(x[j] * inv), -8.0f), 7.0f);
      float b = (j + 1 < e) ? std::min(std::max(round_half_away(x[j + 1] * inv), -8.0f), 7.0f) : 0.0f;
      out[j / 2] = orc_pack_int4(sat_i8(a), sat_i8(b));
    }
  }
}

// The MoE sub-block of one layer for T independent tokens (engine.rs:334-396
// with xb = x[t]): out[t] = sum_k w_k * expert_k(x[t]) in `selected` order.
// `layer_base` is a pointer to the router weights of a layer laid out as in a
// .myai file: W [E][dim] f32, b [E], then E experts.
ORC_API int orc_moe_forward(const float* x, size_t T, const uint8_t* layer_base, size_t dim,
                            size_t hidden, size_t n_experts, size_t top_k, size_t group,
                            float* out, int32_t* sel_out, int threads) {
  const size_t ng_d = (dim + group - 1) / group, ng_h = (hidden + group - 1) / group;
  const size_t gu_bytes = 2 * hidden * ((dim + 1) / 2), gu_cnt = 2 * hidden * ng_d;
  const size_t dn_bytes = dim * ((hidden + 1) / 2), dn_cnt = dim * ng_h;
  const size_t ex_bytes = gu_bytes + gu_cnt * 4 + dn_bytes + dn_cnt * 4;
  const float* rw = reinterpret_cast<const float*>(layer_base);
  const float* rb = rw + n_experts * dim;
  const uint8_t* ex0 = layer_base + n_experts * dim * 4 + n_experts * 4;
  const int nt = threads > 0 ? threads : 1;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nt) if (nt > 1)
  for (long t = 0; t < long(T); ++t) {
    const float* xt = x + size_t(t) * dim;
    std::vector<float> sc(n_experts), hb(hidden), hb2(hidden), y(dim), acc(dim, 0.0f);
    for (size_t e = 0; e < n_experts; ++e) sc[e] = rb[e] + dot_f32(rw + e * dim, xt, dim);
    std::vector<int32_t> sel(top_k);
    std::vector<float> sw(top_k);
    size_t k = softmax_top_k(sc.data(), n_experts, top_k, sel.data(), sw.data());
    for (size_t j = 0; j < k; ++j) {
      const uint8_t* eb = ex0 + size_t(sel[j]) * ex_bytes;
      const float* gus = reinterpret_cast<const float*>(eb + gu_bytes);
      const uint8_t* dn = eb + gu_bytes + gu_cnt * 4;
      const float* dns = reinterpret_cast<const float*>(dn + dn_bytes);
      matmul_i4(hb.data(), eb, gus, xt, hidden, dim, group, 1);
      matmul_i4(hb2.data(), eb + gu_bytes / 2, gus + gu_cnt / 2, xt, hidden, dim, group, 1);
      swiglu(hb.data(), hb2.data(), hidden);
      matmul_i4(y.data(), dn, dns, hb.data(), dim, hidden, group, 1);
      for (size_t i = 0; i < dim; ++i) {
        float p = sw[j] * y[i];
        acc[i] += p;
      }
      if (sel_out) sel_out[size_t(t) * top_k + j] = sel[j];
    }
    std::memcpy(out + size_t(t) * dim, acc.data(), dim * 4);
  }
  return 0;
}

// The expert block (engine.rs:366-380) for rows whose input is already
// quantized (xq, xs, as quantize_f32_to_i8 left it): y = down(swiglu(gate, up))
// of expert[i], experts laid out back to back as in a .myai layer.
ORC_API void orc_expert_rows(const int8_t* xq, const float* xs, const int32_t* expert, size_t n,
                             const uint8_t* experts, size_t dim, size_t hidden, size_t group, float* y,
                             int threads) {
  const size_t ng_d = (dim + group - 1) / group, ng_h = (hidden + group - 1) / group;
  const size_t gu_bytes = 2 * hidden * ((dim + 1) / 2), gu_cnt = 2 * hidden * ng_d;
  const size_t dn_bytes = dim * ((hidden + 1) / 2), dn_cnt = dim * ng_h;
  const size_t ex_bytes = gu_bytes + gu_cnt * 4 + dn_bytes + dn_cnt * 4;
  const int nt = threads > 0 ? threads : 1;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nt) if (nt > 1)
  for (long i = 0; i < long(n); ++i) {
    std::vector<float> g(hidden), u(hidden);
    const uint8_t* eb = experts + size_t(expert[i]) * ex_bytes;
    const float* gus = reinterpret_cast<const float*>(eb + gu_bytes);
    const uint8_t* dn = eb + gu_bytes + gu_cnt * 4;
    const float* dns = reinterpret_cast<const float*>(dn + dn_bytes);
    const int8_t* xr = xq + size_t(i) * dim;
    matmul_i4_q(g.data(), nullptr, eb, gus, xr, xs[i], hidden, dim, group, 1);
    matmul_i4_q(u.data(), nullptr, eb + gu_bytes / 2, gus + gu_cnt / 2, xr, xs[i], hidden, dim, group, 1);
    swiglu(g.data(), u.data(), hidden);
    matmul_i4(y + size_t(i) * dim, dn, dns, g.data(), dim, hidden, group, 1);
  }
}

// ---------------------------------------------------------------------------
// Paged int8 KV cache of the long-context decode workload (a new format, not
// the reference's PagedKVCache): pages of P tokens; the K block and the V block
// of each head in a page (P x hd values, token-major) are quantized as one
// vector with quantize_f32_to_i8's rule (absmax/127, round to nearest even).
// data [page][K|V][head][P x hd] int8 (K blocks token-major [P][hd], V blocks
// dim-major [hd][P]), scales [page][K|V][head] f32. k, v: [n][P][H][hd] f32, the tokens of page page_ids[i] in order.
ORC_API void orc_paged_store(int8_t* data, float* scales, const int32_t* page_ids, size_t n, size_t P,
                             size_t H, size_t hd, const float* k, const float* v) {
  std::vector<float> blk(P * hd);
  for (size_t i = 0; i < n; ++i) {
    const size_t page = size_t(page_ids[i]);
    for (size_t kv = 0; kv < 2; ++kv) {
      const float* src = kv ? v : k;
      for (size_t h = 0; h < H; ++h) {
        for (size_t t = 0; t < P; ++t)
          std::memcpy(&blk[t * hd], src + ((i * P + t) * H + h) * hd, hd * 4);
        const size_t b = (page * 2 + kv) * H + h;
        if (kv == 0) {
          scales[b] = quantize_i8(blk.data(), data + b * P * hd, P * hd);
        } else {  // V blocks are stored dim-major: [hd][P]
          std::vector<int8_t> qb(P * hd);
          scales[b] = quantize_i8(blk.data(), qb.data(), P * hd);
          for (size_t t = 0; t < P; ++t)
            for (size_t d = 0; d < hd; ++d) data[b * P * hd + d * P + t] = qb[t * hd + d];
        }
      }
    }
  }
}

// Decode-step attention of n_seq sequences over that cache: the attention of
// Engine::forward (engine.rs:283-309) on the dequantized rows (value as f32 *
// scale, as KVPage::dequantize_row does, memory.rs:69-74): per head, scores
// soft_cap(dot_f32(q, k_t) / sqrt(hd), 30), softmax, o = sum_t w_t * v_t in t
// order. q, out: [n_seq][H][hd].
ORC_API void orc_paged_attention(const int8_t* data, const float* scales, const int32_t* page_table,
                                 size_t max_pages, const int32_t* lens, size_t n_seq, size_t P, size_t H,
                                 size_t hd, const float* q, float* out, int threads) {
  const float inv_sqrt = 1.0f / std::sqrt(float(hd));
  const int nt = threads > 0 ? threads : 1;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nt) if (nt > 1)
  for (long sh = 0; sh < long(n_seq * H); ++sh) {
    const size_t s = size_t(sh) / H, h = size_t(sh) % H;
    const size_t L = size_t(lens[s]);
    const float* qh = q + (s * H + h) * hd;
    std::vector<float> sc(L), row(hd), o(hd, 0.0f);
    for (size_t t = 0; t < L; ++t) {
      const size_t page = size_t(page_table[s * max_pages + t / P]), off = t % P;
      const size_t b = (page * 2 + 0) * H + h;
      const int8_t* kr = data + b * P * hd + off * hd;
      for (size_t d = 0; d < hd; ++d) row[d] = float(kr[d]) * scales[b];
      sc[t] = soft_cap(dot_f32(qh, row.data(), hd) * inv_sqrt, 30.0f);
    }
    softmax(sc.data(), L);
    for (size_t t = 0; t < L; ++t) {
      const size_t page = size_t(page_table[s * max_pages + t / P]), off = t % P;
      const size_t b = (page * 2 + 1) * H + h;
      const int8_t* vb = data + b * P * hd;
      for (size_t d = 0; d < hd; ++d) {
        float p = sc[t] * (float(vb[d * P + off]) * scales[b]);
        o[d] += p;
      }
    }
    std::memcpy(out + (s * H + h) * hd, o.data(), hd * 4);
  }
}

// ---------------------------------------------------------------------------
// PagedKVCache (src/model/memory.rs:26-201), restated: pages of 256 tokens per
// layer in a map, an LRU queue of (layer, page), eviction of the queue's front
// when the cache holds 16 * n_layers pages (checked before every write, even
// to a page that exists), per-row int8 quantization with scale = max|x|/127
// (1.0 for an all-zero row) and a truncating `as i8` after clamp [-128, 127].
// ---------------------------------------------------------------------------
struct orc_kvc {
  size_t dim, n_layers, max_pages;
  std::vector<std::map<size_t, std::pair<std::vector<int8_t>, std::vector<float>>>> pages;  // k|v, scales
  std::deque<std::pair<size_t, size_t>> lru;
};

namespace {
constexpr size_t kRefPage = 256;

// KVPage::quantize_row (memory.rs:58-66)
void kv_quantize_row(const float* row, size_t n, int8_t* out, float* scale) {
  float mx = 0.0f;
  for (size_t i = 0; i < n; ++i) mx = std::fmax(mx, std::fabs(row[i]));  // fold(0.0, f32::max)
  const float s = mx > 0.0f ? mx / 127.0f : 1.0f;
  *scale = s;
  for (size_t i = 0; i < n; ++i) {
    float v = row[i] / s;
    if (v != v) {
      out[i] = 0;
      continue;
    }
    v = std::min(std::max(v, -128.0f), 127.0f);
    out[i] = int8_t(v);  // truncation toward zero, as `as i8`
  }
}
}  // namespace

ORC_API orc_kvc* orc_kvc_create(size_t kv_dim, size_t n_layers, size_t max_pages_per_layer) {
  orc_kvc* c = new orc_kvc;
  c->dim = kv_dim;
  c->n_layers = n_layers;
  c->max_pages = (max_pages_per_layer ? max_pages_per_layer : 16) * n_layers;
  c->pages.resize(n_layers);
  return c;
}
ORC_API void orc_kvc_free(orc_kvc* c) { delete c; }

ORC_API void orc_kvc_write(orc_kvc* c, size_t layer, size_t pos, const float* k, const float* v) {
  const size_t page = pos / kRefPage, off = pos % kRefPage, d = c->dim;
  size_t total = 0;
  for (auto& m : c->pages) total += m.size();
  if (total >= c->max_pages && !c->lru.empty()) {  // evict_if_full (memory.rs:137-145)
    auto lp = c->lru.front();
    c->lru.pop_front();
    c->pages[lp.first].erase(lp.second);
  }
  for (auto it = c->lru.begin(); it != c->lru.end();)
    it = (it->first == layer && it->second == page) ? c->lru.erase(it) : it + 1;
  c->lru.push_back({layer, page});
  auto& m = c->pages[layer];
  auto f = m.find(page);
  if (f == m.end())
    f = m.emplace(page, std::make_pair(std::vector<int8_t>(2 * kRefPage * d, 0), std::vector<float>(2 * kRefPage, 1.0f)))
            .first;
  kv_quantize_row(k, d, f->second.first.data() + off * d, &f->second.second[off]);
  kv_quantize_row(v, d, f->second.first.data() + (kRefPage + off) * d, &f->second.second[kRefPage + off]);
}

ORC_API int orc_kvc_read(const orc_kvc* c, size_t layer, size_t pos, float* k_out, float* v_out) {
  const size_t page = pos / kRefPage, off = pos % kRefPage, d = c->dim;
  auto f = c->pages[layer].find(page);
  if (f == c->pages[layer].end()) return 0;
  for (size_t i = 0; i < d; ++i) {
    k_out[i] = float(f->second.first[off * d + i]) * f->second.second[off];
    v_out[i] = float(f->second.first[(kRefPage + off) * d + i]) * f->second.second[kRefPage + off];
  }
  return 1;
}

ORC_API void orc_kvc_clear(orc_kvc* c) {
  for (auto& m : c->pages) m.clear();
  c->lru.clear();
}

ORC_API size_t orc_kvc_active_pages(const orc_kvc* c) {
  size_t t = 0;
  for (auto& m : c->pages) t += m.size();
  return t;
}

// ---------------------------------------------------------------------------
// Sampling strategies (src/tensor/sampling.rs:45-165) for a given draw r in
// [0, 1) instead of the clock-seeded random_f32. The descending sorts are
// stable with the lower index first among equal values (sort_unstable_by
// leaves that order unspecified). *margin receives how far r lies from the
// running-sum boundaries of the chosen token (the normalised units r is
// compared in): a draw closer than rounding to a boundary may legitimately
// pick the neighbour in another summation order.
// strategy: 0 greedy, 1 top-k, 2 top-p, 3 min-p.
ORC_API long orc_sample(const float* logits_in, size_t n, int strategy, float temperature, size_t top_k,
                        float top_p, float min_p, float r, float* margin) {
  std::vector<float> l(logits_in, logits_in + n);
  *margin = 1.0f;
  if (strategy == 0) return argmax(l.data(), n);
  auto desc = [&](std::vector<size_t>& idx) {
    std::stable_sort(idx.begin(), idx.end(), [&](size_t a, size_t b) { return l[a] > l[b]; });
  };
  auto pick = [&](const std::vector<size_t>& idx, const std::vector<float>& probs) -> long {
    float cum = 0.0f;
    for (size_t i = 0; i < probs.size(); ++i) {
      const float before = cum;
      cum += probs[i];
      if (r < cum) {
        *margin = std::min(r - before, cum - r);
        return long(idx[i]);
      }
    }
    *margin = 0.0f;
    return long(idx.back());
  };
  if (strategy == 1) {  // sample_top_k (sampling.rs:45-78)
    if (temperature > 0.0f) {
      const float inv_t = 1.0f / temperature;
      for (auto& v : l) v *= inv_t;
    }
    std::vector<size_t> idx(n);
    for (size_t i = 0; i < n; ++i) idx[i] = i;
    desc(idx);
    idx.resize(std::min(top_k, n));
    const float mx = l[idx[0]];
    std::vector<float> probs;
    for (size_t i : idx) probs.push_back(std::exp(l[i] - mx));
    float sum = 0.0f;
    for (float p : probs) sum += p;
    for (auto& p : probs) p /= sum;
    return pick(idx, probs);
  }
  if (temperature > 0.0f && temperature != 1.0f) {
    const float inv_t = 1.0f / temperature;
    for (auto& v : l) v *= inv_t;
  }
  softmax(l.data(), n);
  if (strategy == 2) {  // sample_top_p (sampling.rs:83-124)
    std::vector<size_t> idx(n);
    for (size_t i = 0; i < n; ++i) idx[i] = i;
    desc(idx);
    float cumulative = 0.0f;
    size_t cutoff = n;
    for (size_t rank = 0; rank < n; ++rank) {
      cumulative += l[idx[rank]];
      if (cumulative > top_p) {
        cutoff = rank + 1;
        break;
      }
    }
    idx.resize(cutoff);
    std::vector<float> probs;
    for (size_t i : idx) probs.push_back(l[i]);
    float sum = 0.0f;
    for (float p : probs) sum += p;
    if (sum > 1e-12f)
      for (auto& p : probs) p /= sum;
    return pick(idx, probs);
  }
  // sample_min_p (sampling.rs:129-165)
  float max_prob = 0.0f;
  for (float v : l) max_prob = std::fmax(max_prob, v);
  const float threshold = max_prob * min_p;
  std::vector<size_t> idx;
  for (size_t i = 0; i < n; ++i)
    if (l[i] >= threshold) idx.push_back(i);
  if (idx.empty()) return argmax(l.data(), n);
  std::vector<float> probs;
  for (size_t i : idx) probs.push_back(l[i]);
  float sum = 0.0f;
  for (float p : probs) sum += p;
  if (sum > 1e-12f)
    for (auto& p : probs) p /= sum;
  return pick(idx, probs);
}

ORC_API int orc_hw_threads(void) { return omp_get_num_procs(); }
