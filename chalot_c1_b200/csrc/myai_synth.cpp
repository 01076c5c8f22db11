// myai_synth.cpp — writes a seeded synthetic .myai v2 model.
//
// Weights are drawn N(0, std) and quantized the way the reference's own
// quantizers do it:
//   * int8 tensors (embedding, QKV, O, lm_head): one absmax over the whole
//     tensor, scale = absmax/127, q = round-half-even(clamp(w * (1/scale), ±127))
//     (src/tensor/quantization.rs:56-104); the scale is written into every
//     per-row slot the format has.
//   * int4 expert tensors: per row, per group of `int4_group_size`,
//     scale = absmax/7, q = round-half-away(w * (1/scale)) clamped to [-8, 7]
//     (src/tensor/quantization.rs:131-162), packed low nibble = even element
//     (src/tensor/quantization.rs:122-126).
//   * RMSNorm weights 1.0, router weights N(0, std) in f32, router bias 0,
//     depth router absent.
// The normal deviates come from single-precision Box-Muller over SplitMix64
// counters keyed by (seed, tensor id, element pair), so the file does not
// depend on the thread count.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "capi_internal.h"
#include "myai.h"

namespace chalot {
namespace {

inline uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

struct Rng {
  uint64_t key;
  // Fills out[i] for i in [begin, end) of the stream: element 2p and 2p+1 are
  // the cosine and sine branches of one Box-Muller pair.
  void fill(float* out, size_t begin, size_t end, float std) const {
    for (size_t i = begin & ~size_t(1); i < end; i += 2) {
      uint64_t h = splitmix64(key + i);
      float u1 = float((h >> 40) + 1) * (1.0f / 16777216.0f);  // (0, 1]
      float u2 = float((h >> 16) & 0xFFFFFF) * (1.0f / 16777216.0f);
      float r = std::sqrt(-2.0f * std::log(u1));
      float a = 6.28318530717958647f * u2;
      if (i >= begin) out[i - begin] = r * std::cos(a) * std;
      if (i + 1 >= begin && i + 1 < end) out[i + 1 - begin] = r * std::sin(a) * std;
    }
  }
};

Rng stream(uint64_t seed, uint64_t tensor_id) {
  return Rng{splitmix64(seed * 0x100000001B3ull ^ splitmix64(tensor_id + 0x51ull))};
}

template <class F>
void parallel_for(size_t n, int threads, F f) {
  if (threads <= 1 || n < 4096) {
    f(size_t(0), n);
    return;
  }
  std::vector<std::thread> ts;
  size_t chunk = (n + threads - 1) / threads;
  chunk = (chunk + 63) & ~size_t(63);
  for (int t = 0; t < threads; ++t) {
    size_t b = size_t(t) * chunk, e = std::min(n, b + chunk);
    if (b >= e) break;
    ts.emplace_back([=] { f(b, e); });
  }
  for (auto& t : ts) t.join();
}

class Writer {
 public:
  explicit Writer(FILE* f) : f_(f) {}
  bool put(const void* p, size_t n) {
    if (n && std::fwrite(p, 1, n, f_) != n) return false;
    pos_ += n;
    return true;
  }
  size_t pos() const { return pos_; }

 private:
  FILE* f_;
  size_t pos_ = 0;
};

// Generates an f32 tensor of `n` elements from stream `id`.
std::vector<float> gen(uint64_t seed, uint64_t id, size_t n, float std, int threads) {
  std::vector<float> v(n);
  Rng r = stream(seed, id);
  parallel_for(n, threads, [&](size_t b, size_t e) { r.fill(v.data() + b, b, e, std); });
  return v;
}

// Per-tensor absmax int8 (rows x cols); returns the scale.
float quant_i8_tensor(const std::vector<float>& w, std::vector<int8_t>* q, int threads) {
  const size_t n = w.size();
  std::vector<float> part(std::max(threads, 1), 0.0f);
  std::vector<std::thread> ts;
  size_t chunk = (n + part.size() - 1) / part.size();
  for (size_t t = 0; t < part.size(); ++t) {
    ts.emplace_back([&, t] {
      float m = 0.0f;
      for (size_t i = t * chunk; i < std::min(n, (t + 1) * chunk); ++i) m = std::max(m, std::fabs(w[i]));
      part[t] = m;
    });
  }
  for (auto& t : ts) t.join();
  float amax = 0.0f;
  for (float m : part) amax = std::max(amax, m);
  amax = std::max(amax, 1e-12f);
  const float scale = amax / 127.0f;
  const float inv = 1.0f / scale;
  q->resize(n);
  parallel_for(n, threads, [&](size_t b, size_t e) {
    for (size_t i = b; i < e; ++i) {
      float s = w[i] * inv;
      s = std::min(std::max(s, -127.0f), 127.0f);
      (*q)[i] = int8_t(std::nearbyint(s));
    }
  });
  return scale;
}

// Per-row, per-group int4 quantization of a [rows x cols] tensor.
void quant_i4_rows(const std::vector<float>& w, size_t rows, size_t cols, size_t group,
                   std::vector<uint8_t>* packed, std::vector<float>* scales, int threads) {
  const size_t prow = (cols + 1) / 2, ng = (cols + group - 1) / group;
  packed->assign(rows * prow, 0);
  scales->assign(rows * ng, 0.0f);
  parallel_for(rows, threads, [&](size_t rb, size_t re) {
    std::vector<int8_t> q(cols + 1, 0);
    for (size_t r = rb; r < re; ++r) {
      const float* x = w.data() + r * cols;
      for (size_t g = 0; g < ng; ++g) {
        size_t s = g * group, e = std::min(s + group, cols);
        float amax = 0.0f;
        for (size_t j = s; j < e; ++j) amax = std::max(amax, std::fabs(x[j]));
        amax = std::max(amax, 1e-12f);
        float scale = amax / 7.0f;
        float inv = 1.0f / scale;
        (*scales)[r * ng + g] = scale;
        for (size_t j = s; j < e; ++j) {
          float v = std::round(x[j] * inv);
          q[j] = int8_t(std::min(std::max(v, -8.0f), 7.0f));
        }
      }
      q[cols] = 0;
      uint8_t* out = packed->data() + r * prow;
      for (size_t j = 0; j < prow; ++j) {
        int lo = q[2 * j], hi = (2 * j + 1 < cols) ? q[2 * j + 1] : 0;
        out[j] = uint8_t(((lo + 8) & 0x0F) | (((hi + 8) & 0x0F) << 4));
      }
    }
  });
}

enum TensorKind : uint64_t { kEmbed = 1, kQKV = 2, kO = 3, kRouter = 4, kGateUp = 5, kDown = 6, kOut = 7 };
uint64_t tid(uint64_t kind, uint64_t layer, uint64_t expert) { return (kind << 40) | (layer << 20) | expert; }

}  // namespace

int write_synthetic(const char* path, const chalot_synth_spec& sp, std::string* err) {
  if (!sp.dim || !sp.n_layers || !sp.n_heads || !sp.vocab_size || !sp.hidden_dim ||
      sp.dim % sp.n_heads) {
    *err = "synthetic spec: dim, hidden_dim, n_layers, n_heads, vocab_size must be non-zero and dim % n_heads == 0";
    return CHALOT_ERR_ARG;
  }
  FileHeader h;
  h.magic = kMyaiMagic;
  h.version = 2;
  h.dim = sp.dim;
  h.hidden_dim = sp.hidden_dim;
  h.n_layers = sp.n_layers;
  h.n_heads = sp.n_heads;
  h.vocab_size = sp.vocab_size;
  h.flags = sp.n_experts >= 2 ? 0b111u : 0b011u;
  h.n_experts = sp.n_experts;
  h.top_k = sp.top_k;
  h.int4_group_size = sp.int4_group_size;
  h.depth_router_layer = 0;
  h.max_seq_len = sp.max_seq_len;
  h.rope_theta_x100 = sp.rope_theta_x100;
  const ModelConfig cfg = config_from_header(h);
  const WeightIndex idx = build_index(cfg);
  const int th = sp.n_threads > 0 ? sp.n_threads : int(std::max(1u, std::thread::hardware_concurrency()));
  const float std = sp.weight_std > 0 ? sp.weight_std : 0.02f;
  const uint64_t seed = sp.seed;
  const size_t d = cfg.dim, H = cfg.hidden_dim, V = cfg.vocab_size, G = cfg.int4_group_size;

  FILE* f = std::fopen(path, "wb");
  if (!f) {
    *err = std::string("open for write: ") + path;
    return CHALOT_ERR_IO;
  }
  std::vector<char> fbuf(1 << 22);
  std::setvbuf(f, fbuf.data(), _IOFBF, fbuf.size());
  Writer w(f);
  bool ok = true;
  auto check = [&](size_t expect) {
    if (w.pos() != expect) ok = false;
  };
  uint8_t hdr[kHeaderSize];
  write_header(h, hdr);
  ok &= w.put(hdr, idx.header_bytes);

  auto int8_tensor = [&](uint64_t id, size_t rows, size_t cols) {
    std::vector<float> x = gen(seed, id, rows * cols, std, th);
    std::vector<int8_t> q;
    float s = quant_i8_tensor(x, &q, th);
    ok &= w.put(q.data(), q.size());
    std::vector<float> sc(rows, s);
    ok &= w.put(sc.data(), rows * 4);
  };
  std::vector<float> ones(std::max(d, size_t(1)), 1.0f);

  check(idx.embed_offset);
  int8_tensor(tid(kEmbed, 0, 0), V, d);
  for (size_t l = 0; l < cfg.n_layers && ok; ++l) {
    const LayerIndex& L = idx.layers[l];
    check(L.rms_attn_offset);
    ok &= w.put(ones.data(), d * 4);
    check(L.attn_qkv_offset);
    int8_tensor(tid(kQKV, l, 0), 3 * d, d);
    check(L.attn_out_offset);
    int8_tensor(tid(kO, l, 0), d, d);
    check(L.rms_ffn_offset);
    ok &= w.put(ones.data(), d * 4);
    if (cfg.n_experts >= 2) {
      check(L.router_w_offset);
      std::vector<float> rw = gen(seed, tid(kRouter, l, 0), cfg.n_experts * d, std, th);
      ok &= w.put(rw.data(), rw.size() * 4);
      std::vector<float> rb(cfg.n_experts, 0.0f);
      ok &= w.put(rb.data(), rb.size() * 4);
    }
    for (size_t e = 0; e < cfg.n_experts && ok; ++e) {
      const ExpertIndex& E = L.experts[e];
      std::vector<uint8_t> p;
      std::vector<float> s;
      check(E.gate_up_offset);
      {
        std::vector<float> x = gen(seed, tid(kGateUp, l, e), 2 * H * d, std, th);
        quant_i4_rows(x, 2 * H, d, G, &p, &s, th);
      }
      ok &= w.put(p.data(), p.size());
      ok &= w.put(s.data(), s.size() * 4);
      check(E.down_offset);
      {
        std::vector<float> x = gen(seed, tid(kDown, l, e), d * H, std, th);
        quant_i4_rows(x, d, H, G, &p, &s, th);
      }
      ok &= w.put(p.data(), p.size());
      ok &= w.put(s.data(), s.size() * 4);
    }
  }
  check(idx.final_norm_offset);
  ok &= w.put(ones.data(), d * 4);
  check(idx.output_proj_offset);
  int8_tensor(tid(kOut, 0, 0), V, d);
  check(idx.total_bytes);
  if (std::fclose(f) != 0) ok = false;
  if (!ok) {
    *err = std::string("writing synthetic model failed: ") + path;
    return CHALOT_ERR_IO;
  }
  return CHALOT_OK;
}

}  // namespace chalot
