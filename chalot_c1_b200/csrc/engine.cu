// engine.cu — host engine behind the C ABI: Engine::load / forward / generate /
// sample_from_logits (src/model/engine.rs:94-569) on one B200.
//
// Load parses the .myai header (myai.cpp), copies every tensor the decode path
// reads into one device allocation at 256-byte aligned offsets, builds the
// RoPE tables on the host with the same libm calls as InferenceState::new
// (src/model/state.rs:53-60) and allocates the f32 KV cache
// [layer][max_seq][dim] (state.rs:45, 73-74).
//
// One forward is a fixed sequence of kernels that read the token and position
// from a device StepState, so it is captured once into a CUDA graph and
// replayed for every position. Greedy generation without a penalty or stop
// tokens runs entirely on the device: after each forward the advance kernel
// stores the argmax and feeds either the next prompt token or the argmax back
// in, so prefill + decode is one stream of graph launches with no host round
// trip until the tokens are copied back.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <array>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "batch.h"
#include "capi_internal.h"
#include "devstat.h"
#include "ep_link.h"
#include "kernels.cuh"
#include "moe_layer.h"
#include "myai.h"
#include "pdl.cuh"
#include "persist.h"

namespace chalot {

struct CudaFail {
  int code;
  std::string msg;
};

#define CK(call)                                                                         \
  do {                                                                                   \
    cudaError_t e_ = (call);                                                             \
    if (e_ != cudaSuccess)                                                               \
      throw CudaFail{e_ == cudaErrorMemoryAllocation ? CHALOT_ERR_OOM : CHALOT_ERR_CUDA, \
                     std::string(#call) + ": " + cudaGetErrorString(e_)};                \
  } while (0)

class MappedFile {
 public:
  ~MappedFile() {
    if (p_) munmap(p_, n_);
  }
  bool open(const char* path, std::string* err) {
    int fd = ::open(path, O_RDONLY);
    if (fd < 0) {
      *err = std::string("open: ") + path;
      return false;
    }
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size <= 0) {
      ::close(fd);
      *err = std::string("stat: ") + path;
      return false;
    }
    n_ = size_t(st.st_size);
    p_ = mmap(nullptr, n_, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (p_ == MAP_FAILED) {
      p_ = nullptr;
      *err = "mmap failed";
      return false;
    }
    return true;
  }
  const uint8_t* data() const { return static_cast<const uint8_t*>(p_); }
  size_t size() const { return n_; }

 private:
  void* p_ = nullptr;
  size_t n_ = 0;
};

}  // namespace chalot

#ifdef CHALOT_PHASE_TRACE
namespace chalot {
cudaError_t trace_dense(unsigned long long*, size_t);
cudaError_t trace_moe(unsigned long long*, size_t);
cudaError_t trace_attn(unsigned long long*, size_t);
cudaError_t trace_dense_clear();
cudaError_t trace_moe_clear();
cudaError_t trace_attn_clear();
}  // namespace chalot
#endif

using namespace chalot;

struct chalot_engine {
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;
  ModelConfig cfg;
  WeightIndex idx;
  Dims dims{};
  uint8_t* d_weights = nullptr;
  size_t weight_bytes = 0;
  ExpertPtrs* d_experts = nullptr;
  std::vector<LayerPtrs> layers;
  std::vector<std::vector<ExpertPtrs>> host_experts;
  const int8_t* emb = nullptr;
  const float* emb_s = nullptr;
  const float* final_norm = nullptr;
  const int8_t* out_w = nullptr;
  const float* out_s = nullptr;
  DecodeBufs b{};
  std::vector<void*> allocs;
  StepState* h_state = nullptr;  // pinned: device-state readback
  StepState* h_stage = nullptr;  // pinned: one StepState per in-flight host->device copy
  size_t n_stage = 0, next_stage = 0;
  uint32_t* h_tokens = nullptr;  // pinned, [max_seq]
  uint32_t* d_hist = nullptr;    // [2*max_seq] token history for the penalty
  bool use_graph = true;
  // the persistent one-kernel decode step (k_persist.cu), when the shape fits
  bool use_persist = false;
  PersistArgs pargs{};
  cudaGraphExec_t g_fwd = nullptr;   // embed .. lm_head
  cudaGraphExec_t g_step = nullptr;  // embed .. lm_head + advance
  cudaEvent_t ev[3] = {nullptr, nullptr, nullptr};
  double last_prefill_ms = 0, last_decode_ms = 0;
  uint32_t last_n_prefill = 0, last_n_decode = 0;
  uint64_t rng = 0;  // splitmix64 state of the sampling draws
  // batched decode (chalot_batch_reserve / chalot_forward_batch)
  struct Batch {
    int cap = 0;
    float *kc = nullptr, *vc = nullptr, *x = nullptr, *qkv = nullptr, *q = nullptr, *scores = nullptr;
    float *att = nullptr, *xb = nullptr, *eout = nullptr, *logits = nullptr, *xs = nullptr;
    int8_t* xq = nullptr;
    int32_t *pos = nullptr, *slot = nullptr;
    uint32_t *toks = nullptr, *out = nullptr;
    void* moe_ws = nullptr;
    uint32_t* h_io = nullptr;  // pinned staging: slots, tokens, positions, results
    std::vector<MlExperts> experts;  // per layer, the engine's repacked experts
    // paged K/V (chalot_batch_reserve_paged): kc/vc are pools of n_pages pages
    // of 2^pt_shift positions ([layer][position][dim] each); a slot's pages are
    // taken from the free list as its positions grow and returned by
    // chalot_batch_release
    int pt_shift = -1, maxp = 0, n_pages = 0;  // pt_shift < 0: the flat cache
    int32_t* ptab = nullptr;    // device [cap][maxp]: page of each slot's page index
    int32_t* h_ptab = nullptr;  // pinned copy, uploaded before a forward that changed it
    std::vector<std::vector<int>> slot_pages;
    std::vector<int> free_pages;
  } bt;
  // expert parallelism of the batched forward: this engine computes the
  // experts e with e % world == rank and exchanges token rows with its peers
  std::unique_ptr<EpLink> ep;
  struct EpBufs {
    int cap = 0, world = 0;  // sized for cap tokens per rank and world ranks
    // blocks of R1 = cap*K rows, one per peer
    int8_t* rows = nullptr;     // [world][R1][dim] rows to send
    float* rscale = nullptr;    // [world][R1]
    int8_t* rrows = nullptr;    // [world][R1][dim] rows received
    float* rrscale = nullptr;   // [world][R1]
    int32_t* rexp = nullptr;    // [world][R1] local expert of each received row (-1: padding)
    float* y = nullptr;         // [world][R1][dim] outputs of the received rows
    float* yback = nullptr;     // [world][R1][dim] outputs of my rows
    int32_t* ppos = nullptr;    // [cap*K] row of each of my slots in those blocks
    int32_t* offs = nullptr;    // [E+1] plan offsets (rank-major, then local expert)
    int32_t* cnt = nullptr;     // [2][world*El] counts sent / received
    void* ws = nullptr;         // expert workspace for world*R1 rows
  } epb;

  ~chalot_engine() {
    if (g_fwd) cudaGraphExecDestroy(g_fwd);
    if (g_step) cudaGraphExecDestroy(g_step);
    for (auto& e : ev)
      if (e) cudaEventDestroy(e);
    for (void* p : allocs) cudaFree(p);
    if (d_weights) cudaFree(d_weights);
    if (h_state) cudaFreeHost(h_state);
    if (h_stage) cudaFreeHost(h_stage);
    if (h_tokens) cudaFreeHost(h_tokens);
    if (bt.h_io) cudaFreeHost(bt.h_io);
    if (bt.h_ptab) cudaFreeHost(bt.h_ptab);
    if (stream) cudaStreamDestroy(stream);
  }

  template <class T>
  T* dalloc(size_t n) {
    void* p = nullptr;
    CK(cudaMalloc(&p, std::max<size_t>(n * sizeof(T), 16)));
    CK(cudaMemset(p, 0, std::max<size_t>(n * sizeof(T), 16)));
    allocs.push_back(p);
    return static_cast<T*>(p);
  }

  // One forward: every kernel after the first is launched with programmatic
  // dependent launch so it can load its weights while its predecessor runs.
  // With `marks`, an event is recorded after every kernel (and PDL is off):
  // the per-kernel profile of chalot_profile_forward.
  void record_forward(cudaStream_t s, bool with_advance, cudaEvent_t* marks = nullptr) {
    const Dims& d = dims;
    const bool pdl = marks == nullptr;
    int m = 0;
    auto mark = [&]() {
      if (marks) cudaEventRecordWithFlags(marks[m++], s, cudaEventRecordExternal);
    };
    if (use_persist && !marks) {  // the whole step in one cooperative launch
      CK(launch_persist(pargs, num_sms, s));
      CK(launch_persist_epoch(const_cast<unsigned*>(pargs.epoch), pargs.ll.cnt, s));
      if (with_advance) launch_advance(d, b, s, false);
      return;
    }
    mark();
    launch_embed(d, emb, emb_s, b, s);
    mark();
    for (int l = 0; l < d.n_layers; ++l) {
      const LayerPtrs& L = layers[l];
      // the last layer's down kernel also computes rmsnorm(x, final_norm) for the lm_head
      const float* next_norm = (l + 1 < d.n_layers) ? nullptr : final_norm;
      launch_qkv(d, L, l, b, s, pdl);
      mark();
      launch_scores(d, l, b, s, pdl);
      mark();
      launch_pv(d, l, b, s, pdl);
      mark();
      launch_oproj(d, L, l, b, s, pdl);
      mark();
      launch_gateup(d, L, l, b, s, pdl);
      mark();
      launch_down(d, L, l, next_norm, b, s, pdl);
      mark();
    }
    launch_lmhead(d, out_w, out_s, b, num_sms, s, pdl);
    mark();
    if (with_advance) {
      launch_advance(d, b, s, pdl);
      mark();
    }
  }

  cudaGraphExec_t capture(bool with_advance) {
    cudaGraph_t g = nullptr;
    CK(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
    record_forward(stream, with_advance);
    cudaError_t le = cudaGetLastError();
    CK(cudaStreamEndCapture(stream, &g));
    CK(le);
    cudaGraphExec_t ex = nullptr;
    cudaError_t ie = cudaGraphInstantiate(&ex, g, 0);
    cudaGraphDestroy(g);
    CK(ie);
    return ex;
  }

  void run_forward(bool with_advance) {
    if (use_graph) {
      CK(cudaGraphLaunch(with_advance ? g_step : g_fwd, stream));
    } else {
      record_forward(stream, with_advance);
      CK(cudaGetLastError());
    }
  }

  // After a synchronize: a bounded device wait that gave up leaves b.err set;
  // report it and clear the error word and the last-CTA tickets.
  void check_device_error() {
    unsigned h = 0;
    CK(cudaMemcpy(&h, b.err, sizeof h, cudaMemcpyDeviceToHost));
    if (h) {
      CK(cudaMemset(b.err, 0, 4 * sizeof(unsigned)));
      CK(cudaMemset(b.counters, 0, kTickets * sizeof(unsigned)));
      throw CudaFail{CHALOT_ERR_TIMEOUT, "a device wait for a bulk copy timed out"};
    }
  }

  // Stages the state of the next forward. Each call uses its own pinned slot
  // (the copy is asynchronous: a slot is reused only after n_stage calls, and
  // callers synchronize at least once per n_stage forwards).
  void set_state(uint32_t pos, uint32_t token, uint32_t n_prefill, uint32_t step) {
    StepState* h = h_stage + (next_stage++ % n_stage);
    h->pos = pos;
    h->token = token;
    h->n_prefill = n_prefill;
    h->step = step;
    h->argmax_key = 0ull;
    CK(cudaMemcpyAsync(b.st, h, sizeof(StepState), cudaMemcpyHostToDevice, stream));
  }
};

namespace {

int fail(const CudaFail& f) { return set_error(f.code, f.msg); }

bool check_shapes(const ModelConfig& c, std::string* err) {
  auto bad = [&](const char* m) {
    *err = std::string("unsupported model shape: ") + m;
    return false;
  };
  if (c.dim == 0 || c.n_heads == 0 || c.n_layers == 0 || c.vocab_size == 0 || c.hidden_dim == 0)
    return bad("zero dimension");
  if (c.dim % c.n_heads) return bad("dim is not a multiple of n_heads");
  if (c.dim % 32) return bad("dim must be a multiple of 32");
  if (c.hidden_dim % 32) return bad("hidden_dim must be a multiple of 32");
  if (c.int4_group_size % 32) return bad("int4_group_size must be a multiple of 32");
  if (c.dim % c.int4_group_size || c.hidden_dim % c.int4_group_size)
    return bad("dim and hidden_dim must be multiples of int4_group_size");
  if (c.head_dim % 8 || c.head_dim < 16 || c.head_dim > 256)
    return bad("head_dim must be a multiple of 8 in [16, 256]");
  if (c.dim > 4096) return bad("dim above 4096");
  if (c.hidden_dim > 8192) return bad("hidden_dim above 8192");
  if (c.top_k * c.hidden_dim > 16384) return bad("top_k * hidden_dim above 16384");
  if (c.dim / c.int4_group_size > 64) return bad("dim / int4_group_size above 64");
  if (c.dim % 8) return bad("dim must be a multiple of 8");
  if ((c.hidden_dim / c.int4_group_size) % 4) return bad("hidden_dim / int4_group_size must be a multiple of 4");
  if (c.int4_group_size > 1024 || (c.int4_group_size & (c.int4_group_size - 1)))
    return bad("int4_group_size must be a power of two in [32, 1024]");
  if (c.n_experts > 32) return bad("more than 32 experts");
  if (c.top_k > 8) return bad("top_k above 8");
  if (c.vocab_size >= (1u << 31)) return bad("vocab too large");
  return true;
}

}  // namespace

extern "C" {

__attribute__((visibility("default"))) int chalot_load(const char* path, const chalot_opts* opts,
                                                       chalot_engine** out) {
  if (!path || !out) return set_error(CHALOT_ERR_ARG, "null argument");
  *out = nullptr;
  MappedFile mf;
  std::string err;
  if (!mf.open(path, &err)) return set_error(CHALOT_ERR_IO, err);
  FileHeader h;
  if (!parse_header(mf.data(), mf.size(), &h, &err)) return set_error(CHALOT_ERR_FORMAT, err);
  std::unique_ptr<chalot_engine> e(new chalot_engine());
  e->cfg = config_from_header(h);
  e->idx = build_index(e->cfg);
  const ModelConfig& c = e->cfg;
  if (!check_shapes(c, &err)) return set_error(CHALOT_ERR_ARG, err);
  if (mf.size() < e->idx.total_bytes)
    return set_error(CHALOT_ERR_FORMAT, "file is " + std::to_string(mf.size()) +
                                            " bytes, its header implies " +
                                            std::to_string(e->idx.total_bytes));
  e->device = opts ? opts->device : 0;
  e->use_graph = opts ? opts->use_cuda_graph != 0 : true;
  try {
    CK(cudaSetDevice(e->device));
    CK(cudaDeviceGetAttribute(&e->num_sms, cudaDevAttrMultiProcessorCount, e->device));
    CK(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking));
    Dims& d = e->dims;
    d.dim = int(c.dim);
    d.hidden = int(c.hidden_dim);
    d.n_layers = int(c.n_layers);
    d.n_heads = int(c.n_heads);
    d.head_dim = int(c.head_dim);
    d.vocab = int(c.vocab_size);
    d.max_seq = int(c.max_seq_len);
    d.n_experts = int(c.n_experts);
    d.top_k = int(c.top_k);
    d.group = int(c.int4_group_size);

    // ---- weights: every tensor at a 256-byte aligned device offset ----
    struct Piece {
      size_t src, bytes, dst;
    };
    std::vector<Piece> pieces;
    size_t cur = 0;
    auto place = [&](size_t src, size_t bytes) {
      pieces.push_back({src, bytes, cur});
      size_t at = cur;
      cur = (cur + bytes + 255) & ~size_t(255);
      return at;
    };
    const WeightIndex& ix = e->idx;
    const size_t dim = c.dim, H = c.hidden_dim, V = c.vocab_size, E = c.n_experts;
    struct LOff {
      size_t rms_attn, qkv, qkv_s, o, o_s, rms_ffn, rw, rb;
      std::vector<std::array<size_t, 4>> ex;
    };
    std::vector<LOff> loff(c.n_layers);
    const size_t emb = place(ix.embed_offset, V * dim), emb_s = place(ix.embed_scales_offset, V * 4);
    for (size_t l = 0; l < c.n_layers; ++l) {
      const LayerIndex& L = ix.layers[l];
      LOff& o = loff[l];
      o.rms_attn = place(L.rms_attn_offset, dim * 4);
      o.qkv = place(L.attn_qkv_offset, 3 * dim * dim);
      o.qkv_s = place(L.attn_qkv_scales_offset, 3 * dim * 4);
      o.o = place(L.attn_out_offset, dim * dim);
      o.o_s = place(L.attn_out_scales_offset, dim * 4);
      o.rms_ffn = place(L.rms_ffn_offset, dim * 4);
      o.rw = o.rb = 0;
      if (E >= 2) {
        o.rw = place(L.router_w_offset, E * dim * 4);
        o.rb = place(L.router_b_offset, E * 4);
      }
      for (size_t x = 0; x < E; ++x) {
        const ExpertIndex& X = L.experts[x];
        std::array<size_t, 4> a{place(X.gate_up_offset, X.gate_up_packed_bytes),
                                place(X.gate_up_scales_offset, X.gate_up_scales_count * 4),
                                place(X.down_offset, X.down_packed_bytes),
                                place(X.down_scales_offset, X.down_scales_count * 4)};
        o.ex.push_back(a);
      }
    }
    const size_t fnorm = place(ix.final_norm_offset, dim * 4);
    const size_t outw = place(ix.output_proj_offset, V * dim), outs = place(ix.output_proj_scales_offset, V * 4);
    e->weight_bytes = cur;
    CK(cudaMalloc(&e->d_weights, cur));
    {
      // stage through pinned memory in large chunks
      const size_t chunk = size_t(64) << 20;
      uint8_t* stage[2] = {nullptr, nullptr};
      CK(cudaMallocHost(&stage[0], chunk));
      CK(cudaMallocHost(&stage[1], chunk));
      cudaEvent_t done[2];
      CK(cudaEventCreateWithFlags(&done[0], cudaEventDisableTiming));
      CK(cudaEventCreateWithFlags(&done[1], cudaEventDisableTiming));
      int which = 0;
      size_t fill = 0;
      for (const Piece& p : pieces) {
        size_t done_b = 0;
        while (done_b < p.bytes) {
          size_t n = std::min(p.bytes - done_b, chunk - fill);
          if (fill == 0) CK(cudaEventSynchronize(done[which]));
          std::memcpy(stage[which] + fill, mf.data() + p.src + done_b, n);
          CK(cudaMemcpyAsync(e->d_weights + p.dst + done_b, stage[which] + fill, n,
                             cudaMemcpyHostToDevice, e->stream));
          fill += n;
          done_b += n;
          if (fill == chunk) {
            CK(cudaEventRecord(done[which], e->stream));
            which ^= 1;
            fill = 0;
          }
        }
      }
      CK(cudaStreamSynchronize(e->stream));
      cudaEventDestroy(done[0]);
      cudaEventDestroy(done[1]);
      cudaFreeHost(stage[0]);
      cudaFreeHost(stage[1]);
    }
    uint8_t* W = e->d_weights;
    e->emb = reinterpret_cast<const int8_t*>(W + emb);
    e->emb_s = reinterpret_cast<const float*>(W + emb_s);
    e->final_norm = reinterpret_cast<const float*>(W + fnorm);
    e->out_w = reinterpret_cast<const int8_t*>(W + outw);
    e->out_s = reinterpret_cast<const float*>(W + outs);
    e->d_experts = e->dalloc<ExpertPtrs>(c.n_layers * E);
    std::vector<ExpertPtrs> all;
    for (size_t l = 0; l < c.n_layers; ++l) {
      const LOff& o = loff[l];
      LayerPtrs L{};
      L.rms_attn = reinterpret_cast<const float*>(W + o.rms_attn);
      L.qkv = reinterpret_cast<const int8_t*>(W + o.qkv);
      L.qkv_s = reinterpret_cast<const float*>(W + o.qkv_s);
      L.o = reinterpret_cast<const int8_t*>(W + o.o);
      L.o_s = reinterpret_cast<const float*>(W + o.o_s);
      L.rms_ffn = reinterpret_cast<const float*>(W + o.rms_ffn);
      L.router_w = E >= 2 ? reinterpret_cast<const float*>(W + o.rw) : nullptr;
      L.router_b = E >= 2 ? reinterpret_cast<const float*>(W + o.rb) : nullptr;
      L.experts = e->d_experts + l * E;
      std::vector<ExpertPtrs> exs;
      for (size_t x = 0; x < E; ++x) {
        ExpertPtrs p{W + o.ex[x][0], reinterpret_cast<const float*>(W + o.ex[x][1]), W + o.ex[x][2],
                     reinterpret_cast<const float*>(W + o.ex[x][3])};
        exs.push_back(p);
        all.push_back(p);
      }
      for (size_t x = 0; x < std::min<size_t>(E, 16); ++x) L.ex[x] = exs[x];
      e->host_experts.push_back(exs);
      e->layers.push_back(L);
    }
    CK(cudaMemcpy(e->d_experts, all.data(), all.size() * sizeof(ExpertPtrs), cudaMemcpyHostToDevice));
    // expert int4 rows: file layout -> the kernels' repacked layout, once
    for (size_t l = 0; l < c.n_layers; ++l)
      for (size_t x = 0; x < E; ++x) {
        const ExpertIndex& X = ix.layers[l].experts[x];
        CK(repack_int4(W + loff[l].ex[x][0], X.gate_up_packed_bytes, e->stream));
        CK(repack_int4(W + loff[l].ex[x][2], X.down_packed_bytes, e->stream));
      }
    CK(cudaStreamSynchronize(e->stream));

    // ---- RoPE tables (state.rs:53-60), computed with glibc powf/cosf/sinf ----
    const size_t half = c.head_dim / 2;
    std::vector<float> cosv(c.max_seq_len * half), sinv(c.max_seq_len * half);
    for (size_t pos = 0; pos < c.max_seq_len; ++pos)
      for (size_t i = 0; i < half; ++i) {
        float freq = 1.0f / std::pow(c.rope_theta, float(2 * i) / float(c.head_dim));
        float th = float(pos) * freq;
        cosv[pos * half + i] = std::cos(th);
        sinv[pos * half + i] = std::sin(th);
      }
    float* rc = e->dalloc<float>(cosv.size());
    float* rs = e->dalloc<float>(sinv.size());
    CK(cudaMemcpy(rc, cosv.data(), cosv.size() * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(rs, sinv.data(), sinv.size() * 4, cudaMemcpyHostToDevice));

    // ---- decode buffers ----
    DecodeBufs& b = e->b;
    b.x = e->dalloc<float>(dim);
    b.q = e->dalloc<float>(dim);
    b.att_out = e->dalloc<float>(dim);
    b.scores = e->dalloc<float>(c.n_heads * c.max_seq_len);
    b.kc = e->dalloc<float>(c.n_layers * c.max_seq_len * dim);
    b.vc = e->dalloc<float>(c.n_layers * c.max_seq_len * dim);
    b.rope_cos = rc;
    b.rope_sin = rs;
    b.xq_attn = e->dalloc<int8_t>((dim + 15) & ~size_t(15));
    b.xs_attn = e->dalloc<float>(1);
    b.xq_ffn = e->dalloc<int8_t>((dim + 15) & ~size_t(15));
    b.xs_ffn = e->dalloc<float>(1);
    b.counters = e->dalloc<unsigned>(kTickets);
    b.err = e->dalloc<unsigned>(4);
    b.sel = e->dalloc<int32_t>(std::max<size_t>(c.top_k, 1));
    b.selw = e->dalloc<float>(std::max<size_t>(c.top_k, 1));
    b.h = e->dalloc<float>(std::max<size_t>(c.top_k, 1) * H);
    b.amax = e->dalloc<unsigned>(std::max<size_t>(c.top_k, 1));
    b.xq_h = e->dalloc<int8_t>(std::max<size_t>(c.top_k, 1) * H);
    b.xs_h = e->dalloc<float>(std::max<size_t>(c.top_k, 1));
    b.logits = e->dalloc<float>(V);
    b.st = e->dalloc<StepState>(1);
    b.prompt = e->dalloc<uint32_t>(c.max_seq_len);
    b.out_tokens = e->dalloc<uint32_t>(c.max_seq_len + 1);
    b.router_trace = nullptr;
    e->d_hist = e->dalloc<uint32_t>(2 * c.max_seq_len + 64);
    CK(cudaMallocHost(&e->h_state, sizeof(StepState)));
    e->n_stage = c.max_seq_len + 2;  // a generate call stages at most max_seq states between syncs
    CK(cudaMallocHost(&e->h_stage, e->n_stage * sizeof(StepState)));
    CK(cudaMallocHost(&e->h_tokens, (c.max_seq_len + 1) * sizeof(uint32_t)));
    for (auto& ev : e->ev) CK(cudaEventCreate(&ev));
    {
      // the persistent decode kernel when CHALOT_DECODE=persist asks for it
      // (shapes it does not fit keep the multi-kernel chain)
      const char* mode = std::getenv("CHALOT_DECODE");
      PersistArgs& pa = e->pargs;
      std::string why;
      if (mode && std::strcmp(mode, "persist") == 0 && persist_plan(e->dims, e->num_sms, &pa.plan, &why)) {
        pa.d = e->dims;
        LayerPtrs* dl = e->dalloc<LayerPtrs>(e->layers.size());
        CK(cudaMemcpy(dl, e->layers.data(), e->layers.size() * sizeof(LayerPtrs), cudaMemcpyHostToDevice));
        pa.layers = dl;
        pa.emb = e->emb;
        pa.emb_s = e->emb_s;
        pa.final_norm = e->final_norm;
        pa.out_w = e->out_w;
        pa.out_s = e->out_s;
        pa.b = e->b;
        pa.ll.x = e->dalloc<uint64_t>(2 * dim);
        pa.ll.q = e->dalloc<uint64_t>(3 * dim);
        pa.ll.score = e->dalloc<uint64_t>((size_t)c.n_heads * c.max_seq_len);
        pa.ll.att = e->dalloc<uint64_t>(dim);
        pa.ll.h = e->dalloc<uint64_t>((size_t)c.top_k * H);
        pa.epoch = e->dalloc<unsigned>(1);
        pa.ll.cnt = e->dalloc<unsigned>(kPersistCntWords);
        pa.err = e->b.err;
        pa.trace = e->dalloc<unsigned long long>((size_t)(c.n_layers + 1) * 32);
        if (std::getenv("CHALOT_TRACE_MAX"))  // diagnostics: every CTA's marks, latest kept
          pa.trace_max = e->dalloc<unsigned long long>((size_t)(c.n_layers + 1) * 32);
        e->use_persist = true;
      }
    }
    if (e->use_graph) {
      e->g_fwd = e->capture(false);
      e->g_step = e->capture(true);
    }
    CK(cudaDeviceSynchronize());
  } catch (const CudaFail& f) {
    return fail(f);
  }
  *out = e.release();
  clear_error();
  return CHALOT_OK;
}

__attribute__((visibility("default"))) void chalot_free(chalot_engine* e) { delete e; }

__attribute__((visibility("default"))) int chalot_get_config(const chalot_engine* e,
                                                             chalot_model_config* out) {
  if (!e || !out) return set_error(CHALOT_ERR_ARG, "null argument");
  const ModelConfig& c = e->cfg;
  std::memset(out, 0, sizeof *out);
  out->dim = uint32_t(c.dim);
  out->hidden_dim = uint32_t(c.hidden_dim);
  out->n_layers = uint32_t(c.n_layers);
  out->n_heads = uint32_t(c.n_heads);
  out->head_dim = uint32_t(c.head_dim);
  out->vocab_size = uint32_t(c.vocab_size);
  out->max_seq_len = uint32_t(c.max_seq_len);
  out->n_experts = uint32_t(c.n_experts);
  out->top_k = uint32_t(c.top_k);
  out->int4_group_size = uint32_t(c.int4_group_size);
  out->depth_router_layer = uint32_t(c.depth_router_layer);
  out->rope_theta = c.rope_theta;
  out->total_bytes = e->idx.total_bytes;
  out->expert_bytes = e->idx.layers.empty() || e->idx.layers[0].experts.empty()
                          ? 0
                          : e->idx.layers[0].experts[0].bytes();
  return CHALOT_OK;
}

__attribute__((visibility("default"))) int chalot_forward(chalot_engine* e, uint32_t token,
                                                          uint32_t pos, uint32_t* out_token) {
  if (!e) return set_error(CHALOT_ERR_ARG, "null engine");
  if (token >= e->cfg.vocab_size) return set_error(CHALOT_ERR_ARG, "token id out of range");
  if (pos >= e->cfg.max_seq_len) return set_error(CHALOT_ERR_ARG, "position out of range");
  try {
    CK(cudaSetDevice(e->device));
    e->set_state(pos, token, 0, 0);
    e->run_forward(true);
    CK(cudaMemcpyAsync(e->h_tokens, e->b.out_tokens, sizeof(uint32_t), cudaMemcpyDeviceToHost,
                       e->stream));
    CK(cudaStreamSynchronize(e->stream));
    e->check_device_error();
    if (out_token) *out_token = e->h_tokens[0];
  } catch (const CudaFail& f) {
    return fail(f);
  }
  clear_error();
  return CHALOT_OK;
}

__attribute__((visibility("default"))) int chalot_get_logits(chalot_engine* e, float* dst, size_t n) {
  if (!e || !dst) return set_error(CHALOT_ERR_ARG, "null argument");
  try {
    CK(cudaSetDevice(e->device));
    CK(cudaMemcpyAsync(dst, e->b.logits, std::min(n, e->cfg.vocab_size) * 4, cudaMemcpyDeviceToHost,
                       e->stream));
    CK(cudaStreamSynchronize(e->stream));
  } catch (const CudaFail& f) {
    return fail(f);
  }
  return CHALOT_OK;
}

// Uniform draw in [0, 1) from splitmix64 (24 bits, exact in f32).
static float next_draw(uint64_t* st) {
  uint64_t z = (*st += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return (float)(z >> 40) * (1.0f / 16777216.0f);
}

static uint64_t seed_of(const chalot_sampling* sp) {
  if (sp && sp->seed) return sp->seed;
  return (uint64_t)std::chrono::high_resolution_clock::now().time_since_epoch().count();
}

// Greedy argmax, or the configured strategy for one draw, of the engine's
// logits (the penalty already applied); the token lands in st->argmax_key.
static void launch_pick(chalot_engine* e, const chalot_sampling* sp) {
  if (!sp || sp->strategy == CHALOT_GREEDY || (sp->strategy == CHALOT_MIN_P && sp->min_p > 1.0f)) {
    launch_penalty_argmax(e->dims, e->b, e->d_hist, 0, 1.0f, e->stream);  // argmax only
    return;
  }
  CK(launch_sample(e->b.logits, (int)e->cfg.vocab_size, sp->strategy, sp->temperature, (int)sp->top_k,
                   sp->top_p, sp->min_p, next_draw(&e->rng), &e->b.st->argmax_key, e->stream));
}

__attribute__((visibility("default"))) int chalot_sample_from_logits(chalot_engine* e,
                                                                     const chalot_sampling* sp,
                                                                     const uint32_t* history,
                                                                     size_t n_history,
                                                                     uint32_t* out_token) {
  if (!e || !out_token) return set_error(CHALOT_ERR_ARG, "null argument");
  if (sp && (sp->strategy < CHALOT_GREEDY || sp->strategy > CHALOT_MIN_P))
    return set_error(CHALOT_ERR_ARG, "unknown sampling strategy");
  try {
    CK(cudaSetDevice(e->device));
    if (!e->rng) e->rng = seed_of(sp);
    const float pen = sp ? sp->repetition_penalty : 1.0f;
    size_t w = 0;
    if (pen > 1.0f && n_history > 0 && history) {  // engine.rs:555-560
      w = std::min<size_t>(n_history, sp->repetition_window);
      w = std::min<size_t>(w, 2 * e->cfg.max_seq_len + 64);
      CK(cudaMemcpyAsync(e->d_hist, history + (n_history - w), w * 4, cudaMemcpyHostToDevice,
                         e->stream));
    }
    launch_penalty_argmax(e->dims, e->b, e->d_hist, int(w), w ? pen : 1.0f, e->stream);
    if (sp && sp->strategy != CHALOT_GREEDY) launch_pick(e, sp);
    CK(cudaGetLastError());
    CK(cudaMemcpyAsync(e->h_state, e->b.st, sizeof(StepState), cudaMemcpyDeviceToHost, e->stream));
    CK(cudaStreamSynchronize(e->stream));
    *out_token = uint32_t(e->h_state->argmax_key & 0xffffffffull);
  } catch (const CudaFail& f) {
    return fail(f);
  }
  return CHALOT_OK;
}

__attribute__((visibility("default"))) int chalot_generate(chalot_engine* e, const uint32_t* prompt,
                                                           size_t n_prompt, size_t max_new,
                                                           const chalot_sampling* sp, uint32_t* out,
                                                           size_t* n_out) {
  if (!e || !n_out || (n_prompt && !prompt) || (max_new && !out))
    return set_error(CHALOT_ERR_ARG, "null argument");
  if (sp && (sp->strategy < CHALOT_GREEDY || sp->strategy > CHALOT_MIN_P))
    return set_error(CHALOT_ERR_ARG, "unknown sampling strategy");
  const bool greedy = !sp || sp->strategy == CHALOT_GREEDY;
  const size_t max_seq = e->cfg.max_seq_len, V = e->cfg.vocab_size;
  *n_out = 0;
  // engine.rs:509: n_prefill = min(len, max(max_seq - max_new, 1))
  const size_t room = max_seq > max_new ? max_seq - max_new : 0;
  const size_t n_prefill = std::min(n_prompt, std::max<size_t>(room, 1));
  const size_t n_decode = std::min(max_new, max_seq - std::min(max_seq, n_prefill));
  const float pen = sp ? sp->repetition_penalty : 1.0f;
  const bool penalty = pen > 1.0f;
  const bool stops = sp && sp->n_stop_tokens > 0 && sp->stop_tokens;
  try {
    CK(cudaSetDevice(e->device));
    CK(cudaStreamSynchronize(e->stream));  // every staged state of earlier calls is consumed
    std::vector<uint32_t> clamped(n_prefill);
    for (size_t i = 0; i < n_prefill; ++i) clamped[i] = std::min<uint32_t>(prompt[i], uint32_t(V - 1));
    if (n_prefill)
      CK(cudaMemcpyAsync(const_cast<uint32_t*>(e->b.prompt), clamped.data(), n_prefill * 4,
                         cudaMemcpyHostToDevice, e->stream));
    // the first token processed: prompt[0] or, without a prompt, BOS = 1 (engine.rs:520-524)
    e->set_state(0, n_prefill ? clamped[0] : 1u, uint32_t(n_prefill), 0);
    std::vector<uint32_t> hist(prompt, prompt + n_prompt);
    const size_t total = n_prefill + n_decode;
    CK(cudaEventRecord(e->ev[0], e->stream));
    e->rng = seed_of(sp);
    if (greedy && !penalty && !stops) {
      for (size_t f = 0; f < total; ++f) {
        e->run_forward(true);
        if (f + 1 == n_prefill) CK(cudaEventRecord(e->ev[1], e->stream));
      }
      if (n_prefill == 0) CK(cudaEventRecord(e->ev[1], e->stream));
      CK(cudaEventRecord(e->ev[2], e->stream));
      CK(cudaMemcpyAsync(e->h_tokens, e->b.out_tokens, std::max<size_t>(total, 1) * 4,
                         cudaMemcpyDeviceToHost, e->stream));
      CK(cudaStreamSynchronize(e->stream));
      // the token sampled after forward f (f >= n_prefill-1) is output n_prefill-1..
      size_t cnt = 0;
      for (size_t s = 0; s < n_decode; ++s)
        out[cnt++] = (n_prefill == 0 && s == 0) ? 1u : e->h_tokens[n_prefill + s - 1];
      *n_out = cnt;
    } else {
      // host-driven loop: the penalty needs the history, stop tokens end early,
      // and the sampling strategies need one draw per token
      if (n_prefill == 0) CK(cudaEventRecord(e->ev[1], e->stream));
      uint32_t next = 1;
      size_t cnt = 0;
      auto sample = [&]() -> uint32_t {
        size_t w = 0;
        if (penalty && !hist.empty()) {
          w = std::min<size_t>(hist.size(), sp->repetition_window);
          w = std::min<size_t>(w, 2 * max_seq + 64);
          CK(cudaMemcpyAsync(e->d_hist, hist.data() + (hist.size() - w), w * 4,
                             cudaMemcpyHostToDevice, e->stream));
        }
        launch_penalty_argmax(e->dims, e->b, e->d_hist, int(w), w ? pen : 1.0f, e->stream);
        if (!greedy) launch_pick(e, sp);
        CK(cudaGetLastError());
        CK(cudaMemcpyAsync(e->h_state, e->b.st, sizeof(StepState), cudaMemcpyDeviceToHost, e->stream));
        CK(cudaStreamSynchronize(e->stream));
        return uint32_t(e->h_state->argmax_key & 0xffffffffull);
      };
      for (size_t p = 0; p < n_prefill; ++p) {
        e->set_state(uint32_t(p), clamped[p], 0, 0);
        e->run_forward(false);
        if (p + 1 == n_prefill) CK(cudaEventRecord(e->ev[1], e->stream));
      }
      if (n_prefill) next = sample();
      for (size_t s = 0; s < n_decode; ++s) {
        bool is_stop = false;
        for (uint32_t i = 0; stops && i < sp->n_stop_tokens; ++i) is_stop |= sp->stop_tokens[i] == next;
        if (is_stop) break;
        out[cnt++] = next;
        hist.push_back(next);
        e->set_state(uint32_t(n_prefill + s), next, 0, 0);
        e->run_forward(false);
        next = sample();
      }
      CK(cudaEventRecord(e->ev[2], e->stream));
      CK(cudaStreamSynchronize(e->stream));
      *n_out = cnt;
    }
    e->check_device_error();
    float a = 0, bb = 0;
    CK(cudaEventElapsedTime(&a, e->ev[0], e->ev[1]));
    CK(cudaEventElapsedTime(&bb, e->ev[1], e->ev[2]));
    e->last_prefill_ms = a;
    e->last_decode_ms = bb;
    e->last_n_prefill = uint32_t(n_prefill);
    e->last_n_decode = uint32_t(n_decode);
  } catch (const CudaFail& f) {
    return fail(f);
  }
  clear_error();
  return CHALOT_OK;
}

__attribute__((visibility("default"))) int chalot_last_timing(chalot_engine* e, double* prefill_ms,
                                                              double* decode_ms, uint32_t* n_prefill,
                                                              uint32_t* n_decode) {
  if (!e) return set_error(CHALOT_ERR_ARG, "null engine");
  if (prefill_ms) *prefill_ms = e->last_prefill_ms;
  if (decode_ms) *decode_ms = e->last_decode_ms;
  if (n_prefill) *n_prefill = e->last_n_prefill;
  if (n_decode) *n_decode = e->last_n_decode;
  return CHALOT_OK;
}

__attribute__((visibility("default"))) int chalot_bench_moe_layers(chalot_engine* e, int reps,
                                                                   double* ms_per_layer,
                                                                   double* bytes_per_layer) {
  if (!e || reps <= 0) return set_error(CHALOT_ERR_ARG, "bad argument");
  const Dims& d = e->dims;
  try {
    CK(cudaSetDevice(e->device));
    // A fixed selection per layer in device buffers of its own, so the
    // decode state is untouched.
    const int K = d.top_k, L = d.n_layers;
    DecodeBufs b = e->b;
    int32_t* sel = nullptr;
    float* selw = nullptr;
    float* x = nullptr;
    CK(cudaMalloc(&sel, sizeof(int32_t) * K * L));
    CK(cudaMalloc(&selw, sizeof(float) * K * L));
    CK(cudaMalloc(&x, sizeof(float) * d.dim));
    std::vector<int32_t> hs(K * L);
    std::vector<float> hw(K * L, 1.0f / K);
    for (int l = 0; l < L; ++l)
      for (int k = 0; k < K; ++k) hs[l * K + k] = (l * K + k) % d.n_experts;
    CK(cudaMemcpy(sel, hs.data(), hs.size() * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(selw, hw.data(), hw.size() * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(x, e->b.x, sizeof(float) * d.dim, cudaMemcpyDeviceToDevice));
    b.x = x;
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ex = nullptr;
    CK(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
    for (int l = 0; l < L; ++l) {
      DecodeBufs bl = b;
      bl.sel = sel + l * K;
      bl.selw = selw + l * K;
      launch_gateup(d, e->layers[l], l, bl, e->stream, l > 0);
      launch_down(d, e->layers[l], l, nullptr, bl, e->stream, true);
    }
    CK(cudaStreamEndCapture(e->stream, &g));
    CK(cudaGraphInstantiate(&ex, g, 0));
    cudaGraphDestroy(g);
    CK(cudaGraphLaunch(ex, e->stream));  // warm-up
    CK(cudaEventRecord(e->ev[0], e->stream));
    for (int r = 0; r < reps; ++r) CK(cudaGraphLaunch(ex, e->stream));
    CK(cudaEventRecord(e->ev[1], e->stream));
    CK(cudaStreamSynchronize(e->stream));
    float ms = 0;
    CK(cudaEventElapsedTime(&ms, e->ev[0], e->ev[1]));
    cudaGraphExecDestroy(ex);
    cudaFree(sel);
    cudaFree(selw);
    cudaFree(x);
    if (ms_per_layer) *ms_per_layer = double(ms) / (double(reps) * L);
    if (bytes_per_layer) *bytes_per_layer = double(K) * double(e->idx.layers[0].experts[0].bytes());
  } catch (const CudaFail& f) {
    return fail(f);
  }
  return CHALOT_OK;
}

__attribute__((visibility("default"))) int chalot_decode_trace(chalot_engine* e, unsigned long long* dst,
                                                               size_t n, size_t* n_out) {
  if (!e) return set_error(CHALOT_ERR_ARG, "null engine");
  if (!e->use_persist) return set_error(CHALOT_ERR_STATE, "decode_trace: the engine runs the multi-kernel chain");
  const size_t total = (size_t)(e->cfg.n_layers + 1) * 32;
  if (n_out) *n_out = e->pargs.trace_max ? 2 * total : total;
  if (!dst || n == 0) return CHALOT_OK;
  try {
    CK(cudaSetDevice(e->device));
    CK(cudaStreamSynchronize(e->stream));
    CK(cudaMemcpy(dst, e->pargs.trace, std::min(n, total) * sizeof(unsigned long long), cudaMemcpyDeviceToHost));
    if (e->pargs.trace_max && n >= 2 * total) {  // then the latest-CTA marks, cleared for the next step
      CK(cudaMemcpy(dst + total, e->pargs.trace_max, total * sizeof(unsigned long long), cudaMemcpyDeviceToHost));
      CK(cudaMemset(e->pargs.trace_max, 0, total * sizeof(unsigned long long)));
    }
  } catch (const CudaFail& f) {
    return fail(f);
  }
  return CHALOT_OK;
}

#ifdef CHALOT_PHASE_TRACE
// Copies the phase trace of the forwards since the last clear (instrumented
// builds only): [slot = layer*8 + kind][cta][phase] %globaltimer values.
__attribute__((visibility("default"))) int chalot_phase_trace(unsigned long long* dst, size_t n) {
  n = std::min(n, (size_t)kTraceSlots * kTraceCtas * kTracePhases);
  std::vector<unsigned long long> tmp(n);
  std::memset(dst, 0, n * 8);
  for (auto fn : {trace_dense, trace_moe, trace_attn}) {
    cudaError_t r = fn(tmp.data(), n);
    if (r != cudaSuccess) return set_error(CHALOT_ERR_CUDA, cudaGetErrorString(r));
    for (size_t i = 0; i < n; ++i) dst[i] += tmp[i];
  }
  return CHALOT_OK;
}
__attribute__((visibility("default"))) int chalot_phase_trace_clear(void) {
  for (auto fn : {trace_dense_clear, trace_moe_clear, trace_attn_clear}) {
    cudaError_t r = fn();
    if (r != cudaSuccess) return set_error(CHALOT_ERR_CUDA, cudaGetErrorString(r));
  }
  return CHALOT_OK;
}
#endif

__attribute__((visibility("default"))) int chalot_profile_forward(chalot_engine* e, uint32_t token,
                                                                  uint32_t pos, float* ms, int cap,
                                                                  int* n_out) {
  if (!e || !ms || !n_out) return set_error(CHALOT_ERR_ARG, "null argument");
  if (token >= e->cfg.vocab_size || pos >= e->cfg.max_seq_len)
    return set_error(CHALOT_ERR_ARG, "token or position out of range");
  const int n = 2 + 6 * e->dims.n_layers + 1;  // kernels of one forward (no advance)
  if (cap < n) return set_error(CHALOT_ERR_ARG, "profile buffer too small");
  std::vector<cudaEvent_t> ev(n + 1, nullptr);
  try {
    CK(cudaSetDevice(e->device));
    for (auto& x : ev) CK(cudaEventCreate(&x));
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ex = nullptr;
    CK(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
    e->record_forward(e->stream, false, ev.data());
    CK(cudaStreamEndCapture(e->stream, &g));
    CK(cudaGraphInstantiate(&ex, g, 0));
    cudaGraphDestroy(g);
    for (int rep = 0; rep < 2; ++rep) {  // the second replay is the one reported
      e->set_state(pos, token, 0, 0);
      CK(cudaGraphLaunch(ex, e->stream));
    }
    CK(cudaStreamSynchronize(e->stream));
    for (int i = 0; i < n - 1; ++i) CK(cudaEventElapsedTime(&ms[i], ev[i], ev[i + 1]));
    *n_out = n - 1;
    cudaGraphExecDestroy(ex);
  } catch (const CudaFail& f) {
    for (auto& x : ev)
      if (x) cudaEventDestroy(x);
    return fail(f);
  }
  for (auto& x : ev) cudaEventDestroy(x);
  return CHALOT_OK;
}

// ---- batched decode -------------------------------------------------------------

static MlDims batch_moe_dims(const chalot_engine* e, int n) {
  const ModelConfig& c = e->cfg;
  return MlDims{n, (int)c.dim, (int)c.hidden_dim, (int)c.n_experts, (int)c.top_k, (int)c.int4_group_size};
}

// Batch state for max_seqs slots; page_tokens == 0: the flat K/V cache
// [slot][layer][max_seq][dim], else a pool of n_pages pages of page_tokens
// positions.
static int batch_reserve(chalot_engine* e, uint32_t max_seqs, uint32_t n_pages, uint32_t page_tokens) {
  if (!e) return set_error(CHALOT_ERR_ARG, "null engine");
  const ModelConfig& c = e->cfg;
  if (c.n_experts < 2) return set_error(CHALOT_ERR_ARG, "batch_reserve: batched decode needs a MoE model");
  if (max_seqs == 0 || max_seqs > 1024) return set_error(CHALOT_ERR_ARG, "batch_reserve: max_seqs in [1, 1024]");
  const bool paged = page_tokens != 0;
  if (paged && (page_tokens < 16 || page_tokens > 256 || (page_tokens & (page_tokens - 1))))
    return set_error(CHALOT_ERR_ARG, "batch_reserve: page_tokens must be a power of two in [16, 256]");
  if (paged && (n_pages == 0 || n_pages > (1u << 24)))
    return set_error(CHALOT_ERR_ARG, "batch_reserve: n_pages must be in [1, 2^24]");
  if (paged && e->cfg.head_dim % 16)
    return set_error(CHALOT_ERR_ARG, "batch_reserve: paged K/V needs head_dim % 16 == 0");
  if (e->bt.cap) {
    const bool same = paged ? e->bt.pt_shift >= 0 && (1u << e->bt.pt_shift) == page_tokens &&
                                  (uint32_t)e->bt.n_pages >= n_pages
                            : e->bt.pt_shift < 0;
    if ((int)max_seqs <= e->bt.cap && (same || !paged)) return CHALOT_OK;  // a flat request takes either layout
    return set_error(CHALOT_ERR_STATE, "batch_reserve: already reserved (with fewer slots or another K/V layout)");
  }
  if (const char* m = ml_check(batch_moe_dims(e, (int)max_seqs)))
    return set_error(CHALOT_ERR_ARG, std::string("batch_reserve: ") + m);
  try {
    CK(cudaSetDevice(e->device));
    auto& b = e->bt;
    const size_t S = max_seqs, D = c.dim, L = c.n_layers, M = c.max_seq_len, H = c.n_heads;
    if (paged) {
      b.pt_shift = 0;
      while ((1u << b.pt_shift) < page_tokens) ++b.pt_shift;
      b.maxp = (int)((M + page_tokens - 1) / page_tokens);
      b.n_pages = (int)n_pages;
      b.kc = e->dalloc<float>((size_t)n_pages * L * page_tokens * D);
      b.vc = e->dalloc<float>((size_t)n_pages * L * page_tokens * D);
      b.ptab = e->dalloc<int32_t>(S * b.maxp);
      CK(cudaMallocHost(&b.h_ptab, S * b.maxp * sizeof(int32_t)));
      std::memset(b.h_ptab, 0, S * b.maxp * sizeof(int32_t));
      b.slot_pages.assign(S, {});
      b.free_pages.resize(n_pages);
      for (uint32_t i = 0; i < n_pages; ++i) b.free_pages[i] = (int)(n_pages - 1 - i);  // page 0 first
    } else {
      b.kc = e->dalloc<float>(S * L * M * D);
      b.vc = e->dalloc<float>(S * L * M * D);
    }
    b.x = e->dalloc<float>(S * D);
    b.qkv = e->dalloc<float>(S * 3 * D);
    b.q = e->dalloc<float>(S * D);
    b.scores = e->dalloc<float>(S * H * M);
    b.att = e->dalloc<float>(S * D);
    b.xb = e->dalloc<float>(S * D);
    b.eout = e->dalloc<float>(S * D);
    b.logits = e->dalloc<float>(S * c.vocab_size);
    b.xs = e->dalloc<float>(S);
    b.xq = e->dalloc<int8_t>(S * D);
    b.pos = e->dalloc<int32_t>(S);
    b.slot = e->dalloc<int32_t>(S);
    b.toks = e->dalloc<uint32_t>(S);
    b.out = e->dalloc<uint32_t>(S);
    const MlDims md = batch_moe_dims(e, (int)max_seqs);
    const size_t simt = ml_layout(md, nullptr, nullptr);
    const size_t need = ml_tc_eligible(md) ? ml_tc_layout(md, simt, nullptr, nullptr) : simt;
    b.moe_ws = e->dalloc<unsigned char>(need);
    CK(cudaMallocHost(&b.h_io, 4 * S * sizeof(uint32_t)));
    b.experts.assign(L, MlExperts{});
    for (size_t l = 0; l < L; ++l) {
      for (size_t x = 0; x < c.n_experts && x < 32; ++x) {
        const ExpertPtrs& p = e->host_experts[l][x];
        b.experts[l].ex[x] = MlExpert{p.gu, p.gu_s, p.dn, p.dn_s};
      }
      b.experts[l].repacked = 1;
    }
    b.cap = (int)max_seqs;
  } catch (const CudaFail& f) {
    return fail(f);
  }
  return CHALOT_OK;
}

__attribute__((visibility("default"))) int chalot_batch_reserve(chalot_engine* e, uint32_t max_seqs) {
  return batch_reserve(e, max_seqs, 0, 0);
}

__attribute__((visibility("default"))) int chalot_batch_reserve_paged(chalot_engine* e, uint32_t max_seqs,
                                                                     uint32_t n_pages, uint32_t page_tokens) {
  if (!page_tokens) return set_error(CHALOT_ERR_ARG, "batch_reserve_paged: page_tokens must be positive");
  return batch_reserve(e, max_seqs, n_pages, page_tokens);
}

__attribute__((visibility("default"))) int chalot_batch_release(chalot_engine* e, uint32_t slot) {
  if (!e) return set_error(CHALOT_ERR_ARG, "null engine");
  auto& b = e->bt;
  if ((int)slot >= b.cap) return set_error(CHALOT_ERR_ARG, "batch_release: slot out of range");
  if (b.pt_shift < 0) return CHALOT_OK;  // the flat cache keeps every slot's rows
  for (int p : b.slot_pages[slot]) b.free_pages.push_back(p);
  b.slot_pages[slot].clear();
  return CHALOT_OK;
}

__attribute__((visibility("default"))) int chalot_batch_capacity(chalot_engine* e, uint32_t* max_seqs) {
  if (!e || !max_seqs) return set_error(CHALOT_ERR_ARG, "null argument");
  *max_seqs = (uint32_t)e->bt.cap;
  return CHALOT_OK;
}

__attribute__((visibility("default"))) int chalot_batch_kv_pages(chalot_engine* e, uint32_t* n_free,
                                                                uint32_t* n_total, uint32_t* page_tokens) {
  if (!e) return set_error(CHALOT_ERR_ARG, "null engine");
  const auto& b = e->bt;
  const bool paged = b.pt_shift >= 0;
  if (n_free) *n_free = paged ? (uint32_t)b.free_pages.size() : 0;
  if (n_total) *n_total = paged ? (uint32_t)b.n_pages : 0;
  if (page_tokens) *page_tokens = paged ? 1u << b.pt_shift : 0;
  return CHALOT_OK;
}

// ---- expert parallelism of the batched forward --------------------------------
//
// Every exchange has a fixed size, so the host never waits for the device in
// the middle of a forward: rank r sends each peer a block of R1 = cap*top_k
// rows (the most one rank can route to another; all ranks reserve the same
// max_seqs), of which the first n are real, n coming from the counts exchange
// that precedes the rows. The receiving side marks the padding rows invalid
// (expert -1), which the dispatch of the expert kernels skips.

// Counts per (destination rank, local expert) from the rank-major plan offsets.
__global__ void k_ep_counts(const int32_t* offs, int n, int32_t* cnt) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) cnt[i] = offs[i + 1] - offs[i];
}

// One warp per plan position q: copies the int8 row and the scale of slot
// order[q] into block g (its destination rank) of the send buffer, at row
// q - (first position of rank g), and records that padded row for the slot.
__global__ void k_ep_pack(int n_slots, int K, int D, int G, int El, int R1, const int32_t* offs,
                          const int32_t* order, const int8_t* xq, const float* xs, int8_t* rows, float* rscale,
                          int32_t* ppos) {
  const int q = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (q >= n_slots) return;
  int g = 0;
  while (g + 1 < G && q >= offs[(g + 1) * El]) ++g;
  const int dst = g * R1 + (q - offs[g * El]);
  const int slot = order[q], tok = slot / K;
  const uint4* src = reinterpret_cast<const uint4*>(xq + (size_t)tok * D);
  uint4* o = reinterpret_cast<uint4*>(rows + (size_t)dst * D);
  for (int j = lane; j < D / 16; j += 32) o[j] = src[j];
  if (lane == 0) {
    rscale[dst] = xs[tok];
    ppos[slot] = dst;
  }
}

// Local expert of every received row: block g holds rcnt[g][0..El) rows in
// local-expert order, then padding (-1, skipped by the dispatch).
__global__ void k_ep_row_experts(int G, int El, int R1, const int32_t* rcnt, int32_t* rexp) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= G * R1) return;
  const int g = i / R1, r = i - g * R1;
  int acc = 0, ex = -1;
  for (int k = 0; k < El; ++k) {
    const int c = rcnt[g * El + k];
    if (r >= acc && r < acc + c) ex = k;
    acc += c;
  }
  rexp[i] = ex;
}

// Exchange buffers for `cap` tokens per rank: R1 = cap*top_k rows per peer.
static void ep_reserve(chalot_engine* e) {
  auto& p = e->epb;
  const ModelConfig& c = e->cfg;
  const int G = e->ep->world();
  if (p.cap == e->bt.cap && p.world == G) return;
  const size_t S = e->bt.cap, K = c.top_k, D = c.dim, E = c.n_experts, El = E / G;
  const size_t R = (size_t)G * S * K;  // rows of all blocks, sent or received
  p.rows = e->dalloc<int8_t>(R * D);
  p.rscale = e->dalloc<float>(R);
  p.rrows = e->dalloc<int8_t>(R * D);
  p.rrscale = e->dalloc<float>(R);
  p.rexp = e->dalloc<int32_t>(R);
  p.y = e->dalloc<float>(R * D);
  p.yback = e->dalloc<float>(R * D);
  p.ppos = e->dalloc<int32_t>(S * K);
  p.offs = e->dalloc<int32_t>(E + 1);
  p.cnt = e->dalloc<int32_t>(2 * G * El);
  const MlDims xd{(int)R, (int)D, (int)c.hidden_dim, (int)El, 1, (int)c.int4_group_size};
  const size_t simt = ml_layout(xd, nullptr, nullptr);
  p.ws = e->dalloc<unsigned char>(ml_tc_eligible(xd) ? ml_tc_layout(xd, simt, nullptr, nullptr) : simt);
  p.cap = (int)S;
  p.world = G;
}

// The expert block of layer l for this rank's B tokens (rows b.xb) with the
// experts spread over the group (expert e on rank e % world), into b.eout:
// route, order the (token, choice) slots by destination rank and local expert,
// exchange counts, int8 rows and scales, run the local experts on the rows
// received, send the f32 outputs back and combine them per token in selection
// order (engine.rs:334-401). Every rank takes the same exchanges in the same
// order, B == 0 included; nothing waits for the device. Returns a CHALOT_
// status.
static int ep_moe(chalot_engine* e, int l, int B, const MlDims& md, MlWork w, cudaStream_t s, std::string* msg) {
  auto& p = e->epb;
  auto& b = e->bt;
  const ModelConfig& c = e->cfg;
  EpLink& link = *e->ep;
  const int G = link.world(), rank = link.rank(), E = (int)c.n_experts, El = E / G, K = (int)c.top_k;
  const int R1 = p.cap * K;
  const size_t D = c.dim, R = (size_t)G * R1;
  const LayerPtrs& L = e->layers[l];
  int rc;
  if (B > 0) {
    ml_launch_route(md, b.xb, L.router_w, L.router_b, w, s);
    ml_launch_plan(MlDims{B * K, 0, 0, E, 1, 32}, w, G, p.offs, s);
    k_ep_pack<<<(B * K + 7) / 8, 256, 0, s>>>(B * K, K, (int)D, G, El, R1, p.offs, w.perm, w.xq, w.xs, p.rows,
                                              p.rscale, p.ppos);
  } else {
    CK(cudaMemsetAsync(p.offs, 0, (E + 1) * sizeof(int32_t), s));
  }
  k_ep_counts<<<1, 1024, 0, s>>>(p.offs, G * El, p.cnt);
  CK(cudaGetLastError());
  const std::vector<size_t> cb(G, El * sizeof(int32_t)), rb(G, (size_t)R1 * D), sb(G, (size_t)R1 * 4),
      yb(G, (size_t)R1 * D * 4);
  if ((rc = link.all_to_all(p.cnt, cb.data(), p.cnt + G * El, cb.data(), s, msg)) != CHALOT_OK) return rc;
  if ((rc = link.all_to_all(p.rows, rb.data(), p.rrows, rb.data(), s, msg)) != CHALOT_OK) return rc;
  if ((rc = link.all_to_all(p.rscale, sb.data(), p.rrscale, sb.data(), s, msg)) != CHALOT_OK) return rc;
  k_ep_row_experts<<<(unsigned)((R + 255) / 256), 256, 0, s>>>(G, El, R1, p.cnt + G * El, p.rexp);
  CK(cudaGetLastError());
  const MlDims xd{(int)R, (int)D, (int)c.hidden_dim, El, 1, (int)c.int4_group_size};
  MlWork xw;
  const size_t simt = ml_layout(xd, p.ws, &xw);
  // the blocks hold R rows, mostly padding: the kernels are chosen by the rows a
  // rank receives on average, this rank's B*K (ranks decode similar batches)
  const int live = std::max(B, 1) * K;
  MlDims xe = xd;
  xe.T = std::min(live, (int)R);
  const bool tc = ml_use_tc(xe);
  MlTcWork xt{};
  if (tc) ml_tc_layout(xd, simt, p.ws, &xt);
  xw.sel = p.rexp;  // -1 on padding rows: not dispatched, their outputs are 0
  xw.xq = p.rrows;
  xw.xs = p.rrscale;
  MlExperts X{};
  for (int i = 0; i < El; ++i) X.ex[i] = b.experts[l].ex[rank + G * i];
  X.repacked = b.experts[l].repacked;
  CK(ml_run_rows(xd, X, xw, tc ? &xt : nullptr, p.y, s, live));
  if ((rc = link.all_to_all(p.y, yb.data(), p.yback, yb.data(), s, msg)) != CHALOT_OK) return rc;
  if (B > 0) {
    w.y = p.yback;   // padded blocks of the outputs of my rows
    w.inv = p.ppos;  // slot -> its row there
    ml_launch_combine(MlDims{B, (int)D, 0, 1, K, 32}, w, b.eout, s);
  }
  return CHALOT_OK;
}

__attribute__((visibility("default"))) int chalot_forward_batch(chalot_engine* e, const uint32_t* slots,
                                                                const uint32_t* toks, const uint32_t* pos,
                                                                uint32_t n, uint32_t* out_toks) {
  if (!e || (n && (!slots || !toks || !pos || !out_toks))) return set_error(CHALOT_ERR_ARG, "null argument");
  auto& b = e->bt;
  if (!b.cap) return set_error(CHALOT_ERR_STATE, "forward_batch: call chalot_batch_reserve first");
  if ((int)n > b.cap) return set_error(CHALOT_ERR_ARG, "forward_batch: more tokens than reserved slots");
  const ModelConfig& c = e->cfg;
  for (uint32_t i = 0; i < n; ++i) {
    if ((int)slots[i] >= b.cap) return set_error(CHALOT_ERR_ARG, "forward_batch: slot out of range");
    if (pos[i] >= c.max_seq_len) return set_error(CHALOT_ERR_ARG, "forward_batch: position beyond max_seq_len");
    if (toks[i] >= c.vocab_size) return set_error(CHALOT_ERR_ARG, "forward_batch: token out of range");
    for (uint32_t j = 0; j < i; ++j)
      if (slots[j] == slots[i] && pos[j] == pos[i])
        return set_error(CHALOT_ERR_ARG, "forward_batch: a (slot, position) pair appears twice");
  }
  if (n == 0 && !e->ep) return CHALOT_OK;
  try {
    CK(cudaSetDevice(e->device));
    cudaStream_t s = e->stream;
    CK(cudaStreamSynchronize(s));  // the pinned staging may still feed a previous call
    std::string msg;
    if (e->ep) ep_reserve(e);
    if (n == 0) {  // no tokens here: still take every exchange of the group
      const MlDims md0 = batch_moe_dims(e, 0);
      MlWork w0;
      ml_layout(md0, b.moe_ws, &w0);
      for (int l = 0; l < (int)c.n_layers; ++l)
        if (int rc = ep_moe(e, l, 0, md0, w0, s, &msg)) return set_error(rc, "forward_batch: " + msg);
      return CHALOT_OK;
    }
    if (b.pt_shift >= 0) {  // pages for every position this call writes or attends
      bool grew = false;
      for (uint32_t i = 0; i < n; ++i) {
        auto& pages = b.slot_pages[slots[i]];
        const size_t need = (size_t)(pos[i] >> b.pt_shift) + 1;
        while (pages.size() < need) {
          if (b.free_pages.empty()) return set_error(CHALOT_ERR_OOM, "forward_batch: out of K/V pages");
          pages.push_back(b.free_pages.back());
          b.free_pages.pop_back();
          b.h_ptab[(size_t)slots[i] * b.maxp + pages.size() - 1] = pages.back();
          grew = true;
        }
      }
      if (grew) CK(cudaMemcpyAsync(b.ptab, b.h_ptab, (size_t)b.cap * b.maxp * 4, cudaMemcpyHostToDevice, s));
    }
    uint32_t* io = b.h_io;
    std::memcpy(io, slots, n * 4);
    std::memcpy(io + b.cap, toks, n * 4);
    std::memcpy(io + 2 * b.cap, pos, n * 4);
    CK(cudaMemcpyAsync(b.slot, io, n * 4, cudaMemcpyHostToDevice, s));
    CK(cudaMemcpyAsync(b.toks, io + b.cap, n * 4, cudaMemcpyHostToDevice, s));
    CK(cudaMemcpyAsync(b.pos, io + 2 * b.cap, n * 4, cudaMemcpyHostToDevice, s));
    const int B = (int)n, D = (int)c.dim;
    BatchDims bd{D, (int)c.n_layers, (int)c.n_heads, (int)c.head_dim, (int)c.max_seq_len};
    if (b.pt_shift >= 0) {
      bd.ptab = b.ptab;
      bd.pt_shift = b.pt_shift;
      bd.maxp = b.maxp;
    }
    CK(cudaEventRecord(e->ev[0], s));
    b_embed(bd, B, b.toks, e->emb, e->emb_s, e->layers[0].rms_attn, b.x, b.xq, b.xs, s);
    const MlDims md = batch_moe_dims(e, B);
    MlWork w;
    const size_t simt = ml_layout(md, b.moe_ws, &w);
    const bool tc = ml_use_tc(md);
    MlTcWork t{};
    if (tc) ml_tc_layout(md, simt, b.moe_ws, &t);
    for (int l = 0; l < (int)c.n_layers; ++l) {
      const LayerPtrs& L = e->layers[l];
      b_gemm_i8(B, 3 * D, D, L.qkv, L.qkv_s, b.xq, b.xs, b.qkv, 3 * D, false, s);
      b_rope_kv(bd, l, B, b.pos, b.slot, b.qkv, b.q, b.kc, b.vc, e->b.rope_cos, e->b.rope_sin, s);
      b_attention(bd, l, B, b.pos, b.slot, b.q, b.kc, b.vc, b.scores, b.att, s);
      CK(op_quantize_i8(b.xq, b.xs, b.att, B, D, s));
      b_gemm_i8(B, D, D, L.o, L.o_s, b.xq, b.xs, b.x, D, true, s);  // residual (engine.rs:312-322)
      const float* next_norm = l + 1 < (int)c.n_layers ? e->layers[l + 1].rms_attn : e->final_norm;
      if (e->ep) {
        b_rmsnorm(bd, B, b.x, L.rms_ffn, b.xb, s);
        if (int rc = ep_moe(e, l, B, md, w, s, &msg)) return set_error(rc, "forward_batch: " + msg);
        b_add((long)B * D, b.x, b.eout, s);  // x += expert_out (engine.rs:401)
        b_norm_quant(bd, B, b.x, next_norm, b.xq, b.xs, s);
      } else {  // rmsnorm, MoE block, x += expert_out (engine.rs:325-401) and the next norm + quantize
        CK(ml_run_decode(md, b.x, L.rms_ffn, L.router_w, L.router_b, b.experts[l], w, tc ? &t : nullptr,
                         next_norm, b.xq, b.xs, s));
      }
    }
    b_gemm_i8(B, (int)c.vocab_size, D, e->out_w, e->out_s, b.xq, b.xs, b.logits, (int)c.vocab_size, false, s);
    b_argmax(B, (int)c.vocab_size, b.logits, b.out, s);
    CK(cudaGetLastError());
    CK(cudaEventRecord(e->ev[1], s));
    CK(cudaMemcpyAsync(io + 3 * b.cap, b.out, n * 4, cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    {
      float ms = 0;
      CK(cudaEventElapsedTime(&ms, e->ev[0], e->ev[1]));
      e->last_prefill_ms = 0;
      e->last_decode_ms = ms;
      e->last_n_prefill = 0;
      e->last_n_decode = (uint32_t)n;
    }
    // a tensor-core wait of this forward (or of earlier operator work) that gave up
    if (int rc = devstat_take("forward_batch")) return rc;
    std::memcpy(out_toks, io + 3 * b.cap, n * 4);
  } catch (const CudaFail& f) {
    return fail(f);
  }
  return CHALOT_OK;
}

__attribute__((visibility("default"))) int chalot_get_batch_logits(chalot_engine* e, uint32_t row, float* dst,
                                                                   size_t n) {
  if (!e || !dst) return set_error(CHALOT_ERR_ARG, "null argument");
  if ((int)row >= e->bt.cap) return set_error(CHALOT_ERR_ARG, "get_batch_logits: row out of range");
  try {
    CK(cudaSetDevice(e->device));
    CK(cudaMemcpyAsync(dst, e->bt.logits + (size_t)row * e->cfg.vocab_size,
                       std::min(n, e->cfg.vocab_size) * 4, cudaMemcpyDeviceToHost, e->stream));
    CK(cudaStreamSynchronize(e->stream));
  } catch (const CudaFail& f) {
    return fail(f);
  }
  return CHALOT_OK;
}

__attribute__((visibility("default"))) int chalot_ep_nccl_id(uint8_t* id) {
  if (!id) return set_error(CHALOT_ERR_ARG, "ep_nccl_id: null argument");
  std::string msg;
  const int rc = ep_nccl_unique_id(id, &msg);
  return rc == CHALOT_OK ? CHALOT_OK : set_error(rc, "ep_nccl_id: " + msg);
}

static int ep_check_attach(chalot_engine* e, uint32_t rank, uint32_t world) {
  if (!e) return set_error(CHALOT_ERR_ARG, "ep_attach: null engine");
  if (e->ep) return set_error(CHALOT_ERR_STATE, "ep_attach: already attached");
  const uint32_t E = (uint32_t)e->cfg.n_experts;
  if (E < 2) return set_error(CHALOT_ERR_ARG, "ep_attach: expert parallelism needs a MoE model");
  if (world < 1 || world > E || E % world || rank >= world)
    return set_error(CHALOT_ERR_ARG, "ep_attach: need world dividing n_experts and rank < world");
  return CHALOT_OK;
}

__attribute__((visibility("default"))) int chalot_ep_attach_nccl(chalot_engine* e, uint32_t rank, uint32_t world,
                                                                const uint8_t* id) {
  if (int rc = ep_check_attach(e, rank, world)) return rc;
  if (!id) return set_error(CHALOT_ERR_ARG, "ep_attach: null id");
  std::string msg;
  const int rc = ep_nccl_link((int)rank, (int)world, id, e->device, &e->ep, &msg);
  return rc == CHALOT_OK ? CHALOT_OK : set_error(rc, "ep_attach: " + msg);
}

__attribute__((visibility("default"))) chalot_ep_hub* chalot_ep_hub_create(uint32_t world) {
  if (world < 1 || world > 32) {
    set_error(CHALOT_ERR_ARG, "ep_hub_create: world in [1, 32]");
    return nullptr;
  }
  return reinterpret_cast<chalot_ep_hub*>(ep_hub_create((int)world));
}

__attribute__((visibility("default"))) void chalot_ep_hub_free(chalot_ep_hub* hub) {
  ep_hub_release(reinterpret_cast<EpHub*>(hub));
}

__attribute__((visibility("default"))) int chalot_ep_attach_hub(chalot_engine* e, chalot_ep_hub* hub,
                                                               uint32_t rank) {
  if (!hub) return set_error(CHALOT_ERR_ARG, "ep_attach: null hub");
  EpHub* h = reinterpret_cast<EpHub*>(hub);
  if (int rc = ep_check_attach(e, rank, (uint32_t)ep_hub_world(h))) return rc;
  std::string msg;
  const int rc = ep_hub_link(h, (int)rank, &e->ep, &msg);
  return rc == CHALOT_OK ? CHALOT_OK : set_error(rc, "ep_attach: " + msg);
}

__attribute__((visibility("default"))) int chalot_ep_detach(chalot_engine* e) {
  if (!e) return set_error(CHALOT_ERR_ARG, "ep_detach: null engine");
  if (e->stream) cudaStreamSynchronize(e->stream);
  e->ep.reset();
  return CHALOT_OK;
}

__attribute__((visibility("default"))) int chalot_sample(const float* logits, size_t vocab,
                                                         const chalot_sampling* cfg, float r, uint32_t* out_token,
                                                         void* stream) {
  if (!logits || !cfg || !out_token) return set_error(CHALOT_ERR_ARG, "sample: null argument");
  if (vocab == 0 || vocab > (1u << 30)) return set_error(CHALOT_ERR_ARG, "sample: bad vocab size");
  if (cfg->strategy < CHALOT_GREEDY || cfg->strategy > CHALOT_MIN_P)
    return set_error(CHALOT_ERR_ARG, "sample: unknown strategy");
  if (!(r >= 0.0f && r < 1.0f)) return set_error(CHALOT_ERR_ARG, "sample: r must be in [0, 1)");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned long long* d = nullptr;
  unsigned long long h = 0;
  cudaError_t rc = cudaMallocAsync(reinterpret_cast<void**>(&d), 8, s);
  if (rc == cudaSuccess) rc = cudaMemsetAsync(d, 0, 8, s);
  if (rc == cudaSuccess) {
    if (cfg->strategy == CHALOT_GREEDY || (cfg->strategy == CHALOT_MIN_P && cfg->min_p > 1.0f))
      rc = launch_argmax_op(logits, (int)vocab, d, s);
    else
      rc = launch_sample(logits, (int)vocab, cfg->strategy, cfg->temperature, (int)cfg->top_k, cfg->top_p,
                         cfg->min_p, r, d, s);
  }
  if (rc == cudaSuccess) rc = cudaMemcpyAsync(&h, d, 8, cudaMemcpyDeviceToHost, s);
  if (d) cudaFreeAsync(d, s);
  if (rc == cudaSuccess) rc = cudaStreamSynchronize(s);
  if (rc != cudaSuccess) return set_error(CHALOT_ERR_CUDA, std::string("sample: ") + cudaGetErrorString(rc));
  *out_token = uint32_t(h & 0xffffffffull);
  return CHALOT_OK;
}

// ---- operators ----------------------------------------------------------------

__attribute__((visibility("default"))) int chalot_matmul_i8(float* out, const int8_t* w,
                                                            const float* ws, const float* x,
                                                            size_t out_dim, size_t in_dim,
                                                            void* stream) {
  if (!out || !w || !ws || !x) return set_error(CHALOT_ERR_ARG, "null pointer");
  if (out_dim == 0 || in_dim == 0) return CHALOT_OK;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaError_t r = op_matmul_i8(out, w, ws, x, out_dim, in_dim, sms, static_cast<cudaStream_t>(stream));
  if (r != cudaSuccess) return set_error(r == cudaErrorInvalidValue ? CHALOT_ERR_ARG : CHALOT_ERR_CUDA,
                                         std::string("matmul_i8: ") + cudaGetErrorString(r));
  return CHALOT_OK;
}

__attribute__((visibility("default"))) int chalot_matmul_i4(float* out, const uint8_t* wp,
                                                            const float* ws, const float* x,
                                                            size_t out_dim, size_t in_dim,
                                                            size_t group, void* stream) {
  if (!out || !wp || !ws || !x) return set_error(CHALOT_ERR_ARG, "null pointer");
  if (group == 0) group = kDefaultInt4Group;
  if (group % 2) return set_error(CHALOT_ERR_ARG, "odd int4 group sizes are not supported");
  if (out_dim == 0 || in_dim == 0) return CHALOT_OK;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaError_t r = op_matmul_i4(out, wp, ws, x, out_dim, in_dim, group, sms,
                               static_cast<cudaStream_t>(stream));
  if (r != cudaSuccess) return set_error(r == cudaErrorInvalidValue ? CHALOT_ERR_ARG : CHALOT_ERR_CUDA,
                                         std::string("matmul_i4: ") + cudaGetErrorString(r));
  return CHALOT_OK;
}

__attribute__((visibility("default"))) int chalot_quantize_i8(int8_t* q, float* scale, const float* x,
                                                              size_t n_vec, size_t n, void* stream) {
  if (!q || !scale || !x) return set_error(CHALOT_ERR_ARG, "null pointer");
  if (n_vec == 0 || n == 0) return CHALOT_OK;
  cudaError_t r = op_quantize_i8(q, scale, x, n_vec, n, static_cast<cudaStream_t>(stream));
  if (r != cudaSuccess) return set_error(CHALOT_ERR_CUDA, cudaGetErrorString(r));
  return CHALOT_OK;
}

__attribute__((visibility("default"))) int chalot_router_topk(int32_t* idx, float* weight,
                                                              const float* x, const float* w,
                                                              const float* b, size_t n_tok,
                                                              size_t dim, size_t n_experts,
                                                              size_t top_k, void* stream) {
  if (!idx || !weight || !x || !w || !b) return set_error(CHALOT_ERR_ARG, "null pointer");
  if (n_experts == 0 || top_k == 0 || top_k > n_experts || n_experts > 32)
    return set_error(CHALOT_ERR_ARG, "need 1 <= top_k <= n_experts <= 32");
  if (n_tok == 0) return CHALOT_OK;
  cudaError_t r = op_router_topk(idx, weight, x, w, b, n_tok, dim, n_experts, top_k,
                                 static_cast<cudaStream_t>(stream));
  if (r != cudaSuccess) return set_error(r == cudaErrorInvalidValue ? CHALOT_ERR_ARG : CHALOT_ERR_CUDA,
                                         cudaGetErrorString(r));
  return CHALOT_OK;
}

}  // extern "C"
