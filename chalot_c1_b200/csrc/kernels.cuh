// kernels.cuh — launch interfaces of the sm_100a kernels of the decode path.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace chalot {

// Model dimensions as the kernels see them.
struct Dims {
  int dim, hidden, n_layers, n_heads, head_dim, vocab, max_seq, n_experts, top_k, group;
};

// Device pointers of one expert's tensors (src/model/weight_index.rs:10-23).
struct ExpertPtrs {
  const uint8_t* gu;  // [2*hidden][ceil(dim/2)], gate rows then up rows
  const float* gu_s;  // [2*hidden][ceil(dim/group)]
  const uint8_t* dn;  // [dim][ceil(hidden/2)]
  const float* dn_s;  // [dim][ceil(hidden/group)]
};

// Device pointers of one transformer layer (src/model/weight_index.rs:26-52).
struct LayerPtrs {
  const float* rms_attn;
  const int8_t* qkv;   // [3*dim][dim]: Q rows, K rows, V rows
  const float* qkv_s;  // [3*dim]
  const int8_t* o;     // [dim][dim]
  const float* o_s;    // [dim]
  const float* rms_ffn;
  const float* router_w;  // [E][dim] (MoE only)
  const float* router_b;  // [E]
  const ExpertPtrs* experts;  // device table of E entries
  ExpertPtrs ex[16];          // the same pointers as kernel parameters (E <= 16)
};

// Pointers of expert e: from the kernel parameters when E <= 16 (no memory
// round trip), else from the device table.
__device__ __forceinline__ ExpertPtrs expert_ptrs(const LayerPtrs& L, int E, int e) {
  if (E <= 16) {
    ExpertPtrs r = L.ex[0];
#pragma unroll
    for (int i = 1; i < 16; ++i)
      if (i == e) r = L.ex[i];
    return r;
  }
  return L.experts[e];
}

constexpr int kTickets = 16;

// Per-engine device buffers of the batch-1 decode path.
struct DecodeBufs {
  float* x;          // [dim] residual stream
  float* q;          // [dim] rotated query
  float* att_out;    // [dim]
  float* scores;     // [n_heads][max_seq]
  float* kc;         // [n_layers][max_seq][dim] f32 key cache
  float* vc;         // [n_layers][max_seq][dim] f32 value cache
  const float* rope_cos;  // [max_seq][head_dim/2]
  const float* rope_sin;
  int8_t* xq_attn;   // [dim] quantized attention input (rmsnorm(x) of this layer)
  float* xs_attn;    // [1] its scale
  int8_t* xq_ffn;    // [dim] quantized FFN input
  float* xs_ffn;     // [1] its scale
  unsigned* counters;  // [kTickets] last-CTA tickets: [1] O-projection, [2] down, [8 + j] gate/up of expert j
  unsigned* err;       // [1] set when a bounded wait gave up
  int32_t* sel;      // [top_k] selected experts
  float* selw;       // [top_k] their weights
  float* h;          // [top_k][hidden] SwiGLU output
  unsigned* amax;    // [top_k] absmax bits of h
  int8_t* xq_h;      // [top_k][hidden] quantized h (down-projection input)
  float* xs_h;       // [top_k] its scales
  float* logits;     // [vocab]
  StepState* st;
  const uint32_t* prompt;  // [max_seq] prompt of the running generate call
  uint32_t* out_tokens;    // [max_seq] argmax of every forward
  float* router_trace;     // [n_layers][E] router logits of the last forward (may be null)
};

// ---- decode step (batch 1) ---------------------------------------------------
// Kernels after the first of a forward are launched with programmatic
// dependent launch (`pdl`); see pdl.cuh for the rules they follow.
// x = embedding(token).
void launch_embed(const Dims& d, const int8_t* emb, const float* emb_s, const DecodeBufs& b,
                  cudaStream_t s);
// quantize(rmsnorm(x, rms_attn)) in every CTA, Q/K/V rows, RoPE, KV-cache write.
void launch_qkv(const Dims& d, const LayerPtrs& L, int layer, const DecodeBufs& b, cudaStream_t s,
                bool pdl);
// Scores and softmax.P.V into att_out.
void launch_attention(const Dims& d, int layer, const DecodeBufs& b, cudaStream_t s, bool pdl);
void launch_scores(const Dims& d, int layer, const DecodeBufs& b, cudaStream_t s, bool pdl);
void launch_pv(const Dims& d, int layer, const DecodeBufs& b, cudaStream_t s, bool pdl);
// O rows from quantize(att_out), x += ; the last CTA computes the FFN norm, xq_ffn and the routing.
void launch_oproj(const Dims& d, const LayerPtrs& L, int layer, const DecodeBufs& b,
                  cudaStream_t s, bool pdl);
// Gate/up rows of the routed experts + SwiGLU -> h, absmax(h); the last CTA
// quantizes h into xq_h/xs_h.
void launch_gateup(const Dims& d, const LayerPtrs& L, int layer, const DecodeBufs& b, cudaStream_t s,
                   bool pdl);
// Down rows of every routed expert, gated combine, x += ; with `next_norm`
// (the final norm, after the last layer) the last CTA computes xq_attn for
// the lm_head; null for the other layers.
void launch_down(const Dims& d, const LayerPtrs& L, int layer, const float* next_norm,
                 const DecodeBufs& b, cudaStream_t s, bool pdl);
// Logits from xq_attn (the final-norm input) + argmax.
void launch_lmhead(const Dims& d, const int8_t* w, const float* ws, const DecodeBufs& b,
                   int num_sms, cudaStream_t s, bool pdl);
// Records the argmax of the forward and selects the next token/position.
void launch_advance(const Dims& d, const DecodeBufs& b, cudaStream_t s, bool pdl);
// Repetition penalty on the logits followed by a fresh argmax into st->argmax_key.
// One draw of a sampling strategy (k_sample.cu); the token goes to *out.
cudaError_t launch_sample(const float* logits, int V, int strategy, float temperature, int top_k, float top_p,
                          float min_p, float r, unsigned long long* out, cudaStream_t s);
// argmax with ties to the last index into *out (cleared by the caller).
cudaError_t launch_argmax_op(const float* logits, int V, unsigned long long* out, cudaStream_t s);
void launch_penalty_argmax(const Dims& d, const DecodeBufs& b, const uint32_t* hist, int n_hist,
                           float penalty, cudaStream_t s);

// Converts packed int4 rows (bytes % 4 == 0) in place from the file layout to
// the engine's repacked layout (repack_word in common.cuh).
cudaError_t repack_int4(uint8_t* p, size_t bytes, cudaStream_t s);

// ---- operator entry points ------------------------------------------------------
cudaError_t op_matmul_i8(float* out, const int8_t* w, const float* ws, const float* x,
                         size_t out_dim, size_t in_dim, int num_sms, cudaStream_t s);
cudaError_t op_matmul_i4(float* out, const uint8_t* wp, const float* ws, const float* x,
                         size_t out_dim, size_t in_dim, size_t group, int num_sms, cudaStream_t s);
cudaError_t op_quantize_i8(int8_t* q, float* scale, const float* x, size_t n_vec, size_t n,
                           cudaStream_t s);
cudaError_t op_router_topk(int32_t* idx, float* w, const float* x, const float* rw,
                           const float* rb, size_t n_tok, size_t dim, size_t n_experts,
                           size_t top_k, cudaStream_t s);

}  // namespace chalot
