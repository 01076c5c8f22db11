// persist.h — the persistent batch-1 decode kernel (k_persist.cu).
#pragma once

#include <cuda_runtime.h>

#include <string>

#include "kernels.cuh"

namespace chalot {

constexpr int kPersistThreads = 512;
// broadcast counters (ll.cnt): three groups of 8 lines (32 words apart)
constexpr int kCntXc = 0, kCntH = 32 * 8, kCntXf = 2 * 32 * 8;
constexpr int kPersistCntWords = 3 * 32 * 8;
constexpr int kPvTile = 1024;              // positions of V products per pass
constexpr int kLmStages = 4;               // lm_head ring stages
constexpr int kLmChunk = 2 * (kPersistThreads / 32 - 1);  // lm_head rows per stage: two per compute warp

// Shared-memory plan of one CTA (byte offsets) for a model shape on a GPU.
struct PersistPlan {
  int o_xq, o_xf, o_xb, o_own, o_red, o_bars, o_xp, o_P, o_T, o_xh, o_stage;
  int o_vs, o_pp, o_vt;  // offsets inside the staging area (attention phase)
  int o_hf;              // offset inside the staging area of the f32 h (phase F)
  int o_sq, sqs;         // squares of the norm, [8][sqs] floats
  int ets;               // row stride of the exps by lane, [8][ets] floats (over the products)
  int ps_gu, ps_dn;      // row strides of the group products (floats, 4 mod 32)
  size_t smem;
  int max_pairs, max_rows;
};

// Tagged words (64 bits: the f32 value, then the 32-bit tag) through which
// the CTAs of one step pass values to each other.
struct PersistLL {
  uint64_t* x;      // [2][dim] x after the O projection, after the expert block
  uint64_t* q;      // [3][dim] this step's q, k, v
  uint64_t* score;  // [n_heads][max_seq]
  uint64_t* att;    // [dim] attention output
  uint64_t* h;      // [top_k][hidden] SwiGLU output of the selected experts
  unsigned* cnt;    // [kPersistCntWords] producer counts of the x and h broadcasts (zero at launch)
};

struct PersistArgs {
  Dims d;
  PersistPlan plan;
  const LayerPtrs* layers;  // device array [n_layers]
  const int8_t* emb;
  const float* emb_s;
  const float* final_norm;
  const int8_t* out_w;
  const float* out_s;
  DecodeBufs b;
  PersistLL ll;
  const unsigned* epoch;  // step epoch: advanced after every launch
  unsigned* err;   // set when a bounded wait gave up
  // %globaltimer of CTA 0 at the phase boundaries, [n_layers + 1][16]: per
  // layer 0 start, 1 A (after the barrier), 2 A end, 3 B1, 4 B1 end, 5 B2,
  // 6 B2 end, 7 C, 8 C end, 9 D, 10 expert copies issued, 11 E end, 12 F,
  // 13 F end; then kernel start, lm_head start, lm_head end. May be null.
  unsigned long long* trace;
  unsigned long long* trace_max;  // diagnostics: per mark the latest CTA's time (atomicMax), may be null
};

// False (with the reason) when the shape does not fit the kernel.
bool persist_plan(const Dims& d, int num_sms, PersistPlan* plan, std::string* why);
// One decode step: embedding .. argmax into b.st->argmax_key (cooperative launch).
cudaError_t launch_persist(const PersistArgs& a, int num_sms, cudaStream_t s);
// Advances the step epoch and zeroes the broadcast counters (after each
// launch_persist, in stream order).
cudaError_t launch_persist_epoch(unsigned* epoch, unsigned* cnt, cudaStream_t s);

}  // namespace chalot
