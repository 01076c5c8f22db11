// persist.h — the persistent batch-1 decode kernel (k_persist.cu).
#pragma once

#include <cuda_runtime.h>

#include <string>

#include "kernels.cuh"

namespace chalot {

constexpr int kPersistThreads = 512;
constexpr int kPersistBarWords = 32 * 72;  // grid counter + one 128-byte line per head group
constexpr int kPvTile = 1024;              // positions of V staged per pass

// Shared-memory plan of one CTA (byte offsets) for a model shape on a GPU.
struct PersistPlan {
  int o_xq, o_xf, o_xb, o_own, o_red, o_bars, o_P, o_T, o_xh, o_stage;
  size_t smem;
  int max_pairs, max_rows;
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
  unsigned* bar;   // [kPersistBarWords] barrier counters, zero at launch
  unsigned* amax;  // [2][8] absmax(h) per layer parity and choice, zero at launch
  unsigned* err;   // set when a bounded wait gave up
  // %globaltimer of CTA 0 at the phase boundaries, [n_layers + 1][16]: per
  // layer 0 start, 1 A (after the barrier), 2 A end, 3 B1, 4 B1 end, 5 B2,
  // 6 B2 end, 7 C, 8 C end, 9 D, 10 expert copies issued, 11 E end, 12 F,
  // 13 F end; then kernel start, lm_head start, lm_head end. May be null.
  unsigned long long* trace;
};

// False (with the reason) when the shape does not fit the kernel.
bool persist_plan(const Dims& d, int num_sms, PersistPlan* plan, std::string* why);
// One decode step: embedding .. argmax into b.st->argmax_key (cooperative launch).
cudaError_t launch_persist(const PersistArgs& a, int num_sms, cudaStream_t s);
// Zeroes the barrier counters and absmax slots (after each launch_persist).
cudaError_t launch_persist_reset(unsigned* bar, unsigned* amax, cudaStream_t s);

}  // namespace chalot
