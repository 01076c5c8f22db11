// batch.h — launchers of the batched-decode kernels (k_batch.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

namespace chalot {

// Shapes of the batched decode, and where its K/V rows live: either the
// flat cache [slot][layer][max_seq][dim] (ptab == nullptr) or a pool of pages
// of 2^pt_shift positions, page p holding [layer][position in page][dim], with
// the page of position t of a slot at ptab[slot * maxp + (t >> pt_shift)].
struct BatchDims {
  int dim, n_layers, n_heads, head_dim, max_seq;
  const int32_t* ptab = nullptr;
  int pt_shift = 0, maxp = 0;
};

void b_embed(const BatchDims& d, int B, const uint32_t* toks, const int8_t* emb, const float* emb_s,
             const float* rms0, float* x, int8_t* xq, float* xs, cudaStream_t s);
void b_norm_quant(const BatchDims& d, int B, const float* x, const float* w, int8_t* xq, float* xs,
                  cudaStream_t s);
void b_gemm_i8(int B, int R, int C, const int8_t* W, const float* ws, const int8_t* xq, const float* xs,
               float* out, int ldo, bool add, cudaStream_t s);
// The same GEMM on the tensor cores (k_dense_tc.cu) when eligible: B <= 256,
// C % 128 == 0, W and xq 16-byte aligned.
bool b_gemm_tc_eligible(int B, int C, const int8_t* W, const int8_t* xq);
cudaError_t b_gemm_tc(int B, int R, int C, const int8_t* W, const float* ws, const int8_t* xq, const float* xs,
                      float* out, int ldo, bool add, cudaStream_t s);
void b_rope_kv(const BatchDims& d, int layer, int B, const int32_t* pos, const int32_t* slot, const float* qkv,
               float* q, float* kc, float* vc, const float* rcos, const float* rsin, cudaStream_t s);
void b_attention(const BatchDims& d, int layer, int B, const int32_t* pos, const int32_t* slot, const float* q,
                 const float* kc, const float* vc, float* scores, float* att, cudaStream_t s);
void b_rmsnorm(const BatchDims& d, int B, const float* x, const float* w, float* xb, cudaStream_t s);
void b_add(long n, float* x, const float* y, cudaStream_t s);
void b_argmax(int B, int V, const float* logits, uint32_t* out, cudaStream_t s);

}  // namespace chalot
