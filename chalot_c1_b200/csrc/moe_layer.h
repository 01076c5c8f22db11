// moe_layer.h — host-side interface of the batched MoE layer kernels.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace chalot {

struct MlDims {
  int T, dim, H, E, K, group;
};

// Where each expert's tensors are: gate+up packed int4 [2H][dim/2] (gate rows
// first) and their scales [2H][dim/group], down [dim][H/2] and its scales
// [dim][H/group]. Passed by value to the kernels (32 experts at most).
struct MlExpert {
  const uint8_t* gu;
  const float* gus;
  const uint8_t* dn;
  const float* dns;
};
struct MlExperts {
  MlExpert ex[32];
  int repacked;  // 0: the file's int4 layout, 1: the engine's repacked layout
};

// Device pointers into a caller-provided workspace (ml_layout).
struct MlWork {
  int32_t* sel;   // [T*k] expert of each (token, choice) slot
  float* selw;    // [T*k] its gate weight
  int8_t* xq;     // [T][dim] quantized input rows
  float* xs;      // [T] their scales
  int32_t* perm;  // [T*k] expert-sorted position -> slot
  int32_t* inv;   // [T*k] slot -> position
  int32_t* mb_e;  // 32-slot blocks: expert, first position, slot count
  int32_t* mb_p0;
  int32_t* mb_n;
  int32_t* n_mb;  // number of blocks
  float* h;       // [T*k][H] swiglu(gate, up), by position
  int8_t* hq;     // [T*k][H] quantized h
  float* hs;      // [T*k]
  float* y;       // [T*k][dim] expert outputs, by position
  unsigned* amax; // [T*k] absmax of each h row (float bits): zeroed by the dispatch, raised by the few-slot gate/up
};

// Extra workspace of the tensor-core path (k_moe_tc.cu).
struct MlTcWork {
  int8_t* xp;     // [T*k][dim] quantized x rows in expert-sorted order
  float* xsp;     // [T*k] their scales
  int8_t* w8gu;   // [E*2H][dim] gate/up weights as int8, gate/up interleaved per 64 units
  float* sgu;     // [E*dim/group][2H] their group scales, transposed
  int8_t* w8dn;   // [E*dim][H] down weights as int8
  float* sdn;     // [E*H/group][dim] their group scales, transposed
  unsigned* amax; // [T*k] absmax of each h row (float bits), reduced by the gate/up epilogue
  unsigned long long* key;  // [4] which experts w8gu..sdn hold (0: none); [4] as int: unpack needed
  unsigned* err;  // nonzero when a bounded wait ran out
};

size_t ml_expert_bytes(const MlDims& d);
// E experts back to back in the file layout from `blob`.
MlExperts ml_experts_from_blob(const MlDims& d, const uint8_t* blob);
size_t ml_layout(const MlDims& d, void* base, MlWork* w);
const char* ml_check(const MlDims& d);
cudaError_t ml_run(const MlDims& d, const float* x, const float* rw, const float* rb,
                   const MlExperts& X, const MlWork& w, float* out, cudaStream_t s);

// The batched decode's MoE block with the FFN rmsnorm fused into the router
// and the combine + residual add + next rmsnorm/quantize fused after it
// (t: the tensor-core work, or nullptr for the SIMT/few-slot kernels).
cudaError_t ml_run_decode(const MlDims& d, float* x, const float* norm_ffn, const float* rw, const float* rb,
                          const MlExperts& X, const MlWork& w, const MlTcWork* t, const float* norm_next,
                          int8_t* xq, float* xs, cudaStream_t s);

// Building blocks of the expert-parallel layer (k_moe_layer.cu).
void ml_launch_route(const MlDims& d, const float* x, const float* rw, const float* rb, const MlWork& w,
                     cudaStream_t s);
void ml_launch_plan(const MlDims& d, const MlWork& w, int n_ranks, int32_t* offs, cudaStream_t s);
void ml_launch_combine(const MlDims& d, const MlWork& w, float* out, cudaStream_t s);
// est_rows >= 0: the expected number of live rows (the rest are padding that the
// dispatch skips), which picks the expert kernels' slot tiles.
cudaError_t ml_run_rows(const MlDims& d, const MlExperts& X, const MlWork& w, const MlTcWork* t, float* y,
                        cudaStream_t s, int est_rows = -1);
bool ml_use_tc(const MlDims& d);
cudaError_t ml_run_tc(const MlDims& d, const float* x, const float* rw, const float* rb, const MlExperts& X,
                      const MlWork& w, const MlTcWork& t, float* out, cudaStream_t s);
cudaError_t ml_tc_gather_rows(const MlDims& d, const MlWork& w, const MlTcWork& t, cudaStream_t s);

bool ml_tc_eligible(const MlDims& d);
size_t ml_tc_layout(const MlDims& d, size_t off, void* base, MlTcWork* t);
cudaError_t ml_tc_prepare(const MlDims& d, const MlExperts& X, const MlWork& w, const MlTcWork& t,
                          cudaStream_t s);
cudaError_t ml_tc_gemm(const MlDims& d, bool gate_up, const MlWork& w, const MlTcWork& t,
                       unsigned n_mblocks, cudaStream_t s);
cudaError_t ml_tc_quant(const MlDims& d, const MlWork& w, const MlTcWork& t, cudaStream_t s);

}  // namespace chalot
