// moe_ep.cu — C ABI of the building blocks of an expert-parallel MoE layer.
//
// Expert e lives on rank e % n_ranks. Per layer each rank: routes its own
// tokens (chalot_moe_route), orders the (token, choice) slots by destination
// rank and local expert (chalot_moe_plan), gathers the int8 rows in that order
// (chalot_moe_gather), exchanges counts, rows and scales with the other ranks
// (the caller's all-to-all; int8 rows are exact and 4x smaller than f32),
// computes the experts it holds on the rows it received (chalot_moe_experts),
// sends the f32 outputs back, and combines them in selection order
// (chalot_moe_combine). Every step keeps the reference's per-token arithmetic
// (src/model/engine.rs:334-401), so the result is bit-identical to
// chalot_moe_layer on one GPU.
#include <cuda_runtime.h>

#include <string>

#include "capi_internal.h"
#include "devstat.h"
#include "moe_layer.h"

using namespace chalot;

namespace {

int cuda_fail(const char* what, cudaError_t r) {
  return set_error(CHALOT_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(r));
}

bool experts_dims(const chalot_moe_desc* d, size_t n_rows, MlDims* out, std::string* why) {
  if (!d) {
    *why = "null descriptor";
    return false;
  }
  MlDims m{(int)n_rows, (int)d->dim, (int)d->hidden_dim, (int)d->n_experts, 1, (int)(d->group ? d->group : 32)};
  // the router checks do not apply: a rank may hold a single expert
  MlDims c = m;
  c.E = 2;
  c.K = 1;
  if (const char* e = ml_check(c)) {
    *why = e;
    return false;
  }
  if (m.E < 1 || m.E > 32) {
    *why = "n_experts (local) must be in [1, 32]";
    return false;
  }
  if (n_rows > (size_t)(1 << 20)) {
    *why = "at most 2^20 rows";
    return false;
  }
  if (!d->experts || (reinterpret_cast<uintptr_t>(d->experts) & 15)) {
    *why = "experts must be non-null and 16-byte aligned";
    return false;
  }
  *out = m;
  return true;
}

size_t experts_need(const MlDims& m, bool* tc) {
  *tc = ml_use_tc(m);
  const size_t simt = ml_layout(m, nullptr, nullptr);
  return *tc ? ml_tc_layout(m, simt, nullptr, nullptr) : simt;
}

}  // namespace

extern "C" {

__attribute__((visibility("default"))) int chalot_moe_route(const chalot_moe_desc* desc, const float* x,
                                                            size_t n_tok, int32_t* sel, float* selw, int8_t* xq,
                                                            float* xs, void* stream) {
  if (!desc) return set_error(CHALOT_ERR_ARG, "moe_route: null descriptor");
  MlDims d{(int)n_tok, (int)desc->dim, (int)desc->hidden_dim, (int)desc->n_experts, (int)desc->top_k,
           (int)(desc->group ? desc->group : 32)};
  if (const char* m = ml_check(d)) return set_error(CHALOT_ERR_ARG, std::string("moe_route: ") + m);
  if (n_tok == 0) return CHALOT_OK;
  if (!x || !sel || !selw || !xq || !xs || !desc->router_w || !desc->router_b)
    return set_error(CHALOT_ERR_ARG, "moe_route: null pointer");
  if (n_tok > 65535u * 1024u) return set_error(CHALOT_ERR_ARG, "moe_route: too many tokens");
  MlWork w{};
  w.sel = sel;
  w.selw = selw;
  w.xq = xq;
  w.xs = xs;
  ml_launch_route(d, x, desc->router_w, desc->router_b, w, static_cast<cudaStream_t>(stream));
  cudaError_t r = cudaGetLastError();
  return r == cudaSuccess ? CHALOT_OK : cuda_fail("moe_route", r);
}

__attribute__((visibility("default"))) int chalot_moe_plan(const int32_t* sel, size_t n_slots, uint32_t n_experts,
                                                           uint32_t n_ranks, int32_t* order, int32_t* pos,
                                                           int32_t* offsets, void* stream) {
  if (n_experts < 1 || n_experts > 32 || n_ranks < 1 || n_experts % n_ranks)
    return set_error(CHALOT_ERR_ARG, "moe_plan: need 1 <= n_experts <= 32 and n_ranks dividing n_experts");
  if (n_slots > (size_t)(1 << 20)) return set_error(CHALOT_ERR_ARG, "moe_plan: at most 2^20 slots");
  if (!offsets) return set_error(CHALOT_ERR_ARG, "moe_plan: null offsets");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n_slots == 0) {
    cudaError_t r = cudaMemsetAsync(offsets, 0, (n_experts + 1) * sizeof(int32_t), s);
    return r == cudaSuccess ? CHALOT_OK : cuda_fail("moe_plan", r);
  }
  if (!sel || !order || !pos) return set_error(CHALOT_ERR_ARG, "moe_plan: null pointer");
  MlDims d{(int)n_slots, 0, 0, (int)n_experts, 1, 32};
  MlWork w{};
  w.sel = const_cast<int32_t*>(sel);
  w.perm = order;
  w.inv = pos;
  ml_launch_plan(d, w, (int)n_ranks, offsets, s);
  cudaError_t r = cudaGetLastError();
  return r == cudaSuccess ? CHALOT_OK : cuda_fail("moe_plan", r);
}

__attribute__((visibility("default"))) int chalot_moe_gather(const int8_t* xq, const float* xs, const int32_t* order,
                                                             size_t n_slots, uint32_t top_k, size_t dim, int8_t* rows,
                                                             float* row_scales, void* stream) {
  if (n_slots == 0) return CHALOT_OK;
  if (!xq || !xs || !order || !rows || !row_scales) return set_error(CHALOT_ERR_ARG, "moe_gather: null pointer");
  if (top_k < 1 || dim == 0 || dim % 16 || n_slots % top_k)
    return set_error(CHALOT_ERR_ARG, "moe_gather: need top_k >= 1, dim % 16 == 0, n_slots % top_k == 0");
  if (((reinterpret_cast<uintptr_t>(xq) | reinterpret_cast<uintptr_t>(rows)) & 15))
    return set_error(CHALOT_ERR_ARG, "moe_gather: row buffers must be 16-byte aligned");
  MlDims d{(int)(n_slots / top_k), (int)dim, 0, 1, (int)top_k, 32};
  MlWork w{};
  w.xq = const_cast<int8_t*>(xq);
  w.xs = const_cast<float*>(xs);
  w.perm = const_cast<int32_t*>(order);
  MlTcWork t{};
  t.xp = rows;
  t.xsp = row_scales;
  cudaError_t r = ml_tc_gather_rows(d, w, t, static_cast<cudaStream_t>(stream));
  return r == cudaSuccess ? CHALOT_OK : cuda_fail("moe_gather", r);
}

__attribute__((visibility("default"))) size_t chalot_moe_experts_workspace_size(const chalot_moe_desc* local,
                                                                                size_t n_rows) {
  MlDims m;
  std::string why;
  if (!experts_dims(local, n_rows, &m, &why)) {
    set_error(CHALOT_ERR_ARG, "moe_experts: " + why);
    return 0;
  }
  bool tc;
  return experts_need(m, &tc);
}

__attribute__((visibility("default"))) int chalot_moe_experts(const chalot_moe_desc* local, const int8_t* rows,
                                                              const float* row_scales, const int32_t* row_expert,
                                                              size_t n_rows, float* y, void* workspace,
                                                              size_t workspace_bytes, void* stream) {
  MlDims m;
  std::string why;
  if (!experts_dims(local, n_rows, &m, &why)) return set_error(CHALOT_ERR_ARG, "moe_experts: " + why);
  if (n_rows == 0) return CHALOT_OK;
  if (!rows || !row_scales || !row_expert || !y) return set_error(CHALOT_ERR_ARG, "moe_experts: null pointer");
  if (int rc = devstat_poll("moe_experts", static_cast<cudaStream_t>(stream))) return rc;
  bool tc;
  const size_t need = experts_need(m, &tc);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return set_error(CHALOT_ERR_ARG, "moe_experts: workspace too small or not 256-byte aligned (need " +
                                         std::to_string(need) + " bytes)");
  MlWork w;
  const size_t simt = ml_layout(m, workspace, &w);
  MlTcWork t{};
  if (tc) ml_tc_layout(m, simt, workspace, &t);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t r = cudaMemcpyAsync(w.sel, row_expert, n_rows * 4, cudaMemcpyDeviceToDevice, s);
  if (r == cudaSuccess) r = cudaMemcpyAsync(w.xq, rows, n_rows * m.dim, cudaMemcpyDeviceToDevice, s);
  if (r == cudaSuccess) r = cudaMemcpyAsync(w.xs, row_scales, n_rows * 4, cudaMemcpyDeviceToDevice, s);
  if (r == cudaSuccess) r = ml_run_rows(m, ml_experts_from_blob(m, local->experts), w, tc ? &t : nullptr, y, s);
  return r == cudaSuccess ? CHALOT_OK : cuda_fail("moe_experts", r);
}

__attribute__((visibility("default"))) int chalot_moe_combine(const float* y, const int32_t* pos, const float* selw,
                                                              size_t n_tok, uint32_t top_k, size_t dim, float* out,
                                                              void* stream) {
  if (n_tok == 0) return CHALOT_OK;
  if (!y || !pos || !selw || !out) return set_error(CHALOT_ERR_ARG, "moe_combine: null pointer");
  if (top_k < 1 || dim == 0 || n_tok > 65535u * 1024u) return set_error(CHALOT_ERR_ARG, "moe_combine: bad sizes");
  MlDims d{(int)n_tok, (int)dim, 0, 1, (int)top_k, 32};
  MlWork w{};
  w.y = const_cast<float*>(y);
  w.inv = const_cast<int32_t*>(pos);
  w.selw = const_cast<float*>(selw);
  ml_launch_combine(d, w, out, static_cast<cudaStream_t>(stream));
  cudaError_t r = cudaGetLastError();
  return r == cudaSuccess ? CHALOT_OK : cuda_fail("moe_combine", r);
}

}  // extern "C"
