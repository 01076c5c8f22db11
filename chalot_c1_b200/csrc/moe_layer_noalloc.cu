// moe_layer_noalloc.cu — chalot_moe_layer_noalloc: the batched MoE layer with
// its scratch in a fixed device array of this library instead of a
// caller-provided workspace.
//
// Some callers cannot allocate device memory at the point where they run a
// layer: a host whose allocator owns the whole device budget and hands out no
// extra buffers (a serving process that reserves the GPU's memory at start-up,
// a Rust or Go host that binds only plain pointers), or a latency-critical
// loop that must not pay cudaMalloc's implicit device synchronisation. This
// entry point needs nothing from them beyond the inputs and outputs: the
// intermediate buffers (router choices, quantized rows, expert-sorted slots,
// the SwiGLU activations and the expert outputs) live in g_moe_scratch below.
//
// The array is a file-scope __device__ variable: every GPU that loads this
// library holds kNoAllocScratchBytes of it until the process exits. In host
// code its name is only a host-side stand-in, so the kernels are given the
// device address that cudaGetSymbolAddress returns; that lookup runs on the
// first call on each device (with that device current), so the first call on
// a device should come before any stream capture on it. The address is kept
// for the life of the process: after cudaDeviceReset the library's device
// copy may move, so this entry point must not be used across a device reset.
// Every call on a device shares the one array and it keeps the last call's
// contents: each call
// writes every scratch byte it reads, so nothing has to start at zero, and two
// calls whose executions overlap on the GPU (different streams, or different
// host threads without ordering) race on the array.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "capi_internal.h"
#include "moe_layer.h"

namespace chalot {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;  // 4 MiB per device
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_moe_scratch[kNoAllocScratchBytes];

std::mutex g_addr_mu;
void* g_addr[kMaxDevices] = {};

// Device address of g_moe_scratch on the current device (looked up once).
cudaError_t scratch_address(void** out) {
  int dev = 0;
  cudaError_t r = cudaGetDevice(&dev);
  if (r != cudaSuccess) return r;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_addr_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    r = cudaGetSymbolAddress(&p, g_moe_scratch);
    if (r != cudaSuccess) return r;
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return cudaSuccess;
}

}  // namespace
}  // namespace chalot

using namespace chalot;

extern "C" {

__attribute__((visibility("default"))) int chalot_moe_layer_noalloc(const chalot_moe_desc* desc,
                                                                    const float* x, size_t n_tok,
                                                                    float* out, int32_t* sel_out,
                                                                    float* selw_out, void* stream) {
  if (!desc) return set_error(CHALOT_ERR_ARG, "moe_layer_noalloc: null descriptor");
  if (n_tok == 0) return CHALOT_OK;
  // validation as chalot_moe_layer does it (0: invalid, chalot_last_error says why)
  if (chalot_moe_workspace_size(desc, n_tok) == 0) return CHALOT_ERR_ARG;
  const MlDims d{(int)n_tok, (int)desc->dim, (int)desc->hidden_dim, (int)desc->n_experts,
                 (int)desc->top_k, (int)(desc->group ? desc->group : 32)};
  // the scratch of the path this entry point runs (ml_run), whatever path
  // chalot_moe_layer would pick for the shape
  const size_t need = ml_layout(d, nullptr, nullptr);
  if (need > kNoAllocScratchBytes)
    return set_error(CHALOT_ERR_ARG, "moe_layer_noalloc: " + std::to_string(n_tok) +
                                         " tokens need " + std::to_string(need) +
                                         " bytes of scratch, above the fixed " +
                                         std::to_string(kNoAllocScratchBytes) +
                                         "; use chalot_moe_layer with a workspace");
  if (!x || !out) return set_error(CHALOT_ERR_ARG, "moe_layer_noalloc: null x or out");
  void* base = nullptr;
  cudaError_t r = scratch_address(&base);
  if (r != cudaSuccess)
    return set_error(CHALOT_ERR_CUDA, std::string("moe_layer_noalloc: scratch address: ") +
                                          cudaGetErrorString(r));
  MlWork w;
  ml_layout(d, base, &w);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  r = ml_run(d, x, desc->router_w, desc->router_b, ml_experts_from_blob(d, desc->experts), w, out, s);
  const size_t N = n_tok * d.K;
  if (r == cudaSuccess && sel_out) r = cudaMemcpyAsync(sel_out, w.sel, N * 4, cudaMemcpyDeviceToDevice, s);
  if (r == cudaSuccess && selw_out)
    r = cudaMemcpyAsync(selw_out, w.selw, N * 4, cudaMemcpyDeviceToDevice, s);
  if (r != cudaSuccess)
    return set_error(CHALOT_ERR_CUDA, std::string("moe_layer_noalloc: ") + cudaGetErrorString(r));
  return CHALOT_OK;
}

}  // extern "C"
