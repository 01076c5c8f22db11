// ep_comm.cu — the expert-parallel MoE layer inside the library, its token
// exchange over NVLink peer memory (chalot_ep_comm_*, chalot_moe_layer_ep).
//
// Expert e lives on rank e % world (one process per GPU of one node). Each
// rank owns an exchange arena in its GPU memory, exported with a CUDA IPC
// handle and mapped by every other rank (plain peer loads and stores over
// NVLink, no multicast, no library collective):
//   meta[world]        per source rank: its slot counts per local expert of
//                      this rank, where its block starts in its own plan, and
//                      two tags (rows sent, outputs returned)
//   recv_rows[world]   per source rank: the int8 rows it sent to this rank
//   recv_scale[world]  their f32 quantization scales
//   back_y             this rank's slots' expert outputs, in plan order,
//                      written by the ranks that hold the experts
// One layer call on each rank (all ranks call in the same order; the call
// counter is the tag, so no word of an earlier call can match):
//   1. route (router, softmax_top_k, quantize x: the reference's per-token
//      arithmetic) and plan: a stable counting sort of the (token, choice)
//      slots by destination rank, then by the destination's local expert;
//   2. dispatch: every slot's int8 row and scale stored straight into the
//      destination rank's arena; then the counts and the tag;
//   3. every rank waits (bounded) for the tags of all sources, runs its local
//      experts on the received rows (tile GEMMs or tcgen05 tensor cores);
//   4. return: each output row stored into its source rank's back_y at the
//      slot's plan position; then the tag;
//   5. every rank waits for the returns and combines per token in selection
//      order (engine.rs:390-396).
// Counts and offsets never leave the device; nothing is padded on the wire.
// Shipping int8 rows is exact, so the layer is bit-identical to
// chalot_moe_layer on one GPU. Reuse of the arena across calls is safe without
// double buffering: a rank starts call c+1 only after every rank returned its
// call-c outputs, i.e. after every rank finished reading its call-c rows.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "capi_internal.h"
#include "common.cuh"
#include "devstat.h"
#include "moe_layer.h"

namespace chalot {
namespace {

constexpr int kEpMaxWorld = 8;
constexpr int kEpMaxLocal = 32;
constexpr unsigned long long kEpWaitNs = 5ull * 1000 * 1000 * 1000;  // 5 s: every rank must call

struct EpMeta {
  int counts[kEpMaxLocal];  // slots per local expert of the receiving rank
  int start;                // first position of the block in the source's plan
  unsigned tag_rows;        // the source's rows, counts and start are written
  unsigned tag_back;        // this rank (as expert holder) returned the source's outputs
  int pad[29];
};
static_assert(sizeof(EpMeta) == 256, "EpMeta is one 256-byte block");

struct EpArena {  // byte offsets inside every rank's arena (the same on all ranks)
  size_t meta, rows, scale, back, bytes;
};

EpArena arena_layout(int world, size_t cap_rows, int dim) {
  EpArena a{};
  size_t off = 0;
  auto take = [&](size_t b) {
    const size_t o = off;
    off += (b + 255) & ~size_t(255);
    return o;
  };
  a.meta = take(sizeof(EpMeta) * world);
  a.rows = take((size_t)world * cap_rows * dim);
  a.scale = take((size_t)world * cap_rows * 4);
  a.back = take(cap_rows * (size_t)dim * 4);
  a.bytes = off;
  return a;
}

struct EpPeers {
  unsigned char* base[kEpMaxWorld];  // every rank's arena as this rank addresses it
};

CHALOT_DEV unsigned long long ep_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Waits until *flag == tag (a peer's store), bounded; false on timeout (the
// device-check word records it).
CHALOT_DEV bool ep_wait(const volatile unsigned* flag, unsigned tag, unsigned* err) {
  if (*flag == tag) return true;
  const unsigned long long t0 = ep_now();
  while (*flag != tag) {
    __nanosleep(64);
    if (ep_now() - t0 > kEpWaitNs) {
      *(volatile unsigned*)err = 1u;
      return false;
    }
  }
  return true;
}

// One warp per plan position q: the slot's int8 row and scale into its
// destination rank's arena, at the slot's place in this rank's block there.
__global__ void __launch_bounds__(256) k_ep_dispatch(EpPeers peers, EpArena a, int rank, int world, int El, int K,
                                                     int dim, size_t cap_rows, const int32_t* __restrict__ order,
                                                     const int32_t* __restrict__ offs, const int8_t* __restrict__ xq,
                                                     const float* __restrict__ xs, int n_pos) {
  const int lane = threadIdx.x & 31;
  const int q = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (q < n_pos) {
    int r = 0;
    while (r + 1 < world && q >= offs[(r + 1) * El]) ++r;
    const int i = q - offs[r * El];
    const int tok = order[q] / K;
    unsigned char* dst = peers.base[r];
    const uint4* src = reinterpret_cast<const uint4*>(xq + (size_t)tok * dim);
    uint4* drow = reinterpret_cast<uint4*>(dst + a.rows + ((size_t)rank * cap_rows + i) * dim);
    for (int j = lane; j < dim / 16; j += 32) drow[j] = __ldg(src + j);
    if (lane == 0) reinterpret_cast<float*>(dst + a.scale)[(size_t)rank * cap_rows + i] = xs[tok];
  }
  __threadfence_system();
}

// Thread r: the counts and block start of destination r into its arena's
// meta[rank], then (after a system-wide fence) the tag.
__global__ void k_ep_signal_rows(EpPeers peers, EpArena a, int rank, int world, int El,
                                 const int32_t* __restrict__ offs, unsigned tag) {
  const int r = threadIdx.x;
  if (r >= world) return;
  EpMeta* m = reinterpret_cast<EpMeta*>(peers.base[r] + a.meta) + rank;
  for (int j = 0; j < El; ++j) m->counts[j] = offs[r * El + j + 1] - offs[r * El + j];
  m->start = offs[r * El];
  __threadfence_system();
  *(volatile unsigned*)&m->tag_rows = tag;
}

// Block (source s, chunk): waits for s's rows, then the local expert of every
// received row of s (-1 past s's count, skipped by the expert kernels).
__global__ void __launch_bounds__(256) k_ep_recv_index(EpArena a, unsigned char* mine, int El, size_t cap_rows,
                                                       unsigned tag, int32_t* row_expert, unsigned* err) {
  const int s = blockIdx.y;
  const EpMeta* m = reinterpret_cast<const EpMeta*>(mine + a.meta) + s;
  __shared__ int ok_s, cum[kEpMaxLocal + 1];
  if (threadIdx.x == 0) {
    ok_s = ep_wait(&m->tag_rows, tag, err) ? 1 : 0;
    __threadfence_system();
    cum[0] = 0;
    for (int j = 0; j < El; ++j) cum[j + 1] = cum[j] + ((volatile const int*)m->counts)[j];
  }
  __syncthreads();
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= cap_rows) return;
  int e = -1;
  if (ok_s && (int)i < cum[El]) {
    e = 0;
    while ((int)i >= cum[e + 1]) ++e;
  }
  row_expert[(size_t)s * cap_rows + i] = e;
}

// One warp per received row (s, i): its output row into source s's back_y at
// the row's place in s's plan.
__global__ void __launch_bounds__(256) k_ep_return(EpPeers peers, EpArena a, unsigned char* mine, int rank, int El,
                                                   int dim, size_t cap_rows, const float* __restrict__ y, int world) {
  const int lane = threadIdx.x & 31;
  const size_t row = (size_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row < (size_t)world * cap_rows) {
    const int s = (int)(row / cap_rows), i = (int)(row % cap_rows);
    const EpMeta* m = reinterpret_cast<const EpMeta*>(mine + a.meta) + s;
    int n = 0;
    for (int j = 0; j < El; ++j) n += m->counts[j];
    if (i < n) {
      const float4* src = reinterpret_cast<const float4*>(y + row * dim);
      float4* dst = reinterpret_cast<float4*>(peers.base[s] + a.back) + ((size_t)m->start + i) * (dim / 4);
      for (int j = lane; j < dim / 4; j += 32) dst[j] = src[j];
    }
  }
  __threadfence_system();
}

__global__ void k_ep_signal_back(EpPeers peers, EpArena a, int rank, int world, unsigned tag) {
  const int s = threadIdx.x;
  if (s >= world) return;
  __threadfence_system();
  EpMeta* m = reinterpret_cast<EpMeta*>(peers.base[s] + a.meta) + rank;
  *(volatile unsigned*)&m->tag_back = tag;
}

__global__ void k_ep_wait_back(EpArena a, unsigned char* mine, int world, unsigned tag, unsigned* err) {
  const int r = threadIdx.x;
  if (r < world) {
    const EpMeta* m = reinterpret_cast<const EpMeta*>(mine + a.meta) + r;
    ep_wait(&m->tag_back, tag, err);
  }
  __threadfence_system();
}

}  // namespace
}  // namespace chalot

using namespace chalot;

struct chalot_ep_comm {
  int rank = 0, world = 1, device = 0;
  int dim = 0, hidden = 0, E = 0, K = 0, group = 32;
  size_t max_tokens = 0, cap_rows = 0;
  EpArena arena{};
  unsigned char* mine = nullptr;  // this rank's arena (cudaMalloc, exported)
  EpPeers peers{};
  bool connected = false;
  unsigned tag = 0;
  // local scratch
  int32_t *sel = nullptr, *order = nullptr, *pos = nullptr, *offs = nullptr, *row_expert = nullptr;
  float *selw = nullptr, *xs = nullptr, *y = nullptr;
  int8_t* xq = nullptr;
  void* ws = nullptr;
  size_t ws_bytes = 0;
  std::vector<void*> allocs;

  ~chalot_ep_comm() {
    if (cudaSetDevice(device) != cudaSuccess) return;
    for (int r = 0; r < world; ++r)
      if (r != rank && peers.base[r]) cudaIpcCloseMemHandle(peers.base[r]);
    for (void* p : allocs) cudaFree(p);
    if (mine) cudaFree(mine);
  }
};

namespace {

MlDims ep_local_dims(const chalot_ep_comm* c) {
  return MlDims{(int)(c->world * c->cap_rows), c->dim, c->hidden, c->E / c->world, 1, c->group};
}

int ep_fail(const char* what, cudaError_t r) {
  return set_error(CHALOT_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(r));
}

}  // namespace

extern "C" {

__attribute__((visibility("default"))) int chalot_ep_comm_create(uint32_t rank, uint32_t world,
                                                                  const chalot_moe_desc* desc, size_t max_tokens,
                                                                  chalot_ep_comm** out, uint8_t* handle) {
  if (!desc || !out || !handle) return set_error(CHALOT_ERR_ARG, "ep_comm_create: null argument");
  if (world < 1 || world > (uint32_t)kEpMaxWorld || rank >= world)
    return set_error(CHALOT_ERR_ARG, "ep_comm_create: need 1 <= world <= 8 and rank < world");
  if (desc->n_experts < 2 || desc->n_experts % world || desc->n_experts / world > (uint32_t)kEpMaxLocal)
    return set_error(CHALOT_ERR_ARG, "ep_comm_create: n_experts must be >= 2 and a multiple of world");
  MlDims full{(int)max_tokens, (int)desc->dim, (int)desc->hidden_dim, (int)desc->n_experts, (int)desc->top_k,
              (int)(desc->group ? desc->group : 32)};
  if (const char* m = ml_check(full)) return set_error(CHALOT_ERR_ARG, std::string("ep_comm_create: ") + m);
  if (max_tokens == 0 || max_tokens * desc->top_k * world > (size_t)(1 << 20))
    return set_error(CHALOT_ERR_ARG, "ep_comm_create: max_tokens * top_k * world must be in [1, 2^20]");
  auto c = std::make_unique<chalot_ep_comm>();
  c->rank = (int)rank;
  c->world = (int)world;
  c->dim = full.dim;
  c->hidden = full.H;
  c->E = full.E;
  c->K = full.K;
  c->group = full.group;
  c->max_tokens = max_tokens;
  c->cap_rows = max_tokens * full.K;
  cudaError_t r = cudaGetDevice(&c->device);
  if (r != cudaSuccess) return ep_fail("ep_comm_create", r);
  c->arena = arena_layout(c->world, c->cap_rows, c->dim);
  auto alloc = [&](size_t bytes, void** p) {
    cudaError_t e = cudaMalloc(p, std::max<size_t>(bytes, 256));
    if (e == cudaSuccess) {
      c->allocs.push_back(*p);
      e = cudaMemset(*p, 0, std::max<size_t>(bytes, 256));
    }
    return e;
  };
  r = cudaMalloc(reinterpret_cast<void**>(&c->mine), c->arena.bytes);
  if (r == cudaSuccess) r = cudaMemset(c->mine, 0, c->arena.bytes);
  const size_t N = c->cap_rows, R = (size_t)c->world * c->cap_rows;
  if (r == cudaSuccess) r = alloc(N * 4, reinterpret_cast<void**>(&c->sel));
  if (r == cudaSuccess) r = alloc(N * 4, reinterpret_cast<void**>(&c->selw));
  if (r == cudaSuccess) r = alloc(max_tokens * (size_t)c->dim, reinterpret_cast<void**>(&c->xq));
  if (r == cudaSuccess) r = alloc(max_tokens * 4, reinterpret_cast<void**>(&c->xs));
  if (r == cudaSuccess) r = alloc(N * 4, reinterpret_cast<void**>(&c->order));
  if (r == cudaSuccess) r = alloc(N * 4, reinterpret_cast<void**>(&c->pos));
  if (r == cudaSuccess) r = alloc((size_t)(c->E + 1) * 4, reinterpret_cast<void**>(&c->offs));
  if (r == cudaSuccess) r = alloc(R * 4, reinterpret_cast<void**>(&c->row_expert));
  if (r == cudaSuccess) r = alloc(R * (size_t)c->dim * 4, reinterpret_cast<void**>(&c->y));
  if (r == cudaSuccess) {
    const MlDims m = ep_local_dims(c.get());
    const size_t simt = ml_layout(m, nullptr, nullptr);
    c->ws_bytes = ml_use_tc(m) ? ml_tc_layout(m, simt, nullptr, nullptr) : simt;
    r = alloc(c->ws_bytes, &c->ws);
  }
  cudaIpcMemHandle_t h;
  if (r == cudaSuccess) r = cudaIpcGetMemHandle(&h, c->mine);
  if (r != cudaSuccess) return ep_fail("ep_comm_create", r);
  std::memcpy(handle, &h, sizeof h);
  c->peers.base[c->rank] = c->mine;
  *out = c.release();
  return CHALOT_OK;
}

__attribute__((visibility("default"))) int chalot_ep_comm_connect(chalot_ep_comm* c, const uint8_t* all_handles) {
  if (!c || !all_handles) return set_error(CHALOT_ERR_ARG, "ep_comm_connect: null argument");
  if (c->connected) return set_error(CHALOT_ERR_STATE, "ep_comm_connect: already connected");
  cudaError_t r = cudaSetDevice(c->device);
  for (int p = 0; p < c->world && r == cudaSuccess; ++p) {
    if (p == c->rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, all_handles + (size_t)p * CHALOT_EP_HANDLE_BYTES, sizeof h);
    void* ptr = nullptr;
    r = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (r == cudaSuccess) c->peers.base[p] = static_cast<unsigned char*>(ptr);
  }
  if (r != cudaSuccess) return ep_fail("ep_comm_connect (peer arena)", r);
  c->connected = true;
  return CHALOT_OK;
}

__attribute__((visibility("default"))) void chalot_ep_comm_free(chalot_ep_comm* c) { delete c; }

__attribute__((visibility("default"))) int chalot_moe_layer_ep(chalot_ep_comm* c, const chalot_moe_desc* desc,
                                                               const float* x, size_t n_tok, float* out,
                                                               int32_t* sel_out, float* selw_out, void* stream) {
  if (!c || !desc) return set_error(CHALOT_ERR_ARG, "moe_layer_ep: null argument");
  if (!c->connected) return set_error(CHALOT_ERR_STATE, "moe_layer_ep: connect the group first");
  if ((int)desc->dim != c->dim || (int)desc->hidden_dim != c->hidden || (int)desc->n_experts != c->E ||
      (int)desc->top_k != c->K || (int)(desc->group ? desc->group : 32) != c->group)
    return set_error(CHALOT_ERR_ARG, "moe_layer_ep: descriptor shape differs from the group's");
  if (n_tok > c->max_tokens) return set_error(CHALOT_ERR_ARG, "moe_layer_ep: more tokens than the group reserved");
  if (n_tok > 0 && (!x || !out)) return set_error(CHALOT_ERR_ARG, "moe_layer_ep: null x or out");
  if (!desc->router_w || !desc->router_b || !desc->experts || (reinterpret_cast<uintptr_t>(desc->experts) & 15))
    return set_error(CHALOT_ERR_ARG, "moe_layer_ep: null router or experts (16-byte aligned)");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (int rc = devstat_poll("moe_layer_ep", s)) return rc;
  unsigned* err = devstat_word();
  if (!err) return set_error(CHALOT_ERR_CUDA, "moe_layer_ep: device status word unavailable");
  const unsigned tag = ++c->tag;
  const int El = c->E / c->world, K = c->K, dim = c->dim;
  const int N = (int)(n_tok * K);
  // 1. route and plan (every rank takes every step, n_tok == 0 included)
  MlDims d{(int)n_tok, dim, c->hidden, c->E, K, c->group};
  MlWork w{};
  w.sel = c->sel;
  w.selw = c->selw;
  w.xq = c->xq;
  w.xs = c->xs;
  w.perm = c->order;
  w.inv = c->pos;
  cudaError_t r = cudaSuccess;
  if (n_tok > 0) {
    ml_launch_route(d, x, desc->router_w, desc->router_b, w, s);
    MlDims dp{N, 0, 0, c->E, 1, 32};
    ml_launch_plan(dp, w, c->world, c->offs, s);
  } else {
    r = cudaMemsetAsync(c->offs, 0, (size_t)(c->E + 1) * 4, s);
  }
  // 2. rows to their expert ranks, then counts and the tag
  if (r == cudaSuccess && N > 0)
    k_ep_dispatch<<<(N + 7) / 8, 256, 0, s>>>(c->peers, c->arena, c->rank, c->world, El, K, dim, c->cap_rows,
                                              c->order, c->offs, c->xq, c->xs, N);
  if (r == cudaSuccess) k_ep_signal_rows<<<1, 32, 0, s>>>(c->peers, c->arena, c->rank, c->world, El, c->offs, tag);
  // 3. wait for every source; the local experts on the rows received
  const dim3 gi((unsigned)((c->cap_rows + 255) / 256), (unsigned)c->world);
  if (r == cudaSuccess)
    k_ep_recv_index<<<gi, 256, 0, s>>>(c->arena, c->mine, El, c->cap_rows, tag, c->row_expert, err);
  if (r == cudaSuccess) r = cudaGetLastError();
  if (r == cudaSuccess) {
    const MlDims m = ep_local_dims(c);
    MlWork lw;
    const size_t simt = ml_layout(m, c->ws, &lw);
    MlTcWork t{};
    const bool tc = ml_use_tc(m);
    if (tc) ml_tc_layout(m, simt, c->ws, &t);
    // the received rows in place: no copy into the workspace
    lw.xq = reinterpret_cast<int8_t*>(c->mine + c->arena.rows);
    lw.xs = reinterpret_cast<float*>(c->mine + c->arena.scale);
    lw.sel = c->row_expert;
    MlExperts X{};
    {
      MlDims dx{1, dim, c->hidden, El, 1, c->group};
      X = ml_experts_from_blob(dx, desc->experts);
    }
    r = ml_run_rows(m, X, lw, tc ? &t : nullptr, c->y, s);
  }
  // 4. outputs back to their sources, then the tag
  if (r == cudaSuccess) {
    const size_t rows = (size_t)c->world * c->cap_rows;
    k_ep_return<<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(c->peers, c->arena, c->mine, c->rank, El, dim,
                                                           c->cap_rows, c->y, c->world);
    k_ep_signal_back<<<1, 32, 0, s>>>(c->peers, c->arena, c->rank, c->world, tag);
    k_ep_wait_back<<<1, 32, 0, s>>>(c->arena, c->mine, c->world, tag, err);
    r = cudaGetLastError();
  }
  // 5. combine per token in selection order
  if (r == cudaSuccess && n_tok > 0) {
    MlWork cw{};
    cw.y = reinterpret_cast<float*>(c->mine + c->arena.back);
    cw.inv = c->pos;
    cw.selw = c->selw;
    ml_launch_combine(d, cw, out, s);
    if (sel_out) r = cudaMemcpyAsync(sel_out, c->sel, (size_t)N * 4, cudaMemcpyDeviceToDevice, s);
    if (r == cudaSuccess && selw_out) r = cudaMemcpyAsync(selw_out, c->selw, (size_t)N * 4, cudaMemcpyDeviceToDevice, s);
    if (r == cudaSuccess) r = cudaGetLastError();
  }
  return r == cudaSuccess ? CHALOT_OK : ep_fail("moe_layer_ep", r);
}

}  // extern "C"
