// kv_cache.cu — the reference-shaped paged KV cache (PagedKVCache,
// src/model/memory.rs:100-201) with its pages in device memory.
//
// Semantics kept from the reference:
//   * pages of 256 tokens per layer, found through a per-layer page map;
//   * write(layer, pos, k, v): evict the front of the LRU queue when the cache
//     holds max_pages_per_layer * n_layers pages (checked before every write,
//     even to a page that exists), move (layer, page) to the back of the
//     queue, create the page if absent (zeros, scales 1.0), then quantize the
//     K and V rows (memory.rs:126-171);
//   * quantize_row: scale = max|x| / 127 (1.0 when the row is all zeros),
//     q = (x / scale).clamp(-128, 127) truncated toward zero (NaN -> 0)
//     (memory.rs:58-66); dequantize: q as f32 * scale (memory.rs:69-74);
//   * read(layer, pos): false when the page is absent; reads do not touch the
//     LRU queue.
// The page map, the LRU queue and the free slots live on the host; a batch of
// writes is resolved on the host in order (so evictions inside a batch act as
// sequential writes would) and then applied by one init and one quantize
// kernel. Device layout: slot s = [K|V][256][kv_dim] int8 and [K|V][256] f32.
#include <cuda_runtime.h>

#include <algorithm>
#include <deque>
#include <string>
#include <unordered_map>
#include <vector>

#include "capi_internal.h"
#include "common.cuh"

namespace chalot {
namespace {

constexpr uint32_t kRefPageTokens = 256;

struct RowJob {  // one token row to quantize (or read)
  int slot, off, src;
};

__global__ void k_kv_init(int8_t* data, float* scales, const int* slots, int n, int dim) {
  const int s = slots[blockIdx.x];
  int8_t* d = data + (size_t)s * 2 * kRefPageTokens * dim;
  for (size_t i = threadIdx.x; i < (size_t)2 * kRefPageTokens * dim; i += blockDim.x) d[i] = 0;
  for (int i = threadIdx.x; i < 2 * (int)kRefPageTokens; i += blockDim.x) scales[(size_t)s * 2 * kRefPageTokens + i] = 1.0f;
}

// KVPage::quantize_row for the K row (blockIdx.y == 0) or the V row (1) of job blockIdx.x.
__global__ void k_kv_write(int8_t* data, float* scales, const RowJob* jobs, const float* __restrict__ k,
                           const float* __restrict__ v, int dim) {
  __shared__ float red[33];
  const RowJob j = jobs[blockIdx.x];
  const int kv = blockIdx.y;
  const float* row = (kv ? v : k) + (size_t)j.src * dim;
  float mx = 0.0f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) mx = fmaxf(mx, fabsf(row[i]));  // NaN-ignoring, as f32::max
  mx = warp_max(mx);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, red[w]);
    red[32] = m > 0.0f ? div_rn(m, 127.0f) : 1.0f;
  }
  __syncthreads();
  const float s = red[32];
  const size_t base = (size_t)j.slot * 2 * kRefPageTokens + (size_t)kv * kRefPageTokens + j.off;
  int8_t* out = data + base * dim;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const float q = div_rn(row[i], s);
    out[i] = (q != q) ? 0 : (int8_t)__float2int_rz(fminf(fmaxf(q, -128.0f), 127.0f));
  }
  if (threadIdx.x == 0) scales[base] = s;
}

// KVPage::dequantize_row of the K and V rows of job blockIdx.x into out row j.src.
__global__ void k_kv_read(const int8_t* data, const float* scales, const RowJob* jobs, float* k_out,
                          float* v_out, int dim) {
  const RowJob j = jobs[blockIdx.x];
  for (int kv = 0; kv < 2; ++kv) {
    const size_t base = (size_t)j.slot * 2 * kRefPageTokens + (size_t)kv * kRefPageTokens + j.off;
    const float s = scales[base];
    float* out = (kv ? v_out : k_out) + (size_t)j.src * dim;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) out[i] = __fmul_rn((float)data[base * dim + i], s);
  }
}

}  // namespace
}  // namespace chalot

using namespace chalot;

struct chalot_kv_cache {
  uint32_t dim = 0, n_layers = 0, cap = 0;
  int device = 0;
  int8_t* data = nullptr;
  float* scales = nullptr;
  std::vector<std::unordered_map<uint32_t, int>> pages;  // per layer: page id -> slot
  std::deque<std::pair<uint32_t, uint32_t>> lru;         // (layer, page), front = least recent
  std::vector<int> free_slots;
  std::vector<uint32_t> gen;  // per slot: bumped when the slot gets a new page
  cudaStream_t stream = nullptr;
  RowJob* d_jobs = nullptr;
  int* d_slots = nullptr;
  float* d_rows = nullptr;  // staging for host rows
  size_t jobs_cap = 0, rows_cap = 0, slots_cap = 0;

  size_t active() const {
    size_t t = 0;
    for (auto& m : pages) t += m.size();
    return t;
  }
  // PagedKVCache::get_or_create_page (memory.rs:148-160): returns the slot; *created set when new.
  int get_or_create(uint32_t layer, uint32_t page, bool* created) {
    if (active() >= cap && !lru.empty()) {  // evict_if_full
      auto lp = lru.front();
      lru.pop_front();
      auto it = pages[lp.first].find(lp.second);
      if (it != pages[lp.first].end()) {
        free_slots.push_back(it->second);
        pages[lp.first].erase(it);
      }
    }
    for (auto it = lru.begin(); it != lru.end();)
      it = (it->first == layer && it->second == page) ? lru.erase(it) : it + 1;
    lru.push_back({layer, page});
    auto f = pages[layer].find(page);
    *created = false;
    if (f != pages[layer].end()) return f->second;
    const int s = free_slots.back();
    free_slots.pop_back();
    ++gen[s];
    pages[layer][page] = s;
    *created = true;
    return s;
  }
};

namespace {

int kv_fail(const char* what, cudaError_t r) {
  return set_error(CHALOT_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(r));
}

template <typename T>
cudaError_t ensure(T** p, size_t* cap, size_t n) {
  if (n <= *cap) return cudaSuccess;
  if (*p) cudaFree(*p);
  *p = nullptr;
  const size_t c = std::max<size_t>(n, 64);
  cudaError_t r = cudaMalloc(reinterpret_cast<void**>(p), c * sizeof(T));
  *cap = r == cudaSuccess ? c : 0;
  return r;
}

// Resolves n writes in order on the host and applies them on the device.
// k/v are device rows [n][dim].
int apply_writes(chalot_kv_cache* c, uint32_t layer, const uint32_t* pos, size_t n, const float* k, const float* v,
                 cudaStream_t s) {
  std::vector<RowJob> jobs;
  std::vector<uint32_t> job_gen;
  std::vector<int> created;
  jobs.reserve(n);
  for (size_t i = 0; i < n; ++i) {
    bool made = false;
    const int slot = c->get_or_create(layer, pos[i] / kRefPageTokens, &made);
    if (made) created.push_back(slot);
    jobs.push_back({slot, (int)(pos[i] % kRefPageTokens), (int)i});
    job_gen.push_back(c->gen[slot]);
  }
  // keep what sequential writes would leave: rows of pages evicted later in the
  // batch are gone, and of several writes to one row the last one stands
  std::vector<RowJob> keep;
  std::unordered_map<long long, size_t> last;
  for (size_t i = 0; i < jobs.size(); ++i) {
    if (job_gen[i] != c->gen[jobs[i].slot]) continue;
    const long long key = (long long)jobs[i].slot * kRefPageTokens + jobs[i].off;
    auto it = last.find(key);
    if (it != last.end()) keep[it->second] = jobs[i];
    else {
      last[key] = keep.size();
      keep.push_back(jobs[i]);
    }
  }
  std::vector<int> init;  // pages created in this batch and still held: start from zeros
  for (int sl : created)
    if (std::find(init.begin(), init.end(), sl) == init.end()) {
      bool held = false;
      for (auto& m : c->pages)
        for (auto& kvp : m) held |= kvp.second == sl;
      if (held) init.push_back(sl);
    }
  cudaError_t r = cudaSuccess;
  if (!init.empty()) {
    r = ensure(&c->d_slots, &c->slots_cap, init.size());
    if (r == cudaSuccess) r = cudaMemcpyAsync(c->d_slots, init.data(), init.size() * sizeof(int), cudaMemcpyHostToDevice, s);
    if (r == cudaSuccess) {
      k_kv_init<<<(unsigned)init.size(), 256, 0, s>>>(c->data, c->scales, c->d_slots, (int)init.size(), (int)c->dim);
      r = cudaGetLastError();
    }
    if (r == cudaSuccess) r = cudaStreamSynchronize(s);  // `init` is a host vector
  }
  if (r == cudaSuccess && !keep.empty()) {
    r = ensure(&c->d_jobs, &c->jobs_cap, keep.size());
    if (r == cudaSuccess)
      r = cudaMemcpyAsync(c->d_jobs, keep.data(), keep.size() * sizeof(RowJob), cudaMemcpyHostToDevice, s);
    if (r == cudaSuccess) {
      k_kv_write<<<dim3((unsigned)keep.size(), 2), 256, 0, s>>>(c->data, c->scales, c->d_jobs, k, v, (int)c->dim);
      r = cudaGetLastError();
    }
    if (r == cudaSuccess) r = cudaStreamSynchronize(s);  // `keep` is a host vector
  }
  return r == cudaSuccess ? CHALOT_OK : kv_fail("kv_write", r);
}

}  // namespace

extern "C" {

__attribute__((visibility("default"))) int chalot_kv_create(uint32_t kv_dim, uint32_t n_layers,
                                                            uint32_t max_pages_per_layer, int device,
                                                            chalot_kv_cache** out) {
  if (!out) return set_error(CHALOT_ERR_ARG, "kv_create: null out");
  *out = nullptr;
  if (kv_dim == 0 || n_layers == 0) return set_error(CHALOT_ERR_ARG, "kv_create: kv_dim and n_layers must be positive");
  auto* c = new chalot_kv_cache;
  c->dim = kv_dim;
  c->n_layers = n_layers;
  c->cap = (max_pages_per_layer ? max_pages_per_layer : 16) * n_layers;
  c->device = device;
  c->pages.resize(n_layers);
  c->gen.assign(c->cap, 0);
  for (int s = (int)c->cap - 1; s >= 0; --s) c->free_slots.push_back(s);
  cudaError_t r = cudaSetDevice(device);
  if (r == cudaSuccess) r = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
  if (r == cudaSuccess) r = cudaMalloc(&c->data, (size_t)c->cap * 2 * kRefPageTokens * kv_dim);
  if (r == cudaSuccess) r = cudaMalloc(&c->scales, (size_t)c->cap * 2 * kRefPageTokens * sizeof(float));
  if (r != cudaSuccess) {
    chalot_kv_free(c);
    return set_error(r == cudaErrorMemoryAllocation ? CHALOT_ERR_OOM : CHALOT_ERR_CUDA,
                     std::string("kv_create: ") + cudaGetErrorString(r));
  }
  *out = c;
  return CHALOT_OK;
}

__attribute__((visibility("default"))) void chalot_kv_free(chalot_kv_cache* c) {
  if (!c) return;
  cudaSetDevice(c->device);
  if (c->stream) cudaStreamSynchronize(c->stream);
  if (c->data) cudaFree(c->data);
  if (c->scales) cudaFree(c->scales);
  if (c->d_jobs) cudaFree(c->d_jobs);
  if (c->d_slots) cudaFree(c->d_slots);
  if (c->d_rows) cudaFree(c->d_rows);
  if (c->stream) cudaStreamDestroy(c->stream);
  delete c;
}

__attribute__((visibility("default"))) int chalot_kv_write(chalot_kv_cache* c, uint32_t layer, uint32_t pos,
                                                           const float* k, const float* v) {
  if (!c || !k || !v) return set_error(CHALOT_ERR_ARG, "kv_write: null pointer");
  if (layer >= c->n_layers) return set_error(CHALOT_ERR_ARG, "kv_write: layer out of range");
  cudaError_t r = cudaSetDevice(c->device);
  if (r == cudaSuccess) r = ensure(&c->d_rows, &c->rows_cap, (size_t)2 * c->dim);
  if (r == cudaSuccess) r = cudaMemcpyAsync(c->d_rows, k, c->dim * 4, cudaMemcpyHostToDevice, c->stream);
  if (r == cudaSuccess) r = cudaMemcpyAsync(c->d_rows + c->dim, v, c->dim * 4, cudaMemcpyHostToDevice, c->stream);
  if (r != cudaSuccess) return kv_fail("kv_write", r);
  return apply_writes(c, layer, &pos, 1, c->d_rows, c->d_rows + c->dim, c->stream);
}

__attribute__((visibility("default"))) int chalot_kv_write_batch(chalot_kv_cache* c, uint32_t layer,
                                                                 const uint32_t* pos, size_t n, const float* k,
                                                                 const float* v, void* stream) {
  if (!c || (n && (!pos || !k || !v))) return set_error(CHALOT_ERR_ARG, "kv_write_batch: null pointer");
  if (layer >= c->n_layers) return set_error(CHALOT_ERR_ARG, "kv_write_batch: layer out of range");
  if (n == 0) return CHALOT_OK;
  cudaError_t r = cudaSetDevice(c->device);
  if (r != cudaSuccess) return kv_fail("kv_write_batch", r);
  return apply_writes(c, layer, pos, n, k, v, stream ? static_cast<cudaStream_t>(stream) : c->stream);
}

__attribute__((visibility("default"))) int chalot_kv_gather(chalot_kv_cache* c, uint32_t layer, const uint32_t* pos,
                                                            size_t n, float* k_out, float* v_out, uint8_t* found,
                                                            void* stream) {
  if (!c || (n && (!pos || !k_out || !v_out || !found))) return set_error(CHALOT_ERR_ARG, "kv_gather: null pointer");
  if (layer >= c->n_layers) return set_error(CHALOT_ERR_ARG, "kv_gather: layer out of range");
  std::vector<RowJob> jobs;
  for (size_t i = 0; i < n; ++i) {
    auto f = c->pages[layer].find(pos[i] / kRefPageTokens);
    found[i] = f != c->pages[layer].end();
    if (found[i]) jobs.push_back({f->second, (int)(pos[i] % kRefPageTokens), (int)i});
  }
  if (jobs.empty()) return CHALOT_OK;
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
  cudaError_t r = cudaSetDevice(c->device);
  if (r == cudaSuccess) r = ensure(&c->d_jobs, &c->jobs_cap, jobs.size());
  if (r == cudaSuccess) r = cudaMemcpyAsync(c->d_jobs, jobs.data(), jobs.size() * sizeof(RowJob), cudaMemcpyHostToDevice, s);
  if (r == cudaSuccess) {
    k_kv_read<<<(unsigned)jobs.size(), 256, 0, s>>>(c->data, c->scales, c->d_jobs, k_out, v_out, (int)c->dim);
    r = cudaGetLastError();
  }
  if (r == cudaSuccess) r = cudaStreamSynchronize(s);  // `jobs` is a host vector
  return r == cudaSuccess ? CHALOT_OK : kv_fail("kv_gather", r);
}

__attribute__((visibility("default"))) int chalot_kv_read(chalot_kv_cache* c, uint32_t layer, uint32_t pos,
                                                          float* k_out, float* v_out, int* found) {
  if (!c || !k_out || !v_out || !found) return set_error(CHALOT_ERR_ARG, "kv_read: null pointer");
  if (layer >= c->n_layers) return set_error(CHALOT_ERR_ARG, "kv_read: layer out of range");
  uint8_t f = 0;
  cudaError_t r = cudaSetDevice(c->device);
  if (r == cudaSuccess) r = ensure(&c->d_rows, &c->rows_cap, (size_t)2 * c->dim);
  if (r != cudaSuccess) return kv_fail("kv_read", r);
  int rc = chalot_kv_gather(c, layer, &pos, 1, c->d_rows, c->d_rows + c->dim, &f, c->stream);
  if (rc != CHALOT_OK) return rc;
  *found = f;
  if (!f) return CHALOT_OK;  // outputs untouched, as PagedKVCache::read leaves them
  r = cudaMemcpyAsync(k_out, c->d_rows, c->dim * 4, cudaMemcpyDeviceToHost, c->stream);
  if (r == cudaSuccess) r = cudaMemcpyAsync(v_out, c->d_rows + c->dim, c->dim * 4, cudaMemcpyDeviceToHost, c->stream);
  if (r == cudaSuccess) r = cudaStreamSynchronize(c->stream);
  return r == cudaSuccess ? CHALOT_OK : kv_fail("kv_read", r);
}

__attribute__((visibility("default"))) int chalot_kv_clear(chalot_kv_cache* c) {
  if (!c) return set_error(CHALOT_ERR_ARG, "kv_clear: null cache");
  for (auto& m : c->pages) {
    for (auto& kvp : m) c->free_slots.push_back(kvp.second);
    m.clear();
  }
  c->lru.clear();
  return CHALOT_OK;
}

__attribute__((visibility("default"))) size_t chalot_kv_active_pages(const chalot_kv_cache* c) {
  return c ? c->active() : 0;
}

__attribute__((visibility("default"))) float chalot_kv_memory_mb(const chalot_kv_cache* c) {
  if (!c) return 0.0f;
  const size_t bytes_per_page = (size_t)kRefPageTokens * c->dim * 2 + (size_t)kRefPageTokens * 8;
  return (float)(c->active() * bytes_per_page) / 1e6f;  // memory.rs:129-133
}

}  // extern "C"
