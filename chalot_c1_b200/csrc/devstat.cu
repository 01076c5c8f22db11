// devstat.cu — the device-check flags of the operator entry points
// (devstat.h): two words per device in mapped pinned host memory, written by
// kernels with plain stores (no atomics across the bus) and read by the host
// without a copy or an event.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "capi_internal.h"
#include "devstat.h"

namespace chalot {
namespace {

constexpr int kMaxDevices = 64;

struct Flags {
  unsigned* host = nullptr;  // [2] mapped pinned: timeout, bad page
  unsigned* dev = nullptr;   // the same words as the device addresses them
};

std::mutex g_mu;
Flags g_flags[kMaxDevices];

int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -1;
  return dev;
}

// The current device's flags, allocated on first use.
Flags* flags() {
  const int dev = current_device();
  if (dev < 0) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  Flags& f = g_flags[dev];
  if (!f.host) {
    void* h = nullptr;
    if (cudaHostAlloc(&h, 2 * sizeof(unsigned), cudaHostAllocMapped) != cudaSuccess) return nullptr;
    void* d = nullptr;
    if (cudaHostGetDevicePointer(&d, h, 0) != cudaSuccess) {
      cudaFreeHost(h);
      return nullptr;
    }
    f.host = static_cast<unsigned*>(h);
    f.host[0] = f.host[1] = 0u;
    f.dev = static_cast<unsigned*>(d);
  }
  return &f;
}

}  // namespace

unsigned* devstat_word() {
  Flags* f = flags();
  return f ? f->dev : nullptr;
}

int devstat_poll(const char* who, cudaStream_t) {
  const int dev = current_device();
  if (dev < 0) return CHALOT_OK;
  unsigned* h = g_flags[dev].host;
  if (!h) return CHALOT_OK;
  volatile unsigned* v = h;
  const unsigned timeout = v[0], bad_page = v[1];
  if (!timeout && !bad_page) return CHALOT_OK;
  v[0] = 0u;
  v[1] = 0u;
  const std::string w = who ? who : "device";
  if (timeout)
    return set_error(CHALOT_ERR_TIMEOUT, w + ": a bounded device wait (bulk copy or tensor-core pipeline) "
                                             "gave up in earlier work; its output is invalid");
  return set_error(CHALOT_ERR_ARG, w + ": a page id outside [0, n_pages) was passed to earlier work; "
                                       "that page was skipped and the output is invalid");
}

int devstat_take(const char* who) { return devstat_poll(who, nullptr); }

}  // namespace chalot

using namespace chalot;

extern "C" {

__attribute__((visibility("default"))) int chalot_device_status(void* stream) {
  cudaError_t r = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (r != cudaSuccess) return set_error(CHALOT_ERR_CUDA, std::string("device_status: ") + cudaGetErrorString(r));
  return devstat_take("device_status");
}

}  // extern "C"
