// devstat.cu — the sticky device-check word of the operator entry points and
// its asynchronous readback (devstat.h).
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "capi_internal.h"
#include "devstat.h"

namespace chalot {
namespace {

__device__ unsigned g_dev_status;

constexpr int kMaxDevices = 64;

struct Readback {
  unsigned* host = nullptr;   // pinned: the last readback of the word
  cudaEvent_t ev = nullptr;   // recorded after that readback
  bool posted = false;
};

std::mutex g_mu;
Readback g_rb[kMaxDevices];

int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -1;
  return dev;
}

int report(unsigned bits, const char* who) {
  const std::string w = who ? who : "device";
  if (bits & kDevErrTimeout)
    return set_error(CHALOT_ERR_TIMEOUT, w + ": a bounded device wait (bulk copy or tensor-core pipeline) "
                                             "gave up in earlier work; its output is invalid");
  return set_error(CHALOT_ERR_ARG, w + ": a page id outside [0, n_pages) was passed to earlier work; "
                                       "that page was skipped and the output is invalid");
}

}  // namespace

unsigned* devstat_word() {
  // Looked up on every call: the address belongs to the current device's
  // module instance.
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_dev_status) != cudaSuccess) return nullptr;
  return static_cast<unsigned*>(p);
}

int devstat_poll(const char* who, cudaStream_t s) {
  const int dev = current_device();
  if (dev < 0) return CHALOT_OK;
  std::lock_guard<std::mutex> lk(g_mu);
  Readback& rb = g_rb[dev];
  if (!rb.posted || cudaEventQuery(rb.ev) != cudaSuccess) return CHALOT_OK;
  const unsigned bits = *reinterpret_cast<volatile unsigned*>(rb.host);
  if (!bits) return CHALOT_OK;
  *reinterpret_cast<volatile unsigned*>(rb.host) = 0u;
  rb.posted = false;
  if (unsigned* w = devstat_word()) cudaMemsetAsync(w, 0, sizeof(unsigned), s);
  return report(bits, who);
}

cudaError_t devstat_post(cudaStream_t s) {
  const int dev = current_device();
  if (dev < 0) return cudaErrorInvalidDevice;
  unsigned* w = devstat_word();
  if (!w) return cudaGetLastError();
  std::lock_guard<std::mutex> lk(g_mu);
  Readback& rb = g_rb[dev];
  cudaError_t r = cudaSuccess;
  if (!rb.host) {
    void* h = nullptr;
    r = cudaHostAlloc(&h, sizeof(unsigned), cudaHostAllocDefault);
    if (r != cudaSuccess) return r;
    rb.host = static_cast<unsigned*>(h);
    *rb.host = 0u;
    r = cudaEventCreateWithFlags(&rb.ev, cudaEventDisableTiming);
    if (r != cudaSuccess) return r;
  }
  r = cudaMemcpyAsync(rb.host, w, sizeof(unsigned), cudaMemcpyDeviceToHost, s);
  if (r == cudaSuccess) r = cudaEventRecord(rb.ev, s);
  if (r == cudaSuccess) rb.posted = true;
  return r;
}

int devstat_take(const char* who) {
  unsigned* w = devstat_word();
  if (!w) return CHALOT_OK;
  unsigned bits = 0;
  if (cudaMemcpy(&bits, w, sizeof bits, cudaMemcpyDeviceToHost) != cudaSuccess || !bits) return CHALOT_OK;
  cudaMemset(w, 0, sizeof(unsigned));
  const int dev = current_device();
  if (dev >= 0) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_rb[dev].host) *reinterpret_cast<volatile unsigned*>(g_rb[dev].host) = 0u;
    g_rb[dev].posted = false;
  }
  return report(bits, who);
}

}  // namespace chalot

using namespace chalot;

extern "C" {

__attribute__((visibility("default"))) int chalot_device_status(void* stream) {
  cudaError_t r = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (r != cudaSuccess) return set_error(CHALOT_ERR_CUDA, std::string("device_status: ") + cudaGetErrorString(r));
  return devstat_take("device_status");
}

}  // extern "C"
