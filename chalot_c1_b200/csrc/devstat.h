// devstat.h — device-side checks of the asynchronous operators, reported to
// the host without a synchronisation per call.
//
// Kernels of the operator entry points (the tensor-core MoE layer, the paged
// KV store and attention) record what they cannot report by return value —
// a bounded wait that ran out, a page id outside the pool — by OR-ing a bit
// into one sticky word per device. Every such call, after enqueueing its
// kernels, enqueues a 4-byte readback of that word into pinned host memory
// and records an event; the next operator call on that device looks at the
// readback once its event has completed and, if a bit is set, clears the word
// and returns the error. chalot_device_status(stream) synchronises `stream`
// and reports at once. Errors therefore surface at the latest on the next
// operator call after the failing work has finished, with no environment
// variable and no stream synchronisation inside the calls.
#pragma once

#include <cuda_runtime.h>

namespace chalot {

constexpr unsigned kDevErrTimeout = 1u;  // a bounded wait on a bulk copy or the tensor cores gave up
constexpr unsigned kDevErrBadPage = 2u;  // a page id outside [0, n_pages): that page was skipped

// Device address of the current device's sticky word (nullptr on a CUDA error).
unsigned* devstat_word();
// At the start of an operator call: CHALOT_OK, or the status of a device check
// of earlier work whose readback has completed (the word is then cleared on
// stream `s` and the message names `who`).
int devstat_poll(const char* who, cudaStream_t s);
// After an operator enqueued its kernels on `s`: readback of the word.
cudaError_t devstat_post(cudaStream_t s);
// After the caller synchronised the work: CHALOT_OK or the recorded error
// (cleared).
int devstat_take(const char* who);

}  // namespace chalot
