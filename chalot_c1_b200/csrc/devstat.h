// devstat.h — device-side checks of the asynchronous operators, reported to
// the host without a synchronisation or a copy per call.
//
// Kernels of the operator entry points (the tensor-core MoE layer, the paged
// KV store and attention) record what they cannot report by return value —
// a bounded wait that ran out, a page id outside the pool — by storing 1 into
// one of two words per device that live in mapped pinned host memory
// (devstat_word: word 0 a timeout, word 1 a bad page id; plain stores, no
// atomics across the bus). The next operator call on that device reads the
// words, and if one is set, clears them and returns the error;
// chalot_device_status(stream) synchronises `stream` first. Errors therefore
// surface at the latest on the next operator call after the failing work has
// finished, with no environment variable, no stream synchronisation and no
// copy inside the calls.
#pragma once

#include <cuda_runtime.h>

namespace chalot {

// Device address of the current device's two flag words (nullptr on a CUDA
// error): [0] a bounded wait on a bulk copy or the tensor cores gave up,
// [1] a page id outside [0, n_pages) (that page was skipped).
unsigned* devstat_word();
// At the start of an operator call: CHALOT_OK, or the status of a device check
// of earlier work (the flags are then cleared and the message names `who`).
int devstat_poll(const char* who, cudaStream_t s);
// After the caller synchronised the work: the same.
int devstat_take(const char* who);

}  // namespace chalot
