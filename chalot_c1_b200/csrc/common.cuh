// common.cuh — device helpers shared by the sm_100a kernels.
//
// Every float operation on a parity-critical path is written with an explicit
// round-to-nearest intrinsic (__fmul_rn, __fadd_rn, div_rn, __fsqrt_rn), so
// the compiler can neither contract it into an FMA nor reorder it; the library
// is also compiled with --fmad=false. The orders mirror the reference's AVX2
// code (citations at each helper).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "libm_f32.h"

namespace chalot {

using libm::div_rn;  // exact division, fast path (libm_f32.h)

#define CHALOT_DEV __device__ __forceinline__

// Per-forward state read by every kernel of a decode step, so one captured
// graph serves every position.
struct StepState {
  uint32_t pos;        // position of the token being processed
  uint32_t token;      // token id being processed
  uint32_t n_prefill;  // prompt tokens fed before decoding starts
  uint32_t step;       // forwards run so far in this generate call
  unsigned long long argmax_key;  // (ordered logit << 32) | index of the max
};

// ---- float helpers --------------------------------------------------------

// One lane of fast_exp_avx2 (src/tensor/normalization.rs:165-200, identical to
// src/tensor/activations.rs:92-127): n = floor(x/ln2 as x*inv_ln2),
// r = x - n*ln2, Horner c5..c0 without FMA, 2^n assembled as (n+127)<<23.
CHALOT_DEV float fast_exp(float x) {
  const float ln2 = 0.693147180559945309f;
  const float inv_ln2 = 1.442695040888963407f;
  float n = floorf(__fmul_rn(x, inv_ln2));
  float r = __fsub_rn(x, __fmul_rn(n, ln2));
  float p = 0.008333333333f;
  p = __fadd_rn(__fmul_rn(p, r), 0.041666666666f);
  p = __fadd_rn(__fmul_rn(p, r), 0.166666666666f);
  p = __fadd_rn(__fmul_rn(p, r), 0.5f);
  p = __fadd_rn(__fmul_rn(p, r), 1.0f);
  p = __fadd_rn(__fmul_rn(p, r), 1.0f);
  // cvtps_epi32 of an integral value; out-of-range gives 0x80000000.
  int32_t ni = (n >= -2147483648.0f && n < 2147483648.0f) ? (int32_t)n : INT32_MIN;
  uint32_t e = ((uint32_t)ni + 127u) << 23;
  return __fmul_rn(p, __uint_as_float(e));
}

// Horizontal sum of 8 lanes: (lane j + lane j+4), movehl, shuffle
// (e.g. src/tensor/normalization.rs:45-50).
CHALOT_DEV float hsum8(const float s[8]) {
  float t0 = __fadd_rn(s[0], s[4]), t1 = __fadd_rn(s[1], s[5]);
  float t2 = __fadd_rn(s[2], s[6]), t3 = __fadd_rn(s[3], s[7]);
  return __fadd_rn(__fadd_rn(t0, t2), __fadd_rn(t1, t3));
}

// libm expf as the reference gets it from glibc (libm::exp_f32, the same
// method and rounding; libm_f32.h). Out of line: it runs only for the few tail
// elements of a softmax or SwiGLU, and inlined next to fast_exp under a
// select, its double arithmetic and table lookup would run for every element.
static __device__ __noinline__ float expf_cr(float x) { return libm::exp_f32(x); }

// SwiGLU of one element at index i of a vector of length n: the first
// floor(n/8)*8 elements use fast_exp, the tail uses libm exp
// (src/tensor/activations.rs:59-87).
CHALOT_DEV float swiglu_elem(float g, float u, size_t i, size_t n) {
  float e;
  if (i < (n & ~size_t(7)))
    e = fast_exp(__fsub_rn(0.0f, g));
  else
    e = expf_cr(-g);
  float silu = div_rn(g, __fadd_rn(1.0f, e));
  return __fmul_rn(silu, u);
}

// Scale and reciprocal of quantize_f32_to_i8 from the absolute maximum
// (src/tensor/quantization.rs:77-80).
CHALOT_DEV void quant_scale(float amax, float* scale, float* inv) {
  amax = fmaxf(amax, 1e-12f);
  float s = div_rn(amax, 127.0f);
  *scale = s;
  *inv = div_rn(1.0f, s);
}

// AVX2 quantization of one element: clamp(x*inv, ±127) then cvtps_epi32
// (round to nearest even) (src/tensor/quantization.rs:86-99).
CHALOT_DEV int8_t quant_elem(float x, float inv) {
  float s = __fmul_rn(x, inv);
  s = (s < 127.0f) ? s : 127.0f;
  s = (s > -127.0f) ? s : -127.0f;
  return (int8_t)__float2int_rn(s);
}

// Scalar tail of the same quantizer: .round() (half away from zero).
CHALOT_DEV int8_t quant_elem_tail(float x, float inv) {
  float s = roundf(__fmul_rn(x, inv));
  s = fminf(fmaxf(s, -127.0f), 127.0f);
  return (int8_t)(int)s;
}

CHALOT_DEV int8_t quant_any(float x, float inv, size_t i, size_t n) {
  return (i < (n & ~size_t(7))) ? quant_elem(x, inv) : quant_elem_tail(x, inv);
}

// Total order key of a logit for the argmax (larger key = larger value; equal
// values compare equal, with -0 folded into +0).
CHALOT_DEV uint32_t ordered_key(float v) {
  if (v == 0.0f) v = 0.0f;
  uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// ---- reductions -------------------------------------------------------------

CHALOT_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

CHALOT_DEV int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide max of non-negative floats; `red` holds >= 32 floats.
CHALOT_DEV float block_max(float v, float* red) {
  v = warp_max(v);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float r = (threadIdx.x < (unsigned)nw) ? red[threadIdx.x] : -INFINITY;
  if (wid == 0) r = warp_max(r);
  if (threadIdx.x == 0) red[0] = r;
  __syncthreads();
  r = red[0];
  __syncthreads();
  return r;
}

// ---- int8/int4 dot helpers -----------------------------------------------------

// 16 int8 weights (one uint4) times 16 int8 activations.
CHALOT_DEV int dot16_i8(uint4 w, uint4 x, int acc) {
  acc = __dp4a((int)w.x, (int)x.x, acc);
  acc = __dp4a((int)w.y, (int)x.y, acc);
  acc = __dp4a((int)w.z, (int)x.z, acc);
  acc = __dp4a((int)w.w, (int)x.w, acc);
  return acc;
}

// 32 int4 weights packed in one uint4 (low nibble = even column, stored
// value = weight + 8) against 32 activations stored as [8 even, 8 odd] per
// 8-column block: xe/xo pairs, i.e. x_perm[4*j .. 4*j+3] = even columns of
// word j and x_perm[16 + 4*j ..] = odd columns. Returns sum(nibble * x)
// (the caller subtracts 8 * sum(x) for the group). Nibbles 0..15 read the
// same as signed bytes, so the signed dp4a form is exact.
CHALOT_DEV int dot32_u4(uint4 w, const uint4& xe, const uint4& xo, int acc) {
  const uint32_t m = 0x0F0F0F0Fu;
  acc = __dp4a((int)(w.x & m), (int)xe.x, acc);
  acc = __dp4a((int)((w.x >> 4) & m), (int)xo.x, acc);
  acc = __dp4a((int)(w.y & m), (int)xe.y, acc);
  acc = __dp4a((int)((w.y >> 4) & m), (int)xo.y, acc);
  acc = __dp4a((int)(w.z & m), (int)xe.z, acc);
  acc = __dp4a((int)((w.z >> 4) & m), (int)xo.z, acc);
  acc = __dp4a((int)(w.w & m), (int)xe.w, acc);
  acc = __dp4a((int)((w.w >> 4) & m), (int)xo.w, acc);
  return acc;
}

// Repacked int4 layout used by the engine (applied once at load): in every
// 32-bit word (8 columns 8j..8j+7) byte b holds column 8j+b in its low nibble
// and column 8j+4+b in its high nibble, each as a 4-bit two's complement
// value. Then (w << 4) & 0xF0F0F0F0 is 16*w for columns 8j..8j+3 and
// w & 0xF0F0F0F0 is 16*w for columns 8j+4..8j+7, as signed bytes, so dp4a
// against the activations in natural order gives 16 * the exact int32 dot.
CHALOT_DEV uint32_t repack_word(uint32_t w) {
  const uint32_t lo0 = w & 0xF, hi0 = (w >> 4) & 0xF, lo1 = (w >> 8) & 0xF, hi1 = (w >> 12) & 0xF;
  const uint32_t lo2 = (w >> 16) & 0xF, hi2 = (w >> 20) & 0xF, lo3 = (w >> 24) & 0xF, hi3 = (w >> 28) & 0xF;
  // columns 0..7 of the word in the file: lo0 hi0 lo1 hi1 lo2 hi2 lo3 hi3 (value + 8)
  const uint32_t b0 = lo0 | (lo2 << 4), b1 = hi0 | (hi2 << 4), b2 = lo1 | (lo3 << 4), b3 = hi1 | (hi3 << 4);
  return (b0 | (b1 << 8) | (b2 << 16) | (b3 << 24)) ^ 0x88888888u;  // value + 8 -> two's complement
}

// Exact int32 dot of 32 repacked int4 weights (one uint4) with 32 int8
// activations in natural order (x0: columns 0..15, x1: columns 16..31).
CHALOT_DEV int dot32_rp(uint4 w, const uint4& x0, const uint4& x1) {
  const uint32_t m = 0xF0F0F0F0u;
  int acc = 0;
  acc = __dp4a((int)((w.x << 4) & m), (int)x0.x, acc);
  acc = __dp4a((int)(w.x & m), (int)x0.y, acc);
  acc = __dp4a((int)((w.y << 4) & m), (int)x0.z, acc);
  acc = __dp4a((int)(w.y & m), (int)x0.w, acc);
  acc = __dp4a((int)((w.z << 4) & m), (int)x1.x, acc);
  acc = __dp4a((int)(w.z & m), (int)x1.y, acc);
  acc = __dp4a((int)((w.w << 4) & m), (int)x1.z, acc);
  acc = __dp4a((int)(w.w & m), (int)x1.w, acc);
  return acc >> 4;  // every product is 16 * w * x: the division is exact
}

// One 16-byte shared-memory load as a single vector instruction. Passing
// *(const uint4*)p straight into a helper that reads the four words one by
// one lets the compiler emit four 32-bit loads instead, which at a 32-byte
// lane stride is an 8-way bank conflict.
CHALOT_DEV uint4 lds16(const void* p) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"((uint32_t)__cvta_generic_to_shared(p)));
  return v;
}
CHALOT_DEV float4 lds16f(const float* p) {
  const uint4 v = lds16(p);
  return make_float4(__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z), __uint_as_float(v.w));
}

// Streaming 16-byte load of a weight (read once: evict-first). A compiler
// builtin, so it stays ordered with the griddepcontrol barriers.
CHALOT_DEV uint4 ldg_stream(const void* p) { return __ldcs(reinterpret_cast<const uint4*>(p)); }

}  // namespace chalot
