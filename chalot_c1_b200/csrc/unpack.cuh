// unpack.cuh — 32 int4 columns (16 bytes) to 32 int8 in column order, from
// either int4 layout:
//   file layout  (quantization.rs:114-126): byte k holds column 2k in the low
//                nibble and 2k+1 in the high one, value + 8;
//   repacked     (repack_word, the engine's device layout): in word j, byte b
//                holds column 8j+b low and 8j+4+b high, two's complement.
#pragma once

#include <stdint.h>

namespace chalot {

// nibble n (0..15) at each byte -> n - 8, without borrows between bytes
__device__ __forceinline__ uint32_t nib_minus8(uint32_t n) { return (n + 0x78787878u) ^ 0x80808080u; }

__device__ __forceinline__ void unpack32_any(uint4 p, uint4* dst, bool repacked) {
  const uint32_t in[4] = {p.x, p.y, p.z, p.w};
  uint32_t o[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t lo = in[i] & 0x0F0F0F0Fu, hi = (in[i] >> 4) & 0x0F0F0F0Fu;
    if (repacked) {  // two's complement nibbles: flip to value + 8 first
      o[2 * i] = nib_minus8(lo ^ 0x08080808u);
      o[2 * i + 1] = nib_minus8(hi ^ 0x08080808u);
    } else {  // interleave even (low) and odd (high) columns
      o[2 * i] = nib_minus8(__byte_perm(lo, hi, 0x5140));
      o[2 * i + 1] = nib_minus8(__byte_perm(lo, hi, 0x7362));
    }
  }
  dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
  dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
}

}  // namespace chalot
