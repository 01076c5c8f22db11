// tmap.h — 2-D TMA tensor maps over row-major device matrices (host side).
#pragma once

#include <cuda.h>
#include <stddef.h>
#include <stdint.h>

namespace chalot {

// Map over a row-major [rows][cols] matrix (cols contiguous, element size
// `esize`), box (box_c columns x box_r rows), optional 128-byte swizzle.
// False when the driver entry point is missing or the driver rejects the
// shape (base not 16-byte aligned, row stride not a multiple of 16 bytes, ...).
bool make_map(CUtensorMap* m, CUtensorMapDataType dt, size_t esize, const void* ptr, uint64_t cols,
              uint64_t rows, uint32_t box_c, uint32_t box_r, bool swizzle);

}  // namespace chalot
