// Host-side construction of TMA tensor maps (CUtensorMap) for row-major 2-D
// f16/bf16 matrices. cuTensorMapEncodeTiled is a driver API entry point; it is
// fetched once through cudaGetDriverEntryPoint so the library links only
// against the CUDA runtime.
#pragma once

#include <cstdint>

#include <cuda.h>

namespace zcb {

enum class TmaSwizzle { None, B64, B128 };

// Encodes a map for a row-major matrix of `rows` x `cols` elements with a
// leading dimension of `ld` elements, copied in boxes of box_rows x box_cols.
// Returns false (map untouched) if the driver rejects the parameters.
bool make_tma_2d(CUtensorMap* map, const void* base, bool bf16, int64_t rows, int64_t cols,
                 int64_t ld, int box_rows, int box_cols, TmaSwizzle swizzle);

// True when a matrix can be described by a TMA map: 16-byte aligned base and
// a leading dimension whose byte size is a multiple of 16.
inline bool tma_compatible(const void* base, int64_t ld_elems) {
  return (reinterpret_cast<uintptr_t>(base) & 15u) == 0 && ((ld_elems * 2) & 15) == 0 &&
         ld_elems > 0 && ld_elems * 2 < (int64_t(1) << 40);
}

}  // namespace zcb
