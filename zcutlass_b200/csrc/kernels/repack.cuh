// Copy of a 2-byte-element matrix between arbitrary layouts, for the generic
// path: operands TMA cannot describe (leading dimensions that are not a
// multiple of 8 elements, pointers aligned to 2 bytes only) are packed into
// 16-byte-aligned rows so the tcgen05 kernels can run on them, and a packed
// result is copied out to a D with such a layout.
//
//   dst[r][c] = c < cols ? src[r][c] : 0      for r < rows, c < cols_out
//
// One thread writes 8 consecutive elements of a row: a 16-byte load when the
// source chunk is 16-byte aligned and inside the row, else 2-byte loads (the
// threads of a warp still cover consecutive bytes, so loads coalesce); a
// 16-byte store when the destination chunk is aligned and whole, else 2-byte
// stores. Values are copied bit for bit (no rounding).
#pragma once

#include <cstdint>

namespace zcb {
namespace repack {

constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads) copy2d_u16_kernel(uint16_t* dst, int64_t ld_dst, const uint16_t* src,
                                                             int64_t ld_src, int64_t rows, int64_t cols,
                                                             int64_t cols_out) {
  const int64_t chunks = (cols_out + 7) / 8;
  const int64_t total = rows * chunks;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int64_t r = i / chunks;
    const int64_t c0 = (i - r * chunks) * 8;
    const uint16_t* s = src + r * ld_src + c0;
    uint16_t* d = dst + r * ld_dst + c0;
    uint16_t v[8];
    if (c0 + 8 <= cols && (reinterpret_cast<uintptr_t>(s) & 15u) == 0) {
      const uint4 u = *reinterpret_cast<const uint4*>(s);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[2 * j] = static_cast<uint16_t>(w[j] & 0xffffu);
        v[2 * j + 1] = static_cast<uint16_t>(w[j] >> 16);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = c0 + j < cols ? s[j] : uint16_t(0);
    }
    if (c0 + 8 <= cols_out && (reinterpret_cast<uintptr_t>(d) & 15u) == 0) {
      uint4 u;
      u.x = uint32_t(v[0]) | (uint32_t(v[1]) << 16);
      u.y = uint32_t(v[2]) | (uint32_t(v[3]) << 16);
      u.z = uint32_t(v[4]) | (uint32_t(v[5]) << 16);
      u.w = uint32_t(v[6]) | (uint32_t(v[7]) << 16);
      *reinterpret_cast<uint4*>(d) = u;
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (c0 + j < cols_out) d[j] = v[j];
    }
  }
}

}  // namespace repack
}  // namespace zcb
