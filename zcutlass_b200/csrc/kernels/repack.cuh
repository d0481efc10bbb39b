// Copy of a 2-byte-element matrix between arbitrary layouts, for the generic
// path: operands TMA cannot describe (leading dimensions that are not a
// multiple of 8 elements, pointers aligned to 2 bytes only) are packed into
// 16-byte-aligned rows so the tcgen05 kernels can run on them, and a packed
// result is copied out to a D with such a layout.
//
//   dst[r][c] = c < cols ? src[r][c] : 0      for r < rows, c < cols_out
//
// One thread writes 8 consecutive elements of a row. It reads them with
// 16-byte loads of the aligned words that hold them -- one word when the
// chunk starts on a 16-byte boundary, else two, joined with funnel shifts --
// and loads only words that hold at least one element of the row inside
// `cols` (such a word lies in the same 16-byte-aligned block as that element,
// so inside the caller's allocation). Stores are 16 bytes wide when the
// destination chunk is aligned and whole, 4 bytes when it is 4-byte aligned,
// else 2. Values are copied bit for bit (no rounding).
#pragma once

#include <cstdint>

namespace zcb {
namespace repack {

constexpr int kThreads = 256;

// Bytes [sh, sh + 16) of the 32 bytes w0 w1 (sh even, 0..14), as 4 words.
__device__ __forceinline__ uint4 extract16(const uint4& w0, const uint4& w1, uint32_t sh) {
  const uint32_t W[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
  const uint32_t q = sh >> 2, half = (sh & 2u) * 8u;  // word offset, 0 or 16 bits
  uint32_t o[5];
#pragma unroll
  for (int i = 0; i < 5; ++i) {
    // W[q + i] without a runtime-indexed array (q is 0..3)
    const uint32_t a = q == 0 ? W[i] : q == 1 ? W[i + 1] : q == 2 ? W[i + 2] : W[i + 3];
    o[i] = a;
  }
  uint4 r;
  r.x = __funnelshift_r(o[0], o[1], half);
  r.y = __funnelshift_r(o[1], o[2], half);
  r.z = __funnelshift_r(o[2], o[3], half);
  r.w = __funnelshift_r(o[3], o[4], half);
  return r;
}

__global__ void __launch_bounds__(kThreads) copy2d_u16_kernel(uint16_t* dst, int64_t ld_dst, const uint16_t* src,
                                                             int64_t ld_src, int64_t rows, int64_t cols,
                                                             int64_t cols_out) {
  const int64_t chunks = (cols_out + 7) / 8;
  const int64_t total = rows * chunks;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int64_t r = i / chunks;
    const int64_t c0 = (i - r * chunks) * 8;
    const int64_t valid = cols - c0 < 8 ? (cols - c0 > 0 ? cols - c0 : 0) : 8;  // elements of the chunk in the row
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (valid > 0) {
      const uintptr_t b = reinterpret_cast<uintptr_t>(src + r * ld_src + c0);
      const uint32_t sh = static_cast<uint32_t>(b & 15u);
      const uint4* w = reinterpret_cast<const uint4*>(b - sh);
      const uint4 w0 = w[0];
      // the second word holds elements from (16 - sh) / 2 on: load it only if one of them is in the row
      const uint4 w1 = sh != 0 && static_cast<int64_t>((16u - sh) / 2u) < valid ? w[1] : make_uint4(0u, 0u, 0u, 0u);
      v = sh == 0 ? w0 : extract16(w0, w1, sh);
      if (valid < 8) {  // zero the elements past the row's end
        uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (j >= valid) u[j >> 1] &= (j & 1) ? 0x0000ffffu : 0xffff0000u;
        v = make_uint4(u[0], u[1], u[2], u[3]);
      }
    }
    uint16_t* d = dst + r * ld_dst + c0;
    const uintptr_t da = reinterpret_cast<uintptr_t>(d);
    if (c0 + 8 <= cols_out && (da & 15u) == 0) {
      *reinterpret_cast<uint4*>(d) = v;
    } else if (c0 + 8 <= cols_out && (da & 3u) == 0) {
      uint32_t* d32 = reinterpret_cast<uint32_t*>(d);
      d32[0] = v.x;
      d32[1] = v.y;
      d32[2] = v.z;
      d32[3] = v.w;
    } else {
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (c0 + j < cols_out) d[j] = static_cast<uint16_t>((j & 1) ? (u[j >> 1] >> 16) : (u[j >> 1] & 0xffffu));
    }
  }
}

}  // namespace repack
}  // namespace zcb
