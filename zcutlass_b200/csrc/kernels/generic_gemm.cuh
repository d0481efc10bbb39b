// Fully predicated CUDA-core GEMM for layouts TMA cannot describe: leading
// dimensions that are not multiples of 8 elements, base pointers that are not
// 16-byte aligned, and tiny problems where a 128-row tensor-core tile would be
// almost all padding. Supports alpha/beta/bias exactly like the tensor-core
// path and accumulates in FP32 in increasing-k order.
#pragma once

#include <cstdint>

#include "sm100_ptx.cuh"

namespace zcb {

struct GenericGemmParams {
  int64_t m, n, k;
  const void* a;
  int64_t lda;
  const void* b;
  int64_t ldb;
  const void* c;
  int64_t ldc;
  void* d;
  int64_t ldd;
  const void* bias;
  float alpha, beta;
  int b_col_major;  // B[k][n] at n*ldb + k instead of k*ldb + n
};

namespace generic {

constexpr int kTile = 64;
constexpr int kTileK = 16;
constexpr int kThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kThreads) gemm_kernel(const GenericGemmParams p) {
  __shared__ float as[kTileK][kTile + 1];  // [k][m]
  __shared__ float bs[kTileK][kTile + 1];  // [k][n]
  const T* A = static_cast<const T*>(p.a);
  const T* B = static_cast<const T*>(p.b);
  const T* C = static_cast<const T*>(p.c);
  const T* bias = static_cast<const T*>(p.bias);
  T* D = static_cast<T*>(p.d);
  // Launched with programmatic stream serialization: wait for the previous
  // kernel on the stream before touching global memory.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t tiles_m = (p.m + kTile - 1) / kTile;

  for (int64_t tmi = blockIdx.y; tmi < tiles_m; tmi += gridDim.y) {
    const int64_t m0 = tmi * kTile, n0 = static_cast<int64_t>(blockIdx.x) * kTile;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;

    for (int64_t k0 = 0; k0 < p.k; k0 += kTileK) {
      for (int idx = threadIdx.x; idx < kTile * kTileK; idx += kThreads) {
        const int r = idx / kTileK, kk = idx % kTileK;
        const int64_t gm = m0 + r, gk = k0 + kk;
        as[kk][r] = (gm < p.m && gk < p.k) ? Elem<T>::to_float(A[gm * p.lda + gk]) : 0.0f;
      }
      for (int idx = threadIdx.x; idx < kTile * kTileK; idx += kThreads) {
        const int kk = idx / kTile, cidx = idx % kTile;
        const int64_t gk = k0 + kk, gn = n0 + cidx;
        const int64_t off = p.b_col_major ? gn * p.ldb + gk : gk * p.ldb + gn;
        bs[kk][cidx] = (gk < p.k && gn < p.n) ? Elem<T>::to_float(B[off]) : 0.0f;
      }
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < kTileK; ++kk) {
        float a[4], b[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) a[i] = as[kk][ty + 16 * i];
#pragma unroll
        for (int j = 0; j < 4; ++j) b[j] = bs[kk][tx + 16 * j];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
      }
      __syncthreads();
    }

#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t gm = m0 + ty + 16 * i;
      if (gm >= p.m) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t gn = n0 + tx + 16 * j;
        if (gn >= p.n) continue;
        float v = p.alpha * acc[i][j];
        if (p.beta != 0.0f) v += p.beta * Elem<T>::to_float(C[gm * p.ldc + gn]);
        if (bias != nullptr) v += Elem<T>::to_float(bias[gn]);
        D[gm * p.ldd + gn] = Elem<T>::from_float(v);
      }
    }
  }
}

}  // namespace generic
}  // namespace zcb
