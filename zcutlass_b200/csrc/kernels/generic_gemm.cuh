// Fully predicated tensor-core GEMM for layouts TMA cannot describe: leading
// dimensions that are not multiples of 8 elements, base pointers that are not
// 16-byte aligned (any 2-byte aligned address works), and C/D/bias that the
// tcgen05 epilogue cannot store or vector-load. Supports alpha/beta/bias
// exactly like the tcgen05 path, FP32 accumulation.
//
// Tile 128 x 128 x 32, 8 warps (2 along M x 4 along N, 64 x 32 each) issuing
// mma.sync m16n8k16 from shared memory; operands come in through predicated
// 2-byte global loads (zero outside the matrix), are held in registers while
// the previous K slice is multiplied, and are stored to a double-buffered,
// K-contiguous shared tile (A as [m][k], B as [n][k], rows padded to 80 bytes
// so fragment reads are bank-conflict free). The epilogue writes D with
// predicated scalar stores, so nothing outside [M, N] is touched.
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

constexpr int kTileM = 128;
constexpr int kTileN = 128;
constexpr int kTileK = 32;
constexpr int kThreads = 256;
constexpr int kRow = kTileK + 8;                         // halves per shared row (80 bytes)
constexpr int kLoads = kTileM * kTileK / kThreads;       // elements of A (and of B) per thread per slice
static_assert(kTileM == kTileN, "A and B slices share the load schedule");

template <bool kBf16>
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  if constexpr (kBf16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const GenericGemmParams p) {
  __shared__ __align__(16) uint16_t as[2][kTileM * kRow];  // [m][k]
  __shared__ __align__(16) uint16_t bs[2][kTileN * kRow];  // [n][k]
  const uint16_t* A = static_cast<const uint16_t*>(p.a);
  const uint16_t* B = static_cast<const uint16_t*>(p.b);
  const T* C = static_cast<const T*>(p.c);
  const T* bias = static_cast<const T*>(p.bias);
  T* D = static_cast<T*>(p.d);
  // Launched with programmatic stream serialization: wait for the previous
  // kernel on the stream before touching global memory.
  griddep_wait();
  griddep_launch_dependents();

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int wm = warp >> 2, wn = warp & 3;  // warp tile: rows wm*64.., cols wn*32..
  const int64_t tiles_m = (p.m + kTileM - 1) / kTileM;
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * kTileN;
  const int num_kt = static_cast<int>((p.k + kTileK - 1) / kTileK);

  for (int64_t tmi = blockIdx.y; tmi < tiles_m; tmi += gridDim.y) {
    const int64_t m0 = tmi * kTileM;
    uint16_t ra[kLoads], rb[kLoads];

    // Element i of this thread's share of a slice: A row/col along K
    // (consecutive threads read consecutive k); B along its contiguous axis.
    auto load = [&](int64_t k0) {
#pragma unroll
      for (int i = 0; i < kLoads; ++i) {
        const int idx = tid + i * kThreads;
        const int r = idx / kTileK, kk = idx % kTileK;
        const int64_t gm = m0 + r, gk = k0 + kk;
        ra[i] = (gm < p.m && gk < p.k) ? A[gm * p.lda + gk] : uint16_t(0);
      }
#pragma unroll
      for (int i = 0; i < kLoads; ++i) {
        const int idx = tid + i * kThreads;
        int nn, kk;
        if (p.b_col_major) {
          nn = idx / kTileK;
          kk = idx % kTileK;
        } else {
          kk = idx / kTileN;
          nn = idx % kTileN;
        }
        const int64_t gn = n0 + nn, gk = k0 + kk;
        const int64_t off = p.b_col_major ? gn * p.ldb + gk : gk * p.ldb + gn;
        rb[i] = (gn < p.n && gk < p.k) ? B[off] : uint16_t(0);
      }
    };
    auto store = [&](int buf) {
#pragma unroll
      for (int i = 0; i < kLoads; ++i) {
        const int idx = tid + i * kThreads;
        as[buf][(idx / kTileK) * kRow + idx % kTileK] = ra[i];
      }
#pragma unroll
      for (int i = 0; i < kLoads; ++i) {
        const int idx = tid + i * kThreads;
        const int nn = p.b_col_major ? idx / kTileK : idx % kTileN;
        const int kk = p.b_col_major ? idx % kTileK : idx / kTileN;
        bs[buf][nn * kRow + kk] = rb[i];
      }
    };

    float acc[4][4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.0f;

    if (num_kt > 0) {
      load(0);
      store(0);
    }
    __syncthreads();
    for (int kt = 0; kt < num_kt; ++kt) {
      const int buf = kt & 1;
      if (kt + 1 < num_kt) load(static_cast<int64_t>(kt + 1) * kTileK);  // in flight during the MMAs
      const uint16_t* sa = as[buf];
      const uint16_t* sb = bs[buf];
#pragma unroll
      for (int ks = 0; ks < kTileK; ks += 16) {
        uint32_t af[4][4], bf[4][2];
#pragma unroll
        for (int mi = 0; mi < 4; ++mi) {
          const int r = wm * 64 + mi * 16 + g;
          af[mi][0] = *reinterpret_cast<const uint32_t*>(sa + r * kRow + ks + 2 * t);
          af[mi][1] = *reinterpret_cast<const uint32_t*>(sa + (r + 8) * kRow + ks + 2 * t);
          af[mi][2] = *reinterpret_cast<const uint32_t*>(sa + r * kRow + ks + 2 * t + 8);
          af[mi][3] = *reinterpret_cast<const uint32_t*>(sa + (r + 8) * kRow + ks + 2 * t + 8);
        }
#pragma unroll
        for (int ni = 0; ni < 4; ++ni) {
          const int cidx = wn * 32 + ni * 8 + g;
          bf[ni][0] = *reinterpret_cast<const uint32_t*>(sb + cidx * kRow + ks + 2 * t);
          bf[ni][1] = *reinterpret_cast<const uint32_t*>(sb + cidx * kRow + ks + 2 * t + 8);
        }
#pragma unroll
        for (int mi = 0; mi < 4; ++mi)
#pragma unroll
          for (int ni = 0; ni < 4; ++ni) mma_16816<Elem<T>::kBf16>(acc[mi][ni], af[mi], bf[ni]);
      }
      if (kt + 1 < num_kt) store(buf ^ 1);  // that buffer was last read before the previous barrier
      __syncthreads();
    }

    // Accumulator fragment: e = 0,1 -> (row g, cols 2t, 2t+1); e = 2,3 -> row g + 8.
#pragma unroll
    for (int mi = 0; mi < 4; ++mi) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int64_t gm = m0 + wm * 64 + mi * 16 + g + half * 8;
        if (gm >= p.m) continue;
#pragma unroll
        for (int ni = 0; ni < 4; ++ni) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int64_t gn = n0 + wn * 32 + ni * 8 + 2 * t + e;
            if (gn >= p.n) continue;
            float v = p.alpha * acc[mi][ni][half * 2 + e];
            if (p.beta != 0.0f) v += p.beta * Elem<T>::to_float(C[gm * p.ldc + gn]);
            if (bias != nullptr) v += Elem<T>::to_float(bias[gn]);
            D[gm * p.ldd + gn] = Elem<T>::from_float(v);
          }
        }
      }
    }
  }
}

}  // namespace generic
}  // namespace zcb
