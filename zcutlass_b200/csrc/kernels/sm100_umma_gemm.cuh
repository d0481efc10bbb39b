// Persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   D[M,N] = alpha * A[M,K] * B[K,N] + beta * C[M,N] + bias[N]     (row-major, f16/bf16)
//
// Roles (192 threads = 6 warps, one CTA per SM, grid = min(tiles, #SMs)):
//   warp 0      TMA producer: per K-block loads A (128x64, K-major, 128B swizzle)
//               and B into a STAGES-deep shared-memory ring. Row-major B [K,N]
//               arrives as BN/64 boxes of 64(k)x64(n), N-major; column-major B
//               (a PyTorch [N,K] weight) as one BNx64 box, K-major.
//   warp 1      owns TMEM (allocates 2*BN columns = two accumulators) and one
//               elected thread issues tcgen05.mma (M=128, N=BN, K=16) per
//               16-wide K slice; tcgen05.commit frees ring slots and publishes
//               finished accumulators.
//   warps 2-5   epilogue: tcgen05.ld 32 rows x 32 columns, alpha/beta/bias in
//               registers, convert, write a 32x32 tile to a swizzled shared
//               buffer and TMA-store it. Double-buffered TMEM lets the epilogue
//               of tile i overlap the main loop of tile i+1.
//
// Ragged M/N/K need no special code: TMA loads zero-fill outside the tensor and
// TMA stores clip, so the only host-side requirements are 16-byte aligned base
// pointers and leading dimensions that are multiples of 8 elements.
#pragma once

#include "sm100_ptx.cuh"

namespace zcb {

enum : uint32_t { kEpiHasC = 1u, kEpiHasBias = 2u };

struct UmmaGemmParams {
  int m, n, k;
  int tiles_m, tiles_n, num_kb, total_tiles;
  int group_m;  // raster: tiles are visited in bands of group_m tile-rows
  float alpha, beta;
  const void* c;
  int64_t ldc;
  const void* bias;
  void* d;  // used for the ragged last column chunk only (see epilogue)
  int64_t ldd;
  uint32_t epi_flags;
  int* error_word;
  // A split by rows over several buffers (TmaMapSet): rows [i * a_rows_per_part,
  // (i + 1) * a_rows_per_part) come from map i. 0 / 1 for a single buffer.
  int a_rows_per_part;
  int a_parts;
};

namespace umma {

constexpr int kBlockM = 128;
constexpr int kBlockK = 64;  // 64 x 2 B = one 128-byte swizzle row
constexpr int kUmmaK = 16;
constexpr int kThreads = 192;
constexpr int kEpiWarps = 4;
constexpr int kEpiCols = 32;  // columns per epilogue chunk

__host__ __device__ constexpr uint32_t tmem_cols_for(int bn) {
  return (2 * bn) <= 32 ? 32 : (2 * bn) <= 64 ? 64 : (2 * bn) <= 128 ? 128 : (2 * bn) <= 256 ? 256 : 512;
}

// A stage holds KSUB sub-blocks of 64 K: one TMA unit streams faster with
// larger stages at the same bytes in flight (mid-size problems, where few
// tiles per SM leave each SM's load rate as the limit).
template <int BN, int STAGES, int KSUB = 1>
struct Smem {
  static constexpr int kASubBytes = kBlockM * kBlockK * 2;     // 16 KiB
  static constexpr int kBChunkBytes = kBlockK * 128;           // one 64(N) x 64(K) box: 8 KiB
  static constexpr int kBSubBytes = (BN / 64) * kBChunkBytes;  // BN=256: 32 KiB
  static constexpr int kABytes = KSUB * kASubBytes;
  static constexpr int kBBytes = KSUB * kBSubBytes;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kEpiBufBytes = 32 * kEpiCols * 2;       // 2 KiB
  static constexpr int kAOff = 0;
  static constexpr int kBOff = STAGES * kABytes;
  static constexpr int kEpiOff = kBOff + STAGES * kBBytes;
  static constexpr int kBarOff = kEpiOff + kEpiWarps * 2 * kEpiBufBytes;
  static constexpr int kNumBars = 2 * STAGES + 5;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kBytes = kMiscOff + 16;
  static constexpr int kDynamicBytes = kBytes + 1024;  // slack to align the base to 1024
  static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "BN must be 64..256 in steps of 64");
  static_assert(kDynamicBytes <= 232448, "shared memory budget exceeded");
};

__device__ __forceinline__ void raster_tile(int tile, const UmmaGemmParams& p, int& tm, int& tn) {
  const int per_group = p.group_m * p.tiles_n;
  const int g = tile / per_group;
  const int first_m = g * p.group_m;
  const int gm = min(p.tiles_m - first_m, p.group_m);
  const int local = tile - g * per_group;
  tm = first_m + local % gm;
  tn = local / gm;
}

// Error codes written to the error word: (site << 4) | role.
enum : int {
  kErrProducerEmpty = (1 << 4) | 1,
  kErrMmaTmemEmpty = (2 << 4) | 2,
  kErrMmaFull = (3 << 4) | 2,
  kErrEpiTmemFull = (4 << 4) | 3,
};

template <typename T, int BN>
__device__ __forceinline__ void load_row_chunk(const T* src, int valid, float (&out)[32]) {
  // src points at 32 consecutive elements of one row; `valid` of them are in bounds.
  if (valid >= 32) {
    const uint4* v = reinterpret_cast<const uint4*>(src);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 u = __ldg(v + j);
      const float2 f0 = Elem<T>::unpack(u.x), f1 = Elem<T>::unpack(u.y);
      const float2 f2 = Elem<T>::unpack(u.z), f3 = Elem<T>::unpack(u.w);
      out[8 * j + 0] = f0.x; out[8 * j + 1] = f0.y; out[8 * j + 2] = f1.x; out[8 * j + 3] = f1.y;
      out[8 * j + 4] = f2.x; out[8 * j + 5] = f2.y; out[8 * j + 6] = f3.x; out[8 * j + 7] = f3.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) out[i] = i < valid ? Elem<T>::to_float(src[i]) : 0.0f;
  }
}

// Stores the first `valid` (< 32) of 32 packed 16-bit values to dst; fully
// unrolled so `packed` stays in registers.
template <typename T>
__device__ __forceinline__ void store_row_prefix(T* dst, const uint32_t (&packed)[16], int valid) {
  uint16_t* d = reinterpret_cast<uint16_t*>(dst);
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    if (i < valid) d[i] = static_cast<uint16_t>((i & 1) ? (packed[i >> 1] >> 16) : (packed[i >> 1] & 0xffffu));
  }
}

// kBKMajor: B is given column-major (B[k][n] at n*ldb + k, i.e. a PyTorch
// [N, K] weight); its tiles are then K-major like A's.
template <typename T, int BN, int STAGES, bool kBKMajor, int kAParts = 1, int KSUB = 1>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ TmaMapSet<kAParts> amaps, const __grid_constant__ CUtensorMap tmap_b,
                const __grid_constant__ CUtensorMap tmap_d, const UmmaGemmParams p) {
  using L = Smem<BN, STAGES, KSUB>;
  constexpr uint32_t kTmemCols = tmem_cols_for(BN);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* tmem_full = empty + STAGES;   // [2]
  uint64_t* tmem_empty = tmem_full + 2;   // [2]
  uint64_t* drain = tmem_empty + 2;       // [1], abort path only
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMiscOff + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tmem_full[b], 1);
      mbar_init(&tmem_empty[b], kEpiWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    for (int i = 0; i < kAParts; ++i) tma_prefetch_desc(&amaps.map[i]);
    tma_prefetch_desc(&tmap_b);
    tma_prefetch_desc(&tmap_d);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();  // inputs/outputs may belong to the previous kernel on the stream
  griddep_launch_dependents();
  const WaitCtx ctx{abort_flag, p.error_word};

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.total_tiles; tile += gridDim.x) {
        int tm, tn;
        raster_tile(tile, p, tm, tn);
        const int m0 = tm * kBlockM, n0 = tn * BN;
        const CUtensorMap* tmap_a = map_for_row(amaps, m0, p.a_rows_per_part, p.a_parts);
        for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
          const uint32_t s = it % STAGES;
          if (!mbar_wait(&empty[s], ((it / STAGES) & 1u) ^ 1u, ctx, kErrProducerEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], L::kStageBytes);
#pragma unroll
          for (int sub = 0; sub < KSUB; ++sub) {
            const int k0 = (kb * KSUB + sub) * kBlockK;
            uint8_t* a_dst = smem + L::kAOff + s * L::kABytes + sub * L::kASubBytes;
            uint8_t* b_dst = smem + L::kBOff + s * L::kBBytes + sub * L::kBSubBytes;
            tma_load_2d(a_dst, tmap_a, &full[s], k0, m0);
            if constexpr (kBKMajor) {
              tma_load_2d(b_dst, &tmap_b, &full[s], k0, n0);
            } else {
#pragma unroll
              for (int j = 0; j < BN / 64; ++j)
                tma_load_2d(b_dst + j * L::kBChunkBytes, &tmap_b, &full[s], n0 + 64 * j, k0);
            }
          }
        }
      }
      if (!ok) {
        // Unwind: let the loads already issued land before the CTA can exit.
        const uint32_t first = it > static_cast<uint32_t>(STAGES) ? it - STAGES : 0u;
        for (uint32_t j = first; j < it; ++j)
          mbar_wait_quiet(&full[j % STAGES], (j / STAGES) & 1u, 200000000ull);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdesc = umma_idesc_f16<Elem<T>::kBf16>(kBlockM, BN, false, !kBKMajor);
      uint32_t it = 0;
      int t = 0;
      bool ok = true, issued = false;
      for (int tile = blockIdx.x; ok && tile < p.total_tiles; tile += gridDim.x, ++t) {
        const uint32_t buf = t & 1, use = t >> 1;
        if (!mbar_wait(&tmem_empty[buf], (use & 1u) ^ 1u, ctx, kErrMmaTmemEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
          const uint32_t s = it % STAGES;
          if (!mbar_wait(&full[s], (it / STAGES) & 1u, ctx, kErrMmaFull)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
#pragma unroll
          for (int sub = 0; sub < KSUB; ++sub) {
            const uint32_t a_addr = smem_addr(smem + L::kAOff + s * L::kABytes + sub * L::kASubBytes);
            const uint32_t b_addr = smem_addr(smem + L::kBOff + s * L::kBBytes + sub * L::kBSubBytes);
#pragma unroll
            for (int kk = 0; kk < kBlockK / kUmmaK; ++kk) {
              // A: K-major rows of 128 B; a 16-wide K slice starts 32 B further in.
              const uint64_t a_desc = smem_desc_sw128(a_addr + kk * 32, 16, 1024);
              // B N-major: 64-column atoms are kBChunkBytes apart (LBO), 8-row
              // K groups 1024 B apart (SBO); a K slice of 16 rows is 2048 B.
              // B K-major: same form as A.
              const uint64_t b_desc = kBKMajor
                                          ? smem_desc_sw128(b_addr + kk * 32, 16, 1024)
                                          : smem_desc_sw128(b_addr + kk * 2048, L::kBChunkBytes, 1024);
              umma_f16_ss(d_tmem, a_desc, b_desc, kIdesc, (kb | sub | kk) != 0 ? 1u : 0u);
            }
          }
          issued = true;
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&tmem_full[buf]);
      }
      if (!ok && issued) {
        // Unwind: wait for MMAs in flight before TMEM is released.
        umma_commit(drain);
        mbar_wait_quiet(drain, 0, 200000000ull);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lanes this warp may read: 32*quarter ..
    const int e = warp - 2;
    uint8_t* stage_base = smem + L::kEpiOff + e * 2 * L::kEpiBufBytes;
    const T* cptr = static_cast<const T*>(p.c);
    const T* bptr = static_cast<const T*>(p.bias);
    const bool has_c = (p.epi_flags & kEpiHasC) != 0;
    const bool has_bias = (p.epi_flags & kEpiHasBias) != 0;
    uint32_t chunk_ctr = 0;
    int t = 0;
    for (int tile = blockIdx.x; tile < p.total_tiles; tile += gridDim.x, ++t) {
      int tm, tn;
      raster_tile(tile, p, tm, tn);
      const int m0 = tm * kBlockM, n0 = tn * BN;
      const uint32_t buf = t & 1, use = t >> 1;
      const bool ok = mbar_wait(&tmem_full[buf], use & 1u, ctx, kErrEpiTmemFull);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after_sync();
      const int row = m0 + quarter * 32 + lane;
      const bool row_ok = row < p.m;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * BN;
#pragma unroll 1
      for (int c = 0; c < BN / kEpiCols; ++c) {
        const int nc = n0 + c * kEpiCols;
        if (nc >= p.n) break;  // uniform across the warp
        uint32_t acc[32];
        tmem_ld_32x32b_x32(t_row + c * kEpiCols, acc);
        float cv[32], bv[32];
        if (has_c) {
          if (row_ok)
            load_row_chunk<T, BN>(cptr + static_cast<int64_t>(row) * p.ldc + nc, p.n - nc, cv);
          else
#pragma unroll
            for (int i = 0; i < 32; ++i) cv[i] = 0.0f;
        }
        if (has_bias) load_row_chunk<T, BN>(bptr + nc, p.n - nc, bv);
        tmem_ld_wait();
        uint32_t packed[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float v0 = p.alpha * __uint_as_float(acc[2 * i]);
          float v1 = p.alpha * __uint_as_float(acc[2 * i + 1]);
          if (has_c) {
            v0 += p.beta * cv[2 * i];
            v1 += p.beta * cv[2 * i + 1];
          }
          if (has_bias) {
            v0 += bv[2 * i];
            v1 += bv[2 * i + 1];
          }
          packed[i] = Elem<T>::pack(v0, v1);
        }
        if (nc + kEpiCols > p.n) {
          // Ragged last chunk: a TMA store clips the inner dimension in 16-byte
          // units, which would touch D's padding columns when N is not a
          // multiple of 8. Store exactly the in-bounds elements instead.
          if (row_ok) store_row_prefix(static_cast<T*>(p.d) + static_cast<int64_t>(row) * p.ldd + nc, packed, p.n - nc);
          continue;
        }
        uint8_t* sb = stage_base + (chunk_ctr & 1u) * L::kEpiBufBytes;
        if (lane == 0) bulk_wait_group_read<1>();  // the store that last used `sb` has read it
        __syncwarp();
        // 64-byte swizzle (matches the D tensor map): 16-byte unit j of row r
        // sits at unit j ^ ((r >> 1) & 3); conflict-free for 8 consecutive rows.
        uint4* srow = reinterpret_cast<uint4*>(sb + lane * 64);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          srow[j ^ ((lane >> 1) & 3)] =
              make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmap_d, sb, nc, m0 + quarter * 32);
          bulk_commit_group();
        }
        ++chunk_ctr;
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tmem_empty[buf]);
    }
    if (lane == 0) bulk_wait_group<0>();
    __syncwarp();
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace umma
}  // namespace zcb
