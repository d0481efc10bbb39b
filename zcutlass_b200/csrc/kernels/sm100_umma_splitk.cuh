// Cluster split-K tcgen05 GEMM for sm_100a: mid-size problems whose output
// has too few 128 x BN tiles to occupy every SM (M of a few hundred tokens,
// e.g. 256 x 4096 x 4096 has 32 tiles of 128 x 256 for 148 SMs).
//
//   D[M,N] = alpha * A[M,K] * B[K,N] + beta * C[M,N] + bias[N]     (row-major, f16/bf16)
//
// One thread-block cluster of S CTAs computes one BM x BN output tile; CTA r
// of the cluster runs K blocks [r*KB/S, (r+1)*KB/S) through the same
// warp-specialised pipeline as the persistent kernel (warp 0 TMA producer,
// warp 1 MMA issuer, warps 2-5 epilogue). With BM = 256 the CTA holds two
// 128 x BN accumulators in TMEM (all 512 columns for BN = 256) and every B
// tile it loads feeds both, which halves the bytes the SM's TMA unit moves
// per FLOP -- the limit for these HBM-streaming shapes. Afterwards, for each
// 128-row half h of the tile:
//   1. the epilogue warps copy half h of the FP32 partial from TMEM into this
//      CTA's shared memory ([128][BN + 4] floats, over the drained ring);
//   2. cluster barrier: every CTA's half h is in place;
//   3. CTA r owns rows [r*128/S, (r+1)*128/S) of the half: each thread reads a
//      4-column group of its rows from every CTA's partial through distributed
//      shared memory (ld.shared::cluster.v4), adds them in CTA order -- the
//      sum does not depend on timing -- applies alpha/beta/bias, rounds once
//      and stores 4 outputs (8 bytes) to D;
//   4. cluster barrier: no CTA overwrites or leaves while a peer still reads.
// No global scratch memory is used. Ragged M/N/K: TMA zero-fills loads
// outside A and B; rows and columns outside D are never stored.
#pragma once

#include "sm100_ptx.cuh"
#include "sm100_umma_gemm.cuh"  // kEpiHasC / kEpiHasBias

namespace zcb {

struct SplitKParams {
  int m, n, k;
  int num_kb;  // K blocks of 64
  int splits;  // CTAs per cluster, along K
  float alpha, beta;
  const void* c;
  int64_t ldc;
  const void* bias;
  void* d;
  int64_t ldd;
  uint32_t epi_flags;
  int* error_word;
};

namespace splitk {

constexpr int kBlockM = 128;
constexpr int kBlockK = 64;
constexpr int kUmmaK = 16;
constexpr int kThreads = 192;
constexpr int kEpiWarps = 4;
constexpr int kMaxSplits = 8;  // portable cluster size
constexpr int kUnroll = 2;     // reduction groups per thread per pass

// A stage holds KSUB sub-blocks of 64 K (larger stages stream faster per SM
// at the same bytes in flight).
template <int BM, int BN, int STAGES, int KSUB = 1>
struct Smem {
  static constexpr int kASubBytes = BM * kBlockK * 2;       // 16 or 32 KiB
  static constexpr int kBChunkBytes = kBlockK * 128;        // 64(n) x 64(k) box: 8 KiB
  static constexpr int kBSubBytes = (BN / 64) * kBChunkBytes;
  static constexpr int kABytes = KSUB * kASubBytes;
  static constexpr int kBBytes = KSUB * kBSubBytes;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kAOff = 0;
  static constexpr int kBOff = STAGES * kABytes;
  static constexpr int kRingBytes = STAGES * kStageBytes;
  // FP32 partial, row stride BN + 4 floats: the TMEM-to-shared copy (a row
  // per thread, 16-byte stores) is free of bank conflicts.
  static constexpr int kRedStride = BN + 4;
  static constexpr int kRedBytes = kBlockM * kRedStride * 4;
  static constexpr int kBarOff = kRingBytes;
  static constexpr int kNumBars = 2 * STAGES + 2;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kBytes = kMiscOff + 16;
  static constexpr int kDynamicBytes = kBytes + 1024;
  static_assert(BN == 128 || BN == 256, "BN must be 128 or 256");
  static_assert(BM == 128 || BM == 256, "BM must be 128 or 256");
  static_assert(kRedBytes <= kRingBytes, "the partial tile must fit in the drained pipeline ring");
  static_assert(kDynamicBytes <= 232448, "shared memory budget exceeded");
};

enum : int {
  kErrProducerEmpty = (20 << 4) | 1,
  kErrMmaFull = (21 << 4) | 2,
  kErrEpiTmemFull = (22 << 4) | 3,
};

__device__ __forceinline__ float4 ld_dsmem_v4(uint32_t local_addr, uint32_t rank) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(map_shared_rank(local_addr, rank))
               : "memory");
  return v;
}

template <typename T>
__device__ __forceinline__ float4 load4(const T* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);  // 8-byte aligned by the launch contract
  const float2 lo = Elem<T>::unpack(u.x), hi = Elem<T>::unpack(u.y);
  return make_float4(lo.x, lo.y, hi.x, hi.y);
}

// Epilogue of 4 consecutive outputs of one row: alpha * sum (+ beta * C)
// (+ bias), rounded once; an 8-byte store when all 4 are inside N.
template <typename T>
__device__ __forceinline__ void store_group(T* dptr, const T* cptr, const T* bptr, const SplitKParams& p, bool has_c,
                                            bool has_bias, int row, int col, const float4& sum) {
  float v[4] = {p.alpha * sum.x, p.alpha * sum.y, p.alpha * sum.z, p.alpha * sum.w};
  const int valid = p.n - col < 4 ? p.n - col : 4;
  if (valid == 4) {
    if (has_c) {
      const float4 cv = load4(cptr + static_cast<int64_t>(row) * p.ldc + col);
      v[0] += p.beta * cv.x;
      v[1] += p.beta * cv.y;
      v[2] += p.beta * cv.z;
      v[3] += p.beta * cv.w;
    }
    if (has_bias) {
      const float4 bv = load4(bptr + col);
      v[0] += bv.x;
      v[1] += bv.y;
      v[2] += bv.z;
      v[3] += bv.w;
    }
    uint2 out;
    out.x = Elem<T>::pack(v[0], v[1]);
    out.y = Elem<T>::pack(v[2], v[3]);
    *reinterpret_cast<uint2*>(dptr + static_cast<int64_t>(row) * p.ldd + col) = out;
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (j < valid) {
        float x = v[j];
        if (has_c) x += p.beta * Elem<T>::to_float(cptr[static_cast<int64_t>(row) * p.ldc + col + j]);
        if (has_bias) x += Elem<T>::to_float(bptr[col + j]);
        dptr[static_cast<int64_t>(row) * p.ldd + col + j] = Elem<T>::from_float(x);
      }
    }
  }
}

// kBKMajor: B is column-major (a PyTorch [N, K] weight): its tiles are K-major.
template <typename T, int BM, int BN, int STAGES, bool kBKMajor, int KSUB = 1>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                const SplitKParams p) {
  using L = Smem<BM, BN, STAGES, KSUB>;
  constexpr int kHalves = BM / kBlockM;
  constexpr uint32_t kTmemCols = kHalves * BN;  // accumulator h at columns [h*BN, (h+1)*BN)
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* tmem_full = empty + STAGES;
  uint64_t* drain = tmem_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMiscOff + 4);
  float* red = reinterpret_cast<float*>(smem);  // over the ring, once the main loop is done

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // the cluster spans gridDim.x == p.splits
  const int n0 = blockIdx.y * BN;
  const int m0 = blockIdx.z * BM;
  const int kb_begin = static_cast<int>((static_cast<int64_t>(rank) * p.num_kb) / p.splits);
  const int kb_end = static_cast<int>((static_cast<int64_t>(rank + 1) * p.num_kb) / p.splits);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tmem_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
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
  bool epi_ok = false;  // epilogue warps: the accumulator is complete

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int kb = kb_begin; kb < kb_end; ++kb, ++it) {
        const uint32_t s = it % STAGES;
        if (!mbar_wait(&empty[s], ((it / STAGES) & 1u) ^ 1u, ctx, kErrProducerEmpty)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[s], L::kStageBytes);
#pragma unroll
        for (int sub = 0; sub < KSUB; ++sub) {
          const int k0 = (kb * KSUB + sub) * kBlockK;
          uint8_t* b_dst = smem + L::kBOff + s * L::kBBytes + sub * L::kBSubBytes;
          tma_load_2d(smem + L::kAOff + s * L::kABytes + sub * L::kASubBytes, &tmap_a, &full[s], k0, m0);
          if constexpr (kBKMajor) {
            tma_load_2d(b_dst, &tmap_b, &full[s], k0, n0);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(b_dst + j * L::kBChunkBytes, &tmap_b, &full[s], n0 + 64 * j, k0);
          }
        }
      }
      if (!ok) {
        const uint32_t first = it > static_cast<uint32_t>(STAGES) ? it - STAGES : 0u;
        for (uint32_t j = first; j < it; ++j) mbar_wait_quiet(&full[j % STAGES], (j / STAGES) & 1u, 200000000ull);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t kIdesc = umma_idesc_f16<Elem<T>::kBf16>(kBlockM, BN, false, !kBKMajor);
      uint32_t it = 0;
      bool ok = true, issued = false;
      for (int kb = kb_begin; kb < kb_end; ++kb, ++it) {
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
            const uint64_t b_desc = kBKMajor ? smem_desc_sw128(b_addr + kk * 32, 16, 1024)
                                             : smem_desc_sw128(b_addr + kk * 2048, L::kBChunkBytes, 1024);
#pragma unroll
            for (int h = 0; h < kHalves; ++h) {  // rows [128h, 128h + 128) of the A tile: 16 KiB apart
              const uint64_t a_desc = smem_desc_sw128(a_addr + h * 16384 + kk * 32, 16, 1024);
              umma_f16_ss(tmem_base + h * BN, a_desc, b_desc, kIdesc, (it | sub | kk) != 0 ? 1u : 0u);
            }
          }
        }
        issued = true;
        umma_commit(&empty[s]);
      }
      if (ok && issued) {
        umma_commit(tmem_full);
      } else if (ok) {
        mbar_arrive(tmem_full);  // no K blocks for this CTA: its partial is zero
      } else if (issued) {
        umma_commit(drain);
        mbar_wait_quiet(drain, 0, 200000000ull);
      }
    }
    __syncwarp();
  } else {
    epi_ok = mbar_wait(tmem_full, 0, ctx, kErrEpiTmemFull);
    epi_ok = __all_sync(0xffffffffu, epi_ok);
  }

  const T* cptr = static_cast<const T*>(p.c);
  const T* bptr = static_cast<const T*>(p.bias);
  T* dptr = static_cast<T*>(p.d);
  const bool has_c = (p.epi_flags & kEpiHasC) != 0;
  const bool has_bias = (p.epi_flags & kEpiHasBias) != 0;
  const int r_begin = static_cast<int>((rank * kBlockM) / p.splits);
  const int r_end = static_cast<int>(((rank + 1) * kBlockM) / p.splits);
  constexpr int kGroups = BN / 4;  // 4-column groups per row
  const int total = (r_end - r_begin) * kGroups;
  const uint32_t red_addr = smem_addr(red);

#pragma unroll 1
  for (int h = 0; h < kHalves; ++h) {
    // Half h of the partial from TMEM to shared memory: thread = row of the half.
    if (warp >= 2 && epi_ok) {
      tc_fence_after_sync();
      const int quarter = warp & 3;
      const int row = quarter * 32 + lane;
      float4* dst = reinterpret_cast<float4*>(red + row * L::kRedStride);
      if (kb_end > kb_begin) {
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + h * BN;
#pragma unroll 1
        for (int c = 0; c < BN / 32; c += 2) {  // two 32-column loads in flight per wait
          uint32_t acc[2][32];
          tmem_ld_32x32b_x32(taddr + c * 32, acc[0]);
          tmem_ld_32x32b_x32(taddr + (c + 1) * 32, acc[1]);
          tmem_ld_wait();
#pragma unroll
          for (int q = 0; q < 2; ++q)
#pragma unroll
            for (int j = 0; j < 8; ++j)
              dst[(c + q) * 8 + j] = make_float4(__uint_as_float(acc[q][4 * j]), __uint_as_float(acc[q][4 * j + 1]),
                                                 __uint_as_float(acc[q][4 * j + 2]), __uint_as_float(acc[q][4 * j + 3]));
        }
      } else {
#pragma unroll 4
        for (int j = 0; j < BN / 4; ++j) dst[j] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }

    // Every thread of every CTA reaches both cluster barriers of every half,
    // on the abort path too, so no CTA waits for a peer that left.
    tc_fence_before_sync();
    __syncwarp();
    cluster_sync_all();

    if (*abort_flag == 0) {  // an aborted CTA has no partial; its error code is already recorded
      // kUnroll groups per thread per pass, every DSMEM load of the pass issued
      // before the first sum: the remote-load latency is paid once per pass.
#pragma unroll 1
      for (int g0 = threadIdx.x; g0 < total; g0 += kThreads * kUnroll) {
        float4 part[kUnroll][kMaxSplits];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int g = g0 + u * kThreads;
          if (g >= total) continue;
          const int rl = r_begin + g / kGroups;
          const int cl = (g % kGroups) * 4;
          const uint32_t off = static_cast<uint32_t>((rl * L::kRedStride + cl) * 4);
#pragma unroll
          for (int s = 0; s < kMaxSplits; ++s)
            if (s < p.splits) part[u][s] = ld_dsmem_v4(red_addr + off, static_cast<uint32_t>(s));
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int g = g0 + u * kThreads;
          if (g >= total) continue;
          const int rl = r_begin + g / kGroups;
          const int cl = (g % kGroups) * 4;
          const int row = m0 + h * kBlockM + rl, col = n0 + cl;
          if (row >= p.m || col >= p.n) continue;
          float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int s = 0; s < kMaxSplits; ++s) {
            if (s < p.splits) {  // in CTA order: the result does not depend on timing
              sum.x += part[u][s].x;
              sum.y += part[u][s].y;
              sum.z += part[u][s].z;
              sum.w += part[u][s].w;
            }
          }
          store_group<T>(dptr, cptr, bptr, p, has_c, has_bias, row, col, sum);
        }
      }
    }
    __syncwarp();
    cluster_sync_all();  // peers are done reading this half before it is overwritten or freed
  }

  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace splitk
}  // namespace zcb
