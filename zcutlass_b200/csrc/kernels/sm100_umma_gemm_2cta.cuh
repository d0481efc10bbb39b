// Persistent tcgen05 GEMM on CTA pairs (cta_group::2), 256 x 256 output tiles.
//
// A cluster of two CTAs on the two SMs of a TPC computes one 256x256 tile per
// step: the leader (cluster rank 0) issues tcgen05.mma.cta_group::2 with
// M = 256, N = 256, K = 16; each CTA supplies its own 128 rows of A and its own
// 128 columns of B from its shared memory, and each CTA's TMEM receives its
// 128 rows x 256 columns of the accumulator. Compared with the one-CTA
// 128x256 tile this halves the B bytes every SM loads and reads from shared
// memory per MMA, which is what lets the tensor pipe stay busy.
//
// Roles per CTA (192 threads), as in the one-CTA kernel:
//   warp 0     TMA producer for this CTA's half tiles. Both CTAs' loads signal
//              the leader's `full` barrier (.cta_group::2 form, no multicast);
//              each waits on its own `empty` barrier.
//   warp 1     TMEM (cta_group::2 alloc of 512 columns in both CTAs); on the
//              leader one thread issues the MMAs and multicasts tcgen05.commit
//              to both CTAs' `empty` / `tmem_full` barriers.
//   warps 2-5  epilogue on this CTA's 128 rows (TMEM -> registers -> swizzled
//              shared -> TMA store), then arrive on the leader's `tmem_empty`.
// Every wait is bounded (see sm100_ptx.cuh); both CTAs meet at a cluster
// barrier before TMEM is released, also on the abort path.
#pragma once

#include "sm100_umma_gemm.cuh"

namespace zcb {
namespace umma2 {

constexpr int kHalfM = 128;    // rows per CTA
constexpr int kBlockM = 256;   // rows per pair
constexpr int kHalfN = 128;    // B columns per CTA
constexpr int kBlockN = 256;   // output columns per pair
constexpr int kBlockK = 64;
constexpr int kThreads = 192;
constexpr int kEpiWarps = 4;
constexpr int kEpiCols = 32;
constexpr uint32_t kTmemCols = 512;  // two 256-column accumulators

// A stage holds KSUB sub-blocks of 64 K per CTA.
template <int STAGES, int KSUB = 1>
struct Smem {
  static constexpr int kASubBytes = kHalfM * kBlockK * 2;  // 16 KiB
  static constexpr int kBChunkBytes = kBlockK * 128;       // 64(n) x 64(k) N-major box: 8 KiB
  static constexpr int kBSubBytes = kHalfN * kBlockK * 2;  // 16 KiB
  static constexpr int kABytes = KSUB * kASubBytes;
  static constexpr int kBBytes = KSUB * kBSubBytes;
  static constexpr int kStageBytes = kABytes + kBBytes;  // per CTA
  static constexpr int kEpiBufBytes = 32 * kEpiCols * 2;
  static constexpr int kAOff = 0;
  static constexpr int kBOff = STAGES * kABytes;
  static constexpr int kEpiOff = kBOff + STAGES * kBBytes;
  static constexpr int kBarOff = kEpiOff + kEpiWarps * 2 * kEpiBufBytes;
  static constexpr int kNumBars = 2 * STAGES + 5;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kBytes = kMiscOff + 16;
  static constexpr int kDynamicBytes = kBytes + 1024;
  static_assert(kDynamicBytes <= 232448, "shared memory budget exceeded");
};

enum : int {
  kErrProducerEmpty = (8 << 4) | 1,
  kErrMmaTmemEmpty = (9 << 4) | 2,
  kErrMmaFull = (10 << 4) | 2,
  kErrEpiTmemFull = (11 << 4) | 3,
};

template <typename T, int STAGES, bool kBKMajor, int kAParts = 1, int KSUB = 1>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ TmaMapSet<kAParts> amaps, const __grid_constant__ CUtensorMap tmap_b,
                const __grid_constant__ CUtensorMap tmap_d, const UmmaGemmParams p) {
  using L = Smem<STAGES, KSUB>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);  // used in the leader
  uint64_t* empty = full + STAGES;
  uint64_t* tmem_full = empty + STAGES;  // [2]
  uint64_t* tmem_empty = tmem_full + 2;  // [2], used in the leader
  uint64_t* drain = tmem_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMiscOff + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tmem_full[b], 1);
      mbar_init(&tmem_empty[b], 2 * kEpiWarps);
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
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before_sync();
  cluster_sync_all();  // barrier inits and TMEM allocation visible to the peer
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();  // inputs/outputs may belong to the previous kernel on the stream
  griddep_launch_dependents();
  const WaitCtx ctx{abort_flag, p.error_word};
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < p.total_tiles; tile += npairs) {
        int tm, tn;
        umma::raster_tile(tile, p, tm, tn);
        const int m0 = tm * kBlockM + static_cast<int>(rank) * kHalfM;
        const int nb = tn * kBlockN + static_cast<int>(rank) * kHalfN;
        const CUtensorMap* tmap_a = map_for_row(amaps, m0, p.a_rows_per_part, p.a_parts);
        for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
          const uint32_t s = it % STAGES;
          if (!mbar_wait(&empty[s], ((it / STAGES) & 1u) ^ 1u, ctx, kErrProducerEmpty)) {
            ok = false;
            break;
          }
          const uint32_t full_leader = map_shared_rank(smem_addr(&full[s]), 0);
          if (leader) mbar_arrive_expect_tx(&full[s], 2 * L::kStageBytes);
#pragma unroll
          for (int sub = 0; sub < KSUB; ++sub) {
            const int k0 = (kb * KSUB + sub) * kBlockK;
            tma_load_2d_pair(smem + L::kAOff + s * L::kABytes + sub * L::kASubBytes, tmap_a, full_leader, k0, m0);
            uint8_t* sb = smem + L::kBOff + s * L::kBBytes + sub * L::kBSubBytes;
            if constexpr (kBKMajor) {
              tma_load_2d_pair(sb, &tmap_b, full_leader, k0, nb);
            } else {
              tma_load_2d_pair(sb, &tmap_b, full_leader, nb, k0);
              tma_load_2d_pair(sb + L::kBChunkBytes, &tmap_b, full_leader, nb + 64, k0);
            }
          }
        }
      }
      if (!ok) {
        // Unwind: loads already issued must land before the CTAs can exit.
        if (leader) {
          const uint32_t first = it > static_cast<uint32_t>(STAGES) ? it - STAGES : 0u;
          for (uint32_t j = first; j < it; ++j)
            mbar_wait_quiet(&full[j % STAGES], (j / STAGES) & 1u, 200000000ull);
        } else {
          for (int i = 0; i < 1000; ++i) sleep_ns(1000);  // the follower cannot poll the leader's barrier
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (leader && lane == 0) {
      constexpr uint32_t kIdesc = umma_idesc_f16<Elem<T>::kBf16>(kBlockM, kBlockN, false, !kBKMajor);
      uint32_t it = 0;
      int t = 0;
      bool ok = true, issued = false;
      for (int tile = pair; ok && tile < p.total_tiles; tile += npairs, ++t) {
        const uint32_t buf = t & 1, use = t >> 1;
        if (!mbar_wait(&tmem_empty[buf], (use & 1u) ^ 1u, ctx, kErrMmaTmemEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + buf * kBlockN;
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
            for (int kk = 0; kk < kBlockK / 16; ++kk) {
              const uint64_t a_desc = smem_desc_sw128(a_addr + kk * 32, 16, 1024);
              const uint64_t b_desc = kBKMajor ? smem_desc_sw128(b_addr + kk * 32, 16, 1024)
                                               : smem_desc_sw128(b_addr + kk * 2048, L::kBChunkBytes, 1024);
              umma_f16_ss_pair(d_tmem, a_desc, b_desc, kIdesc, (kb | sub | kk) != 0 ? 1u : 0u);
            }
          }
          issued = true;
          umma_commit_pair_multicast(&empty[s], 0x3);
        }
        if (!ok) break;
        umma_commit_pair_multicast(&tmem_full[buf], 0x3);
      }
      if (!ok && issued) {
        umma_commit_pair_multicast(drain, 0x1);
        mbar_wait_quiet(drain, 0, 200000000ull);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quarter = warp & 3;
    const int e = warp - 2;
    uint8_t* stage_base = smem + L::kEpiOff + e * 2 * L::kEpiBufBytes;
    const T* cptr = static_cast<const T*>(p.c);
    const T* bptr = static_cast<const T*>(p.bias);
    const bool has_c = (p.epi_flags & kEpiHasC) != 0;
    const bool has_bias = (p.epi_flags & kEpiHasBias) != 0;
    uint32_t chunk_ctr = 0;
    int t = 0;
    for (int tile = pair; tile < p.total_tiles; tile += npairs, ++t) {
      int tm, tn;
      umma::raster_tile(tile, p, tm, tn);
      const int m0 = tm * kBlockM + static_cast<int>(rank) * kHalfM;
      const int n0 = tn * kBlockN;
      const uint32_t buf = t & 1, use = t >> 1;
      const bool ok = mbar_wait(&tmem_full[buf], use & 1u, ctx, kErrEpiTmemFull);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after_sync();
      const int row = m0 + quarter * 32 + lane;
      const bool row_ok = row < p.m;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * kBlockN;
#pragma unroll 1
      for (int c = 0; c < kBlockN / kEpiCols; ++c) {
        const int nc = n0 + c * kEpiCols;
        if (nc >= p.n) break;
        uint32_t acc[32];
        tmem_ld_32x32b_x32(t_row + c * kEpiCols, acc);
        float cv[32], bv[32];
        if (has_c) {
          if (row_ok)
            umma::load_row_chunk<T, kBlockN>(cptr + static_cast<int64_t>(row) * p.ldc + nc, p.n - nc, cv);
          else
#pragma unroll
            for (int i = 0; i < 32; ++i) cv[i] = 0.0f;
        }
        if (has_bias) umma::load_row_chunk<T, kBlockN>(bptr + nc, p.n - nc, bv);
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
          // Ragged last chunk: store exactly the in-bounds elements (a TMA store
          // clips the inner dimension in 16-byte units).
          if (row_ok) umma::store_row_prefix(static_cast<T*>(p.d) + static_cast<int64_t>(row) * p.ldd + nc, packed, p.n - nc);
          continue;
        }
        uint8_t* sb = stage_base + (chunk_ctr & 1u) * L::kEpiBufBytes;
        if (lane == 0) bulk_wait_group_read<1>();
        __syncwarp();
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
      if (lane == 0) mbar_arrive_cluster(map_shared_rank(smem_addr(&tmem_empty[buf]), 0));
    }
    if (lane == 0) bulk_wait_group<0>();
    __syncwarp();
  }

  tc_fence_before_sync();
  __syncwarp();
  cluster_sync_all();  // no CTA leaves while its peer may still touch its memory
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

}  // namespace umma2
}  // namespace zcb
