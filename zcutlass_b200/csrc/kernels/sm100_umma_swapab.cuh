// Small-M (decode) tcgen05 GEMM for sm_100a: swap A and B so the weight
// matrix fills the 128-row MMA dimension and the few tokens sit on MMA-N.
//
//   D^T[N, M] = B^T[N, K] * A^T[K, M]
//   MMA operand "A" = a 128(n) x 64(k) tile of B[K,N]   (N-major, 128B swizzle)
//   MMA operand "B" = an MP(m) x 64(k) tile of A[M,K]   (K-major, 128B swizzle)
//   accumulator     = TMEM lanes = n (128), columns = m (MP = M padded to 16/32/64)
//
// The weights are streamed exactly once, so the kernel is HBM-bound; to keep
// enough loads in flight it splits K across the CTAs of a thread-block cluster
// (cluster = splits x 1 x 1, all working on the same 128-column slice of N).
// Each CTA parks its FP32 partial in its own shared memory, the cluster
// synchronises, and CTA r reduces its share of the tile's 32 groups of 4
// rows of D^T (groups [r*32/S, (r+1)*32/S)) by reading every peer's partial
// through distributed shared memory (ld.shared::cluster.v4, all CTAs' loads of
// a pass in flight at once: the remote-load latency is paid once per pass,
// and one pass covers M <= 16), then applies alpha/beta/bias and writes D
// with coalesced stores. No global scratch memory is used.
#pragma once

#include "sm100_ptx.cuh"

namespace zcb {

struct SwapAbParams {
  int m, n, k;
  int num_kb, splits;
  float alpha, beta;
  const void* c;
  int64_t ldc;
  void* d;
  int64_t ldd;
  const void* bias;
  uint32_t epi_flags;  // kEpiHasC | kEpiHasBias (same bits as the persistent kernel)
  int* error_word;
};

namespace swapab {

constexpr int kBlockN = 128;  // rows of D^T per CTA (MMA M)
constexpr int kBlockK = 64;   // one 128-byte swizzle row of K; a stage holds KSUB of them
constexpr int kThreads = 192;
constexpr int kMaxSplits = 8;  // cluster size limit (portable)
constexpr int kRedUnroll = 2;  // reduction groups (4 outputs each) per thread per pass

// A pipeline stage holds KSUB K sub-blocks of 64: TMA streams a weight
// matrix at ~4.7 TB/s with 16 KiB per stage but ~5.7 TB/s with >= 32 KiB
// (measured on B200, independent of ring depth), so decode uses KSUB = 2.
template <int MP, int STAGES, int KSUB = 1>
struct Smem {
  static constexpr int kWChunkBytes = kBlockK * 128;       // 64(n) x 64(k) box: 8 KiB
  static constexpr int kWSubBytes = 2 * kWChunkBytes;       // 128(n) x 64(k): 16 KiB
  static constexpr int kXSubBytes = MP * 128;               // MP(m) x 64(k)
  static constexpr int kWBytes = KSUB * kWSubBytes;
  static constexpr int kXBytes = KSUB * kXSubBytes;
  static constexpr int kStageBytes = kWBytes + kXBytes;
  static constexpr int kWOff = 0;
  static constexpr int kXOff = STAGES * kWBytes;
  static constexpr int kRedOff = kXOff + STAGES * kXBytes;  // MP x 128 floats, [m][n]
  static constexpr int kBarOff = kRedOff + MP * kBlockN * 4;
  static constexpr int kNumBars = 2 * STAGES + 2;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kBytes = kMiscOff + 16;
  static constexpr int kDynamicBytes = kBytes + 1024;
  static_assert(MP == 16 || MP == 32 || MP == 64, "MP must be 16, 32 or 64");
  static_assert(kDynamicBytes <= 232448, "shared memory budget exceeded");
};

enum : int {
  kErrProducerEmpty = (5 << 4) | 1,
  kErrMmaFull = (6 << 4) | 2,
  kErrEpiTmemFull = (7 << 4) | 3,
};

__device__ __forceinline__ float4 ld_dsmem_v4f(uint32_t local_addr, uint32_t rank) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(map_shared_rank(local_addr, rank))
               : "memory");
  return v;
}

__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// kWKMajor: the weight matrix is column-major B (a PyTorch [N, K] weight), so
// its 128(n) x 64(k) tile is one K-major box instead of two N-major boxes.
// p.num_kb counts K blocks of KSUB * 64.
template <typename T, int MP, int STAGES, int KSUB, bool kWKMajor>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                const SwapAbParams p) {
  using L = Smem<MP, STAGES, KSUB>;
  constexpr uint32_t kTmemCols = MP < 32 ? 32 : MP;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* tmem_full = empty + STAGES;
  uint64_t* drain = tmem_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMiscOff + 4);
  float* red = reinterpret_cast<float*>(smem + L::kRedOff);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t split = cluster_ctarank();
  const int n0 = blockIdx.y * kBlockN;
  const int kb_begin = static_cast<int>((static_cast<int64_t>(split) * p.num_kb) / p.splits);
  const int kb_end = static_cast<int>((static_cast<int64_t>(split + 1) * p.num_kb) / p.splits);

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
    tma_prefetch_desc(&tmap_w);
    tma_prefetch_desc(&tmap_x);
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
    if (lane == 0) {
      const uint64_t stream_once = l2_policy_evict_first();  // weights: read once
      const uint64_t keep = l2_policy_evict_last();          // tokens: read by every CTA
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
          uint8_t* w = smem + L::kWOff + s * L::kWBytes + sub * L::kWSubBytes;
          if constexpr (kWKMajor) {
            tma_load_2d_hint(w, &tmap_w, &full[s], k0, n0, stream_once);
          } else {
            tma_load_2d_hint(w, &tmap_w, &full[s], n0, k0, stream_once);
            tma_load_2d_hint(w + L::kWChunkBytes, &tmap_w, &full[s], n0 + 64, k0, stream_once);
          }
          tma_load_2d_hint(smem + L::kXOff + s * L::kXBytes + sub * L::kXSubBytes, &tmap_x, &full[s], k0, 0,
                           keep);
        }
      }
      if (!ok) {
        const uint32_t first = it > static_cast<uint32_t>(STAGES) ? it - STAGES : 0u;
        for (uint32_t j = first; j < it; ++j)
          mbar_wait_quiet(&full[j % STAGES], (j / STAGES) & 1u, 200000000ull);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // A operand (weights) is MN-major for row-major B, K-major for
      // column-major B; the B operand (tokens) is always K-major.
      constexpr uint32_t kIdesc = umma_idesc_f16<Elem<T>::kBf16>(kBlockN, MP, !kWKMajor, false);
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
          const uint32_t w_addr = smem_addr(smem + L::kWOff + s * L::kWBytes + sub * L::kWSubBytes);
          const uint32_t x_addr = smem_addr(smem + L::kXOff + s * L::kXBytes + sub * L::kXSubBytes);
#pragma unroll
          for (int kk = 0; kk < kBlockK / 16; ++kk) {
            const uint64_t a_desc = kWKMajor ? smem_desc_sw128(w_addr + kk * 32, 16, 1024)
                                             : smem_desc_sw128(w_addr + kk * 2048, L::kWChunkBytes, 1024);
            const uint64_t b_desc = smem_desc_sw128(x_addr + kk * 32, 16, 1024);
            umma_f16_ss(tmem_base, a_desc, b_desc, kIdesc, (it | sub | kk) != 0 ? 1u : 0u);
          }
        }
        issued = true;
        umma_commit(&empty[s]);
      }
      if (ok) {
        umma_commit(tmem_full);
      } else if (issued) {
        umma_commit(drain);
        mbar_wait_quiet(drain, 0, 200000000ull);
      }
    }
    __syncwarp();
  } else {
    // Park this CTA's partial tile in shared memory as red[m][n_local].
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const bool ok = mbar_wait(tmem_full, 0, ctx, kErrEpiTmemFull);
    if (__all_sync(0xffffffffu, ok)) {
      tc_fence_after_sync();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll
      for (int c = 0; c < MP / 16; ++c) {
        uint32_t acc[16];
        tmem_ld_32x32b_x16(taddr + c * 16, acc);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) red[(c * 16 + j) * kBlockN + row] = __uint_as_float(acc[j]);
      }
    }
  }

  // Every thread of every CTA in the cluster reaches both cluster barriers,
  // also on the abort path, so no CTA can wait on a peer that left.
  tc_fence_before_sync();
  __syncwarp();
  cluster_sync_all();

  {
    const T* cptr = static_cast<const T*>(p.c);
    const T* bptr = static_cast<const T*>(p.bias);
    T* dptr = static_cast<T*>(p.d);
    const bool has_c = (p.epi_flags & kEpiHasC) != 0;
    const bool has_bias = (p.epi_flags & kEpiHasBias) != 0;
    constexpr int kGroups = kBlockN / 4;  // groups of 4 rows of D^T (4 consecutive n)
    const int g_begin = static_cast<int>((split * kGroups) / p.splits);
    const int g_end = static_cast<int>(((split + 1) * kGroups) / p.splits);
    const int groups = g_end - g_begin;
    const uint32_t red_addr = smem_addr(red);
    const int total = groups * p.m;  // work items: (token mi, group g)
    // Every thread of the CTA takes kRedUnroll items per pass, every remote
    // load of the pass issued before the first sum.
#pragma unroll 1
    for (int i0 = threadIdx.x; i0 < total; i0 += kThreads * kRedUnroll) {
      float4 part[kRedUnroll][kMaxSplits];
#pragma unroll
      for (int u = 0; u < kRedUnroll; ++u) {
        const int idx = i0 + u * kThreads;
        if (idx >= total) continue;
        const uint32_t off = static_cast<uint32_t>(((idx / groups) * kBlockN + 4 * (g_begin + idx % groups)) * 4);
#pragma unroll
        for (int s = 0; s < kMaxSplits; ++s)
          if (s < p.splits) part[u][s] = ld_dsmem_v4f(red_addr + off, static_cast<uint32_t>(s));
      }
#pragma unroll
      for (int u = 0; u < kRedUnroll; ++u) {
        const int idx = i0 + u * kThreads;
        if (idx >= total) continue;
        const int mi = idx / groups;
        const int nb = n0 + 4 * (g_begin + idx % groups);
        float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);  // in split order: the result does not depend on timing
#pragma unroll
        for (int s = 0; s < kMaxSplits; ++s) {
          if (s < p.splits) {
            sum.x += part[u][s].x;
            sum.y += part[u][s].y;
            sum.z += part[u][s].z;
            sum.w += part[u][s].w;
          }
        }
        const float v4[4] = {sum.x, sum.y, sum.z, sum.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int n = nb + j;
          if (n >= p.n) continue;
          float v = p.alpha * v4[j];
          if (has_c) v += p.beta * Elem<T>::to_float(cptr[static_cast<int64_t>(mi) * p.ldc + n]);
          if (has_bias) v += Elem<T>::to_float(bptr[n]);
          dptr[static_cast<int64_t>(mi) * p.ldd + n] = Elem<T>::from_float(v);
        }
      }
    }
  }

  __syncwarp();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace swapab
}  // namespace zcb
