// Stream-K small-M (decode) tcgen05 GEMM for sm_100a.
//
// Same swap-AB MMA as sm100_umma_swapab.cuh (weights on MMA-M = 128 rows of N,
// tokens on MMA-N = MP), but the work is divided so that every SM streams an
// equal share of the weight matrix:
//
//   units  = tiles_n x num_kb            (one unit = a 128(n) x 64(k) weight block)
//   CTA c  = units [c*U/G, (c+1)*U/G)    (G = min(#SMs, U) CTAs, one per SM)
//
// A CTA's range splits into segments, one per n-tile it touches. A segment
// that covers a tile's whole K range is finished in place. Otherwise the CTA
// writes its FP32 partial (MP x 128) to a workspace slot and arrives on the
// tile's counter; the CTA that arrives last sums the tile's partials in
// segment order -- the same order whoever arrives last, so results are
// deterministic -- and applies alpha/beta/bias. Each CTA owns two partial
// slots (its first and its last tile; tiles in between are always whole).
//
// Tile counters hold (epoch << 32 | arrivals). A launch carries a fresh epoch,
// so a counter left behind by an earlier (or aborted) launch reads as zero,
// and the last arriver resets the count so a replayed CUDA graph with the
// same epoch starts clean too.
#pragma once

#include "sm100_ptx.cuh"
#include "sm100_umma_gemm.cuh"  // kEpiHasC / kEpiHasBias

namespace zcb {

struct SwapAbSkParams {
  int m, n, k;
  int num_kb, tiles_n;
  long long total_units;
  int grid;
  float alpha, beta;
  const void* c;
  int64_t ldc;
  void* d;
  int64_t ldd;
  const void* bias;
  uint32_t epi_flags;
  float* partials;                // [grid * 2][MP][128] FP32
  unsigned long long* counters;   // [tiles_n]
  uint32_t epoch;
  int* error_word;
};

namespace swapab_sk {

constexpr int kBlockN = 128;
constexpr int kBlockK = 64;
constexpr int kThreads = 192;
constexpr int kEpiThreads = 128;

// A stage (and a stream-K unit) holds KSUB K sub-blocks of 64 (see the
// stage-size note in sm100_umma_swapab.cuh).
template <int MP, int STAGES, int KSUB = 1>
struct Smem {
  static constexpr int kWChunkBytes = kBlockK * 128;
  static constexpr int kWSubBytes = 2 * kWChunkBytes;  // 128(n) x 64(k)
  static constexpr int kXSubBytes = MP * 128;          // MP(m) x 64(k)
  static constexpr int kWBytes = KSUB * kWSubBytes;
  static constexpr int kXBytes = KSUB * kXSubBytes;
  static constexpr int kStageBytes = kWBytes + kXBytes;
  static constexpr int kWOff = 0;
  static constexpr int kXOff = STAGES * kWBytes;
  static constexpr int kBarOff = kXOff + STAGES * kXBytes;
  static constexpr int kNumBars = 2 * STAGES + 5;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kBytes = kMiscOff + 32;
  static constexpr int kDynamicBytes = kBytes + 1024;
  static_assert(MP == 16 || MP == 32 || MP == 64, "MP must be 16, 32 or 64");
  static_assert(kDynamicBytes <= 232448, "shared memory budget exceeded");
};

enum : int {
  kErrProducerEmpty = (12 << 4) | 1,
  kErrMmaTmemEmpty = (13 << 4) | 2,
  kErrMmaFull = (13 << 4) | 4,
  kErrEpiTmemFull = (14 << 4) | 3,
};

// Segment of CTA `cta` on n-tile `t`: k-blocks [kb0, kb1).
struct Segment {
  int tile, kb0, kb1;
};

__device__ __forceinline__ long long unit_begin(long long cta, const SwapAbSkParams& p) {
  return cta * p.total_units / p.grid;
}

// CTA whose unit range contains unit u.
__device__ __forceinline__ int cta_of_unit(long long u, const SwapAbSkParams& p) {
  const long long c = ((u + 1) * p.grid - 1) / p.total_units;
  return static_cast<int>(c < p.grid - 1 ? c : p.grid - 1);
}

__device__ __forceinline__ void named_bar_epi() { asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory"); }

// Arrives on a tile counter; returns how many CTAs arrived before (this launch).
__device__ __forceinline__ uint32_t arrive_counter(unsigned long long* ctr, uint32_t epoch) {
  unsigned long long cur = *reinterpret_cast<volatile unsigned long long*>(ctr);
  for (;;) {
    const bool same = static_cast<uint32_t>(cur >> 32) == epoch;
    const unsigned long long want = same ? cur + 1 : ((static_cast<unsigned long long>(epoch) << 32) | 1ull);
    const unsigned long long prev = atomicCAS(ctr, cur, want);
    if (prev == cur) return same ? static_cast<uint32_t>(cur & 0xffffffffull) : 0u;
    cur = prev;
  }
}

__device__ __forceinline__ void tmem_ld_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// p.num_kb counts K blocks of KSUB * 64 (one stream-K unit each).
template <typename T, int MP, int STAGES, int KSUB, bool kWKMajor>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                const SwapAbSkParams p) {
  using L = Smem<MP, STAGES, KSUB>;
  constexpr uint32_t kTmemCols = 2 * MP < 32 ? 32 : 2 * MP;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* tmem_full = empty + STAGES;  // [2]
  uint64_t* tmem_empty = tmem_full + 2;  // [2]
  uint64_t* drain = tmem_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMiscOff + 4);
  volatile uint32_t* order_slot = reinterpret_cast<volatile uint32_t*>(smem + L::kMiscOff + 8);
  volatile int* vote = reinterpret_cast<volatile int*>(smem + L::kMiscOff + 16);  // [4]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  const long long u0 = unit_begin(cta, p), u1 = unit_begin(cta + 1, p);
  const int first_tile = static_cast<int>(u0 / p.num_kb);
  const int last_tile = static_cast<int>((u1 - 1) / p.num_kb);
  auto segment = [&](int t) {
    const long long lo = static_cast<long long>(t) * p.num_kb;
    Segment s;
    s.tile = t;
    s.kb0 = static_cast<int>((u0 > lo ? u0 : lo) - lo);
    s.kb1 = static_cast<int>((u1 < lo + p.num_kb ? u1 : lo + p.num_kb) - lo);
    return s;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tmem_full[b], 1);
      mbar_init(&tmem_empty[b], 4);
    }
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
      const uint64_t stream_once = l2_policy_evict_first();
      const uint64_t keep = l2_policy_evict_last();
      uint32_t it = 0;
      bool ok = true;
      for (int t = first_tile; ok && t <= last_tile; ++t) {
        const Segment sg = segment(t);
        const int n0 = t * kBlockN;
        for (int kb = sg.kb0; kb < sg.kb1; ++kb, ++it) {
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
      }
      if (!ok) {
        const uint32_t first = it > static_cast<uint32_t>(STAGES) ? it - STAGES : 0u;
        for (uint32_t j = first; j < it; ++j) mbar_wait_quiet(&full[j % STAGES], (j / STAGES) & 1u, 200000000ull);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t kIdesc = umma_idesc_f16<Elem<T>::kBf16>(kBlockN, MP, !kWKMajor, false);
      uint32_t it = 0;
      int seg = 0;
      bool ok = true, issued = false;
      for (int t = first_tile; ok && t <= last_tile; ++t, ++seg) {
        const Segment sg = segment(t);
        const uint32_t buf = seg & 1, use = seg >> 1;
        if (!mbar_wait(&tmem_empty[buf], (use & 1u) ^ 1u, ctx, kErrMmaTmemEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + buf * MP;
        for (int kb = sg.kb0; kb < sg.kb1; ++kb, ++it) {
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
              umma_f16_ss(d_tmem, a_desc, b_desc, kIdesc, (kb != sg.kb0 || sub != 0 || kk != 0) ? 1u : 0u);
            }
          }
          issued = true;
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&tmem_full[buf]);
      }
      if (!ok && issued) {
        umma_commit(drain);
        mbar_wait_quiet(drain, 0, 200000000ull);
      }
    }
    __syncwarp();
  } else {
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;  // n within the tile
    const int tid = threadIdx.x - 64;     // 0..127 across the four epilogue warps
    const T* cptr = static_cast<const T*>(p.c);
    const T* bptr = static_cast<const T*>(p.bias);
    T* dptr = static_cast<T*>(p.d);
    const bool has_c = (p.epi_flags & kEpiHasC) != 0;
    const bool has_bias = (p.epi_flags & kEpiHasBias) != 0;
    int seg = 0;
    for (int t = first_tile; t <= last_tile; ++t, ++seg) {
      const Segment sg = segment(t);
      const uint32_t buf = seg & 1, use = seg >> 1;
      // The four epilogue warps take every branch below together (the partial
      // path has named barriers): vote on the wait's outcome first. Every
      // path into the vote is a bounded wait, so the vote always completes.
      const bool ok = mbar_wait(&tmem_full[buf], use & 1u, ctx, kErrEpiTmemFull);
      const bool warp_ok = __all_sync(0xffffffffu, ok);
      if (lane == 0) vote[quarter] = warp_ok ? 1 : 0;
      named_bar_epi();
      const bool all_ok = (vote[0] & vote[1] & vote[2] & vote[3]) != 0;
      named_bar_epi();  // votes read before the next segment rewrites them
      if (!all_ok) break;
      tc_fence_after_sync();
      float acc[MP];
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * MP;
#pragma unroll
      for (int c = 0; c < MP / 16; ++c) {
        uint32_t r[16];
        tmem_ld_x16(taddr + c * 16, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[c * 16 + j] = __uint_as_float(r[j]);
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tmem_empty[buf]);

      const int n = t * kBlockN + row;
      const bool whole = sg.kb0 == 0 && sg.kb1 == p.num_kb;
      bool finish = whole;
      if (!whole) {
        const int my_slot = 2 * cta + (t == first_tile ? 0 : 1);
        float* mine = p.partials + static_cast<size_t>(my_slot) * MP * kBlockN;
#pragma unroll
        for (int mi = 0; mi < MP; ++mi)
          if (mi < p.m) mine[mi * kBlockN + row] = acc[mi];
        __threadfence();
        named_bar_epi();
        const long long tlo = static_cast<long long>(t) * p.num_kb;
        const int c_first = cta_of_unit(tlo, p);
        const int c_last = cta_of_unit(tlo + p.num_kb - 1, p);
        const uint32_t nseg = static_cast<uint32_t>(c_last - c_first + 1);
        if (tid == 0) {
          const uint32_t before = arrive_counter(p.counters + t, p.epoch);
          if (before + 1 == nseg) *reinterpret_cast<volatile unsigned long long*>(p.counters + t) =
              static_cast<unsigned long long>(p.epoch) << 32;  // last arriver resets the count
          *order_slot = before;
        }
        named_bar_epi();
        finish = *order_slot + 1 == nseg;
        if (finish) {
          __threadfence();
          // Sum every segment's partial in segment order (deterministic).
          float sum[MP];
#pragma unroll
          for (int mi = 0; mi < MP; ++mi) sum[mi] = 0.0f;
          for (int cj = c_first; cj <= c_last; ++cj) {
            if (cj == cta) {
#pragma unroll
              for (int mi = 0; mi < MP; ++mi) sum[mi] += acc[mi];
            } else {
              const int first_of_cj = static_cast<int>(unit_begin(cj, p) / p.num_kb);
              const int slot = 2 * cj + (t == first_of_cj ? 0 : 1);
              const float* part = p.partials + static_cast<size_t>(slot) * MP * kBlockN;
#pragma unroll
              for (int mi = 0; mi < MP; ++mi)
                if (mi < p.m) sum[mi] += __ldcg(part + mi * kBlockN + row);
            }
          }
#pragma unroll
          for (int mi = 0; mi < MP; ++mi) acc[mi] = sum[mi];
        }
      }
      if (finish && n < p.n) {
        const float bv = has_bias ? Elem<T>::to_float(bptr[n]) : 0.0f;
#pragma unroll
        for (int mi = 0; mi < MP; ++mi) {
          if (mi < p.m) {
            float v = p.alpha * acc[mi];
            if (has_c) v += p.beta * Elem<T>::to_float(cptr[static_cast<int64_t>(mi) * p.ldc + n]);
            v += bv;
            dptr[static_cast<int64_t>(mi) * p.ldd + n] = Elem<T>::from_float(v);
          }
        }
      }
    }
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace swapab_sk
}  // namespace zcb
