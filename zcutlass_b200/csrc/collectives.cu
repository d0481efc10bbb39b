// NVLink SHARP (NVLS) collectives over a multicast mapping, for the
// tensor-parallel row-parallel linears.
//
// All-reduce of a symmetric buffer in place, as three launches on one stream:
//   1. barrier: every rank has finished writing its partial;
//   2. reduce: every rank reduces its 1/world slice -- multimem.ld_reduce
//      reads the slice from every GPU's copy through the NVSwitch, which adds
//      them with FP32 accumulation -- and multimem.st writes the sum back to
//      every GPU's copy (each 16-byte word crosses NVLink once per direction
//      per GPU);
//   3. barrier: every slice has been written everywhere.
// The barrier is a counter in symmetric memory: each rank adds 1 to every
// rank's copy with one multimem.red and waits, bounded, until its own copy
// reaches world * (number of barriers so far). The counter only grows, so a
// rank that runs ahead into the next barrier cannot release a slow one early.
// The number of barriers so far is itself kept on the device (the word after
// the counter, written only by this rank's barrier kernels, which run in
// stream order), so the launches carry no per-call value and can be captured
// once in a CUDA graph and replayed.
#include <algorithm>
#include <cstdint>
#include <mutex>

#include <cuda_runtime_api.h>

#include "kernels/sm100_ptx.cuh"
#include "launchers.hpp"

namespace zcb {
namespace {

// Error codes written to the device error word: (site << 4) | role.
enum : int { kErrNvlsBarrierPre = (16 << 4) | 1, kErrNvlsBarrierPost = (16 << 4) | 2 };

__global__ void __launch_bounds__(32) nvls_barrier_kernel(uint32_t* mc_flag, uint32_t* flag, uint32_t world,
                                                          uint64_t timeout_ns, int err_code, int* error_word) {
  if (threadIdx.x != 0) return;
  const uint32_t gen = flag[1] + 1u;
  flag[1] = gen;
  const uint32_t target = world * gen;
  // Release: this GPU's earlier writes (the previous kernels on this stream)
  // are visible system-wide before any peer sees the increment.
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  asm volatile("multimem.red.release.sys.global.add.u32 [%0], %1;" ::"l"(mc_flag), "r"(1u) : "memory");
  const uint64_t t0 = global_timer_ns();
  while (true) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if (static_cast<int32_t>(v - target) >= 0) break;
    if (global_timer_ns() - t0 > timeout_ns) {
      if (error_word != nullptr) atomicCAS(error_word, 0, err_code);
      break;
    }
    __nanosleep(64);
  }
}

template <bool kBf16>
__device__ __forceinline__ uint4 multimem_ld_reduce_add(const uint8_t* addr) {
  uint4 v;
  if constexpr (kBf16) {
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(addr)
                 : "memory");
  } else {
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.f16x2 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(addr)
                 : "memory");
  }
  return v;
}

template <bool kBf16>
__device__ __forceinline__ void multimem_st(uint8_t* addr, const uint4& v) {
  if constexpr (kBf16) {
    asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(addr), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
  } else {
    asm volatile("multimem.st.relaxed.sys.global.v4.f16x2 [%0], {%1, %2, %3, %4};" ::"l"(addr), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
  }
}

// Launch shape, from a sweep of threads x unroll x blocks at 8 ranks: with
// 32 MiB / 64 MiB, reduction alone or broadcast alone each runs at ~560 GB/s
// per GPU whatever the shape, but run together they contend in the switch
// and the time grows with the number of blocks (64 MiB: 160 us at 16-32
// blocks, 205 us at 256). 32 blocks x 256 threads x 4 reductions in flight
// (16 KiB outstanding per block) is at the minimum, and leaves the other
// SMs to a concurrently running GEMM.
constexpr int kArThreads = 256;
constexpr int kArUnroll = 4;
constexpr int kArMaxBlocks = 32;

// Reduces 16-byte words [lo, lo + n) across all ranks. kBroadcast: the sums go
// back to every rank's copy (all-reduce); otherwise only to this rank's copy
// at `local` (reduce-scatter). When the device error word is already set --
// the barrier before this launch gave up waiting, so some peers' partials may
// be incomplete -- the kernel does nothing: the caller reads the error word
// and must not use the buffer, and no half-reduced sum is written over it.
template <bool kBf16, bool kBroadcast>
__global__ void __launch_bounds__(kArThreads) nvls_reduce_kernel(uint8_t* mc, uint8_t* local, int64_t lo, int64_t n,
                                                                 const int* error_word) {
  if (error_word != nullptr && *reinterpret_cast<const volatile int*>(error_word) != 0) return;
  uint8_t* base = mc + lo * 16;
  uint8_t* dst = local + lo * 16;
  const int64_t step = static_cast<int64_t>(gridDim.x) * kArThreads * kArUnroll;
  for (int64_t j = static_cast<int64_t>(blockIdx.x) * kArThreads * kArUnroll + threadIdx.x; j < n; j += step) {
    uint4 v[kArUnroll];
#pragma unroll
    for (int u = 0; u < kArUnroll; ++u) {
      const int64_t idx = j + static_cast<int64_t>(u) * kArThreads;
      if (idx < n) v[u] = multimem_ld_reduce_add<kBf16>(base + idx * 16);
    }
#pragma unroll
    for (int u = 0; u < kArUnroll; ++u) {
      const int64_t idx = j + static_cast<int64_t>(u) * kArThreads;
      if (idx < n) {
        if constexpr (kBroadcast) {
          multimem_st<kBf16>(base + idx * 16, v[u]);
        } else {
          *reinterpret_cast<uint4*>(dst + idx * 16) = v[u];
        }
      }
    }
  }
}

// These kernels use no shared memory, but an SM only changes its L1/shared
// split while it is empty: keep the split at maximum shared memory so their
// blocks never hold an SM in a configuration a concurrently launched GEMM CTA
// (about 200 KB of shared memory) cannot use.
constexpr int kMaxDevices = 64;
std::once_flag g_carveout_once[kMaxDevices];

cudaError_t ensure_carveout(int device) {
  if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
  cudaError_t result = cudaSuccess;
  std::call_once(g_carveout_once[device], [&result] {
    const int carve = cudaSharedmemCarveoutMaxShared;
    for (const void* k : {reinterpret_cast<const void*>(&nvls_barrier_kernel),
                          reinterpret_cast<const void*>(&nvls_reduce_kernel<true, true>),
                          reinterpret_cast<const void*>(&nvls_reduce_kernel<false, true>),
                          reinterpret_cast<const void*>(&nvls_reduce_kernel<true, false>),
                          reinterpret_cast<const void*>(&nvls_reduce_kernel<false, false>)}) {
      const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, carve);
      if (e != cudaSuccess && result == cudaSuccess) result = e;
    }
  });
  return result;
}

}  // namespace

namespace {

// barrier -> reduce words [lo, lo + n) -> barrier, all on `stream`.
cudaError_t launch_reduce(void* mc_ptr, void* local_ptr, int64_t lo, int64_t n, bool bf16, bool broadcast,
                          uint32_t* mc_flag, uint32_t* flag, int world, cudaStream_t stream) {
  const DeviceInfo* info = current_device_info();
  if (info == nullptr) return cudaErrorInvalidDevice;
  const cudaError_t ce = ensure_carveout(info->ordinal);
  if (ce != cudaSuccess) return ce;
  const int64_t per_block = static_cast<int64_t>(kArThreads) * kArUnroll;
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((n + per_block - 1) / per_block, kArMaxBlocks));
  const uint32_t w = static_cast<uint32_t>(world);
  auto* mc = static_cast<uint8_t*>(mc_ptr);
  auto* local = static_cast<uint8_t*>(local_ptr);
  const dim3 grid(static_cast<unsigned>(blocks));

  nvls_barrier_kernel<<<1, 32, 0, stream>>>(mc_flag, flag, w, kWaitTimeoutNs, kErrNvlsBarrierPre, info->error_word);
  if (broadcast) {
    if (bf16) nvls_reduce_kernel<true, true><<<grid, kArThreads, 0, stream>>>(mc, local, lo, n, info->error_word);
    else nvls_reduce_kernel<false, true><<<grid, kArThreads, 0, stream>>>(mc, local, lo, n, info->error_word);
  } else {
    if (bf16) nvls_reduce_kernel<true, false><<<grid, kArThreads, 0, stream>>>(mc, local, lo, n, info->error_word);
    else nvls_reduce_kernel<false, false><<<grid, kArThreads, 0, stream>>>(mc, local, lo, n, info->error_word);
  }
  nvls_barrier_kernel<<<1, 32, 0, stream>>>(mc_flag, flag, w, kWaitTimeoutNs, kErrNvlsBarrierPost, info->error_word);
  count_launches(3);
  return cudaGetLastError();
}

bool common_args_ok(const void* mc_ptr, int64_t nbytes, const uint32_t* mc_flag, const uint32_t* flag, int rank,
                    int world) {
  return mc_ptr != nullptr && nbytes > 0 && (nbytes & 15) == 0 && (reinterpret_cast<uintptr_t>(mc_ptr) & 15) == 0 &&
         mc_flag != nullptr && flag != nullptr && (reinterpret_cast<uintptr_t>(mc_flag) & 3) == 0 &&
         (reinterpret_cast<uintptr_t>(flag) & 7) == 0 && world >= 1 && rank >= 0 && rank < world;
}

}  // namespace

cudaError_t launch_nvls_allreduce(void* mc_ptr, int64_t nbytes, bool bf16, uint32_t* mc_flag, uint32_t* flag,
                                  int rank, int world, cudaStream_t stream) {
  if (!common_args_ok(mc_ptr, nbytes, mc_flag, flag, rank, world)) return cudaErrorInvalidValue;
  const int64_t words = nbytes / 16;
  const int64_t lo = words * rank / world;
  const int64_t n = words * (rank + 1) / world - lo;
  return launch_reduce(mc_ptr, mc_ptr, lo, n, bf16, true, mc_flag, flag, world, stream);
}

cudaError_t launch_nvls_barrier(uint32_t* mc_flag, uint32_t* flag, int world, cudaStream_t stream) {
  if (mc_flag == nullptr || flag == nullptr || (reinterpret_cast<uintptr_t>(mc_flag) & 3) != 0 ||
      (reinterpret_cast<uintptr_t>(flag) & 7) != 0 || world < 1) {
    return cudaErrorInvalidValue;
  }
  const DeviceInfo* info = current_device_info();
  if (info == nullptr) return cudaErrorInvalidDevice;
  const cudaError_t ce = ensure_carveout(info->ordinal);
  if (ce != cudaSuccess) return ce;
  nvls_barrier_kernel<<<1, 32, 0, stream>>>(mc_flag, flag, static_cast<uint32_t>(world), kWaitTimeoutNs,
                                             kErrNvlsBarrierPre, info->error_word);
  count_launches(1);
  return cudaGetLastError();
}

cudaError_t launch_nvls_reduce_scatter(void* mc_ptr, void* local_ptr, int64_t nbytes, bool bf16, uint32_t* mc_flag,
                                       uint32_t* flag, int rank, int world, cudaStream_t stream) {
  if (!common_args_ok(mc_ptr, nbytes, mc_flag, flag, rank, world) || local_ptr == nullptr ||
      (reinterpret_cast<uintptr_t>(local_ptr) & 15) != 0 || nbytes % (16 * static_cast<int64_t>(world)) != 0) {
    return cudaErrorInvalidValue;
  }
  const int64_t n = nbytes / 16 / world;  // equal contiguous slices, one per rank
  return launch_reduce(mc_ptr, local_ptr, n * rank, n, bf16, false, mc_flag, flag, world, stream);
}

}  // namespace zcb
