// Kernel launchers: the only place that turns host arguments into CUDA
// launches. Everything here assumes the arguments already passed validation.
#pragma once

#include <cstdint>

#include <cuda_runtime_api.h>

namespace zcb {

struct LaunchArgs {
  int64_t m, n, k;
  const void* a;
  int64_t lda;
  const void* b;
  int64_t ldb;
  const void* c;  // null when beta == 0
  int64_t ldc;
  void* d;
  int64_t ldd;
  const void* bias;
  float alpha, beta;
  bool bf16;
  bool b_col_major;  // B[k][n] at n*ldb + k (PyTorch [N, K] weight)
  cudaStream_t stream;
  // Rows of A gathered from several buffers (persistent kernels, column-major
  // B): rows [i * a_rows_per_part, (i + 1) * a_rows_per_part) are read from
  // a_parts[i], each a full [M, K] matrix with leading dimension lda.
  const void* const* a_parts = nullptr;
  int a_nparts = 0;
  int64_t a_rows_per_part = 0;
};

constexpr int kMaxAParts = 8;

// Per-device facts, cached on first use.
struct DeviceInfo {
  int ordinal = -1;
  int cc_major = 0, cc_minor = 0;
  int sm_count = 0;
  int max_smem_optin = 0;
  int* error_word = nullptr;  // device address of this device's error word
};
const DeviceInfo* current_device_info();

// Persistent tcgen05 kernel, 128 x bn tiles (bn in {128, 256}).
cudaError_t launch_umma_gemm(const LaunchArgs& args, int bn);
// Persistent tcgen05 kernel on CTA pairs (cta_group::2), 256 x 256 tiles.
cudaError_t launch_umma_pair_gemm(const LaunchArgs& args);
// Swap-AB tcgen05 kernel for small M (M <= 32): split-K across a thread-block
// cluster, reduced through distributed shared memory.
cudaError_t launch_umma_swapab_gemm(const LaunchArgs& args, int* splits_used);
// Stream-K swap-AB kernel for small M (M <= 64): every SM streams an equal
// share of the weights; partial tiles are reduced through a per-stream
// workspace owned by the library.
cudaError_t launch_umma_swapab_sk_gemm(const LaunchArgs& args);
bool swapab_prefer_streamk(int64_t n, int64_t k, int sm_count);
// False only while `stream` is being captured into a CUDA graph and its
// stream-K workspace does not yet fit an (m, n, k) problem (a first-use
// allocation is not allowed during capture).
bool swapab_sk_ready_for_stream(int64_t m, int64_t n, int64_t k, cudaStream_t stream);
// Predicated CUDA-core kernel for TMA-incompatible layouts.
cudaError_t launch_generic_gemm(const LaunchArgs& args);
// TMA-incompatible layouts on the tcgen05 kernels: the operands TMA cannot
// describe (and C, bias, D where the chosen kernel needs them aligned) are
// copied into 16-byte-aligned rows of a per-(device, stream) scratch buffer
// owned by the library, grown on first use.
cudaError_t launch_repack_gemm(const LaunchArgs& args);
size_t repack_scratch_bytes(const LaunchArgs& args);
// False only while `stream` is being captured into a CUDA graph and its
// scratch buffer does not yet hold `bytes` (allocation is not allowed then).
bool repack_ready_for_stream(size_t bytes, cudaStream_t stream);

// Cluster split-K tcgen05 kernel, one bm x bn tile (128 x 128, 128 x 256 or
// 256 x 256) per cluster of `splits` CTAs along K, reduced through distributed
// shared memory.
cudaError_t launch_umma_splitk_gemm(const LaunchArgs& args, int bm, int bn, int splits);

// Shape heuristics shared by dispatch and telemetry.
enum class PersistentConfig { Pair256x256, Cta128x256, Cta128x128, SplitK256x256, SplitK128x256, SplitK128x128, Cta128x64 };
// The persistent configurations only (no split-K): for paths whose kernels
// need one CTA (pair) per output tile.
PersistentConfig choose_persistent(int64_t m, int64_t n, int sm_count);
struct TileChoice {
  PersistentConfig config;
  int splits;  // CTAs per cluster along K (split-K configurations), else 1
};
// Every configuration, split-K included; ZCUTLASS_SPLITK=<s> fixes the split
// count of the split-K configurations (tests).
TileChoice choose_tiles(int64_t m, int64_t n, int64_t k, int sm_count);
// Split count for a split-K launch of bm x bn tiles when the kernel is used
// outside choose_tiles' choice (forced): ZCUTLASS_SPLITK, else as many CTAs
// per tile as the SMs allow, at most 8 and at most one per K block.
int splitk_default_splits(int64_t m, int64_t n, int64_t k, int bm, int bn, int sm_count);
int swapab_choose_splits(int64_t n, int64_t k, int sm_count);

// In-place NVLS all-reduce (sum) of `nbytes` of f16/bf16 at multicast
// address `mc_ptr` (collectives.cu): barrier, each rank reduces and
// broadcasts its slice, barrier. The barriers use two symmetric u32 words:
// flag[0] the cross-rank counter (multicast address `mc_flag`), flag[1] this
// rank's barrier count.
cudaError_t launch_nvls_allreduce(void* mc_ptr, int64_t nbytes, bool bf16, uint32_t* mc_flag, uint32_t* flag,
                                  int rank, int world, cudaStream_t stream);
// The cross-rank barrier alone (same words and contract as the collectives).
cudaError_t launch_nvls_barrier(uint32_t* mc_flag, uint32_t* flag, int world, cudaStream_t stream);
// Reduce-scatter with the same barriers: rank r sums bytes
// [r * nbytes / world, (r + 1) * nbytes / world) over all ranks into its own
// copy at local_ptr (nbytes a multiple of 16 * world).
cudaError_t launch_nvls_reduce_scatter(void* mc_ptr, void* local_ptr, int64_t nbytes, bool bf16, uint32_t* mc_flag,
                                       uint32_t* flag, int rank, int world, cudaStream_t stream);
int read_and_clear_error_word(bool clear);
// Stream-K decode GEMM with its scratch in a fixed device array (no
// allocation); returns a zcutlass status code. Arguments must already have
// passed the generic validation.
int gemm_decode_noalloc(const LaunchArgs& args);
// Runs a kernel whose bounded mbarrier wait can never be satisfied; returns
// the error code it recorded (expected non-zero), or -1 on a CUDA error.
int selftest_bounded_wait(uint32_t timeout_us);
uint64_t launch_count();
void count_launches(uint64_t n);

}  // namespace zcb
