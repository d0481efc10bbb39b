// Kernel instantiation and launch. Compiled for sm_100a only.
#include "launchers.hpp"

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <mutex>

#include "kernels/generic_gemm.cuh"
#include "kernels/repack.cuh"
#include "kernels/sm100_umma_gemm.cuh"
#include "kernels/sm100_umma_gemm_2cta.cuh"
#include "kernels/sm100_umma_swapab.cuh"
#include "kernels/sm100_umma_splitk.cuh"
#include "kernels/sm100_umma_swapab_sk.cuh"
#include "tma_desc.hpp"

#include <map>
#include <utility>

namespace zcb {

// One error word per device (each device loading the library gets its own
// copy of this variable). Kernels set it when a bounded wait expires.
__device__ int g_device_error_word = 0;

namespace {

constexpr int kMaxDevices = 64;
std::atomic<uint64_t> g_launches{0};

// Decode (swap-AB) kernels stage 2 x 64 of K per pipeline slot: 32 KiB of
// weights per stage, which TMA streams at ~5.7 TB/s (16 KiB stages: ~4.7).
constexpr int kDecodeKsub = 2;
constexpr int kDecodeKBlock = 64 * kDecodeKsub;

struct DeviceSlot {
  std::once_flag once;
  DeviceInfo info;
  // Bit i set once cudaFuncSetAttribute ran for kernel configuration i.
  std::atomic<uint64_t> attr_done{0};
  // Resident CTA pairs of each cluster-launched configuration (0 = not queried).
  int max_active_pairs[64] = {};
  // Resident clusters of each split-K configuration by cluster size (0 = not queried).
  int max_active_clusters[64][9] = {};
};
DeviceSlot g_devices[kMaxDevices];

DeviceSlot* current_slot() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  DeviceSlot* slot = &g_devices[dev];
  std::call_once(slot->once, [slot, dev] {
    DeviceInfo info;
    info.ordinal = dev;
    cudaDeviceGetAttribute(&info.cc_major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&info.cc_minor, cudaDevAttrComputeCapabilityMinor, dev);
    cudaDeviceGetAttribute(&info.sm_count, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&info.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    void* word = nullptr;
    if (cudaGetSymbolAddress(&word, g_device_error_word) == cudaSuccess) {
      info.error_word = static_cast<int*>(word);
    }
    slot->info = info;
  });
  return slot;
}

// Programmatic stream serialization: a GEMM may be launched while the
// previous kernel on its stream is still finishing, so its prologue (barrier
// init, TMEM allocation, descriptor prefetch) and launch latency overlap that
// kernel's tail; every kernel waits (griddepcontrol.wait) before its first
// global memory access. ZCUTLASS_PDL=0 launches without it.
bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("ZCUTLASS_PDL");
    return v == nullptr || v[0] != '0';
  }();
  return on;
}

void add_pdl_attr(cudaLaunchAttribute* attrs, unsigned int& n) {
  if (!pdl_enabled()) return;
  attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[n].val.programmaticStreamSerializationAllowed = 1;
  ++n;
}

// Sets the dynamic shared memory limit of `kernel` once per device.
template <typename Kernel>
cudaError_t ensure_smem_attr(DeviceSlot* slot, int config_bit, Kernel kernel, int bytes) {
  const uint64_t bit = uint64_t(1) << config_bit;
  if (slot->attr_done.load(std::memory_order_acquire) & bit) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) slot->attr_done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

// The A tensor maps: one for the single buffer, or one per row block when
// the rows come from several buffers (a.a_nparts > 1).
template <int AP>
bool make_a_maps(TmaMapSet<AP>* set, const LaunchArgs& a, int box_rows, int box_k) {
  const int parts = AP == 1 ? 1 : a.a_nparts;
  if (parts < 1 || parts > AP) return false;
  for (int i = 0; i < AP; ++i) {
    const void* base = AP == 1 ? a.a : a.a_parts[i < parts ? i : 0];
    if (!make_tma_2d(&set->map[i], base, a.bf16, a.m, a.k, a.lda, box_rows, box_k, TmaSwizzle::B128)) return false;
  }
  return true;
}

template <typename T, int BN, int STAGES, bool KM, int AP = 1, int KSUB = 1>
cudaError_t launch_umma_t(const LaunchArgs& a, DeviceSlot* slot, int config_bit) {
  using L = umma::Smem<BN, STAGES, KSUB>;
  TmaMapSet<AP> ta;
  CUtensorMap tb, td;
  const bool bf16 = a.bf16;
  const bool b_ok = KM ? make_tma_2d(&tb, a.b, bf16, a.n, a.k, a.ldb, BN, umma::kBlockK, TmaSwizzle::B128)
                       : make_tma_2d(&tb, a.b, bf16, a.k, a.n, a.ldb, umma::kBlockK, 64, TmaSwizzle::B128);
  if (!b_ok || !make_a_maps(&ta, a, umma::kBlockM, umma::kBlockK) ||
      !make_tma_2d(&td, a.d, bf16, a.m, a.n, a.ldd, 32, umma::kEpiCols, TmaSwizzle::B64)) {
    return cudaErrorInvalidValue;
  }
  UmmaGemmParams p{};
  p.m = static_cast<int>(a.m);
  p.n = static_cast<int>(a.n);
  p.k = static_cast<int>(a.k);
  p.tiles_m = static_cast<int>((a.m + umma::kBlockM - 1) / umma::kBlockM);
  p.tiles_n = static_cast<int>((a.n + BN - 1) / BN);
  p.num_kb = static_cast<int>((a.k + KSUB * umma::kBlockK - 1) / (KSUB * umma::kBlockK));
  p.total_tiles = p.tiles_m * p.tiles_n;
  p.group_m = std::min(p.tiles_m, 16);
  p.alpha = a.alpha;
  p.beta = a.beta;
  p.c = a.c;
  p.ldc = a.ldc;
  p.bias = a.bias;
  p.d = a.d;
  p.ldd = a.ldd;
  p.epi_flags = (a.beta != 0.0f ? kEpiHasC : 0u) | (a.bias != nullptr ? kEpiHasBias : 0u);
  p.error_word = slot->info.error_word;
  p.a_rows_per_part = AP == 1 ? 0 : static_cast<int>(a.a_rows_per_part);
  p.a_parts = AP == 1 ? 1 : a.a_nparts;

  auto kernel = umma::gemm_kernel<T, BN, STAGES, KM, AP, KSUB>;
  cudaError_t e = ensure_smem_attr(slot, config_bit, kernel, L::kDynamicBytes);
  if (e != cudaSuccess) return e;
  const int grid = std::min(p.total_tiles, slot->info.sm_count);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(umma::kThreads, 1, 1);
  cfg.dynamicSmemBytes = L::kDynamicBytes;
  cfg.stream = a.stream;
  cudaLaunchAttribute attr[1];
  unsigned int nattr = 0;
  add_pdl_attr(attr, nattr);
  cfg.attrs = attr;
  cfg.numAttrs = nattr;
  e = cudaLaunchKernelEx(&cfg, kernel, ta, tb, td, p);
  g_launches.fetch_add(1, std::memory_order_relaxed);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

template <typename T, int MP, int STAGES, bool KM>
cudaError_t launch_swapab_t(const LaunchArgs& a, DeviceSlot* slot, int config_bit, int splits) {
  using L = swapab::Smem<MP, STAGES, kDecodeKsub>;
  CUtensorMap tw, tx;
  const bool bf16 = a.bf16;
  // Weights: the B matrix ([K, N] row-major, or [N, K] when column-major);
  // tokens: the A matrix [M, K].
  const bool w_ok =
      KM ? make_tma_2d(&tw, a.b, bf16, a.n, a.k, a.ldb, swapab::kBlockN, swapab::kBlockK, TmaSwizzle::B128)
         : make_tma_2d(&tw, a.b, bf16, a.k, a.n, a.ldb, swapab::kBlockK, 64, TmaSwizzle::B128);
  if (!w_ok ||
      !make_tma_2d(&tx, a.a, bf16, a.m, a.k, a.lda, MP, swapab::kBlockK, TmaSwizzle::B128)) {
    return cudaErrorInvalidValue;
  }
  SwapAbParams p{};
  p.m = static_cast<int>(a.m);
  p.n = static_cast<int>(a.n);
  p.k = static_cast<int>(a.k);
  p.num_kb = static_cast<int>((a.k + kDecodeKBlock - 1) / kDecodeKBlock);
  p.splits = splits;
  p.alpha = a.alpha;
  p.beta = a.beta;
  p.c = a.c;
  p.ldc = a.ldc;
  p.d = a.d;
  p.ldd = a.ldd;
  p.bias = a.bias;
  p.epi_flags = (a.beta != 0.0f ? kEpiHasC : 0u) | (a.bias != nullptr ? kEpiHasBias : 0u);
  p.error_word = slot->info.error_word;

  auto kernel = swapab::gemm_kernel<T, MP, STAGES, kDecodeKsub, KM>;
  cudaError_t e = ensure_smem_attr(slot, config_bit, kernel, L::kDynamicBytes);
  if (e != cudaSuccess) return e;

  const int tiles_n = static_cast<int>((a.n + swapab::kBlockN - 1) / swapab::kBlockN);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(splits), static_cast<unsigned>(tiles_n), 1);
  cfg.blockDim = dim3(swapab::kThreads, 1, 1);
  cfg.dynamicSmemBytes = L::kDynamicBytes;
  cfg.stream = a.stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(splits);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  unsigned int nattr = 1;
  add_pdl_attr(attr, nattr);
  cfg.attrs = attr;
  cfg.numAttrs = nattr;
  e = cudaLaunchKernelEx(&cfg, kernel, tw, tx, p);
  g_launches.fetch_add(1, std::memory_order_relaxed);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

template <typename T, int STAGES, bool KM, int AP = 1, int KSUB = 1>
cudaError_t launch_umma2_t(const LaunchArgs& a, DeviceSlot* slot, int config_bit) {
  using L = umma2::Smem<STAGES, KSUB>;
  TmaMapSet<AP> ta;
  CUtensorMap tb, td;
  const bool bf16 = a.bf16;
  const bool b_ok =
      KM ? make_tma_2d(&tb, a.b, bf16, a.n, a.k, a.ldb, umma2::kHalfN, umma2::kBlockK, TmaSwizzle::B128)
         : make_tma_2d(&tb, a.b, bf16, a.k, a.n, a.ldb, umma2::kBlockK, 64, TmaSwizzle::B128);
  if (!b_ok || !make_a_maps(&ta, a, umma2::kHalfM, umma2::kBlockK) ||
      !make_tma_2d(&td, a.d, bf16, a.m, a.n, a.ldd, 32, umma2::kEpiCols, TmaSwizzle::B64)) {
    return cudaErrorInvalidValue;
  }
  UmmaGemmParams p{};
  p.m = static_cast<int>(a.m);
  p.n = static_cast<int>(a.n);
  p.k = static_cast<int>(a.k);
  p.tiles_m = static_cast<int>((a.m + umma2::kBlockM - 1) / umma2::kBlockM);
  p.tiles_n = static_cast<int>((a.n + umma2::kBlockN - 1) / umma2::kBlockN);
  p.num_kb = static_cast<int>((a.k + KSUB * umma2::kBlockK - 1) / (KSUB * umma2::kBlockK));
  p.total_tiles = p.tiles_m * p.tiles_n;
  p.group_m = std::min(p.tiles_m, 8);
  p.alpha = a.alpha;
  p.beta = a.beta;
  p.c = a.c;
  p.ldc = a.ldc;
  p.bias = a.bias;
  p.d = a.d;
  p.ldd = a.ldd;
  p.epi_flags = (a.beta != 0.0f ? kEpiHasC : 0u) | (a.bias != nullptr ? kEpiHasBias : 0u);
  p.error_word = slot->info.error_word;
  p.a_rows_per_part = AP == 1 ? 0 : static_cast<int>(a.a_rows_per_part);
  p.a_parts = AP == 1 ? 1 : a.a_nparts;

  auto kernel = umma2::gemm_kernel<T, STAGES, KM, AP, KSUB>;
  cudaError_t e = ensure_smem_attr(slot, config_bit, kernel, L::kDynamicBytes);
  if (e != cudaSuccess) return e;

  cudaLaunchConfig_t cfg{};
  cfg.blockDim = dim3(umma2::kThreads, 1, 1);
  cfg.dynamicSmemBytes = L::kDynamicBytes;
  cfg.stream = a.stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;  // the occupancy query below sees the cluster shape only
  // Persistent grid: as many CTA pairs as can be resident at once (queried
  // once per device), never more than there are tiles.
  int& max_pairs = slot->max_active_pairs[config_bit];
  if (max_pairs == 0) {
    cfg.gridDim = dim3(static_cast<unsigned>(slot->info.sm_count & ~1), 1, 1);
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) != cudaSuccess || clusters <= 0)
      clusters = slot->info.sm_count / 2;
    max_pairs = clusters;
  }
  cfg.gridDim = dim3(static_cast<unsigned>(2 * std::min(p.total_tiles, max_pairs)), 1, 1);
  unsigned int nattr = 1;
  add_pdl_attr(attr, nattr);
  cfg.numAttrs = nattr;
  e = cudaLaunchKernelEx(&cfg, kernel, ta, tb, td, p);
  g_launches.fetch_add(1, std::memory_order_relaxed);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

template <typename T, int BM, int BN, int STAGES, bool KM, int KSUB = 1>
cudaError_t launch_splitk_t(const LaunchArgs& a, DeviceSlot* slot, int config_bit, int splits) {
  using L = splitk::Smem<BM, BN, STAGES, KSUB>;
  CUtensorMap ta, tb;
  const bool bf16 = a.bf16;
  const bool b_ok = KM ? make_tma_2d(&tb, a.b, bf16, a.n, a.k, a.ldb, BN, splitk::kBlockK, TmaSwizzle::B128)
                       : make_tma_2d(&tb, a.b, bf16, a.k, a.n, a.ldb, splitk::kBlockK, 64, TmaSwizzle::B128);
  if (!b_ok || !make_tma_2d(&ta, a.a, bf16, a.m, a.k, a.lda, BM, splitk::kBlockK, TmaSwizzle::B128))
    return cudaErrorInvalidValue;
  const int64_t tiles_m = (a.m + BM - 1) / BM;
  const int64_t tiles_n = (a.n + BN - 1) / BN;
  if (tiles_m > 65535 || tiles_n > 65535) return cudaErrorInvalidValue;
  SplitKParams p{};
  p.m = static_cast<int>(a.m);
  p.n = static_cast<int>(a.n);
  p.k = static_cast<int>(a.k);
  p.num_kb = static_cast<int>((a.k + KSUB * splitk::kBlockK - 1) / (KSUB * splitk::kBlockK));
  p.alpha = a.alpha;
  p.beta = a.beta;
  p.c = a.c;
  p.ldc = a.ldc;
  p.bias = a.bias;
  p.d = a.d;
  p.ldd = a.ldd;
  p.epi_flags = (a.beta != 0.0f ? kEpiHasC : 0u) | (a.bias != nullptr ? kEpiHasBias : 0u);
  p.error_word = slot->info.error_word;

  auto kernel = splitk::gemm_kernel<T, BM, BN, STAGES, KM, KSUB>;
  cudaError_t e = ensure_smem_attr(slot, config_bit, kernel, L::kDynamicBytes);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg{};
  cfg.blockDim = dim3(splitk::kThreads, 1, 1);
  cfg.dynamicSmemBytes = L::kDynamicBytes;
  cfg.stream = a.stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;  // the occupancy query sees the cluster shape only
  // The whole grid should be resident at once (every cluster is one wave of
  // work): fewer CTAs per cluster when that many clusters of `splits` CTAs
  // cannot be co-resident (a cluster must fit in one GPC).
  splits = std::max(1, std::min(std::min(splits, splitk::kMaxSplits), p.num_kb));
  for (; splits > 1; --splits) {
    int& active = slot->max_active_clusters[config_bit][splits];
    if (active == 0) {
      attr[0].val.clusterDim.x = static_cast<unsigned>(splits);
      cfg.gridDim = dim3(static_cast<unsigned>(splits), static_cast<unsigned>(tiles_n), static_cast<unsigned>(tiles_m));
      int clusters = 0;
      if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) != cudaSuccess || clusters <= 0) {
        (void)cudaGetLastError();
        clusters = -1;  // unknown: do not trust this cluster size
      }
      active = clusters;
    }
    if (active >= tiles_m * tiles_n) break;
  }
  p.splits = splits;
  attr[0].val.clusterDim.x = static_cast<unsigned>(splits);
  cfg.gridDim = dim3(static_cast<unsigned>(splits), static_cast<unsigned>(tiles_n), static_cast<unsigned>(tiles_m));
  unsigned int nattr = 1;
  add_pdl_attr(attr, nattr);
  cfg.numAttrs = nattr;
  e = cudaLaunchKernelEx(&cfg, kernel, ta, tb, p);
  g_launches.fetch_add(1, std::memory_order_relaxed);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

// Stream-K workspace, one per (device, stream): tile counters followed by the
// FP32 partial slots. Kernels on one stream run in order, so they can share
// it; kernels on different streams may overlap, so they never do. Grown on
// demand (after draining the stream that used the old buffer); the counter
// region is zeroed when allocated and epoch-tagged afterwards.
struct StreamKWorkspace {
  void* base = nullptr;
  size_t counter_bytes = 0;  // fixed-size counter region at the front
  size_t partial_bytes = 0;  // partial slots after it
  uint32_t epoch = 0;
};
std::mutex g_ws_mutex;
std::map<std::pair<int, cudaStream_t>, StreamKWorkspace> g_ws;

cudaError_t acquire_workspace(int dev, cudaStream_t stream, size_t counter_need, size_t partial_need,
                              unsigned long long** counters, float** partials, uint32_t* epoch) {
  std::lock_guard<std::mutex> lock(g_ws_mutex);
  StreamKWorkspace& ws = g_ws[{dev, stream}];
  if (ws.counter_bytes < counter_need || ws.partial_bytes < partial_need) {
    if (ws.base != nullptr) {
      cudaError_t e = cudaStreamSynchronize(stream);  // the old buffer may still be in use
      if (e != cudaSuccess) return e;
      cudaFree(ws.base);
      ws = StreamKWorkspace{nullptr, 0, 0, ws.epoch};
    }
    const size_t ctr = std::max<size_t>((counter_need + 255) & ~size_t(255), size_t(64) << 10);
    const size_t part = std::max<size_t>((partial_need + 255) & ~size_t(255), size_t(4) << 20);
    cudaError_t e = cudaMalloc(&ws.base, ctr + part);
    if (e != cudaSuccess) return e;
    e = cudaMemsetAsync(ws.base, 0, ctr, stream);  // counters start at (epoch 0, count 0)
    if (e != cudaSuccess) return e;
    ws.counter_bytes = ctr;
    ws.partial_bytes = part;
  }
  ws.epoch = ws.epoch + 1 == 0 ? 1 : ws.epoch + 1;  // never 0: zeroed counters read as stale
  *counters = static_cast<unsigned long long*>(ws.base);
  *partials = reinterpret_cast<float*>(static_cast<char*>(ws.base) + ws.counter_bytes);
  *epoch = ws.epoch;
  return cudaSuccess;
}

// Workspace bytes the stream-K kernel needs for (m, n, k): tile counters and
// two partial slots per CTA (MP = m rounded up to 16, 32 or 64).
void swapab_sk_needs(int64_t m, int64_t n, int64_t k, int sm_count, size_t* counter_need, size_t* partial_need) {
  const int mp = m <= 16 ? 16 : (m <= 32 ? 32 : 64);
  const int64_t tiles_n = (n + swapab_sk::kBlockN - 1) / swapab_sk::kBlockN;
  const int64_t num_kb = (k + kDecodeKBlock - 1) / kDecodeKBlock;
  const int64_t grid = std::min<int64_t>(tiles_n * num_kb, sm_count);
  *counter_need = size_t(tiles_n) * 8;
  *partial_need = size_t(2) * grid * mp * swapab_sk::kBlockN * sizeof(float);
}

template <typename T, int MP, int STAGES, bool KM>
cudaError_t launch_swapab_sk_t(const LaunchArgs& a, DeviceSlot* slot, int config_bit) {
  using L = swapab_sk::Smem<MP, STAGES, kDecodeKsub>;
  CUtensorMap tw, tx;
  const bool bf16 = a.bf16;
  const bool w_ok =
      KM ? make_tma_2d(&tw, a.b, bf16, a.n, a.k, a.ldb, swapab_sk::kBlockN, swapab_sk::kBlockK, TmaSwizzle::B128)
         : make_tma_2d(&tw, a.b, bf16, a.k, a.n, a.ldb, swapab_sk::kBlockK, 64, TmaSwizzle::B128);
  if (!w_ok || !make_tma_2d(&tx, a.a, bf16, a.m, a.k, a.lda, MP, swapab_sk::kBlockK, TmaSwizzle::B128)) {
    return cudaErrorInvalidValue;
  }
  SwapAbSkParams p{};
  p.m = static_cast<int>(a.m);
  p.n = static_cast<int>(a.n);
  p.k = static_cast<int>(a.k);
  p.num_kb = static_cast<int>((a.k + kDecodeKBlock - 1) / kDecodeKBlock);
  p.tiles_n = static_cast<int>((a.n + swapab_sk::kBlockN - 1) / swapab_sk::kBlockN);
  p.total_units = static_cast<long long>(p.num_kb) * p.tiles_n;
  p.grid = static_cast<int>(std::min<long long>(p.total_units, slot->info.sm_count));
  p.alpha = a.alpha;
  p.beta = a.beta;
  p.c = a.c;
  p.ldc = a.ldc;
  p.d = a.d;
  p.ldd = a.ldd;
  p.bias = a.bias;
  p.epi_flags = (a.beta != 0.0f ? kEpiHasC : 0u) | (a.bias != nullptr ? kEpiHasBias : 0u);
  p.error_word = slot->info.error_word;
  cudaError_t e = acquire_workspace(slot->info.ordinal, a.stream, size_t(p.tiles_n) * 8,
                                    size_t(2) * p.grid * MP * swapab_sk::kBlockN * sizeof(float), &p.counters,
                                    &p.partials, &p.epoch);
  if (e != cudaSuccess) return e;

  auto kernel = swapab_sk::gemm_kernel<T, MP, STAGES, kDecodeKsub, KM>;
  e = ensure_smem_attr(slot, config_bit, kernel, L::kDynamicBytes);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(p.grid), 1, 1);
  cfg.blockDim = dim3(swapab_sk::kThreads, 1, 1);
  cfg.dynamicSmemBytes = L::kDynamicBytes;
  cfg.stream = a.stream;
  cudaLaunchAttribute attr[1];
  unsigned int nattr = 0;
  add_pdl_attr(attr, nattr);
  cfg.attrs = attr;
  cfg.numAttrs = nattr;
  e = cudaLaunchKernelEx(&cfg, kernel, tw, tx, p);
  g_launches.fetch_add(1, std::memory_order_relaxed);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_generic_t(const LaunchArgs& a) {
  GenericGemmParams p{a.m,   a.n,   a.k,   a.a,     a.lda,  a.b,   a.ldb,
                      a.c,   a.ldc, a.d,   a.ldd,   a.bias, a.alpha, a.beta,
                      a.b_col_major ? 1 : 0};
  const int64_t tiles_n = (a.n + generic::kTileN - 1) / generic::kTileN;
  const int64_t tiles_m = (a.m + generic::kTileM - 1) / generic::kTileM;
  if (tiles_n > 2147483647LL) return cudaErrorInvalidValue;
  const dim3 grid(static_cast<unsigned>(tiles_n), static_cast<unsigned>(std::min<int64_t>(tiles_m, 65535)));
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(generic::kThreads, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = a.stream;
  cudaLaunchAttribute attr[1];
  unsigned int nattr = 0;
  add_pdl_attr(attr, nattr);
  cfg.attrs = attr;
  cfg.numAttrs = nattr;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, generic::gemm_kernel<T>, p);
  g_launches.fetch_add(1, std::memory_order_relaxed);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

// Kernel configuration bits for ensure_smem_attr: one per instantiation,
// the column-major-B variant of configuration c uses bit c + kCfgColMajorB.
enum : int {
  kCfgUmmaBf16N256 = 0,
  kCfgUmmaF16N256,
  kCfgUmmaBf16N128,
  kCfgUmmaF16N128,
  kCfgSwapBf16M16,
  kCfgSwapF16M16,
  kCfgSwapBf16M32,
  kCfgSwapF16M32,
  kCfgSwapBf16M64,
  kCfgSwapF16M64,
  kCfgPairBf16,
  kCfgPairF16,
  kCfgSkBf16M16,
  kCfgSkF16M16,
  kCfgSkBf16M32,
  kCfgSkF16M32,
  kCfgSkBf16M64,
  kCfgSkF16M64,
  // row-gathered A (column-major B only)
  kCfgGatherPairBf16,
  kCfgGatherPairF16,
  kCfgGatherUmmaBf16N256,
  kCfgGatherUmmaF16N256,
  kCfgGatherUmmaBf16N128,
  kCfgGatherUmmaF16N128,
  kCfgSplitKBf16N256,
  kCfgSplitKF16N256,
  kCfgSplitKBf16N128,
  kCfgSplitKF16N128,
  kCfgSplitKBf16M256,
  kCfgSplitKF16M256,
  kCfgUmmaBf16N64,
  kCfgUmmaF16N64,
  kCfgColMajorB = 32,
};

template <bool KM>
cudaError_t launch_swapab_sk_km(const LaunchArgs& a, DeviceSlot* slot) {
  const int off = KM ? kCfgColMajorB : 0;
  if (a.m <= 16) {
    return a.bf16 ? launch_swapab_sk_t<__nv_bfloat16, 16, 6, KM>(a, slot, kCfgSkBf16M16 + off)
                  : launch_swapab_sk_t<half, 16, 6, KM>(a, slot, kCfgSkF16M16 + off);
  }
  if (a.m <= 32) {
    return a.bf16 ? launch_swapab_sk_t<__nv_bfloat16, 32, 5, KM>(a, slot, kCfgSkBf16M32 + off)
                  : launch_swapab_sk_t<half, 32, 5, KM>(a, slot, kCfgSkF16M32 + off);
  }
  return a.bf16 ? launch_swapab_sk_t<__nv_bfloat16, 64, 4, KM>(a, slot, kCfgSkBf16M64 + off)
                : launch_swapab_sk_t<half, 64, 4, KM>(a, slot, kCfgSkF16M64 + off);
}

template <bool KM>
cudaError_t launch_umma_km(const LaunchArgs& a, DeviceSlot* slot, int bn) {
  const int off = KM ? kCfgColMajorB : 0;
  if (bn == 256) {
    return a.bf16 ? launch_umma_t<__nv_bfloat16, 256, 4, KM>(a, slot, kCfgUmmaBf16N256 + off)
                  : launch_umma_t<half, 256, 4, KM>(a, slot, kCfgUmmaF16N256 + off);
  }
  if (bn == 64) {
    return a.bf16 ? launch_umma_t<__nv_bfloat16, 64, 4, KM, 1, 2>(a, slot, kCfgUmmaBf16N64 + off)
                  : launch_umma_t<half, 64, 4, KM, 1, 2>(a, slot, kCfgUmmaF16N64 + off);
  }
  return a.bf16 ? launch_umma_t<__nv_bfloat16, 128, 3, KM, 1, 2>(a, slot, kCfgUmmaBf16N128 + off)
                : launch_umma_t<half, 128, 3, KM, 1, 2>(a, slot, kCfgUmmaF16N128 + off);
}

template <bool KM>
cudaError_t launch_splitk_km(const LaunchArgs& a, DeviceSlot* slot, int bm, int bn, int splits) {
  const int off = KM ? kCfgColMajorB : 0;
  if (bm == 256) {
    return a.bf16 ? launch_splitk_t<__nv_bfloat16, 256, 256, 3, KM>(a, slot, kCfgSplitKBf16M256 + off, splits)
                  : launch_splitk_t<half, 256, 256, 3, KM>(a, slot, kCfgSplitKF16M256 + off, splits);
  }
  if (bn == 256) {
    return a.bf16 ? launch_splitk_t<__nv_bfloat16, 128, 256, 4, KM>(a, slot, kCfgSplitKBf16N256 + off, splits)
                  : launch_splitk_t<half, 128, 256, 4, KM>(a, slot, kCfgSplitKF16N256 + off, splits);
  }
  return a.bf16 ? launch_splitk_t<__nv_bfloat16, 128, 128, 3, KM, 2>(a, slot, kCfgSplitKBf16N128 + off, splits)
                : launch_splitk_t<half, 128, 128, 3, KM, 2>(a, slot, kCfgSplitKF16N128 + off, splits);
}

template <bool KM>
cudaError_t launch_swapab_km(const LaunchArgs& a, DeviceSlot* slot, int splits) {
  const int off = KM ? kCfgColMajorB : 0;
  if (a.m <= 16) {
    return a.bf16 ? launch_swapab_t<__nv_bfloat16, 16, 5, KM>(a, slot, kCfgSwapBf16M16 + off, splits)
                  : launch_swapab_t<half, 16, 5, KM>(a, slot, kCfgSwapF16M16 + off, splits);
  }
  if (a.m <= 32) {
    return a.bf16 ? launch_swapab_t<__nv_bfloat16, 32, 5, KM>(a, slot, kCfgSwapBf16M32 + off, splits)
                  : launch_swapab_t<half, 32, 5, KM>(a, slot, kCfgSwapF16M32 + off, splits);
  }
  return a.bf16 ? launch_swapab_t<__nv_bfloat16, 64, 4, KM>(a, slot, kCfgSwapBf16M64 + off, splits)
                : launch_swapab_t<half, 64, 4, KM>(a, slot, kCfgSwapF16M64 + off, splits);
}

}  // namespace

const DeviceInfo* current_device_info() {
  DeviceSlot* slot = current_slot();
  return slot ? &slot->info : nullptr;
}

TileChoice choose_tiles(int64_t m, int64_t n, int64_t k, int sm_count) {
  // Time model in SM clocks, fitted on B200 to graph-timed runs (bf16, 148
  // SMs, B column-major, weights rotated past L2) of every configuration on
  // M x N x K = 64 / 128 / 256 / 512 / 1024 x 4096^2, 256 x 8192^2,
  // 256 x 1536^2, 256 x 2048 x 1536, 256 x 14336 x 4096, 1024^3 and
  // 8192 x 28672 x 4096:
  //   persistent: waves x K blocks x clocks per K block of one tile + fixed
  //     (CTA pair 256x256: 800 + 5000, 128x256: 820 + 7000, 128x128: 560 + 5000,
  //     128x64: 454 + 6290; the last two stream two 64-wide K blocks per stage);
  //   split-K (one wave): ceil(K blocks / S) x clocks per K block + fixed,
  //     the fixed part being mostly the cross-CTA reduction of the FP32
  //     partial through distributed shared memory (128x128, two 64-wide K
  //     blocks per stage: 560 + 12900,
  //     128x256: 990 + 15500, 256x256: 1450 + 40000).
  // It picks the fastest measured configuration on each of those shapes
  // (within 3 %).
  const int64_t kb = (k + 63) / 64;
  struct Cand {
    PersistentConfig cfg;
    int tile_m, tile_n, units;  // units: CTAs (or CTA pairs) resident at once
    double per_kb, fixed;
    bool split;
  };
  const int pairs = sm_count / 2;
  const Cand cands[] = {
      {PersistentConfig::Pair256x256, 256, 256, pairs, 800.0, 5000.0, false},
      {PersistentConfig::Cta128x256, 128, 256, sm_count, 820.0, 7000.0, false},
      {PersistentConfig::Cta128x128, 128, 128, sm_count, 560.0, 5000.0, false},
      {PersistentConfig::Cta128x64, 128, 64, sm_count, 454.0, 6290.0, false},
      {PersistentConfig::SplitK256x256, 256, 256, sm_count, 1450.0, 40000.0, true},
      {PersistentConfig::SplitK128x256, 128, 256, sm_count, 990.0, 15500.0, true},
      {PersistentConfig::SplitK128x128, 128, 128, sm_count, 560.0, 12900.0, true},
  };
  const char* forced = std::getenv("ZCUTLASS_SPLITK");
  const int forced_splits = forced != nullptr ? std::atoi(forced) : 0;
  TileChoice best{choose_persistent(m, n, sm_count), 1};
  double best_cost = 1e300;
  for (const Cand& c : cands) {
    const int64_t tiles = ((m + c.tile_m - 1) / c.tile_m) * ((n + c.tile_n - 1) / c.tile_n);
    if (tiles <= 0 || kb <= 0) continue;
    double cost;
    int splits = 1;
    if (!c.split) {
      cost = double((tiles + c.units - 1) / c.units) * double(kb) * c.per_kb + c.fixed;
    } else {
      if (tiles * 2 > sm_count) continue;  // split-K only when the tiles alone leave SMs idle
      int64_t s = std::min<int64_t>({int64_t(splitk::kMaxSplits), sm_count / tiles, kb / 2});
      if (forced_splits > 0) s = std::min<int64_t>(std::min<int64_t>(forced_splits, splitk::kMaxSplits), kb);
      if (s < 2) continue;
      splits = static_cast<int>(s);
      cost = double((kb + s - 1) / s) * c.per_kb + c.fixed;
    }
    if (cost < best_cost * 0.999) {
      best_cost = cost;
      best = {c.cfg, splits};
    }
  }
  return best;
}

int splitk_default_splits(int64_t m, int64_t n, int64_t k, int bm, int bn, int sm_count) {
  const int64_t kb = (k + 63) / 64;
  const int64_t tiles = std::max<int64_t>(1, ((m + bm - 1) / bm) * ((n + bn - 1) / bn));
  const char* forced = std::getenv("ZCUTLASS_SPLITK");
  int64_t s = forced != nullptr && std::atoi(forced) > 0 ? std::atoi(forced) : sm_count / tiles;
  s = std::min<int64_t>({s, int64_t(splitk::kMaxSplits), kb});
  return static_cast<int>(std::max<int64_t>(s, 1));
}

PersistentConfig choose_persistent(int64_t m, int64_t n, int sm_count) {
  // Wave-quantisation cost model: time ~ waves * per-SM tile area / relative
  // efficiency, where a wave is one tile per SM (one 256x256 tile per CTA
  // pair). Efficiencies are the measured throughput ratios of the kernels on
  // large problems (pair 256x256 : 128x256 : 128x128).
  struct Cand {
    PersistentConfig cfg;
    int tile_m, tile_n, units;
    double per_sm_area, eff;
  };
  const int pairs = sm_count / 2;
  const Cand cands[] = {
      {PersistentConfig::Pair256x256, 256, 256, pairs, 256.0 * 256.0 / 2.0, 1.0},
      {PersistentConfig::Cta128x256, 128, 256, sm_count, 128.0 * 256.0, 0.86},
      {PersistentConfig::Cta128x128, 128, 128, sm_count, 128.0 * 128.0, 0.72},
  };
  PersistentConfig best = PersistentConfig::Cta128x128;
  double best_cost = 1e300;
  for (const Cand& c : cands) {
    const int64_t tiles = ((m + c.tile_m - 1) / c.tile_m) * ((n + c.tile_n - 1) / c.tile_n);
    const int64_t waves = (tiles + c.units - 1) / c.units;
    const double cost = static_cast<double>(waves) * c.per_sm_area / c.eff;
    if (cost < best_cost * 0.999) {
      best_cost = cost;
      best = c.cfg;
    }
  }
  return best;
}

int swapab_choose_splits(int64_t n, int64_t k, int sm_count) {
  const int64_t tiles_n = (n + swapab::kBlockN - 1) / swapab::kBlockN;
  const int64_t num_kb = (k + kDecodeKBlock - 1) / kDecodeKBlock;
  int64_t s = sm_count / std::max<int64_t>(tiles_n, 1);
  s = std::min<int64_t>(s, 8);
  s = std::min<int64_t>(s, num_kb);
  return static_cast<int>(std::max<int64_t>(s, 1));
}

cudaError_t launch_umma_gemm(const LaunchArgs& a, int bn) {
  DeviceSlot* slot = current_slot();
  if (slot == nullptr) return cudaErrorInvalidDevice;
  if (a.a_nparts > 1) {
    if (!a.b_col_major || a.a_nparts > kMaxAParts || bn == 64) return cudaErrorInvalidValue;
    if (bn == 256) {
      return a.bf16 ? launch_umma_t<__nv_bfloat16, 256, 4, true, kMaxAParts>(a, slot, kCfgGatherUmmaBf16N256)
                    : launch_umma_t<half, 256, 4, true, kMaxAParts>(a, slot, kCfgGatherUmmaF16N256);
    }
    return a.bf16 ? launch_umma_t<__nv_bfloat16, 128, 6, true, kMaxAParts>(a, slot, kCfgGatherUmmaBf16N128)
                  : launch_umma_t<half, 128, 6, true, kMaxAParts>(a, slot, kCfgGatherUmmaF16N128);
  }
  return a.b_col_major ? launch_umma_km<true>(a, slot, bn) : launch_umma_km<false>(a, slot, bn);
}

cudaError_t launch_umma_splitk_gemm(const LaunchArgs& a, int bm, int bn, int splits) {
  DeviceSlot* slot = current_slot();
  if (slot == nullptr) return cudaErrorInvalidDevice;
  return a.b_col_major ? launch_splitk_km<true>(a, slot, bm, bn, splits)
                       : launch_splitk_km<false>(a, slot, bm, bn, splits);
}

cudaError_t launch_umma_pair_gemm(const LaunchArgs& a) {
  DeviceSlot* slot = current_slot();
  if (slot == nullptr) return cudaErrorInvalidDevice;
  if (a.a_nparts > 1) {
    if (!a.b_col_major || a.a_nparts > kMaxAParts) return cudaErrorInvalidValue;
    return a.bf16 ? launch_umma2_t<__nv_bfloat16, 6, true, kMaxAParts>(a, slot, kCfgGatherPairBf16)
                  : launch_umma2_t<half, 6, true, kMaxAParts>(a, slot, kCfgGatherPairF16);
  }
  const int off = a.b_col_major ? kCfgColMajorB : 0;
  if (a.b_col_major) {
    return a.bf16 ? launch_umma2_t<__nv_bfloat16, 3, true, 1, 2>(a, slot, kCfgPairBf16 + off)
                  : launch_umma2_t<half, 3, true, 1, 2>(a, slot, kCfgPairF16 + off);
  }
  return a.bf16 ? launch_umma2_t<__nv_bfloat16, 3, false, 1, 2>(a, slot, kCfgPairBf16 + off)
                : launch_umma2_t<half, 3, false, 1, 2>(a, slot, kCfgPairF16 + off);
}

cudaError_t launch_umma_swapab_sk_gemm(const LaunchArgs& a) {
  DeviceSlot* slot = current_slot();
  if (slot == nullptr) return cudaErrorInvalidDevice;
  return a.b_col_major ? launch_swapab_sk_km<true>(a, slot) : launch_swapab_sk_km<false>(a, slot);
}

bool swapab_sk_ready_for_stream(int64_t m, int64_t n, int64_t k, cudaStream_t stream) {
  cudaStreamCaptureStatus status = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &status) != cudaSuccess) {
    (void)cudaGetLastError();  // no device (host-only telemetry): not capturing
    return true;
  }
  if (status == cudaStreamCaptureStatusNone) return true;
  DeviceSlot* slot = current_slot();
  if (slot == nullptr) return false;
  size_t counter_need = 0, partial_need = 0;
  swapab_sk_needs(m, n, k, slot->info.sm_count, &counter_need, &partial_need);
  std::lock_guard<std::mutex> lock(g_ws_mutex);
  const auto it = g_ws.find({slot->info.ordinal, stream});
  return it != g_ws.end() && it->second.counter_bytes >= counter_need && it->second.partial_bytes >= partial_need;
}

bool swapab_prefer_streamk(int64_t n, int64_t k, int sm_count) {
  // Cluster split-K fills tiles_n x splits SMs; stream-K always fills all of
  // them. Prefer stream-K unless split-K already covers ~95% of the SMs.
  const int64_t tiles_n = (n + swapab::kBlockN - 1) / swapab::kBlockN;
  const int64_t used = tiles_n * swapab_choose_splits(n, k, sm_count);
  return used * 100 < static_cast<int64_t>(sm_count) * 95;
}

cudaError_t launch_umma_swapab_gemm(const LaunchArgs& a, int* splits_used) {
  DeviceSlot* slot = current_slot();
  if (slot == nullptr) return cudaErrorInvalidDevice;
  const int splits = swapab_choose_splits(a.n, a.k, slot->info.sm_count);
  if (splits_used) *splits_used = splits;
  return a.b_col_major ? launch_swapab_km<true>(a, slot, splits) : launch_swapab_km<false>(a, slot, splits);
}

cudaError_t launch_generic_gemm(const LaunchArgs& a) {
  return a.bf16 ? launch_generic_t<__nv_bfloat16>(a) : launch_generic_t<half>(a);
}

// ---------------------------------------------------------------- generic path through packed operands
//
// Operands TMA cannot describe are copied once into 16-byte-aligned rows of a
// per-(device, stream) scratch buffer, the tcgen05 kernels run on the packed
// copies, and a packed D is copied out. The copies cost one pass over the
// packed operands, against one pass per output tile for repacking inside the
// GEMM's main loop.

namespace {

struct RepackScratch {
  void* base = nullptr;
  size_t bytes = 0;
};
std::mutex g_rp_mutex;
std::map<std::pair<int, cudaStream_t>, RepackScratch> g_rp;

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
int64_t round8(int64_t x) { return (x + 7) & ~int64_t(7); }
size_t round256(size_t x) { return (x + 255) & ~size_t(255); }

struct RepackPlan {
  bool small;  // M <= 64: the swap-AB kernels, which read C / bias and write D element by element
  bool a, b, c, bias, d;
  size_t off_a, off_b, off_c, off_bias, off_d, bytes;
};

RepackPlan plan_repack(const LaunchArgs& a) {
  RepackPlan p{};
  p.small = a.m <= 64;
  p.a = !tma_compatible(a.a, a.lda);
  p.b = !tma_compatible(a.b, a.ldb);
  if (!p.small) {
    p.c = a.c != nullptr && (!aligned16(a.c) || (a.ldc & 7) != 0);
    p.bias = a.bias != nullptr && !aligned16(a.bias);
    p.d = !tma_compatible(a.d, a.ldd);
  }
  size_t off = 0;
  const auto take = [&off](bool used, size_t bytes) {
    const size_t at = off;
    if (used) off += round256(bytes);
    return at;
  };
  p.off_a = take(p.a, size_t(a.m) * round8(a.k) * 2);
  p.off_b = take(p.b, a.b_col_major ? size_t(a.n) * round8(a.k) * 2 : size_t(a.k) * round8(a.n) * 2);
  p.off_c = take(p.c, size_t(a.m) * round8(a.n) * 2);
  p.off_bias = take(p.bias, size_t(round8(a.n)) * 2);
  p.off_d = take(p.d, size_t(a.m) * round8(a.n) * 2);
  p.bytes = off;
  return p;
}

cudaError_t launch_copy2d(void* dst, int64_t ld_dst, const void* src, int64_t ld_src, int64_t rows, int64_t cols,
                          int64_t cols_out, int sm_count, cudaStream_t stream) {
  const int64_t work = rows * ((cols_out + 7) / 8);
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((work + repack::kThreads - 1) / repack::kThreads,
                                                                int64_t(sm_count) * 8));
  repack::copy2d_u16_kernel<<<static_cast<unsigned>(blocks), repack::kThreads, 0, stream>>>(
      static_cast<uint16_t*>(dst), ld_dst, static_cast<const uint16_t*>(src), ld_src, rows, cols, cols_out);
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return cudaGetLastError();
}

}  // namespace

size_t repack_scratch_bytes(const LaunchArgs& a) { return plan_repack(a).bytes; }

bool repack_ready_for_stream(size_t bytes, cudaStream_t stream) {
  cudaStreamCaptureStatus status = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &status) != cudaSuccess) {
    (void)cudaGetLastError();  // no device (host-only telemetry): not capturing
    return true;
  }
  if (status == cudaStreamCaptureStatusNone) return true;
  DeviceSlot* slot = current_slot();
  if (slot == nullptr) return false;
  std::lock_guard<std::mutex> lock(g_rp_mutex);
  const auto it = g_rp.find({slot->info.ordinal, stream});
  return it != g_rp.end() && it->second.bytes >= bytes;
}

cudaError_t launch_repack_gemm(const LaunchArgs& a) {
  DeviceSlot* slot = current_slot();
  if (slot == nullptr) return cudaErrorInvalidDevice;
  const RepackPlan plan = plan_repack(a);
  char* base = nullptr;
  if (plan.bytes > 0) {
    std::lock_guard<std::mutex> lock(g_rp_mutex);
    RepackScratch& sc = g_rp[{slot->info.ordinal, a.stream}];
    if (sc.bytes < plan.bytes) {
      if (sc.base != nullptr) {
        const cudaError_t e = cudaStreamSynchronize(a.stream);  // the old buffer may still be in use
        if (e != cudaSuccess) return e;
        cudaFree(sc.base);
        sc = RepackScratch{};
      }
      const size_t want = std::max<size_t>(plan.bytes, size_t(16) << 20);
      const cudaError_t e = cudaMalloc(&sc.base, want);
      if (e != cudaSuccess) return e;
      sc.bytes = want;
    }
    base = static_cast<char*>(sc.base);
  }
  const int sms = slot->info.sm_count;
  LaunchArgs b = a;
  cudaError_t e = cudaSuccess;
  if (plan.a) {
    b.a = base + plan.off_a;
    b.lda = round8(a.k);
    e = launch_copy2d(base + plan.off_a, b.lda, a.a, a.lda, a.m, a.k, b.lda, sms, a.stream);
    if (e != cudaSuccess) return e;
  }
  if (plan.b) {
    const int64_t rows = a.b_col_major ? a.n : a.k, cols = a.b_col_major ? a.k : a.n;
    b.b = base + plan.off_b;
    b.ldb = round8(cols);
    e = launch_copy2d(base + plan.off_b, b.ldb, a.b, a.ldb, rows, cols, b.ldb, sms, a.stream);
    if (e != cudaSuccess) return e;
  }
  if (plan.c) {
    b.c = base + plan.off_c;
    b.ldc = round8(a.n);
    e = launch_copy2d(base + plan.off_c, b.ldc, a.c, a.ldc, a.m, a.n, b.ldc, sms, a.stream);
    if (e != cudaSuccess) return e;
  }
  if (plan.bias) {
    b.bias = base + plan.off_bias;
    e = launch_copy2d(base + plan.off_bias, 0, a.bias, 0, 1, a.n, round8(a.n), sms, a.stream);
    if (e != cudaSuccess) return e;
  }
  if (plan.d) {
    b.d = base + plan.off_d;
    b.ldd = round8(a.n);
  }
  if (plan.small) {
    e = launch_umma_swapab_gemm(b, nullptr);
  } else {
    const TileChoice tc = choose_tiles(a.m, a.n, a.k, sms);
    switch (tc.config) {
      case PersistentConfig::Pair256x256:
        e = launch_umma_pair_gemm(b);
        break;
      case PersistentConfig::Cta128x256:
        e = launch_umma_gemm(b, 256);
        break;
      case PersistentConfig::Cta128x128:
        e = launch_umma_gemm(b, 128);
        break;
      case PersistentConfig::Cta128x64:
        e = launch_umma_gemm(b, 64);
        break;
      case PersistentConfig::SplitK256x256:
        e = launch_umma_splitk_gemm(b, 256, 256, tc.splits);
        break;
      case PersistentConfig::SplitK128x256:
        e = launch_umma_splitk_gemm(b, 128, 256, tc.splits);
        break;
      case PersistentConfig::SplitK128x128:
        e = launch_umma_splitk_gemm(b, 128, 128, tc.splits);
        break;
    }
  }
  if (e != cudaSuccess) return e;
  if (plan.d) e = launch_copy2d(a.d, a.ldd, b.d, b.ldd, a.m, a.n, a.n, sms, a.stream);
  return e;
}

int read_and_clear_error_word(bool clear) {
  int value = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  if (cudaMemcpyFromSymbol(&value, g_device_error_word, sizeof(int)) != cudaSuccess) return -1;
  if (clear && value != 0) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_device_error_word, &zero, sizeof(int)) != cudaSuccess) return -1;
  }
  return value;
}

uint64_t launch_count() { return g_launches.load(std::memory_order_relaxed); }
void count_launches(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

// One thread waits on an mbarrier that nothing ever arrives on, with the same
// bounded wait the GEMM kernels use but a caller-chosen limit. The wait must
// give up, record kSelftestCode in the error word and let the kernel return.
constexpr int kSelftestCode = (15 << 4) | 15;

__global__ void selftest_bounded_wait_kernel(uint64_t timeout_ns, int* error_word) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  abort_flag = 0;
  fence_mbarrier_init();
  WaitCtx ctx{&abort_flag, error_word, timeout_ns};
  (void)mbar_wait(&bar, 0, ctx, kSelftestCode);
}

int selftest_bounded_wait(uint32_t timeout_us) {
  DeviceSlot* slot = current_slot();
  if (slot == nullptr || slot->info.error_word == nullptr) return -1;
  if (read_and_clear_error_word(true) < 0) return -1;
  selftest_bounded_wait_kernel<<<1, 32>>>(static_cast<uint64_t>(timeout_us) * 1000ull, slot->info.error_word);
  g_launches.fetch_add(1, std::memory_order_relaxed);
  if (cudaGetLastError() != cudaSuccess) return -1;
  return read_and_clear_error_word(true);
}

// ---------------------------------------------------------------- decode without allocation
//
// Some callers cannot allocate device memory at call time (inside an
// allocator or memory-pool callback, or in a process that reserves all device
// memory at start-up and allocates nothing afterwards). For them the stream-K
// decode kernel can run with its
// scratch -- tile counters and FP32 partial tiles -- in this fixed array
// instead of the per-stream workspace. The array is part of the library
// image: every device that loads the library holds it until exit.

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;  // 16 MiB
constexpr size_t kNoAllocCounterBytes = size_t(64) << 10;   // 8192 tile counters

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

struct NoAllocSlot {
  std::once_flag once;
  void* ptr = nullptr;  // device address of g_noalloc_scratch on this device
  cudaError_t err = cudaSuccess;
};
NoAllocSlot g_noalloc[kMaxDevices];

template <typename T, int MP, int STAGES, bool KM>
cudaError_t launch_swapab_sk_scratch_t(const LaunchArgs& a, DeviceSlot* slot, int config_bit,
                                       unsigned char* scratch) {
  using L = swapab_sk::Smem<MP, STAGES, kDecodeKsub>;
  CUtensorMap tw, tx;
  const bool bf16 = a.bf16;
  const bool w_ok =
      KM ? make_tma_2d(&tw, a.b, bf16, a.n, a.k, a.ldb, swapab_sk::kBlockN, swapab_sk::kBlockK, TmaSwizzle::B128)
         : make_tma_2d(&tw, a.b, bf16, a.k, a.n, a.ldb, swapab_sk::kBlockK, 64, TmaSwizzle::B128);
  if (!w_ok || !make_tma_2d(&tx, a.a, bf16, a.m, a.k, a.lda, MP, swapab_sk::kBlockK, TmaSwizzle::B128)) {
    return cudaErrorInvalidValue;
  }
  SwapAbSkParams p{};
  p.m = static_cast<int>(a.m);
  p.n = static_cast<int>(a.n);
  p.k = static_cast<int>(a.k);
  p.num_kb = static_cast<int>((a.k + kDecodeKBlock - 1) / kDecodeKBlock);
  p.tiles_n = static_cast<int>((a.n + swapab_sk::kBlockN - 1) / swapab_sk::kBlockN);
  p.total_units = static_cast<long long>(p.num_kb) * p.tiles_n;
  p.grid = static_cast<int>(std::min<long long>(p.total_units, slot->info.sm_count));
  p.alpha = a.alpha;
  p.beta = a.beta;
  p.c = a.c;
  p.ldc = a.ldc;
  p.d = a.d;
  p.ldd = a.ldd;
  p.bias = a.bias;
  p.epi_flags = (a.beta != 0.0f ? kEpiHasC : 0u) | (a.bias != nullptr ? kEpiHasBias : 0u);
  p.error_word = slot->info.error_word;
  p.counters = reinterpret_cast<unsigned long long*>(scratch);
  p.partials = reinterpret_cast<float*>(scratch + kNoAllocCounterBytes);
  p.epoch = 1;
  // The array keeps the previous call's counters: zero the ones this call uses.
  cudaError_t e = cudaMemsetAsync(p.counters, 0, size_t(p.tiles_n) * sizeof(unsigned long long), a.stream);
  if (e != cudaSuccess) return e;
  auto kernel = swapab_sk::gemm_kernel<T, MP, STAGES, kDecodeKsub, KM>;
  e = ensure_smem_attr(slot, config_bit, kernel, L::kDynamicBytes);
  if (e != cudaSuccess) return e;
  kernel<<<p.grid, swapab_sk::kThreads, L::kDynamicBytes, a.stream>>>(tw, tx, p);
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return cudaGetLastError();
}

template <bool KM>
cudaError_t launch_noalloc_km(const LaunchArgs& a, DeviceSlot* slot, unsigned char* scratch) {
  const int off = KM ? kCfgColMajorB : 0;
  if (a.m <= 16) {
    return a.bf16 ? launch_swapab_sk_scratch_t<__nv_bfloat16, 16, 6, KM>(a, slot, kCfgSkBf16M16 + off, scratch)
                  : launch_swapab_sk_scratch_t<half, 16, 6, KM>(a, slot, kCfgSkF16M16 + off, scratch);
  }
  if (a.m <= 32) {
    return a.bf16 ? launch_swapab_sk_scratch_t<__nv_bfloat16, 32, 5, KM>(a, slot, kCfgSkBf16M32 + off, scratch)
                  : launch_swapab_sk_scratch_t<half, 32, 5, KM>(a, slot, kCfgSkF16M32 + off, scratch);
  }
  return a.bf16 ? launch_swapab_sk_scratch_t<__nv_bfloat16, 64, 4, KM>(a, slot, kCfgSkBf16M64 + off, scratch)
                : launch_swapab_sk_scratch_t<half, 64, 4, KM>(a, slot, kCfgSkF16M64 + off, scratch);
}

}  // namespace

int gemm_decode_noalloc(const LaunchArgs& a) {
  constexpr int kSuccess = 0, kInvalidArgument = 1, kRuntimeError = 3;
  DeviceSlot* slot = current_slot();
  if (slot == nullptr) return kRuntimeError;
  if (slot->info.cc_major != 10 || slot->info.cc_minor != 0) return kInvalidArgument;
  if (a.m < 1 || a.m > 64 || a.n > INT32_MAX || a.k > INT32_MAX) return kInvalidArgument;
  if (!tma_compatible(a.a, a.lda) || !tma_compatible(a.b, a.ldb)) return kInvalidArgument;
  // Size check before any device work.
  const int mp = a.m <= 16 ? 16 : a.m <= 32 ? 32 : 64;
  const long long tiles_n = (a.n + swapab_sk::kBlockN - 1) / swapab_sk::kBlockN;
  const long long units = tiles_n * ((a.k + kDecodeKBlock - 1) / kDecodeKBlock);
  const long long grid = std::min<long long>(units, slot->info.sm_count);
  const size_t partial_bytes = size_t(2) * grid * mp * swapab_sk::kBlockN * sizeof(float);
  if (size_t(tiles_n) * sizeof(unsigned long long) > kNoAllocCounterBytes ||
      kNoAllocCounterBytes + partial_bytes > kNoAllocScratchBytes) {
    return kInvalidArgument;
  }
  // Set-up, once per device with that device current: the host-side name of a
  // __device__ array is not a device address, so look the address up.
  NoAllocSlot& ns = g_noalloc[slot->info.ordinal];
  std::call_once(ns.once, [&ns] {
    ns.err = cudaGetSymbolAddress(&ns.ptr, g_noalloc_scratch);
    if (ns.err == cudaSuccess && ns.ptr == nullptr) ns.err = cudaErrorInvalidSymbol;
  });
  if (ns.err != cudaSuccess) return kRuntimeError;
  auto* scratch = static_cast<unsigned char*>(ns.ptr);
  const cudaError_t e =
      a.b_col_major ? launch_noalloc_km<true>(a, slot, scratch) : launch_noalloc_km<false>(a, slot, scratch);
  return e == cudaSuccess ? kSuccess : kRuntimeError;
}

}  // namespace zcb
