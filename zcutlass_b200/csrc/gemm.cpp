// Host GEMM layer: validation, the built-in operation table, dispatch and the
// selection telemetry.
//
// Contract followed from supercatking/zcutlass src/gemm.cu:
//   validate_desc      gemm.cu:256-293  (same checks, same order, same codes)
//   make_arguments     gemm.cu:462-478
//   classify family    gemm.cu:480-496  (kept verbatim in meaning for telemetry)
//   gemm()             gemm.cu:609-629  (zero-size -> Success without writes)
//   selected_kernel_*  gemm.cu:631-688  (host-only, dummy non-null pointers)
//   can_implement / get_workspace_size / version  gemm.cu:695-756
// The operation table itself is new: four sm_100a kernel families plus a
// predicated CUDA-core kernel for layouts TMA cannot express.
#include "zcutlass/gemm.hpp"

#include <climits>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "launchers.hpp"
#include "tma_desc.hpp"

namespace zcutlass {
namespace {

using gemm_api::EpilogueKind;
using gemm_api::GemmArguments;
using gemm_api::GemmOperation;
using gemm_api::GemmOperationDescription;
using gemm_api::GemmPreference;
using gemm_api::ShapeFamily;

Status validate_desc(const GemmDesc& desc, const void* A, const void* B, const void* C,
                     const void* D) {
  if (desc.m < 0 || desc.n < 0 || desc.k < 0) return Status::InvalidArgument;
  if (desc.m == 0 || desc.n == 0 || desc.k == 0) return Status::Success;
  if (A == nullptr || B == nullptr || D == nullptr) return Status::InvalidArgument;
  if (desc.beta != 0.0f && C == nullptr) return Status::InvalidArgument;
  // Column-major B (an additive extension: B[k][n] at n*ldb + k) needs ldb >= K.
  const int64_t ldb_min = desc.b_layout == layout::LayoutKind::ColumnMajor ? desc.k : desc.n;
  if (desc.lda < desc.k || desc.ldb < ldb_min || desc.ldd < desc.n) return Status::InvalidArgument;
  if (desc.beta != 0.0f && desc.ldc < desc.n) return Status::InvalidArgument;
  if (desc.a_type != desc.b_type || desc.a_type != desc.c_type || desc.a_type != desc.d_type)
    return Status::NotSupported;
  if (!is_supported_gemm_storage_dtype(desc.a_type)) return Status::NotSupported;
  if (desc.a_layout != layout::LayoutKind::RowMajor ||
      desc.c_layout != layout::LayoutKind::RowMajor ||
      desc.d_layout != layout::LayoutKind::RowMajor)
    return Status::NotSupported;
  return Status::Success;
}

GemmArguments make_arguments(const GemmDesc& desc, const void* A, const void* B, const void* C,
                             void* D) {
  GemmArguments args{};
  args.problem = {desc.m, desc.n, desc.k};
  args.A = {A, desc.a_type, desc.a_layout, desc.lda};
  args.B = {B, desc.b_type, desc.b_layout, desc.ldb};
  args.C = {C, desc.c_type, desc.c_layout, desc.ldc};
  args.D = {D, desc.d_type, desc.d_layout, desc.ldd};
  args.alpha = desc.alpha;
  args.beta = desc.beta;
  args.bias = desc.bias;
  args.stream = desc.stream;
  return args;
}

GemmDesc desc_from_arguments(const GemmArguments& args) {
  GemmDesc d{args.problem.m, args.problem.n, args.problem.k, args.A.ld,   args.B.ld,
             args.C.ld,      args.D.ld,      args.A.dtype,   args.B.dtype, args.C.dtype,
             args.D.dtype,   args.alpha,     args.beta,      args.bias,    args.stream,
             args.A.layout,  args.B.layout,  args.C.layout,  args.D.layout};
  return d;
}

// Reference shape families (telemetry only; dispatch below uses its own rules).
ShapeFamily classify_shape_family(const GemmArguments& args) {
  const int64_t m = args.problem.m, n = args.problem.n, k = args.problem.k;
  if (args.beta != 0.0f || args.A.ld != k || args.B.ld != n || args.C.ld != n || args.D.ld != n)
    return ShapeFamily::Fallback;
  if (m <= 16 && n >= 1024 && k >= 1024) return ShapeFamily::Decode;
  if (m >= 32 && m <= 256 && n >= 1024 && k >= 1024) return ShapeFamily::Prefill;
  if (m >= 512 && n >= 512 && k >= 512) return ShapeFamily::Large;
  return ShapeFamily::Fallback;
}

bool env_truthy(const char* name) {
  const char* v = std::getenv(name);
  return v != nullptr && v[0] != '\0' && std::strcmp(v, "0") != 0 && std::strcmp(v, "false") != 0 &&
         std::strcmp(v, "FALSE") != 0;
}

// ZCUTLASS_EXPERIMENTAL_KERNELS / ZCUTLASS_EXPERIMENTAL_KERNEL keep their
// reference meaning (gemm.cu:322-331) for operations marked experimental.
bool experimental_allowed(const char* name) {
  if (!env_truthy("ZCUTLASS_EXPERIMENTAL_KERNELS")) return false;
  const char* filter = std::getenv("ZCUTLASS_EXPERIMENTAL_KERNEL");
  return filter == nullptr || filter[0] == '\0' || std::strstr(name, filter) != nullptr;
}

// ZCUTLASS_FORCE_KERNEL=<substring>: only operations whose name contains the
// substring are eligible (used by tests to pin one kernel family).
// A forced operation skips the shape heuristics (tile-width choice, M buckets)
// but keeps every hard requirement of its kernel.
bool force_filter_active() {
  const char* filter = std::getenv("ZCUTLASS_FORCE_KERNEL");
  return filter != nullptr && filter[0] != '\0';
}

bool force_filter_allows(const char* name) {
  const char* filter = std::getenv("ZCUTLASS_FORCE_KERNEL");
  return filter == nullptr || filter[0] == '\0' || std::strstr(name, filter) != nullptr;
}

// Device facts used by selection. With no CUDA device visible (host-only
// tooling, CPU test runners) selection answers for a B200: cc 10.0, 148 SMs.
struct SelectDevice {
  int cc_major, cc_minor, sm_count;
};

SelectDevice select_device() {
  const zcb::DeviceInfo* info = zcb::current_device_info();
  if (info == nullptr) return {10, 0, 148};
  return {info->cc_major, info->cc_minor, info->sm_count > 0 ? info->sm_count : 148};
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

enum class Kind { UmmaPair, UmmaPersistent, UmmaSplitK, UmmaSwapAb, UmmaSwapAbStreamK, Repack, Generic };

class Sm100Operation final : public GemmOperation {
 public:
  Sm100Operation(const char* name, DType type, Kind kind, int tile_m, int tile_n, int tile_k,
                 int stages, ShapeFamily family, EpilogueKind epilogue)
      : kind_(kind), bf16_(type == DType::BF16) {
    desc_.name = name;
    desc_.a_type = desc_.b_type = desc_.c_type = desc_.d_type = type;
    desc_.accum_type = DType::F32;
    desc_.min_arch = kind == Kind::Generic ? arch::ArchKind::Sm80 : arch::ArchKind::Sm100;
    desc_.op_class = kind == Kind::Generic ? arch::OpClass::TensorOp : arch::OpClass::Tcgen05;
    desc_.tile_m = tile_m;
    desc_.tile_n = tile_n;
    desc_.tile_k = tile_k;
    desc_.family = family;
    desc_.requires_aligned_tiles = kind != Kind::Generic && kind != Kind::Repack;
    desc_.supports_beta = true;
    desc_.supports_bias = true;
    // Stream-K decode: correct and deterministic, but its partial-tile fixup
    // makes it slower than cluster split-K on every measured decode shape, so
    // it runs only when experimental kernels are enabled (or it is forced).
    desc_.experimental = kind == Kind::UmmaSwapAbStreamK;
    desc_.pipeline_stages = stages;
    desc_.epilogue = epilogue;
  }

  const GemmOperationDescription& description() const override { return desc_; }

  bool can_implement(const GemmArguments& args, const GemmPreference&) const override {
    const DType t = desc_.a_type;
    if (args.A.dtype != t || args.B.dtype != t || args.C.dtype != t || args.D.dtype != t) return false;
    if (args.A.layout != layout::LayoutKind::RowMajor || args.C.layout != layout::LayoutKind::RowMajor ||
        args.D.layout != layout::LayoutKind::RowMajor)
      return false;
    if (!force_filter_allows(desc_.name)) return false;
    if (desc_.experimental && !force_filter_active() && !experimental_allowed(desc_.name)) return false;
    const int64_t m = args.problem.m, n = args.problem.n, k = args.problem.k;
    if (kind_ == Kind::Generic) return true;
    if (kind_ == Kind::Repack) return can_repack(args, m, n, k);

    // tcgen05 kernels: sm_100a code runs on compute capability 10.0 exactly.
    const SelectDevice dev = select_device();
    if (dev.cc_major != 10 || dev.cc_minor != 0) return false;
    if (m > INT_MAX || n > INT_MAX || k > INT_MAX) return false;
    if (!zcb::tma_compatible(args.A.data, args.A.ld) || !zcb::tma_compatible(args.B.data, args.B.ld))
      return false;

    const bool forced = force_filter_active();
    if (kind_ == Kind::UmmaSwapAb || kind_ == Kind::UmmaSwapAbStreamK) {
      const int mp = desc_.tile_m;
      if (m > mp) return false;
      // The stream-K workspace is allocated on a stream's first use, which a
      // CUDA graph capture forbids: while capturing, only a stream whose
      // workspace already fits qualifies (split-K takes the call otherwise).
      if (kind_ == Kind::UmmaSwapAbStreamK && !zcb::swapab_sk_ready_for_stream(m, n, k, args.stream)) return false;
      if (forced) return true;
      if (mp > 16 && m <= mp / 2) return false;
      if (n < 128 || k < 128) return false;
      // Split-K takes every bucketed shape; an enabled stream-K operation
      // (listed first) takes the shapes where split-K would idle SMs.
      return kind_ == Kind::UmmaSwapAb || zcb::swapab_prefer_streamk(n, k, dev.sm_count);
    }
    // Persistent and split-K kernels: D goes out through TMA or aligned vector
    // stores; C and bias are read with vector loads.
    if (!zcb::tma_compatible(args.D.data, args.D.ld)) return false;
    if (args.beta != 0.0f && (!aligned16(args.C.data) || (args.C.ld & 7) != 0)) return false;
    if (args.bias != nullptr && !aligned16(args.bias)) return false;
    if (forced) return true;
    using PC = zcb::PersistentConfig;
    const PC want = zcb::choose_tiles(m, n, k, dev.sm_count).config;
    switch (kind_) {
      case Kind::UmmaPair:
        return want == PC::Pair256x256;
      case Kind::UmmaSplitK:
        return want == (desc_.tile_m == 256   ? PC::SplitK256x256
                        : desc_.tile_n == 256 ? PC::SplitK128x256
                                              : PC::SplitK128x128);
      default:
        return want == (desc_.tile_n == 256   ? PC::Cta128x256
                        : desc_.tile_n == 128 ? PC::Cta128x128
                                              : PC::Cta128x64);
    }
  }

  // Packed-operand path: shapes large enough that one copy pass pays off
  // (N, K >= 128, M*N*K >= 2^22) whose layout keeps the tcgen05 kernels out.
  bool can_repack(const GemmArguments& args, int64_t m, int64_t n, int64_t k) const {
    const SelectDevice dev = select_device();
    if (dev.cc_major != 10 || dev.cc_minor != 0) return false;
    if (m > INT_MAX || n > INT_MAX || k > INT_MAX) return false;
    const zcb::LaunchArgs la = launch_args(args);
    if (!force_filter_active()) {
      if (n < 128 || k < 128 || m * n * k < (int64_t(1) << 22)) return false;
      const bool small = m <= 64;
      const bool regular = zcb::tma_compatible(la.a, la.lda) && zcb::tma_compatible(la.b, la.ldb) &&
                           (small || (zcb::tma_compatible(la.d, la.ldd) &&
                                      (la.c == nullptr || (aligned16(la.c) && (la.ldc & 7) == 0)) &&
                                      (la.bias == nullptr || aligned16(la.bias))));
      if (regular) return false;
    }
    return zcb::repack_ready_for_stream(zcb::repack_scratch_bytes(la), args.stream);
  }

  zcb::LaunchArgs launch_args(const GemmArguments& args) const {
    zcb::LaunchArgs la{};
    la.m = args.problem.m;
    la.n = args.problem.n;
    la.k = args.problem.k;
    la.a = args.A.data;
    la.lda = args.A.ld;
    la.b = args.B.data;
    la.ldb = args.B.ld;
    la.c = args.beta != 0.0f ? args.C.data : nullptr;
    la.ldc = args.C.ld;
    la.d = args.D.data;
    la.ldd = args.D.ld;
    la.bias = args.bias;
    la.alpha = args.alpha;
    la.beta = args.beta;
    la.bf16 = bf16_;
    la.b_col_major = args.B.layout == layout::LayoutKind::ColumnMajor;
    la.stream = args.stream;
    return la;
  }

  Status run(const GemmArguments& args, const GemmPreference&) const override {
    const zcb::LaunchArgs la = launch_args(args);
    cudaError_t e = cudaSuccess;
    switch (kind_) {
      case Kind::UmmaPair:
        e = zcb::launch_umma_pair_gemm(la);
        break;
      case Kind::UmmaPersistent:
        e = zcb::launch_umma_gemm(la, desc_.tile_n);
        break;
      case Kind::UmmaSplitK: {
        using PC = zcb::PersistentConfig;
        const SelectDevice dev = select_device();
        const zcb::TileChoice tc = zcb::choose_tiles(la.m, la.n, la.k, dev.sm_count);
        const PC mine = desc_.tile_m == 256 ? PC::SplitK256x256 : desc_.tile_n == 256 ? PC::SplitK128x256
                                                                                      : PC::SplitK128x128;
        const int splits = tc.config == mine ? tc.splits
                                             : zcb::splitk_default_splits(la.m, la.n, la.k, desc_.tile_m,
                                                                          desc_.tile_n, dev.sm_count);
        e = zcb::launch_umma_splitk_gemm(la, desc_.tile_m, desc_.tile_n, splits);
        break;
      }
      case Kind::UmmaSwapAbStreamK:
        e = zcb::launch_umma_swapab_sk_gemm(la);
        break;
      case Kind::UmmaSwapAb:
        e = zcb::launch_umma_swapab_gemm(la, nullptr);
        break;
      case Kind::Repack:
        e = zcb::launch_repack_gemm(la);
        break;
      case Kind::Generic:
        e = zcb::launch_generic_gemm(la);
        break;
    }
    return e == cudaSuccess ? Status::Success : Status::RuntimeError;
  }

 private:
  GemmOperationDescription desc_;
  Kind kind_;
  bool bf16_;
};

std::once_flag g_register_once;

void register_builtin_operations() {
  using K = Kind;
  using F = ShapeFamily;
  using E = EpilogueKind;
  // First match wins: small-M swap-AB buckets, then the cluster split-K and
  // persistent kernels (split-K 256x256 / 128x256 / 128x128, CTA-pair 256x256, or
  // one-CTA 128x256 / 128x128 tiles, whichever the cost model in
  // choose_tiles picks), then the same kernels on packed copies of operands
  // TMA cannot describe, then the predicated CUDA-core kernel that accepts
  // any layout (small problems, or a capture without scratch).
  static const Sm100Operation ops[] = {
      {"zcutlass_sm100_tcgen05_bf16_16x128x64_swapab_streamk", DType::BF16, K::UmmaSwapAbStreamK, 16, 128, 64, 12, F::Decode, E::RegisterLinear},
      {"zcutlass_sm100_tcgen05_f16_16x128x64_swapab_streamk", DType::F16, K::UmmaSwapAbStreamK, 16, 128, 64, 12, F::Decode, E::RegisterLinear},
      {"zcutlass_sm100_tcgen05_bf16_32x128x64_swapab_streamk", DType::BF16, K::UmmaSwapAbStreamK, 32, 128, 64, 11, F::Decode, E::RegisterLinear},
      {"zcutlass_sm100_tcgen05_f16_32x128x64_swapab_streamk", DType::F16, K::UmmaSwapAbStreamK, 32, 128, 64, 11, F::Decode, E::RegisterLinear},
      {"zcutlass_sm100_tcgen05_bf16_64x128x64_swapab_streamk", DType::BF16, K::UmmaSwapAbStreamK, 64, 128, 64, 9, F::Prefill, E::RegisterLinear},
      {"zcutlass_sm100_tcgen05_f16_64x128x64_swapab_streamk", DType::F16, K::UmmaSwapAbStreamK, 64, 128, 64, 9, F::Prefill, E::RegisterLinear},
      {"zcutlass_sm100_tcgen05_bf16_16x128x64_swapab_splitk", DType::BF16, K::UmmaSwapAb, 16, 128, 64, 10, F::Decode, E::RegisterLinear},
      {"zcutlass_sm100_tcgen05_f16_16x128x64_swapab_splitk", DType::F16, K::UmmaSwapAb, 16, 128, 64, 10, F::Decode, E::RegisterLinear},
      {"zcutlass_sm100_tcgen05_bf16_32x128x64_swapab_splitk", DType::BF16, K::UmmaSwapAb, 32, 128, 64, 9, F::Decode, E::RegisterLinear},
      {"zcutlass_sm100_tcgen05_f16_32x128x64_swapab_splitk", DType::F16, K::UmmaSwapAb, 32, 128, 64, 9, F::Decode, E::RegisterLinear},
      {"zcutlass_sm100_tcgen05_bf16_64x128x64_swapab_splitk", DType::BF16, K::UmmaSwapAb, 64, 128, 64, 7, F::Prefill, E::RegisterLinear},
      {"zcutlass_sm100_tcgen05_f16_64x128x64_swapab_splitk", DType::F16, K::UmmaSwapAb, 64, 128, 64, 7, F::Prefill, E::RegisterLinear},
      {"zcutlass_sm100_tcgen05_bf16_256x256x64_splitk_cluster", DType::BF16, K::UmmaSplitK, 256, 256, 64, 3, F::Prefill, E::RegisterLinear},
      {"zcutlass_sm100_tcgen05_f16_256x256x64_splitk_cluster", DType::F16, K::UmmaSplitK, 256, 256, 64, 3, F::Prefill, E::RegisterLinear},
      {"zcutlass_sm100_tcgen05_bf16_128x256x64_splitk_cluster", DType::BF16, K::UmmaSplitK, 128, 256, 64, 4, F::Prefill, E::RegisterLinear},
      {"zcutlass_sm100_tcgen05_f16_128x256x64_splitk_cluster", DType::F16, K::UmmaSplitK, 128, 256, 64, 4, F::Prefill, E::RegisterLinear},
      {"zcutlass_sm100_tcgen05_bf16_128x128x64_splitk_cluster", DType::BF16, K::UmmaSplitK, 128, 128, 64, 3, F::Prefill, E::RegisterLinear},
      {"zcutlass_sm100_tcgen05_f16_128x128x64_splitk_cluster", DType::F16, K::UmmaSplitK, 128, 128, 64, 3, F::Prefill, E::RegisterLinear},
      {"zcutlass_sm100_tcgen05_bf16_256x256x64_2cta_persistent", DType::BF16, K::UmmaPair, 256, 256, 64, 3, F::Large, E::TmemRegisterTma},
      {"zcutlass_sm100_tcgen05_f16_256x256x64_2cta_persistent", DType::F16, K::UmmaPair, 256, 256, 64, 3, F::Large, E::TmemRegisterTma},
      {"zcutlass_sm100_tcgen05_bf16_128x256x64_ws_persistent", DType::BF16, K::UmmaPersistent, 128, 256, 64, 4, F::Large, E::TmemRegisterTma},
      {"zcutlass_sm100_tcgen05_f16_128x256x64_ws_persistent", DType::F16, K::UmmaPersistent, 128, 256, 64, 4, F::Large, E::TmemRegisterTma},
      {"zcutlass_sm100_tcgen05_bf16_128x128x64_ws_persistent", DType::BF16, K::UmmaPersistent, 128, 128, 64, 3, F::Prefill, E::TmemRegisterTma},
      {"zcutlass_sm100_tcgen05_f16_128x128x64_ws_persistent", DType::F16, K::UmmaPersistent, 128, 128, 64, 3, F::Prefill, E::TmemRegisterTma},
      {"zcutlass_sm100_tcgen05_bf16_128x64x64_ws_persistent", DType::BF16, K::UmmaPersistent, 128, 64, 64, 4, F::Prefill, E::TmemRegisterTma},
      {"zcutlass_sm100_tcgen05_f16_128x64x64_ws_persistent", DType::F16, K::UmmaPersistent, 128, 64, 64, 4, F::Prefill, E::TmemRegisterTma},
      {"zcutlass_sm100_tcgen05_bf16_repack_generic", DType::BF16, K::Repack, 128, 128, 64, 4, F::Fallback, E::RegisterLinear},
      {"zcutlass_sm100_tcgen05_f16_repack_generic", DType::F16, K::Repack, 128, 128, 64, 4, F::Fallback, E::RegisterLinear},
      {"zcutlass_sm100_mma_bf16_128x128x32_generic", DType::BF16, K::Generic, 128, 128, 32, 2, F::Fallback, E::RegisterLinear},
      {"zcutlass_sm100_mma_f16_128x128x32_generic", DType::F16, K::Generic, 128, 128, 32, 2, F::Fallback, E::RegisterLinear},
  };
  auto& manifest = gemm_api::global_manifest();
  for (const auto& op : ops) manifest.append(&op);
}

void ensure_registered() { std::call_once(g_register_once, register_builtin_operations); }

const void* const kDummy = reinterpret_cast<const void*>(uintptr_t(256));

// Telemetry answers for the descriptor's shape, types and layouts only: the
// selection runs as for a call outside any stream capture, and never passes
// desc.stream to the CUDA runtime (a descriptor may outlive its stream).
const GemmOperationDescription* select_description(const GemmDesc& desc) {
  ensure_registered();
  GemmArguments args = make_arguments(desc, kDummy, kDummy, desc.beta != 0.0f ? kDummy : nullptr,
                                      const_cast<void*>(kDummy));
  args.stream = nullptr;
  const GemmOperation* op = gemm_api::global_manifest().find_best(args, {});
  return op != nullptr ? &op->description() : nullptr;
}

bool telemetry_valid(const GemmDesc& desc) {
  return validate_desc(desc, kDummy, kDummy, desc.beta != 0.0f ? kDummy : nullptr, kDummy) ==
         Status::Success;
}

}  // namespace

namespace gemm_api {
void initialize_builtin_operations() { ensure_registered(); }
}  // namespace gemm_api

Status gemm(const GemmDesc& desc, const void* A, const void* B, const void* C, void* D) {
  const Status validation = validate_desc(desc, A, B, C, D);
  if (validation != Status::Success) return validation;
  if (desc.m == 0 || desc.n == 0 || desc.k == 0) return Status::Success;
  ensure_registered();
  const GemmArguments args = make_arguments(desc, A, B, C, D);
  const GemmOperation* op = gemm_api::global_manifest().find_best(args, {});
  if (op == nullptr) return Status::NotSupported;
  return op->run(args, {});
}

Status gemm_gather_a(const GemmDesc& desc, const void* const* a_parts, int parts, const void* B, const void* C,
                     void* D) {
  if (a_parts == nullptr || parts < 1 || parts > zcb::kMaxAParts) return Status::InvalidArgument;
  const Status validation = validate_desc(desc, a_parts[0], B, C, D);
  if (validation != Status::Success) return validation;
  if (desc.m == 0 || desc.n == 0 || desc.k == 0) return Status::Success;
  for (int i = 0; i < parts; ++i)
    if (a_parts[i] == nullptr) return Status::InvalidArgument;
  // Served by the persistent tcgen05 kernels only: TMA-describable operands,
  // a [N, K] weight, and row blocks that never split a tile.
  if (desc.b_layout != layout::LayoutKind::ColumnMajor) return Status::NotSupported;
  const SelectDevice dev = select_device();
  if (dev.cc_major != 10 || dev.cc_minor != 0) return Status::NotSupported;
  if (desc.m > INT_MAX || desc.n > INT_MAX || desc.k > INT_MAX || desc.m % parts != 0) return Status::NotSupported;
  for (int i = 0; i < parts; ++i)
    if (!zcb::tma_compatible(a_parts[i], desc.lda)) return Status::NotSupported;
  if (!zcb::tma_compatible(B, desc.ldb) || !zcb::tma_compatible(D, desc.ldd)) return Status::NotSupported;
  if (desc.beta != 0.0f && (!aligned16(C) || (desc.ldc & 7) != 0)) return Status::NotSupported;
  if (desc.bias != nullptr && !aligned16(desc.bias)) return Status::NotSupported;
  const int64_t rows_per_part = desc.m / parts;
  const zcb::PersistentConfig want = zcb::choose_persistent(desc.m, desc.n, dev.sm_count);
  const bool pair = want == zcb::PersistentConfig::Pair256x256 && rows_per_part % 256 == 0;
  if (!pair && rows_per_part % 128 != 0) return Status::NotSupported;

  zcb::LaunchArgs la{};
  la.m = desc.m;
  la.n = desc.n;
  la.k = desc.k;
  la.a = a_parts[0];
  la.lda = desc.lda;
  la.b = B;
  la.ldb = desc.ldb;
  la.c = desc.beta != 0.0f ? C : nullptr;
  la.ldc = desc.ldc;
  la.d = D;
  la.ldd = desc.ldd;
  la.bias = desc.bias;
  la.alpha = desc.alpha;
  la.beta = desc.beta;
  la.bf16 = desc.a_type == DType::BF16;
  la.b_col_major = true;
  la.stream = desc.stream;
  la.a_parts = a_parts;
  la.a_nparts = parts;
  la.a_rows_per_part = rows_per_part;
  const cudaError_t e = pair ? zcb::launch_umma_pair_gemm(la)
                             : zcb::launch_umma_gemm(la, want == zcb::PersistentConfig::Cta128x128 ? 128 : 256);
  if (e == cudaErrorInvalidValue) return Status::NotSupported;
  return e == cudaSuccess ? Status::Success : Status::RuntimeError;
}

Status gemm(const gemm_api::GemmArguments& args) {
  return gemm(desc_from_arguments(args), args.A.data, args.B.data, args.C.data, args.D.data);
}

Status can_implement(const gemm_api::GemmArguments& args) {
  return validate_desc(desc_from_arguments(args), args.A.data, args.B.data, args.C.data, args.D.data);
}

size_t get_workspace_size(const gemm_api::GemmArguments&) { return 0; }

const char* selected_kernel_name(const GemmDesc& desc) {
  if (!telemetry_valid(desc)) return "none";
  const auto* d = select_description(desc);
  return d != nullptr ? d->name : "none";
}

const char* selected_kernel_family(const GemmDesc& desc) {
  if (!telemetry_valid(desc)) return "none";
  const GemmArguments args = make_arguments(desc, kDummy, kDummy, desc.beta != 0.0f ? kDummy : nullptr,
                                            const_cast<void*>(kDummy));
  return gemm_api::shape_family_name(classify_shape_family(args));
}

const char* selected_kernel_path(const GemmDesc& desc) {
  const auto* d = select_description(desc);
  if (d == nullptr) return "none";
  if (d->experimental) return d->requires_aligned_tiles ? "experimental_fast" : "experimental_fallback";
  return d->requires_aligned_tiles ? "fast" : "fallback";
}

int selected_kernel_tile_m(const GemmDesc& desc) {
  const auto* d = select_description(desc);
  return d != nullptr ? d->tile_m : 0;
}

int selected_kernel_tile_n(const GemmDesc& desc) {
  const auto* d = select_description(desc);
  return d != nullptr ? d->tile_n : 0;
}

int selected_kernel_tile_k(const GemmDesc& desc) {
  const auto* d = select_description(desc);
  return d != nullptr ? d->tile_k : 0;
}

int selected_kernel_pipeline_stages(const GemmDesc& desc) {
  const auto* d = select_description(desc);
  return d != nullptr ? d->pipeline_stages : 0;
}

const char* selected_kernel_epilogue_kind(const GemmDesc& desc) {
  const auto* d = select_description(desc);
  return d != nullptr ? gemm_api::epilogue_kind_name(d->epilogue) : "none";
}

int registered_gemm_operation_count() {
  ensure_registered();
  return gemm_api::global_manifest().size();
}

int version_major() { return 0; }
int version_minor() { return 2; }
int version_patch() { return 0; }

}  // namespace zcutlass
