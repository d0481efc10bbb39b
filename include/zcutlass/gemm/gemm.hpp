// The GEMM entry points: D = alpha * A * B + beta * C + bias.
//
//   A: [M, K] row-major, leading dimension lda >= K
//   B: [K, N] row-major, leading dimension ldb >= N
//   C: [M, N] row-major, ldc >= N (read only when beta != 0; may be null otherwise)
//   D: [M, N] row-major, ldd >= N; columns N..ldd-1 are never written
//   bias: optional [N] vector of the same dtype, added after the alpha/beta blend
//   All pointers are caller-owned device memory; all dtypes must be equal (F16 or BF16).
//   Accumulation is FP32; the result is rounded to the storage type once.
//
// Interface mirrors supercatking/zcutlass include/zcutlass/gemm/gemm.hpp:14-89:
// GemmDesc keeps the same positional field order (callers brace-initialise it),
// and every function keeps its name, arguments and Status meaning. Work is
// enqueued asynchronously on desc.stream (nullptr = legacy default stream).
#pragma once

#include <cstddef>
#include <cstdint>

#include <cuda_runtime_api.h>

#include "zcutlass/layout/layout.hpp"
#include "zcutlass/numeric_types.hpp"
#include "zcutlass/status.hpp"

namespace zcutlass::gemm_api {

struct GemmCoord {
  int64_t m = 0;
  int64_t n = 0;
  int64_t k = 0;
};

struct TensorRef {
  const void* data = nullptr;
  DType dtype = DType::F16;
  layout::LayoutKind layout = layout::LayoutKind::RowMajor;
  int64_t ld = 0;
};

struct TensorRefMutable {
  void* data = nullptr;
  DType dtype = DType::F16;
  layout::LayoutKind layout = layout::LayoutKind::RowMajor;
  int64_t ld = 0;
};

struct GemmArguments {
  GemmCoord problem;
  TensorRef A;
  TensorRef B;
  TensorRef C;
  TensorRefMutable D;
  float alpha = 1.0f;
  float beta = 0.0f;
  const void* bias = nullptr;
  cudaStream_t stream = nullptr;
};

}  // namespace zcutlass::gemm_api

namespace zcutlass {

struct GemmDesc {
  int64_t m;
  int64_t n;
  int64_t k;
  int64_t lda;
  int64_t ldb;
  int64_t ldc;
  int64_t ldd;
  DType a_type;
  DType b_type;
  DType c_type;
  DType d_type;
  float alpha;
  float beta;
  const void* bias;
  cudaStream_t stream;
  layout::LayoutKind a_layout = layout::LayoutKind::RowMajor;
  layout::LayoutKind b_layout = layout::LayoutKind::RowMajor;
  layout::LayoutKind c_layout = layout::LayoutKind::RowMajor;
  layout::LayoutKind d_layout = layout::LayoutKind::RowMajor;
};

// Validates, selects a kernel from the manifest and enqueues it.
Status gemm(const GemmDesc& desc, const void* A, const void* B, const void* C, void* D);

Status gemm(const gemm_api::GemmArguments& args);

// Addition without a reference counterpart: the same GEMM with the rows of A
// gathered from `parts` buffers (1..8), e.g. the row shards of a sequence-
// parallel activation in peer-mapped memory of each tensor-parallel rank.
// Rows [i * M / parts, (i + 1) * M / parts) are read from a_parts[i], which
// points to a full [M, K] row-major matrix with leading dimension desc.lda
// (only its own rows are read). B must be column-major (a [N, K] weight).
// NotSupported unless M is a multiple of parts and every block of rows is a
// multiple of 128 (of 256 where the 256 x 256 two-CTA tiles are chosen), and
// every operand satisfies the tcgen05 kernels' alignment rules.
Status gemm_gather_a(const GemmDesc& desc, const void* const* a_parts, int parts, const void* B, const void* C,
                     void* D);
// Argument validation only (same contract as the reference: no kernel selection).
Status can_implement(const gemm_api::GemmArguments& args);
// Always 0: no kernel in this library needs a caller-provided workspace.
size_t get_workspace_size(const gemm_api::GemmArguments& args);

// Host-only selection telemetry: which operation gemm() would run for `desc`.
// These never launch anything; "none"/0 when validation fails or nothing matches.
const char* selected_kernel_name(const GemmDesc& desc);
const char* selected_kernel_family(const GemmDesc& desc);
const char* selected_kernel_path(const GemmDesc& desc);
int selected_kernel_tile_m(const GemmDesc& desc);
int selected_kernel_tile_n(const GemmDesc& desc);
int selected_kernel_tile_k(const GemmDesc& desc);
int selected_kernel_pipeline_stages(const GemmDesc& desc);
const char* selected_kernel_epilogue_kind(const GemmDesc& desc);
int registered_gemm_operation_count();

}  // namespace zcutlass
