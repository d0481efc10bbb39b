// extern "C" entry points declared in include/zcutlass_c.h. Each converts the
// flat C arguments into the C++ API types and forwards; no logic lives here.
#include "zcutlass_c.h"

#include "zcutlass/gemm.hpp"

#include "launchers.hpp"

namespace {

zcutlass::GemmDesc to_desc(const zcutlass_gemm_desc* d) {
  zcutlass::GemmDesc g{d->m,
                       d->n,
                       d->k,
                       d->lda,
                       d->ldb,
                       d->ldc,
                       d->ldd,
                       static_cast<zcutlass::DType>(d->a_type),
                       static_cast<zcutlass::DType>(d->b_type),
                       static_cast<zcutlass::DType>(d->c_type),
                       static_cast<zcutlass::DType>(d->d_type),
                       d->alpha,
                       d->beta,
                       d->bias,
                       static_cast<cudaStream_t>(d->stream),
                       static_cast<zcutlass::layout::LayoutKind>(d->a_layout),
                       static_cast<zcutlass::layout::LayoutKind>(d->b_layout),
                       static_cast<zcutlass::layout::LayoutKind>(d->c_layout),
                       static_cast<zcutlass::layout::LayoutKind>(d->d_layout)};
  return g;
}

}  // namespace

extern "C" {

int zcutlass_gemm(const zcutlass_gemm_desc* desc, const void* A, const void* B, const void* C,
                  void* D) {
  if (desc == nullptr) return ZCUTLASS_INVALID_ARGUMENT;
  return static_cast<int>(zcutlass::gemm(to_desc(desc), A, B, C, D));
}

int zcutlass_gemm_rowmajor(int64_t m, int64_t n, int64_t k, const void* A, int64_t lda,
                           const void* B, int64_t ldb, const void* C, int64_t ldc, void* D,
                           int64_t ldd, int32_t dtype, float alpha, float beta, const void* bias,
                           void* stream) {
  const zcutlass::DType t = static_cast<zcutlass::DType>(dtype);
  zcutlass::GemmDesc g{m, n, k, lda, ldb, ldc, ldd, t, t, t, t, alpha, beta, bias,
                       static_cast<cudaStream_t>(stream)};
  return static_cast<int>(zcutlass::gemm(g, A, B, C, D));
}

int zcutlass_gemm_gather_a(const zcutlass_gemm_desc* desc, const void* const* a_parts, int32_t parts,
                           const void* B, const void* C, void* D) {
  if (desc == nullptr) return ZCUTLASS_INVALID_ARGUMENT;
  return static_cast<int>(zcutlass::gemm_gather_a(to_desc(desc), a_parts, parts, B, C, D));
}

int zcutlass_can_implement(const zcutlass_gemm_desc* desc, const void* A, const void* B,
                           const void* C, const void* D) {
  if (desc == nullptr) return ZCUTLASS_INVALID_ARGUMENT;
  const zcutlass::GemmDesc g = to_desc(desc);
  zcutlass::gemm_api::GemmArguments args{};
  args.problem = {g.m, g.n, g.k};
  args.A = {A, g.a_type, g.a_layout, g.lda};
  args.B = {B, g.b_type, g.b_layout, g.ldb};
  args.C = {C, g.c_type, g.c_layout, g.ldc};
  args.D = {const_cast<void*>(D), g.d_type, g.d_layout, g.ldd};
  args.alpha = g.alpha;
  args.beta = g.beta;
  args.bias = g.bias;
  args.stream = g.stream;
  return static_cast<int>(zcutlass::can_implement(args));
}

size_t zcutlass_get_workspace_size(const zcutlass_gemm_desc*) {
  return zcutlass::get_workspace_size(zcutlass::gemm_api::GemmArguments{});
}

const char* zcutlass_selected_kernel_name(const zcutlass_gemm_desc* desc) {
  return desc ? zcutlass::selected_kernel_name(to_desc(desc)) : "none";
}
const char* zcutlass_selected_kernel_family(const zcutlass_gemm_desc* desc) {
  return desc ? zcutlass::selected_kernel_family(to_desc(desc)) : "none";
}
const char* zcutlass_selected_kernel_path(const zcutlass_gemm_desc* desc) {
  return desc ? zcutlass::selected_kernel_path(to_desc(desc)) : "none";
}
int zcutlass_selected_kernel_tile_m(const zcutlass_gemm_desc* desc) {
  return desc ? zcutlass::selected_kernel_tile_m(to_desc(desc)) : 0;
}
int zcutlass_selected_kernel_tile_n(const zcutlass_gemm_desc* desc) {
  return desc ? zcutlass::selected_kernel_tile_n(to_desc(desc)) : 0;
}
int zcutlass_selected_kernel_tile_k(const zcutlass_gemm_desc* desc) {
  return desc ? zcutlass::selected_kernel_tile_k(to_desc(desc)) : 0;
}
int zcutlass_selected_kernel_pipeline_stages(const zcutlass_gemm_desc* desc) {
  return desc ? zcutlass::selected_kernel_pipeline_stages(to_desc(desc)) : 0;
}
const char* zcutlass_selected_kernel_epilogue_kind(const zcutlass_gemm_desc* desc) {
  return desc ? zcutlass::selected_kernel_epilogue_kind(to_desc(desc)) : "none";
}
int zcutlass_registered_gemm_operation_count(void) {
  return zcutlass::registered_gemm_operation_count();
}

const char* zcutlass_status_to_string(int status) {
  return zcutlass::status_to_string(static_cast<zcutlass::Status>(status));
}
const char* zcutlass_dtype_name(int dtype) {
  return zcutlass::dtype_name(static_cast<zcutlass::DType>(dtype));
}
int zcutlass_dtype_bits(int dtype) { return zcutlass::dtype_bits(static_cast<zcutlass::DType>(dtype)); }
int zcutlass_version_major(void) { return zcutlass::version_major(); }
int zcutlass_version_minor(void) { return zcutlass::version_minor(); }
int zcutlass_version_patch(void) { return zcutlass::version_patch(); }

int zcutlass_device_error(int clear) { return zcb::read_and_clear_error_word(clear != 0); }

uint64_t zcutlass_gemm_kernel_launches(void) { return zcb::launch_count(); }

int zcutlass_selftest_bounded_wait(uint32_t timeout_us) { return zcb::selftest_bounded_wait(timeout_us); }

int zcutlass_nvls_allreduce(void* mc_ptr, int64_t nbytes, int32_t dtype, void* mc_flag, void* flag, int32_t rank,
                            int32_t world, void* stream) {
  if (dtype != ZCUTLASS_F16 && dtype != ZCUTLASS_BF16) return ZCUTLASS_NOT_SUPPORTED;
  const cudaError_t e = zcb::launch_nvls_allreduce(mc_ptr, nbytes, dtype == ZCUTLASS_BF16,
                                                   static_cast<uint32_t*>(mc_flag), static_cast<uint32_t*>(flag), rank,
                                                   world, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? ZCUTLASS_SUCCESS
                          : (e == cudaErrorInvalidValue ? ZCUTLASS_INVALID_ARGUMENT : ZCUTLASS_RUNTIME_ERROR);
}

int zcutlass_nvls_barrier(void* mc_flag, void* flag, int32_t world, void* stream) {
  const cudaError_t e = zcb::launch_nvls_barrier(static_cast<uint32_t*>(mc_flag), static_cast<uint32_t*>(flag), world,
                                                 static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? ZCUTLASS_SUCCESS
                          : (e == cudaErrorInvalidValue ? ZCUTLASS_INVALID_ARGUMENT : ZCUTLASS_RUNTIME_ERROR);
}

int zcutlass_nvls_reduce_scatter(void* mc_ptr, void* local_ptr, int64_t nbytes, int32_t dtype, void* mc_flag,
                                 void* flag, int32_t rank, int32_t world, void* stream) {
  if (dtype != ZCUTLASS_F16 && dtype != ZCUTLASS_BF16) return ZCUTLASS_NOT_SUPPORTED;
  const cudaError_t e = zcb::launch_nvls_reduce_scatter(mc_ptr, local_ptr, nbytes, dtype == ZCUTLASS_BF16,
                                                        static_cast<uint32_t*>(mc_flag), static_cast<uint32_t*>(flag),
                                                        rank, world, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? ZCUTLASS_SUCCESS
                          : (e == cudaErrorInvalidValue ? ZCUTLASS_INVALID_ARGUMENT : ZCUTLASS_RUNTIME_ERROR);
}

// For callers that may not allocate device memory at call time (see the
// header): same validation as zcutlass_gemm, then the stream-K decode kernel
// with its scratch in the library's fixed device array.
int zcutlass_gemm_decode_noalloc(int64_t m, int64_t n, int64_t k, const void* A, int64_t lda,
                                 const void* B, int64_t ldb, int32_t b_col_major, const void* C,
                                 int64_t ldc, void* D, int64_t ldd, int32_t dtype, float alpha,
                                 float beta, const void* bias, void* stream) {
  const zcutlass::DType t = static_cast<zcutlass::DType>(dtype);
  const zcutlass::layout::LayoutKind b_layout =
      b_col_major ? zcutlass::layout::LayoutKind::ColumnMajor : zcutlass::layout::LayoutKind::RowMajor;
  zcutlass::gemm_api::GemmArguments args{};
  args.problem = {m, n, k};
  args.A = {A, t, zcutlass::layout::LayoutKind::RowMajor, lda};
  args.B = {B, t, b_layout, ldb};
  args.C = {C, t, zcutlass::layout::LayoutKind::RowMajor, ldc};
  args.D = {D, t, zcutlass::layout::LayoutKind::RowMajor, ldd};
  args.alpha = alpha;
  args.beta = beta;
  args.bias = bias;
  args.stream = static_cast<cudaStream_t>(stream);
  const zcutlass::Status v = zcutlass::can_implement(args);
  if (v != zcutlass::Status::Success) return static_cast<int>(v);
  if (m == 0 || n == 0 || k == 0) return ZCUTLASS_SUCCESS;
  zcb::LaunchArgs la{};
  la.m = m;
  la.n = n;
  la.k = k;
  la.a = A;
  la.lda = lda;
  la.b = B;
  la.ldb = ldb;
  la.c = beta != 0.0f ? C : nullptr;
  la.ldc = ldc;
  la.d = D;
  la.ldd = ldd;
  la.bias = bias;
  la.alpha = alpha;
  la.beta = beta;
  la.bf16 = t == zcutlass::DType::BF16;
  la.b_col_major = b_col_major != 0;
  la.stream = static_cast<cudaStream_t>(stream);
  return zcb::gemm_decode_noalloc(la);
}

}  // extern "C"
