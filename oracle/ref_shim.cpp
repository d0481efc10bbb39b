// TEST INFRASTRUCTURE ONLY. A flat C binding of the *reference* library
// (supercatking/zcutlass, built from its own src/*.cu by oracle/Makefile into
// oracle/_ref/libzcutlass_ref.so). Tests use it to run the reference's own
// GEMM (its WMMA kernels, the ones it dispatches to on compute capability 10.0)
// on the same inputs as ours; bench.py may time it as a comparator. Nothing in
// the product links this file.
//
// Binds: zcutlass::gemm(GemmDesc, A, B, C, D)    include/zcutlass/gemm/gemm.hpp:72-76
//        zcutlass::selected_kernel_name(GemmDesc) include/zcutlass/gemm/gemm.hpp:80
#include "zcutlass/gemm.hpp"

#include <cstdint>

namespace {

zcutlass::GemmDesc flat_desc(int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb,
                             int64_t ldc, int64_t ldd, int dtype, float alpha, float beta,
                             const void* bias, void* stream) {
  const auto t = static_cast<zcutlass::DType>(dtype);
  zcutlass::GemmDesc d{m, n, k, lda, ldb, ldc, ldd, t, t, t, t, alpha, beta, bias,
                       static_cast<cudaStream_t>(stream)};
  return d;
}

}  // namespace

extern "C" {

int zref_gemm(int64_t m, int64_t n, int64_t k, const void* A, int64_t lda, const void* B,
              int64_t ldb, const void* C, int64_t ldc, void* D, int64_t ldd, int dtype,
              float alpha, float beta, const void* bias, void* stream) {
  return static_cast<int>(zcutlass::gemm(
      flat_desc(m, n, k, lda, ldb, ldc, ldd, dtype, alpha, beta, bias, stream), A, B, C, D));
}

const char* zref_selected_kernel_name(int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb,
                                      int64_t ldc, int64_t ldd, int dtype, float alpha, float beta,
                                      const void* bias) {
  return zcutlass::selected_kernel_name(
      flat_desc(m, n, k, lda, ldb, ldc, ldd, dtype, alpha, beta, bias, nullptr));
}

}  // extern "C"
