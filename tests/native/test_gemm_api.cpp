// Native C++ test of the zcutlass C++ API (include/zcutlass/gemm.hpp), the
// boundary C++ callers compile against. Structured like the reference's own
// test program (supercatking/zcutlass tests/test_gemm.cu:737-791): numeric
// cases over the same shapes (ragged sizes, padded leading dimensions,
// alpha/beta/bias), zero-size problems (test_gemm.cu:439-473), invalid
// arguments (:475-567) and selection telemetry (:569-735). Each numeric case
// runs through zcutlass::gemm(GemmDesc, ...) and its twin through
// zcutlass::gemm(GemmArguments), and is checked against the CPU oracle
// (oracle/gemm_oracle.cpp, linked as liboracle.so; test infrastructure) under
// the same bounds as the Python suite: the reference test's absolute
// tolerance, relative Frobenius error, and |out - ref| <= 4 ulp * (1 + |ref|).
// Padding columns of D must keep their sentinel value.
//
// Exit status 0 when every check passes; one line per failure otherwise.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "zcutlass/gemm.hpp"

extern "C" {
void oracle_make_tensor(int64_t rows, int64_t cols, int64_t ld, int seed, int dtype, uint16_t* out);
void oracle_gemm(int64_t m, int64_t n, int64_t k, const uint16_t* A, int64_t lda, const uint16_t* B, int64_t ldb,
                 const uint16_t* C, int64_t ldc, const uint16_t* bias, float alpha, float beta, int dtype,
                 int threads, float* out);
float oracle_bits_to_float(uint16_t v, int dtype);
uint16_t oracle_float_to_bits(float v, int dtype);
}

namespace {

using zcutlass::DType;
using zcutlass::GemmDesc;
using zcutlass::Status;
using zcutlass::layout::LayoutKind;

int g_failures = 0;
int g_checks = 0;

void fail(const std::string& what) {
  ++g_failures;
  std::printf("FAIL %s\n", what.c_str());
}

void expect(bool ok, const std::string& what) {
  ++g_checks;
  if (!ok) fail(what);
}

template <typename T>
struct DeviceBuffer {
  T* ptr = nullptr;
  explicit DeviceBuffer(size_t count) {
    if (count > 0 && cudaMalloc(&ptr, count * sizeof(T)) != cudaSuccess) ptr = nullptr;
  }
  ~DeviceBuffer() {
    if (ptr != nullptr) cudaFree(ptr);
  }
  DeviceBuffer(const DeviceBuffer&) = delete;
  DeviceBuffer& operator=(const DeviceBuffer&) = delete;
};

struct Case {
  const char* name;
  DType dtype;
  int64_t m, n, k;
  float alpha, beta;
  bool bias;
  int pad_a, pad_b, pad_c, pad_d;
};

double ulp_at_one(DType t) { return t == DType::F16 ? std::ldexp(1.0, -10) : std::ldexp(1.0, -7); }
double ref_abs_tol(DType t) { return t == DType::F16 ? 0.16 : 0.55; }
double rel_fro_tol(DType t) { return t == DType::F16 ? 1e-3 : 5e-3; }

// Runs one case through both C++ entry points and checks both results.
void run_case(const Case& c) {
  const int dt = static_cast<int>(c.dtype);
  const int64_t lda = c.k + c.pad_a, ldb = c.n + c.pad_b, ldc = c.n + c.pad_c, ldd = c.n + c.pad_d;
  std::vector<uint16_t> a(c.m * lda), b(c.k * ldb), cm(c.m * ldc), bias(c.n);
  oracle_make_tensor(c.m, c.k, lda, 17, dt, a.data());
  oracle_make_tensor(c.k, c.n, ldb, 29, dt, b.data());
  oracle_make_tensor(c.m, c.n, ldc, 41, dt, cm.data());
  oracle_make_tensor(1, c.n, c.n, 53, dt, bias.data());
  std::vector<float> ref(c.m * c.n);
  const unsigned hw = std::thread::hardware_concurrency();
  oracle_gemm(c.m, c.n, c.k, a.data(), lda, b.data(), ldb, cm.data(), ldc, c.bias ? bias.data() : nullptr, c.alpha,
              c.beta, dt, hw > 0 ? static_cast<int>(hw) : 1, ref.data());

  DeviceBuffer<uint16_t> da(a.size()), db(b.size()), dc(cm.size()), dbias(bias.size()), dd(c.m * ldd);
  if (da.ptr == nullptr || db.ptr == nullptr || dc.ptr == nullptr || dbias.ptr == nullptr || dd.ptr == nullptr) {
    fail(std::string(c.name) + ": cudaMalloc");
    return;
  }
  cudaMemcpy(da.ptr, a.data(), a.size() * 2, cudaMemcpyHostToDevice);
  cudaMemcpy(db.ptr, b.data(), b.size() * 2, cudaMemcpyHostToDevice);
  cudaMemcpy(dc.ptr, cm.data(), cm.size() * 2, cudaMemcpyHostToDevice);
  cudaMemcpy(dbias.ptr, bias.data(), bias.size() * 2, cudaMemcpyHostToDevice);
  const uint16_t sentinel = oracle_float_to_bits(-77.0f, dt);

  for (int entry = 0; entry < 2; ++entry) {
    const std::string name = std::string(c.name) + (entry == 0 ? " [GemmDesc]" : " [GemmArguments]");
    std::vector<uint16_t> d(c.m * ldd, sentinel);
    cudaMemcpy(dd.ptr, d.data(), d.size() * 2, cudaMemcpyHostToDevice);
    Status st;
    if (entry == 0) {
      const GemmDesc desc{c.m,     c.n,     c.k,     lda,          ldb, ldc, ldd, c.dtype,
                          c.dtype, c.dtype, c.dtype, c.alpha, c.beta, c.bias ? dbias.ptr : nullptr, nullptr};
      st = zcutlass::gemm(desc, da.ptr, db.ptr, c.beta != 0.0f ? dc.ptr : nullptr, dd.ptr);
    } else {
      zcutlass::gemm_api::GemmArguments args{};
      args.problem = {c.m, c.n, c.k};
      args.A = {da.ptr, c.dtype, LayoutKind::RowMajor, lda};
      args.B = {db.ptr, c.dtype, LayoutKind::RowMajor, ldb};
      args.C = {c.beta != 0.0f ? dc.ptr : nullptr, c.dtype, LayoutKind::RowMajor, ldc};
      args.D = {dd.ptr, c.dtype, LayoutKind::RowMajor, ldd};
      args.alpha = c.alpha;
      args.beta = c.beta;
      args.bias = c.bias ? dbias.ptr : nullptr;
      st = zcutlass::gemm(args);
    }
    const cudaError_t ce = cudaDeviceSynchronize();
    expect(st == Status::Success, name + ": status " + zcutlass::status_to_string(st));
    expect(ce == cudaSuccess, name + ": " + cudaGetErrorString(ce));
    if (st != Status::Success || ce != cudaSuccess) continue;
    cudaMemcpy(d.data(), dd.ptr, d.size() * 2, cudaMemcpyDeviceToHost);

    double err2 = 0.0, ref2 = 0.0, max_abs = 0.0, worst = 0.0;
    int64_t pad_bad = 0;
    for (int64_t i = 0; i < c.m; ++i) {
      for (int64_t j = 0; j < ldd; ++j) {
        if (j >= c.n) {
          pad_bad += d[i * ldd + j] != sentinel;
          continue;
        }
        const double out = oracle_bits_to_float(d[i * ldd + j], dt);
        const double r = ref[i * c.n + j];
        const double e = std::fabs(out - r);
        err2 += e * e;
        ref2 += r * r;
        max_abs = std::max(max_abs, e);
        worst = std::max(worst, e / (4.0 * ulp_at_one(c.dtype) * (1.0 + std::fabs(r))));
        if (!std::isfinite(out)) worst = INFINITY;
      }
    }
    const double rel = std::sqrt(err2) / (ref2 > 0.0 ? std::sqrt(ref2) : 1.0);
    char buf[256];
    std::snprintf(buf, sizeof buf, ": rel_fro %.3e max_abs %.3e bound %.3f pad %lld kernel %s", rel, max_abs, worst,
                  static_cast<long long>(pad_bad), entry == 0 ? "" : "");
    expect(max_abs <= ref_abs_tol(c.dtype), name + buf);
    expect(rel <= rel_fro_tol(c.dtype), name + buf);
    expect(worst <= 1.0, name + buf);
    expect(pad_bad == 0, name + buf);
  }
}

// K = 0 or M/N = 0: Success, and D is not written (test_gemm.cu:439-473).
void run_zero_size() {
  uint16_t host[64];
  const uint16_t sentinel = 0x1234;
  for (auto& v : host) v = sentinel;
  DeviceBuffer<uint16_t> dd(64), da(64), db(64);
  cudaMemcpy(dd.ptr, host, sizeof host, cudaMemcpyHostToDevice);
  const int64_t shapes[][3] = {{0, 8, 8}, {8, 0, 8}, {8, 8, 0}};
  for (const auto& s : shapes) {
    const GemmDesc desc{s[0], s[1], s[2], 8, 8, 8, 8, DType::F16, DType::F16, DType::F16, DType::F16, 1.0f, 0.0f,
                        nullptr, nullptr};
    const Status st = zcutlass::gemm(desc, da.ptr, db.ptr, nullptr, dd.ptr);
    expect(st == Status::Success, "zero size " + std::to_string(s[0]) + "x" + std::to_string(s[1]) + "x" +
                                      std::to_string(s[2]) + " status");
  }
  cudaDeviceSynchronize();
  uint16_t back[64];
  cudaMemcpy(back, dd.ptr, sizeof back, cudaMemcpyDeviceToHost);
  expect(std::memcmp(back, host, sizeof host) == 0, "zero size: D untouched");
}

// Argument errors: the reference's status codes (test_gemm.cu:475-567).
void run_invalid_arguments() {
  DeviceBuffer<uint16_t> buf(1 << 16);
  const void* p = buf.ptr;
  void* q = buf.ptr;
  auto desc = [](int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc, int64_t ldd) {
    return GemmDesc{m, n, k, lda, ldb, ldc, ldd, DType::BF16, DType::BF16, DType::BF16, DType::BF16, 1.0f, 0.0f,
                    nullptr, nullptr};
  };
  struct Bad {
    const char* name;
    GemmDesc d;
    const void* a;
    const void* b;
    const void* c;
    void* out;
    Status want;
  };
  GemmDesc mixed = desc(16, 16, 16, 16, 16, 16, 16);
  mixed.b_type = DType::F16;
  GemmDesc fp8 = desc(16, 16, 16, 16, 16, 16, 16);
  fp8.a_type = fp8.b_type = fp8.c_type = fp8.d_type = DType::E4M3;
  GemmDesc beta_no_c = desc(16, 16, 16, 16, 16, 16, 16);
  beta_no_c.beta = 1.0f;
  GemmDesc col_a = desc(16, 16, 16, 16, 16, 16, 16);
  col_a.a_layout = LayoutKind::ColumnMajor;
  const Bad cases[] = {
      {"negative m", desc(-1, 16, 16, 16, 16, 16, 16), p, p, nullptr, q, Status::InvalidArgument},
      {"lda < k", desc(16, 16, 32, 16, 16, 16, 16), p, p, nullptr, q, Status::InvalidArgument},
      {"ldb < n", desc(16, 32, 16, 16, 16, 32, 32), p, p, nullptr, q, Status::InvalidArgument},
      {"ldd < n", desc(16, 32, 16, 16, 32, 32, 16), p, p, nullptr, q, Status::InvalidArgument},
      {"null A", desc(16, 16, 16, 16, 16, 16, 16), nullptr, p, nullptr, q, Status::InvalidArgument},
      {"null D", desc(16, 16, 16, 16, 16, 16, 16), p, p, nullptr, nullptr, Status::InvalidArgument},
      {"beta without C", beta_no_c, p, p, nullptr, q, Status::InvalidArgument},
      {"mixed dtypes", mixed, p, p, nullptr, q, Status::NotSupported},
      {"fp8", fp8, p, p, nullptr, q, Status::NotSupported},
      {"column-major A", col_a, p, p, nullptr, q, Status::NotSupported},
  };
  for (const Bad& c : cases) {
    const Status st = zcutlass::gemm(c.d, c.a, c.b, c.c, c.out);
    expect(st == c.want, std::string("invalid argument '") + c.name + "': got " + zcutlass::status_to_string(st) +
                             ", want " + zcutlass::status_to_string(c.want));
  }
  expect(cudaDeviceSynchronize() == cudaSuccess, "invalid arguments: no launch failed");
}

// Selection telemetry: a family per shape bucket and a tcgen05 kernel for
// every aligned bucket (test_gemm.cu:569-735 checks its own kernel names).
void run_dispatch() {
  auto sel = [](int64_t m, int64_t n, int64_t k) {
    return GemmDesc{m, n, k, k, n, n, n, DType::BF16, DType::BF16, DType::BF16, DType::BF16, 1.0f, 0.0f,
                    nullptr, nullptr};
  };
  const std::string decode = zcutlass::selected_kernel_name(sel(8, 4096, 4096));
  const std::string large = zcutlass::selected_kernel_name(sel(8192, 8192, 4096));
  expect(decode.find("swapab") != std::string::npos, "dispatch decode -> swap-AB, got " + decode);
  expect(large.find("tcgen05") != std::string::npos, "dispatch large -> tcgen05, got " + large);
  expect(std::string(zcutlass::selected_kernel_family(sel(8, 4096, 4096))) == "decode", "family decode");
  expect(std::string(zcutlass::selected_kernel_family(sel(8192, 8192, 4096))) == "large", "family large");
  GemmDesc odd = sel(300, 301, 299);  // odd leading dimensions: TMA cannot describe them
  expect(std::string(zcutlass::selected_kernel_name(odd)).find("generic") != std::string::npos, "dispatch odd ld");
  expect(zcutlass::selected_kernel_tile_m(sel(8192, 8192, 4096)) > 0, "tile_m reported");
  expect(std::string(zcutlass::selected_kernel_name(sel(-1, 8, 8))) == "none", "invalid desc -> none");
  expect(zcutlass::registered_gemm_operation_count() > 0, "operations registered");
  expect(zcutlass::get_workspace_size(zcutlass::gemm_api::GemmArguments{}) == 0, "workspace 0");
}

}  // namespace

int main() {
  int devices = 0;
  if (cudaGetDeviceCount(&devices) != cudaSuccess || devices == 0) {
    std::printf("no CUDA device\n");
    return 2;
  }
  // The reference program's case list (tests/test_gemm.cu:754-785), with
  // its padding pattern, plus two multi-tile shapes per dtype.
  const Case cases[] = {
      {"f16 tiny padded bias", DType::F16, 15, 17, 19, 1.0f, 0.25f, true, 1, 1, 1, 1},
      {"f16 16x16", DType::F16, 16, 16, 16, 1.0f, 0.0f, false, 0, 0, 0, 0},
      {"f16 rectangular", DType::F16, 65, 129, 31, 0.75f, 0.5f, true, 1, 1, 1, 1},
      {"f16 ragged alpha no-bias padded A/D", DType::F16, 31, 63, 17, -0.5f, 0.0f, false, 2, 0, 0, 9},
      {"f16 ragged beta no-bias", DType::F16, 47, 64, 33, 0.5f, -0.25f, false, 0, 0, 0, 0},
      {"f16 llm-smoke", DType::F16, 8, 256, 256, 1.0f, 0.0f, false, 0, 0, 0, 0},
      {"f16 prefill 64x1024x1024", DType::F16, 64, 1024, 1024, 1.0f, 0.0f, true, 0, 0, 0, 0},
      {"f16 large 1024x2048x512", DType::F16, 1024, 2048, 512, 1.0f, 0.0f, false, 0, 0, 0, 8},
      {"bf16 tiny padded bias", DType::BF16, 13, 19, 23, 1.0f, 0.25f, true, 1, 1, 1, 1},
      {"bf16 16x16", DType::BF16, 16, 16, 16, 1.0f, 0.0f, false, 0, 0, 0, 0},
      {"bf16 rectangular", DType::BF16, 67, 127, 29, 0.75f, 0.5f, true, 1, 1, 1, 1},
      {"bf16 ragged alpha no-bias padded B/C/D", DType::BF16, 29, 61, 15, -0.75f, 0.0f, false, 0, 4, 6, 10},
      {"bf16 ragged beta no-bias", DType::BF16, 45, 64, 31, 0.5f, -0.25f, false, 0, 0, 0, 0},
      {"bf16 llm-smoke", DType::BF16, 8, 256, 256, 1.0f, 0.0f, false, 0, 0, 0, 0},
      {"bf16 prefill 32x1024x1024", DType::BF16, 32, 1024, 1024, 1.0f, 0.0f, true, 0, 0, 0, 0},
      {"bf16 large 2048x1024x1536", DType::BF16, 2048, 1024, 1536, 0.5f, 1.0f, true, 0, 0, 0, 8},
  };
  for (const Case& c : cases) run_case(c);
  run_zero_size();
  run_invalid_arguments();
  run_dispatch();
  std::printf("zcutlass C++ API test: %d checks, %d failures\n", g_checks, g_failures);
  return g_failures == 0 ? 0 : 1;
}
