// TEST INFRASTRUCTURE ONLY. This is the parity oracle for the zcutlass GEMM
// hot path: a CPU restatement of the reference's host GEMM. Only tests/,
// __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it; the
// product library never links or calls anything in oracle/.
//
// What it restates (supercatking/zcutlass, paths relative to that project):
//   oracle_gemm        tests/test_gemm.cu:130-162  `reference()`:
//                      FP32 accumulation in increasing k, one multiply and one
//                      add per step (no fused multiply-add), then
//                      alpha*acc (+ beta*C when beta != 0) (+ bias[col]),
//                      rounded once to the storage type (round-to-nearest-even).
//                      The same epilogue order as the device kernels,
//                      src/gemm.cu:240-250 (bias added unscaled by alpha).
//   oracle_make_tensor tests/test_gemm.cu:118-128 `make_tensor`: std::mt19937
//                      seeded per tensor, std::uniform_real_distribution<float>
//                      over [-0.35, 0.35), padding columns (col >= cols) set to 0.
//   oracle_gemm_f64    the same GEMM accumulated in FP64 for selected rows,
//                      used to bound large-shape error without a full CPU GEMM.
// Storage values cross this ABI as raw 16-bit patterns (uint16_t).
//
// Build: oracle/Makefile (g++ -O3 -ffp-contract=off, so the compiler cannot
// fuse the multiply and the add and change the rounding).
#include <cmath>
#include <cstdint>
#include <cstring>
#include <random>
#include <thread>
#include <vector>

namespace {

enum { kF16 = 0, kBF16 = 1 };

float bits_to_float(uint32_t u) {
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

uint32_t float_to_bits(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return u;
}

// bfloat16 is the top half of an IEEE binary32.
float bf16_to_float(uint16_t h) { return bits_to_float(static_cast<uint32_t>(h) << 16); }

// Round-to-nearest-even binary32 -> bfloat16; NaN stays a quiet NaN.
uint16_t float_to_bf16(float f) {
  const uint32_t u = float_to_bits(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((u >> 16) | 0x0040u);
  const uint32_t lsb = (u >> 16) & 1u;
  return static_cast<uint16_t>((u + 0x7fffu + lsb) >> 16);
}

// IEEE binary16 -> binary32 (exact).
float f16_to_float(uint16_t h) {
  const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1fu;
  const uint32_t man = h & 0x3ffu;
  if (exp == 0) {
    // zero or subnormal: man * 2^-24
    const float v = std::ldexp(static_cast<float>(man), -24);
    return sign ? -v : v;
  }
  if (exp == 31) return bits_to_float(sign | 0x7f800000u | (man << 13));
  return bits_to_float(sign | ((exp + 112u) << 23) | (man << 13));
}

// binary32 -> binary16, round-to-nearest-even, overflow to infinity,
// gradual underflow to subnormals.
uint16_t float_to_f16(float f) {
  const uint32_t u = float_to_bits(f);
  const uint16_t sign = static_cast<uint16_t>((u >> 16) & 0x8000u);
  const uint32_t absu = u & 0x7fffffffu;
  if (absu > 0x7f800000u) return static_cast<uint16_t>(sign | 0x7e00u);  // NaN
  if (absu >= 0x477ff000u) return static_cast<uint16_t>(sign | 0x7c00u);  // >= 65520 rounds to inf
  const int exp = static_cast<int>(absu >> 23) - 127;
  if (exp >= -14) {
    // normal half: keep 10 mantissa bits of the 23, rounding the other 13
    uint32_t man = absu & 0x7fffffu;
    uint32_t h = static_cast<uint32_t>(exp + 15) << 10 | (man >> 13);
    const uint32_t rest = man & 0x1fffu;
    if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) ++h;  // carry may bump the exponent
    return static_cast<uint16_t>(sign | h);
  }
  // subnormal half: value = q * 2^-24 with q = round(|f| * 2^24)
  const float scaled = bits_to_float(absu) * 16777216.0f;  // exact power-of-two scaling
  const float q = std::nearbyint(scaled);                   // ties-to-even in the default mode
  return static_cast<uint16_t>(sign | static_cast<uint16_t>(q));
}

float to_float(uint16_t v, int dtype) { return dtype == kBF16 ? bf16_to_float(v) : f16_to_float(v); }
uint16_t from_float(float v, int dtype) { return dtype == kBF16 ? float_to_bf16(v) : float_to_f16(v); }

// Rows [r0, r1) of the FP32 oracle. Loop order keeps, for every output
// element, the reference's accumulation order (k = 0, 1, ..., K-1) while
// letting the compiler vectorise across columns.
void gemm_rows(int64_t r0, int64_t r1, int64_t n, int64_t k, const uint16_t* A, int64_t lda,
               const uint16_t* B, int64_t ldb, const uint16_t* C, int64_t ldc,
               const uint16_t* bias, float alpha, float beta, int dtype, float* out) {
  std::vector<float> acc(static_cast<size_t>(n));
  std::vector<float> brow(static_cast<size_t>(n));
  for (int64_t r = r0; r < r1; ++r) {
    std::fill(acc.begin(), acc.end(), 0.0f);
    for (int64_t kk = 0; kk < k; ++kk) {
      const float a = to_float(A[r * lda + kk], dtype);
      const uint16_t* bk = B + kk * ldb;
      for (int64_t c = 0; c < n; ++c) brow[c] = to_float(bk[c], dtype);
      float* accp = acc.data();
      const float* bp = brow.data();
      for (int64_t c = 0; c < n; ++c) {
        const float prod = a * bp[c];
        accp[c] = accp[c] + prod;
      }
    }
    for (int64_t c = 0; c < n; ++c) {
      float value = alpha * acc[c];
      if (beta != 0.0f) value += beta * to_float(C[r * ldc + c], dtype);
      if (bias != nullptr) value += to_float(bias[c], dtype);
      out[r * n + c] = to_float(from_float(value, dtype), dtype);
    }
  }
}

}  // namespace

extern "C" {

// Exposed so tests can check the conversions against numpy / torch.
uint16_t oracle_float_to_bits(float v, int dtype) { return from_float(v, dtype); }
float oracle_bits_to_float(uint16_t v, int dtype) { return to_float(v, dtype); }

// Fills out[rows * ld] exactly like the reference test's make_tensor<T>.
void oracle_make_tensor(int64_t rows, int64_t cols, int64_t ld, int seed, int dtype,
                        uint16_t* out) {
  std::mt19937 rng(static_cast<std::mt19937::result_type>(seed));
  std::uniform_real_distribution<float> dist(-0.35f, 0.35f);
  for (int64_t i = 0; i < rows; ++i)
    for (int64_t j = 0; j < ld; ++j) out[i * ld + j] = from_float(j < cols ? dist(rng) : 0.0f, dtype);
}

// out[m * n] (dense, ld = n) receives the reference result as float (already
// rounded to the storage type). C may be null when beta == 0; bias may be null.
void oracle_gemm(int64_t m, int64_t n, int64_t k, const uint16_t* A, int64_t lda,
                 const uint16_t* B, int64_t ldb, const uint16_t* C, int64_t ldc,
                 const uint16_t* bias, float alpha, float beta, int dtype, int threads,
                 float* out) {
  if (threads <= 1 || m < 2) {
    gemm_rows(0, m, n, k, A, lda, B, ldb, C, ldc, bias, alpha, beta, dtype, out);
    return;
  }
  const int64_t t = std::min<int64_t>(threads, m);
  std::vector<std::thread> pool;
  for (int64_t i = 0; i < t; ++i) {
    const int64_t r0 = m * i / t, r1 = m * (i + 1) / t;
    pool.emplace_back(gemm_rows, r0, r1, n, k, A, lda, B, ldb, C, ldc, bias, alpha, beta, dtype,
                      out);
  }
  for (auto& th : pool) th.join();
}

// FP64-accumulated, unrounded result for the listed rows: out[nrows * n].
void oracle_gemm_f64_rows(int64_t n, int64_t k, const uint16_t* A, int64_t lda, const uint16_t* B,
                          int64_t ldb, const uint16_t* C, int64_t ldc, const uint16_t* bias,
                          float alpha, float beta, int dtype, const int64_t* rows, int64_t nrows,
                          double* out) {
  std::vector<double> acc(static_cast<size_t>(n));
  for (int64_t i = 0; i < nrows; ++i) {
    const int64_t r = rows[i];
    std::fill(acc.begin(), acc.end(), 0.0);
    for (int64_t kk = 0; kk < k; ++kk) {
      const double a = to_float(A[r * lda + kk], dtype);
      const uint16_t* bk = B + kk * ldb;
      for (int64_t c = 0; c < n; ++c) acc[c] += a * static_cast<double>(to_float(bk[c], dtype));
    }
    for (int64_t c = 0; c < n; ++c) {
      double value = static_cast<double>(alpha) * acc[c];
      if (beta != 0.0f) value += static_cast<double>(beta) * to_float(C[r * ldc + c], dtype);
      if (bias != nullptr) value += to_float(bias[c], dtype);
      out[i * n + c] = value;
    }
  }
}

}  // extern "C"
