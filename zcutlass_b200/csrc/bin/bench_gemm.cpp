// zcutlass_bench: native GEMM benchmark (built as zcutlass_b200/zcutlass_bench).
//
// Same command line, suites, timing method and schema-v1 JSONL records as the
// reference harness (benchmarks/bench_gemm.cu in supercatking/zcutlass:
// options 120-160, suites 162-216, CUDA-event median 238-263, TFLOP/s 265-268,
// record 270-330, cuBLAS comparator 392-412), against this library's C++ API.
// Additions: --b-layout col (a PyTorch [N,K] weight), --bias, --rotate R
// (R copies of A/B/C/D cycled per launch so each launch reads HBM, not L2),
// --force-kernel SUBSTR (sets ZCUTLASS_FORCE_KERNEL) and per-record GB/s.
#include <cublas_v2.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <iomanip>
#include <iostream>
#include <random>
#include <sstream>
#include <string>
#include <vector>

#include "zcutlass/gemm.hpp"

namespace {

#define CHECK_CUDA(expr)                                                                   \
  do {                                                                                     \
    cudaError_t e_ = (expr);                                                               \
    if (e_ != cudaSuccess) {                                                               \
      std::cerr << "CUDA error " << __FILE__ << ":" << __LINE__ << ": " << cudaGetErrorString(e_) \
                << std::endl;                                                              \
      std::exit(1);                                                                        \
    }                                                                                      \
  } while (0)

#define CHECK_CUBLAS(expr)                                                                 \
  do {                                                                                     \
    cublasStatus_t s_ = (expr);                                                            \
    if (s_ != CUBLAS_STATUS_SUCCESS) {                                                     \
      std::cerr << "cuBLAS error " << __FILE__ << ":" << __LINE__ << ": " << int(s_) << std::endl; \
      std::exit(1);                                                                        \
    }                                                                                      \
  } while (0)

struct Options {
  int64_t m = 256, n = 4096, k = 4096;
  std::string dtype = "f16";
  std::string suite = "single";
  std::string providers = "zcutlass,cublas";
  std::string output;
  std::string b_layout = "row";
  std::string force_kernel;
  std::string experimental_kernel;
  int warmup = 10, iterations = 50, rotate = 1;
  float alpha = 1.0f, beta = 0.0f;
  bool bias = false, json = false, append = false, experimental = false;
  bool graph = false;
};

struct Shape {
  int64_t m, n, k;
};

void usage() {
  std::cout << "Usage: zcutlass_bench [--m M --n N --k K] [--dtype f16|bf16|both]\n"
               "  [--suite single|correctness|smoke|llm|llm-v1.5|llm-canonical|llm-decode|llm-prefill|square|ragged]\n"
               "  [--providers zcutlass,cublas] [--json] [--output FILE] [--append]\n"
               "  [--warmup N] [--iterations N] [--alpha X] [--beta X] [--bias]\n"
               "  [--b-layout row|col] [--rotate R] [--force-kernel SUBSTR]\n"
               "  [--experimental-kernels] [--experimental-kernel NAME] [--graph]\n"
               "  --graph: capture the timed launches in one CUDA graph and report the\n"
               "           device time per launch (no host launch latency in the figure)\n";
}

Options parse(int argc, char** argv) {
  Options o;
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    auto val = [&]() -> const char* {
      if (i + 1 >= argc) {
        std::cerr << "Missing value for " << a << std::endl;
        std::exit(2);
      }
      return argv[++i];
    };
    if (a == "--m") o.m = std::atoll(val());
    else if (a == "--n") o.n = std::atoll(val());
    else if (a == "--k") o.k = std::atoll(val());
    else if (a == "--dtype") o.dtype = val();
    else if (a == "--suite") o.suite = val();
    else if (a == "--providers") o.providers = val();
    else if (a == "--output") o.output = val();
    else if (a == "--append") o.append = true;
    else if (a == "--warmup") o.warmup = std::atoi(val());
    else if (a == "--iterations") o.iterations = std::atoi(val());
    else if (a == "--alpha") o.alpha = static_cast<float>(std::atof(val()));
    else if (a == "--beta") o.beta = static_cast<float>(std::atof(val()));
    else if (a == "--bias") o.bias = true;
    else if (a == "--b-layout") o.b_layout = val();
    else if (a == "--rotate") o.rotate = std::max(1, std::atoi(val()));
    else if (a == "--force-kernel") o.force_kernel = val();
    else if (a == "--json") o.json = true;
    else if (a == "--graph") o.graph = true;
    else if (a == "--experimental-kernels") o.experimental = true;
    else if (a == "--experimental-kernel") {
      o.experimental = true;
      o.experimental_kernel = val();
    } else if (a == "--help") {
      usage();
      std::exit(0);
    } else {
      std::cerr << "Unknown argument: " << a << std::endl;
      std::exit(2);
    }
  }
  return o;
}

std::vector<Shape> make_shapes(const Options& o) {
  const std::string& s = o.suite;
  if (s == "single") return {{o.m, o.n, o.k}};
  if (s == "smoke") return {{1, 1024, 1024}, {8, 2048, 2048}, {64, 4096, 4096}, {256, 2048, 8192}};
  if (s == "correctness") return {{15, 17, 19}, {16, 16, 16}, {65, 129, 31}, {67, 127, 29}};
  if (s == "square") return {{512, 512, 512}, {1024, 1024, 1024}, {2048, 2048, 2048}, {4096, 4096, 4096}};
  if (s == "ragged") return {{63, 127, 65}, {65, 129, 127}, {127, 255, 129}, {257, 511, 255}};
  if (s == "llm-v1.5" || s == "llm-canonical")
    return {{8, 4096, 4096}, {128, 4096, 4096}, {128, 16384, 4096}, {128, 4096, 16384}, {4096, 4096, 4096}};
  if (s == "llm" || s == "llm-decode" || s == "llm-prefill") {
    std::vector<Shape> v;
    std::vector<int64_t> ms = {1, 8, 16, 64, 256, 1024};
    if (s == "llm-decode") ms = {1, 2, 4, 8, 16};
    if (s == "llm-prefill") ms = {64, 128, 256, 512, 1024};
    for (int64_t h : {1024, 2048, 4096, 8192}) {
      for (int64_t m : ms) {
        v.push_back({m, h, h});
        v.push_back({m, 4 * h, h});
        v.push_back({m, h, 4 * h});
      }
    }
    v.push_back({1024, 1024, 1024});
    v.push_back({2048, 2048, 2048});
    v.push_back({4096, 4096, 4096});
    return v;
  }
  std::cerr << "Unknown suite: " << s << std::endl;
  std::exit(2);
}

bool provider_on(const Options& o, const char* p) {
  return o.providers == "all" || o.providers.find(p) != std::string::npos;
}

template <typename T>
T from_float(float v);
template <>
half from_float<half>(float v) { return __float2half_rn(v); }
template <>
__nv_bfloat16 from_float<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

template <typename T>
cudaDataType cuda_type();
template <>
cudaDataType cuda_type<half>() { return CUDA_R_16F; }
template <>
cudaDataType cuda_type<__nv_bfloat16>() { return CUDA_R_16BF; }

template <typename T>
zcutlass::DType z_dtype();
template <>
zcutlass::DType z_dtype<half>() { return zcutlass::DType::F16; }
template <>
zcutlass::DType z_dtype<__nv_bfloat16>() { return zcutlass::DType::BF16; }

template <typename T>
std::vector<T> make_tensor(size_t count, int seed) {
  std::mt19937 rng(seed);
  std::uniform_real_distribution<float> dist(-0.25f, 0.25f);
  std::vector<T> v(count);
  for (T& x : v) x = from_float<T>(dist(rng));
  return v;
}

template <typename Fn>
float time_ms(Fn&& fn, int warmup, int iterations) {
  for (int i = 0; i < warmup; ++i) fn(i);
  CHECK_CUDA(cudaDeviceSynchronize());
  cudaEvent_t start, stop;
  CHECK_CUDA(cudaEventCreate(&start));
  CHECK_CUDA(cudaEventCreate(&stop));
  std::vector<float> samples;
  for (int i = 0; i < iterations; ++i) {
    CHECK_CUDA(cudaEventRecord(start));
    fn(i);
    CHECK_CUDA(cudaEventRecord(stop));
    CHECK_CUDA(cudaEventSynchronize(stop));
    float ms = 0.0f;
    CHECK_CUDA(cudaEventElapsedTime(&ms, start, stop));
    samples.push_back(ms);
  }
  CHECK_CUDA(cudaEventDestroy(start));
  CHECK_CUDA(cudaEventDestroy(stop));
  std::sort(samples.begin(), samples.end());
  return samples[samples.size() / 2];
}

// Device time per launch: `iterations` calls captured once in a CUDA graph on
// `stream` (programmatic dependent launch between them as in a serving
// graph), replayed, and divided by the count. The reference's per-launch
// event timing above also counts the host's launch latency.
template <typename Fn>
float time_graph_ms(Fn&& fn, int warmup, int iterations, cudaStream_t stream) {
  for (int i = 0; i < warmup; ++i) fn(i);
  CHECK_CUDA(cudaStreamSynchronize(stream));
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  CHECK_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
  for (int i = 0; i < iterations; ++i) fn(i);
  CHECK_CUDA(cudaStreamEndCapture(stream, &graph));
  CHECK_CUDA(cudaGraphInstantiate(&exec, graph, 0));
  CHECK_CUDA(cudaGraphLaunch(exec, stream));
  CHECK_CUDA(cudaStreamSynchronize(stream));
  cudaEvent_t start, stop;
  CHECK_CUDA(cudaEventCreate(&start));
  CHECK_CUDA(cudaEventCreate(&stop));
  CHECK_CUDA(cudaEventRecord(start, stream));
  CHECK_CUDA(cudaGraphLaunch(exec, stream));
  CHECK_CUDA(cudaEventRecord(stop, stream));
  CHECK_CUDA(cudaEventSynchronize(stop));
  float ms = 0.0f;
  CHECK_CUDA(cudaEventElapsedTime(&ms, start, stop));
  CHECK_CUDA(cudaEventDestroy(start));
  CHECK_CUDA(cudaEventDestroy(stop));
  CHECK_CUDA(cudaGraphExecDestroy(exec));
  CHECK_CUDA(cudaGraphDestroy(graph));
  return ms / iterations;
}

double algorithmic_bytes(const Shape& s, const Options& o) {
  return 2.0 * (double(s.m) * s.k + double(s.k) * s.n + double(s.m) * s.n) +
         (o.beta != 0.0f ? 2.0 * double(s.m) * s.n : 0.0) + (o.bias ? 2.0 * s.n : 0.0);
}

zcutlass::GemmDesc make_desc(const Shape& s, const Options& o, zcutlass::DType t, const void* bias) {
  const bool col = o.b_layout == "col";
  zcutlass::GemmDesc d{s.m, s.n, s.k, s.k, col ? s.k : s.n, s.n, s.n, t, t, t, t, o.alpha, o.beta,
                       bias, nullptr};
  if (col) d.b_layout = zcutlass::layout::LayoutKind::ColumnMajor;
  return d;
}

void emit_record(std::ostream& out, const Options& o, const Shape& s, const char* provider,
                 const char* kernel, float ms, const cudaDeviceProp& prop) {
  const zcutlass::DType t = o.dtype == "f16" ? zcutlass::DType::F16 : zcutlass::DType::BF16;
  const zcutlass::GemmDesc desc = make_desc(s, o, t, o.bias ? reinterpret_cast<const void*>(256) : nullptr);
  const bool z = std::string(provider) == "zcutlass";
  const double tf = 2.0 * double(s.m) * s.n * s.k / (double(ms) * 1e-3) / 1e12;
  const double gbs = algorithmic_bytes(s, o) / (double(ms) * 1e-3) / 1e9;
  out << std::fixed << std::setprecision(4) << "{\"schema_version\":1"
      << ",\"problem\":{\"operation\":\"gemm\",\"m\":" << s.m << ",\"n\":" << s.n << ",\"k\":" << s.k
      << ",\"dtype\":\"" << o.dtype << "\",\"layout\":\"row," << o.b_layout << ",row,row\",\"alpha\":" << o.alpha
      << ",\"beta\":" << o.beta << ",\"bias\":" << (o.bias ? "true" : "false") << "}"
      << ",\"provider\":\"" << provider << "\",\"status\":\"success\",\"kernel\":\"" << kernel << "\""
      << ",\"performance\":{\"warmup_iterations\":" << o.warmup << ",\"profiling_iterations\":" << o.iterations
      << ",\"median_ms\":" << ms << ",\"tflops\":" << tf << ",\"gbps\":" << gbs << ",\"rotate\":" << o.rotate
      << ",\"timing\":\"" << (o.graph ? "cuda_graph_mean" : "per_launch_events_median") << "\"}"
      << ",\"environment\":{\"gpu_name\":\"" << prop.name << "\",\"sm\":" << prop.major << prop.minor
      << ",\"zcutlass_version\":\"" << zcutlass::version_major() << "." << zcutlass::version_minor() << "."
      << zcutlass::version_patch() << "\",\"registered_gemm_operations\":"
      << zcutlass::registered_gemm_operation_count() << "}"
      << ",\"tags\":{\"suite\":\"" << o.suite << "\",\"shape_family\":\"" << zcutlass::selected_kernel_family(desc)
      << "\",\"kernel_path\":\"" << (z ? zcutlass::selected_kernel_path(desc) : "external")
      << "\",\"tile_m\":" << (z ? zcutlass::selected_kernel_tile_m(desc) : 0)
      << ",\"tile_n\":" << (z ? zcutlass::selected_kernel_tile_n(desc) : 0)
      << ",\"tile_k\":" << (z ? zcutlass::selected_kernel_tile_k(desc) : 0)
      << ",\"pipeline_stages\":" << (z ? zcutlass::selected_kernel_pipeline_stages(desc) : 0)
      << ",\"epilogue_kind\":\"" << (z ? zcutlass::selected_kernel_epilogue_kind(desc) : "external")
      << "\",\"experimental_kernels\":" << (o.experimental ? "true" : "false")
      << ",\"experimental_kernel_filter\":\"" << o.experimental_kernel << "\"}}" << std::endl;
}

template <typename T>
void run_shape(const Shape& s, const Options& o, cublasHandle_t handle, const cudaDeviceProp& prop,
               std::ostream* out) {
  const bool col = o.b_layout == "col";
  const int64_t lda = s.k, ldb = col ? s.k : s.n, ldc = s.n, ldd = s.n;
  const size_t a_n = size_t(s.m * lda), b_n = size_t((col ? s.n : s.k) * ldb), c_n = size_t(s.m * ldc);
  const int R = o.rotate;
  std::vector<T*> A(R), B(R), C(R), D(R);
  const std::vector<T> ha = make_tensor<T>(a_n, 11), hb = make_tensor<T>(b_n, 23), hc = make_tensor<T>(c_n, 37);
  const std::vector<T> hbias = make_tensor<T>(size_t(s.n), 53);
  for (int r = 0; r < R; ++r) {
    CHECK_CUDA(cudaMalloc(&A[r], a_n * sizeof(T)));
    CHECK_CUDA(cudaMalloc(&B[r], b_n * sizeof(T)));
    CHECK_CUDA(cudaMalloc(&C[r], c_n * sizeof(T)));
    CHECK_CUDA(cudaMalloc(&D[r], c_n * sizeof(T)));
    CHECK_CUDA(cudaMemcpy(A[r], ha.data(), a_n * sizeof(T), cudaMemcpyHostToDevice));
    CHECK_CUDA(cudaMemcpy(B[r], hb.data(), b_n * sizeof(T), cudaMemcpyHostToDevice));
    CHECK_CUDA(cudaMemcpy(C[r], hc.data(), c_n * sizeof(T), cudaMemcpyHostToDevice));
  }
  T* bias = nullptr;
  CHECK_CUDA(cudaMalloc(&bias, size_t(s.n) * sizeof(T)));
  CHECK_CUDA(cudaMemcpy(bias, hbias.data(), size_t(s.n) * sizeof(T), cudaMemcpyHostToDevice));
  zcutlass::GemmDesc desc = make_desc(s, o, z_dtype<T>(), o.bias ? bias : nullptr);
  cudaStream_t stream = nullptr;
  if (o.graph) {
    CHECK_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    desc.stream = stream;
    CHECK_CUBLAS(cublasSetStream(handle, stream));
  }

  auto z_fn = [&](int i) {
    const int r = i % R;
    const zcutlass::Status st = zcutlass::gemm(desc, A[r], B[r], o.beta != 0.0f ? C[r] : nullptr, D[r]);
    if (st != zcutlass::Status::Success) {
      std::cerr << "zcutlass::gemm failed: " << zcutlass::status_to_string(st) << std::endl;
      std::exit(1);
    }
  };
  const float alpha = o.alpha, beta = o.beta;
  auto blas_fn = [&](int i) {
    const int r = i % R;
    if (beta != 0.0f) CHECK_CUDA(cudaMemcpyAsync(D[r], C[r], c_n * sizeof(T), cudaMemcpyDeviceToDevice, stream));
    // Row-major D = A * B is column-major D^T = B^T * A^T.
    CHECK_CUBLAS(cublasGemmEx(handle, col ? CUBLAS_OP_T : CUBLAS_OP_N, CUBLAS_OP_N, int(s.n), int(s.m), int(s.k),
                              &alpha, B[r], cuda_type<T>(), int(ldb), A[r], cuda_type<T>(), int(lda), &beta,
                              D[r], cuda_type<T>(), int(ldd), CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT_TENSOR_OP));
  };

  float z_ms = 0.0f, b_ms = 0.0f;
  if (provider_on(o, "zcutlass")) {
    z_ms = o.graph ? time_graph_ms(z_fn, o.warmup, o.iterations, stream) : time_ms(z_fn, o.warmup, o.iterations);
    if (out) emit_record(*out, o, s, "zcutlass", zcutlass::selected_kernel_name(desc), z_ms, prop);
  }
  if (provider_on(o, "cublas")) {
    b_ms = o.graph ? time_graph_ms(blas_fn, o.warmup, o.iterations, stream) : time_ms(blas_fn, o.warmup, o.iterations);
    if (out) emit_record(*out, o, s, "cublas", "cublasGemmEx", b_ms, prop);
  }
  if (stream != nullptr) {
    CHECK_CUBLAS(cublasSetStream(handle, nullptr));
    CHECK_CUDA(cudaStreamDestroy(stream));
    desc.stream = nullptr;  // the telemetry below must not see the destroyed stream
  }
  const double flops = 2.0 * double(s.m) * s.n * s.k;
  const double z_tf = z_ms > 0 ? flops / (z_ms * 1e-3) / 1e12 : 0.0;
  const double b_tf = b_ms > 0 ? flops / (b_ms * 1e-3) / 1e12 : 0.0;
  const double z_gb = z_ms > 0 ? algorithmic_bytes(s, o) / (z_ms * 1e-3) / 1e9 : 0.0;
  const double speedup = (z_ms > 0 && b_ms > 0) ? b_ms / z_ms : 0.0;
  if (o.json) {
    std::cout << std::fixed << std::setprecision(4) << "{\"m\":" << s.m << ",\"n\":" << s.n << ",\"k\":" << s.k
              << ",\"dtype\":\"" << o.dtype << "\",\"b_layout\":\"" << o.b_layout << "\",\"zcutlass_ms\":" << z_ms
              << ",\"kernel\":\"" << zcutlass::selected_kernel_name(desc) << "\",\"shape_family\":\""
              << zcutlass::selected_kernel_family(desc) << "\",\"kernel_path\":\""
              << zcutlass::selected_kernel_path(desc) << "\",\"tile_m\":" << zcutlass::selected_kernel_tile_m(desc)
              << ",\"tile_n\":" << zcutlass::selected_kernel_tile_n(desc)
              << ",\"tile_k\":" << zcutlass::selected_kernel_tile_k(desc)
              << ",\"pipeline_stages\":" << zcutlass::selected_kernel_pipeline_stages(desc)
              << ",\"epilogue_kind\":\"" << zcutlass::selected_kernel_epilogue_kind(desc) << "\""
              << ",\"cublas_ms\":" << b_ms << ",\"zcutlass_tflops\":" << z_tf << ",\"zcutlass_gbps\":" << z_gb
              << ",\"cublas_tflops\":" << b_tf << ",\"speedup\":" << speedup << "}" << std::endl;
  } else {
    std::cout << std::fixed << std::setprecision(4) << "m=" << s.m << " n=" << s.n << " k=" << s.k
              << " dtype=" << o.dtype << " B=" << o.b_layout << " kernel=" << zcutlass::selected_kernel_name(desc)
              << " zcutlass=" << z_ms << " ms (" << z_tf << " TFLOP/s, " << z_gb << " GB/s) cublas=" << b_ms
              << " ms (" << b_tf << " TFLOP/s) speedup=" << speedup << "x" << std::endl;
  }
  for (int r = 0; r < R; ++r) {
    CHECK_CUDA(cudaFree(A[r]));
    CHECK_CUDA(cudaFree(B[r]));
    CHECK_CUDA(cudaFree(C[r]));
    CHECK_CUDA(cudaFree(D[r]));
  }
  CHECK_CUDA(cudaFree(bias));
}

}  // namespace

int main(int argc, char** argv) {
  Options o = parse(argc, argv);
  if (o.experimental) {
    setenv("ZCUTLASS_EXPERIMENTAL_KERNELS", "1", 1);
    if (!o.experimental_kernel.empty()) setenv("ZCUTLASS_EXPERIMENTAL_KERNEL", o.experimental_kernel.c_str(), 1);
  }
  if (!o.force_kernel.empty()) setenv("ZCUTLASS_FORCE_KERNEL", o.force_kernel.c_str(), 1);
  if (o.iterations <= 0 || o.warmup < 0) {
    std::cerr << "Invalid warmup/iteration counts" << std::endl;
    return 2;
  }
  if (o.b_layout != "row" && o.b_layout != "col") {
    std::cerr << "--b-layout must be row or col" << std::endl;
    return 2;
  }
  int device = 0;
  CHECK_CUDA(cudaGetDevice(&device));
  cudaDeviceProp prop{};
  CHECK_CUDA(cudaGetDeviceProperties(&prop, device));
  if (!o.json) std::cout << "GPU: " << prop.name << " sm_" << prop.major << prop.minor << std::endl;
  cublasHandle_t handle = nullptr;
  CHECK_CUBLAS(cublasCreate(&handle));
  std::ofstream file;
  std::ostream* out = nullptr;
  if (!o.output.empty()) {
    file.open(o.output, o.append ? std::ios::app : std::ios::out);
    if (!file) {
      std::cerr << "Failed to open output file: " << o.output << std::endl;
      return 2;
    }
    out = &file;
  }
  for (const Shape& s : make_shapes(o)) {
    if (o.dtype == "f16") {
      run_shape<half>(s, o, handle, prop, out);
    } else if (o.dtype == "bf16") {
      run_shape<__nv_bfloat16>(s, o, handle, prop, out);
    } else if (o.dtype == "both") {
      Options a = o;
      a.dtype = "f16";
      run_shape<half>(s, a, handle, prop, out);
      a.dtype = "bf16";
      run_shape<__nv_bfloat16>(s, a, handle, prop, out);
    } else {
      std::cerr << "Unsupported dtype: " << o.dtype << std::endl;
      return 2;
    }
  }
  CHECK_CUBLAS(cublasDestroy(handle));
  return 0;
}
