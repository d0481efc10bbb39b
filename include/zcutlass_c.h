/*
 * zcutlass C ABI: plain pointers, sizes and enums, no C++ or torch types.
 *
 * Every function below is a flat C entry point for the C++ API declared in
 * include/zcutlass/gemm.hpp and is what an FFI (ctypes, cffi, JNI, cgo) binds.
 * Each one cites the reference interface it replaces, in
 * supercatking/zcutlass (paths relative to that project):
 *
 *   zcutlass_gemm               <- zcutlass::gemm(GemmDesc, A, B, C, D)
 *                                  include/zcutlass/gemm/gemm.hpp:72-76, src/gemm.cu:609-629
 *   zcutlass_gemm_rowmajor      <- same call with the GemmDesc fields passed flat
 *                                  (what python/zcutlass_torch/csrc/zcutlass_torch.cpp:67-83 builds)
 *   zcutlass_can_implement      <- zcutlass::can_implement(GemmArguments)  gemm.hpp:78, gemm.cu:718-739
 *   zcutlass_get_workspace_size <- zcutlass::get_workspace_size            gemm.hpp:79, gemm.cu:741-744
 *   zcutlass_selected_kernel_*  <- zcutlass::selected_kernel_*             gemm.hpp:80-88, gemm.cu:631-688
 *   zcutlass_registered_gemm_operation_count <- gemm.hpp:89, gemm.cu:690-693
 *   zcutlass_status_to_string   <- zcutlass::status_to_string              status.hpp:14
 *   zcutlass_dtype_name / _bits <- numeric_types.hpp:43-44
 *   zcutlass_version_*          <- gemm.hpp (umbrella) :13-15
 *
 * Entry points with no reference counterpart (Blackwell additions):
 *   zcutlass_device_error       read/clear the device-side error word that the
 *                               tcgen05 kernels set when a bounded wait expires
 *   zcutlass_gemm_kernel_launches  number of kernel launches this library made
 *   zcutlass_selftest_bounded_wait runs a kernel whose bounded wait must expire
 *   zcutlass_gemm_decode_noalloc   decode GEMM that allocates nothing
 *   zcutlass_nvls_allreduce     row-parallel all-reduce over NVLink SHARP
 *   zcutlass_nvls_reduce_scatter   reduce-scatter over NVLink SHARP
 *   zcutlass_nvls_barrier       the collectives' cross-rank barrier alone
 *   zcutlass_gemm_gather_a      GEMM reading row blocks of A from several buffers
 *
 * Integer enum values equal the C++ enum values (Status, DType, LayoutKind).
 * Return values of type int that carry a status use zcutlass_status values.
 */
#ifndef ZCUTLASS_C_H_
#define ZCUTLASS_C_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* zcutlass::Status */
enum zcutlass_status {
  ZCUTLASS_SUCCESS = 0,
  ZCUTLASS_INVALID_ARGUMENT = 1,
  ZCUTLASS_NOT_SUPPORTED = 2,
  ZCUTLASS_RUNTIME_ERROR = 3
};

/* zcutlass::DType */
enum zcutlass_dtype {
  ZCUTLASS_F16 = 0,
  ZCUTLASS_BF16 = 1,
  ZCUTLASS_F32 = 2,
  ZCUTLASS_TF32 = 3,
  ZCUTLASS_E4M3 = 4,
  ZCUTLASS_E5M2 = 5,
  ZCUTLASS_E2M1 = 6
};

/* zcutlass::layout::LayoutKind */
enum zcutlass_layout { ZCUTLASS_ROW_MAJOR = 0, ZCUTLASS_COLUMN_MAJOR = 1 };

/* Field-for-field C image of zcutlass::GemmDesc (same order). `stream` is a
 * cudaStream_t passed as an opaque pointer (NULL = legacy default stream). */
typedef struct zcutlass_gemm_desc {
  int64_t m, n, k;
  int64_t lda, ldb, ldc, ldd;
  int32_t a_type, b_type, c_type, d_type;
  float alpha, beta;
  const void* bias;
  void* stream;
  int32_t a_layout, b_layout, c_layout, d_layout;
} zcutlass_gemm_desc;

int zcutlass_gemm(const zcutlass_gemm_desc* desc, const void* A, const void* B, const void* C,
                  void* D);

/* Row-major GEMM with every argument flat; all four tensors share `dtype`. */
int zcutlass_gemm_rowmajor(int64_t m, int64_t n, int64_t k, const void* A, int64_t lda,
                           const void* B, int64_t ldb, const void* C, int64_t ldc, void* D,
                           int64_t ldd, int32_t dtype, float alpha, float beta,
                           const void* bias, void* stream);

/* zcutlass_gemm with the rows of A gathered from `parts` (1..8) buffers; no
 * reference counterpart (see zcutlass::gemm_gather_a in
 * include/zcutlass/gemm/gemm.hpp for the contract). Returns
 * ZCUTLASS_NOT_SUPPORTED when the layout cannot be served by its kernels. */
int zcutlass_gemm_gather_a(const zcutlass_gemm_desc* desc, const void* const* a_parts, int32_t parts,
                           const void* B, const void* C, void* D);

int zcutlass_can_implement(const zcutlass_gemm_desc* desc, const void* A, const void* B,
                           const void* C, const void* D);
size_t zcutlass_get_workspace_size(const zcutlass_gemm_desc* desc);

const char* zcutlass_selected_kernel_name(const zcutlass_gemm_desc* desc);
const char* zcutlass_selected_kernel_family(const zcutlass_gemm_desc* desc);
const char* zcutlass_selected_kernel_path(const zcutlass_gemm_desc* desc);
int zcutlass_selected_kernel_tile_m(const zcutlass_gemm_desc* desc);
int zcutlass_selected_kernel_tile_n(const zcutlass_gemm_desc* desc);
int zcutlass_selected_kernel_tile_k(const zcutlass_gemm_desc* desc);
int zcutlass_selected_kernel_pipeline_stages(const zcutlass_gemm_desc* desc);
const char* zcutlass_selected_kernel_epilogue_kind(const zcutlass_gemm_desc* desc);
int zcutlass_registered_gemm_operation_count(void);

const char* zcutlass_status_to_string(int status);
const char* zcutlass_dtype_name(int dtype);
int zcutlass_dtype_bits(int dtype);
int zcutlass_version_major(void);
int zcutlass_version_minor(void);
int zcutlass_version_patch(void);

/* Device-side error word of the current device: 0 when clean, otherwise a code
 * (site * 16 + role) written by the first kernel whose bounded wait expired.
 * Synchronises the device. `clear` != 0 resets the word to 0 afterwards. */
int zcutlass_device_error(int clear);

/* Number of kernel launches this library has enqueued since load (all devices). */
uint64_t zcutlass_gemm_kernel_launches(void);

/* Decode GEMM that allocates nothing (no counterpart in the reference).
 *
 * For callers that cannot call cudaMalloc: code inside a custom allocator or
 * memory-pool callback (an allocation there would re-enter the allocator), and
 * serving processes that reserve all device memory at start-up and forbid any
 * device allocation afterwards. The regular entry points may
 * allocate a per-stream workspace the first time the stream-K decode kernel
 * runs on a stream; this one runs that kernel with its scratch in a fixed
 * 16 MiB array compiled into the library (every GPU that loads the library
 * holds it until the process exits) and calls no cudaMalloc, cudaFree or
 * allocating library routine.
 *
 *   D[M,N] = alpha * A[M,K] * B + beta * C + bias[N]   (f16/bf16, FP32 accumulate)
 *   B is [K,N] row-major (b_col_major = 0) or a [N,K] weight (b_col_major = 1).
 *
 * Limits: 1 <= M <= 64; A and B 16-byte aligned with lda, ldb multiples of 8;
 * N <= 1,048,576 (8192 tile counters of 128 columns in the first 64 KiB).
 * The FP32 partial tiles take 2 * G * MP * 512 bytes (G = min(#SMs,
 * ceil(N/128) * ceil(K/128)), MP = 16, 32 or 64 by M): at most 9.7 MB on a
 * 148-SM B200, always within the rest of the 16 MiB, so on B200 only M and N
 * limit a call. Anything outside these limits returns
 * ZCUTLASS_INVALID_ARGUMENT without launching; other argument errors return
 * the same codes as zcutlass_gemm.
 * The first call on each device looks up the scratch array's device address
 * (cudaGetSymbolAddress); make that first call before any stream capture.
 * All calls share the one array and each call clears the counters it uses
 * on `stream` before its kernel: calls whose kernels overlap on the GPU (on
 * different streams) race, so serialise them. */
int zcutlass_gemm_decode_noalloc(int64_t m, int64_t n, int64_t k, const void* A, int64_t lda,
                                 const void* B, int64_t ldb, int32_t b_col_major, const void* C,
                                 int64_t ldc, void* D, int64_t ldd, int32_t dtype, float alpha,
                                 float beta, const void* bias, void* stream);

/* Tensor-parallel all-reduce over NVLink SHARP (no reference counterpart: the
 * reference leaves the row-parallel all-reduce to vLLM/NCCL). Sums, in place,
 * `nbytes` (a multiple of 16) of f16/bf16 held at the same offset of a
 * symmetric buffer on every rank; `mc_ptr` is that data's multicast address
 * (16-byte aligned). Rank `rank` reduces its 1/world slice with FP32
 * accumulation in the switch and broadcasts it.
 *
 * The call brackets the reduction with two cross-rank barriers of its own
 * (every partial written before; every slice written after), kept in two
 * uint32 words of symmetric memory (8-byte aligned): `flag` is their local
 * address, `mc_flag` the multicast address of the first. Both words must be
 * 0 on every rank before the first call; word 0 counts arrivals from all
 * ranks, word 1 this rank's barriers. Calls that share the words must run in
 * one stream order on each rank, and every rank of the group must make the
 * same calls in the same order. The launches take no per-call state from the
 * host, so they may be captured in a CUDA graph and replayed. A barrier that
 * waits longer than two seconds gives up and sets the device error word
 * (zcutlass_device_error) instead of hanging.
 * Asynchronous on `stream` (three kernel launches). */
int zcutlass_nvls_allreduce(void* mc_ptr, int64_t nbytes, int32_t dtype, void* mc_flag, void* flag,
                            int32_t rank, int32_t world, void* stream);

/* The cross-rank barrier of the two collectives on its own (no reference
 * counterpart): same barrier words and contract. Every rank's earlier work on
 * `stream` is complete and visible to all ranks when it returns on the
 * stream (bounded wait: two seconds, then the device error word). */
int zcutlass_nvls_barrier(void* mc_flag, void* flag, int32_t world, void* stream);

/* Reduce-scatter over NVLink SHARP (no reference counterpart), for a
 * sequence-parallel layer: same buffer, barrier and ordering contract as
 * zcutlass_nvls_allreduce. `nbytes` (a multiple of 16 * world) is split into
 * `world` equal contiguous slices; rank r sums slice r over all ranks (FP32
 * accumulation in the switch) and stores it into its own copy, `local_ptr`
 * being the local address of the data `mc_ptr` maps. The other slices of the
 * local copy are left as they were. After the call returns on the stream,
 * every rank's slice is final on that rank (the closing barrier), so peers
 * may read it. */
int zcutlass_nvls_reduce_scatter(void* mc_ptr, void* local_ptr, int64_t nbytes, int32_t dtype, void* mc_flag,
                                 void* flag, int32_t rank, int32_t world, void* stream);

/* Failure-detection self test (no reference counterpart): launches one kernel
 * whose bounded mbarrier wait is never satisfied, with a limit of `timeout_us`
 * microseconds. The wait gives up, records an error code and the kernel
 * returns; the call synchronises and returns that code (non-zero), clearing
 * the error word, or -1 if CUDA itself failed. The device stays usable. */
int zcutlass_selftest_bounded_wait(uint32_t timeout_us);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* ZCUTLASS_C_H_ */
