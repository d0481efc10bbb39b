"""TEST INFRASTRUCTURE ONLY: numpy/ctypes front end of oracle/liboracle.so.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import
this module; the product never does. It restates the reference's host GEMM
(tests/test_gemm.cu:130-162 in supercatking/zcutlass) and its seeded input
generator (tests/test_gemm.cu:118-128); see oracle/gemm_oracle.cpp for the
exact arithmetic.

Parity pins (checked by tests/test_oracle.py):
  * tests/golden/*.npz: inputs and outputs of the reference's own CPU path
    (python/zcutlass_torch/overlay.py _fallback / linear, run in this
    container by tests/golden/make_golden.py);
  * on a GPU box, the reference library itself (oracle/_ref/libzcutlass_ref.so,
    built from its src/*.cu) on the reference test cases.

Error metrics named by the product spec:
  rel_frobenius(out, ref) = ||out - ref||_F / ||ref||_F   (<= 1e-3 f16, <= 5e-3 bf16)
  |out - ref| <= 4 * ulp(out) * (1 + |ref|) elementwise, where ulp(out) is the
      unit in the last place of the output type at 1.0 (2^-10 for f16, 2^-7
      for bf16). The (1 + |ref|) factor makes the bound absolute near zero and
      relative for large values. (Reading ulp at the magnitude of each output
      instead would fail every result that cancels to near zero, whatever the
      summation order: there the FP32 accumulation error is ~1e-7 absolute.)
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_SO = HERE / "_ref" / "libzcutlass_ref.so"

F16, BF16 = 0, 1
# Reference test tolerances (tests/test_gemm.cu:91-102): absolute.
REF_ABS_TOL = {F16: 0.16, BF16: 0.55}
# Product tolerances (relative Frobenius).
REL_FRO_TOL = {F16: 1e-3, BF16: 5e-3}
MANTISSA_BITS = {F16: 10, BF16: 7}
MIN_NORMAL_EXP = {F16: -14, BF16: -126}

_u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(dtype=np.int64, flags="C_CONTIGUOUS")
_LIB = None


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not ORACLE_SO.exists():
            raise ImportError(f"{ORACLE_SO} missing: run `make -C oracle`")
        L = ctypes.CDLL(str(ORACLE_SO))
        L.oracle_make_tensor.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                                         ctypes.c_int, _u16p]
        L.oracle_make_tensor.restype = None
        L.oracle_gemm.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _u16p, ctypes.c_int64,
                                  _u16p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                                  ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_int, _f32p]
        L.oracle_gemm.restype = None
        L.oracle_gemm_f64_rows.argtypes = [ctypes.c_int64, ctypes.c_int64, _u16p, ctypes.c_int64, _u16p,
                                           ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                                           ctypes.c_float, ctypes.c_float, ctypes.c_int, _i64p,
                                           ctypes.c_int64, _f64p]
        L.oracle_gemm_f64_rows.restype = None
        L.oracle_float_to_bits.argtypes = [ctypes.c_float, ctypes.c_int]
        L.oracle_float_to_bits.restype = ctypes.c_uint16
        L.oracle_bits_to_float.argtypes = [ctypes.c_uint16, ctypes.c_int]
        L.oracle_bits_to_float.restype = ctypes.c_float
        _LIB = L
    return _LIB


def make_tensor(rows: int, cols: int, ld: int, seed: int, dtype: int) -> np.ndarray:
    """Reference make_tensor<T>: [rows, ld] uint16 bit patterns, padding = 0."""
    out = np.empty((rows, ld), dtype=np.uint16)
    lib().oracle_make_tensor(rows, cols, ld, seed, dtype, out)
    return out


def bits_to_float(bits: np.ndarray, dtype: int) -> np.ndarray:
    """Exact widening of f16/bf16 bit patterns to float32 (numpy, no oracle call)."""
    b = np.ascontiguousarray(bits, dtype=np.uint16)
    if dtype == BF16:
        return (b.astype(np.uint32) << 16).view(np.float32)
    return b.view(np.float16).astype(np.float32)


def float_to_bits(x: np.ndarray, dtype: int) -> np.ndarray:
    """Round-to-nearest-even narrowing of float32 to f16/bf16 bit patterns."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if dtype == F16:
        with np.errstate(over="ignore"):  # values beyond the f16 range become inf, as in the kernels
            return x.astype(np.float16).view(np.uint16)
    u = x.view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def gemm(a: np.ndarray, b: np.ndarray, m: int, n: int, k: int, dtype: int, *, c: np.ndarray | None = None,
         bias: np.ndarray | None = None, alpha: float = 1.0, beta: float = 0.0, threads: int | None = None,
         lda: int | None = None, ldb: int | None = None, ldc: int | None = None) -> np.ndarray:
    """Reference GEMM on uint16 bit patterns; returns float32 [m, n] (already
    rounded to the storage type). a: [m, lda], b: [k, ldb], c: [m, ldc]."""
    a = np.ascontiguousarray(a, dtype=np.uint16)
    b = np.ascontiguousarray(b, dtype=np.uint16)
    lda = a.shape[1] if lda is None else lda
    ldb = b.shape[1] if ldb is None else ldb
    cp = None
    if beta != 0.0:
        if c is None:
            raise ValueError("beta != 0 needs C")
        c = np.ascontiguousarray(c, dtype=np.uint16)
        ldc = c.shape[1] if ldc is None else ldc
        cp = c.ctypes.data
    biasp = None
    if bias is not None:
        bias = np.ascontiguousarray(bias, dtype=np.uint16)
        biasp = bias.ctypes.data
    out = np.empty((m, n), dtype=np.float32)
    threads = threads if threads is not None else min(os.cpu_count() or 1, 32)
    lib().oracle_gemm(m, n, k, a, lda, b, ldb, cp, ldc or n, biasp, alpha, beta, dtype, threads, out)
    return out


def gemm_f64_rows(a: np.ndarray, b: np.ndarray, rows: np.ndarray, n: int, k: int, dtype: int, *,
                  c: np.ndarray | None = None, bias: np.ndarray | None = None, alpha: float = 1.0,
                  beta: float = 0.0) -> np.ndarray:
    """FP64-accumulated, unrounded rows of the same GEMM: [len(rows), n]."""
    a = np.ascontiguousarray(a, dtype=np.uint16)
    b = np.ascontiguousarray(b, dtype=np.uint16)
    rows = np.ascontiguousarray(rows, dtype=np.int64)
    cp, ldc = None, n
    if beta != 0.0:
        c = np.ascontiguousarray(c, dtype=np.uint16)
        cp, ldc = c.ctypes.data, c.shape[1]
    biasp = None
    if bias is not None:
        bias = np.ascontiguousarray(bias, dtype=np.uint16)
        biasp = bias.ctypes.data
    out = np.empty((rows.shape[0], n), dtype=np.float64)
    lib().oracle_gemm_f64_rows(n, k, a, a.shape[1], b, b.shape[1], cp, ldc, biasp, alpha, beta, dtype, rows,
                               rows.shape[0], out)
    return out


def ulp(x: np.ndarray, dtype: int) -> np.ndarray:
    """Spacing of the storage type at |x| (subnormal spacing below the normal range)."""
    ax = np.abs(np.asarray(x, dtype=np.float64))
    e = np.floor(np.log2(np.maximum(ax, 2.0 ** MIN_NORMAL_EXP[dtype])))
    return np.exp2(e - MANTISSA_BITS[dtype])


def rel_frobenius(out: np.ndarray, ref: np.ndarray) -> float:
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    denom = np.linalg.norm(ref)
    return float(np.linalg.norm(out - ref) / (denom if denom > 0 else 1.0))


def type_ulp(dtype: int) -> float:
    """Unit in the last place of the storage type at 1.0."""
    return 2.0 ** -MANTISSA_BITS[dtype]


def max_abs_violation(out: np.ndarray, ref: np.ndarray, dtype: int, ulps: float = 4.0) -> float:
    """max(|out-ref| / (ulps * ulp_T * (1+|ref|))); <= 1 passes."""
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    bound = ulps * type_ulp(dtype) * (1.0 + np.abs(ref))
    return float(np.max(np.abs(out - ref) / bound)) if out.size else 0.0


def check(out: np.ndarray, ref: np.ndarray, dtype: int, *, rel_tol: float | None = None,
          ulps: float = 4.0) -> dict:
    """Applies both product bounds; returns the metrics (raises AssertionError on failure)."""
    rel = rel_frobenius(out, ref)
    viol = max_abs_violation(out, ref, dtype, ulps)
    tol = REL_FRO_TOL[dtype] if rel_tol is None else rel_tol
    metrics = {"rel_frobenius": rel, "max_abs_bound_ratio": viol,
               "max_abs": float(np.max(np.abs(np.asarray(out, np.float64) - ref))) if np.size(out) else 0.0}
    assert np.all(np.isfinite(out)), f"non-finite output {metrics}"
    assert rel <= tol, f"relative Frobenius error {rel:.3e} > {tol:.1e} {metrics}"
    assert viol <= 1.0, f"max-abs error beyond {ulps} ulp*(1+|ref|) {metrics}"
    return metrics


class RefLib:
    """The reference library built from its own sources (GPU box only)."""

    def __init__(self) -> None:
        if not REF_SO.exists():
            raise ImportError(f"{REF_SO} missing: run `make -C oracle ref` where the reference is present")
        L = ctypes.CDLL(str(REF_SO))
        v, i64 = ctypes.c_void_p, ctypes.c_int64
        L.zref_gemm.argtypes = [i64, i64, i64, v, i64, v, i64, v, i64, v, i64, ctypes.c_int, ctypes.c_float,
                                ctypes.c_float, v, v]
        L.zref_gemm.restype = ctypes.c_int
        L.zref_selected_kernel_name.argtypes = [i64, i64, i64, i64, i64, i64, i64, ctypes.c_int,
                                                ctypes.c_float, ctypes.c_float, v]
        L.zref_selected_kernel_name.restype = ctypes.c_char_p
        self.lib = L

    def gemm(self, m, n, k, a, lda, b, ldb, c, ldc, d, ldd, dtype, alpha, beta, bias, stream=None) -> int:
        return self.lib.zref_gemm(m, n, k, a, lda, b, ldb, c, ldc, d, ldd, dtype, alpha, beta, bias, stream)

    def selected_kernel_name(self, m, n, k, lda, ldb, ldc, ldd, dtype, alpha=1.0, beta=0.0, bias=None) -> str:
        return self.lib.zref_selected_kernel_name(m, n, k, lda, ldb, ldc, ldd, dtype, alpha, beta,
                                                  bias).decode()
