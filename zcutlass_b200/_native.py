"""ctypes binding of the C ABI in include/zcutlass_c.h (libzcutlass.so).

This is the FFI a non-C++ host binds; tests call the kernels through it with
raw device pointers. The library is loaded from this package directory only
(an in-tree build, see zcutlass_b200/build.py); if it is missing the import
fails loudly -- there is no fallback implementation.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

PKG = Path(__file__).resolve().parent
CORE_SO = PKG / "libzcutlass.so"

# zcutlass::Status
SUCCESS, INVALID_ARGUMENT, NOT_SUPPORTED, RUNTIME_ERROR = 0, 1, 2, 3
STATUS_NAMES = {0: "Success", 1: "InvalidArgument", 2: "NotSupported", 3: "RuntimeError"}
# zcutlass::DType
F16, BF16, F32, TF32, E4M3, E5M2, E2M1 = range(7)
# zcutlass::layout::LayoutKind
ROW_MAJOR, COLUMN_MAJOR = 0, 1


class GemmDesc(ctypes.Structure):
    """Field-for-field image of zcutlass_gemm_desc / zcutlass::GemmDesc."""

    _fields_ = [
        ("m", ctypes.c_int64),
        ("n", ctypes.c_int64),
        ("k", ctypes.c_int64),
        ("lda", ctypes.c_int64),
        ("ldb", ctypes.c_int64),
        ("ldc", ctypes.c_int64),
        ("ldd", ctypes.c_int64),
        ("a_type", ctypes.c_int32),
        ("b_type", ctypes.c_int32),
        ("c_type", ctypes.c_int32),
        ("d_type", ctypes.c_int32),
        ("alpha", ctypes.c_float),
        ("beta", ctypes.c_float),
        ("bias", ctypes.c_void_p),
        ("stream", ctypes.c_void_p),
        ("a_layout", ctypes.c_int32),
        ("b_layout", ctypes.c_int32),
        ("c_layout", ctypes.c_int32),
        ("d_layout", ctypes.c_int32),
    ]


def make_desc(m, n, k, lda, ldb, ldc, ldd, dtype, alpha=1.0, beta=0.0, bias=None, stream=None,
              a_layout=ROW_MAJOR, b_layout=ROW_MAJOR, c_layout=ROW_MAJOR, d_layout=ROW_MAJOR,
              a_type=None, b_type=None, c_type=None, d_type=None) -> GemmDesc:
    """Builds a GemmDesc the way the reference tests brace-initialise one."""
    return GemmDesc(m, n, k, lda, ldb, ldc, ldd,
                    dtype if a_type is None else a_type, dtype if b_type is None else b_type,
                    dtype if c_type is None else c_type, dtype if d_type is None else d_type,
                    alpha, beta, bias, stream, a_layout, b_layout, c_layout, d_layout)


_P = ctypes.POINTER(GemmDesc)
_v = ctypes.c_void_p
_i64 = ctypes.c_int64

# name -> (restype, argtypes); every symbol include/zcutlass_c.h declares.
SIGNATURES = {
    "zcutlass_gemm": (ctypes.c_int, [_P, _v, _v, _v, _v]),
    "zcutlass_gemm_rowmajor": (ctypes.c_int, [_i64, _i64, _i64, _v, _i64, _v, _i64, _v, _i64, _v, _i64,
                                              ctypes.c_int32, ctypes.c_float, ctypes.c_float, _v, _v]),
    "zcutlass_can_implement": (ctypes.c_int, [_P, _v, _v, _v, _v]),
    "zcutlass_gemm_gather_a": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_void_p), ctypes.c_int32, _v, _v, _v]),
    "zcutlass_get_workspace_size": (ctypes.c_size_t, [_P]),
    "zcutlass_selected_kernel_name": (ctypes.c_char_p, [_P]),
    "zcutlass_selected_kernel_family": (ctypes.c_char_p, [_P]),
    "zcutlass_selected_kernel_path": (ctypes.c_char_p, [_P]),
    "zcutlass_selected_kernel_tile_m": (ctypes.c_int, [_P]),
    "zcutlass_selected_kernel_tile_n": (ctypes.c_int, [_P]),
    "zcutlass_selected_kernel_tile_k": (ctypes.c_int, [_P]),
    "zcutlass_selected_kernel_pipeline_stages": (ctypes.c_int, [_P]),
    "zcutlass_selected_kernel_epilogue_kind": (ctypes.c_char_p, [_P]),
    "zcutlass_registered_gemm_operation_count": (ctypes.c_int, []),
    "zcutlass_status_to_string": (ctypes.c_char_p, [ctypes.c_int]),
    "zcutlass_dtype_name": (ctypes.c_char_p, [ctypes.c_int]),
    "zcutlass_dtype_bits": (ctypes.c_int, [ctypes.c_int]),
    "zcutlass_version_major": (ctypes.c_int, []),
    "zcutlass_version_minor": (ctypes.c_int, []),
    "zcutlass_version_patch": (ctypes.c_int, []),
    "zcutlass_device_error": (ctypes.c_int, [ctypes.c_int]),
    "zcutlass_gemm_kernel_launches": (ctypes.c_uint64, []),
    "zcutlass_selftest_bounded_wait": (ctypes.c_int, [ctypes.c_uint32]),
    "zcutlass_nvls_allreduce": (ctypes.c_int, [_v, _i64, ctypes.c_int32, _v, _v, ctypes.c_int32, ctypes.c_int32,
                                               _v]),
    "zcutlass_nvls_barrier": (ctypes.c_int, [_v, _v, ctypes.c_int32, _v]),
    "zcutlass_nvls_reduce_scatter": (ctypes.c_int, [_v, _v, _i64, ctypes.c_int32, _v, _v, ctypes.c_int32,
                                                    ctypes.c_int32, _v]),
    "zcutlass_gemm_decode_noalloc": (ctypes.c_int, [_i64, _i64, _i64, _v, _i64, _v, _i64, ctypes.c_int32, _v, _i64,
                                                    _v, _i64, ctypes.c_int32, ctypes.c_float, ctypes.c_float, _v,
                                                    _v]),
}

_LIB: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """Loads libzcutlass.so (once) and declares every exported signature."""
    global _LIB
    if _LIB is None:
        if not CORE_SO.exists():
            raise ImportError(
                f"{CORE_SO} is missing: build it with `python -m zcutlass_b200.build` "
                "(there is no non-native fallback)")
        handle = ctypes.CDLL(str(CORE_SO))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = handle
    return _LIB


def _s(b: bytes | None) -> str:
    return b.decode() if b is not None else "null"


def gemm(desc: GemmDesc, a, b, c, d) -> int:
    return lib().zcutlass_gemm(ctypes.byref(desc), a, b, c, d)


def gemm_rowmajor(m, n, k, a, lda, b, ldb, c, ldc, d, ldd, dtype, alpha=1.0, beta=0.0, bias=None,
                  stream=None) -> int:
    return lib().zcutlass_gemm_rowmajor(m, n, k, a, lda, b, ldb, c, ldc, d, ldd, dtype, alpha, beta,
                                        bias, stream)


def gemm_gather_a(desc: GemmDesc, a_parts, b, c, d) -> int:
    """zcutlass_gemm_gather_a: rows of A in len(a_parts) row blocks, block i read from a_parts[i]."""
    arr = (ctypes.c_void_p * max(1, len(a_parts)))(*a_parts)
    return lib().zcutlass_gemm_gather_a(ctypes.byref(desc), arr, len(a_parts), b, c, d)


def can_implement(desc: GemmDesc, a, b, c, d) -> int:
    return lib().zcutlass_can_implement(ctypes.byref(desc), a, b, c, d)


def get_workspace_size(desc: GemmDesc) -> int:
    return int(lib().zcutlass_get_workspace_size(ctypes.byref(desc)))


def selected_kernel(desc: GemmDesc) -> dict:
    """All selection telemetry for one descriptor (host only, nothing launches)."""
    L = lib()
    r = ctypes.byref(desc)
    return {
        "kernel_name": _s(L.zcutlass_selected_kernel_name(r)),
        "shape_family": _s(L.zcutlass_selected_kernel_family(r)),
        "kernel_path": _s(L.zcutlass_selected_kernel_path(r)),
        "tile": {"m": L.zcutlass_selected_kernel_tile_m(r), "n": L.zcutlass_selected_kernel_tile_n(r),
                 "k": L.zcutlass_selected_kernel_tile_k(r)},
        "pipeline_stages": L.zcutlass_selected_kernel_pipeline_stages(r),
        "epilogue_kind": _s(L.zcutlass_selected_kernel_epilogue_kind(r)),
        "registered_gemm_operations": L.zcutlass_registered_gemm_operation_count(),
    }


def status_name(status: int) -> str:
    return _s(lib().zcutlass_status_to_string(status))


def version() -> tuple[int, int, int]:
    L = lib()
    return (L.zcutlass_version_major(), L.zcutlass_version_minor(), L.zcutlass_version_patch())


def device_error(clear: bool = True) -> int:
    return lib().zcutlass_device_error(1 if clear else 0)


def kernel_launches() -> int:
    return int(lib().zcutlass_gemm_kernel_launches())
