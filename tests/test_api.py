"""Host-side contract of libzcutlass.so, checked without a GPU.

Every call here returns before any CUDA work: argument validation, zero-size
problems and selection telemetry are host-only. Follows the reference's
run_invalid_argument_tests / run_zero_size_tests / run_dispatch_tests
(tests/test_gemm.cu:438-733 in supercatking/zcutlass), with the dispatch
expectations re-derived for this library's sm_100a operation table (selection
answers for a B200 when no device is visible).
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from zcutlass_b200 import _native as N

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "zcutlass_c.h"
P = 0x100  # dummy 16-byte-aligned, non-null pointer: never dereferenced here


def header_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(zcutlass_[a-z_0-9]+)\s*\(", text)))


def test_library_exports_every_header_symbol():
    lib = N.lib()
    names = header_functions()
    assert len(names) >= 20
    for name in names:
        assert hasattr(lib, name), f"{name} declared in include/zcutlass_c.h but not exported"
    assert set(names) == set(N.SIGNATURES), "ctypes binding and header disagree"


def test_torch_ops_library_present():
    assert (ROOT / "zcutlass_b200" / "libzcutlass_torch.so").exists()


def test_version_and_names():
    assert N.version() == (0, 2, 0)
    L = N.lib()
    assert [N.status_name(i) for i in range(4)] == ["Success", "InvalidArgument", "NotSupported", "RuntimeError"]
    assert [L.zcutlass_dtype_name(i).decode() for i in range(7)] == ["f16", "bf16", "f32", "tf32", "e4m3", "e5m2",
                                                                      "e2m1"]
    assert [L.zcutlass_dtype_bits(i) for i in range(7)] == [16, 16, 32, 32, 8, 8, 4]


def desc16(**kw):
    base = dict(m=16, n=16, k=16, lda=16, ldb=16, ldc=16, ldd=16, dtype=N.F16)
    base.update(kw)
    return N.make_desc(**base)


def test_invalid_arguments():
    # tests/test_gemm.cu:475-567, same order and codes
    d = desc16()
    assert N.gemm(d, None, P, None, P) == N.INVALID_ARGUMENT  # null A
    assert N.gemm(d, P, None, None, P) == N.INVALID_ARGUMENT  # null B
    assert N.gemm(d, P, P, None, None) == N.INVALID_ARGUMENT  # null D
    assert N.gemm(desc16(beta=1.0), P, P, None, P) == N.INVALID_ARGUMENT  # beta without C
    assert N.gemm(desc16(m=-1), P, P, None, P) == N.INVALID_ARGUMENT
    assert N.gemm(desc16(lda=15), P, P, None, P) == N.INVALID_ARGUMENT
    assert N.gemm(desc16(ldb=15), P, P, None, P) == N.INVALID_ARGUMENT
    assert N.gemm(desc16(ldd=15), P, P, None, P) == N.INVALID_ARGUMENT
    assert N.gemm(desc16(beta=1.0, ldc=15), P, P, P, P) == N.INVALID_ARGUMENT
    assert N.gemm(desc16(b_type=N.BF16), P, P, None, P) == N.NOT_SUPPORTED  # mixed dtypes
    assert N.gemm(desc16(dtype=N.F32), P, P, None, P) == N.NOT_SUPPORTED
    assert N.gemm(desc16(a_layout=N.COLUMN_MAJOR), P, P, None, P) == N.NOT_SUPPORTED
    assert N.gemm(desc16(d_layout=N.COLUMN_MAJOR), P, P, None, P) == N.NOT_SUPPORTED
    assert N.gemm(desc16(c_layout=N.COLUMN_MAJOR), P, P, None, P) == N.NOT_SUPPORTED
    # column-major B is accepted (extension) but then needs ldb >= K
    assert N.can_implement(desc16(b_layout=N.COLUMN_MAJOR, n=32, ldb=16, ldc=32, ldd=32), P, P, None, P) == N.SUCCESS
    assert N.can_implement(desc16(b_layout=N.COLUMN_MAJOR, k=32, lda=32, ldb=16), P, P, None, P) == \
        N.INVALID_ARGUMENT
    # flat entry point validates the same way
    assert N.gemm_rowmajor(16, 16, 16, None, 16, P, 16, None, 16, P, 16, N.F16) == N.INVALID_ARGUMENT
    assert N.lib().zcutlass_gemm(None, P, P, None, P) == N.INVALID_ARGUMENT


def test_can_implement_and_workspace():
    d = desc16()
    assert N.can_implement(d, P, P, None, P) == N.SUCCESS
    assert N.get_workspace_size(d) == 0


@pytest.mark.parametrize("dtype", [N.F16, N.BF16])
def test_zero_sizes_succeed_without_touching_memory(dtype):
    # tests/test_gemm.cu:438-473: null tensors are fine when there is no work
    assert N.gemm(desc16(m=0, dtype=dtype), None, None, None, None) == N.SUCCESS
    assert N.gemm(desc16(n=0, dtype=dtype), None, None, None, None) == N.SUCCESS
    assert N.gemm(desc16(k=0, beta=1.0, dtype=dtype), None, None, None, None) == N.SUCCESS


def sel(m, n, k, dtype=N.BF16, **kw):
    lda = kw.pop("lda", k)
    ldb = kw.pop("ldb", n)
    return N.selected_kernel(N.make_desc(m, n, k, lda, ldb, n, n, dtype, **kw))


def test_registered_operation_count():
    assert N.lib().zcutlass_registered_gemm_operation_count() == 30


def test_shape_families_follow_reference_rules():
    # classify_shape_family (src/gemm.cu:480-496)
    assert sel(8, 4096, 4096)["shape_family"] == "decode"
    assert sel(128, 4096, 4096)["shape_family"] == "prefill"
    assert sel(4096, 4096, 4096)["shape_family"] == "large"
    assert sel(8, 256, 256)["shape_family"] == "fallback"
    assert sel(4096, 4096, 4096, beta=1.0)["shape_family"] == "fallback"
    assert sel(64, 256, 256, lda=260)["shape_family"] == "fallback"


def test_dispatch_table_on_b200():
    big = sel(8192, 28672, 4096)
    assert "256x256x64_2cta_persistent" in big["kernel_name"]
    assert big["kernel_path"] == "fast" and big["epilogue_kind"] == "tmem_register_tma"
    assert big["tile"] == {"m": 256, "n": 256, "k": 64} and big["pipeline_stages"] == 3
    assert "bf16_16x128x64_swapab" in sel(8, 4096, 4096)["kernel_name"]
    assert "f16_32x128x64_swapab" in sel(20, 4096, 4096, dtype=N.F16)["kernel_name"]
    assert "64x128x64_swapab" in sel(64, 1024, 1024)["kernel_name"]
    # mid-M: too few output tiles for 148 SMs -> cluster split-K
    assert "128x128x64_splitk_cluster" in sel(256, 4096, 4096)["kernel_name"]
    assert "128x128x64_splitk_cluster" in sel(128, 4096, 4096)["kernel_name"]
    # one wave of 128 x 128 tiles with the two-block stages beats splitting K
    assert "128x128x64_ws_persistent" in sel(512, 4096, 4096)["kernel_name"]
    assert "128x64x64_ws_persistent" in sel(1024, 1024, 1024)["kernel_name"]
    assert "_persistent" in sel(4096, 2048, 1536)["kernel_name"]  # 128 pair tiles: no split
    # layouts TMA cannot describe go to the predicated kernel
    padded = sel(64, 256, 256, lda=259)
    assert "generic" in padded["kernel_name"] and padded["kernel_path"] == "fallback"
    assert "generic" in sel(15, 17, 19)["kernel_name"]
    # column-major B selects the same families
    col = N.selected_kernel(N.make_desc(8192, 4096, 4096, 4096, 4096, 4096, 4096, N.BF16,
                                        b_layout=N.COLUMN_MAJOR))
    assert "2cta" in col["kernel_name"]
    # invalid descriptors report "none"
    assert sel(-1, 16, 16)["kernel_name"] == "none"


def test_force_kernel_filter(monkeypatch):
    monkeypatch.setenv("ZCUTLASS_FORCE_KERNEL", "_128x256x64_ws")
    assert "128x256x64_ws_persistent" in sel(8192, 8192, 8192)["kernel_name"]
    monkeypatch.setenv("ZCUTLASS_FORCE_KERNEL", "_generic")
    assert "generic" in sel(8192, 8192, 8192)["kernel_name"]
    monkeypatch.setenv("ZCUTLASS_FORCE_KERNEL", "no_such_kernel")
    assert sel(8192, 8192, 8192)["kernel_name"] == "none"


def test_experimental_flags_do_not_change_default_dispatch(monkeypatch):
    base = sel(128, 4096, 4096)["kernel_name"]
    monkeypatch.setenv("ZCUTLASS_EXPERIMENTAL_KERNELS", "1")
    monkeypatch.setenv("ZCUTLASS_EXPERIMENTAL_KERNEL", "anything")
    assert sel(128, 4096, 4096)["kernel_name"] == base


def test_experimental_streamk_decode(monkeypatch):
    # the stream-K decode family is experimental (reference semantics: gated by
    # ZCUTLASS_EXPERIMENTAL_KERNELS and the ZCUTLASS_EXPERIMENTAL_KERNEL filter)
    d = sel(16, 7168, 8192)
    assert "swapab_splitk" in d["kernel_name"] and d["kernel_path"] == "fast"
    monkeypatch.setenv("ZCUTLASS_EXPERIMENTAL_KERNELS", "1")
    e = sel(16, 7168, 8192)
    assert "swapab_streamk" in e["kernel_name"] and e["kernel_path"] == "experimental_fast"
    monkeypatch.setenv("ZCUTLASS_EXPERIMENTAL_KERNEL", "no_match")
    assert "swapab_splitk" in sel(16, 7168, 8192)["kernel_name"]


def test_gemm_desc_layout_matches_c_header():
    # field order and sizes of zcutlass_gemm_desc (positional brace-init in C++)
    names = [f[0] for f in N.GemmDesc._fields_]
    assert names[:7] == ["m", "n", "k", "lda", "ldb", "ldc", "ldd"]
    assert names[7:11] == ["a_type", "b_type", "c_type", "d_type"]
    assert ctypes.sizeof(N.GemmDesc) == 7 * 8 + 4 * 4 + 2 * 4 + 2 * 8 + 4 * 4


def test_gather_a_argument_checks():
    """zcutlass_gemm_gather_a rejects bad part lists and layouts its kernels
    cannot serve before launching anything (no GPU needed)."""
    P = 1 << 20  # 16-byte aligned dummy addresses; nothing is dereferenced on these paths

    def call(m, n, k, parts, *, col=True, ptrs=None):
        desc = N.make_desc(m, n, k, k, k if col else n, n, n, N.BF16,
                           b_layout=N.COLUMN_MAJOR if col else N.ROW_MAJOR)
        ptrs = [P * (i + 1) for i in range(parts)] if ptrs is None else ptrs
        arr = (ctypes.c_void_p * max(1, len(ptrs)))(*ptrs)
        return N.lib().zcutlass_gemm_gather_a(ctypes.byref(desc), arr, parts, P * 16, None, P * 32)

    assert call(1024, 1024, 1024, 0, ptrs=[P]) == N.INVALID_ARGUMENT
    assert call(1024, 1024, 1024, 9) == N.INVALID_ARGUMENT
    assert call(1024, 1024, 1024, 2, ptrs=[P, None]) == N.INVALID_ARGUMENT
    assert call(1024, 1024, 1024, 4, col=False) == N.NOT_SUPPORTED      # B must be a [N, K] weight
    assert call(1000, 1024, 1024, 8) == N.NOT_SUPPORTED                 # 125-row blocks split tiles
    assert call(1024, 1024, 1024, 3) == N.NOT_SUPPORTED                 # M not a multiple of parts
    assert call(0, 1024, 1024, 4) == N.SUCCESS                          # zero size: nothing to do
    assert N.lib().zcutlass_gemm_gather_a(None, None, 1, None, None, None) == N.INVALID_ARGUMENT


def test_nvls_collective_argument_checks():
    lib = N.lib()
    flag = 1 << 20
    assert lib.zcutlass_nvls_reduce_scatter(None, flag, 4096, N.BF16, flag, flag, 0, 2, None) == N.INVALID_ARGUMENT
    # 4096 + 16 bytes do not split into 2 slices of whole 16-byte words
    assert lib.zcutlass_nvls_reduce_scatter(flag, flag, 4096 + 16, N.BF16, flag, flag, 0, 2, None) == \
        N.INVALID_ARGUMENT
    assert lib.zcutlass_nvls_reduce_scatter(flag, flag, 4096, N.BF16, flag, flag, 2, 2, None) == \
        N.INVALID_ARGUMENT  # rank out of range
    assert lib.zcutlass_nvls_reduce_scatter(flag, flag, 4096, N.F32, flag, flag, 0, 2, None) == N.NOT_SUPPORTED
    assert lib.zcutlass_nvls_allreduce(flag, 4096, N.BF16, flag, flag + 4, 0, 2, None) == \
        N.INVALID_ARGUMENT  # barrier words must be 8-byte aligned
    assert lib.zcutlass_nvls_barrier(None, flag, 2, None) == N.INVALID_ARGUMENT
