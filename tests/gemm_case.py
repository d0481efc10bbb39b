"""Helpers shared by the GPU parity tests: one GEMM case run through the C ABI
(include/zcutlass_c.h) with device buffers from torch, checked against the
oracle. Mirrors run_case in the reference's tests/test_gemm.cu:263-411
(seeded inputs, padded leading dimensions, a sentinel-filled D whose padding
columns must stay untouched)."""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from oracle import oracle
from zcutlass_b200 import _native

SENTINEL = {oracle.F16: -7.5, oracle.BF16: -6.5}  # tests/test_gemm.cu:104-115
CODE = {"f16": oracle.F16, "bf16": oracle.BF16}


def to_device(bits: np.ndarray):
    import torch

    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).cuda()


def to_host(t) -> np.ndarray:
    return t.cpu().numpy().view(np.uint16)


@dataclass
class Case:
    name: str
    dtype: int
    m: int
    n: int
    k: int
    alpha: float = 1.0
    beta: float = 0.0
    bias: bool = False
    pad_a: int = 0
    pad_b: int = 0
    pad_c: int = 0
    pad_d: int = 0
    b_col_major: bool = False
    gen: str = "mt19937"  # "mt19937" = reference make_tensor; "normal" = BASELINE distributions
    seed: int = 0

    @property
    def lda(self) -> int:
        return self.k + self.pad_a

    @property
    def ldb(self) -> int:
        return (self.k if self.b_col_major else self.n) + self.pad_b

    @property
    def ldc(self) -> int:
        return self.n + self.pad_c

    @property
    def ldd(self) -> int:
        return self.n + self.pad_d


def make_inputs(c: Case):
    """Returns (A[m,lda], B (row-major [k,ldb] or col-major [n,ldb]), C[m,ldc], bias[n]) as uint16."""
    if c.gen == "mt19937":
        a = oracle.make_tensor(c.m, c.k, c.lda, 17, c.dtype)
        b = (oracle.make_tensor(c.n, c.k, c.ldb, 29, c.dtype) if c.b_col_major
             else oracle.make_tensor(c.k, c.n, c.ldb, 29, c.dtype))
        cm = oracle.make_tensor(c.m, c.n, c.ldc, 41, c.dtype)
        bias = oracle.make_tensor(1, c.n, c.n, 53, c.dtype)[0]
        return a, b, cm, bias
    rng = np.random.default_rng(c.seed)
    f = lambda x: oracle.float_to_bits(x.astype(np.float32), c.dtype)  # noqa: E731
    a = np.zeros((c.m, c.lda), np.float32)
    a[:, : c.k] = rng.standard_normal((c.m, c.k))
    shape_b = (c.n, c.ldb) if c.b_col_major else (c.k, c.ldb)
    b = np.zeros(shape_b, np.float32)
    if c.b_col_major:
        b[:, : c.k] = rng.standard_normal((c.n, c.k)) / np.sqrt(c.k)
    else:
        b[:, : c.n] = rng.standard_normal((c.k, c.n)) / np.sqrt(c.k)
    cm = np.zeros((c.m, c.ldc), np.float32)
    cm[:, : c.n] = rng.standard_normal((c.m, c.n))
    bias = rng.standard_normal(c.n) * 0.1
    return f(a), f(b), f(cm), f(bias)


def oracle_result(c: Case, a, b, cm, bias) -> np.ndarray:
    b_rm = np.ascontiguousarray(b[:, : c.k].T) if c.b_col_major else b
    return oracle.gemm(a, b_rm, c.m, c.n, c.k, c.dtype, c=cm, bias=bias if c.bias else None, alpha=c.alpha,
                       beta=c.beta, lda=c.lda, ldb=b_rm.shape[1], ldc=c.ldc)


def run_zcutlass(c: Case, a, b, cm, bias, *, rowmajor_entry: bool = False):
    """Runs the case through the C ABI; returns (status, D[m, ldd] uint16)."""
    import torch

    da, db, dc, dbias = to_device(a), to_device(b), to_device(cm), to_device(bias)
    d0 = np.full((c.m, c.ldd), oracle.float_to_bits(np.float32(SENTINEL[c.dtype]), c.dtype), np.uint16)
    dd = to_device(d0)
    cptr = dc.data_ptr() if c.beta != 0.0 else None
    bptr = dbias.data_ptr() if c.bias else None
    if rowmajor_entry:
        assert not c.b_col_major
        st = _native.gemm_rowmajor(c.m, c.n, c.k, da.data_ptr(), c.lda, db.data_ptr(), c.ldb, cptr, c.ldc,
                                   dd.data_ptr(), c.ldd, c.dtype, c.alpha, c.beta, bptr, None)
    else:
        desc = _native.make_desc(c.m, c.n, c.k, c.lda, c.ldb, c.ldc, c.ldd, c.dtype, c.alpha, c.beta, bptr,
                                 None, b_layout=_native.COLUMN_MAJOR if c.b_col_major else _native.ROW_MAJOR)
        st = _native.gemm(desc, da.data_ptr(), db.data_ptr(), cptr, dd.data_ptr())
    torch.cuda.synchronize()
    return st, to_host(dd)


def selected(c: Case) -> dict:
    desc = _native.make_desc(c.m, c.n, c.k, c.lda, c.ldb, c.ldc, c.ldd, c.dtype, c.alpha, c.beta,
                             256 if c.bias else None, None,
                             b_layout=_native.COLUMN_MAJOR if c.b_col_major else _native.ROW_MAJOR)
    return _native.selected_kernel(desc)


def check_case(c: Case, *, rowmajor_entry: bool = False) -> dict:
    """Runs one case and applies every check; returns metrics for reporting."""
    a, b, cm, bias = make_inputs(c)
    ref = oracle_result(c, a, b, cm, bias)
    st, d = run_zcutlass(c, a, b, cm, bias, rowmajor_entry=rowmajor_entry)
    assert st == _native.SUCCESS, f"{c.name}: status {_native.STATUS_NAMES.get(st, st)}"
    assert _native.device_error(clear=True) == 0, f"{c.name}: device-side wait timed out"
    out = oracle.bits_to_float(d[:, : c.n], c.dtype)
    # padding columns of D are never written (tests/test_gemm.cu:392-403)
    if c.ldd > c.n:
        pad = d[:, c.n:]
        bad = np.argwhere(pad != d.dtype.type(oracle.float_to_bits(np.float32(SENTINEL[c.dtype]), c.dtype)))
        assert bad.size == 0, (f"{c.name}: output padding overwritten at {bad.shape[0]} places, "
                               f"first (row, col) {tuple(int(v) for v in bad[0]) if bad.size else None} "
                               f"(col relative to n={c.n})")
    # reference test tolerance (absolute) and the product bounds
    max_abs = float(np.max(np.abs(out - ref))) if out.size else 0.0
    assert max_abs <= oracle.REF_ABS_TOL[c.dtype], f"{c.name}: max_abs {max_abs}"
    m = oracle.check(out, ref, c.dtype)
    m["kernel"] = selected(c)["kernel_name"]
    return m
