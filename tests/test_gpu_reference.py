"""The reference library itself on the B200, as a second checker.

oracle/_ref/libzcutlass_ref.so is the reference's own src/*.cu compiled for
sm_100a (oracle/Makefile); on compute capability 10.0 it dispatches to its
WMMA kernels. On the reference's own test cases (tests/test_gemm.cu:754-786)
its output must agree with the oracle under the reference test's tolerance,
which pins the oracle to the reference's device arithmetic, and our kernels
must agree with both. A timing comparison on the layer shapes is printed.
"""

from __future__ import annotations

import numpy as np
import pytest

from gemm_case import Case, SENTINEL, make_inputs, oracle_result, run_zcutlass, to_device, to_host
from oracle import oracle
from test_gpu_gemm import REFERENCE_CASES
from zcutlass_b200 import _native


@pytest.fixture(scope="module")
def ref_lib():
    try:
        return oracle.RefLib()
    except ImportError as exc:
        pytest.skip(str(exc))


def run_reference(ref, c: Case, a, b, cm, bias):
    import torch

    da, db, dc, dbias = to_device(a), to_device(b), to_device(cm), to_device(bias)
    dd = to_device(np.full((c.m, c.ldd), oracle.float_to_bits(np.float32(SENTINEL[c.dtype]), c.dtype), np.uint16))
    st = ref.gemm(c.m, c.n, c.k, da.data_ptr(), c.lda, db.data_ptr(), c.ldb,
                  dc.data_ptr() if c.beta != 0.0 else None, c.ldc, dd.data_ptr(), c.ldd, c.dtype, c.alpha, c.beta,
                  dbias.data_ptr() if c.bias else None, None)
    torch.cuda.synchronize()
    return st, to_host(dd)


@pytest.mark.gpu
@pytest.mark.parametrize("case", REFERENCE_CASES, ids=[c[0] for c in REFERENCE_CASES])
def test_reference_library_agrees_with_oracle_and_ours(cuda_device, ref_lib, case):
    name, dt, m, n, k, alpha, beta, bias, pads = case
    c = Case(name, dt, m, n, k, alpha, beta, bias, *pads)
    a, b, cm, bv = make_inputs(c)
    expect = oracle_result(c, a, b, cm, bv)
    st, d_ref = run_reference(ref_lib, c, a, b, cm, bv)
    assert st == 0, f"reference status {st}"
    ref_out = oracle.bits_to_float(d_ref[:, :n], dt)
    # the reference test's own criterion (tests/test_gemm.cu:91-102, 366-374)
    assert float(np.max(np.abs(ref_out - expect))) <= oracle.REF_ABS_TOL[dt]
    # and the product bounds hold for the reference too on these cases
    oracle.check(ref_out, expect, dt)
    st2, d_ours = run_zcutlass(c, a, b, cm, bv)
    assert st2 == 0
    ours = oracle.bits_to_float(d_ours[:, :n], dt)
    oracle.check(ours, ref_out.astype(np.float64), dt)


@pytest.mark.gpu
def test_reference_dispatch_on_b200(cuda_device, ref_lib):
    # On cc 10.0 the reference runs WMMA kernels; its sm_120 explicit-MMA family is gated off.
    name = ref_lib.selected_kernel_name(128, 4096, 4096, 4096, 4096, 4096, 4096, oracle.F16)
    assert "tensorop" in name and "sm120_mma" not in name


@pytest.mark.gpu
def test_speed_against_reference_kernels(cuda_device, ref_lib, capsys):
    """Times both libraries on the Llama-3-8B prefill linears (row-major B, the
    only layout the reference accepts) and the cfg0 shape; prints the table."""
    import torch

    # the last two: odd leading dimensions, which TMA cannot describe (our generic path)
    shapes = [(8192, 6144, 4096), (8192, 4096, 4096), (8192, 28672, 4096), (8192, 4096, 14336), (256, 4096, 4096),
              (2047, 3001, 1999), (4095, 4097, 4093)]
    rows = []
    for m, n, k in shapes:
        a = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
        b = torch.randn(k, n, device="cuda", dtype=torch.bfloat16) / k ** 0.5
        d1 = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
        d2 = torch.empty_like(d1)
        desc = _native.make_desc(m, n, k, k, n, n, n, _native.BF16)

        def ours():
            assert _native.gemm(desc, a.data_ptr(), b.data_ptr(), None, d1.data_ptr()) == 0

        def theirs():
            assert ref_lib.gemm(m, n, k, a.data_ptr(), k, b.data_ptr(), n, None, n, d2.data_ptr(), n,
                                oracle.BF16, 1.0, 0.0, None) == 0

        times = []
        for fn in (ours, theirs):
            fn()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(5):
                fn()
            e1.record()
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1) / 5)
        flops = 2.0 * m * n * k
        rows.append((m, n, k, times[0], times[1], flops / times[0] / 1e9, flops / times[1] / 1e9,
                     _native.selected_kernel(desc)["kernel_name"]))
        ab = torch.testing.assert_close
        ab(d1.float(), d2.float(), rtol=5e-2, atol=5e-2)
    with capsys.disabled():
        print("\n  m      n      k   ours_ms  ref_ms   ours_TF  ref_TF  speedup  our kernel")
        for m, n, k, t0, t1, f0, f1, kern in rows:
            print(f"{m:6d} {n:6d} {k:6d} {t0:8.3f} {t1:8.3f} {f0:8.1f} {f1:7.1f} {t1 / t0:7.1f}x  {kern}")
    assert all(r[3] < r[4] for r in rows)
