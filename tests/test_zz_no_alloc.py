"""The decode GEMM entry point that allocates nothing: zcutlass_gemm_decode_noalloc.

Some callers cannot allocate device memory at the moment they call the GEMM:
code inside an allocator or memory-pool callback (a cudaMalloc there would
re-enter the allocator), and serving processes that reserve all device memory
up front and forbid any allocation after start-up. The regular entry points
may allocate a per-stream workspace the first time the stream-K decode kernel
runs on a stream; this entry point runs that kernel with its scratch in a
fixed array compiled into the library.

The test calls it through the C ABI twice in a row -- the second call finds
the first call's counters and partial tiles still in the shared scratch -- and
checks both results against zcutlass_gemm on the same inputs and against the
oracle, with the same tolerances as the other GPU tests. It also checks that
repeated calls allocate no device memory, that problems beyond the scratch
limit are rejected before any launch, and that zero-size problems succeed.
The file name makes pytest collect it last; it also passes alone in a fresh
process.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle
from zcutlass_b200 import _native

DUMMY = 0x1000  # aligned, never dereferenced: these calls return before any launch


def _noalloc(m, n, k, a, lda, b, ldb, col, c, ldc, d, ldd, dtype, alpha=1.0, beta=0.0, bias=None, stream=None):
    return _native.lib().zcutlass_gemm_decode_noalloc(m, n, k, a, lda, b, ldb, 1 if col else 0, c, ldc, d, ldd,
                                                       dtype, alpha, beta, bias, stream)


def _case(m, n, k, dtype, col, beta, with_bias, seed):
    import torch

    tdt = torch.bfloat16 if dtype == oracle.BF16 else torch.float16
    g = torch.Generator(device="cpu").manual_seed(seed)
    a = torch.randn(m, k, generator=g).to(tdt).cuda()
    w = ((torch.randn(n, k, generator=g) if col else torch.randn(k, n, generator=g)) / k ** 0.5).to(tdt).cuda()
    c = torch.randn(m, n, generator=g).to(tdt).cuda()
    bias = (torch.randn(n, generator=g) * 0.1).to(tdt).cuda() if with_bias else None
    return a, w, c, bias


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k,dtype,col,beta,with_bias", [
    (16, 4096, 4096, oracle.BF16, True, 0.0, True),
    (7, 1000, 520, oracle.F16, False, 0.5, False),
    (48, 2048, 1536, oracle.BF16, True, 1.0, True),
])
def test_noalloc_matches_gemm_twice(cuda_device, m, n, k, dtype, col, beta, with_bias):
    import torch

    a, w, c, bias = _case(m, n, k, dtype, col, beta, with_bias, seed=m + n)
    ldb = k if col else n
    cptr = c.data_ptr() if beta != 0.0 else None
    bptr = bias.data_ptr() if bias is not None else None
    ref = torch.empty(m, n, dtype=a.dtype, device="cuda")
    desc = _native.make_desc(m, n, k, k, ldb, n, n, dtype, 1.0, beta, bptr, None,
                             b_layout=_native.COLUMN_MAJOR if col else _native.ROW_MAJOR)
    assert _native.gemm(desc, a.data_ptr(), w.data_ptr(), cptr, ref.data_ptr()) == _native.SUCCESS
    torch.cuda.synchronize()
    ref_np = ref.float().cpu().numpy()
    # the oracle on the same bit patterns (B as the [K, N] row-major matrix it reads)
    bits = lambda t: t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    oracle_ref = oracle.gemm(bits(a), bits(w.t() if col else w), m, n, k, dtype, c=bits(c) if beta != 0.0 else None,
                             bias=bits(bias) if bias is not None else None, alpha=1.0, beta=beta)

    outs = []
    for call in range(2):
        d = torch.full((m, n), -3.0, dtype=a.dtype, device="cuda")
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        st = _noalloc(m, n, k, a.data_ptr(), k, w.data_ptr(), ldb, col, cptr, n, d.data_ptr(), n, dtype, 1.0, beta,
                      bptr)
        assert st == _native.SUCCESS, _native.status_name(st)
        torch.cuda.synchronize()
        if call == 1:  # after the first call's one-time set-up: no device allocation at all
            assert torch.cuda.mem_get_info()[0] == free_before
        assert _native.device_error(clear=True) == 0
        out = d.float().cpu().numpy()
        oracle.check(out, ref_np.astype(np.float64), dtype)  # against zcutlass_gemm
        oracle.check(out, oracle_ref, dtype)  # against the oracle
        outs.append(out)
    np.testing.assert_array_equal(outs[0], outs[1])  # the scratch left by call 1 does not leak into call 2


@pytest.mark.gpu
def test_noalloc_limits(cuda_device):
    bf16 = oracle.BF16
    # M beyond the decode buckets
    assert _noalloc(65, 256, 256, DUMMY, 256, DUMMY, 256, True, None, 256, DUMMY, 256, bf16) == \
        _native.INVALID_ARGUMENT
    # more tile counters than the scratch holds (N > 1,048,576)
    n = 1 << 21
    assert _noalloc(1, n, 128, DUMMY, 128, DUMMY, 128, True, None, n, DUMMY, n, bf16) == _native.INVALID_ARGUMENT
    # leading dimension TMA cannot describe
    assert _noalloc(8, 256, 250, DUMMY, 250, DUMMY, 250, True, None, 256, DUMMY, 256, bf16) == \
        _native.INVALID_ARGUMENT
    # generic validation first, same codes as zcutlass_gemm
    assert _noalloc(8, 256, 256, None, 256, DUMMY, 256, True, None, 256, DUMMY, 256, bf16) == \
        _native.INVALID_ARGUMENT
    assert _noalloc(8, 256, 256, DUMMY, 256, DUMMY, 256, True, None, 256, DUMMY, 256, _native.F32) == \
        _native.NOT_SUPPORTED
    # nothing to do: success without touching memory
    assert _noalloc(0, 256, 256, None, 256, None, 256, True, None, 256, None, 256, bf16) == _native.SUCCESS
