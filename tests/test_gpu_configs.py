"""Every named benchmark configuration against the oracle, at full size.

The reference benchmarks these shape sets (benchmarks/bench_gemm.cu:162-216
for the square bucket sweep; tools/benchmark_torch_llm_overlay.py:97-105 for
the decoder-layer linears). Each point runs through the C ABI with the
product's own distributions (A ~ N(0,1), W ~ N(0,1/K), C ~ N(0,1),
bias ~ N(0,0.1), cast to the storage type) and is checked against the
oracle's FP64-accumulated rows -- every row for M <= 16, 16 sampled rows
(first and last included) above that -- under both product bounds
(relative Frobenius <= 1e-3 f16 / 5e-3 bf16, |out-ref| <= 4 ulp (1+|ref|)).

  cfg1  square N = K in {1024, 2048, 4096, 8192} x M in {1, 16, 64, 256, 1024}
        x {no bias, bias} x beta in {0, 1}, f16 and bf16, B row-major [K, N]
        (the sweep's plain GEMM layout): 160 points;
  cfg2  the Qwen2-1.5B layer at M = 4096, o_proj included;
  cfg4  Llama-3-70B TP=8 shards in f16 and bf16: prefill at M = 16384 and
        decode at M in {1, 8, 16, 32}, weights in the PyTorch [N, K] layout.
Inputs are generated once per (dtype, shape) and sliced by M.
"""

from __future__ import annotations

import functools

import numpy as np
import pytest

from oracle import oracle
from zcutlass_b200 import _native

F16, BF16 = oracle.F16, oracle.BF16
DT_NAME = {F16: "f16", BF16: "bf16"}


def _bits(t) -> np.ndarray:
    import torch

    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


@functools.lru_cache(maxsize=2)
def _operands(dtype: int, m_max: int, n: int, k: int, col: bool, seed: int):
    """Device tensors (A[m_max,k], B, C[m_max,n], bias[n]) and B's bit
    patterns as the oracle reads them ([k, n] row-major). B is [n, k] on the
    device when col (PyTorch weight) else [k, n]. Drawn on the GPU from a
    seeded generator (full-size host generation would take minutes)."""
    import torch

    tdt = torch.bfloat16 if dtype == BF16 else torch.float16
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randn(m_max, k, generator=g, device="cuda").to(tdt)
    b = (torch.randn(*((n, k) if col else (k, n)), generator=g, device="cuda") * k ** -0.5).to(tdt)
    c = torch.randn(m_max, n, generator=g, device="cuda").to(tdt)
    bias = (torch.randn(n, generator=g, device="cuda") * 0.1).to(tdt)
    b_rm = _bits(b.t() if col else b)
    return a, b, c, bias, b_rm


def _check_point(name, dtype, m, n, k, col, bias, beta, m_max, seed=11):
    import torch

    a_all, b, c_all, bvec, b_rm = _operands(dtype, m_max, n, k, col, seed)
    a, cm = a_all[:m], c_all[:m]
    d = torch.empty(m, n, device="cuda", dtype=a.dtype)
    desc = _native.make_desc(m, n, k, k, k if col else n, n, n, dtype, 1.0, beta,
                             bvec.data_ptr() if bias else None, None,
                             b_layout=_native.COLUMN_MAJOR if col else _native.ROW_MAJOR)
    st = _native.gemm(desc, a.data_ptr(), b.data_ptr(), cm.data_ptr() if beta != 0.0 else None, d.data_ptr())
    torch.cuda.synchronize()
    assert st == _native.SUCCESS, f"{name}: {_native.STATUS_NAMES.get(st, st)}"
    assert _native.device_error(clear=True) == 0, f"{name}: device-side wait timed out"
    if m <= 16:
        rows = np.arange(m)
    else:
        rng = np.random.default_rng(m * 7 + n)
        rows = np.unique(np.concatenate([[0, m - 1], rng.integers(0, m, size=14)]))
    idx = torch.as_tensor(rows, device="cuda")
    # the oracle reads row r of A and C at index r of these row-gathered copies
    a_rows, c_rows = _bits(a[idx]), _bits(cm[idx])
    ref = oracle.gemm_f64_rows(a_rows, b_rm, np.arange(rows.size), n, k, dtype, c=c_rows,
                               bias=_bits(bvec) if bias else None, alpha=1.0, beta=beta)
    out = oracle.bits_to_float(_bits(d[idx]), dtype)
    metrics = oracle.check(out, ref, dtype)
    assert float(np.max(np.abs(out - ref))) <= oracle.REF_ABS_TOL[dtype]
    return metrics


# ---------------------------------------------------------------- cfg1: the bucket sweep

CFG1_M = (1, 16, 64, 256, 1024)
CFG1_H = (1024, 2048, 4096, 8192)


def _cfg1_points():
    out = []
    for dt in (F16, BF16):
        for h in CFG1_H:
            for m in CFG1_M:
                for bias in (False, True):
                    for beta in (0.0, 1.0):
                        out.append(pytest.param(dt, h, m, bias, beta,
                                                id=f"cfg1-{DT_NAME[dt]}-h{h}-m{m}-bias{int(bias)}-beta{int(beta)}"))
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("dt,h,m,bias,beta", _cfg1_points())
def test_cfg1_bucket_sweep(cuda_device, dt, h, m, bias, beta):
    _check_point(f"cfg1 {DT_NAME[dt]} h{h} m{m}", dt, m, h, h, False, bias, beta, max(CFG1_M))


# ---------------------------------------------------------------- cfg2 / cfg4: layer linears

CFG2 = [  # (name, n, k, bias) at M = 4096, bf16
    ("qkv", 2048, 1536, True),
    ("o_proj", 1536, 1536, False),
    ("gate_up", 17920, 1536, False),
    ("down", 1536, 8960, False),
]

CFG4 = [  # Llama-3-70B per-GPU shards at TP=8: (name, n, k)
    ("qkv", 1280, 8192),
    ("o_proj", 8192, 1024),
    ("gate_up", 7168, 8192),
    ("down", 8192, 3584),
]


@pytest.mark.gpu
@pytest.mark.parametrize("name,n,k,bias", CFG2, ids=[f"cfg2-{c[0]}" for c in CFG2])
def test_cfg2_qwen2_layer(cuda_device, name, n, k, bias):
    _check_point(f"cfg2 {name}", BF16, 4096, n, k, True, bias, 0.0, 4096)


@pytest.mark.gpu
@pytest.mark.parametrize("dt", [F16, BF16], ids=["f16", "bf16"])
@pytest.mark.parametrize("name,n,k", CFG4, ids=[f"cfg4-prefill-{c[0]}" for c in CFG4])
def test_cfg4_prefill_m16384(cuda_device, name, n, k, dt):
    _check_point(f"cfg4 prefill {name}", dt, 16384, n, k, True, False, 0.0, 16384)


@pytest.mark.gpu
@pytest.mark.parametrize("dt", [F16, BF16], ids=["f16", "bf16"])
@pytest.mark.parametrize("m", [1, 8, 16, 32])
@pytest.mark.parametrize("name,n,k", CFG4, ids=[f"cfg4-decode-{c[0]}" for c in CFG4])
def test_cfg4_decode(cuda_device, name, n, k, m, dt):
    _check_point(f"cfg4 decode {name} m{m}", dt, m, n, k, True, False, 0.0, 32)
