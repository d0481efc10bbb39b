"""GPU parity tests: every kernel family against the oracle, through the C ABI.

Cases follow the reference's own test list (tests/test_gemm.cu:754-786 in
supercatking/zcutlass: tiny padded+bias, 16^3, rectangular with alpha/beta/bias,
ragged alpha/beta, llm-smoke, the 64/32 x 1024 x 1024 prefill smokes) plus
forced runs of each sm_100a family over ragged shapes, both B layouts and
every epilogue combination.
"""

from __future__ import annotations

import numpy as np
import pytest

from gemm_case import Case, check_case, make_inputs, oracle_result, run_zcutlass, selected, to_device, to_host
from oracle import oracle
from zcutlass_b200 import _native

F16, BF16 = oracle.F16, oracle.BF16

REFERENCE_CASES = [
    # name, dtype, m, n, k, alpha, beta, bias, pads (a, b, c, d)
    ("f16 tiny padded bias", F16, 15, 17, 19, 1.0, 0.25, True, (3, 5, 7, 11)),
    ("f16 16x16", F16, 16, 16, 16, 1.0, 0.0, False, (0, 0, 0, 0)),
    ("f16 rectangular", F16, 65, 129, 31, 0.75, 0.5, True, (3, 5, 7, 11)),
    ("f16 ragged alpha no-bias padded A/D", F16, 31, 63, 17, -0.5, 0.0, False, (2, 0, 0, 9)),
    ("f16 ragged beta no-bias", F16, 47, 64, 33, 0.5, -0.25, False, (0, 0, 0, 0)),
    ("f16 llm-smoke", F16, 8, 256, 256, 1.0, 0.0, False, (0, 0, 0, 0)),
    ("f16 prefill smoke", F16, 64, 1024, 1024, 1.0, 0.0, False, (0, 0, 0, 0)),
    ("f16 m32 prefill smoke", F16, 32, 1024, 1024, 1.0, 0.0, False, (0, 0, 0, 0)),
    ("f16 n64 prefill bias smoke", F16, 64, 1024, 1024, 1.0, 0.0, True, (0, 0, 0, 0)),
    ("bf16 tiny padded bias", BF16, 13, 19, 23, 1.0, 0.25, True, (3, 5, 7, 11)),
    ("bf16 16x16", BF16, 16, 16, 16, 1.0, 0.0, False, (0, 0, 0, 0)),
    ("bf16 rectangular", BF16, 67, 127, 29, 0.75, 0.5, True, (3, 5, 7, 11)),
    ("bf16 ragged alpha no-bias padded B/C/D", BF16, 29, 61, 15, -0.75, 0.0, False, (0, 4, 6, 10)),
    ("bf16 ragged beta no-bias", BF16, 45, 64, 31, 0.5, -0.25, False, (0, 0, 0, 0)),
    ("bf16 llm-smoke", BF16, 8, 256, 256, 1.0, 0.0, False, (0, 0, 0, 0)),
    ("bf16 prefill smoke", BF16, 64, 1024, 1024, 1.0, 0.0, False, (0, 0, 0, 0)),
    ("bf16 m32 prefill smoke", BF16, 32, 1024, 1024, 1.0, 0.0, False, (0, 0, 0, 0)),
    ("bf16 n64 prefill bias smoke", BF16, 64, 1024, 1024, 1.0, 0.0, True, (0, 0, 0, 0)),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", REFERENCE_CASES, ids=[c[0] for c in REFERENCE_CASES])
def test_reference_cases(cuda_device, case):
    name, dt, m, n, k, alpha, beta, bias, pads = case
    c = Case(name, dt, m, n, k, alpha, beta, bias, *pads)
    check_case(c)


@pytest.mark.gpu
def test_rowmajor_entry_point(cuda_device):
    c = Case("flat entry", BF16, 200, 384, 320, 0.5, 1.0, True)
    check_case(c, rowmajor_entry=True)


# ---------------------------------------------------------------- forced families

FAMILIES = {
    "pair256": "_256x256x64_2cta_persistent",
    "persistent256": "_128x256x64_ws_persistent",
    "persistent128": "_128x128x64_ws_persistent",
    "persistent64": "_128x64x64_ws_persistent",
    "swapab16": "_16x128x64_swapab_splitk",
    "swapab32": "_32x128x64_swapab_splitk",
    "swapab64": "_64x128x64_swapab_splitk",
    "sk16": "_16x128x64_swapab_streamk",
    "sk32": "_32x128x64_swapab_streamk",
    "sk64": "_64x128x64_swapab_streamk",
    "generic": "x32_generic",
    "repack": "_repack_generic",
    "splitk256": "_128x256x64_splitk_cluster",
    "splitk128": "_128x128x64_splitk_cluster",
    "splitkm256": "_256x256x64_splitk_cluster",
}

# (m, n, k) per family: ragged edges in every dimension, K tails, multi-tile.
FAMILY_SHAPES = {
    # (300, ...): the second tile row's follower CTA (rows 384..511) lies wholly outside M.
    "pair256": [(256, 256, 64), (300, 520, 200), (1000, 777, 1032), (2048, 4096, 1024), (4096, 1536, 8960)],
    "persistent256": [(128, 256, 64), (300, 520, 200), (1000, 777, 1032), (2048, 4096, 1024)],
    "persistent128": [(128, 128, 64), (129, 136, 72), (513, 1000, 520), (1536, 2048, 1536)],
    "persistent64": [(128, 64, 64), (129, 72, 72), (513, 1000, 520), (256, 4096, 4096)],
    "swapab16": [(1, 128, 128), (7, 300, 200), (16, 1000, 4096), (13, 4096, 1032)],
    "swapab32": [(17, 128, 128), (32, 520, 777), (25, 2048, 2048)],
    "swapab64": [(33, 256, 256), (64, 1000, 1000), (48, 4096, 1536)],
    # stream-K: one tile split over 128 CTAs, a 12-unit problem (every tile
    # shared by several CTAs), ragged edges, and decode-sized layers
    "sk16": [(1, 128, 8192), (7, 300, 200), (16, 1000, 4096), (13, 7168, 1032), (16, 8192, 1024)],
    "sk32": [(17, 128, 128), (32, 520, 777), (25, 2048, 8192)],
    "sk64": [(33, 256, 256), (64, 1000, 1000), (48, 4096, 1536)],
    # cluster split-K: one tile, ragged edges, the cfg0 shape, several tile rows
    "splitk256": [(128, 256, 64), (300, 520, 200), (256, 4096, 4096), (1000, 777, 1032)],
    "splitk128": [(129, 136, 72), (513, 1000, 520), (256, 2048, 1536)],
    "splitkm256": [(256, 256, 64), (300, 520, 200), (256, 4096, 4096), (1000, 777, 1032), (129, 1024, 2048)],
    # odd leading dimensions (pads 3/5/7/11) on several 128 x 128 tiles, K tails of 1..31
    "generic": [(5, 7, 9), (100, 200, 50), (130, 70, 300), (1000, 777, 1032), (257, 1300, 2101)],
    # the same odd layouts on the tcgen05 kernels through packed copies: the
    # small-M (swap-AB), split-K and persistent routes
    "repack": [(5, 7, 9), (60, 300, 200), (100, 200, 50), (257, 1300, 2101), (1000, 777, 1032), (2047, 3001, 1999)],
}

EPILOGUES = [  # (alpha, beta, bias)
    (1.0, 0.0, False),
    (0.75, 0.5, True),
    (-1.25, 1.0, False),
    (1.0, 0.0, True),
]


def _family_params():
    out = []
    for fam, shapes in FAMILY_SHAPES.items():
        for shape in shapes:
            for dt in (F16, BF16):
                for col in (False, True):
                    out.append((fam, shape, dt, col))
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("fam,shape,dt,col", _family_params(),
                         ids=lambda v: str(v).replace(" ", ""))
def test_forced_family(cuda_device, monkeypatch, fam, shape, dt, col):
    monkeypatch.setenv("ZCUTLASS_FORCE_KERNEL", FAMILIES[fam])
    m, n, k = shape
    if fam in ("generic", "repack"):
        pads = (3, 5, 7, 11)
    else:
        # TMA families need leading dimensions that are multiples of 8 elements;
        # pad ragged sizes up to that, and give D 8 extra columns so the
        # padding sentinel is checked on the TMA store path too.
        pads = ((-k) % 8, (-(k if col else n)) % 8, (-n) % 8, (-n) % 8 + 8)
    for i, (alpha, beta, bias) in enumerate(EPILOGUES):
        if i and m * n * k > 2**31:
            break  # large shapes: plain epilogue only (the rest is covered on small shapes)
        c = Case(f"{fam} {shape} {i}", dt, m, n, k, alpha, beta, bias, *pads, b_col_major=col, gen="normal",
                 seed=i)
        sel = selected(c)
        assert FAMILIES[fam] in sel["kernel_name"], sel
        check_case(c)


@pytest.mark.gpu
@pytest.mark.parametrize("splits", [1, 2, 3, 5, 8])
@pytest.mark.parametrize("tile", ["128x128", "128x256", "256x256"])
def test_splitk_split_counts(cuda_device, monkeypatch, splits, tile):
    """Every cluster size the split-K kernel can get, on a ragged problem whose
    K blocks do not divide evenly (17 blocks of 64, the last one partial)."""
    monkeypatch.setenv("ZCUTLASS_FORCE_KERNEL", f"_{tile}x64_splitk_cluster")
    monkeypatch.setenv("ZCUTLASS_SPLITK", str(splits))
    for dt in (F16, BF16):
        for i, (alpha, beta, bias) in enumerate(EPILOGUES):
            c = Case(f"splitk{tile} s{splits} {i}", dt, 200, 600, 1080, alpha, beta, bias, 0, 0, 0, 8,
                     b_col_major=(i % 2 == 1), gen="normal", seed=splits * 10 + i)
            assert f"_{tile}x64_splitk_cluster" in selected(c)["kernel_name"]
            check_case(c)


# ---------------------------------------------------------------- config shapes

# Full-size BASELINE shapes, checked on sampled rows against an FP64-accumulated oracle.
CONFIG_SHAPES = [
    ("cfg0 256x4096x4096+bias", BF16, 256, 4096, 4096, True),
    ("cfg2 qkv", BF16, 4096, 2048, 1536, True),
    ("cfg2 gate_up", BF16, 4096, 17920, 1536, False),
    ("cfg2 down", BF16, 4096, 1536, 8960, False),
    ("cfg3 qkv", BF16, 8192, 6144, 4096, False),
    ("cfg3 gate_up", BF16, 8192, 28672, 4096, False),
    ("cfg3 down", BF16, 8192, 4096, 14336, False),
    ("cfg4 decode gate_up m16", F16, 16, 7168, 8192, False),
    ("cfg4 decode down m1", BF16, 1, 8192, 3584, False),
    ("cfg4 decode o m32", BF16, 32, 8192, 1024, False),
    ("cfg1 h8192 m1024 beta", F16, 1024, 8192, 8192, True),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", CONFIG_SHAPES, ids=[c[0] for c in CONFIG_SHAPES])
@pytest.mark.parametrize("col", [False, True], ids=["B_rowmajor", "B_colmajor"])
def test_config_shapes_sampled(cuda_device, case, col):
    name, dt, m, n, k, bias = case
    beta = 1.0 if "beta" in name else 0.0
    c = Case(name, dt, m, n, k, 1.0, beta, bias, b_col_major=col, gen="normal", seed=7)
    a, b, cm, bvec = make_inputs(c)
    st, d = run_zcutlass(c, a, b, cm, bvec)
    assert st == _native.SUCCESS
    assert _native.device_error(clear=True) == 0
    rng = np.random.default_rng(1)
    rows = np.unique(np.concatenate([[0, m - 1], rng.integers(0, m, size=min(m, 14))]))
    b_rm = np.ascontiguousarray(b[:, :k].T) if col else b
    ref = oracle.gemm_f64_rows(a, b_rm, rows, n, k, dt, c=cm, bias=bvec if bias else None, alpha=1.0, beta=beta)
    out = oracle.bits_to_float(d[rows, :n], dt)
    oracle.check(out, ref, dt)


# ---------------------------------------------------------------- stream-K specifics


def _sk_run(m, n, k, dtype, stream=None, repeats=1):
    import torch

    g = torch.Generator(device="cpu").manual_seed(3)
    tdt = torch.bfloat16 if dtype == BF16 else torch.float16
    a = torch.randn(m, k, generator=g).to(tdt).cuda()
    w = (torch.randn(n, k, generator=g) / k ** 0.5).to(tdt).cuda()
    outs = []
    for _ in range(repeats):
        d = torch.empty(m, n, dtype=tdt, device="cuda")
        desc = _native.make_desc(m, n, k, k, k, n, n, dtype, stream=stream, b_layout=_native.COLUMN_MAJOR)
        assert _native.gemm(desc, a.data_ptr(), w.data_ptr(), None, d.data_ptr()) == 0
        outs.append(d)
    return a, w, outs


@pytest.mark.gpu
def test_streamk_is_deterministic(cuda_device, monkeypatch):
    import torch

    monkeypatch.setenv("ZCUTLASS_FORCE_KERNEL", "_16x128x64_swapab_streamk")
    _, _, outs = _sk_run(16, 7168, 8192, BF16, repeats=4)
    torch.cuda.synchronize()
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    assert _native.device_error(clear=True) == 0


@pytest.mark.gpu
def test_streamk_in_cuda_graph_replays(cuda_device, monkeypatch):
    """The counters reset themselves, so a captured launch (fixed epoch)
    replays correctly; interleaved shapes on one stream share the workspace."""
    import torch

    monkeypatch.setenv("ZCUTLASS_FORCE_KERNEL", "_swapab_streamk")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        a, w, (ref,) = _sk_run(8, 1280, 8192, BF16, stream=s.cuda_stream)  # allocates the workspace
        a2, w2, (ref2,) = _sk_run(32, 4096, 1024, BF16, stream=s.cuda_stream)
        torch.cuda.synchronize()
        d = torch.empty_like(ref)
        d2 = torch.empty_like(ref2)
        desc = _native.make_desc(8, 1280, 8192, 8192, 8192, 1280, 1280, BF16, stream=s.cuda_stream,
                                 b_layout=_native.COLUMN_MAJOR)
        desc2 = _native.make_desc(32, 4096, 1024, 1024, 1024, 4096, 4096, BF16, stream=s.cuda_stream,
                                  b_layout=_native.COLUMN_MAJOR)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            desc.stream = torch.cuda.current_stream().cuda_stream
            desc2.stream = desc.stream
            assert _native.gemm(desc, a.data_ptr(), w.data_ptr(), None, d.data_ptr()) == 0
            assert _native.gemm(desc2, a2.data_ptr(), w2.data_ptr(), None, d2.data_ptr()) == 0
        for _ in range(3):
            d.zero_()
            d2.zero_()
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(d, ref) and torch.equal(d2, ref2)
    assert _native.device_error(clear=True) == 0


@pytest.mark.gpu
def test_streamk_capture_on_fresh_stream_falls_back(cuda_device, monkeypatch):
    """With the experimental stream-K kernel enabled, a decode GEMM captured on
    a stream that has no stream-K workspace yet (its allocation is not allowed
    during capture) is served by split-K instead of failing the capture."""
    import torch

    monkeypatch.setenv("ZCUTLASS_EXPERIMENTAL_KERNELS", "1")
    m, n, k = 8, 1280, 8192
    g0 = torch.Generator(device="cpu").manual_seed(5)
    a = torch.randn(m, k, generator=g0).to(torch.bfloat16).cuda()
    w = (torch.randn(n, k, generator=g0) / k ** 0.5).to(torch.bfloat16).cuda()
    s = torch.cuda.Stream()
    desc = _native.make_desc(m, n, k, k, k, n, n, BF16, stream=s.cuda_stream, b_layout=_native.COLUMN_MAJOR)
    assert "swapab_streamk" in _native.selected_kernel(desc)["kernel_name"]  # outside capture
    d = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        desc.stream = torch.cuda.current_stream().cuda_stream
        assert _native.gemm(desc, a.data_ptr(), w.data_ptr(), None, d.data_ptr()) == 0
    d.zero_()
    g.replay()
    torch.cuda.synchronize()
    ref = torch.nn.functional.linear(a.float(), w.float())
    rel = float((d.float() - ref).norm() / ref.norm())
    assert rel < 5e-3, rel
    assert _native.device_error(clear=True) == 0


# ---------------------------------------------------------------- row-gathered A

GATHER_CASES = [  # (m, n, k, parts, alpha, beta, bias)
    (256, 2048, 512, 2, 1.0, 0.0, False),     # 128-row blocks: one-CTA kernel
    (1024, 1536, 520, 4, 0.75, 0.5, True),    # ragged K, epilogue with C and bias
    (2048, 4096, 1024, 8, 1.0, 0.0, False),   # 256-row blocks: two-CTA tiles
    (4096, 3584, 1024, 8, 1.0, 0.0, True),    # TP8 gate_up shard width at 4096 tokens
]


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k,parts,alpha,beta,bias", GATHER_CASES)
def test_gemm_gather_a(cuda_device, m, n, k, parts, alpha, beta, bias):
    """zcutlass_gemm_gather_a reads row block i of A from buffer i only: every
    buffer holds a full [M, K] matrix whose other rows are garbage."""
    import torch

    c = Case(f"gather {m}x{n}x{k}/{parts}", BF16, m, n, k, alpha, beta, bias, b_col_major=True, gen="normal",
             seed=parts)
    a, b, cm, bias_bits = make_inputs(c)
    ref = oracle_result(c, a, b, cm, bias_bits)
    rows = m // parts
    bufs = []
    for i in range(parts):
        junk = np.full_like(a, oracle.float_to_bits(np.float32(1000.0 + i), BF16))
        junk[i * rows:(i + 1) * rows] = a[i * rows:(i + 1) * rows]
        bufs.append(to_device(junk))
    db, dc, dbias = to_device(b), to_device(cm), to_device(bias_bits)
    dd = torch.empty(m, n, device="cuda", dtype=torch.int16)
    desc = _native.make_desc(m, n, k, k, k, n, n, BF16, alpha, beta, dbias.data_ptr() if bias else None, None,
                             b_layout=_native.COLUMN_MAJOR)
    st = _native.gemm_gather_a(desc, [t.data_ptr() for t in bufs], db.data_ptr(),
                               dc.data_ptr() if beta != 0.0 else None, dd.data_ptr())
    torch.cuda.synchronize()
    assert st == _native.SUCCESS, _native.STATUS_NAMES.get(st, st)
    assert _native.device_error(clear=True) == 0
    out = oracle.bits_to_float(to_host(dd), BF16)
    oracle.check(out, ref, BF16)


@pytest.mark.gpu
def test_repack_path_in_cuda_graph(cuda_device):
    """The packed-operand path replayed from a CUDA graph equals its eager
    result bit for bit; a capture on a stream that has no scratch buffer yet is
    served by the predicated kernel instead (no allocation while capturing)."""
    import torch

    m, n, k = 300, 1000, 1031  # K odd: A and B cannot be described by TMA
    g0 = torch.Generator(device="cpu").manual_seed(9)
    a = torch.randn(m, k, generator=g0).to(torch.bfloat16).cuda()
    b = (torch.randn(k, n, generator=g0) / k ** 0.5).to(torch.bfloat16).cuda()
    s = torch.cuda.Stream()
    desc = _native.make_desc(m, n, k, k, n, n, n, BF16, stream=s.cuda_stream)
    assert "repack_generic" in _native.selected_kernel(desc)["kernel_name"]
    ref = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    with torch.cuda.stream(s):
        assert _native.gemm(desc, a.data_ptr(), b.data_ptr(), None, ref.data_ptr()) == 0  # sizes the scratch
    torch.cuda.synchronize()
    d = torch.empty_like(ref)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        desc.stream = torch.cuda.current_stream().cuda_stream
        assert _native.gemm(desc, a.data_ptr(), b.data_ptr(), None, d.data_ptr()) == 0
    for _ in range(2):
        d.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(d, ref)
    del g
    # a fresh stream has no scratch: the capture takes the predicated kernel
    s2 = torch.cuda.Stream()
    d2 = torch.empty_like(ref)
    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g2, stream=s2):
        desc.stream = torch.cuda.current_stream().cuda_stream
        assert _native.gemm(desc, a.data_ptr(), b.data_ptr(), None, d2.data_ptr()) == 0
    g2.replay()
    torch.cuda.synchronize()
    rel = float((d2.float() - ref.float()).norm() / ref.float().norm())
    assert rel < 5e-3, rel
    assert _native.device_error(clear=True) == 0
