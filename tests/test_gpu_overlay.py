"""The PyTorch operators, overlay and vLLM LinearMethod on the GPU.

Follows tools/check_torch_overlay.py and tools/check_vllm_linear_method.py in
the reference (forced hits, the selected-config telemetry, a policy fallback
counted as shape_not_target_bucket), plus the native [N, K] weight path.
Where the reference compares with torch at rtol=atol=1e-2 / 5e-2, these
tests hold every result the library computes to the product bounds against
the oracle on the same bit patterns (relative Frobenius <= 1e-3 f16 /
5e-3 bf16 and |out-ref| <= 4 ulp (1+|ref|)); results of a fallback, which
torch computes, are compared with torch.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle
from zcutlass_b200 import _native, torch_ops

CODE = {torch.float16: oracle.F16, torch.bfloat16: oracle.BF16}


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def oracle_check(out, a, b_kn, *, bias=None, c=None, alpha=1.0, beta=0.0):
    """out (device, [.., N]) against the oracle GEMM of a [M, K] and b_kn [K, N]."""
    dt = CODE[a.dtype]
    a2 = a.reshape(-1, a.shape[-1])
    m, k = a2.shape
    n = b_kn.shape[1]
    ref = oracle.gemm(_bits(a2), _bits(b_kn), m, n, k, dt, c=_bits(c) if beta != 0.0 else None,
                      bias=_bits(bias) if bias is not None else None, alpha=alpha, beta=beta)
    got = out.reshape(m, n).float().cpu().numpy()
    return oracle.check(got, ref, dt)


@pytest.fixture(scope="module")
def ops(cuda_device):
    torch_ops.load()
    return torch.ops


@pytest.mark.gpu
def test_torch_ops_match_torch(ops):
    from zcutlass_torch import ZCutlassGemmOverlay, selected_gemm_config

    a = torch.randn(8, 64, device="cuda", dtype=torch.float16)
    b = torch.randn(64, 128, device="cuda", dtype=torch.float16)
    bias = torch.randn(128, device="cuda", dtype=torch.float16)
    expected = torch.matmul(a, b) + bias
    launches = _native.kernel_launches()
    ov = ZCutlassGemmOverlay(force_zcutlass=True)
    actual = ov.gemm(a, b, bias=bias)
    assert _native.kernel_launches() > launches
    oracle_check(actual, a, b, bias=bias)
    cfg = selected_gemm_config(a, b, bias=bias)
    assert ov.last_kernel_name == cfg["kernel_name"] and ov.last_tile == cfg["tile"]
    assert ov.stats.hits == 1
    policy = ZCutlassGemmOverlay()
    torch.testing.assert_close(policy.gemm(a, b, bias=bias), expected, rtol=1e-2, atol=1e-2)
    assert policy.stats.fallback_reasons.get("shape_not_target_bucket") == 1


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_gemm_alpha_beta_bias_and_out(ops, dtype):
    m, n, k = 300, 520, 264
    a = torch.randn(m, k, device="cuda", dtype=dtype)
    b = torch.randn(k, n, device="cuda", dtype=dtype) / k ** 0.5
    c = torch.randn(m, n, device="cuda", dtype=dtype)
    bias = torch.randn(n, device="cuda", dtype=dtype)
    for op in (ops.zcutlass_torch.gemm, ops.zcutlass.gemm):
        oracle_check(op(a, b, c, bias, 0.5, 2.0), a, b, bias=bias, c=c, alpha=0.5, beta=2.0)
    d = torch.empty(m, n, device="cuda", dtype=dtype)
    ops.zcutlass.gemm_out(a, b, c, bias, 0.5, 2.0, d)
    oracle_check(d, a, b, bias=bias, c=c, alpha=0.5, beta=2.0)
    with pytest.raises(RuntimeError):
        ops.zcutlass_torch.gemm(a, b.t())  # shape mismatch raises like the reference op


@pytest.mark.gpu
def test_linear_native_weight(ops):
    from zcutlass_torch import ZCutlassGemmOverlay

    x = torch.randn(4, 512, 1024, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(4096, 1024, device="cuda", dtype=torch.bfloat16) / 32
    bias = torch.randn(4096, device="cuda", dtype=torch.bfloat16)
    y = ops.zcutlass.linear(x, w, bias)
    assert y.shape == (4, 512, 4096)
    oracle_check(y, x, w.t(), bias=bias)
    ov = ZCutlassGemmOverlay(native_weight_layout=True, routing_policy=None, force_zcutlass=True)
    y2 = ov.linear(x[0], w, bias)
    oracle_check(y2, x[0], w.t(), bias=bias)
    assert ov.stats.hits == 1 and ov.last_kernel_path == "zcutlass"


@pytest.mark.gpu
@pytest.mark.parametrize("native", [False, True])
def test_vllm_linear_method_on_gpu(ops, native):
    vllm_linear = pytest.importorskip("vllm.model_executor.layers.linear")
    from zcutlass_vllm import install_zcutlass_unquantized_linear_method

    class DummyVllmLinear(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.weight = torch.nn.Parameter(torch.randn(2048, 1536, device="cuda", dtype=torch.float16) / 40,
                                             requires_grad=False)
            self.bias = torch.nn.Parameter(torch.randn(2048, device="cuda", dtype=torch.float16) * 0.1,
                                           requires_grad=False)
            self.prefix = "model.layers.0.self_attn.qkv_proj"
            self.quant_method = vllm_linear.UnquantizedLinearMethod()

    layer = DummyVllmLinear()
    m = install_zcutlass_unquantized_linear_method(layer, promoted_families=("prefill",), native_weight_layout=native)
    x = torch.randn(256, 1536, device="cuda", dtype=torch.float16)
    y = m.apply(layer, x, layer.bias)
    oracle_check(y, x, layer.weight.t(), bias=layer.bias)
    assert m.stats.hits == 1 and m.last_trace["fallback_reason"] is None
    assert m.last_trace["weight_cache"] == ("native" if native else "miss")
    # decode-sized call: unpromoted family delegates to vLLM's own GEMM
    y8 = m.apply(layer, x[:8], layer.bias)  # computed by vLLM (torch), compared with torch
    ref = torch.nn.functional.linear(x, layer.weight, layer.bias)
    torch.testing.assert_close(y8, ref[:8], rtol=5e-2, atol=5e-2)
    assert m.last_trace["fallback_reason"] == "family_not_promoted"
