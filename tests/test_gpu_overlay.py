"""The PyTorch operators, overlay and vLLM LinearMethod on the GPU.

Follows tools/check_torch_overlay.py and tools/check_vllm_linear_method.py in
the reference (forced hits compared with torch at rtol=atol=1e-2 / 5e-2, the
selected-config telemetry, a policy fallback counted as
shape_not_target_bucket), plus the native [N, K] weight path.
"""

from __future__ import annotations

import pytest
import torch

from zcutlass_b200 import _native, torch_ops


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
    torch.testing.assert_close(actual, expected, rtol=1e-2, atol=1e-2)
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
    ref = (0.5 * (a.float() @ b.float()) + 2.0 * c.float() + bias.float())
    tol = 2e-2 if dtype == torch.float16 else 6e-2
    for op in (ops.zcutlass_torch.gemm, ops.zcutlass.gemm):
        torch.testing.assert_close(op(a, b, c, bias, 0.5, 2.0).float(), ref, rtol=tol, atol=tol)
    d = torch.empty(m, n, device="cuda", dtype=dtype)
    ops.zcutlass.gemm_out(a, b, c, bias, 0.5, 2.0, d)
    torch.testing.assert_close(d.float(), ref, rtol=tol, atol=tol)
    with pytest.raises(RuntimeError):
        ops.zcutlass_torch.gemm(a, b.t())  # shape mismatch raises like the reference op


@pytest.mark.gpu
def test_linear_native_weight(ops):
    from zcutlass_torch import ZCutlassGemmOverlay

    x = torch.randn(4, 512, 1024, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(4096, 1024, device="cuda", dtype=torch.bfloat16) / 32
    bias = torch.randn(4096, device="cuda", dtype=torch.bfloat16)
    ref = torch.nn.functional.linear(x.float(), w.float(), bias.float())
    y = ops.zcutlass.linear(x, w, bias)
    assert y.shape == (4, 512, 4096)
    torch.testing.assert_close(y.float(), ref, rtol=3e-2, atol=3e-2)
    ov = ZCutlassGemmOverlay(native_weight_layout=True, routing_policy=None, force_zcutlass=True)
    y2 = ov.linear(x[0], w, bias)
    torch.testing.assert_close(y2.float(), ref[0], rtol=3e-2, atol=3e-2)
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
    ref = torch.nn.functional.linear(x, layer.weight, layer.bias)
    torch.testing.assert_close(y, ref, rtol=5e-2, atol=5e-2)
    assert m.stats.hits == 1 and m.last_trace["fallback_reason"] is None
    assert m.last_trace["weight_cache"] == ("native" if native else "miss")
    # decode-sized call: unpromoted family delegates to vLLM's own GEMM
    y8 = m.apply(layer, x[:8], layer.bias)
    torch.testing.assert_close(y8, ref[:8], rtol=5e-2, atol=5e-2)
    assert m.last_trace["fallback_reason"] == "family_not_promoted"
