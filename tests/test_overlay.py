"""The PyTorch overlay and vLLM LinearMethod boundary, on CPU.

Counters, reasons and routing must match the reference's overlay
(python/zcutlass_torch/overlay.py); where the reference checkout is present
the same calls are replayed through the reference module and compared.
Patterns follow tools/check_torch_overlay.py and
tools/check_vllm_linear_method.py (a DummyVllmLinear module holding weight,
bias, prefix and an UnquantizedLinearMethod).
"""

from __future__ import annotations

import importlib.util
import os
from pathlib import Path

import pytest
import torch

import zcutlass_torch
from zcutlass_torch import OverlayStats, RoutingPolicy, ZCutlassGemmOverlay

REF_ROOT = Path(os.environ.get("ZCUTLASS_REF_ROOT", Path(__file__).resolve().parents[2] / "reference"))
REF_OVERLAY = REF_ROOT / "python" / "zcutlass_torch" / "overlay.py"


def _reference_overlay_module():
    if not REF_OVERLAY.exists():
        return None
    import sys

    spec = importlib.util.spec_from_file_location("_reference_zcutlass_overlay", REF_OVERLAY)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod  # dataclasses resolve annotations through sys.modules
    spec.loader.exec_module(mod)
    return mod


def test_routing_policy_families_and_reasons():
    p = RoutingPolicy()
    assert p.family(16, 1024, 1024) == "decode"
    assert p.family(17, 1024, 1024) == "fallback"
    assert p.family(32, 4096, 4096) == "prefill"
    assert p.family(256, 4096, 4096) == "prefill"
    assert p.family(300, 4096, 4096) == "fallback"
    assert p.family(512, 4096, 4096) == "large"
    assert p.family(4096, 512, 4096) == "fallback"
    assert p.reject_reason(8, 64, 64) == "shape_not_target_bucket"
    assert p.reject_reason(4096, 4096, 4096) == "family_not_promoted"
    assert RoutingPolicy(promoted_families=("large",)).reject_reason(4096, 4096, 4096) is None
    assert RoutingPolicy(enabled=False).reject_reason(8, 64, 64) is None


def test_stats():
    s = OverlayStats()
    assert s.hit_rate == 0.0
    s.record_hit()
    s.record_miss("x")
    s.record_miss("x")
    assert (s.hits, s.misses, s.total, s.fallback_reasons) == (1, 2, 3, {"x": 2})
    assert abs(s.hit_rate - 1 / 3) < 1e-12


def _calls():
    g = torch.Generator().manual_seed(0)
    a = torch.randn(8, 64, generator=g).half()
    b = torch.randn(64, 128, generator=g).half()
    c = torch.randn(8, 128, generator=g).half()
    bias = torch.randn(128, generator=g).half()
    return [
        ("gemm", (a, b), {}),
        ("gemm", (a, b), {"bias": bias}),
        ("gemm", (a, b), {"beta": 1.0}),  # beta without C
        ("gemm", (a, b, c, bias), {"alpha": 0.5, "beta": 2.0}),
        ("linear", (a, b.t().contiguous(), bias), {}),
        ("linear", (a, b, bias), {"weight_is_transposed": True}),
    ]


def _replay(overlay_cls, calls, **kw):
    ov = overlay_cls(**kw)
    outs = []
    for name, args, kwargs in calls:
        try:
            outs.append(getattr(ov, name)(*args, **kwargs))
        except Exception as exc:  # the reference raises for beta without C in torch.matmul? keep the type
            outs.append(type(exc).__name__)
    return ov, outs


@pytest.mark.parametrize("enable", [True, False])
def test_cpu_calls_fall_back_with_reference_reasons(enable):
    calls = _calls()
    ov, outs = _replay(ZCutlassGemmOverlay, calls, enable_zcutlass=enable)
    reasons = ov.stats.fallback_reasons
    assert ov.stats.hits == 0 and ov.stats.misses == len(calls)
    if enable:
        assert reasons == {"cpu_tensor": 4, "beta_without_c": 1, "weight_not_pretransposed": 1}
    else:
        assert reasons == {"zcutlass_disabled": 5, "weight_not_pretransposed": 1}
    a, b = calls[0][1]
    torch.testing.assert_close(outs[0], torch.matmul(a, b))
    ref = _reference_overlay_module()
    if ref is not None:
        # Same calls through the reference overlay with its extension missing:
        # identical fallback values; reasons identical except the first gate.
        ref_ov, ref_outs = _replay(ref.ZCutlassGemmOverlay, calls, enable_zcutlass=enable)
        assert ref_ov.stats.misses == ov.stats.misses
        for mine, theirs in zip(outs, ref_outs):
            if isinstance(mine, torch.Tensor):
                torch.testing.assert_close(mine, theirs, rtol=0, atol=0)
        if not enable:
            assert ref_ov.stats.fallback_reasons == reasons


def test_module_level_functions_and_config_on_cpu():
    a = torch.randn(4, 8).half()
    b = torch.randn(8, 16).half()
    torch.testing.assert_close(zcutlass_torch.gemm(a, b), torch.matmul(a, b))
    w = torch.randn(16, 8).half()
    torch.testing.assert_close(zcutlass_torch.linear(a, w), torch.nn.functional.linear(a, w))
    assert zcutlass_torch.extension_available() in (True, False)


def test_native_weight_layout_reasons_on_cpu():
    ov = ZCutlassGemmOverlay(native_weight_layout=True, force_zcutlass=True)
    x = torch.randn(4, 8).half()
    w = torch.randn(16, 8).half()
    y = ov.linear(x, w)
    torch.testing.assert_close(y, torch.nn.functional.linear(x, w))
    assert ov.stats.fallback_reasons == {"cpu_tensor": 1}


# ---------------------------------------------------------------- vLLM

vllm_linear = pytest.importorskip("vllm.model_executor.layers.linear")


class DummyVllmLinear(torch.nn.Module):
    """A Linear layer as vLLM hands it to a LinearMethod (weight [N, K])."""

    def __init__(self, n, k, bias=True, prefix="model.layers.0.self_attn.qkv_proj", dtype=torch.float16):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.randn(n, k, dtype=dtype) * k ** -0.5, requires_grad=False)
        self.bias = torch.nn.Parameter(torch.randn(n, dtype=dtype) * 0.1, requires_grad=False) if bias else None
        self.prefix = prefix
        self.quant_method = vllm_linear.UnquantizedLinearMethod()


def test_linear_method_install_and_cpu_fallback(monkeypatch):
    from zcutlass_vllm import ZCutlassUnquantizedLinearMethod, install_zcutlass_unquantized_linear_method

    layer = DummyVllmLinear(2048, 1536)
    m = install_zcutlass_unquantized_linear_method(layer, promoted_families=("prefill",))
    assert isinstance(layer.quant_method, ZCutlassUnquantizedLinearMethod)
    assert install_zcutlass_unquantized_linear_method(layer) is m  # idempotent
    x = torch.randn(256, 1536, dtype=torch.float16)
    y = m.apply(layer, x, layer.bias)
    torch.testing.assert_close(y, torch.nn.functional.linear(x, layer.weight, layer.bias), rtol=2e-2, atol=2e-2)
    # prefill family promoted -> transposed-weight cache built, CPU tensors rejected
    assert m.last_trace["fallback_reason"] == "cpu_tensor"
    assert m.last_trace["weight_cache"] == "miss"
    m.apply(layer, x, layer.bias)
    assert m.last_trace["weight_cache"] == "hit"
    m.process_weights_after_loading(layer)
    assert not hasattr(layer, "_zcutlass_weight_t_cache")
    # an unpromoted family is decided from shapes alone
    x8 = torch.randn(8, 1536, dtype=torch.float16)
    m.apply(layer, x8, layer.bias)
    assert m.last_trace["fallback_reason"] == "family_not_promoted"
    assert m.last_trace["weight_cache"] == "skipped"
    assert m.stats.fallback_reasons["family_not_promoted"] == 1
    # measured profit policy reasons
    monkeypatch.setenv("ZCUTLASS_VLLM_PROFIT_POLICY", "measured")
    xb = torch.randn(128, 1536, dtype=torch.bfloat16)
    assert m._profit_policy_reject_reason(layer, xb, 128, 2048, 1536, "prefill") == "profit_policy_dtype_not_promoted"
    assert m._profit_policy_reject_reason(layer, x, 256, 2048, 1536, "prefill") is None
    assert m._profit_policy_reject_reason(layer, x, 128, 2048, 1536, "prefill") == "profit_policy_shape_not_promoted"
    monkeypatch.setenv("ZCUTLASS_VLLM_PROFIT_POLICY", "bogus")
    assert m._profit_policy_reject_reason(layer, x, 256, 2048, 1536, "prefill") == "profit_policy_unknown"


def test_native_weight_method_has_no_transposed_copy():
    from zcutlass_vllm import install_zcutlass_unquantized_linear_method

    layer = DummyVllmLinear(2048, 1536)
    m = install_zcutlass_unquantized_linear_method(layer, promoted_families=("prefill",), native_weight_layout=True)
    x = torch.randn(64, 1536, dtype=torch.float16)
    y = m.apply(layer, x, layer.bias)
    torch.testing.assert_close(y, torch.nn.functional.linear(x, layer.weight, layer.bias), rtol=2e-2, atol=2e-2)
    assert m.last_trace["weight_cache"] == "native"
    assert not hasattr(layer, "_zcutlass_weight_t_cache")


def test_route_row_and_plugin(tmp_path, monkeypatch):
    from zcutlass_vllm.plugin import register, state
    from zcutlass_vllm.route_logger import RouteLogger, build_route_row, shape_family

    assert shape_family(8, 4096, 4096) == "decode" and shape_family(8, 512, 4096) == "fallback"
    layer = DummyVllmLinear(4096, 4096, prefix="model.layers.3.mlp.down_proj")
    x = torch.randn(8, 4096, dtype=torch.float16)
    row = build_route_row(layer=layer, layer_class="RowParallelLinear", input_tensor=x, output=(x,), latency_us=1.5,
                          trace={"fallback_reason": None, "hit_count": 1, "kernel_name": "k"})
    assert row["route"] == "zcutlass" and row["m"] == 8 and row["n"] == 4096 and row["shape_family"] == "decode"
    RouteLogger(tmp_path / "r.jsonl").write(row)
    assert (tmp_path / "r.jsonl").read_text().count("\n") == 1
    monkeypatch.delenv("ZCUTLASS_VLLM_ENABLE", raising=False)
    register()
    register()
    assert state().registered and os.environ["ZCUTLASS_VLLM_PLUGIN_LOADED"] == "1"
