"""The drop-in packages' routing tables against the reference's, on CPU.

tests/golden/reference_boundary_tables.json holds, in order, the fallback
reasons each reference decision point returns, the keys of an adapter trace
and the columns of a route row, read from the reference's sources by
tests/golden/make_boundary_tables.py. The rule tables of zcutlass_b200 must
list the same reasons in the same order, and -- checked here with duck-typed
operands, so no GPU is needed -- a call that breaks several rules reports
the first of them.
"""

from __future__ import annotations

import json
from pathlib import Path

import pytest
import torch

from zcutlass_b200.routing import first_reason
from zcutlass_b200.zcutlass_torch import overlay as ov
from zcutlass_b200.zcutlass_vllm import linear as adapter_mod
from zcutlass_b200.zcutlass_vllm import linear_method as method_mod
from zcutlass_b200.zcutlass_vllm import oot_linear as oot_mod
from zcutlass_b200.zcutlass_vllm import route_logger

REF = json.loads((Path(__file__).parent / "golden" / "reference_boundary_tables.json").read_text())


def reasons(*tables):
    return [r.reason for t in tables for r in t]


def test_overlay_reason_order():
    assert reasons(ov._GATE_RULES, ov._SHAPE_RULES, ov._OPERAND_RULES) == REF["overlay_reject_reasons"]
    assert reasons(ov._POLICY_RULES) == REF["policy_reject_reasons"]
    fams = [b.family for b in ov.RoutingPolicy().buckets()] + ["fallback"]
    assert fams == REF["policy_families"]


def test_vllm_reason_orders():
    assert reasons(adapter_mod.FAST_RULES) == REF["adapter_fast_reasons"]
    assert reasons(adapter_mod.SHAPE_RULES) == REF["method_delegate_reasons"]
    assert reasons(method_mod.PROFIT_RULES) == REF["profit_policy_reasons"]
    assert reasons(oot_mod.INSTALL_SKIP_RULES) == REF["install_skip_reasons"]


def test_route_row_columns():
    row = route_logger.build_route_row(layer=object(), layer_class="X", input_tensor=None, output=None,
                                       latency_us=0.0, trace=None)
    assert list(row) == REF["route_row_keys"]


def test_adapter_trace_keys():
    a = adapter_mod.ZCutlassVllmLinearAdapter()
    x, w = torch.randn(4, 8), torch.randn(8, 16)
    a.run(x, w, weight_is_transposed=True, fallback_fn=lambda: x @ w)
    assert list(a.last_trace) == REF["adapter_trace_keys"]
    assert a.last_trace["fallback_reason"] == "shape_not_target_bucket"
    assert (a.stats.calls, a.stats.hits, a.stats.misses) == (1, 0, 1)


class FakeTensor:
    """Just the attributes the overlay's rules read."""

    def __init__(self, shape, *, cuda=True, contiguous=True, dtype=torch.float16):
        self.shape = tuple(shape)
        self.is_cuda = cuda
        self._contig = contiguous
        self.dtype = dtype

    def dim(self):
        return len(self.shape)

    def is_contiguous(self):
        return self._contig


def _good():
    return dict(a=FakeTensor((64, 32)), b=FakeTensor((32, 48)), c=FakeTensor((64, 48)), bias=FakeTensor((48,)),
                beta=1.0)


# For every operand reason, one way to break exactly that rule.
BREAKS = {
    "beta_without_c": lambda d: d.update(c=None),
    "cpu_tensor": lambda d: d.update(a=FakeTensor((64, 32), cuda=False)),
    "rank_not_2": lambda d: d.update(b=FakeTensor((32, 48, 1))),
    "inner_dimension_mismatch": lambda d: d.update(b=FakeTensor((31, 48))),
    "non_contiguous_ab": lambda d: d.update(b=FakeTensor((32, 48), contiguous=False)),
    "mixed_dtype": lambda d: d.update(b=FakeTensor((32, 48), dtype=torch.bfloat16)),
    "unsupported_dtype": lambda d: d.update(a=FakeTensor((64, 32), dtype=torch.float32),
                                            b=FakeTensor((32, 48), dtype=torch.float32),
                                            c=FakeTensor((64, 48), dtype=torch.float32),
                                            bias=FakeTensor((48,), dtype=torch.float32)),
    "cpu_c_tensor": lambda d: d.update(c=FakeTensor((64, 48), cuda=False)),
    "c_shape_mismatch": lambda d: d.update(c=FakeTensor((64, 47))),
    "c_dtype_mismatch": lambda d: d.update(c=FakeTensor((64, 48), dtype=torch.bfloat16)),
    "non_contiguous_c": lambda d: d.update(c=FakeTensor((64, 48), contiguous=False)),
    "cpu_bias_tensor": lambda d: d.update(bias=FakeTensor((48,), cuda=False)),
    "bias_shape_mismatch": lambda d: d.update(bias=FakeTensor((47,))),
    "bias_dtype_mismatch": lambda d: d.update(bias=FakeTensor((48,), dtype=torch.bfloat16)),
    "non_contiguous_bias": lambda d: d.update(bias=FakeTensor((48,), contiguous=False)),
}
OPERAND_ORDER = REF["overlay_reject_reasons"][2:]


def _first(d):
    call = ov._Call(**d)
    return first_reason(ov._SHAPE_RULES, call) or first_reason(ov._OPERAND_RULES, call)


def test_operand_rules_fire_alone():
    assert _first(_good()) is None
    assert sorted(BREAKS) == sorted(OPERAND_ORDER)
    for reason, brk in BREAKS.items():
        d = _good()
        brk(d)
        assert _first(d) == reason, reason


@pytest.mark.parametrize("i", range(len(OPERAND_ORDER) - 1))
def test_earlier_rule_wins(i):
    """Breaking rules i and j > i reports rule i (the reference's order)."""
    for j in range(i + 1, len(OPERAND_ORDER)):
        first, later = OPERAND_ORDER[i], OPERAND_ORDER[j]
        d = _good()
        BREAKS[later](d)
        BREAKS[first](d)
        if first in ("beta_without_c",) or (first == "unsupported_dtype" and later.endswith("dtype_mismatch")):
            continue  # applying the first break rewrites the operand the later one broke
        assert _first(d) == first, (first, later)


def test_profit_policy_first_reason(monkeypatch):
    layer = type("L", (), {"bias": None, "prefix": "model.layers.0.mlp.down_proj"})()
    x = FakeTensor((128, 1536), dtype=torch.bfloat16)
    m = method_mod.ZCutlassUnquantizedLinearMethod.__new__(method_mod.ZCutlassUnquantizedLinearMethod)
    monkeypatch.setenv("ZCUTLASS_VLLM_PROFIT_POLICY", "measured")
    # every profit rule is broken: the first one (dtype) is reported
    assert m._profit_policy_reject_reason(layer, x, 128, 2048, 1536, "decode") == "profit_policy_dtype_not_promoted"
    for word in ("off", "all", "experimental", ""):
        monkeypatch.setenv("ZCUTLASS_VLLM_PROFIT_POLICY", word)
        assert m._profit_policy_reject_reason(layer, x, 128, 2048, 1536, "decode") is None
