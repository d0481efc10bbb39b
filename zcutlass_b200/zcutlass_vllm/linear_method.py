"""vLLM LinearMethod that sends selected unquantized Linear layers to zcutlass.

Public surface of the reference's method (python/zcutlass_vllm/linear_method.py
in supercatking/zcutlass): ZCutlassUnquantizedLinearMethod (create_weights /
process_weights_after_loading / apply, `stats`, `last_trace` with its
`weight_cache` key), clear_zcutlass_weight_cache and
install_zcutlass_unquantized_linear_method. apply() decides misses from the
layer's shapes and the profit policy (ZCUTLASS_VLLM_PROFIT_POLICY) before the
weight is touched, then runs the adapter on a [K, N] copy of the weight that
is made once and reused while the weight's storage is unchanged.

B200 addition (opt-in, native_weight_layout=True): the vLLM weight stays in
its [N, K] layout and runs as column-major B, so no [K, N] copy exists
(weight_cache = "native"); that removes the second copy of every routed
weight from device memory.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Optional

from ..routing import Rule, env_word, first_reason
from .linear import SHAPE_RULES, LinearShape, ZCutlassVllmLinearAdapter, fast_reason

try:  # vLLM is optional outside serving environments
    from vllm.model_executor.layers.linear import LinearMethodBase, UnquantizedLinearMethod
except Exception:  # pragma: no cover - exercised without vLLM
    LinearMethodBase = object  # type: ignore[assignment,misc]
    UnquantizedLinearMethod = None  # type: ignore[assignment]

FALLBACK_PATH = "vllm_unquantized_fallback"

# ---------------------------------------------------------------- profit policy

# Policy words that route everything the family policy allows.
PASS_THROUGH_POLICIES = frozenset({"", "0", "off", "none", "false", "disabled", "all", "experimental"})
HALF_DTYPE_NAMES = frozenset({"torch.float16", "float16", "f16", "half", "torch.half"})
# The one (m, n, k) the reference measured as profitable: f16 prefill qkv_proj with bias.
MEASURED_SHAPES = frozenset({(256, 2048, 1536)})


@dataclass(frozen=True)
class ProfitCase:
    policy: str
    dtype: str
    family: str
    has_bias: bool
    prefix: str
    mnk: tuple[int, int, int]


# `measured` keeps only the profitable subset; reasons in the reference's
# order (python/zcutlass_vllm/linear_method.py:85-111).
PROFIT_RULES = (
    Rule("profit_policy_unknown", lambda c: c.policy != "measured"),
    Rule("profit_policy_dtype_not_promoted", lambda c: c.dtype not in HALF_DTYPE_NAMES),
    Rule("profit_policy_family_not_promoted", lambda c: c.family != "prefill"),
    Rule("profit_policy_bias_not_promoted", lambda c: not c.has_bias),
    Rule("profit_policy_layer_not_promoted", lambda c: "qkv_proj" not in c.prefix),
    Rule("profit_policy_shape_not_promoted", lambda c: c.mnk not in MEASURED_SHAPES),
)


def profit_policy() -> str:
    return env_word("ZCUTLASS_VLLM_PROFIT_POLICY", "off")


# ---------------------------------------------------------------- [K, N] weight copies

_CACHE_ATTR = "_zcutlass_weight_t_cache"


def _storage_key(weight) -> tuple:
    """Changes whenever the weight's storage, shape, dtype or device does."""
    ptr = int(weight.data_ptr()) if hasattr(weight, "data_ptr") else 0
    return ptr, tuple(weight.shape), str(weight.dtype), str(weight.device)


def transposed_weight(layer, enabled: bool = True) -> tuple[Any, str]:
    """(contiguous [K, N] copy of layer.weight, how it was obtained: "hit",
    "miss" (made and kept on the layer) or "disabled" (made, not kept))."""
    w = layer.weight
    if not enabled:
        return w.t().contiguous(), "disabled"
    key = _storage_key(w)
    kept = getattr(layer, _CACHE_ATTR, None)
    if kept is not None and kept[0] == key:
        return kept[1], "hit"
    copy = w.t().contiguous()
    setattr(layer, _CACHE_ATTR, (key, copy))
    return copy, "miss"


def clear_zcutlass_weight_cache(layer) -> None:
    """Drops the layer's kept [K, N] copy, if any."""
    if hasattr(layer, _CACHE_ATTR):
        delattr(layer, _CACHE_ATTR)


# ---------------------------------------------------------------- the method


class ZCutlassUnquantizedLinearMethod(LinearMethodBase):  # type: ignore[misc,valid-type]
    """vLLM unquantized Linear with zcutlass-first routing."""

    def __init__(self, delegate: Optional[Any] = None, *, promoted_families: tuple[str, ...] = (),
                 force_zcutlass: bool = False, materialize_inputs: bool = True,
                 cache_transposed_weight: bool = True, native_weight_layout: bool = False) -> None:
        if UnquantizedLinearMethod is None:
            raise ImportError("vLLM is required to construct ZCutlassUnquantizedLinearMethod")
        self.delegate = delegate if delegate is not None else UnquantizedLinearMethod()
        self.adapter = ZCutlassVllmLinearAdapter(promoted_families=promoted_families, force_zcutlass=force_zcutlass,
                                                 materialize_inputs=materialize_inputs)
        self.cache_transposed_weight = cache_transposed_weight
        self.native_weight_layout = native_weight_layout
        self.last_weight_cache = "unknown"

    stats = property(lambda self: self.adapter.stats)
    last_trace = property(lambda self: self.adapter.last_trace)

    def create_weights(self, *args: Any, **kwargs: Any):
        return self.delegate.create_weights(*args, **kwargs)

    def process_weights_after_loading(self, layer) -> None:
        if hasattr(self.delegate, "process_weights_after_loading"):
            self.delegate.process_weights_after_loading(layer)
        clear_zcutlass_weight_cache(layer)

    def _profit_policy_reject_reason(self, layer, x, m: int, n: int, k: int, family: str) -> Optional[str]:
        policy = profit_policy()
        if policy in PASS_THROUGH_POLICIES:
            return None
        case = ProfitCase(policy, str(getattr(x, "dtype", "")).lower(), family, getattr(layer, "bias", None) is not None,
                          str(getattr(layer, "prefix", "")).lower(), (m, n, k))
        return first_reason(PROFIT_RULES, case)

    def _delegate_without_transpose_reason(self, layer, x) -> Optional[tuple[str, str]]:
        """(reason, family) when this call goes to vLLM's own GEMM whatever the
        operands hold: decided from shapes and policy, before any weight copy."""
        if self.adapter.force_zcutlass:
            return None
        shape = LinearShape.of(x, getattr(layer, "weight", None), self.adapter.routing_policy, weight_nk=True)
        fast = fast_reason(SHAPE_RULES, shape)
        if fast is not None:
            return fast
        reason = self._profit_policy_reject_reason(layer, x, shape.m, shape.n, shape.k, shape.family)
        return None if reason is None else (reason, shape.family)

    def apply(self, layer, x, bias=None):
        def vllm_gemm():
            return self.delegate.apply(layer, x, bias)

        early = self._delegate_without_transpose_reason(layer, x)
        if early is not None:
            self.last_weight_cache = "skipped"
            self.adapter.record_delegation(early[0], early[1], FALLBACK_PATH)
            out = vllm_gemm()
        elif self.native_weight_layout:
            self.last_weight_cache = "native"
            out = self.adapter.run_native(x, layer.weight, bias, fallback_fn=vllm_gemm, fallback_path_name=FALLBACK_PATH)
        else:
            weight_kn, self.last_weight_cache = transposed_weight(layer, self.cache_transposed_weight)
            out = self.adapter.run(x, weight_kn, bias, weight_is_transposed=True, fallback_fn=vllm_gemm,
                                   fallback_path_name=FALLBACK_PATH)
        if self.adapter.last_trace is not None:
            self.adapter.last_trace["weight_cache"] = self.last_weight_cache
        return out


def install_zcutlass_unquantized_linear_method(layer, *, promoted_families: tuple[str, ...] = (),
                                               force_zcutlass: bool = False, materialize_inputs: bool = True,
                                               cache_transposed_weight: bool = True,
                                               native_weight_layout: bool = False) -> ZCutlassUnquantizedLinearMethod:
    """Wraps one vLLM Linear layer's UnquantizedLinearMethod (idempotent)."""
    if UnquantizedLinearMethod is None:
        raise ImportError("vLLM is required to install ZCutlassUnquantizedLinearMethod")
    current = getattr(layer, "quant_method", None)
    if isinstance(current, ZCutlassUnquantizedLinearMethod):
        return current
    if current is not None and not isinstance(current, UnquantizedLinearMethod):
        raise TypeError("zcutlass can only wrap vLLM UnquantizedLinearMethod layers in v1.5")
    layer.quant_method = ZCutlassUnquantizedLinearMethod(
        current, promoted_families=promoted_families, force_zcutlass=force_zcutlass,
        materialize_inputs=materialize_inputs, cache_transposed_weight=cache_transposed_weight,
        native_weight_layout=native_weight_layout)
    return layer.quant_method
