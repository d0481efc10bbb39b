"""vLLM LinearMethod that routes selected Linear layers to zcutlass.

Mirrors ZCutlassUnquantizedLinearMethod (python/zcutlass_vllm/linear_method.py
in supercatking/zcutlass): wraps vLLM's UnquantizedLinearMethod, decides misses
from shapes before touching the weight (61-83), the measured profit policy
ZCUTLASS_VLLM_PROFIT_POLICY and its reason strings (85-111), a transposed
weight cache keyed on (data_ptr, shape, dtype, device) (113-134), apply()
(136-161) and the installer (169-198).

B200 addition (opt-in, native_weight_layout=True): the vLLM weight stays in
its [N, K] layout and goes to the kernels as column-major B; no transposed
copy is made or cached (trace key weight_cache = "native").
"""

from __future__ import annotations

import os
from typing import Any, Optional

from .linear import ZCutlassVllmLinearAdapter

try:  # vLLM is optional outside serving environments
    from vllm.model_executor.layers.linear import LinearMethodBase, UnquantizedLinearMethod
except Exception:  # pragma: no cover - exercised without vLLM
    LinearMethodBase = object  # type: ignore[assignment,misc]
    UnquantizedLinearMethod = None  # type: ignore[assignment]


_HALF_NAMES = ("torch.float16", "float16", "f16", "half", "torch.half")


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

    @property
    def stats(self):
        return self.adapter.stats

    @property
    def last_trace(self):
        return self.adapter.last_trace

    def create_weights(self, *args: Any, **kwargs: Any):
        return self.delegate.create_weights(*args, **kwargs)

    def process_weights_after_loading(self, layer) -> None:
        if hasattr(self.delegate, "process_weights_after_loading"):
            self.delegate.process_weights_after_loading(layer)
        clear_zcutlass_weight_cache(layer)

    def _delegate_without_transpose_reason(self, layer, x) -> tuple[str, str] | None:
        if self.adapter.force_zcutlass:
            return None
        xs = getattr(x, "shape", None)
        ws = getattr(getattr(layer, "weight", None), "shape", None)
        if xs is None or ws is None or len(xs) != 2 or len(ws) != 2:
            return ("rank_not_2", "unknown")
        m, k = int(xs[0]), int(xs[1])
        n, weight_k = int(ws[0]), int(ws[1])
        if k != weight_k:
            return ("inner_dimension_mismatch", "unknown")
        family = self.adapter.routing_policy.family(m, n, k)
        if family == "fallback":
            return ("shape_not_target_bucket", family)
        if family not in self.adapter.promoted_families:
            return ("family_not_promoted", family)
        reason = self._profit_policy_reject_reason(layer, x, m, n, k, family)
        return (reason, family) if reason is not None else None

    def _profit_policy_reject_reason(self, layer, x, m: int, n: int, k: int, family: str) -> str | None:
        """ZCUTLASS_VLLM_PROFIT_POLICY: off/all/experimental route everything the
        family policy allows; `measured` keeps only the subset the reference
        measured as profitable (f16 prefill qkv_proj with bias, 256x2048x1536)."""
        policy = os.environ.get("ZCUTLASS_VLLM_PROFIT_POLICY", "off").strip().lower()
        if policy in ("", "0", "off", "none", "false", "disabled", "all", "experimental"):
            return None
        if policy != "measured":
            return "profit_policy_unknown"
        if str(getattr(x, "dtype", "")).lower() not in _HALF_NAMES:
            return "profit_policy_dtype_not_promoted"
        if family != "prefill":
            return "profit_policy_family_not_promoted"
        if getattr(layer, "bias", None) is None:
            return "profit_policy_bias_not_promoted"
        if "qkv_proj" not in str(getattr(layer, "prefix", "")).lower():
            return "profit_policy_layer_not_promoted"
        if (m, n, k) == (256, 2048, 1536):
            return None
        return "profit_policy_shape_not_promoted"

    def _transposed_weight(self, layer):
        weight = layer.weight
        if not self.cache_transposed_weight:
            self.last_weight_cache = "disabled"
            return weight.t().contiguous()
        signature = (int(weight.data_ptr()) if hasattr(weight, "data_ptr") else 0, tuple(weight.shape),
                     str(weight.dtype), str(weight.device))
        cached = getattr(layer, "_zcutlass_weight_t_cache", None)
        if cached is not None and cached[0] == signature:
            self.last_weight_cache = "hit"
            return cached[1]
        weight_t = weight.t().contiguous()
        setattr(layer, "_zcutlass_weight_t_cache", (signature, weight_t))
        self.last_weight_cache = "miss"
        return weight_t

    def apply(self, layer, x, bias=None):
        fast = self._delegate_without_transpose_reason(layer, x)
        if fast is not None:
            reason, family = fast
            self.last_weight_cache = "skipped"
            self.adapter._record_fallback_trace(reason=reason, family=family,
                                                fallback_path_name="vllm_unquantized_fallback")
        elif self.native_weight_layout:
            self.last_weight_cache = "native"
            out = self.adapter.run_native(x, layer.weight, bias,
                                          fallback_fn=lambda: self.delegate.apply(layer, x, bias),
                                          fallback_path_name="vllm_unquantized_fallback")
            self._tag_trace()
            return out
        else:
            weight_t = self._transposed_weight(layer)
            out = self.adapter.run(x, weight_t, bias, weight_is_transposed=True,
                                   fallback_fn=lambda: self.delegate.apply(layer, x, bias),
                                   fallback_path_name="vllm_unquantized_fallback")
            self._tag_trace()
            return out
        self._tag_trace()
        return self.delegate.apply(layer, x, bias)

    def _tag_trace(self) -> None:
        if self.adapter.last_trace is not None:
            self.adapter.last_trace["weight_cache"] = self.last_weight_cache


def clear_zcutlass_weight_cache(layer) -> None:
    if hasattr(layer, "_zcutlass_weight_t_cache"):
        delattr(layer, "_zcutlass_weight_t_cache")


def install_zcutlass_unquantized_linear_method(layer, *, promoted_families: tuple[str, ...] = (),
                                               force_zcutlass: bool = False, materialize_inputs: bool = True,
                                               cache_transposed_weight: bool = True,
                                               native_weight_layout: bool = False) -> ZCutlassUnquantizedLinearMethod:
    """Replaces one vLLM Linear layer's unquantized method with the zcutlass wrapper."""
    if UnquantizedLinearMethod is None:
        raise ImportError("vLLM is required to install ZCutlassUnquantizedLinearMethod")
    current = getattr(layer, "quant_method", None)
    if isinstance(current, ZCutlassUnquantizedLinearMethod):
        return current
    if current is not None and not isinstance(current, UnquantizedLinearMethod):
        raise TypeError("zcutlass can only wrap vLLM UnquantizedLinearMethod layers in v1.5")
    method = ZCutlassUnquantizedLinearMethod(current, promoted_families=promoted_families,
                                             force_zcutlass=force_zcutlass, materialize_inputs=materialize_inputs,
                                             cache_transposed_weight=cache_transposed_weight,
                                             native_weight_layout=native_weight_layout)
    layer.quant_method = method
    return method
