"""Out-of-tree vLLM Linear classes that install the zcutlass LinearMethod.

Public surface of the reference's OOT module (python/zcutlass_vllm/oot_linear.py
in supercatking/zcutlass): ZCutlassOotLinearMixin and
register_oot_linear_layers(), which registers subclasses of vLLM's
ColumnParallelLinear, MergedColumnParallelLinear, QKVParallelLinear and
RowParallelLinear through PluggableLayer.register_oot. A constructed layer
installs the method when ZCUTLASS_VLLM_ENABLE is on, its prefix passes
ZCUTLASS_VLLM_LAYER_FILTER and the measured profit policy does not skip it
(`INSTALL_SKIP_RULES`); ZCUTLASS_VLLM_ALLOW_FAMILIES lists the promoted
families; forwards of installed layers write route rows when route logging is
on. vLLM still performs RowParallelLinear's tensor-parallel all-reduce.

ZCUTLASS_VLLM_NATIVE_WEIGHT=1 (B200 addition) installs the method with
native_weight_layout=True: weights run in their [N, K] layout, no copy.
"""

from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Any, Optional

from ..routing import Rule, env_flag, env_list, first_reason
from .linear_method import HALF_DTYPE_NAMES, install_zcutlass_unquantized_linear_method, profit_policy
from .route_logger import build_route_row, make_route_logger

DEFAULT_LAYER_FILTER = ("qkv_proj", "gate_up_proj", "down_proj", "o_proj")
TARGET_LAYER_CLASS_NAMES = ("QKVParallelLinear", "MergedColumnParallelLinear", "ColumnParallelLinear",
                            "RowParallelLinear")


def layer_selected(prefix: str) -> bool:
    """ZCUTLASS_VLLM_LAYER_FILTER: comma-separated name fragments ("*" or
    "all" selects every layer; an empty list none)."""
    tokens = env_list("ZCUTLASS_VLLM_LAYER_FILTER", DEFAULT_LAYER_FILTER)
    if {"*", "all"} & set(tokens):
        return True
    return any(t in prefix for t in tokens)


@dataclass(frozen=True)
class _LayerFacts:
    prefix: str
    weight_dtype: str


# Install skips under the measured profit policy, in the reference's order
# (python/zcutlass_vllm/oot_linear.py:41-52).
INSTALL_SKIP_RULES = (
    Rule("profit_policy_layer_not_promoted", lambda f: "qkv_proj" not in f.prefix),
    Rule("profit_policy_dtype_not_promoted", lambda f: f.weight_dtype not in HALF_DTYPE_NAMES),
)


def install_skip_reason(layer: Any) -> Optional[str]:
    if profit_policy() != "measured":
        return None
    facts = _LayerFacts(str(getattr(layer, "prefix", "")).lower(),
                        str(getattr(getattr(layer, "weight", None), "dtype", "")).lower())
    return first_reason(INSTALL_SKIP_RULES, facts)


class ZCutlassOotLinearMixin:
    """Mixed into the registered vLLM Linear subclasses."""

    def _zcutlass_post_init(self) -> None:
        self._zcutlass_route_logger = make_route_logger()
        self._zcutlass_install_error = None
        self._zcutlass_target_layer = False
        self._zcutlass_overlay_method = None
        if not (env_flag("ZCUTLASS_VLLM_ENABLE") and layer_selected(str(getattr(self, "prefix", "")))):
            return
        self._zcutlass_install_error = install_skip_reason(self)
        if self._zcutlass_install_error is not None:
            return
        self._zcutlass_target_layer = True
        try:
            self._zcutlass_overlay_method = install_zcutlass_unquantized_linear_method(
                self, promoted_families=env_list("ZCUTLASS_VLLM_ALLOW_FAMILIES", ()), materialize_inputs=True,
                cache_transposed_weight=True, native_weight_layout=env_flag("ZCUTLASS_VLLM_NATIVE_WEIGHT"))
        except Exception as exc:
            self._zcutlass_install_error = str(exc)

    def _zcutlass_log_forward(self, input_tensor: Any, output: Any, latency_us: float) -> None:
        logger = getattr(self, "_zcutlass_route_logger", None)
        if logger is None or not getattr(self, "_zcutlass_target_layer", False):
            return
        trace = getattr(getattr(self, "quant_method", None), "last_trace", None)
        logger.write(build_route_row(layer=self, layer_class=type(self).__name__, input_tensor=input_tensor,
                                     output=output, latency_us=latency_us, trace=trace,
                                     install_error=getattr(self, "_zcutlass_install_error", None)))

    def forward(self, input_):
        logging = getattr(self, "_zcutlass_route_logger", None) is not None and \
            getattr(self, "_zcutlass_target_layer", False)
        if not logging:
            return super().forward(input_)
        t0 = time.perf_counter_ns()
        output = super().forward(input_)
        self._zcutlass_log_forward(input_, output, (time.perf_counter_ns() - t0) / 1000.0)
        return output


_REGISTERED = False


def _ours(cls) -> bool:
    return str(getattr(cls, "__module__", "")).startswith(("zcutlass_vllm", "zcutlass_b200"))


def register_oot_linear_layers() -> bool:
    """Registers the zcutlass OOT classes with vLLM (idempotent). Leaves the
    registry alone when another package already registered one of the names."""
    global _REGISTERED
    if _REGISTERED:
        return True
    if not env_flag("ZCUTLASS_VLLM_ENABLE"):
        return False
    from vllm.model_executor.custom_op import PluggableLayer, op_registry_oot
    from vllm.model_executor.layers import linear as vllm_linear

    if any(name in op_registry_oot and not _ours(op_registry_oot[name]) for name in TARGET_LAYER_CLASS_NAMES):
        return False
    for name in TARGET_LAYER_CLASS_NAMES:
        if name in op_registry_oot:
            continue
        base = getattr(vllm_linear, name)

        def _init(self, *args: Any, __base=base, **kwargs: Any) -> None:
            __base.__init__(self, *args, **kwargs)
            self._zcutlass_post_init()

        PluggableLayer.register_oot(name=name)(
            type(f"ZCutlass{name}", (ZCutlassOotLinearMixin, base), {"__init__": _init, "__module__": __name__}))
    _REGISTERED = all(name in op_registry_oot for name in TARGET_LAYER_CLASS_NAMES)
    return _REGISTERED
