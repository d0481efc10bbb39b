"""Out-of-tree vLLM Linear classes that install the zcutlass LinearMethod.

Mirrors python/zcutlass_vllm/oot_linear.py in supercatking/zcutlass: the
layer filter (ZCUTLASS_VLLM_LAYER_FILTER, default qkv_proj/gate_up_proj/
down_proj/o_proj), ZCUTLASS_VLLM_ALLOW_FAMILIES, the measured-profit install
skip, per-forward route logging, and OOT subclasses of Column/MergedColumn/
QKV/RowParallelLinear registered through PluggableLayer.register_oot. vLLM
still performs the tensor-parallel all-reduce of RowParallelLinear.

ZCUTLASS_VLLM_NATIVE_WEIGHT=1 (new) installs the method with
native_weight_layout=True: weights are consumed in their [N, K] layout.
"""

from __future__ import annotations

import os
import time
from typing import Any

from .linear_method import install_zcutlass_unquantized_linear_method
from .route_logger import build_route_row, csv_env, env_enabled, make_route_logger

DEFAULT_LAYER_FILTER = ("qkv_proj", "gate_up_proj", "down_proj", "o_proj")
TARGET_LAYER_CLASS_NAMES = ("QKVParallelLinear", "MergedColumnParallelLinear", "ColumnParallelLinear",
                            "RowParallelLinear")

_REGISTERED = False


def _layer_filter() -> tuple[str, ...]:
    return csv_env("ZCUTLASS_VLLM_LAYER_FILTER", DEFAULT_LAYER_FILTER)


def _allow_families() -> tuple[str, ...]:
    return csv_env("ZCUTLASS_VLLM_ALLOW_FAMILIES", ())


def _matches_layer_filter(prefix: str) -> bool:
    filters = _layer_filter()
    if not filters:
        return False
    if "*" in filters or "all" in filters:
        return True
    return any(prefix.endswith(tok) or tok in prefix for tok in filters)


def _skip_install_for_profit_policy(layer: Any) -> str | None:
    if os.environ.get("ZCUTLASS_VLLM_PROFIT_POLICY", "off").strip().lower() != "measured":
        return None
    if "qkv_proj" not in str(getattr(layer, "prefix", "")).lower():
        return "profit_policy_layer_not_promoted"
    dtype = str(getattr(getattr(layer, "weight", None), "dtype", "")).lower()
    if dtype not in ("torch.float16", "float16", "f16", "half", "torch.half"):
        return "profit_policy_dtype_not_promoted"
    return None


class ZCutlassOotLinearMixin:
    """Installed on selected vLLM Linear classes."""

    def _zcutlass_post_init(self) -> None:
        self._zcutlass_route_logger = make_route_logger()
        self._zcutlass_install_error = None
        self._zcutlass_target_layer = False
        self._zcutlass_overlay_method = None
        if not env_enabled("ZCUTLASS_VLLM_ENABLE"):
            return
        if not _matches_layer_filter(str(getattr(self, "prefix", ""))):
            return
        skip = _skip_install_for_profit_policy(self)
        if skip is not None:
            self._zcutlass_install_error = skip
            return
        self._zcutlass_target_layer = True
        try:
            self._zcutlass_overlay_method = install_zcutlass_unquantized_linear_method(
                self, promoted_families=_allow_families(), materialize_inputs=True, cache_transposed_weight=True,
                native_weight_layout=env_enabled("ZCUTLASS_VLLM_NATIVE_WEIGHT"))
        except Exception as exc:
            self._zcutlass_install_error = str(exc)

    def _zcutlass_log_forward(self, input_tensor: Any, output: Any, latency_us: float) -> None:
        logger = getattr(self, "_zcutlass_route_logger", None)
        if logger is None or not getattr(self, "_zcutlass_target_layer", False):
            return
        trace = getattr(getattr(self, "quant_method", None), "last_trace", None)
        logger.write(build_route_row(layer=self, layer_class=self.__class__.__name__, input_tensor=input_tensor,
                                     output=output, latency_us=latency_us, trace=trace,
                                     install_error=getattr(self, "_zcutlass_install_error", None)))

    def forward(self, input_):
        if getattr(self, "_zcutlass_route_logger", None) is None or not getattr(self, "_zcutlass_target_layer", False):
            return super().forward(input_)
        t0 = time.perf_counter_ns()
        output = super().forward(input_)
        self._zcutlass_log_forward(input_, output, (time.perf_counter_ns() - t0) / 1000.0)
        return output


def register_oot_linear_layers() -> bool:
    """Registers the zcutlass OOT classes with vLLM (idempotent)."""
    global _REGISTERED
    if _REGISTERED:
        return True
    if not env_enabled("ZCUTLASS_VLLM_ENABLE"):
        return False
    from vllm.model_executor.custom_op import PluggableLayer, op_registry_oot
    from vllm.model_executor.layers.linear import (
        ColumnParallelLinear,
        MergedColumnParallelLinear,
        QKVParallelLinear,
        RowParallelLinear,
    )

    if any(name in op_registry_oot
           and not str(getattr(op_registry_oot[name], "__module__", "")).startswith(("zcutlass_vllm", "zcutlass_b200"))
           for name in TARGET_LAYER_CLASS_NAMES):
        return False
    bases = {"ColumnParallelLinear": ColumnParallelLinear, "MergedColumnParallelLinear": MergedColumnParallelLinear,
             "QKVParallelLinear": QKVParallelLinear, "RowParallelLinear": RowParallelLinear}
    for name, base in bases.items():
        if name in op_registry_oot:
            continue

        def _init(self, *args: Any, __base=base, **kwargs: Any) -> None:
            __base.__init__(self, *args, **kwargs)
            self._zcutlass_post_init()

        cls = type(f"ZCutlass{name}", (ZCutlassOotLinearMixin, base), {"__init__": _init, "__module__": __name__})
        PluggableLayer.register_oot(name=name)(cls)
    _REGISTERED = all(name in op_registry_oot for name in TARGET_LAYER_CLASS_NAMES)
    return _REGISTERED
