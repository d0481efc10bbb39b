"""Per-forward JSONL route rows for vLLM Linear layers.

Same environment switches, row keys and shape families as the reference
(python/zcutlass_vllm/route_logger.py:13-127 in supercatking/zcutlass):
ZCUTLASS_VLLM_LOG_ROUTES / ZCUTLASS_VLLM_ROUTE_LOG, _MODEL_ID, _ARCHITECTURE.
"""

from __future__ import annotations

import json
import os
import time
from pathlib import Path
from typing import Any


def env_enabled(name: str, default: bool = False) -> bool:
    value = os.environ.get(name)
    if value is None:
        return default
    return value not in ("", "0", "false", "False", "FALSE", "no", "No", "NO")


def csv_env(name: str, default: tuple[str, ...] = ()) -> tuple[str, ...]:
    value = os.environ.get(name)
    if value is None or value.strip() == "":
        return default
    return tuple(part.strip() for part in value.split(",") if part.strip())


def tensor_shape(value: Any) -> list[int]:
    shape = getattr(value, "shape", None)
    return [int(d) for d in shape] if shape is not None else []


def tensor_dtype(value: Any) -> str:
    dtype = getattr(value, "dtype", None)
    return str(dtype) if dtype is not None else "unknown"


def first_tensor(value: Any) -> Any:
    return value[0] if isinstance(value, tuple) and value else value


def shape_family(m: int, n: int, k: int) -> str:
    if n >= 1024 and k >= 1024:
        if m <= 16:
            return "decode"
        if 32 <= m <= 256:
            return "prefill"
        if m >= 512:
            return "large"
    return "fallback"


class RouteLogger:
    """Append-only JSONL writer."""

    def __init__(self, path: str | os.PathLike[str]) -> None:
        self.path = Path(path)

    def write(self, row: dict[str, Any]) -> None:
        self.path.parent.mkdir(parents=True, exist_ok=True)
        with self.path.open("a", encoding="utf-8") as fh:
            fh.write(json.dumps(row, sort_keys=True, default=str) + "\n")


def make_route_logger() -> RouteLogger | None:
    if not env_enabled("ZCUTLASS_VLLM_LOG_ROUTES"):
        return None
    path = os.environ.get("ZCUTLASS_VLLM_ROUTE_LOG")
    return RouteLogger(path) if path else None


def build_route_row(*, layer: Any, layer_class: str, input_tensor: Any, output: Any, latency_us: float,
                    trace: dict[str, Any] | None, install_error: str | None = None) -> dict[str, Any]:
    trace = trace or {}
    in_shape = tensor_shape(input_tensor)
    w_shape = tensor_shape(getattr(layer, "weight", None))
    m = int(in_shape[0]) if len(in_shape) >= 2 else 0
    k = int(in_shape[-1]) if len(in_shape) >= 2 else 0
    n = int(w_shape[0]) if len(w_shape) >= 2 else 0
    reason = trace.get("fallback_reason")
    route = "zcutlass" if reason is None and trace.get("hit_count", 0) else "fallback"
    return {
        "ts_ns": time.time_ns(),
        "pid": os.getpid(),
        "rank": os.environ.get("RANK", ""),
        "local_rank": os.environ.get("LOCAL_RANK", ""),
        "tp_rank": getattr(layer, "tp_rank", ""),
        "tp_size": getattr(layer, "tp_size", ""),
        "model_id": os.environ.get("ZCUTLASS_VLLM_MODEL_ID", ""),
        "architecture": os.environ.get("ZCUTLASS_VLLM_ARCHITECTURE", ""),
        "layer_prefix": getattr(layer, "prefix", ""),
        "layer_class": layer_class,
        "input_shape": in_shape,
        "weight_shape": w_shape,
        "output_shape": tensor_shape(first_tensor(output)),
        "dtype": tensor_dtype(input_tensor),
        "bias": getattr(layer, "bias", None) is not None,
        "m": m,
        "n": n,
        "k": k,
        "shape_family": shape_family(m, n, k),
        "route": route,
        "fallback_reason": reason,
        "kernel_path": trace.get("kernel_path", ""),
        "kernel_name": trace.get("kernel_name", ""),
        "tile": trace.get("tile", {}),
        "selected_config": trace.get("selected_config"),
        "weight_cache": trace.get("weight_cache", ""),
        "materialize_inputs": trace.get("materialize_inputs", False),
        "latency_us": latency_us,
        "layer_hits": trace.get("hit_count", 0),
        "layer_misses": trace.get("miss_count", 0),
        "fallback_reasons": trace.get("fallback_reasons", {}),
        "install_error": install_error,
    }
