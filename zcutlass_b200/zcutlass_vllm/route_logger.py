"""Per-forward JSONL route rows for the vLLM Linear layers zcutlass serves.

Same switches and row schema as the reference's route log
(python/zcutlass_vllm/route_logger.py in supercatking/zcutlass), which its
serving reports parse: ZCUTLASS_VLLM_LOG_ROUTES turns logging on,
ZCUTLASS_VLLM_ROUTE_LOG names the file, ZCUTLASS_VLLM_MODEL_ID and
ZCUTLASS_VLLM_ARCHITECTURE tag the rows. A row is assembled from the
`ROW_FIELDS` table: one (key, getter) per column, in the reference's key order.
"""

from __future__ import annotations

import json
import os
import time
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Callable, Optional

from ..routing import default_family, env_flag, env_list

# The reference's helper names, kept importable under them.
env_enabled = env_flag
csv_env = env_list
shape_family = default_family


def tensor_shape(value: Any) -> list[int]:
    shape = getattr(value, "shape", None)
    return [] if shape is None else [int(d) for d in shape]


def tensor_dtype(value: Any) -> str:
    dtype = getattr(value, "dtype", None)
    return "unknown" if dtype is None else str(dtype)


def first_tensor(value: Any) -> Any:
    """vLLM Linear forwards return (output, bias) tuples; the output is first."""
    return value[0] if isinstance(value, tuple) and value else value


class RouteLogger:
    """Appends one JSON object per line."""

    def __init__(self, path: str | os.PathLike[str]) -> None:
        self.path = Path(path)

    def write(self, row: dict[str, Any]) -> None:
        self.path.parent.mkdir(parents=True, exist_ok=True)
        with self.path.open("a", encoding="utf-8") as fh:
            fh.write(json.dumps(row, sort_keys=True, default=str) + "\n")


def make_route_logger() -> Optional[RouteLogger]:
    path = os.environ.get("ZCUTLASS_VLLM_ROUTE_LOG") if env_flag("ZCUTLASS_VLLM_LOG_ROUTES") else None
    return RouteLogger(path) if path else None


@dataclass
class _Forward:
    """Everything one row is read from."""

    layer: Any
    layer_class: str
    input_tensor: Any
    output: Any
    latency_us: float
    trace: dict
    install_error: Optional[str]

    def __post_init__(self) -> None:
        x = tensor_shape(self.input_tensor)
        w = tensor_shape(getattr(self.layer, "weight", None))
        # m = leading input dim, k = last input dim, n = weight rows ([N, K] weights)
        self.m, self.k = (int(x[0]), int(x[-1])) if len(x) >= 2 else (0, 0)
        self.n = int(w[0]) if len(w) >= 2 else 0
        self.in_shape, self.w_shape = x, w

    def t(self, key: str, default: Any = None) -> Any:
        return self.trace.get(key, default)


def _route(f: _Forward) -> str:
    return "zcutlass" if f.t("fallback_reason") is None and f.t("hit_count", 0) else "fallback"


# (row key, getter), in the reference's column order (route_logger.py:73-127).
ROW_FIELDS: tuple[tuple[str, Callable[[_Forward], Any]], ...] = (
    ("ts_ns", lambda f: time.time_ns()),
    ("pid", lambda f: os.getpid()),
    ("rank", lambda f: os.environ.get("RANK", "")),
    ("local_rank", lambda f: os.environ.get("LOCAL_RANK", "")),
    ("tp_rank", lambda f: getattr(f.layer, "tp_rank", "")),
    ("tp_size", lambda f: getattr(f.layer, "tp_size", "")),
    ("model_id", lambda f: os.environ.get("ZCUTLASS_VLLM_MODEL_ID", "")),
    ("architecture", lambda f: os.environ.get("ZCUTLASS_VLLM_ARCHITECTURE", "")),
    ("layer_prefix", lambda f: getattr(f.layer, "prefix", "")),
    ("layer_class", lambda f: f.layer_class),
    ("input_shape", lambda f: f.in_shape),
    ("weight_shape", lambda f: f.w_shape),
    ("output_shape", lambda f: tensor_shape(first_tensor(f.output))),
    ("dtype", lambda f: tensor_dtype(f.input_tensor)),
    ("bias", lambda f: getattr(f.layer, "bias", None) is not None),
    ("m", lambda f: f.m),
    ("n", lambda f: f.n),
    ("k", lambda f: f.k),
    ("shape_family", lambda f: default_family(f.m, f.n, f.k)),
    ("route", _route),
    ("fallback_reason", lambda f: f.t("fallback_reason")),
    ("kernel_path", lambda f: f.t("kernel_path", "")),
    ("kernel_name", lambda f: f.t("kernel_name", "")),
    ("tile", lambda f: f.t("tile", {})),
    ("selected_config", lambda f: f.t("selected_config")),
    ("weight_cache", lambda f: f.t("weight_cache", "")),
    ("materialize_inputs", lambda f: f.t("materialize_inputs", False)),
    ("latency_us", lambda f: f.latency_us),
    ("layer_hits", lambda f: f.t("hit_count", 0)),
    ("layer_misses", lambda f: f.t("miss_count", 0)),
    ("fallback_reasons", lambda f: f.t("fallback_reasons", {})),
    ("install_error", lambda f: f.install_error),
)


def build_route_row(*, layer: Any, layer_class: str, input_tensor: Any, output: Any, latency_us: float,
                    trace: Optional[dict[str, Any]], install_error: Optional[str] = None) -> dict[str, Any]:
    f = _Forward(layer, layer_class, input_tensor, output, latency_us, trace or {}, install_error)
    return {key: get(f) for key, get in ROW_FIELDS}
