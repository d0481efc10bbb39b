"""Linear-call adapter that vLLM integrations route through.

Mirrors ZCutlassVllmLinearAdapter (python/zcutlass_vllm/linear.py in
supercatking/zcutlass): VllmLinearStats (24-41), the fast-delegate reasons
checked before touching the extension (86-121), delegation to a framework
fallback for misses, per-call trace dicts, and ZCUTLASS_VLLM_TRACE_CONFIG
(141-242). Reason strings and trace keys are the reference's.
"""

from __future__ import annotations

import os
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, Optional

from ..zcutlass_torch import RoutingPolicy, ZCutlassGemmOverlay, selected_gemm_config


def _env_enabled(name: str, default: bool = True) -> bool:
    value = os.environ.get(name)
    if value is None:
        return default
    return value not in ("", "0", "false", "False", "FALSE", "no", "No", "NO")


@dataclass
class VllmLinearStats:
    calls: int = 0
    hits: int = 0
    misses: int = 0
    fallback_reasons: Dict[str, int] = field(default_factory=dict)

    def update_from_overlay(self, overlay: ZCutlassGemmOverlay) -> None:
        self.calls += 1
        self.hits += overlay.stats.hits
        self.misses += overlay.stats.misses
        for reason, count in overlay.stats.fallback_reasons.items():
            self.fallback_reasons[reason] = self.fallback_reasons.get(reason, 0) + count

    @property
    def hit_rate(self) -> float:
        total = self.hits + self.misses
        return self.hits / total if total else 0.0


_NO_TILE = {"m": 0, "n": 0, "k": 0}


class ZCutlassVllmLinearAdapter:
    """Routes one Linear call to zcutlass or to a framework fallback."""

    def __init__(self, *, promoted_families: tuple[str, ...] = (), force_zcutlass: bool = False,
                 materialize_inputs: bool = False) -> None:
        self.promoted_families = promoted_families
        self.force_zcutlass = force_zcutlass
        self.materialize_inputs = materialize_inputs
        self.routing_policy = RoutingPolicy(promoted_families=promoted_families)
        self.stats = VllmLinearStats()
        self.last_trace: Optional[dict[str, Any]] = None

    def _trace(self, overlay_like: dict) -> dict:
        overlay_like.update(promoted_families=self.promoted_families, force_zcutlass=self.force_zcutlass,
                            materialize_inputs=self.materialize_inputs)
        return overlay_like

    def _record_fallback_trace(self, *, reason: str, family: str = "unknown", fallback_path_name: str) -> None:
        self.stats.calls += 1
        self.stats.misses += 1
        self.stats.fallback_reasons[reason] = self.stats.fallback_reasons.get(reason, 0) + 1
        self.last_trace = self._trace({
            "family": family, "kernel_path": fallback_path_name, "kernel_name": fallback_path_name,
            "tile": dict(_NO_TILE), "selected_config": None, "fallback_reason": reason, "hit_count": 0,
            "miss_count": 1, "fallback_reasons": {reason: 1},
        })

    def _fast_delegate_reason(self, x, weight, bias, *, weight_is_transposed: bool) -> tuple[str, str] | None:
        """A miss decided from shapes alone, before any extension/config query."""
        if self.force_zcutlass:
            return None
        if not weight_is_transposed:
            return ("weight_not_pretransposed", "unknown")
        xs, ws = getattr(x, "shape", None), getattr(weight, "shape", None)
        if xs is None or ws is None or len(xs) != 2 or len(ws) != 2:
            return ("rank_not_2", "unknown")
        m, k = int(xs[0]), int(xs[1])
        if k != int(ws[0]):
            return ("inner_dimension_mismatch", "unknown")
        family = self.routing_policy.family(m, int(ws[1]), k)
        if family == "fallback":
            return ("shape_not_target_bucket", family)
        if family not in self.promoted_families:
            return ("family_not_promoted", family)
        return None

    def __call__(self, x, weight, bias=None, *, weight_is_transposed: bool = False):
        return self.run(x, weight, bias, weight_is_transposed=weight_is_transposed)

    def run(self, x, weight, bias=None, *, weight_is_transposed: bool = False,
            fallback_fn: Optional[Callable[[], Any]] = None, fallback_path_name: str = "framework_fallback"):
        """One Linear call. With `fallback_fn`, misses delegate to it (vLLM's own
        GEMM) instead of the overlay's PyTorch expression."""
        if self.materialize_inputs and hasattr(x, "is_contiguous") and not x.is_contiguous():
            x = x.contiguous()
        if fallback_fn is not None:
            fast = self._fast_delegate_reason(x, weight, bias, weight_is_transposed=weight_is_transposed)
            if fast is not None:
                reason, family = fast
                self._record_fallback_trace(reason=reason, family=family, fallback_path_name=fallback_path_name)
                return fallback_fn()
        overlay = ZCutlassGemmOverlay(routing_policy=self.routing_policy, force_zcutlass=self.force_zcutlass)
        if fallback_fn is None:
            out = overlay.linear(x, weight, bias, weight_is_transposed=weight_is_transposed)
        elif not weight_is_transposed:
            overlay.stats.record_miss("weight_not_pretransposed")
            self._mark_fallback(overlay, "weight_not_pretransposed", fallback_path_name)
            overlay.last_family = "unknown"
            out = fallback_fn()
        else:
            reason = overlay._reject_reason(x, weight, None, bias, 0.0)
            if reason is not None:
                overlay.stats.record_miss(reason)
                self._mark_fallback(overlay, reason, fallback_path_name)
                out = fallback_fn()
            else:
                config = (selected_gemm_config(x, weight, None, bias, 1.0, 0.0)
                          if _env_enabled("ZCUTLASS_VLLM_TRACE_CONFIG", True) else None)
                overlay._record_hit(config)
                if config is None:
                    overlay.last_family = self.routing_policy.family(int(x.shape[0]), int(weight.shape[1]),
                                                                     int(x.shape[1]))
                    overlay.last_kernel_name = "zcutlass_untraced"
                import torch

                out = torch.ops.zcutlass_torch.gemm(x, weight, None, bias, 1.0, 0.0)
        self.stats.update_from_overlay(overlay)
        self.last_trace = self._trace({
            "family": overlay.last_family, "kernel_path": overlay.last_kernel_path,
            "kernel_name": overlay.last_kernel_name, "tile": overlay.last_tile,
            "selected_config": overlay.last_config, "fallback_reason": overlay.last_fallback_reason,
            "hit_count": overlay.stats.hits, "miss_count": overlay.stats.misses,
            "fallback_reasons": dict(overlay.stats.fallback_reasons),
        })
        return out

    def run_native(self, x, weight, bias=None, *, fallback_fn: Callable[[], Any],
                   fallback_path_name: str = "framework_fallback"):
        """One Linear call with the weight in its stored [N, K] layout, consumed
        by the kernels as column-major B (no transposed copy)."""
        if self.materialize_inputs and hasattr(x, "is_contiguous") and not x.is_contiguous():
            x = x.contiguous()
        overlay = ZCutlassGemmOverlay(routing_policy=self.routing_policy, force_zcutlass=self.force_zcutlass)
        reason = overlay._reject_reason(x, weight, None, bias, 0.0, b_is_nk=True)
        if reason is not None:
            overlay.stats.record_miss(reason)
            self._mark_fallback(overlay, reason, fallback_path_name)
            out = fallback_fn()
        else:
            import torch

            overlay._record_hit(None)
            overlay.last_kernel_path = "zcutlass"
            overlay.last_kernel_name = "zcutlass_linear_native_weight"
            out = torch.ops.zcutlass.linear(x, weight, bias)
        self.stats.update_from_overlay(overlay)
        self.last_trace = self._trace({
            "family": overlay.last_family, "kernel_path": overlay.last_kernel_path,
            "kernel_name": overlay.last_kernel_name, "tile": overlay.last_tile,
            "selected_config": overlay.last_config, "fallback_reason": overlay.last_fallback_reason,
            "hit_count": overlay.stats.hits, "miss_count": overlay.stats.misses,
            "fallback_reasons": dict(overlay.stats.fallback_reasons),
        })
        return out

    @staticmethod
    def _mark_fallback(overlay: ZCutlassGemmOverlay, reason: str, path_name: str) -> None:
        overlay.last_kernel_path = path_name
        overlay.last_kernel_name = path_name
        overlay.last_tile = dict(_NO_TILE)
        overlay.last_config = None
        overlay.last_fallback_reason = reason


def make_linear_adapter(**kwargs: Any) -> ZCutlassVllmLinearAdapter:
    return ZCutlassVllmLinearAdapter(**kwargs)
