"""The Linear-call adapter that the vLLM integration routes through.

Public surface of the reference's adapter (python/zcutlass_vllm/linear.py in
supercatking/zcutlass): ZCutlassVllmLinearAdapter with run() / __call__,
its cumulative VllmLinearStats (calls, hits, misses, fallback_reasons,
hit_rate), the per-call `last_trace` dict with the reference's keys, and
make_linear_adapter. With a `fallback_fn` (vLLM's own GEMM) a call whose
shape alone decides a miss delegates before the extension is touched; the
reasons and their order are the `FAST_RULES` table. ZCUTLASS_VLLM_TRACE_CONFIG=0
skips the selected-config query on hits (kernel_name "zcutlass_untraced").

B200 addition: run_native() takes the weight in its stored [N, K] layout and
runs it as column-major B, without a transposed copy.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable, Optional

from ..routing import Rule, Tally, env_flag, first_reason
from ..zcutlass_torch import RoutingPolicy, ZCutlassGemmOverlay, selected_gemm_config
from ..zcutlass_torch.overlay import _Call


class VllmLinearStats(Tally):
    """Cumulative over every call of one adapter; `calls` counts calls."""

    def __init__(self) -> None:
        super().__init__()
        self.calls = 0

    def update_from_overlay(self, overlay: ZCutlassGemmOverlay) -> None:
        self.calls += 1
        self.absorb(overlay.stats)


@dataclass(frozen=True)
class LinearShape:
    """The shapes of one Linear call: x [m, k] and a weight that is [wk, n]
    (pre-transposed) or [n, wk] (vLLM's stored layout)."""

    ranks_ok: bool
    m: int = 0
    k: int = 0
    n: int = 0
    wk: int = 0
    family: str = "unknown"
    promoted: tuple[str, ...] = ()
    transposed: bool = True

    @classmethod
    def of(cls, x, weight, policy: RoutingPolicy, *, weight_nk: bool, transposed: bool = True) -> "LinearShape":
        xs, ws = getattr(x, "shape", None), getattr(weight, "shape", None)
        if xs is None or ws is None or len(xs) != 2 or len(ws) != 2:
            return cls(False, promoted=policy.promoted_families, transposed=transposed)
        n, wk = (int(ws[0]), int(ws[1])) if weight_nk else (int(ws[1]), int(ws[0]))
        m, k = int(xs[0]), int(xs[1])
        return cls(True, m, k, n, wk, policy.family(m, n, k), policy.promoted_families, transposed)


# Misses decided from shapes alone, in the reference's order
# (python/zcutlass_vllm/linear.py:86-121 and linear_method.py:61-83).
SHAPE_RULES = (
    Rule("rank_not_2", lambda s: not s.ranks_ok),
    Rule("inner_dimension_mismatch", lambda s: s.k != s.wk),
    Rule("shape_not_target_bucket", lambda s: s.family == "fallback"),
    Rule("family_not_promoted", lambda s: s.family not in s.promoted),
)
FAST_RULES = (Rule("weight_not_pretransposed", lambda s: not s.transposed),) + SHAPE_RULES
# The reason strings above that are reported before the family is known.
_FAMILY_UNKNOWN = frozenset({"weight_not_pretransposed", "rank_not_2", "inner_dimension_mismatch"})


def fast_reason(rules, shape: LinearShape) -> Optional[tuple[str, str]]:
    """(reason, family) of the first rule that holds, or None."""
    reason = first_reason(rules, shape)
    if reason is None:
        return None
    return reason, "unknown" if reason in _FAMILY_UNKNOWN else shape.family


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

    # ------------------------------------------------------------ traces

    def _settings(self) -> dict:
        return {"promoted_families": self.promoted_families, "force_zcutlass": self.force_zcutlass,
                "materialize_inputs": self.materialize_inputs}

    def _close(self, overlay: ZCutlassGemmOverlay) -> None:
        """Folds one call's overlay into the cumulative stats and the trace."""
        self.stats.update_from_overlay(overlay)
        r = overlay.route
        self.last_trace = {
            "family": r.family, "kernel_path": r.kernel_path, "kernel_name": r.kernel_name, "tile": r.tile,
            "selected_config": r.config, "fallback_reason": r.fallback_reason, "hit_count": overlay.stats.hits,
            "miss_count": overlay.stats.misses, "fallback_reasons": overlay.stats.fallback_reasons,
            **self._settings(),
        }

    def record_delegation(self, reason: str, family: str, path: str) -> None:
        """A miss decided before any overlay ran (shapes or policy)."""
        overlay = self._overlay()
        overlay.miss(reason, family, path)
        self._close(overlay)

    # ------------------------------------------------------------ calls

    def _overlay(self) -> ZCutlassGemmOverlay:
        return ZCutlassGemmOverlay(routing_policy=self.routing_policy, force_zcutlass=self.force_zcutlass)

    def _prepare(self, x):
        if self.materialize_inputs and hasattr(x, "is_contiguous") and not x.is_contiguous():
            return x.contiguous()
        return x

    def __call__(self, x, weight, bias=None, *, weight_is_transposed: bool = False):
        return self.run(x, weight, bias, weight_is_transposed=weight_is_transposed)

    def run(self, x, weight, bias=None, *, weight_is_transposed: bool = False,
            fallback_fn: Optional[Callable[[], Any]] = None, fallback_path_name: str = "framework_fallback"):
        """One Linear call. `weight` is [K, N] when weight_is_transposed, else
        [N, K]. Without `fallback_fn` misses run the overlay's PyTorch path;
        with it, they delegate to it (vLLM's own GEMM)."""
        x = self._prepare(x)
        if fallback_fn is None:
            overlay = self._overlay()
            out = overlay.linear(x, weight, bias, weight_is_transposed=weight_is_transposed)
            self._close(overlay)
            return out
        if not self.force_zcutlass:
            shape = LinearShape.of(x, weight, self.routing_policy, weight_nk=False, transposed=weight_is_transposed)
            fast = fast_reason(FAST_RULES, shape)
            if fast is not None:
                self.record_delegation(fast[0], fast[1], fallback_path_name)
                return fallback_fn()
        overlay = self._overlay()
        if not weight_is_transposed:
            overlay.miss("weight_not_pretransposed", "unknown", fallback_path_name)
            out = fallback_fn()
        else:
            reason, family = overlay.decide(_Call(x, weight, None, bias, 0.0))
            if reason is not None:
                overlay.miss(reason, family, fallback_path_name)
                out = fallback_fn()
            else:
                out = self._hit(overlay, family, x, weight, bias)
        self._close(overlay)
        return out

    def _hit(self, overlay: ZCutlassGemmOverlay, family: str, x, weight, bias):
        import torch

        traced = env_flag("ZCUTLASS_VLLM_TRACE_CONFIG", True)
        config = selected_gemm_config(x, weight, None, bias, 1.0, 0.0) if traced else None
        overlay.hit(family, config, "zcutlass_untraced")  # the name only shows without a config
        return torch.ops.zcutlass_torch.gemm(x, weight, None, bias, 1.0, 0.0)

    def run_native(self, x, weight, bias=None, *, fallback_fn: Callable[[], Any],
                   fallback_path_name: str = "framework_fallback"):
        """One Linear call with the weight in its stored [N, K] layout, run as
        column-major B (no transposed copy)."""
        import torch

        x = self._prepare(x)
        overlay = self._overlay()
        reason, family = overlay.decide(_Call(x, weight, None, bias, 0.0, b_is_nk=True))
        if reason is not None:
            overlay.miss(reason, family, fallback_path_name)
            out = fallback_fn()
        else:
            overlay.hit(family, None, "zcutlass_linear_native_weight")
            out = torch.ops.zcutlass.linear(x, weight, bias)
        self._close(overlay)
        return out


def make_linear_adapter(**kwargs: Any) -> ZCutlassVllmLinearAdapter:
    return ZCutlassVllmLinearAdapter(**kwargs)
