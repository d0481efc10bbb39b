"""Opt-in PyTorch overlay: sends chosen GEMM / Linear call sites to zcutlass.

Public surface of the reference overlay (python/zcutlass_torch/overlay.py in
supercatking/zcutlass), kept so its users can switch packages: OverlayStats,
RoutingPolicy, ZCutlassGemmOverlay with gemm() / linear() and the last_*
telemetry attributes, selected_gemm_config, extension_available and the
module-level gemm / linear. A call either runs torch.ops.zcutlass_torch.gemm
(a hit) or the stock PyTorch expression, counted under the first reason of
the rule tables below (a miss). The overlay never hooks PyTorch globally.

B200 additions, both opt-in so default counters match the reference:
  * native_weight_layout=True: linear() routes a PyTorch [N, K] weight straight
    to the kernels as column-major B (torch.ops.zcutlass.linear) instead of
    requiring a pre-transposed copy;
  * if a CUDA device is present but the native extension cannot be loaded,
    the first routed call raises instead of falling back silently (on hosts
    without CUDA the `extension_unavailable` reason stands).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

from ..routing import Bucket, Rule, Tally, classify, first_reason


def _torch():
    import torch

    return torch


def _load_extension() -> bool:
    """True once torch.ops.zcutlass_torch is registered; False on hosts without
    CUDA; raises on a CUDA host where the native library does not load."""
    from zcutlass_b200 import torch_ops

    try:
        torch_ops.load()
    except Exception as exc:
        if _torch().cuda.is_available():
            raise RuntimeError(f"zcutlass native extension failed to load on a CUDA host: {exc}") from exc
        return False
    return True


def extension_available() -> bool:
    return _load_extension()


def selected_gemm_config(a, b, c=None, bias=None, alpha: float = 1.0, beta: float = 0.0):
    """Dispatch metadata for one GEMM call site (None without the extension)."""
    if not _load_extension():
        return None
    from zcutlass_b200 import torch_ops

    return dict(torch_ops.selected_gemm_config(a, b, c, bias, float(alpha), float(beta)))


class OverlayStats(Tally):
    """hits / misses / fallback_reasons / total / hit_rate of one overlay."""


@dataclass(frozen=True)
class RoutingPolicy:
    """Which GEMM shapes go to zcutlass without `force_zcutlass`.

    A shape belongs to the first family whose M range holds m, once n and k
    reach min_n / min_k: decode m <= decode_max_m, prefill
    prefill_min_m..prefill_max_m, large m >= large_min_m; anything else is
    `fallback` (reason shape_not_target_bucket). Only families named in
    `promoted_families` are routed (else family_not_promoted)."""

    enabled: bool = True
    min_n: int = 1024
    min_k: int = 1024
    decode_max_m: int = 16
    prefill_min_m: int = 32
    prefill_max_m: int = 256
    large_min_m: int = 512
    promoted_families: tuple[str, ...] = ()

    def buckets(self) -> tuple[Bucket, ...]:
        return (Bucket("decode", 0, self.decode_max_m), Bucket("prefill", self.prefill_min_m, self.prefill_max_m),
                Bucket("large", self.large_min_m, float("inf")))

    def family(self, m: int, n: int, k: int) -> str:
        return classify(m, n, k, self.buckets(), self.min_n, self.min_k)

    def reject_reason(self, m: int, n: int, k: int) -> Optional[str]:
        if not self.enabled:
            return None
        fam = self.family(m, n, k)
        return first_reason(_POLICY_RULES, (fam, self.promoted_families))


# (family, promoted families) -> reason; python/zcutlass_torch/overlay.py:84-92.
_POLICY_RULES = (
    Rule("shape_not_target_bucket", lambda s: s[0] == "fallback"),
    Rule("family_not_promoted", lambda s: s[0] not in s[1]),
)


@dataclass
class _Call:
    """One GEMM call as the rule tables see it. `b` is [K, N], or a PyTorch
    [N, K] weight when b_is_nk."""

    a: object
    b: object
    c: object = None
    bias: object = None
    beta: float = 0.0
    b_is_nk: bool = False

    @property
    def m(self) -> int:
        return int(self.a.shape[0])

    @property
    def k(self) -> int:
        return int(self.a.shape[1])

    @property
    def b_k(self) -> int:
        return int(self.b.shape[1 if self.b_is_nk else 0])

    @property
    def n(self) -> int:
        return int(self.b.shape[0 if self.b_is_nk else 1])


def _half_types():
    torch = _torch()
    return (torch.float16, torch.bfloat16)


# Checks up to the point where (m, n, k) is known -- the family is recorded
# after them -- then operand layout and types, in the reference's order
# (python/zcutlass_torch/overlay.py:159-191). C checks apply only when C is
# given, bias checks only when a bias is given.
_SHAPE_RULES = (
    Rule("beta_without_c", lambda q: q.c is None and q.beta != 0.0),
    Rule("cpu_tensor", lambda q: not (q.a.is_cuda and q.b.is_cuda)),
    Rule("rank_not_2", lambda q: q.a.dim() != 2 or q.b.dim() != 2),
    Rule("inner_dimension_mismatch", lambda q: q.k != q.b_k),
)
_OPERAND_RULES = (
    Rule("non_contiguous_ab", lambda q: not (q.a.is_contiguous() and q.b.is_contiguous())),
    Rule("mixed_dtype", lambda q: q.a.dtype != q.b.dtype),
    Rule("unsupported_dtype", lambda q: q.a.dtype not in _half_types()),
    Rule("cpu_c_tensor", lambda q: q.c is not None and not q.c.is_cuda),
    Rule("c_shape_mismatch", lambda q: q.c is not None and tuple(q.c.shape) != (q.m, q.n)),
    Rule("c_dtype_mismatch", lambda q: q.c is not None and q.c.dtype != q.a.dtype),
    Rule("non_contiguous_c", lambda q: q.c is not None and not q.c.is_contiguous()),
    Rule("cpu_bias_tensor", lambda q: q.bias is not None and not q.bias.is_cuda),
    Rule("bias_shape_mismatch", lambda q: q.bias is not None and (q.bias.dim() != 1 or q.bias.shape[0] != q.n)),
    Rule("bias_dtype_mismatch", lambda q: q.bias is not None and q.bias.dtype != q.a.dtype),
    Rule("non_contiguous_bias", lambda q: q.bias is not None and not q.bias.is_contiguous()),
)
# Gates on the overlay itself, tried first (overlay.py:155-158).
_GATE_RULES = (
    Rule("zcutlass_disabled", lambda ov: not ov.enable_zcutlass),
    Rule("extension_unavailable", lambda ov: not ov._ensure_loaded()),
)


@dataclass(frozen=True)
class Route:
    """Where the last call went: the overlay's last_* attributes."""

    family: str = "unknown"
    kernel_path: str = "unknown"
    kernel_name: str = "unknown"
    tile: dict = field(default_factory=lambda: {"m": 0, "n": 0, "k": 0})
    config: Optional[dict] = None
    fallback_reason: Optional[str] = None

    @classmethod
    def fallback(cls, family: str, reason: str, path: str = "pytorch_fallback") -> "Route":
        return cls(family=family, kernel_path=path, kernel_name=path, fallback_reason=reason)

    @classmethod
    def hit(cls, family: str, config: Optional[dict], kernel_name: str = "unknown") -> "Route":
        if config is None:
            return cls(family=family, kernel_path="zcutlass", kernel_name=kernel_name)
        return cls(family=str(config.get("shape_family", family)), kernel_path=str(config.get("kernel_path", "zcutlass")),
                   kernel_name=str(config.get("kernel_name", "unknown")),
                   tile=dict(config.get("tile", {"m": 0, "n": 0, "k": 0})), config=config)


def _stock_gemm(a, b, c, bias, alpha: float, beta: float):
    """What an un-routed call computes: the reference's fallback expression,
    term by term in its order (python/zcutlass_torch/overlay.py:130-145)."""
    out = _torch().matmul(a, b)
    if alpha != 1.0:
        out = out * alpha
    if c is not None and beta != 0.0:
        out = out + c * beta
    if bias is not None:
        out = out + bias
    return out


class ZCutlassGemmOverlay:
    """Explicit, per-call-site GEMM overlay; never hooks PyTorch globally."""

    def __init__(self, enable_zcutlass: bool = True, *, routing_policy: Optional[RoutingPolicy] = None,
                 force_zcutlass: bool = False, native_weight_layout: bool = False) -> None:
        self.enable_zcutlass = enable_zcutlass
        self.routing_policy = routing_policy or RoutingPolicy()
        self.force_zcutlass = force_zcutlass
        self.native_weight_layout = native_weight_layout
        self.stats = OverlayStats()
        self.route = Route()
        self._loaded = False

    # last_* telemetry, as the reference's users read it
    last_family = property(lambda self: self.route.family)
    last_kernel_path = property(lambda self: self.route.kernel_path)
    last_kernel_name = property(lambda self: self.route.kernel_name)
    last_tile = property(lambda self: self.route.tile)
    last_config = property(lambda self: self.route.config)
    last_fallback_reason = property(lambda self: self.route.fallback_reason)

    def _ensure_loaded(self) -> bool:
        if self.enable_zcutlass and not self._loaded:
            self._loaded = _load_extension()
        return self.enable_zcutlass and self._loaded

    def decide(self, call: _Call) -> tuple[Optional[str], str]:
        """(first reason this call cannot run on zcutlass or None, its family).
        The family is known once the shape checks pass, "unknown" before."""
        reason = first_reason(_GATE_RULES, self) or first_reason(_SHAPE_RULES, call)
        if reason is not None:
            return reason, "unknown"
        family = self.routing_policy.family(call.m, call.n, call.k)
        reason = first_reason(_OPERAND_RULES, call)
        if reason is None and not self.force_zcutlass:
            reason = self.routing_policy.reject_reason(call.m, call.n, call.k)
        return reason, family

    def miss(self, reason: str, family: str = "unknown", path: str = "pytorch_fallback") -> None:
        self.stats.record_miss(reason)
        self.route = Route.fallback(family, reason, path)

    def hit(self, family: str, config: Optional[dict], kernel_name: str = "unknown") -> None:
        self.stats.record_hit()
        self.route = Route.hit(family, config, kernel_name)

    def gemm(self, a, b, c=None, bias=None, alpha: float = 1.0, beta: float = 0.0):
        reason, family = self.decide(_Call(a, b, c, bias, beta))
        if reason is not None:
            self.miss(reason, family)
            return _stock_gemm(a, b, c, bias, alpha, beta)
        self.hit(family, selected_gemm_config(a, b, c, bias, alpha, beta))
        return _torch().ops.zcutlass_torch.gemm(a, b, c, bias, float(alpha), float(beta))

    def linear(self, x, weight, bias=None, *, weight_is_transposed: bool = False):
        """Linear call site. `weight` is [N, K] (PyTorch layout) unless
        weight_is_transposed=True, in which case it is a contiguous [K, N]."""
        torch = _torch()
        if weight_is_transposed:
            return self.gemm(x, weight, None, bias, 1.0, 0.0)
        if not self.native_weight_layout:
            # the reference counts this miss without touching last_* telemetry
            self.stats.record_miss("weight_not_pretransposed")
            return torch.nn.functional.linear(x, weight, bias)
        reason, family = self.decide(_Call(x, weight, None, bias, 0.0, b_is_nk=True))
        if reason is not None:
            self.miss(reason, family)
            return torch.nn.functional.linear(x, weight, bias)
        self.hit(family, None, "zcutlass_linear_native_weight")
        return torch.ops.zcutlass.linear(x, weight, bias)


_DEFAULT_OVERLAY = ZCutlassGemmOverlay()


def gemm(a, b, c=None, bias=None, alpha: float = 1.0, beta: float = 0.0):
    return _DEFAULT_OVERLAY.gemm(a, b, c, bias, alpha, beta)


def linear(x, weight, bias=None, *, weight_is_transposed: bool = False):
    return _DEFAULT_OVERLAY.linear(x, weight, bias, weight_is_transposed=weight_is_transposed)


__all__ = ["OverlayStats", "Route", "RoutingPolicy", "ZCutlassGemmOverlay", "extension_available", "gemm", "linear",
           "selected_gemm_config"]
