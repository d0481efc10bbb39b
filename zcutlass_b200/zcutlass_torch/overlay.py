"""Opt-in PyTorch overlay for the zcutlass GEMM.

Interface and routing contract mirror the reference overlay
(python/zcutlass_torch/overlay.py in supercatking/zcutlass):

  OverlayStats         hits / misses / fallback_reasons / total / hit_rate   (35-54)
  RoutingPolicy        decode / prefill / large / fallback buckets and the
                       shape_not_target_bucket / family_not_promoted reasons (57-92)
  ZCutlassGemmOverlay  gemm(): reject reasons checked in the same order with
                       the same strings (147-196); rejected calls run the
                       stock PyTorch expression (130-145) and are counted;
                       accepted calls run torch.ops.zcutlass_torch.gemm (198-216)
                       linear(): F.linear unless the weight is pre-transposed (218-231)

B200 additions, both opt-in so default counters match the reference:
  * native_weight_layout=True: linear() routes a PyTorch [N, K] weight straight
    to the kernels as column-major B (torch.ops.zcutlass.linear) instead of
    requiring a pre-transposed copy;
  * if a CUDA device is present but the native extension cannot be loaded,
    construction of the first route raises instead of silently falling back
    (on hosts without CUDA the reference's `extension_unavailable` reason stands).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, Optional


def _torch():
    import torch

    return torch


def _load_extension() -> bool:
    from zcutlass_b200 import torch_ops

    try:
        torch_ops.load()
    except Exception as exc:
        torch = _torch()
        if torch.cuda.is_available():
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


@dataclass
class OverlayStats:
    hits: int = 0
    misses: int = 0
    fallback_reasons: Dict[str, int] = field(default_factory=dict)

    def record_hit(self) -> None:
        self.hits += 1

    def record_miss(self, reason: str) -> None:
        self.misses += 1
        self.fallback_reasons[reason] = self.fallback_reasons.get(reason, 0) + 1

    @property
    def total(self) -> int:
        return self.hits + self.misses

    @property
    def hit_rate(self) -> float:
        return self.hits / self.total if self.total else 0.0


@dataclass(frozen=True)
class RoutingPolicy:
    """Shape policy: which GEMM shapes an overlay sends to zcutlass.

    Families (same thresholds as the reference): decode m <= 16, prefill
    32 <= m <= 256, large m >= 512, each with n, k >= 1024; everything else is
    `fallback`. Only families listed in `promoted_families` are routed unless
    the overlay is forced."""

    enabled: bool = True
    min_n: int = 1024
    min_k: int = 1024
    decode_max_m: int = 16
    prefill_min_m: int = 32
    prefill_max_m: int = 256
    large_min_m: int = 512
    promoted_families: tuple[str, ...] = ()

    def family(self, m: int, n: int, k: int) -> str:
        if n < self.min_n or k < self.min_k:
            return "fallback"
        if m <= self.decode_max_m:
            return "decode"
        if self.prefill_min_m <= m <= self.prefill_max_m:
            return "prefill"
        if m >= self.large_min_m:
            return "large"
        return "fallback"

    def reject_reason(self, m: int, n: int, k: int) -> Optional[str]:
        if not self.enabled:
            return None
        fam = self.family(m, n, k)
        if fam == "fallback":
            return "shape_not_target_bucket"
        if fam not in self.promoted_families:
            return "family_not_promoted"
        return None


_NO_TILE = {"m": 0, "n": 0, "k": 0}


class ZCutlassGemmOverlay:
    """Explicit, per-call-site GEMM overlay; never hooks PyTorch globally."""

    def __init__(self, enable_zcutlass: bool = True, *, routing_policy: Optional[RoutingPolicy] = None,
                 force_zcutlass: bool = False, native_weight_layout: bool = False) -> None:
        self.enable_zcutlass = enable_zcutlass
        self.routing_policy = routing_policy or RoutingPolicy()
        self.force_zcutlass = force_zcutlass
        self.native_weight_layout = native_weight_layout
        self.stats = OverlayStats()
        self._loaded = False
        self.last_family = "unknown"
        self.last_kernel_path = "unknown"
        self.last_kernel_name = "unknown"
        self.last_tile = dict(_NO_TILE)
        self.last_config: Optional[dict] = None
        self.last_fallback_reason: Optional[str] = None

    def _ensure_loaded(self) -> bool:
        if not self.enable_zcutlass:
            return False
        if not self._loaded:
            self._loaded = _load_extension()
        return self._loaded

    def _clear_last(self) -> None:
        self.last_family = "unknown"
        self.last_kernel_path = "unknown"
        self.last_kernel_name = "unknown"
        self.last_tile = dict(_NO_TILE)
        self.last_config = None
        self.last_fallback_reason = None

    def _fallback(self, reason: str, a, b, c=None, bias=None, alpha: float = 1.0, beta: float = 0.0):
        torch = _torch()
        self.stats.record_miss(reason)
        self.last_kernel_path = "pytorch_fallback"
        self.last_kernel_name = "pytorch_fallback"
        self.last_tile = dict(_NO_TILE)
        self.last_config = None
        self.last_fallback_reason = reason
        out = torch.matmul(a, b)
        if alpha != 1.0:
            out = out * alpha
        if c is not None and beta != 0.0:
            out = out + c * beta
        if bias is not None:
            out = out + bias
        return out

    def _reject_reason(self, a, b, c=None, bias=None, beta: float = 0.0, *, b_is_nk: bool = False) -> Optional[str]:
        """First reason (in the reference's order) this call cannot run on
        zcutlass, or None. b is [K, N], or a PyTorch [N, K] weight when b_is_nk."""
        torch = _torch()
        self._clear_last()
        if not self.enable_zcutlass:
            return "zcutlass_disabled"
        if not self._ensure_loaded():
            return "extension_unavailable"
        if c is None and beta != 0.0:
            return "beta_without_c"
        if not a.is_cuda or not b.is_cuda:
            return "cpu_tensor"
        if a.dim() != 2 or b.dim() != 2:
            return "rank_not_2"
        if a.shape[1] != b.shape[1 if b_is_nk else 0]:
            return "inner_dimension_mismatch"
        m, k, n = int(a.shape[0]), int(a.shape[1]), int(b.shape[0 if b_is_nk else 1])
        self.last_family = self.routing_policy.family(m, n, k)
        if not a.is_contiguous() or not b.is_contiguous():
            return "non_contiguous_ab"
        if a.dtype != b.dtype:
            return "mixed_dtype"
        if a.dtype not in (torch.float16, torch.bfloat16):
            return "unsupported_dtype"
        if c is not None:
            if not c.is_cuda:
                return "cpu_c_tensor"
            if tuple(c.shape) != (m, n):
                return "c_shape_mismatch"
            if c.dtype != a.dtype:
                return "c_dtype_mismatch"
            if not c.is_contiguous():
                return "non_contiguous_c"
        if bias is not None:
            if not bias.is_cuda:
                return "cpu_bias_tensor"
            if bias.dim() != 1 or bias.shape[0] != n:
                return "bias_shape_mismatch"
            if bias.dtype != a.dtype:
                return "bias_dtype_mismatch"
            if not bias.is_contiguous():
                return "non_contiguous_bias"
        if not self.force_zcutlass:
            return self.routing_policy.reject_reason(m, n, k)
        return None

    def _record_hit(self, config: Optional[dict]) -> None:
        self.stats.record_hit()
        self.last_config = config
        if config is not None:
            self.last_family = str(config.get("shape_family", self.last_family))
            self.last_kernel_path = str(config.get("kernel_path", "zcutlass"))
            self.last_kernel_name = str(config.get("kernel_name", "unknown"))
            self.last_tile = dict(config.get("tile", _NO_TILE))
        else:
            self.last_kernel_path = "zcutlass"
            self.last_kernel_name = "unknown"
            self.last_tile = dict(_NO_TILE)
        self.last_fallback_reason = None

    def gemm(self, a, b, c=None, bias=None, alpha: float = 1.0, beta: float = 0.0):
        reason = self._reject_reason(a, b, c, bias, beta)
        if reason is not None:
            return self._fallback(reason, a, b, c, bias, alpha, beta)
        torch = _torch()
        self._record_hit(selected_gemm_config(a, b, c, bias, alpha, beta))
        return torch.ops.zcutlass_torch.gemm(a, b, c, bias, float(alpha), float(beta))

    def linear(self, x, weight, bias=None, *, weight_is_transposed: bool = False):
        """Linear call site. `weight` is [N, K] (PyTorch layout) unless
        weight_is_transposed=True, in which case it is a contiguous [K, N]."""
        torch = _torch()
        if weight_is_transposed:
            return self.gemm(x, weight, None, bias, 1.0, 0.0)
        if not self.native_weight_layout:
            self.stats.record_miss("weight_not_pretransposed")
            return torch.nn.functional.linear(x, weight, bias)
        # Native [N, K] weight: the same checks as gemm(), on the weight as stored.
        reason = self._reject_reason(x, weight, None, bias, 0.0, b_is_nk=True)
        if reason is not None:
            self.stats.record_miss(reason)
            self.last_kernel_path = "pytorch_fallback"
            self.last_kernel_name = "pytorch_fallback"
            self.last_fallback_reason = reason
            return torch.nn.functional.linear(x, weight, bias)
        self._record_hit(None)
        self.last_kernel_path = "zcutlass"
        self.last_kernel_name = "zcutlass_linear_native_weight"
        return torch.ops.zcutlass.linear(x, weight, bias)


_DEFAULT_OVERLAY = ZCutlassGemmOverlay()


def gemm(a, b, c=None, bias=None, alpha: float = 1.0, beta: float = 0.0):
    return _DEFAULT_OVERLAY.gemm(a, b, c, bias, alpha, beta)


def linear(x, weight, bias=None, *, weight_is_transposed: bool = False):
    return _DEFAULT_OVERLAY.linear(x, weight, bias, weight_is_transposed=weight_is_transposed)
