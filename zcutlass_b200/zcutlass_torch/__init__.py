"""Drop-in for the reference's `zcutlass_torch` package (same public names as
python/zcutlass_torch/__init__.py:1-19 in supercatking/zcutlass)."""

from .overlay import (
    OverlayStats,
    RoutingPolicy,
    ZCutlassGemmOverlay,
    extension_available,
    gemm,
    linear,
    selected_gemm_config,
)

__all__ = [
    "OverlayStats",
    "RoutingPolicy",
    "ZCutlassGemmOverlay",
    "extension_available",
    "gemm",
    "linear",
    "selected_gemm_config",
]
