"""Import path of the reference's `zcutlass_torch.overlay` module."""

from zcutlass_b200.zcutlass_torch.overlay import *  # noqa: F401,F403
from zcutlass_b200.zcutlass_torch.overlay import (  # noqa: F401
    OverlayStats,
    RoutingPolicy,
    ZCutlassGemmOverlay,
    _load_extension,
    extension_available,
    gemm,
    linear,
    selected_gemm_config,
)
