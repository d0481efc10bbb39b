"""Drop-in for the reference's `zcutlass_vllm` package (public names of
python/zcutlass_vllm/__init__.py in supercatking/zcutlass, minus the toy model)."""

from .linear import ZCutlassVllmLinearAdapter, make_linear_adapter
from .linear_method import (
    ZCutlassUnquantizedLinearMethod,
    clear_zcutlass_weight_cache,
    install_zcutlass_unquantized_linear_method,
)
from .oot_linear import register_oot_linear_layers
from .plugin import is_registered, register

__all__ = [
    "ZCutlassUnquantizedLinearMethod",
    "ZCutlassVllmLinearAdapter",
    "clear_zcutlass_weight_cache",
    "install_zcutlass_unquantized_linear_method",
    "make_linear_adapter",
    "register_oot_linear_layers",
    "is_registered",
    "register",
]
