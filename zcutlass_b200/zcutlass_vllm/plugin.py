"""vLLM general-plugin entry point (`vllm.general_plugins: zcutlass_overlay`).

register() runs once per process (vLLM may call it repeatedly): it probes the
native extension, registers the OOT Linear classes when ZCUTLASS_VLLM_ENABLE
is on, and publishes what it found as PluginState and as the environment
variables the reference's serving tools read (python/zcutlass_vllm/plugin.py
in supercatking/zcutlass): ZCUTLASS_VLLM_PLUGIN_LOADED,
ZCUTLASS_TORCH_EXTENSION_AVAILABLE, ZCUTLASS_VLLM_MODEL_REGISTERED,
ZCUTLASS_VLLM_OOT_LINEAR_REGISTERED. The reference also registers a toy
model (a registry probe); that is not part of the GEMM path, so
model_registered stays False.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Optional

from ..routing import env_flag


@dataclass
class PluginState:
    registered: bool = False
    extension_available: Optional[bool] = None
    model_registered: bool = False
    oot_linear_registered: bool = False
    message: str = ""


_STATE = PluginState()

# exported variable -> the state field it reports
_EXPORTS = {
    "ZCUTLASS_TORCH_EXTENSION_AVAILABLE": "extension_available",
    "ZCUTLASS_VLLM_MODEL_REGISTERED": "model_registered",
    "ZCUTLASS_VLLM_OOT_LINEAR_REGISTERED": "oot_linear_registered",
}


def _probe() -> None:
    from ..zcutlass_torch import extension_available

    _STATE.extension_available = extension_available()
    if env_flag("ZCUTLASS_VLLM_ENABLE"):
        try:
            from .oot_linear import register_oot_linear_layers

            _STATE.oot_linear_registered = register_oot_linear_layers()
        except Exception:
            _STATE.oot_linear_registered = False
    _STATE.message = "zcutlass vLLM overlay plugin loaded"


def register() -> None:
    """Registers the zcutlass overlay with a vLLM process; safe to call repeatedly."""
    if _STATE.registered:
        return
    try:
        _probe()
    except Exception as exc:  # pragma: no cover - defensive in vLLM worker processes
        _STATE.extension_available = False
        _STATE.oot_linear_registered = False
        _STATE.message = f"zcutlass vLLM overlay plugin failed to inspect extension: {exc}"
    os.environ["ZCUTLASS_VLLM_PLUGIN_LOADED"] = "1"
    for var, attr in _EXPORTS.items():
        os.environ[var] = "1" if getattr(_STATE, attr) else "0"
    _STATE.registered = True


def is_registered() -> bool:
    return _STATE.registered


def state() -> PluginState:
    return _STATE
