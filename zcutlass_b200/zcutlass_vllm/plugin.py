"""vLLM general-plugin entry point (`vllm.general_plugins: zcutlass_overlay`).

Mirrors python/zcutlass_vllm/plugin.py in supercatking/zcutlass: idempotent
register(), PluginState, and the ZCUTLASS_VLLM_* / ZCUTLASS_TORCH_* environment
exports that report what loaded. The reference's toy model registration
(a registry probe, python/zcutlass_vllm/model.py) is not carried over; the
state reports model_registered = False.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Optional


@dataclass
class PluginState:
    registered: bool = False
    extension_available: Optional[bool] = None
    model_registered: bool = False
    oot_linear_registered: bool = False
    message: str = ""


_STATE = PluginState()
_OFF = (None, "", "0", "false", "False", "FALSE")


def register() -> None:
    """Registers the zcutlass overlay with a vLLM process; safe to call repeatedly."""
    if _STATE.registered:
        return
    try:
        from ..zcutlass_torch import extension_available

        _STATE.extension_available = extension_available()
        _STATE.model_registered = False
        if os.environ.get("ZCUTLASS_VLLM_ENABLE") not in _OFF:
            try:
                from .oot_linear import register_oot_linear_layers

                _STATE.oot_linear_registered = register_oot_linear_layers()
            except Exception:
                _STATE.oot_linear_registered = False
        _STATE.message = "zcutlass vLLM overlay plugin loaded"
    except Exception as exc:  # pragma: no cover - defensive in vLLM worker processes
        _STATE.extension_available = False
        _STATE.oot_linear_registered = False
        _STATE.message = f"zcutlass vLLM overlay plugin failed to inspect extension: {exc}"
    os.environ["ZCUTLASS_VLLM_PLUGIN_LOADED"] = "1"
    os.environ["ZCUTLASS_TORCH_EXTENSION_AVAILABLE"] = "1" if _STATE.extension_available else "0"
    os.environ["ZCUTLASS_VLLM_MODEL_REGISTERED"] = "1" if _STATE.model_registered else "0"
    os.environ["ZCUTLASS_VLLM_OOT_LINEAR_REGISTERED"] = "1" if _STATE.oot_linear_registered else "0"
    _STATE.registered = True


def is_registered() -> bool:
    return _STATE.registered


def state() -> PluginState:
    return _STATE
