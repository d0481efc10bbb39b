"""zcutlass_b200: a dense FP16/BF16 GEMM library for NVIDIA B200 (sm_100a).

Drop-in for the hot path of supercatking/zcutlass: row-major
D = alpha * A @ B + beta * C + bias with FP32 accumulation, behind the same
C++ API (include/zcutlass/gemm.hpp), a flat C ABI (include/zcutlass_c.h), the
`torch.ops.zcutlass_torch.gemm` operator with its opt-in overlay
(zcutlass_b200.zcutlass_torch) and the vLLM LinearMethod plugin
(zcutlass_b200.zcutlass_vllm). Tensor-parallel linears live in zcutlass_b200.tp.

Native code is required: importing a submodule that needs libzcutlass.so
raises if it has not been built (`python -m zcutlass_b200.build`).
"""

from __future__ import annotations

__all__ = ["build", "native", "torch_ops"]


def native():
    """The ctypes binding of the C ABI (loads libzcutlass.so)."""
    from . import _native

    _native.lib()
    return _native
