"""PyTorch operators backed by libzcutlass_torch.so.

Loading registers (CUDA dispatch key only):
    torch.ops.zcutlass_torch.gemm(A, B, C=None, bias=None, alpha=1.0, beta=0.0) -> D
    torch.ops.zcutlass.gemm(...)        same op, product namespace
    torch.ops.zcutlass.gemm_out(A, B, C, bias, alpha, beta, D) -> ()
    torch.ops.zcutlass.linear(x, weight[N, K], bias=None) -> y

`selected_gemm_config` mirrors the reference's extension query
(python/zcutlass_torch/csrc/zcutlass_torch.cpp:91-149 in supercatking/zcutlass):
same checks, same dict keys, answered by the C ABI telemetry.
"""

from __future__ import annotations

from pathlib import Path

from . import _native

TORCH_SO = Path(__file__).resolve().parent / "libzcutlass_torch.so"
_LOADED = False


def load() -> None:
    """Registers the torch operators; raises if the extension was not built."""
    global _LOADED
    if _LOADED:
        return
    import torch

    if not TORCH_SO.exists():
        raise ImportError(f"{TORCH_SO} is missing: build it with `python -m zcutlass_b200.build`")
    _native.lib()  # same process-wide copy of libzcutlass.so the operators link against
    torch.ops.load_library(str(TORCH_SO))
    _LOADED = True


def available() -> bool:
    try:
        load()
    except Exception:
        return False
    return True


def _dtype_code(t) -> int:
    import torch

    if t.dtype == torch.float16:
        return _native.F16
    if t.dtype == torch.bfloat16:
        return _native.BF16
    raise RuntimeError("zcutlass only supports float16 and bfloat16 tensors")


def _check_2d(t, name: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if t.dim() != 2:
        raise RuntimeError(f"{name} must be rank-2")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be row-major contiguous")
    _dtype_code(t)


def selected_gemm_config(a, b, c=None, bias=None, alpha: float = 1.0, beta: float = 0.0) -> dict:
    """Dispatch metadata for one GEMM call site (host only, nothing launches)."""
    _check_2d(a, "A")
    _check_2d(b, "B")
    if a.dtype != b.dtype:
        raise RuntimeError("A and B dtype must match")
    if a.shape[1] != b.shape[0]:
        raise RuntimeError("A.shape[1] must equal B.shape[0]")
    if a.device != b.device:
        raise RuntimeError("A and B must be on the same CUDA device")
    if c is not None:
        _check_2d(c, "C")
        if c.dtype != a.dtype or c.device != a.device or tuple(c.shape) != (a.shape[0], b.shape[1]):
            raise RuntimeError("C must match A/B in dtype and device and be [A.shape[0], B.shape[1]]")
    if bias is not None:
        if not bias.is_cuda or bias.dim() != 1 or not bias.is_contiguous():
            raise RuntimeError("bias must be a contiguous rank-1 CUDA tensor")
        if bias.dtype != a.dtype or bias.shape[0] != b.shape[1]:
            raise RuntimeError("bias must match A/B dtype and have length B.shape[1]")
    t = _dtype_code(a)
    desc = _native.make_desc(a.shape[0], b.shape[1], a.shape[1], a.stride(0), b.stride(0),
                             c.stride(0) if c is not None else b.shape[1], b.shape[1], t,
                             float(alpha), float(beta), bias.data_ptr() if bias is not None else None)
    with _device_of(a):
        return _native.selected_kernel(desc)


class _device_of:
    """Makes `t.device` current so selection sees the right device's properties."""

    def __init__(self, t) -> None:
        self.t = t

    def __enter__(self):
        import torch

        self.ctx = torch.cuda.device(self.t.device)
        return self.ctx.__enter__()

    def __exit__(self, *exc):
        return self.ctx.__exit__(*exc)


def gemm(a, b, c=None, bias=None, alpha: float = 1.0, beta: float = 0.0):
    import torch

    load()
    return torch.ops.zcutlass.gemm(a, b, c, bias, float(alpha), float(beta))


def gemm_out(a, b, d, c=None, bias=None, alpha: float = 1.0, beta: float = 0.0):
    import torch

    load()
    torch.ops.zcutlass.gemm_out(a, b, c, bias, float(alpha), float(beta), d)
    return d


def linear(x, weight, bias=None):
    import torch

    load()
    return torch.ops.zcutlass.linear(x, weight, bias)
