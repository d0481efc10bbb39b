"""TEST/BENCH INFRASTRUCTURE ONLY: the reference's CPU path, restated.

The reference has no CPU GEMM of its own; a GEMM that cannot run on its
kernels falls back to stock PyTorch inside its overlay:

  ZCutlassGemmOverlay._fallback   python/zcutlass_torch/overlay.py:130-145
      out = torch.matmul(a, b); out *= alpha (if != 1); out += c*beta (if C and
      beta != 0); out += bias (if given)
  ZCutlassGemmOverlay.linear      python/zcutlass_torch/overlay.py:218-231
      torch.nn.functional.linear(x, weight, bias) when the weight is not
      pre-transposed (the path BASELINE config 0 times on the host cores).

bench.py times these on the host cores as the CPU baseline
(`cpu_baseline.kind = "port"`) and as `--impl reference`. Nothing in the
product imports this module.
"""

from __future__ import annotations


def gemm(a, b, c=None, bias=None, alpha: float = 1.0, beta: float = 0.0):
    import torch

    out = torch.matmul(a, b)
    if alpha != 1.0:
        out = out * alpha
    if c is not None and beta != 0.0:
        out = out + c * beta
    if bias is not None:
        out = out + bias
    return out


def linear(x, weight, bias=None):
    import torch

    return torch.nn.functional.linear(x, weight, bias)
