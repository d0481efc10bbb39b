"""Regenerates tests/golden/reference_cpu_path.npz from the reference itself.

Runs the reference's own CPU path -- ZCutlassGemmOverlay with the extension
disabled, i.e. its `_fallback` (python/zcutlass_torch/overlay.py:130-145) for
`gemm` and `torch.nn.functional.linear` for `linear` (overlay.py:218-231) --
on seeded inputs, and stores inputs, outputs and the overlay's fallback
counters as small fixtures. It must run where the reference checkout exists
(ZCUTLASS_REF_ROOT, else a `reference` directory beside this repository); the tests only
read the .npz it writes.

    python tests/golden/make_golden.py
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
OUT = HERE / "reference_cpu_path.npz"
REF_ROOT = Path(os.environ.get("ZCUTLASS_REF_ROOT", HERE.parents[2] / "reference"))

# The reference's numeric test cases (tests/test_gemm.cu:754-786), shrunk where
# K*N would make the fixture large, plus LLM-shaped small cases.
CASES = [
    # name, dtype, m, n, k, alpha, beta, bias
    ("f16 tiny bias beta", "f16", 15, 17, 19, 1.0, 0.25, True),
    ("f16 16x16", "f16", 16, 16, 16, 1.0, 0.0, False),
    ("f16 rectangular", "f16", 65, 129, 31, 0.75, 0.5, True),
    ("f16 ragged alpha", "f16", 31, 63, 17, -0.5, 0.0, False),
    ("f16 ragged beta", "f16", 47, 64, 33, 0.5, -0.25, False),
    ("f16 llm-smoke", "f16", 8, 256, 256, 1.0, 0.0, False),
    ("bf16 tiny bias beta", "bf16", 13, 19, 23, 1.0, 0.25, True),
    ("bf16 16x16", "bf16", 16, 16, 16, 1.0, 0.0, False),
    ("bf16 rectangular", "bf16", 67, 127, 29, 0.75, 0.5, True),
    ("bf16 ragged alpha", "bf16", 29, 61, 15, -0.75, 0.0, False),
    ("bf16 ragged beta", "bf16", 45, 64, 31, 0.5, -0.25, False),
    ("bf16 llm-smoke", "bf16", 8, 256, 256, 1.0, 0.0, False),
    ("bf16 cfg0-shaped bias", "bf16", 16, 256, 512, 1.0, 0.0, True),
    ("f16 prefill-shaped", "f16", 64, 128, 512, 1.0, 1.0, True),
]


def main() -> int:
    import torch

    sys.path.insert(0, str(REF_ROOT / "python"))
    from zcutlass_torch.overlay import ZCutlassGemmOverlay  # the reference package

    dt = {"f16": torch.float16, "bf16": torch.bfloat16}
    g = torch.Generator().manual_seed(0)
    arrays: dict[str, np.ndarray] = {}
    names = []
    for i, (name, dname, m, n, k, alpha, beta, bias) in enumerate(CASES):
        t = dt[dname]
        a = torch.randn(m, k, generator=g).to(t)
        b = (torch.randn(k, n, generator=g) / k ** 0.5).to(t)
        c = torch.randn(m, n, generator=g).to(t)
        bv = (torch.randn(n, generator=g) * 0.1).to(t)
        ov = ZCutlassGemmOverlay(enable_zcutlass=False)
        out = ov.gemm(a, b, c if beta != 0.0 else None, bv if bias else None, alpha, beta)
        assert ov.stats.misses == 1 and ov.stats.fallback_reasons == {"zcutlass_disabled": 1}
        assert ov.last_kernel_path == "pytorch_fallback"
        # linear(): stock F.linear on the [N, K] weight (not pre-transposed)
        lin = ov.linear(a, b.t().contiguous(), bv if bias else None)
        assert ov.stats.fallback_reasons.get("weight_not_pretransposed") == 1
        p = f"c{i}_"
        bits = lambda x: x.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
        arrays[p + "a"] = bits(a)
        arrays[p + "b"] = bits(b)
        arrays[p + "c"] = bits(c)
        arrays[p + "bias"] = bits(bv)
        arrays[p + "gemm_out"] = bits(out)
        arrays[p + "linear_out"] = bits(lin)
        arrays[p + "meta"] = np.array([m, n, k, 1 if dname == "bf16" else 0, 1 if bias else 0], np.int64)
        arrays[p + "scalars"] = np.array([alpha, beta], np.float32)
        names.append(name)
    arrays["names"] = np.array(names)
    arrays["torch_version"] = np.array(torch.__version__)
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(CASES)} cases)")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
