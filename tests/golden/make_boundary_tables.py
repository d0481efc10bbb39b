"""Regenerates tests/golden/reference_boundary_tables.json from the reference's sources.

The drop-in packages keep the reference's routing interface: the fallback
reason strings, the order in which they are tried, the keys of a vLLM
adapter trace and the columns of a route-log row. This script reads those
from the reference's Python sources with `ast` (nothing is imported or run)
and writes them as ordered lists; tests/test_boundary_tables.py compares the
package's rule tables with them. It must run where the reference checkout
exists (ZCUTLASS_REF_ROOT, else a `reference` directory beside this
repository); the test only reads the JSON it writes.

    python tests/golden/make_boundary_tables.py
"""

from __future__ import annotations

import ast
import json
import os
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "reference_boundary_tables.json"
REF_ROOT = Path(os.environ.get("ZCUTLASS_REF_ROOT", HERE.parents[2] / "reference"))
PY = REF_ROOT / "python"


def _function(path: Path, qualname: str) -> ast.FunctionDef:
    tree = ast.parse(path.read_text())
    parts = qualname.split(".")
    scope = tree.body
    node = None
    for part in parts:
        node = next(n for n in scope if isinstance(n, (ast.ClassDef, ast.FunctionDef)) and n.name == part)
        scope = node.body
    return node


def _returned_strings(fn: ast.FunctionDef) -> list[str]:
    """String constants returned (alone, or first in a returned tuple), in source order."""
    out = []
    for node in ast.walk(fn):
        if isinstance(node, ast.Return) and node.value is not None:
            v = node.value
            if isinstance(v, ast.Tuple) and v.elts:
                v = v.elts[0]
            if isinstance(v, ast.Constant) and isinstance(v.value, str):
                out.append((node.lineno, v.value))
    return [s for _, s in sorted(out)]


def _dict_keys(fn: ast.FunctionDef, last: bool = False) -> list[str]:
    """Keys of the first (or last) dict literal in the function."""
    dicts = sorted((n for n in ast.walk(fn) if isinstance(n, ast.Dict) and n.keys and
                    all(isinstance(k, ast.Constant) for k in n.keys)), key=lambda n: n.lineno)
    d = dicts[-1] if last else dicts[0]
    return [k.value for k in d.keys]


def main() -> int:
    overlay = PY / "zcutlass_torch" / "overlay.py"
    vllm = PY / "zcutlass_vllm"
    tables = {
        "overlay_reject_reasons": _returned_strings(_function(overlay, "ZCutlassGemmOverlay._reject_reason")),
        "policy_reject_reasons": _returned_strings(_function(overlay, "RoutingPolicy.reject_reason")),
        "policy_families": _returned_strings(_function(overlay, "RoutingPolicy.family")),
        "adapter_fast_reasons": _returned_strings(
            _function(vllm / "linear.py", "ZCutlassVllmLinearAdapter._fast_delegate_reason")),
        "adapter_trace_keys": _dict_keys(_function(vllm / "linear.py", "ZCutlassVllmLinearAdapter.run"), last=True),
        "method_delegate_reasons": _returned_strings(
            _function(vllm / "linear_method.py", "ZCutlassUnquantizedLinearMethod._delegate_without_transpose_reason")),
        "profit_policy_reasons": _returned_strings(
            _function(vllm / "linear_method.py", "ZCutlassUnquantizedLinearMethod._profit_policy_reject_reason")),
        "install_skip_reasons": _returned_strings(_function(vllm / "oot_linear.py", "_skip_install_for_profit_policy")),
        "route_row_keys": _dict_keys(_function(vllm / "route_logger.py", "build_route_row")),
    }
    OUT.write_text(json.dumps(tables, indent=1) + "\n")
    print(f"wrote {OUT}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
