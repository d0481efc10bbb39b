"""Benchmark regression gate over schema-v1 JSONL (the records zcutlass_bench
writes with --output).

Mirrors the reference's gate (tools/check_benchmark_regression.py): records of
one provider are matched between a baseline and a candidate file by
(operation, m, n, k, dtype, layout, alpha, beta); the gate fails when any
matched shape is slower than --max-slowdown (candidate_ms / baseline_ms) or
when the geometric mean of baseline_ms / candidate_ms is below
--min-geomean-speedup, and, unless --allow-missing, when a baseline shape has
no candidate record. Same options, same exit codes (0 pass, 1 fail, usage
errors exit with a message), same tab-separated report and optional Markdown
table.

    python -m zcutlass_b200.regression_gate base.jsonl cand.jsonl --shape-family decode
"""

from __future__ import annotations

import argparse
import json
import math
import sys
from pathlib import Path
from typing import NamedTuple


class ShapeKey(NamedTuple):
    operation: str
    m: int
    n: int
    k: int
    dtype: str
    layout: str
    alpha: float
    beta: float

    def label(self) -> str:
        return (f"{self.operation} {self.dtype} {self.m}x{self.n}x{self.k} "
                f"layout={self.layout} alpha={self.alpha:g} beta={self.beta:g}")


class Timing(NamedTuple):
    median_ms: float
    kernel: str


def read_records(path: Path, provider: str, tags: dict[str, str]) -> dict[ShapeKey, Timing]:
    """Successful records of `provider` whose tags match, keyed by shape (a
    later record of the same shape replaces an earlier one)."""
    out: dict[ShapeKey, Timing] = {}
    for no, line in enumerate(path.read_text().splitlines(), 1):
        if not line.strip():
            continue
        try:
            rec = json.loads(line)
        except json.JSONDecodeError as exc:
            raise SystemExit(f"{path}:{no}: invalid JSONL: {exc}") from exc
        if rec.get("provider") != provider or rec.get("status", "success") != "success":
            continue
        rtags = rec.get("tags", {})
        if any(str(rtags.get(k, "")) != v for k, v in tags.items()):
            continue
        prob = rec["problem"]
        key = ShapeKey(str(prob.get("operation", "gemm")), int(prob["m"]), int(prob["n"]), int(prob["k"]),
                       str(prob.get("dtype") or prob.get("a_type") or "unknown"),
                       str(prob.get("layout", "row,row,row,row")), float(prob.get("alpha", 1.0)),
                       float(prob.get("beta", 0.0)))
        out[key] = Timing(float(rec["performance"]["median_ms"]), str(rec.get("kernel", "")))
    return out


def _num(x: float) -> str:
    return "n/a" if math.isnan(x) else f"{x:.4f}"


def compare(base: dict[ShapeKey, Timing], cand: dict[ShapeKey, Timing], max_slowdown: float,
            min_geomean: float, allow_missing: bool):
    """Returns (rows, geomean, failures); rows = (key, base, cand, base_ms / cand_ms)."""
    failures: list[str] = []
    missing = [k for k in base if k not in cand]
    if missing and not allow_missing:
        failures.append(f"missing candidate records: {len(missing)}")
    rows = []
    for key in sorted(set(base) & set(cand), key=ShapeKey.label):
        b, c = base[key], cand[key]
        speedup = b.median_ms / c.median_ms if c.median_ms > 0 else math.nan
        rows.append((key, b, c, speedup))
        slowdown = c.median_ms / b.median_ms if b.median_ms > 0 else math.inf
        if slowdown > max_slowdown:
            failures.append(f"{key.label()} slowed {slowdown:.4f}x ({b.median_ms:.4f} ms -> {c.median_ms:.4f} ms)")
    logs = [math.log(r[3]) for r in rows if r[3] > 0 and not math.isnan(r[3])]
    geomean = math.exp(sum(logs) / len(logs)) if logs else math.nan
    if math.isnan(geomean) or geomean < min_geomean:
        failures.append(f"geomean speedup {_num(geomean)}x below required {min_geomean:.4f}x")
    return rows, geomean, failures


def markdown(rows) -> str:
    out = ["# Benchmark Regression Check", "",
           "| Shape | Baseline ms | Candidate ms | Baseline / candidate | Candidate kernel |",
           "| --- | ---: | ---: | ---: | --- |"]
    for key, b, c, sp in rows:
        out.append(f"| {key.label()} | {b.median_ms:.4f} | {c.median_ms:.4f} | {sp:.4f}x | `{c.kernel}` |")
    return "\n".join(out) + "\n"


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description="Gate a candidate benchmark JSONL against a baseline.")
    ap.add_argument("baseline", type=Path)
    ap.add_argument("candidate", type=Path)
    ap.add_argument("--provider", default="zcutlass")
    ap.add_argument("--tag", action="append", default=[], help="KEY=VALUE filter on the records' tags")
    ap.add_argument("--shape-family", help="shortcut for --tag shape_family=VALUE")
    ap.add_argument("--max-slowdown", type=float, default=1.05)
    ap.add_argument("--min-geomean-speedup", type=float, default=0.98)
    ap.add_argument("--allow-missing", action="store_true")
    ap.add_argument("--markdown", type=Path)
    args = ap.parse_args(argv)

    tags: dict[str, str] = {}
    for item in args.tag:
        if "=" not in item:
            raise SystemExit(f"Invalid --tag '{item}', expected KEY=VALUE")
        k, v = item.split("=", 1)
        tags[k] = v
    if args.shape_family:
        tags["shape_family"] = args.shape_family

    base = read_records(args.baseline, args.provider, tags)
    cand = read_records(args.candidate, args.provider, tags)
    if not base:
        raise SystemExit(f"No baseline records found for provider '{args.provider}' in {args.baseline}")
    if not cand:
        raise SystemExit(f"No candidate records found for provider '{args.provider}' in {args.candidate}")

    rows, geomean, failures = compare(base, cand, args.max_slowdown, args.min_geomean_speedup, args.allow_missing)
    print("shape\tbaseline_ms\tcandidate_ms\tbaseline/candidate\tcandidate_kernel")
    for key, b, c, sp in rows:
        print(f"{key.label()}\t{b.median_ms:.4f}\t{c.median_ms:.4f}\t{sp:.4f}\t{c.kernel}")
    print(f"geomean_speedup\t{_num(geomean)}x")
    if args.markdown:
        args.markdown.parent.mkdir(parents=True, exist_ok=True)
        args.markdown.write_text(markdown(rows))
        print(f"wrote {args.markdown}")
    if failures:
        print("benchmark regression gate failed:", file=sys.stderr)
        for f in failures:
            print(f"- {f}", file=sys.stderr)
        return 1
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
