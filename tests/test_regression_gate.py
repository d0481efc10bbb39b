"""The schema-v1 benchmark regression gate (zcutlass_b200.regression_gate):
same matching, thresholds and exit codes as the reference's
tools/check_benchmark_regression.py."""

from __future__ import annotations

import json

import pytest

from zcutlass_b200 import regression_gate as gate


def _rec(m, n, k, ms, *, provider="zcutlass", family="decode", status="success", beta=0.0, kernel="k"):
    return {"schema_version": 1,
            "problem": {"operation": "gemm", "m": m, "n": n, "k": k, "dtype": "bf16", "layout": "row,col,row,row",
                        "alpha": 1.0, "beta": beta},
            "provider": provider, "status": status, "kernel": kernel,
            "performance": {"median_ms": ms}, "tags": {"suite": "llm", "shape_family": family}}


def _write(path, recs):
    path.write_text("\n".join(json.dumps(r) for r in recs) + "\n\n")
    return path


def test_pass_within_tolerance(tmp_path, capsys):
    base = _write(tmp_path / "b.jsonl", [_rec(16, 1280, 8192, 0.010), _rec(16, 8192, 1024, 0.008)])
    cand = _write(tmp_path / "c.jsonl", [_rec(16, 1280, 8192, 0.0102), _rec(16, 8192, 1024, 0.0075)])
    md = tmp_path / "out" / "gate.md"
    assert gate.main([str(base), str(cand), "--markdown", str(md)]) == 0
    out = capsys.readouterr().out
    assert "geomean_speedup" in out and "gemm bf16 16x1280x8192 layout=row,col,row,row" in out
    assert md.read_text().startswith("# Benchmark Regression Check")


def test_fails_on_per_shape_slowdown(tmp_path, capsys):
    base = _write(tmp_path / "b.jsonl", [_rec(1, 4096, 4096, 0.010), _rec(8, 4096, 4096, 0.010)])
    cand = _write(tmp_path / "c.jsonl", [_rec(1, 4096, 4096, 0.0107), _rec(8, 4096, 4096, 0.0090)])
    assert gate.main([str(base), str(cand)]) == 1
    assert "slowed 1.0700x" in capsys.readouterr().err


def test_fails_on_geomean(tmp_path):
    base = _write(tmp_path / "b.jsonl", [_rec(1, 1024, 1024, 1.0), _rec(2, 1024, 1024, 1.0)])
    cand = _write(tmp_path / "c.jsonl", [_rec(1, 1024, 1024, 1.04), _rec(2, 1024, 1024, 1.04)])
    # each shape is within 1.05x, the geomean 0.9615 is below 0.98
    assert gate.main([str(base), str(cand)]) == 1
    assert gate.main([str(base), str(cand), "--min-geomean-speedup", "0.95"]) == 0


def test_missing_records_and_filters(tmp_path):
    base = _write(tmp_path / "b.jsonl", [_rec(1, 512, 512, 1.0), _rec(4096, 4096, 4096, 2.0, family="large"),
                                        _rec(1, 512, 512, 9.0, provider="cublas"),
                                        _rec(2, 512, 512, 9.0, status="failed")])
    cand = _write(tmp_path / "c.jsonl", [_rec(4096, 4096, 4096, 2.0, family="large")])
    assert gate.main([str(base), str(cand)]) == 1  # the decode shape is missing
    assert gate.main([str(base), str(cand), "--allow-missing"]) == 0
    assert gate.main([str(base), str(cand), "--shape-family", "large"]) == 0
    assert gate.main([str(base), str(cand), "--tag", "suite=llm", "--tag", "shape_family=large"]) == 0
    with pytest.raises(SystemExit):  # no candidate records for that family
        gate.main([str(base), str(cand), "--shape-family", "decode"])
    with pytest.raises(SystemExit):
        gate.main([str(base), str(cand), "--tag", "badtag"])


def test_invalid_jsonl(tmp_path):
    base = tmp_path / "b.jsonl"
    base.write_text('{"provider": "zcutlass"\n')
    cand = _write(tmp_path / "c.jsonl", [_rec(1, 512, 512, 1.0)])
    with pytest.raises(SystemExit, match="invalid JSONL"):
        gate.main([str(base), str(cand)])


def test_beta_is_part_of_the_key(tmp_path):
    base = _write(tmp_path / "b.jsonl", [_rec(64, 1024, 1024, 1.0, beta=1.0)])
    cand = _write(tmp_path / "c.jsonl", [_rec(64, 1024, 1024, 1.0, beta=0.0)])
    assert gate.main([str(base), str(cand)]) == 1  # different key: missing, and no rows for the geomean
