"""Tensor parallelism on 2+ GPUs of one node: the library's NVLS all-reduce and
the row/column-parallel linears against the CPU oracle. Runs
tests/tp_multi_gpu_worker.py under torch.distributed.run (one process per
GPU, NCCL, rendezvous on 127.0.0.1); skipped on a single-GPU box."""

from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.gpu
def test_tensor_parallel_multi_gpu(tmp_path):
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 or more GPUs")
    world = min(n, 8)
    report = tmp_path / "tp_report.json"
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           str(ROOT / "tests" / "tp_multi_gpu_worker.py"), str(report)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=420, cwd=ROOT, env=dict(os.environ))
    assert r.returncode == 0, f"stdout:\n{r.stdout[-4000:]}\nstderr:\n{r.stderr[-6000:]}"
    rep = json.loads(report.read_text())
    print(json.dumps(rep))
    assert rep["world"] == world
    assert rep["row_parallel_nccl"]["bound_ratio"] <= 1.0
    if "nvls_unavailable" not in rep:
        assert rep["nvls_allreduce"]["calls"] == 6
        assert rep["row_parallel_nvls"]["bound_ratio"] <= 1.0
        assert rep["sequence_parallel"]["copy"]["exact_fraction_vs_allreduce"] == 1.0
        assert rep["sequence_parallel"]["fused"]["rel_frobenius"] < 5e-3


@pytest.mark.gpu
@pytest.mark.parametrize("comm", ["auto", "nccl"])
def test_bench_two_gpus_exits(comm):
    """bench.py at TP2 as the driver launches it (one rank per GPU, CUDA graphs
    holding the NCCL or NVLS all-reduces) prints its line and exits 0: every
    captured graph is freed before the process group is destroyed."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 or more GPUs")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           str(ROOT / "bench.py"), "--gpus", "2", "--steps", "3", "--warmup", "3", "--comm", comm]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=330, cwd=ROOT, env=dict(os.environ))
    assert r.returncode == 0, f"rc {r.returncode}\nstdout:\n{r.stdout[-3000:]}\nstderr:\n{r.stderr[-5000:]}"
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout[-3000:]
    line = json.loads(lines[0])
    assert line["n_gpus"] == 2 and line["value"] > 0 and line["e2e"]["value"] > 0
    assert "teardown did not finish" not in r.stderr


@pytest.mark.gpu
def test_vllm_tensor_parallel_native_weight(tmp_path):
    """vLLM's Column/RowParallelLinear with the zcutlass LinearMethod on native
    [N, K] weight shards, the all-reduce left to vLLM, against the oracle
    (tests/vllm_tp_worker.py)."""
    pytest.importorskip("vllm.model_executor.layers.linear")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 or more GPUs")
    report = tmp_path / "vllm_tp.json"
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           str(ROOT / "tests" / "vllm_tp_worker.py"), str(report)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=420, cwd=ROOT, env=dict(os.environ))
    assert r.returncode == 0, f"stdout:\n{r.stdout[-3000:]}\nstderr:\n{r.stderr[-6000:]}"
    rep = json.loads(report.read_text())
    assert rep["world"] == 2 and rep["weight_cache"] == "native"
    assert rep["row"]["bound_ratio"] <= 1.0
