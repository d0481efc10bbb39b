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
        assert rep["sequence_parallel"]["rel_frobenius"] < 1e-3
