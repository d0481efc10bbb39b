"""Tensor-parallel sharding on world_size-2 `gloo` CPU ranks.

The GEMM itself is replaced by a CPU matmul (the reference's CPU path,
oracle/overlay_fallback.py) so the test checks only what the multi-rank code
adds: column shards, row shards, the chunked all-reduce, the bias added once,
and that a rank leaving early turns the survivor's next collective into an
error instead of a hang.
"""

from __future__ import annotations

import os
import socket
import sys
import traceback
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cpu_linear(x, weight, bias, out):
    from oracle import overlay_fallback

    out.copy_(overlay_fallback.linear(x, weight, bias))


def _init(rank, world, port, timeout_s=60):
    from datetime import timedelta

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))


def _worker_sharding(rank, world, port, errq):
    try:
        sys.path.insert(0, str(ROOT))
        from zcutlass_b200.tp import (ColumnParallelLinear, LayerShape, RowParallelLinear, TPDecoderLinears,
                                      TPGroup, shard_range)

        _init(rank, world, port)
        tp = TPGroup.from_env()
        assert (tp.rank, tp.world_size) == (rank, world)
        g = torch.Generator().manual_seed(123)  # same full weights on every rank
        x = torch.randn(10, 24, generator=g)
        w_col = torch.randn(18, 24, generator=g)
        b_col = torch.randn(18, generator=g)
        w_row = torch.randn(12, 24, generator=g)
        b_row = torch.randn(12, generator=g)

        col = ColumnParallelLinear.from_full(w_col, b_col, tp, linear_fn=_cpu_linear)
        lo, hi = shard_range(18, rank, world)
        torch.testing.assert_close(col(x), torch.nn.functional.linear(x, w_col, b_col)[:, lo:hi])

        for chunks in (1, 3, 16):
            row = RowParallelLinear.from_full(w_row, b_row, tp, chunks=chunks, linear_fn=_cpu_linear)
            klo, khi = shard_range(24, rank, world)
            y = row(x[:, klo:khi].contiguous())
            torch.testing.assert_close(y, torch.nn.functional.linear(x, w_row, b_row), rtol=1e-5, atol=1e-5)

        # The layer wrapper: every rank ends with the same all-reduced output,
        # equal to the unsharded layer computed from the gathered shards.
        shape = LayerShape(hidden=32, intermediate=48, q_heads=4, kv_heads=2, head_dim=8)
        layer = TPDecoderLinears(shape, tp, "cpu", torch.float32, seed=5, chunks=2, linear_fn=_cpu_linear)
        xl = torch.randn(6, 32, generator=g)
        out = layer.forward(xl).clone()

        def gather(t, dim):
            parts = [None] * world
            dist.all_gather_object(parts, t)
            return torch.cat(parts, dim=dim)

        wq = gather(layer.qkv.weight, 0)
        wgu = gather(layer.gate_up.weight, 0)
        qkv_full = xl @ wq.t()
        gu_full = xl @ wgu.t()
        # o_proj / down consume each rank's slice of its own column shard
        o_in = gather(layer.buffers(6, "cpu", torch.float32)["qkv"][:, : layer.o_cols], 1)
        d_in = gather(layer.buffers(6, "cpu", torch.float32)["gate_up"][:, : layer.d_cols], 1)
        wo = gather(layer.o_proj.weight, 1)
        wd = gather(layer.down.weight, 1)
        torch.testing.assert_close(out, d_in @ wd.t(), rtol=1e-4, atol=1e-4)
        torch.testing.assert_close(layer.buffers(6, "cpu", torch.float32)["o"], o_in @ wo.t(), rtol=1e-4, atol=1e-4)
        # gate_up consumes the all-reduced o_proj output (the layer's dependency order)
        bufs = layer.buffers(6, "cpu", torch.float32)
        torch.testing.assert_close(bufs["gate_up"], bufs["o"] @ layer.gate_up.weight.t(), rtol=1e-4, atol=1e-4)
        assert qkv_full.shape == (6, shape.qkv_out) and gu_full.shape == (6, 2 * shape.intermediate)
        assert layer.flops_per_rank(6) > 0
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        errq.put((rank, traceback.format_exc()))
        raise


def _worker_rank_leaves(rank, world, port, errq):
    try:
        sys.path.insert(0, str(ROOT))
        from zcutlass_b200.tp import RowParallelLinear, TPGroup

        _init(rank, world, port, timeout_s=10)
        tp = TPGroup.from_env()
        row = RowParallelLinear(torch.randn(8, 4), None, tp, chunks=2, linear_fn=_cpu_linear)
        row(torch.randn(4, 4))  # one good step on both ranks
        dist.barrier()
        if rank == 1:
            os._exit(0)  # leaves between steps, with nothing in flight
        try:
            row(torch.randn(4, 4))
        except Exception as exc:  # the survivor learns of it as an error, not a hang
            errq.put((rank, f"expected-error:{type(exc).__name__}"))
            return
        errq.put((rank, "no error raised"))
    except Exception:
        errq.put((rank, traceback.format_exc()))


def _run(fn, world=2, timeout=240):
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
        if p.is_alive():
            p.kill()
            pytest.fail("rank did not finish")
    msgs = []
    while not errq.empty():
        msgs.append(errq.get())
    return procs, msgs


def test_tp_sharding_world2_gloo():
    procs, msgs = _run(_worker_sharding)
    assert not msgs, msgs
    assert all(p.exitcode == 0 for p in procs)


def test_rank_leaving_turns_into_error_world2_gloo():
    procs, msgs = _run(_worker_rank_leaves)
    assert msgs and all(m[0] == 0 and m[1].startswith("expected-error") for m in msgs), msgs
