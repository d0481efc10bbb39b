"""One rank of the multi-GPU tensor-parallel parity check (run by
tests/test_gpu_tp.py under torch.distributed.run, one process per GPU).

Checks, against the CPU oracle:
  * zcutlass_nvls_allreduce: every element equals the FP32 sum of the ranks'
    bf16 values rounded once to bf16 (within one bf16 ulp, exact count
    reported), across consecutive calls (barrier epochs) and ragged sizes;
  * RowParallelLinear over the NVLS all-reduce and over NCCL: within the error
    of rounding each rank's partial GEMM to bf16 before the sum;
  * ColumnParallelLinear: each rank's column shard passes the single-GPU
    GEMM bounds;
  * the layer chain: two overlapped row blocks and graph replays against the
    sequential run, and the sequence-parallel step against the all-reduce
    step.
Rank 0 writes a JSON report to argv[1]; any failure raises (non-zero exit).
An optional argv[2] of "sp" runs the sequence-parallel check alone.
"""

from __future__ import annotations

import json
import os
import sys
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from oracle import oracle  # noqa: E402
from zcutlass_b200 import _native  # noqa: E402
from zcutlass_b200.tp import (ColumnParallelLinear, LayerShape, NvlsReducer, RowParallelLinear,  # noqa: E402
                              TPDecoderLinears, TPGroup, shard_range)

BF16 = _native.BF16


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def from_bits(b: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(torch.bfloat16).to(device)


def check_allreduce(red: NvlsReducer, rank: int, world: int, dev) -> dict:
    cols = red.bufs[0].shape[1]
    stats = {"calls": 0, "elements": 0, "exact": 0}
    for it, rows in enumerate([64, 1, 17, 64, 3, 40]):
        g = torch.Generator().manual_seed(1000 + it)  # same parts on every rank
        parts = [(torch.randn(rows, cols, generator=g) * (1 + r)).to(torch.bfloat16) for r in range(world)]
        i, y = red.next_buffer(rows)
        y.copy_(parts[rank].to(dev))
        red.reduce(i, rows)
        torch.cuda.synchronize(dev)
        got = y.float().cpu().double()
        exp = torch.stack([p.float() for p in parts]).sum(0).double()
        ulp = torch.from_numpy(oracle.ulp(exp.numpy(), BF16))
        err = (got - exp).abs()
        assert bool((err <= ulp).all()), f"NVLS all-reduce call {it}: max err/ulp {(err / ulp).max().item():.3f}"
        stats["calls"] += 1
        stats["elements"] += rows * cols
        stats["exact"] += int((got == exp.to(torch.bfloat16).double()).sum())
    code = _native.device_error(True)
    assert code == 0, f"device error word {code} after NVLS all-reduces"
    return stats


def check_row_parallel(tp: TPGroup, dev, use_nvls: bool) -> dict:
    rank, world = tp.rank, tp.world_size
    m, n, k = 96, 512, 384 * world
    x = oracle.make_tensor(m, k, k, 11, BF16)
    w = oracle.make_tensor(n, k, k, 12, BF16)  # [N, K] weight
    bias = oracle.make_tensor(1, n, n, 13, BF16)[0]
    klo, khi = shard_range(k, rank, world)
    row = RowParallelLinear(from_bits(w[:, klo:khi], dev), from_bits(bias, dev), tp, chunks=3)
    if use_nvls:
        assert row.enable_nvls(m), f"NVLS unavailable: {NvlsReducer.last_error}"
    outs = []
    for _ in range(3):  # repeated calls rotate the symmetric buffers
        outs.append(bits(row(from_bits(x[:, klo:khi], dev))))
    assert all(np.array_equal(outs[0], o) for o in outs[1:]), "row-parallel output changed between calls"
    ref = oracle.gemm(x, np.ascontiguousarray(w.T), m, n, k, BF16, bias=bias)
    parts = []
    for r in range(world):
        lo, hi = shard_range(k, r, world)
        parts.append(oracle.gemm(np.ascontiguousarray(x[:, lo:hi]), np.ascontiguousarray(w[:, lo:hi].T), m, n,
                                 hi - lo, BF16, bias=bias if r == 0 else None))
    out = oracle.bits_to_float(outs[0], BF16).astype(np.float64)
    # each partial is rounded to bf16 before the sum, and NCCL's ring rounds
    # every intermediate sum too: allow one bf16 rounding per rank
    bound = world * oracle.type_ulp(BF16) * (1 + np.abs(ref) + sum(np.abs(p) for p in parts))
    viol = float(np.max(np.abs(out - ref) / bound))
    rel = oracle.rel_frobenius(out, ref)
    assert viol <= 1.0 and rel <= 5e-3, f"row-parallel ({'nvls' if use_nvls else 'nccl'}): rel {rel} viol {viol}"
    assert _native.device_error(True) == 0
    return {"rel_frobenius": rel, "bound_ratio": viol}


def check_column_parallel(tp: TPGroup, dev) -> dict:
    m, n, k = 80, 384 * tp.world_size, 512
    x = oracle.make_tensor(m, k, k, 21, BF16)
    w = oracle.make_tensor(n, k, k, 22, BF16)
    bias = oracle.make_tensor(1, n, n, 23, BF16)[0]
    col = ColumnParallelLinear.from_full(from_bits(w, dev), from_bits(bias, dev), tp)
    out = oracle.bits_to_float(bits(col(from_bits(x, dev))), BF16)
    lo, hi = shard_range(n, tp.rank, tp.world_size)
    ref = oracle.gemm(x, np.ascontiguousarray(w[lo:hi].T), m, hi - lo, k, BF16, bias=bias[lo:hi])
    return oracle.check(out, ref, BF16)


def check_layer_overlap(tp: TPGroup, dev, use_nvls: bool) -> dict:
    """The layer chain run as two overlapped row blocks on two streams equals
    the sequential run (same kernels per block, same all-reduce per element)."""
    shape = LayerShape(hidden=1024, intermediate=2048, q_heads=8, kv_heads=2, head_dim=128)
    layer = TPDecoderLinears(shape, tp, dev, torch.bfloat16, seed=3, chunks=2)
    if use_nvls:
        assert layer.enable_nvls(512, lanes=2), f"NVLS unavailable: {NvlsReducer.last_error}"
    g = torch.Generator().manual_seed(77)
    x = torch.randn(512, shape.hidden, generator=g).to(torch.bfloat16).to(dev)
    streams = [torch.cuda.Stream(dev) for _ in range(2)]
    seq = torch.cat([layer.forward(x[:256]).clone(), layer.forward(x[256:]).clone()])
    for _ in range(3):  # several rounds: lanes rotate their symmetric buffers
        ov = torch.cat([y.clone() for y in layer.forward_overlapped(x, streams)])
    torch.cuda.synchronize(dev)
    exact = float((ov == seq).float().mean())
    rel = float((ov.float() - seq.float()).norm() / seq.float().norm())
    assert rel < 1e-3, f"overlapped vs sequential ({'nvls' if use_nvls else 'nccl'}): rel {rel}"
    # the same overlapped step captured once in a CUDA graph and replayed
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, capture_error_mode="thread_local"):
        ys = layer.forward_overlapped(x, streams)
    replays = []
    for _ in range(3):
        graph.replay()
        replays.append(torch.cat([y.clone() for y in ys]))
    torch.cuda.synchronize(dev)
    del graph  # a graph that holds NCCL calls goes before the process group
    graph_exact = all(bool((r == ov).all()) for r in replays)
    graph_rel = max(float((r.float() - ov.float()).norm() / ov.float().norm()) for r in replays)
    # NVLS: same kernels, same per-element reduction -> bit-identical. NCCL may
    # pick another algorithm inside a graph, so only the tolerance applies there.
    assert graph_exact if use_nvls else graph_rel < 1e-3, f"graph replay differs ({'nvls' if use_nvls else 'nccl'})"
    # several layer steps in one graph, the blocks joined only at its ends (bench --layers-per-graph)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, capture_error_mode="thread_local"):
        ys = layer.forward_overlapped_layers(x, streams, 3)
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize(dev)
    layered = torch.cat([y.clone() for y in ys])
    del graph
    layered_rel = float((layered.float() - ov.float()).norm() / ov.float().norm())
    assert bool((layered == ov).all()) if use_nvls else layered_rel < 1e-3, "layered graph differs"
    assert _native.device_error(True) == 0
    return {"exact_fraction": exact, "rel_frobenius": rel, "graph_replays_exact": graph_exact,
            "layered_rel_frobenius": layered_rel}


def check_sequence_parallel(tp: TPGroup, dev) -> dict:
    """The sequence-parallel step (reduce-scatters, qkv / gate_up on the other
    ranks' rows) gives this rank's rows of the all-reduce step's output, for
    both ways of getting those rows:
      * "copy" (peer row blocks copied into local memory, then the same GEMMs
        as the all-reduce step): bit for bit;
      * "fused" (rows read from the owners inside the GEMM): within the BF16
        product tolerance -- the all-reduce step may run these mid-M GEMMs as
        cluster split-K, whose partial sums round differently from the
        gathered persistent kernel's single accumulator.
    Two overlapped lanes and a CUDA graph replay give the step's own bits."""
    shape = LayerShape(hidden=1024, intermediate=2048, q_heads=8, kv_heads=2, head_dim=128)
    layer = TPDecoderLinears(shape, tp, dev, torch.bfloat16, seed=4, chunks=2)
    rows = 256 * tp.world_size
    assert layer.enable_sequence_parallel(rows, lanes=2), f"sequence parallel unavailable: {NvlsReducer.last_error}"
    g = torch.Generator().manual_seed(99)
    x = torch.randn(rows, shape.hidden, generator=g).to(torch.bfloat16).to(dev)
    for lane in range(2):
        layer.sp_inputs[lane].bufs[0][:rows].copy_(x)  # every rank holds all rows; each reads its owners'
    torch.cuda.synchronize(dev)
    dist.barrier()
    ref = layer.forward(x).clone()  # all-reduce path
    r0, r1 = shard_range(rows, tp.rank, tp.world_size)
    streams = [torch.cuda.Stream(dev) for _ in range(2)]
    report = {}
    for mode in ("copy", "fused"):
        layer.sp_gather = mode
        y = layer.forward_sp(rows)[r0:r1].clone()
        torch.cuda.synchronize(dev)
        exact = float((y == ref[r0:r1]).float().mean())
        rel = float((y.float() - ref[r0:r1].float()).norm() / ref[r0:r1].float().norm())
        if mode == "copy":
            assert exact == 1.0, f"sequence-parallel (copy) vs all-reduce step: exact fraction {exact}, rel {rel}"
        assert rel < 5e-3, f"sequence-parallel ({mode}) vs all-reduce step: rel {rel}"
        for _ in range(3):
            ys = [t[r0:r1].clone() for t in layer.forward_sp_overlapped(rows, streams)]
            torch.cuda.synchronize(dev)
            assert all(torch.equal(t, y) for t in ys), f"overlapped sequence-parallel lanes differ ({mode})"
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, capture_error_mode="thread_local"):
            outs = layer.forward_sp_overlapped(rows, streams)
        for _ in range(3):
            graph.replay()
            torch.cuda.synchronize(dev)
            assert all(torch.equal(t[r0:r1], y) for t in outs), f"graph replay of the sequence-parallel step differs ({mode})"
        del graph
        assert _native.device_error(True) == 0
        report[mode] = {"exact_fraction_vs_allreduce": exact, "rel_frobenius": rel}
    return report


def main() -> None:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    tp = TPGroup.from_env()
    report = {"world": world}

    only = sys.argv[2] if len(sys.argv) > 2 else None  # "sp": the sequence-parallel check alone
    red = NvlsReducer.try_create(64, 1024, torch.bfloat16, dev, tp.group)
    ok = torch.tensor([0 if red is None else 1], device=dev, dtype=torch.int32)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if only == "sp":
        assert int(ok.item()) == 1, f"NVLS unavailable: {NvlsReducer.last_error}"
        report["sequence_parallel"] = check_sequence_parallel(tp, dev)
    elif int(ok.item()) == 1:
        report["nvls_allreduce"] = check_allreduce(red, rank, world, dev)
        report["row_parallel_nvls"] = check_row_parallel(tp, dev, True)
    else:
        report["nvls_unavailable"] = NvlsReducer.last_error or "another rank has no multicast"
    if only is None:
        report["row_parallel_nccl"] = check_row_parallel(tp, dev, False)
        report["column_parallel"] = check_column_parallel(tp, dev)
        report["layer_overlap_nccl"] = check_layer_overlap(tp, dev, False)
    if only is None and "nvls_unavailable" not in report:
        report["layer_overlap_nvls"] = check_layer_overlap(tp, dev, True)
        report["sequence_parallel"] = check_sequence_parallel(tp, dev)
    torch.cuda.synchronize(dev)
    dist.barrier()
    if rank == 0:
        Path(sys.argv[1]).write_text(json.dumps(report))
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
