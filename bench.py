#!/usr/bin/env python3
"""Benchmark: Llama-3-8B-shaped prefill linears at TP = --gpus.

One step = the four linears of one decoder layer at M = 8192 tokens, BF16,
in the layer's dependency order (qkv -> o_proj -> gate_up -> down; attention,
norms and the activation are left out): qkv [6144 x 4096] and gate_up
[28672 x 4096] column-parallel (N split over ranks, no communication),
o_proj [4096 x 4096] and down [4096 x 14336] row-parallel (K split, then an
all-reduce of the BF16 partials: the library's NVLS kernel, or NCCL with
--comm nccl). At TP > 1 the 8192 tokens run as two independent 4096-row
blocks on two streams (--micro), so one block's all-reduce overlaps the other
block's GEMMs. The steps are replayed from CUDA graphs of up to 10 consecutive
layer steps (--layers-per-graph) with the blocks joined only at each graph's
ends, as a stack of layers runs: one block's next layer overlaps the other
block's last all-reduce; every step does the whole layer's work. 3573 GFLOP
per step for the whole job, whatever the rank count (strong scaling). --sp 1 runs the sequence-parallel form of the same
step instead (reduce-scatters; qkv / gate_up get the other ranks' rows by
copy-engine copies into local memory, or inside the GEMM with --sp-gather
fused; NVLS only).

    python bench.py                          # N=1, defaults
    torchrun --nproc-per-node N bench.py --gpus N --steps K --warmup W
    python bench.py --impl reference         # the reference's CPU path (host cores)

Prints one JSON line on rank 0. `value` = whole-job TFLOP/s, device-timed
with CUDA events between barriers, max over ranks; `e2e` = the same step
through the C ABI with the input activations copied from pinned host memory
and the layer output copied back inside the timed region (copies on their
own streams, double-buffered). Inputs are larger than L2 (126 MB) every
step, so no explicit flush is done.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "Prefill GEMM TFLOP/s/GPU (% of BF16 dense peak) at TP 1/2/4/8; decode GB/s"
TOKENS = 8192
MEASURED_PEAKS = ROOT / "MEASURED_PEAKS.json"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of
# the dominant kernel at TP1 -- gate_up 8192 x 28672 x 4096 on the 2-CTA
# 256x256 kernel -- from one ncu capture of that exact launch (1113.3 MB read +
# 455.4 MB written; algorithmic 301.9 MB read + 469.8 MB written).
GATE_UP_TRAFFIC_BYTES = 1113329152 + 455350528

NVML_REASONS = {
    0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
    0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
    0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
}


def load_peaks() -> tuple[dict, str]:
    try:
        return json.loads(MEASURED_PEAKS.read_text()), "measured"
    except Exception:
        return dict(FALLBACK_PEAKS), "fallback"


def choose_peak(peaks: dict, sm_mhz_median, sm_max_mhz) -> tuple[float, str]:
    """The bf16 denominator that matches the clocks the timed region ran at.

    MEASURED_PEAKS.json holds a burst figure (cuBLAS timed alone, clocks near
    their maximum) and a sustained one (seconds of back-to-back GEMMs under
    the power cap, with the median SM clock it settled at). A timed region
    whose median SM clock sits nearer the maximum than the sustained clock is
    compared with the burst peak; otherwise with the sustained one."""
    burst, sustained = peaks["bf16_tflops"], peaks["bf16_tflops_sustained"]
    sus_mhz = (peaks.get("clocks_under_load") or {}).get("sm_mhz_median")
    max_mhz = sm_max_mhz or peaks.get("sm_max_mhz")
    if sm_mhz_median is None or sus_mhz is None or max_mhz is None:
        return sustained, "bf16_tflops_sustained (no clock samples to choose by)"
    if sm_mhz_median >= 0.5 * (sus_mhz + max_mhz):
        return burst, (f"bf16_tflops (burst): timed-region median SM clock {sm_mhz_median:.0f} MHz is nearer "
                       f"the maximum {max_mhz:.0f} than the sustained run's {sus_mhz:.0f}")
    return sustained, (f"bf16_tflops_sustained: timed-region median SM clock {sm_mhz_median:.0f} MHz is nearer "
                       f"the sustained run's {sus_mhz:.0f} than the maximum {max_mhz:.0f}")


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML while running."""

    def __init__(self, device_index: int, period_s: float = 0.002) -> None:
        self.idx, self.period = device_index, period_s
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            self._h = pynvml.nvmlDeviceGetHandleByIndex(self.idx)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._nv = pynvml
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        except Exception:
            self._nv = None
        return self

    def _run(self) -> None:
        nv = self._nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((mhz, reasons))
            except Exception:
                pass
            time.sleep(self.period)

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()
        return False

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        mhz = [s[0] for s in self.samples]
        bits = 0
        for _, r in self.samples:
            bits |= r
        reasons = sorted(name for b, name in NVML_REASONS.items() if bits & b and name != "gpu_idle")
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(mhz)}


# ---------------------------------------------------------------- CPU path


def cpu_layer_sample(rows: int, dtype_name: str = "bf16"):
    """The four linears of the layer on `rows` tokens on the host cores, through
    the reference's CPU path (overlay fallback = F.linear), restated in oracle/."""
    import torch

    from oracle import overlay_fallback
    from zcutlass_b200.tp import LLAMA3_8B as S

    dt = torch.bfloat16 if dtype_name == "bf16" else torch.float16
    g = torch.Generator().manual_seed(0)
    x = torch.randn(rows, S.hidden, generator=g).to(dt)
    w = {
        "qkv": (torch.randn(S.qkv_out, S.hidden, generator=g) * S.hidden ** -0.5).to(dt),
        "gate_up": (torch.randn(2 * S.intermediate, S.hidden, generator=g) * S.hidden ** -0.5).to(dt),
        "o": (torch.randn(S.hidden, S.o_in, generator=g) * S.o_in ** -0.5).to(dt),
        "down": (torch.randn(S.hidden, S.intermediate, generator=g) * S.intermediate ** -0.5).to(dt),
    }

    def step():  # the decoder layer's dependency order, as on the GPU
        qkv = overlay_fallback.linear(x, w["qkv"])
        o = overlay_fallback.linear(qkv[:, : S.o_in], w["o"])
        gu = overlay_fallback.linear(o, w["gate_up"])
        return overlay_fallback.linear(gu[:, : S.intermediate], w["down"])

    return step, S.flops(rows)


def cpu_throughput(budget_s: float, steps: int | None = None, warmup: int = 1) -> dict:
    """Times the CPU path on a bounded sample: TFLOP/s with all host threads."""
    import torch

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    step, flops = cpu_layer_sample(64)
    t0 = time.perf_counter()
    step()
    per_row_s = (time.perf_counter() - t0) / 64
    n_steps = steps if steps is not None else 10
    rows = int(max(16, min(TOKENS, budget_s / max(n_steps + warmup, 1) / max(per_row_s, 1e-9))))
    step, flops = cpu_layer_sample(rows)
    for _ in range(warmup):
        step()
    times = []
    for _ in range(n_steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    return {"value": flops / sec / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"layer linears on {rows} of {TOKENS} tokens (bf16 F.linear on CPU, "
                      f"{n_steps} timed steps, median {sec * 1e3:.1f} ms)",
            "steps": n_steps, "ms_per_step": sec * 1e3}


def run_reference(args) -> int:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    cb = cpu_throughput(budget_s=120.0, steps=args.steps, warmup=args.warmup)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(cb["value"], 4), "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": cb["ms_per_step"],
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) activations, N(0,1/K) weights)",
        "config": {"workload": "llama3-8b-layer-prefill-linears", "tokens": TOKENS, "model": "llama3-8b-shaped",
                   "global_batch": TOKENS, "seq_len": TOKENS, "parallelism": "cpu"},
        "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": round(cb["value"], 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- GPU path


def decode_sweep(device, peaks: dict, iters: int = 200) -> list[dict]:
    """Llama-3-70B TP=8 per-GPU decode linears on one GPU:
    achieved HBM GB/s, weights rotated over > 2x L2 so every launch streams HBM.
    The `iters` launches are captured once in a CUDA graph and replayed, as a
    decode step is in serving, so the time is the kernels' and not the host's."""
    import torch

    from zcutlass_b200 import _native

    shapes = {"qkv": (1280, 8192), "o_proj": (8192, 1024), "gate_up": (7168, 8192), "down": (8192, 3584)}
    out = []
    for name, (n, k) in shapes.items():
        wbytes = n * k * 2
        copies = max(2, -(-3 * 126 * 2**20 // wbytes))
        ws = [torch.randn(n, k, device=device, dtype=torch.bfloat16) * k ** -0.5 for _ in range(copies)]
        for m in (1, 8, 16, 32):
            x = torch.randn(m, k, device=device, dtype=torch.bfloat16)
            d = torch.empty(m, n, device=device, dtype=torch.bfloat16)

            def run(i, descs):
                st = _native.gemm(descs[i % copies], x.data_ptr(), ws[i % copies].data_ptr(), None, d.data_ptr())
                assert st == 0, st

            def make_descs():
                stream = torch.cuda.current_stream(device).cuda_stream
                return [_native.make_desc(m, n, k, k, k, n, n, _native.BF16, stream=stream,
                                          b_layout=_native.COLUMN_MAJOR) for _ in ws]

            # warm-up and capture on one stream, so per-stream state (the
            # experimental stream-K workspace) exists before the capture
            side = torch.cuda.Stream(device)
            with torch.cuda.stream(side):
                eager = make_descs()
                for i in range(2 * copies):
                    run(i, eager)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=side, capture_error_mode="thread_local"):
                captured = make_descs()
                for i in range(iters):
                    run(i, captured)
            graph.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            graph.replay()
            e1.record()
            torch.cuda.synchronize()
            del graph
            us = e0.elapsed_time(e1) * 1e3 / iters
            nbytes = 2 * (m * k + n * k + m * n)
            gbs = nbytes / (us * 1e-6) / 1e9
            sel = _native.selected_kernel(eager[0])["kernel_name"]
            out.append({"linear": name, "m": m, "n": n, "k": k, "us": round(us, 2), "GB/s": round(gbs, 1),
                        "frac_hbm": round(gbs / peaks["hbm_gbs"], 3), "kernel": sel})
        del ws
    return out


def capture_steps(fn, copies: int) -> tuple[list, int]:
    """`copies` CUDA graphs of fn() and the library kernel launches one holds.
    No reference to a graph survives outside the returned list."""
    import torch

    from zcutlass_b200 import _native

    graphs, per = [], 0
    for _ in range(copies):
        graphs.append(torch.cuda.CUDAGraph())
        l0 = _native.kernel_launches()
        with torch.cuda.graph(graphs[-1], capture_error_mode="thread_local"):
            fn()
        per = _native.kernel_launches() - l0
    return graphs, per


def teardown(world: int, device, barrier, deadline_s: float = 60.0) -> None:
    """Ends a multi-rank run: every graph is already freed by the caller; a
    final barrier and destroy_process_group run on a helper thread with a
    host-side deadline, and the process exits either way (the JSON line is
    already flushed), so a stuck teardown cannot hold the GPUs."""
    import gc

    import torch
    import torch.distributed as dist

    gc.collect()
    torch.cuda.synchronize()
    if world <= 1:
        return
    done = threading.Event()

    def _end():
        try:
            torch.cuda.set_device(device)  # the CUDA device is per host thread
            barrier()
            dist.destroy_process_group()
        finally:
            done.set()

    threading.Thread(target=_end, daemon=True).start()
    if not done.wait(deadline_s):
        print(f"bench.py: teardown did not finish within {deadline_s:.0f} s; exiting", file=sys.stderr, flush=True)
        sys.stdout.flush()
        os._exit(0)


def run_gpu(args) -> int:
    import torch
    import torch.distributed as dist

    from zcutlass_b200 import _native, torch_ops
    from zcutlass_b200.tp import LLAMA3_8B, TPDecoderLinears, TPGroup, check_device_error, shard_range

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=device)
    torch_ops.load()
    peaks, peaks_src = load_peaks()
    tp = TPGroup.from_env()
    layer = TPDecoderLinears(LLAMA3_8B, tp, device, torch.bfloat16, seed=0, chunks=args.chunks)
    micro = args.micro if args.micro > 0 else (2 if world > 1 else 1)
    comm = "none"
    if world > 1:
        want_nvls = args.comm in ("nvls", "auto")
        comm = "nvls" if want_nvls and layer.enable_nvls(TOKENS, lanes=micro) else "nccl"
    streams = [torch.cuda.Stream(device) for _ in range(micro)] if micro > 1 else None
    args.micro_used = micro
    lane_rows = TOKENS // micro
    # sequence-parallel layer: activations row-sharded between the linears,
    # reduce-scatters instead of all-reduces, peer row blocks copied in (or
    # read inside the GEMMs with --sp-gather fused)
    sp = bool(args.sp) and comm == "nvls" and TOKENS % micro == 0 and layer.enable_sequence_parallel(TOKENS, micro)
    layer.sp_gather = args.sp_gather
    g = torch.Generator(device="cpu").manual_seed(1)
    x_host = torch.randn(TOKENS, LLAMA3_8B.hidden, generator=g).to(torch.bfloat16)
    x = x_host.to(device)
    if sp:
        # every rank holds every input row (each GEMM reads a row block from its
        # owner); lane 0 holds all rows for the sequential breakdown pass
        for j in range(micro):
            rows = TOKENS if j == 0 else lane_rows
            layer.sp_inputs[j].bufs[0][:rows].copy_(x[j * lane_rows: j * lane_rows + rows])
        torch.cuda.synchronize()
        dist.barrier()

    def step(xx, evs=None, outs=None):
        """One layer step; returns (row offset, output block) pieces."""
        if sp:
            if streams is not None:
                return [(j * lane_rows, y) for j, y in enumerate(layer.forward_sp_overlapped(lane_rows, streams))]
            return [(0, layer.forward_sp(TOKENS, events=evs))]
        if streams is not None:
            ys = layer.forward_overlapped(xx, streams, outs)
            return [(shard_range(xx.shape[0], j, micro)[0], y) for j, y in enumerate(ys)]
        return [(0, layer.forward(xx, events=evs, out=None if outs is None else outs[0]))]

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        step(x)
    barrier()
    # At TP > 1 the step is replayed from a CUDA graph: its ~20 launches are
    # host-bound otherwise (the GEMMs of a TP8 step last tens of microseconds).
    use_graph = args.graph == "on" or (args.graph == "auto" and world > 1)
    lpg = min(max(1, args.layers_per_graph), args.steps) if use_graph and streams is not None and not sp else 1
    args.lpg_used = lpg
    graphs, launches_per_step = [], None
    if use_graph:
        # the sequence-parallel step must not reuse an output buffer on
        # consecutive steps (other ranks read it), so it is captured twice.
        # The list is the only owner of the graphs (they may hold NCCL calls):
        # clearing it before destroy_process_group frees them all.
        if lpg > 1:
            # lpg consecutive layer steps per graph (lanes joined at its ends)
            # plus a one-step graph for the remainder of --steps
            graphs, per = capture_steps(lambda: layer.forward_overlapped_layers(x, streams, lpg), 1)
            launches_per_step = per // lpg
            # no name may keep a graph alive past graphs.clear(): they can hold NCCL calls
            graphs += capture_steps(lambda: step(x), 1)[0]
        else:
            graphs, launches_per_step = capture_steps(lambda: step(x), 2 if sp else 1)
        for i in range(4):
            graphs[i % len(graphs)].replay()
        barrier()

    # ---- device-timed steps (inputs resident in HBM)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = _native.kernel_launches()
    with ClockSampler(local) as clocks:
        barrier()
        start.record()
        if lpg > 1:
            for _ in range(args.steps // lpg):
                graphs[0].replay()
            for _ in range(args.steps % lpg):
                graphs[1].replay()
        else:
            for i in range(args.steps):
                if graphs:
                    graphs[i % len(graphs)].replay()
                else:
                    step(x, {"gate_up": ev[i]})
        end.record()
        torch.cuda.synchronize()
    check_device_error()  # a bounded wait that gave up invalidates the timed steps
    launches = _native.kernel_launches() - launches0
    if graphs:  # replays launch what the capture recorded
        launches = launches_per_step * args.steps
    ms = max_over_ranks(start.elapsed_time(end)) / args.steps
    barrier()
    total_flops = LLAMA3_8B.flops(TOKENS)
    value = total_flops / (ms * 1e-3) / 1e12
    live_gate = streams is None and not graphs
    if live_gate:
        gate_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in ev)
    gate_flops = 2.0 * TOKENS * layer.gate_up.weight.shape[0] * layer.gate_up.weight.shape[1]
    sm = clocks.summary()
    peak, peak_rule = choose_peak(peaks, sm["sm_mhz"], sm["sm_max_mhz"])
    # per-linear breakdown (untimed pass; o_proj and down include their all-reduce)
    names = ("qkv", "gate_up", "o_proj", "down")
    bev = [{nm: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for nm in names}
           for _ in range(20)]
    for evs in bev:
        if sp:
            layer.forward_sp(TOKENS, events=evs)
        else:
            layer.forward(x, events=evs)
    torch.cuda.synchronize()
    breakdown = {nm: round(max_over_ranks(statistics.mean(e[nm][0].elapsed_time(e[nm][1]) for e in bev)), 4)
                 for nm in names}
    barrier()
    if not live_gate:  # overlapped or graph-replayed steps: take gate_up from the sequential pass
        gate_ms = statistics.mean(e["gate_up"][0].elapsed_time(e["gate_up"][1]) for e in bev)
    gate_tflops = gate_flops / (gate_ms * 1e-3) / 1e12
    gw = layer.gate_up.weight
    gate_kernel = _native.selected_kernel(_native.make_desc(
        TOKENS, gw.shape[0], gw.shape[1], gw.shape[1], gw.shape[1], gw.shape[0], gw.shape[0], _native.BF16,
        b_layout=_native.COLUMN_MAJOR))["kernel_name"]

    # ---- end to end through the C ABI with pinned host buffers
    if sp:
        e2e = run_e2e_sp(args, layer, streams, lane_rows, x_host, device, barrier, max_over_ranks, total_flops,
                         use_graph)
    else:
        e2e = run_e2e(args, layer, step, x_host, device, barrier, max_over_ranks, total_flops, use_graph)

    line = None
    if rank == 0:
        cfg = {"workload": "llama3-8b-layer-prefill-linears", "model": "llama3-8b-shaped", "tokens": TOKENS,
               "global_batch": TOKENS, "seq_len": TOKENS, "parallelism": f"tp{world}",
               "linears": {"qkv": [6144, 4096], "o_proj": [4096, 4096], "gate_up": [28672, 4096],
                           "down": [4096, 14336]},
               "l2": "inputs larger than L2 every step (436 MB of weights per layer at TP1), no flush",
               "allreduce": {"nvls": "zcutlass_nvls_allreduce (multimem.ld_reduce acc::f32 + multimem.st)",
                             "nccl": f"NCCL all_reduce, {args.chunks} row chunks", "none": "none (TP1)"}[comm],
               "micro_batches": micro, "cuda_graph": use_graph, "layer_steps_per_graph": lpg,
               "sequence_parallel": sp, **({"sp_gather": args.sp_gather} if sp else {}),
               "order": "qkv -> o_proj (+all-reduce) -> gate_up -> down (+all-reduce)"}
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) activations, N(0,1/K) weights)",
            "config": cfg,
            "per_gpu_tflops": round(value / world, 2),
            "frac_of_bf16_peak_per_gpu": round(value / world / peak, 4),
            "roofline": {"bound": "tensor", "kernel": f"gate_up ({gate_kernel})",
                         "timing": "events around gate_up in the timed steps" if live_gate else
                                   "events around gate_up in a sequential pass after the timed steps",
                         "achieved": round(gate_tflops, 2), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(gate_tflops / peak, 4),
                         "peak_source": f"{peak_rule}; of {peaks_src} MEASURED_PEAKS.json",
                         "frac_of_burst": round(gate_tflops / peaks["bf16_tflops"], 4),
                         "frac_of_sustained": round(gate_tflops / peaks["bf16_tflops_sustained"], 4),
                         "algorithmic_flops_per_launch": gate_flops, "avg_launch_ms": round(gate_ms, 4),
                         "traffic": GATE_UP_TRAFFIC_BYTES if world == 1 else None},
            "clocks": sm,
            "linear_ms": breakdown,
            "e2e": e2e,
            "gpu_launches": launches,
        }
    if rank == 0 and world == 1 and not args.skip_decode:
        line["decode"] = decode_sweep(device, peaks)
    if rank == 0 and world == 1 and not args.skip_cpu:
        line["cpu_baseline"] = {k: v for k, v in cpu_throughput(budget_s=10.0).items()
                                if k in ("value", "unit", "cores", "kind", "sample")}
    check_device_error()
    if rank == 0:
        print(json.dumps(line), flush=True)
    graphs.clear()  # the captured graphs (they may hold NCCL calls) go before the process group
    teardown(world, device, barrier)
    return 0


def run_e2e(args, layer, step, x_host, device, barrier, max_over_ranks, total_flops, use_graph=False) -> dict:
    """Same step with host buffers, whole job copying the input once and the
    output once: rank r copies rows [r0, r1) of the layer input from pinned
    host memory (H2D stream), an NCCL all-gather over NVLink assembles the
    full input on every rank, and rank r copies rows [r0, r1) of the
    all-reduced output back (D2H stream). Buffers are double-buffered so the
    copies of step i+1 / i-1 overlap the GEMMs of step i; all inside the timed region."""
    import torch
    import torch.distributed as dist

    from zcutlass_b200.tp import shard_range

    world, rank = layer.tp.world_size, layer.tp.rank
    compute = torch.cuda.current_stream(device)
    h2d_s, d2h_s = torch.cuda.Stream(device), torch.cuda.Stream(device)
    m, hidden = x_host.shape
    r0, r1 = shard_range(m, rank, world)
    hx = x_host[r0:r1].contiguous().pin_memory()
    dx_part = [torch.empty_like(hx, device=device) for _ in range(2)]
    dx = dx_part if world == 1 else [torch.empty(m, hidden, device=device, dtype=hx.dtype) for _ in range(2)]
    dout = [torch.empty(m, layer.shape.hidden, device=device, dtype=hx.dtype) for _ in range(2)]
    res = [None, None]
    streams_n = args.micro_used
    blocks = [shard_range(m, j, streams_n) for j in range(streams_n)]
    hout = [torch.empty(r1 - r0, layer.shape.hidden, dtype=hx.dtype).pin_memory() for _ in range(2)]
    e = lambda: torch.cuda.Event()  # noqa: E731
    h2d_ev, d2h_ev, comp_ev = [e(), e()], [e(), e()], [e(), e()]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    steps = args.steps

    def compute_part(s):
        if world > 1:
            dist.all_gather_into_tensor(dx[s], dx_part[s], group=layer.tp.group)
        # NVLS keeps the output in its lanes' rotating symmetric buffers
        return step(dx[s], outs=None if layer.down.nvls else [dout[s]] if streams_n == 1 else
                    [dout[s][p0:p1] for p0, p1 in blocks])

    graphs, graph_res = [], []

    def run_compute(s):
        if graphs:
            graphs[s].replay()
            return graph_res[s]
        return compute_part(s)

    def loop(n):
        start.record(compute)
        h2d_s.wait_event(start)
        with torch.cuda.stream(h2d_s):
            dx_part[0].copy_(hx, non_blocking=True)
        h2d_ev[0].record(h2d_s)
        for i in range(n):
            s = i % 2
            compute.wait_event(h2d_ev[s])
            if i >= 2:
                compute.wait_event(d2h_ev[s])
            res[s] = run_compute(s)
            comp_ev[s].record(compute)
            if i + 1 < n:
                if i >= 1:
                    h2d_s.wait_event(comp_ev[1 - s])
                with torch.cuda.stream(h2d_s):
                    dx_part[1 - s].copy_(hx, non_blocking=True)
                h2d_ev[1 - s].record(h2d_s)
            d2h_s.wait_event(comp_ev[s])
            with torch.cuda.stream(d2h_s):
                for p0, y in res[s]:  # this rank's rows [r0, r1) from each output block
                    lo, hi = max(r0, p0), min(r1, p0 + y.shape[0])
                    if lo < hi:
                        hout[s][lo - r0:hi - r0].copy_(y[lo - p0:hi - p0], non_blocking=True)
            d2h_ev[s].record(d2h_s)
        compute.wait_event(d2h_ev[(n - 1) % 2])
        end.record(compute)
        torch.cuda.synchronize()

    loop(min(3, steps))
    barrier()
    if use_graph:  # one graph per input/output buffer pair (the copies stay outside)
        for s in range(2):
            graphs.append(torch.cuda.CUDAGraph())
            with torch.cuda.graph(graphs[-1], capture_error_mode="thread_local"):
                graph_res.append(compute_part(s))
        loop(min(3, steps))
        barrier()
    loop(steps)
    ms = max_over_ranks(start.elapsed_time(end)) / steps
    barrier()
    graphs.clear()  # graphs holding NCCL calls go before the process group does
    torch.cuda.synchronize()
    return {"value": round(total_flops / (ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s", "ms_per_step": round(ms, 4),
            "h2d_bytes_per_step": m * hidden * hx.element_size(),
            "d2h_bytes_per_step": m * layer.shape.hidden * hx.element_size(),
            "copies": "whole job: input rows split over ranks (H2D) + NCCL all-gather; output rows split (D2H)",
            "api": "C ABI zcutlass_gemm (include/zcutlass_c.h) via zcutlass_b200.tp"}


def run_e2e_sp(args, layer, streams, lane_rows, x_host, device, barrier, max_over_ranks, total_flops,
               use_graph=False) -> dict:
    """End to end for the sequence-parallel step: each rank copies only its own
    input rows of every row block from pinned host memory into the block's
    input buffer (three rotate), a cross-rank barrier makes every rank's rows
    visible, the step runs (qkv reads the other rows from their owners), and
    each rank copies its own output rows back. No all-gather is needed."""
    import torch

    from zcutlass_b200.tp import shard_range

    world, rank = layer.tp.world_size, layer.tp.rank
    micro = len(streams) if streams is not None else 1
    compute = torch.cuda.current_stream(device)
    h2d_s, d2h_s = torch.cuda.Stream(device), torch.cuda.Stream(device)
    hidden = x_host.shape[1]
    r0, r1 = shard_range(lane_rows, rank, world)
    hx = [x_host[j * lane_rows + r0: j * lane_rows + r1].contiguous().pin_memory() for j in range(micro)]
    hout = [[torch.empty(r1 - r0, layer.shape.hidden, dtype=x_host.dtype).pin_memory() for _ in range(micro)]
            for _ in range(2)]
    e = lambda: torch.cuda.Event()  # noqa: E731
    h2d_ev, comp_ev, d2h_ev = [e() for _ in range(3)], [e() for _ in range(3)], [e(), e()]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def h2d(t):
        with torch.cuda.stream(h2d_s):
            for j in range(micro):
                layer.sp_inputs[j].bufs[t % 3][r0:r1].copy_(hx[j], non_blocking=True)
        h2d_ev[t % 3].record(h2d_s)

    def compute_part(xi):
        layer.sp_inputs[0].barrier()  # every rank's input rows for this step are in
        if streams is not None:
            return layer.forward_sp_overlapped(lane_rows, streams, xi)
        return [layer.forward_sp(lane_rows, xi)]

    graphs, graph_res = [], []

    def loop(n):
        start.record(compute)
        h2d_s.wait_event(start)
        h2d(0)
        for t in range(n):
            xi = t % 3
            compute.wait_event(h2d_ev[xi])
            if t >= 2:
                compute.wait_event(d2h_ev[t % 2])
            if graphs:
                graphs[xi].replay()
                ys = graph_res[xi]
            else:
                ys = compute_part(xi)
            comp_ev[xi].record(compute)
            if t + 1 < n:
                # input buffer (t+1) % 3 was last read by the ranks at step t-2;
                # this rank's step t-1 (its barriers) proves every rank is past it
                if t >= 1:
                    h2d_s.wait_event(comp_ev[(t - 1) % 3])
                h2d(t + 1)
            d2h_s.wait_event(comp_ev[xi])
            with torch.cuda.stream(d2h_s):
                for j in range(micro):
                    hout[t % 2][j].copy_(ys[j][r0:r1], non_blocking=True)
            d2h_ev[t % 2].record(d2h_s)
        compute.wait_event(d2h_ev[(n - 1) % 2])
        end.record(compute)
        torch.cuda.synchronize()

    loop(3)
    barrier()
    if use_graph:  # one graph per input buffer; the row-parallel buffers rotate in step
        for xi in range(3):
            graphs.append(torch.cuda.CUDAGraph())
            with torch.cuda.graph(graphs[-1], capture_error_mode="thread_local"):
                graph_res.append(compute_part(xi))
        loop(3)
        barrier()
    loop(args.steps)
    ms = max_over_ranks(start.elapsed_time(end)) / args.steps
    barrier()
    graphs.clear()
    torch.cuda.synchronize()
    m = lane_rows * micro
    return {"value": round(total_flops / (ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s", "ms_per_step": round(ms, 4),
            "h2d_bytes_per_step": m * hidden * x_host.element_size(),
            "d2h_bytes_per_step": m * layer.shape.hidden * x_host.element_size(),
            "copies": "whole job: each rank copies its own input rows (H2D) and its own output rows (D2H); "
                      "no all-gather (the GEMMs read peer rows)",
            "api": "C ABI zcutlass_gemm_gather_a / zcutlass_nvls_reduce_scatter via zcutlass_b200.tp"}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["zcutlass", "reference"], default="zcutlass")
    ap.add_argument("--chunks", type=int, default=1, help="row chunks of the NCCL row-parallel all-reduce")
    ap.add_argument("--micro", type=int, default=0,
                    help="independent row blocks per step, each on its own stream (0: 2 when TP > 1, else 1)")
    ap.add_argument("--graph", choices=["auto", "on", "off"], default="auto",
                    help="replay each step from a CUDA graph (auto: when TP > 1)")
    ap.add_argument("--layers-per-graph", type=int, default=10,
                    help="at TP > 1 with row blocks: consecutive layer steps captured in one CUDA graph, the "
                         "blocks joined only at its ends (as a stack of layers runs), so one block's next layer "
                         "overlaps another block's last all-reduce; every step does the full layer's work")
    ap.add_argument("--sp", type=int, default=0,
                    help="1: sequence-parallel layer (reduce-scatters, all-gathers fused into the GEMMs; NVLS only)")
    ap.add_argument("--sp-gather", choices=["copy", "fused"], default="copy",
                    help="--sp 1: peer row blocks copied into local memory by the copy engines before a plain GEMM "
                         "(copy), or read from the owners inside the GEMM (fused)")
    ap.add_argument("--comm", choices=["auto", "nvls", "nccl"], default="auto",
                    help="row-parallel all-reduce: the library's NVLS kernel or NCCL (auto: NVLS where the "
                         "GPUs support multicast, else NCCL; measured faster than NCCL at TP2 and TP8)")
    ap.add_argument("--skip-decode", action="store_true")
    ap.add_argument("--skip-cpu", action="store_true")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        return run_reference(args)
    return run_gpu(args)


if __name__ == "__main__":
    sys.exit(main())
