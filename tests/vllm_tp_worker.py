"""One rank of the vLLM tensor-parallel check (run by tests/test_gpu_tp.py under
torch.distributed.run, one process per GPU).

vLLM's own ColumnParallelLinear (qkv_proj-shaped) and RowParallelLinear
(o_proj-shaped) are built inside vLLM's tensor-parallel group, the zcutlass
LinearMethod is installed on both with native_weight_layout=True -- the
weights stay in vLLM's [N, K] shards, no transposed copy exists -- and a
prefill-sized batch goes through column -> row, with the row-parallel
all-reduce left to vLLM (python/zcutlass_vllm/oot_linear.py:158-163 in the
reference). Checked against the CPU oracle on the full, unsharded weights:
the column shard within the single-GPU product bounds, the all-reduced row
output within one f16 rounding per rank (each rank's partial is rounded
before vLLM sums it). Each method must report one hit per call and
weight_cache "native". Rank 0 writes a JSON report to argv[1].
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

from oracle import oracle  # noqa: E402
from zcutlass_b200.tp import shard_range  # noqa: E402

F16 = oracle.F16


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def from_bits(b: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(torch.float16).to(device)


def main() -> None:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from vllm.config import VllmConfig, set_current_vllm_config
    from vllm.distributed import parallel_state as ps

    from zcutlass_vllm import install_zcutlass_unquantized_linear_method

    report = {"world": world}
    with set_current_vllm_config(VllmConfig()):
        ps.set_custom_all_reduce(False)  # vLLM's NCCL all-reduce, as a default serving setup without IPC buffers
        ps.init_distributed_environment(world, rank, "env://", local, backend="nccl")
        ps.initialize_model_parallel(tensor_model_parallel_size=world)
        from vllm.model_executor.layers.linear import ColumnParallelLinear, RowParallelLinear

        m, k, n = 256, 1536, 1024 * world  # M = 256 and N, K >= 1024 per shard: the "prefill" family
        x = oracle.make_tensor(m, k, k, 31, F16)
        wc = oracle.make_tensor(n, k, k, 32, F16)  # column-parallel weight [N, K]
        bc = oracle.make_tensor(1, n, n, 33, F16)[0]
        wr = oracle.make_tensor(k, n, n, 34, F16)  # row-parallel weight [K_out = k, K_in = n]
        with torch.device(dev):  # as vLLM's model loader does: parameters are made on the GPU
            col = ColumnParallelLinear(k, n, bias=True, params_dtype=torch.float16,
                                       prefix="model.layers.0.self_attn.qkv_proj")
            row = RowParallelLinear(n, k, bias=False, params_dtype=torch.float16,
                                    prefix="model.layers.0.self_attn.o_proj")
        assert col.weight.is_cuda and row.weight.is_cuda
        lo, hi = shard_range(n, rank, world)
        assert tuple(col.weight.shape) == (hi - lo, k) and tuple(row.weight.shape) == (k, hi - lo)
        with torch.no_grad():
            col.weight.copy_(from_bits(wc[lo:hi], dev))
            col.bias.copy_(from_bits(bc[lo:hi], dev))
            row.weight.copy_(from_bits(wr[:, lo:hi], dev))
        mc = install_zcutlass_unquantized_linear_method(col, promoted_families=("prefill",), native_weight_layout=True)
        mr = install_zcutlass_unquantized_linear_method(row, promoted_families=("prefill",), native_weight_layout=True)

        y_shard, _ = col(from_bits(x, dev))
        out, _ = row(y_shard)
        torch.cuda.synchronize()
        for name, meth in (("column", mc), ("row", mr)):
            assert meth.stats.hits == 1 and meth.stats.misses == 0, (name, meth.stats)
            assert meth.last_trace["weight_cache"] == "native" and meth.last_trace["fallback_reason"] is None
            assert not hasattr(col if name == "column" else row, "_zcutlass_weight_t_cache")

        # column shard: the single-GPU product bounds
        y_bits = bits(y_shard)
        ref_col = oracle.gemm(x, np.ascontiguousarray(wc[lo:hi].T), m, hi - lo, k, F16, bias=bc[lo:hi])
        report["column"] = oracle.check(oracle.bits_to_float(y_bits, F16), ref_col, F16)

        # row: the oracle on the gathered column output and the full row weight
        parts_bits = [torch.empty_like(y_shard) for _ in range(world)]
        torch.distributed.all_gather(parts_bits, y_shard, group=ps.get_tp_group().device_group)
        y_full = np.concatenate([bits(p) for p in parts_bits], axis=1)
        ref = oracle.gemm(y_full, np.ascontiguousarray(wr.T), m, k, n, F16)
        partials = []
        for r in range(world):
            a, b = shard_range(n, r, world)
            partials.append(oracle.gemm(np.ascontiguousarray(y_full[:, a:b]), np.ascontiguousarray(wr[:, a:b].T), m,
                                        k, b - a, F16))
        got = oracle.bits_to_float(bits(out), F16).astype(np.float64)
        bound = world * oracle.type_ulp(F16) * (1 + np.abs(ref) + sum(np.abs(p) for p in partials))
        viol = float(np.max(np.abs(got - ref) / bound))
        rel = oracle.rel_frobenius(got, ref)
        assert viol <= 1.0 and rel <= 2e-3, f"row-parallel through vLLM: rel {rel} viol {viol}"
        report["row"] = {"rel_frobenius": rel, "bound_ratio": viol}
        report["weight_cache"] = "native"
        if rank == 0:
            Path(sys.argv[1]).write_text(json.dumps(report))
        ps.destroy_model_parallel()
        ps.destroy_distributed_environment()


if __name__ == "__main__":
    main()
