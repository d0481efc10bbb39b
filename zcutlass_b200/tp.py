"""Tensor-parallel linears over one NVLink/NVSwitch node (one process per GPU).

The reference has no multi-GPU code of its own: tensor parallelism reaches its
GEMM only through vLLM's ColumnParallelLinear / RowParallelLinear subclasses
(python/zcutlass_vllm/oot_linear.py:137-163), with the all-reduce done by
vLLM. This module provides the same two shardings natively:

  column-parallel (qkv, gate_up): weight rows (output features) split across
      ranks; every rank computes its slice of the output, no communication.
  row-parallel (o_proj, down): weight columns (input features) split across
      ranks; every rank computes a full-size BF16/F16 partial, then an NCCL
      all-reduce (sum) over NVLink combines them. The GEMM is issued in row
      chunks so the all-reduce of chunk i overlaps the GEMM of chunk i+1.

Weights use the PyTorch [out_features, in_features] layout and go to the
kernels as column-major B (no transposed copy). Every GEMM runs through the
zcutlass C ABI (zcutlass_gemm) on the current stream; `linear_fn` replaces
that call only in tests that check the sharding logic on CPU ranks.
"""

from __future__ import annotations

from dataclasses import dataclass

from . import torch_ops


@dataclass
class TPGroup:
    rank: int = 0
    world_size: int = 1
    group: object = None  # torch.distributed ProcessGroup (None = default group)

    @classmethod
    def from_env(cls, group=None) -> "TPGroup":
        import torch.distributed as dist

        if not dist.is_available() or not dist.is_initialized():
            return cls()
        return cls(dist.get_rank(group), dist.get_world_size(group), group)


def shard_range(total: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [start, stop) slice of `total` owned by `rank` (sizes differ by at most 1)."""
    base, rem = divmod(total, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def _linear_into(x, weight, bias, out) -> None:
    """out[M, N] = x[M, K] @ weight[N, K]^T (+ bias) through the zcutlass kernels."""
    import torch

    from . import _native

    torch_ops.load()
    m, k = x.shape
    n = weight.shape[0]
    t = _native.BF16 if x.dtype == torch.bfloat16 else _native.F16
    desc = _native.make_desc(m, n, k, x.stride(0), weight.stride(0), n, out.stride(0), t, 1.0, 0.0,
                             bias.data_ptr() if bias is not None else None,
                             torch.cuda.current_stream(x.device).cuda_stream, b_layout=_native.COLUMN_MAJOR)
    st = _native.gemm(desc, x.data_ptr(), weight.data_ptr(), None, out.data_ptr())
    if st != _native.SUCCESS:
        raise RuntimeError(f"zcutlass linear failed: {_native.status_name(st)}")


class ColumnParallelLinear:
    """y_shard = x @ W_shard^T + b_shard; W_shard = W[rows owned by this rank]."""

    def __init__(self, weight_shard, bias_shard=None, tp: TPGroup | None = None, linear_fn=None) -> None:
        self.weight = weight_shard
        self.bias = bias_shard
        self.tp = tp or TPGroup()
        self.linear_fn = linear_fn or _linear_into

    @classmethod
    def from_full(cls, weight, bias=None, tp: TPGroup | None = None, linear_fn=None) -> "ColumnParallelLinear":
        tp = tp or TPGroup()
        lo, hi = shard_range(weight.shape[0], tp.rank, tp.world_size)
        return cls(weight[lo:hi].contiguous(), None if bias is None else bias[lo:hi].contiguous(), tp, linear_fn)

    def forward(self, x, out=None):
        import torch

        if out is None:
            out = torch.empty(x.shape[0], self.weight.shape[0], device=x.device, dtype=x.dtype)
        self.linear_fn(x, self.weight, self.bias, out)
        return out

    __call__ = forward


class RowParallelLinear:
    """y = all_reduce_sum(x_shard @ W_shard^T) + b; W_shard = W[:, cols owned by this rank].

    The bias is added once, by rank 0's partial, so the all-reduced sum carries
    it exactly once. `chunks` row blocks let NCCL overlap with the GEMM."""

    def __init__(self, weight_shard, bias=None, tp: TPGroup | None = None, chunks: int = 4,
                 linear_fn=None) -> None:
        self.weight = weight_shard
        self.bias = bias
        self.tp = tp or TPGroup()
        self.chunks = max(1, chunks)
        self.linear_fn = linear_fn or _linear_into

    @classmethod
    def from_full(cls, weight, bias=None, tp: TPGroup | None = None, chunks: int = 4,
                  linear_fn=None) -> "RowParallelLinear":
        tp = tp or TPGroup()
        lo, hi = shard_range(weight.shape[1], tp.rank, tp.world_size)
        return cls(weight[:, lo:hi].contiguous(), bias, tp, chunks, linear_fn)

    def forward(self, x_shard, out=None):
        import torch
        import torch.distributed as dist

        m = x_shard.shape[0]
        if out is None:
            out = torch.empty(m, self.weight.shape[0], device=x_shard.device, dtype=x_shard.dtype)
        bias = self.bias if self.tp.rank == 0 else None
        if self.tp.world_size == 1:
            self.linear_fn(x_shard, self.weight, bias, out)
            return out
        works = []
        chunks = min(self.chunks, m)
        for i in range(chunks):
            r0, r1 = shard_range(m, i, chunks)
            if r1 == r0:
                continue
            self.linear_fn(x_shard[r0:r1], self.weight, bias, out[r0:r1])
            works.append(dist.all_reduce(out[r0:r1], op=dist.ReduceOp.SUM, group=self.tp.group, async_op=True))
        for w in works:
            w.wait()
        return out

    __call__ = forward


@dataclass
class LayerShape:
    """The four linears of one decoder layer (Llama-style)."""

    hidden: int
    intermediate: int
    q_heads: int
    kv_heads: int
    head_dim: int

    @property
    def qkv_out(self) -> int:
        return (self.q_heads + 2 * self.kv_heads) * self.head_dim

    @property
    def o_in(self) -> int:
        return self.q_heads * self.head_dim

    def flops(self, tokens: int) -> float:
        h, i = self.hidden, self.intermediate
        return 2.0 * tokens * (self.qkv_out * h + h * self.o_in + 2 * i * h + h * i)


LLAMA3_8B = LayerShape(4096, 14336, 32, 8, 128)
LLAMA3_70B = LayerShape(8192, 28672, 64, 8, 128)
QWEN2_1_5B = LayerShape(1536, 8960, 12, 2, 128)


class TPDecoderLinears:
    """qkv / o_proj / gate_up / down of one layer, sharded over `tp`.

    forward() runs the four GEMMs the way a decoder layer chains them, with
    the non-GEMM parts (attention, activation) left out: o_proj consumes this
    rank's head slice of the q part of the qkv output, down consumes this
    rank's slice of the gate_up output. Output: the all-reduced down result.
    """

    def __init__(self, shape: LayerShape, tp: TPGroup, device, dtype, seed: int = 0, chunks: int = 4,
                 qkv_bias: bool = False, linear_fn=None) -> None:
        import torch

        self.shape, self.tp = shape, tp
        w = tp.world_size
        h, inter = shape.hidden, shape.intermediate
        g = torch.Generator(device="cpu").manual_seed(seed + 1000 * tp.rank)

        def rnd(*size, scale=1.0):
            return (torch.randn(*size, generator=g) * scale).to(device=device, dtype=dtype)

        qkv_lo, qkv_hi = shard_range(shape.qkv_out, tp.rank, w)
        gu_lo, gu_hi = shard_range(2 * inter, tp.rank, w)
        o_lo, o_hi = shard_range(shape.o_in, tp.rank, w)
        d_lo, d_hi = shard_range(inter, tp.rank, w)
        self.qkv = ColumnParallelLinear(rnd(qkv_hi - qkv_lo, h, scale=h ** -0.5),
                                        rnd(qkv_hi - qkv_lo, scale=0.1) if qkv_bias else None, tp, linear_fn)
        self.gate_up = ColumnParallelLinear(rnd(gu_hi - gu_lo, h, scale=h ** -0.5), None, tp, linear_fn)
        self.o_proj = RowParallelLinear(rnd(h, o_hi - o_lo, scale=shape.o_in ** -0.5), None, tp, chunks, linear_fn)
        self.down = RowParallelLinear(rnd(h, d_hi - d_lo, scale=inter ** -0.5), None, tp, chunks, linear_fn)
        self.o_cols = o_hi - o_lo
        self.d_cols = d_hi - d_lo
        self._bufs = {}

    def flops_per_rank(self, tokens: int) -> float:
        q = self.qkv.weight.shape[0] * self.qkv.weight.shape[1]
        gu = self.gate_up.weight.shape[0] * self.gate_up.weight.shape[1]
        o = self.o_proj.weight.shape[0] * self.o_proj.weight.shape[1]
        d = self.down.weight.shape[0] * self.down.weight.shape[1]
        return 2.0 * tokens * (q + gu + o + d)

    def buffers(self, tokens: int, device, dtype) -> dict:
        import torch

        key = (tokens, str(device), dtype)
        if key not in self._bufs:
            e = lambda *s: torch.empty(*s, device=device, dtype=dtype)  # noqa: E731
            self._bufs[key] = {
                "qkv": e(tokens, self.qkv.weight.shape[0]),
                "gate_up": e(tokens, self.gate_up.weight.shape[0]),
                "o": e(tokens, self.shape.hidden),
                "down": e(tokens, self.shape.hidden),
            }
        return self._bufs[key]

    def forward(self, x, events: dict | None = None, out=None):
        """x: [tokens, hidden] (replicated on every rank). Returns the down output
        (written into `out` when given). `events` (optional) maps a GEMM name to
        a (start, end) CUDA event pair recorded around that GEMM on the current stream."""
        b = self.buffers(x.shape[0], x.device, x.dtype)

        def timed(name, fn):
            if events is not None and name in events:
                events[name][0].record()
                r = fn()
                events[name][1].record()
                return r
            return fn()

        timed("qkv", lambda: self.qkv(x, b["qkv"]))
        timed("gate_up", lambda: self.gate_up(x, b["gate_up"]))
        # o_proj input: this rank's slice of attention output, stood in by the q part of qkv.
        o_in = b["qkv"][:, : self.o_cols]
        timed("o_proj", lambda: self.o_proj(o_in, b["o"]))
        # down input: this rank's slice of act(gate) * up, stood in by the gate_up output.
        d_in = b["gate_up"][:, : self.d_cols]
        return timed("down", lambda: self.down(d_in, b["down"] if out is None else out))
