"""Tensor-parallel linears over one NVLink/NVSwitch node (one process per GPU).

The reference has no multi-GPU code of its own: tensor parallelism reaches its
GEMM only through vLLM's ColumnParallelLinear / RowParallelLinear subclasses
(python/zcutlass_vllm/oot_linear.py:137-163), with the all-reduce done by
vLLM. This module provides the same two shardings natively:

  column-parallel (qkv, gate_up): weight rows (output features) split across
      ranks; every rank computes its slice of the output, no communication.
  row-parallel (o_proj, down): weight columns (input features) split across
      ranks; every rank computes a full-size BF16/F16 partial, then an
      all-reduce (sum) over NVLink combines them: the library's own NVLS
      kernel (multimem reduction in the NVSwitch, FP32 accumulation) on
      symmetric memory when the node supports multicast, else NCCL with the
      GEMM issued in row chunks so the all-reduce of chunk i overlaps the
      GEMM of chunk i+1.

TPDecoderLinears chains the four linears of one decoder layer;
forward_overlapped() runs independent row blocks on separate streams so one
block's all-reduce overlaps another block's GEMMs. forward_sp() is the
sequence-parallel form of the same step: activations stay row-sharded between
the linears, o_proj and down end in an NVLS reduce-scatter, and qkv / gate_up
read the other ranks' rows inside the GEMM (zcutlass_gemm_gather_a: TMA loads
from peer memory, no multicast), so no separate all-gather runs.

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


def check_device_error() -> None:
    """Raises if a kernel of the library recorded an error on the current
    device since the last check (a bounded wait that gave up: an NVLS barrier
    whose peers never arrived, or a GEMM pipeline wait). After such an error
    the outputs of the steps since the last check must not be used: the NVLS
    reduction skips its work once the error word is set. Reading the word
    synchronises the device; call it between steps, not inside a capture."""
    from . import _native

    code = _native.device_error(clear=True)
    if code < 0:
        raise RuntimeError("zcutlass device error word unreadable: the device synchronisation failed")
    if code != 0:
        raise RuntimeError(f"zcutlass device error word 0x{code:x} (site {code >> 4}, role {code & 15}): "
                           "a bounded wait gave up; the results since the last check are invalid")


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

    def forward_gathered(self, x_parts: list[int], rows: int, out) -> None:
        """out = x @ W_shard^T (+ b_shard) where x [rows, K] is sequence-sharded:
        its row block r (rows / len(x_parts) rows) is read by the GEMM straight
        from x_parts[r] -- a full [rows, K] buffer in rank r's memory -- with
        no separate all-gather (zcutlass_gemm_gather_a)."""
        import torch

        from . import _native

        k = self.weight.shape[1]
        n = self.weight.shape[0]
        t = _native.BF16 if self.weight.dtype == torch.bfloat16 else _native.F16
        desc = _native.make_desc(rows, n, k, k, self.weight.stride(0), n, out.stride(0), t, 1.0, 0.0,
                                 self.bias.data_ptr() if self.bias is not None else None,
                                 torch.cuda.current_stream(out.device).cuda_stream, b_layout=_native.COLUMN_MAJOR)
        st = _native.gemm_gather_a(desc, x_parts, self.weight.data_ptr(), None, out.data_ptr())
        if st != _native.SUCCESS:
            raise RuntimeError(f"zcutlass_gemm_gather_a failed: {_native.status_name(st)}")


class NvlsReducer:
    """Row-parallel outputs in symmetric memory with an NVLink SHARP mapping.

    Three symmetric buffers rotate between calls (the consumers of call i --
    this rank's next GEMM, or other ranks reading rows of it -- can still be
    reading buffer i while calls i+1 and i+2 write the others). `reduce`
    sums a partial in place across ranks with the library's NVLS all-reduce
    (zcutlass_nvls_allreduce: FP32 accumulation in the switch, one NVLink
    crossing per byte and direction), which brackets the reduction with its
    own bounded cross-rank barriers on two counter words kept in the same
    symmetric allocation, after the buffers. Every launch is fixed at
    issue time (no per-call values), so a step can be captured in a CUDA
    graph; each replay then alternates nothing -- the buffer a captured call
    uses is the one it used at capture."""

    def __init__(self, max_rows: int, cols: int, dtype, device, group=None, nbufs: int = 3) -> None:
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm

        group = group or dist.group.WORLD
        self.dtype = dtype
        self.nbufs = nbufs
        elem = torch.empty(0, dtype=dtype).element_size()
        region = -(-max_rows * cols * elem // 256) * 256
        raw = symm.empty(nbufs * region + 256, dtype=torch.uint8, device=device)
        self.handle = symm.rendezvous(raw, group)
        if not self.handle.multicast_ptr:
            raise RuntimeError("NVLS multicast is not available for this group")
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.raw = raw
        self.bufs = [raw[i * region: i * region + max_rows * cols * elem].view(dtype).view(max_rows, cols)
                     for i in range(nbufs)]
        self._region_elems = region // elem
        self._peer_views: dict = {}
        # multicast address = multicast base + offset of the local address in the allocation
        self.mc_base = self.handle.multicast_ptr - self.handle.buffer_ptrs[self.rank]
        self.flag = raw.data_ptr() + nbufs * region
        raw[nbufs * region:].zero_()  # barrier counter and barrier count
        self.turn = 0
        torch.cuda.synchronize(device)
        dist.barrier(group)

    last_error: str | None = None  # why the last try_create returned None

    @classmethod
    def try_create(cls, *args, **kwargs):
        """The reducer, or None when the group has no multicast support."""
        try:
            return cls(*args, **kwargs)
        except Exception as exc:  # no symmetric memory / no NVLS on this node
            cls.last_error = f"{type(exc).__name__}: {exc}"
            return None

    def next_buffer(self, rows: int):
        i = self.turn
        self.turn = (self.turn + 1) % self.nbufs
        return i, self.bufs[i][:rows]

    def peer_ptrs(self, i: int) -> list[int]:
        """Address of buffer i in every rank's allocation (peer-mapped), by rank."""
        off = self.bufs[i].data_ptr() - self.handle.buffer_ptrs[self.rank]
        return [int(base) + off for base in self.handle.buffer_ptrs]

    def peer_view(self, r: int, i: int):
        """Buffer i of rank r's allocation as a tensor mapped into this GPU's
        address space (reads and writes cross NVLink)."""
        key = (r, i)
        if key not in self._peer_views:
            rows, cols = self.bufs[i].shape
            self._peer_views[key] = self.handle.get_buffer(r, (rows, cols), self.dtype,
                                                           storage_offset=i * self._region_elems)
        return self._peer_views[key]

    def gather_rows(self, i: int, rows: int) -> None:
        """Copies every other rank's published row block of buffer i
        (rows [r * rows / W, (r + 1) * rows / W) of rank r's copy) into the
        same rows of this rank's copy, one device-to-device copy per rank on
        the current stream: the copy engines move them over NVLink, once, and
        no SM is used. Call after the reduce-scatter that published them
        (its closing barrier orders every rank's stores before these reads);
        the rows overwritten here held this rank's partials for the other
        blocks, which every peer finished reading before that barrier."""
        mine = self.bufs[i]
        for r in range(self.world):
            if r == self.rank:
                continue
            lo, hi = shard_range(rows, r, self.world)
            mine[lo:hi].copy_(self.peer_view(r, i)[lo:hi])

    def _code(self):
        import torch

        from . import _native

        return _native.BF16 if self.dtype == torch.bfloat16 else _native.F16

    def barrier(self) -> None:
        """Cross-rank barrier on the current stream (bounded, device-side)."""
        import torch

        from . import _native

        st = _native.lib().zcutlass_nvls_barrier(self.mc_base + self.flag, self.flag, self.world,
                                                 torch.cuda.current_stream().cuda_stream)
        if st != _native.SUCCESS:
            raise RuntimeError(f"zcutlass_nvls_barrier failed: {_native.status_name(st)}")

    def reduce_scatter(self, i: int, rows: int) -> None:
        """Rank r's rows [r * rows / W, (r + 1) * rows / W) of buffer i become
        the sum over ranks, in place in its own copy (rows a multiple of W)."""
        import torch

        from . import _native

        t = self.bufs[i]
        nbytes = rows * t.shape[1] * t.element_size()
        st = _native.lib().zcutlass_nvls_reduce_scatter(
            self.mc_base + t.data_ptr(), t.data_ptr(), nbytes, self._code(), self.mc_base + self.flag, self.flag,
            self.rank, self.world, torch.cuda.current_stream().cuda_stream)
        if st != _native.SUCCESS:
            raise RuntimeError(f"zcutlass_nvls_reduce_scatter failed: {_native.status_name(st)}")

    def reduce(self, i: int, rows: int) -> None:
        import torch

        from . import _native

        t = self.bufs[i]
        nbytes = rows * t.shape[1] * t.element_size()
        st = _native.lib().zcutlass_nvls_allreduce(
            self.mc_base + t.data_ptr(), nbytes, _native.BF16 if self.dtype == torch.bfloat16 else _native.F16,
            self.mc_base + self.flag, self.flag, self.rank, self.world, torch.cuda.current_stream().cuda_stream)
        if st != _native.SUCCESS:
            raise RuntimeError(f"zcutlass_nvls_allreduce failed: {_native.status_name(st)}")


class RowParallelLinear:
    """y = all_reduce_sum(x_shard @ W_shard^T) + b; W_shard = W[:, cols owned by this rank].

    The bias is added once, by rank 0's partial, so the all-reduced sum carries
    it exactly once. Over NCCL, `chunks` row blocks let the all-reduce of one
    block overlap the GEMM of the next. With enable_nvls() the partial goes
    into symmetric memory and the library's NVLS all-reduce sums it in place;
    each `lane` (a stream that runs its own chain of layers concurrently with
    the others) then has its own buffers and barrier word."""

    def __init__(self, weight_shard, bias=None, tp: TPGroup | None = None, chunks: int = 4,
                 linear_fn=None) -> None:
        self.weight = weight_shard
        self.bias = bias
        self.tp = tp or TPGroup()
        self.chunks = max(1, chunks)
        self.linear_fn = linear_fn or _linear_into
        self.nvls_lanes: list[NvlsReducer] = []  # set by enable_nvls()

    @property
    def nvls(self) -> "NvlsReducer | None":
        return self.nvls_lanes[0] if self.nvls_lanes else None

    def enable_nvls(self, max_rows: int, lanes: int = 1) -> bool:
        """Switch the all-reduce from NCCL to the library's NVLS kernel (if the
        group supports multicast), with `lanes` independent buffer sets of
        `max_rows` rows; returns whether it is active."""
        import torch
        import torch.distributed as dist

        if self.tp.world_size > 1 and len(self.nvls_lanes) < lanes:
            made = [NvlsReducer.try_create(max_rows, self.weight.shape[0], self.weight.dtype,
                                           self.weight.device, self.tp.group)
                    for _ in range(lanes - len(self.nvls_lanes))]
            # every rank must take the same path: use NVLS only if all ranks have it
            ok = torch.tensor([0 if any(r is None for r in made) else 1], device=self.weight.device,
                              dtype=torch.int32)
            dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=self.tp.group)
            if int(ok.item()) == 1:
                self.nvls_lanes.extend(made)
        return len(self.nvls_lanes) >= lanes

    def partial(self, x_shard, out) -> None:
        """This rank's un-reduced term x_shard @ W_shard^T (+ bias on rank 0) into out."""
        self.linear_fn(x_shard, self.weight, self.bias if self.tp.rank == 0 else None, out)

    @classmethod
    def from_full(cls, weight, bias=None, tp: TPGroup | None = None, chunks: int = 4,
                  linear_fn=None) -> "RowParallelLinear":
        tp = tp or TPGroup()
        lo, hi = shard_range(weight.shape[1], tp.rank, tp.world_size)
        return cls(weight[:, lo:hi].contiguous(), bias, tp, chunks, linear_fn)

    def forward(self, x_shard, out=None, lane: int = 0):
        """The all-reduced output. With NVLS and no `out` it is a view of the
        lane's symmetric buffer, valid until the lane's second-next call."""
        import torch
        import torch.distributed as dist

        m = x_shard.shape[0]
        bias = self.bias if self.tp.rank == 0 else None
        if self.nvls_lanes and self.tp.world_size > 1:
            red = self.nvls_lanes[lane]
            # partial into local symmetric memory, then the NVLS all-reduce in place
            i, y = red.next_buffer(m)
            self.linear_fn(x_shard, self.weight, bias, y)
            red.reduce(i, m)
            if out is not None:
                out.copy_(y)
                return out
            return y
        if out is None:
            out = torch.empty(m, self.weight.shape[0], device=x_shard.device, dtype=x_shard.dtype)
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
        self.sp_inputs: list[NvlsReducer] = []  # set by enable_sequence_parallel()
        # How qkv / gate_up see the other ranks' rows in the sequence-parallel
        # step: "copy" brings each peer row block into local memory once (copy
        # engines) and runs the plain GEMM; "fused" reads them inside the GEMM
        # (zcutlass_gemm_gather_a), which re-reads each remote A tile once per
        # N tile.
        self.sp_gather = "copy"

    def enable_nvls(self, max_tokens: int, lanes: int = 1) -> bool:
        """Use the library's NVLS all-reduce for both row-parallel linears."""
        return self.o_proj.enable_nvls(max_tokens, lanes) and self.down.enable_nvls(max_tokens, lanes)

    def enable_sequence_parallel(self, max_tokens: int, lanes: int = 1) -> bool:
        """Symmetric buffers for forward_sp: the NVLS lanes of the row-parallel
        linears plus, per lane, three rotating input buffers. Returns whether
        every rank has them (else the all-reduce path stays in use)."""
        import torch
        import torch.distributed as dist

        if self.tp.world_size < 2 or not self.enable_nvls(max_tokens, lanes):
            return False
        dev, dt = self.qkv.weight.device, self.qkv.weight.dtype
        made = [NvlsReducer.try_create(max_tokens, self.shape.hidden, dt, dev, self.tp.group, nbufs=3)
                for _ in range(lanes)]
        ok = torch.tensor([0 if any(r is None for r in made) else 1], device=dev, dtype=torch.int32)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=self.tp.group)
        self.sp_inputs = made if int(ok.item()) == 1 else []
        return bool(self.sp_inputs)

    def _sp_steps(self, rows: int, lane: int, xi: int, events: dict | None):
        """The sequence-parallel chain of one block of `rows` tokens, as two
        callables (through o_proj's reduce-scatter, then the rest). Rank r owns
        rows [r * rows / W, (r + 1) * rows / W) of the block: its input rows
        sit in buffer xi of the lane's input set, and it ends with the same
        rows of the down output (the sum over ranks). qkv and gate_up get the
        other ranks' rows as `sp_gather` says (copied into this rank's buffer,
        or read from the owners' buffers inside the GEMM); o_proj and down end
        in an NVLS reduce-scatter."""
        b = self.buffers(rows, self.qkv.weight.device, self.qkv.weight.dtype, lane)
        x_in = self.sp_inputs[lane]
        state = {}

        def timed(name, fn):
            if events is not None and name in events:
                events[name][0].record()
                r = fn()
                events[name][1].record()
                return r
            return fn()

        def o_proj():
            red = self.o_proj.nvls_lanes[lane]
            i, y = red.next_buffer(rows)
            self.o_proj.partial(b["qkv"][:, : self.o_cols], y)
            red.reduce_scatter(i, rows)
            state["o"] = (red, i)

        def down():
            red = self.down.nvls_lanes[lane]
            i, y = red.next_buffer(rows)
            self.down.partial(b["gate_up"][:, : self.d_cols], y)
            red.reduce_scatter(i, rows)
            state["y"] = y

        def gathered(col: ColumnParallelLinear, red: NvlsReducer, i: int, out):
            if self.sp_gather == "fused":
                col.forward_gathered(red.peer_ptrs(i), rows, out)
            else:
                red.gather_rows(i, rows)
                col.forward(red.bufs[i][:rows], out=out)

        def first():
            timed("qkv", lambda: gathered(self.qkv, x_in, xi, b["qkv"]))
            timed("o_proj", o_proj)

        def second():
            red, i = state["o"]
            timed("gate_up", lambda: gathered(self.gate_up, red, i, b["gate_up"]))
            timed("down", down)

        return first, second, state

    def forward_sp(self, rows: int, xi: int = 0, events: dict | None = None):
        """Sequence-parallel layer step on lane 0 (see _sp_steps); returns the
        lane's down buffer, whose rows of this rank hold the result."""
        first, second, state = self._sp_steps(rows, 0, xi, events)
        first()
        second()
        return state["y"]

    def forward_sp_overlapped(self, rows: int, streams, xi: int = 0):
        """forward_sp over len(streams) lanes, each a block of `rows` tokens in
        its own input set, issued interleaved on their own streams."""
        import torch

        cur = torch.cuda.current_stream(self.qkv.weight.device)
        chains = [self._sp_steps(rows, j, xi, None) for j in range(len(streams))]
        for s in streams:
            s.wait_stream(cur)
        for phase in (0, 1):
            for j, s in enumerate(streams):
                with torch.cuda.stream(s):
                    chains[j][phase]()
        for s in streams:
            cur.wait_stream(s)
        return [c[2]["y"] for c in chains]

    def flops_per_rank(self, tokens: int) -> float:
        q = self.qkv.weight.shape[0] * self.qkv.weight.shape[1]
        gu = self.gate_up.weight.shape[0] * self.gate_up.weight.shape[1]
        o = self.o_proj.weight.shape[0] * self.o_proj.weight.shape[1]
        d = self.down.weight.shape[0] * self.down.weight.shape[1]
        return 2.0 * tokens * (q + gu + o + d)

    def buffers(self, tokens: int, device, dtype, lane: int = 0) -> dict:
        import torch

        key = (tokens, str(device), dtype, lane)
        if key not in self._bufs:
            e = lambda *s: torch.empty(*s, device=device, dtype=dtype)  # noqa: E731
            self._bufs[key] = {
                "qkv": e(tokens, self.qkv.weight.shape[0]),
                "gate_up": e(tokens, self.gate_up.weight.shape[0]),
                "o": e(tokens, self.shape.hidden),
                "down": e(tokens, self.shape.hidden),
            }
        return self._bufs[key]

    def _steps(self, x, lane: int, out, events: dict | None):
        """The chain for one block of tokens, as two callables: up to and
        including o_proj's all-reduce, then gate_up, down and its all-reduce."""
        b = self.buffers(x.shape[0], x.device, x.dtype, lane)
        state = {}

        def timed(name, fn):
            if events is not None and name in events:
                events[name][0].record()
                r = fn()
                events[name][1].record()
                return r
            return fn()

        def first():
            timed("qkv", lambda: self.qkv(x, b["qkv"]))
            # o_proj input: this rank's heads of the attention output, stood in by the q part of qkv
            o_in = b["qkv"][:, : self.o_cols]
            # with NVLS the row-parallel outputs stay in their symmetric buffers (no copy)
            state["o"] = timed("o_proj", lambda: self.o_proj(o_in, None if self.o_proj.nvls else b["o"], lane))

        def second():
            # gate_up consumes the all-reduced o_proj output (the residual + norm step is left out)
            timed("gate_up", lambda: self.gate_up(state["o"], b["gate_up"]))
            # down input: this rank's slice of act(gate) * up, stood in by the gate_up output
            d_in = b["gate_up"][:, : self.d_cols]
            dst = out if out is not None or self.down.nvls is not None else b["down"]
            state["y"] = timed("down", lambda: self.down(d_in, dst, lane))

        return first, second, state

    def forward(self, x, events: dict | None = None, out=None):
        """x: [tokens, hidden] (replicated on every rank). Runs the four GEMMs in
        a decoder layer's dependency order -- qkv, o_proj (+ all-reduce), gate_up
        on the o_proj output, down (+ all-reduce) -- and returns the down output
        (written into `out` when given). `events` (optional) maps a GEMM name to
        a (start, end) CUDA event pair recorded around that GEMM on the current stream."""
        first, second, state = self._steps(x, 0, out, events)
        first()
        second()
        return state["y"]

    def forward_overlapped(self, x, streams, outs=None):
        """The same layer over len(streams) independent blocks of rows of x (as
        from different sequences), each block's chain on its own stream and
        NVLS lane, issued interleaved so one block's all-reduce overlaps the
        next block's GEMMs. Returns the per-block down outputs (row blocks of
        x in order); `outs` optionally gives their destinations."""
        import torch

        n = len(streams)
        cur = torch.cuda.current_stream(x.device)
        chains = []
        for j in range(n):
            r0, r1 = shard_range(x.shape[0], j, n)
            chains.append(self._steps(x[r0:r1], j, None if outs is None else outs[j], None))
        for s in streams:
            s.wait_stream(cur)
        for phase in (0, 1):
            for j, s in enumerate(streams):
                with torch.cuda.stream(s):
                    chains[j][phase]()
        for s in streams:
            cur.wait_stream(s)
        return [c[2]["y"] for c in chains]

    def forward_overlapped_layers(self, x, streams, layers: int, outs=None):
        """`layers` consecutive layer steps over len(streams) independent row
        blocks, as a stack of decoder layers runs them: each block's chain of
        layers on its own stream and NVLS lane, the blocks joined only at the
        end, so block j's next layer can start while block j + 1 is still in
        the previous layer's all-reduce. Every layer step does the same work as
        forward_overlapped (the input of each layer is x: the linears stand in
        for whole layers). Returns the last layer's per-block outputs."""
        import torch

        n = len(streams)
        cur = torch.cuda.current_stream(x.device)
        for s in streams:
            s.wait_stream(cur)
        chains = []
        for _ in range(layers):
            chains = []
            for j in range(n):
                r0, r1 = shard_range(x.shape[0], j, n)
                chains.append(self._steps(x[r0:r1], j, None if outs is None else outs[j], None))
            for phase in (0, 1):
                for j, s in enumerate(streams):
                    with torch.cuda.stream(s):
                        chains[j][phase]()
        for s in streams:
            cur.wait_stream(s)
        return [c[2]["y"] for c in chains]
