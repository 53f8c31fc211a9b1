"""Tensor-parallel QwQ-32B decoder-layer linear stack on W4A8 linears.

Per layer (the reference's fused-layer benchmark, npu_ops/python/bench_fused_layer.py:63-66;
vLLM's Column/RowParallelLinear sharding):

    qkv     column-parallel  [M, H]      -> [M, QKV/tp]  (q, k and v sections each split, as
                                                         vLLM's QKVParallelLinear does)
    att     the rank's q section, H/tp columns (an attention stand-in: the stack has no
            attention; with per-section shards it is the same map at every tp)
    o_proj  row-parallel     [M, H/tp]   -> [M, H] partial   -> all-reduce
    gate_up column-parallel  [M, H]      -> [M, 2F/tp]  ([gate_shard; up_shard] rows, vLLM's
                                                         MergedColumnParallelLinear order)
    act     silu(gate) * up              -> [M, F/tp]
    down    row-parallel     [M, F/tp]   -> [M, H] partial   -> all-reduce

Row-parallel shards split K at group boundaries (H/tp and F/tp are multiples of the group
size for every tp <= 8 at GK = 128), so each rank's scales are the [G/tp, N] slice.  All
ranks draw the full weights from the same seed and keep their shard, so any tp gives the
same layer as tp = 1 up to the order of the bf16 all-reduce.

The forward takes the linear and all-reduce as callables: the product uses the CUDA op on
prepared weights and NCCL; the CPU tests pass reference arithmetic and gloo.
"""
from __future__ import annotations

import dataclasses
from typing import Callable, Dict, List, Optional, Sequence

import torch

GK = 128


@dataclasses.dataclass(frozen=True)
class Dims:
    hidden: int = 5120
    qkv: int = 7168
    ffn: int = 27648
    gk: int = GK


QWQ = Dims()


@dataclasses.dataclass
class ShardWeights:
    """One linear's shard: int8 codes [N, K] (kept for checking), the packed layout and scales."""
    codes: torch.Tensor
    packed: torch.Tensor
    scale: torch.Tensor        # [G, N] fp32
    K: int
    N: int
    prepared: Optional[object] = None


@dataclasses.dataclass
class LayerShard:
    qkv: ShardWeights
    o: ShardWeights
    gate_up: ShardWeights
    down: ShardWeights


def check_dims(d: Dims, tp: int) -> None:
    for name, k in (("hidden", d.hidden), ("ffn", d.ffn)):
        if k % (tp * d.gk):
            raise ValueError(f"{name}={k} does not split into {tp} group-aligned shards of GK={d.gk}")
    for name, n in (("qkv", d.qkv), ("ffn", d.ffn)):
        if n % (tp * 8):
            raise ValueError(f"{name}={n} does not split into {tp} output shards of a multiple of 8")
    kv = (d.qkv - d.hidden) // 2
    if d.qkv <= d.hidden or (d.qkv - d.hidden) % 2 or kv % (tp * 8):
        raise ValueError(f"qkv={d.qkv} is not q={d.hidden} plus two kv sections that split {tp} ways")


def _full(N: int, K: int, gk: int, gen: torch.Generator, device):
    G = -(-K // gk)
    codes = torch.randint(-8, 8, (N, K), generator=gen, device=device, dtype=torch.int16).to(torch.int8)
    scale = torch.exp(torch.randn(G, N, generator=gen, device=device) * 0.5 - 6.0)
    return codes, scale


def _make(codes: torch.Tensor, scale: torch.Tensor, gk: int, device) -> ShardWeights:
    from . import ops
    codes = codes.to(device).contiguous()
    scale = scale.to(device)
    return ShardWeights(codes=codes, packed=ops.pack_int4_grouped(codes, gk), scale=scale.contiguous(),
                        K=codes.shape[1], N=codes.shape[0])


def column_shard(codes: torch.Tensor, scale: torch.Tensor, rank: int, tp: int):
    """Rows [rank*N/tp, (rank+1)*N/tp) of the output dimension."""
    n = codes.shape[0] // tp
    return codes[rank * n:(rank + 1) * n], scale[:, rank * n:(rank + 1) * n]


def sections_shard(codes: torch.Tensor, scale: torch.Tensor, rank: int, tp: int, sizes: Sequence[int]):
    """The rank's rows of each output section, concatenated in section order (vLLM's
    MergedColumnParallelLinear [gate; up] and QKVParallelLinear [q; k; v])."""
    cs, ss, n0 = [], [], 0
    for n in sizes:
        c, sc = column_shard(codes[n0:n0 + n], scale[:, n0:n0 + n], rank, tp)
        cs.append(c)
        ss.append(sc)
        n0 += n
    return torch.cat(cs, 0), torch.cat(ss, 1)


def merged_column_shard(codes: torch.Tensor, scale: torch.Tensor, rank: int, tp: int):
    """[gate_shard; up_shard] of a [gate; up] weight."""
    f = codes.shape[0] // 2
    return sections_shard(codes, scale, rank, tp, (f, f))


def qkv_shard(codes: torch.Tensor, scale: torch.Tensor, rank: int, tp: int, hidden: int):
    """[q_shard; k_shard; v_shard] of a [q; k; v] weight with q = hidden rows."""
    kv = (codes.shape[0] - hidden) // 2
    return sections_shard(codes, scale, rank, tp, (hidden, kv, kv))


def row_shard(codes: torch.Tensor, scale: torch.Tensor, rank: int, tp: int, gk: int):
    """Columns [rank*K/tp, (rank+1)*K/tp) of the input dimension and their scale groups."""
    k = codes.shape[1] // tp
    g = k // gk
    return codes[:, rank * k:(rank + 1) * k], scale[rank * g:(rank + 1) * g]


def build_layers(n_layers: int, rank: int, tp: int, device, d: Dims = QWQ, seed: int = 1234,
                 prepare: bool = False, gen_device=None) -> List[LayerShard]:
    """Each rank draws the full layer weights from `seed` and keeps its shard.

    The draw happens on `gen_device` (default `device`): torch's CPU and CUDA
    generators give different streams, so ranks must draw on the same kind of
    device to hold shards of one layer."""
    check_dims(d, tp)
    out = []
    gdev = device if gen_device is None else gen_device
    gen = torch.Generator(device=gdev).manual_seed(seed)
    for _ in range(n_layers):
        qkv_c, qkv_s = _full(d.qkv, d.hidden, d.gk, gen, gdev)
        o_c, o_s = _full(d.hidden, d.hidden, d.gk, gen, gdev)
        gu_c, gu_s = _full(2 * d.ffn, d.hidden, d.gk, gen, gdev)
        dn_c, dn_s = _full(d.hidden, d.ffn, d.gk, gen, gdev)
        L = LayerShard(qkv=_make(*qkv_shard(qkv_c, qkv_s, rank, tp, d.hidden), d.gk, device),
                       o=_make(*row_shard(o_c, o_s, rank, tp, d.gk), d.gk, device),
                       gate_up=_make(*merged_column_shard(gu_c, gu_s, rank, tp), d.gk, device),
                       down=_make(*row_shard(dn_c, dn_s, rank, tp, d.gk), d.gk, device))
        del qkv_c, o_c, gu_c, dn_c
        if prepare:
            from . import ops
            for w in (L.qkv, L.o, L.gate_up, L.down):
                w.prepared = ops.prepare_weights(w.packed, w.scale, None, w.K, d.gk)
        out.append(L)
    return out


Linear = Callable[[torch.Tensor, ShardWeights], torch.Tensor]
AllReduce = Callable[[torch.Tensor], None]
# gu [M, 2f] = [gate | up] -> linear(bf16(silu(gate) * up), w): the down projection
# with the activation function applied to its input
SwigluLinear = Callable[[torch.Tensor, ShardWeights], torch.Tensor]


def swiglu(gu: torch.Tensor) -> torch.Tensor:
    """bf16(silu(gate) * up) in fp32 for gu = [gate | up] (the stack's activation)."""
    f = gu.shape[-1] // 2
    return (torch.nn.functional.silu(gu[..., :f].float()) * gu[..., f:].float()).to(torch.bfloat16)


def composed_swiglu_linear(linear: Linear) -> SwigluLinear:
    """The activation as its own step, then the linear (the CPU tests' form)."""
    return lambda gu, w: linear(swiglu(gu), w)


def cuda_linear(x: torch.Tensor, w: ShardWeights) -> torch.Tensor:
    from . import ops
    if w.prepared is not None:
        return ops.linear_prepared(x, w.prepared)
    return ops.linear(x, w.packed, w.scale, None, GK)


def cuda_swiglu_linear(gu: torch.Tensor, w: ShardWeights) -> torch.Tensor:
    """The down projection with silu(gate) * up computed by the op's activation
    quantiser as it reads gu: no elementwise kernels and no [M, f] activation
    tensor between gate_up and down."""
    from . import ops
    if w.prepared is not None:
        return ops.linear_prepared(gu, w.prepared, act="swiglu")
    return ops.linear(gu, w.packed, w.scale, None, GK, act="swiglu")


# (x, w, act) -> the all-reduced output of a row-parallel linear; act None or "swiglu"
RowLinear = Callable[[torch.Tensor, ShardWeights, Optional[str]], torch.Tensor]


def composed_row_linear(linear: Linear, swiglu_linear: SwigluLinear, allreduce: AllReduce) -> RowLinear:
    """The row-parallel linear, then the all-reduce as its own step."""
    def f(x, w, act=None):
        y = swiglu_linear(x, w) if act == "swiglu" else linear(x, w)
        allreduce(y)
        return y
    return f


def fused_row_linear(car) -> RowLinear:
    """The row-parallel linear fused with the one-shot all-reduce
    (``CustomAllReduce.linear_prepared``) on prepared weights."""
    return lambda x, w, act=None: car.linear_prepared(x, w.prepared, act=act)


def layer_forward(h: torch.Tensor, L: LayerShard, tp: int, linear: Linear, allreduce: AllReduce,
                  d: Dims = QWQ, swiglu_linear: Optional[SwigluLinear] = None,
                  row_linear: Optional[RowLinear] = None) -> torch.Tensor:
    swiglu_linear = swiglu_linear or composed_swiglu_linear(linear)
    row_linear = row_linear or composed_row_linear(linear, swiglu_linear, allreduce)
    qkv = linear(h, L.qkv)
    att = qkv[:, : d.hidden // tp]                     # attention stand-in: the rank's q section
    o = row_linear(att, L.o, None)
    gu = linear(o, L.gate_up)
    return row_linear(gu, L.down, "swiglu")


def stack_forward(h: torch.Tensor, layers: Sequence[LayerShard], tp: int, linear: Linear,
                  allreduce: AllReduce, d: Dims = QWQ, swiglu_linear: Optional[SwigluLinear] = None,
                  row_linear: Optional[RowLinear] = None) -> torch.Tensor:
    for L in layers:
        h = layer_forward(h, L, tp, linear, allreduce, d, swiglu_linear, row_linear)
    return h


def _sum_bf16(parts: Sequence[torch.Tensor]) -> torch.Tensor:
    """fp32 sum in rank order, rounded once to bf16: the one-shot all-reduce's arithmetic."""
    acc = parts[0].float()
    for p in parts[1:]:
        acc = acc + p.float()
    return acc.to(torch.bfloat16)


def emulated_stack_forward(h: torch.Tensor, ranks: Sequence[Sequence[LayerShard]], linear: Linear,
                           d: Dims = QWQ, swiglu_linear: Optional[SwigluLinear] = None) -> torch.Tensor:
    """The tp-way sharded stack with every rank's shard on one device: the ranks
    run each layer in lockstep and each all-reduce is the fp32 rank-order sum
    of their partial outputs.  The same sharding and per-rank linears as the
    multi-process stack, so it checks the tensor-parallel arithmetic at TP
    shapes on one GPU."""
    tp = len(ranks)
    swiglu_linear = swiglu_linear or composed_swiglu_linear(linear)
    for li in range(len(ranks[0])):
        Ls = [r[li] for r in ranks]
        att = [linear(h, L.qkv)[:, : d.hidden // tp] for L in Ls]
        o = _sum_bf16([linear(a, L.o) for a, L in zip(att, Ls)])
        h = _sum_bf16([swiglu_linear(linear(o, L.gate_up), L.down) for L in Ls])
    return h


def nccl_allreduce(group=None) -> AllReduce:
    import torch.distributed as dist

    def f(t: torch.Tensor) -> None:
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return f


def _roofline_seconds(layers: Sequence[LayerShard], M: int, hbm_gbs: float, i8_tops: Optional[float]) -> float:
    """Per-rank lower bound: each GEMM at the slower of its HBM and int8 bounds."""
    t = 0.0
    for L in layers:
        for w in (L.qkv, L.o, L.gate_up, L.down):
            G = -(-w.K // GK)
            by = w.N * w.K // 2 + G * w.N * 4 + M * w.K * 2 + M * w.N * 2
            t_mem = by / (hbm_gbs * 1e9)
            t_ops = 2.0 * M * w.N * w.K / (i8_tops * 1e12) if i8_tops else 0.0
            t += max(t_mem, t_ops)
    return t


def custom_allreduce(group=None, max_bytes: Optional[int] = None):
    """The one-shot peer-memory all-reduce (``allreduce.CustomAllReduce``) for
    messages up to ``max_bytes`` (default: M = 64 rows of hidden 5120), NCCL
    beyond."""
    from .allreduce import DEFAULT_MAX_BYTES, CustomAllReduce
    return CustomAllReduce(group=group, max_bytes=max_bytes or DEFAULT_MAX_BYTES)


def bench_stack(world: int, rank: int, dev, ms=(16, 256, 4096), layers: int = 4, iters: int = 10,
                hbm_gbs: float = 6556.5, i8_tops: Optional[float] = None,
                allreduces: Sequence[str] = ("nccl",), parity: bool = True) -> Dict:
    """Time `layers` sharded layers at each M on `world` GPUs (one rank each).

    The step is captured in a CUDA graph (the all-reduces included); the time is
    the max over ranks of CUDA-event time per forward.  Returns tokens/s (M per
    forward) and layer-tokens/s (M x layers per forward) with the roofline
    fraction, per all-reduce (``nccl``; ``custom``: the one-shot kernel for
    small messages, NCCL for the rest; ``fused``: the row-parallel linears fused
    with the one-shot all-reduce, ``custom`` beyond its message limit).

    With ``parity`` and world > 1, each mode also runs one sharded layer and
    rank 0 compares its output with the unsharded layer (tp = 1, the same
    seeded weights and input) at the stack bound (max rel <= 3e-2, cosine >=
    0.9995), and every rank's bits of the timed stack's output are compared.
    One layer, because the stack has no normalisation: SiLU(gate) * up roughly
    squares the magnitude of each layer's input, and random weights take four
    layers past the bf16 range."""
    d = QWQ
    Ls = build_layers(layers, rank, world, dev, d, prepare=True)
    out = {"tp": world, "layers": layers, "dims": dataclasses.asdict(d),
           "note": "attention replaced by the rank's q section of the QKV output; the down projection "
                   "applies silu(gate)*up in its activation quantiser"}
    ref = {}
    if parity and world > 1 and rank == 0:
        L1 = build_layers(1, 0, 1, dev, d, prepare=True)
        for M in ms:
            ref[M] = stack_forward(_stack_input(M, d, dev), L1, 1, cuda_linear, lambda t: None, d,
                                   cuda_swiglu_linear).float()
        del L1
    per = []
    from . import _lib
    for mode in allreduces if world > 1 else ("none",):
        car, row = None, None
        if world == 1:
            ar = (lambda t: None)
        elif mode in ("custom", "fused", "fused_push"):
            car = custom_allreduce()
            ar = car
            if mode != "custom":
                row = fused_row_linear(car)
        else:
            ar = nccl_allreduce()
        # fused_push: the epilogue stores into every rank's slot (W4A8_OPT_AR_PUSH)
        old_opt = _lib.lib().w4a8_set_options(_lib.OPT_AR_PUSH) if mode == "fused_push" else None
        try:
            key = "per_M" if mode in ("nccl", "none") else f"per_M_{mode}"
            out[key], outs = _time_stack(world, dev, Ls, ms, iters, ar, d, hbm_gbs, i8_tops, row)
            if parity and world > 1:
                per += _stack_parity(world, rank, dev, Ls[:1], ms, d, ar, row, mode, outs, ref)
        finally:
            if old_opt is not None:
                _lib.lib().w4a8_set_options(old_opt)
        if car is not None:
            car.check()
            if mode == "fused":
                out["fused_calls"] = car.calls_fused
            car.close()
    if per:
        out["tp_parity"] = {"bound": {"max_rel": 3e-2, "cos": 0.9995}, "layers_compared": 1, "per": per,
                            "ok": all(r.get("ok", True) for r in per)}
    return out


def _stack_parity(world, rank, dev, L1, ms, d, ar, row, mode, outs, ref) -> List[Dict]:
    import torch.distributed as dist
    res = []
    for M in ms:
        y = stack_forward(_stack_input(M, d, dev), L1, world, cuda_linear, ar, d, cuda_swiglu_linear, row)
        # every rank's bits of the 1-layer output and of the timed stack's output
        sums = []
        for t in (y, outs[M]):
            h = t.contiguous().view(torch.int16).to(torch.int64).sum().reshape(1)
            hs = [torch.zeros_like(h) for _ in range(world)]
            dist.all_gather(hs, h)
            sums.append(all(int(x.item()) == int(hs[0].item()) for x in hs))
        if rank == 0:
            yf, r = y.float(), ref[M]
            err = float((yf - r).abs().max() / r.abs().max())
            cos = float((yf * r).sum() / (yf.norm() * r.norm()))
            ok = err <= 3e-2 and cos >= 0.9995 and all(sums)
            res.append({"allreduce": mode, "M": M, "max_rel": err, "cos": cos, "ranks_identical": all(sums),
                        "ok": ok})
    return res


def _stack_input(M: int, d: Dims, dev) -> torch.Tensor:
    gen = torch.Generator(device=dev).manual_seed(99 + M)
    return torch.randn(M, d.hidden, generator=gen, device=dev).to(torch.bfloat16)


def _time_stack(world, dev, Ls, ms, iters, ar, d, hbm_gbs, i8_tops, row=None):
    import torch.distributed as dist
    layers = len(Ls)
    res, outs = [], {}
    for M in ms:
        h0 = _stack_input(M, d, dev)

        def fwd():
            return stack_forward(h0, Ls, world, cuda_linear, ar, d, cuda_swiglu_linear, row)

        for _ in range(2):
            fwd()
        torch.cuda.synchronize()
        graph, y = None, None
        try:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                y = fwd()
        except Exception:
            graph = None
        run = graph.replay if graph is not None else fwd
        for _ in range(2):
            run()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            run()
        e1.record()
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) * 1e-3 / iters
        if world > 1:
            tt = torch.tensor([t], device=dev, dtype=torch.float64)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t = float(tt.item())
        outs[M] = (y if graph is not None else fwd()).clone()
        roof = _roofline_seconds(Ls, M, hbm_gbs, i8_tops)
        res.append({"M": M, "ms_per_forward": 1e3 * t, "tokens_per_s": M / t,
                    "layer_tokens_per_s": M * layers / t, "roofline_frac": roof / t,
                    "graph": graph is not None})
        del graph
    return res, outs
