"""Rank body of the tensor-parallel CPU test (spawned by test_tp_cpu.py).

Runs the sharded layer stack with the reference arithmetic (the oracle) as the
linear and gloo as the all-reduce, plus the unsharded stack in the same
process, and saves both outputs for the parent to compare."""
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
for _p in (REPO, os.path.join(REPO, "vllm-ascend910_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

SMALL = dict(hidden=256, qkv=384, ffn=512, gk=128)


def oracle_linear(gk):
    import numpy as np
    import torch

    import oracle

    def f(x, w):
        xb = x.contiguous().view(torch.int16).numpy().view(np.uint16)
        y, _ = oracle.linear(xb, w.codes.numpy(), w.scale.numpy(), None, gk)
        yb = oracle.f32_to_bf16(np.asarray(y, np.float32))
        return torch.from_numpy(yb.view(np.int16).copy()).view(torch.bfloat16)
    return f


def run(rank, world, port, out_dir, layers=2, M=4):
    import numpy as np
    import torch
    import torch.distributed as dist

    from w4a8_b200 import tp

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        d = tp.Dims(**SMALL)
        lin = oracle_linear(d.gk)

        def ar(t):
            f = t.float()
            dist.all_reduce(f)
            t.copy_(f.to(torch.bfloat16))

        gen = torch.Generator().manual_seed(7)
        h = torch.randn(M, d.hidden, generator=gen).to(torch.bfloat16)
        y = tp.stack_forward(h, tp.build_layers(layers, rank, world, "cpu", d), world, lin, ar, d)
        y1 = tp.stack_forward(h, tp.build_layers(layers, 0, 1, "cpu", d), 1, lin, lambda t: None, d)
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), y=y.float().numpy(), y1=y1.float().numpy())
    finally:
        dist.destroy_process_group()
