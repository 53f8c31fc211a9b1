"""Worker for the multi-GPU custom all-reduce tests (one process per GPU).

Run as ``python tests/ar_worker.py RANK WORLD PORT MODE OUTFILE``; writes a JSON
verdict to OUTFILE.  MODE ``parity``: bit-exact sums against an fp32 rank-order
reference over many sizes, in place and in a replayed CUDA graph, plus the NCCL
fallback.  MODE ``absent``: rank 1 stays alive but skips the last call; rank 0's
wait must run out and ``check()`` must raise (no GPU fault, no hang).
"""
import datetime
import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "vllm-ascend910_b200"))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def inputs(rank, numel, step):
    g = torch.Generator().manual_seed(1000 * step + 17 * rank + numel)
    return (torch.randn(numel, generator=g) * (1 + rank)).to(torch.bfloat16)


def reference(world, numel, step):
    acc = torch.zeros(numel, dtype=torch.float32)
    for r in range(world):
        acc += inputs(r, numel, step).float()
    return acc.to(torch.bfloat16)


def main():
    rank, world, port, mode, out = int(sys.argv[1]), int(sys.argv[2]), sys.argv[3], sys.argv[4], sys.argv[5]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=port)
    if mode != "time":                       # failure paths run with NVLS off; timing compares NCCL's default
        os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    from w4a8_b200 import _lib
    from w4a8_b200.allreduce import CustomAllReduce
    verdict = {"rank": rank, "ok": True, "msgs": []}
    ar = CustomAllReduce(max_bytes=1 << 20)
    try:
        if mode == "parity":
            sizes = [8, 5120, 16 * 5120, 64 * 5120, 1000 * 8, 5120 * 3, 600 * 1024]   # last one: NCCL fallback
            for step, n in enumerate(sizes):
                t = inputs(rank, n, step).to(dev)
                ar(t)
                ok = torch.equal(t.cpu(), reference(world, n, step))
                if n * 2 > ar.max_bytes:
                    # NCCL sums in its own order with bf16 intermediates: bound the error
                    # by the magnitudes summed, not by the (possibly cancelling) result
                    mag = sum(inputs(r, n, step).float().abs() for r in range(world))
                    err = (t.cpu().float() - reference(world, n, step).float()).abs()
                    ok = bool(torch.all(err <= mag * 2.0 ** -6 + 1e-6))
                if not ok:
                    verdict["msgs"].append(["FAILED size", n])
                verdict["ok"] &= bool(ok)
            ar.check()
            # CUDA graph: three calls of different sizes captured once, replayed with new data
            bufs = [torch.empty(n, dtype=torch.bfloat16, device=dev) for n in (5120, 16 * 5120, 4096)]
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                with torch.cuda.graph(g, stream=s):
                    for b in bufs:
                        ar(b)
            torch.cuda.current_stream().wait_stream(s)
            for rep in range(4):
                for i, b in enumerate(bufs):
                    b.copy_(inputs(rank, b.numel(), 100 + 10 * rep + i).to(dev))
                g.replay()
                torch.cuda.synchronize()
                for i, b in enumerate(bufs):
                    ok = torch.equal(b.cpu(), reference(world, b.numel(), 100 + 10 * rep + i))
                    verdict["ok"] &= bool(ok)
                    if not ok:
                        verdict["msgs"].append(["FAILED graph", rep, i])
            ar.check()
            del g
            verdict["calls_custom"], verdict["calls_fallback"] = ar.calls_custom, ar.calls_fallback
            # latency at M = 16 x 5120 against NCCL
            t = torch.randn(16 * 5120, device=dev).to(torch.bfloat16)
            for name, fn in (("custom", lambda: ar(t)),
                             ("nccl", lambda: dist.all_reduce(t, op=dist.ReduceOp.SUM))):
                for _ in range(20):
                    fn()
                torch.cuda.synchronize()
                dist.barrier()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(200):
                    fn()
                e1.record()
                torch.cuda.synchronize()
                verdict[f"us_{name}_m16"] = e0.elapsed_time(e1) * 1e3 / 200
            ar.check()
        elif mode == "time":
            # per-call device time inside a CUDA graph of 50 calls, custom vs NCCL
            verdict["us"] = {}
            for rows in (1, 16, 64):
                t = torch.randn(rows * 5120, device=dev).to(torch.bfloat16)
                for name in ("custom", "nccl"):
                    fn = (lambda: ar(t)) if name == "custom" else (lambda: dist.all_reduce(t, op=dist.ReduceOp.SUM))
                    for _ in range(3):
                        fn()
                    torch.cuda.synchronize()
                    g = torch.cuda.CUDAGraph()
                    s = torch.cuda.Stream()
                    s.wait_stream(torch.cuda.current_stream())
                    with torch.cuda.stream(s):
                        with torch.cuda.graph(g, stream=s):
                            for _ in range(50):
                                fn()
                    torch.cuda.current_stream().wait_stream(s)
                    g.replay()
                    torch.cuda.synchronize()
                    dist.barrier()
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record()
                    for _ in range(5):
                        g.replay()
                    e1.record()
                    torch.cuda.synchronize()
                    verdict["us"][f"{name}_m{rows}"] = e0.elapsed_time(e1) * 1e3 / 250
                    del g
            ar.check()
        elif mode == "absent":
            t = inputs(rank, 5120, 0).to(dev)
            ar(t)
            ar.check()
            dist.barrier()
            if rank == 0:
                t2 = inputs(rank, 5120, 1).to(dev)
                before = t2.clone()
                ar(t2)                                  # rank 1 never joins this call
                try:
                    ar.check()
                    verdict["ok"] = False
                    verdict["msgs"].append("no timeout reported")
                except _lib.W4A8Error as e:
                    verdict["msgs"].append(str(e))
                    verdict["ok"] &= torch.equal(t2.cpu(), before.cpu())   # output left untouched
            dist.barrier()                              # rank 1 stays alive until rank 0 is done
    except Exception as e:  # noqa: BLE001
        verdict["ok"] = False
        verdict["msgs"].append(repr(e))
    finally:
        ar.close()
        dist.destroy_process_group()
        json.dump(verdict, open(out, "w"))


if __name__ == "__main__":
    main()
