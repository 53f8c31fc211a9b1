"""Worker for the multi-GPU custom all-reduce tests (one process per GPU).

Run as ``python tests/ar_worker.py RANK WORLD PORT MODE OUTFILE``; writes a JSON
verdict to OUTFILE.  MODE ``parity``: bit-exact sums against an fp32 rank-order
reference over many sizes, in place and in a replayed CUDA graph, plus the NCCL
fallback.  MODE ``skew``: the reference's barrier gates -- ranks desynchronised
on purpose (skewed launches, changing values, a 200-call run, graph replays,
24 live graphs) -- plus a strided and a misaligned message, which take the
staged form of the one-shot path on one rank while the other passes a dense
tensor.  MODE ``fused``: the row-parallel linear fused with the all-reduce
against the linear followed by the all-reduce, bit for bit.  MODE ``absent``: rank 1 stays alive but skips the last call; rank 0's
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


def skew_value(r, step):
    """Per-rank message value, exact in bf16 (multiples of 0.25 below 64), with
    partial sums exact in fp32: a read of last step's slot gives a visibly wrong
    sum, not a rounding difference."""
    return (r + 1) * 4.0 + (step % 16) * 0.25


def skew_gates(ar, rank, world, dev, verdict):
    """The ranks are desynchronised on purpose before the calls, so only the
    kernel's own flags keep them together (the reference's barrier gates,
    npu_ops/python/test_peer_barrier.py:1-26):
      0. one message laid out differently on different ranks (staged path);
      1. skewed launch: rank r sleeps r * 25 ms before its call;
      2. skewed with the values changing every step;
      3. 200 calls with a random skew and no host barrier, checked every step;
      4. one captured graph replayed 20 times with new values and skewed replays;
      5. 24 graphs of different sizes alive at once, replayed in order."""
    import random
    n = 16 * 5120
    x = torch.empty(n, dtype=torch.bfloat16, device=dev)

    def expect(step):
        # the kernel sums in fp32 (exact here) and rounds once to bf16
        return float(torch.tensor(sum(skew_value(r, step) for r in range(world))).to(torch.bfloat16))

    def check(t, step, what):
        ok = bool(torch.all(t == expect(step)).item())
        if not ok:
            verdict["msgs"].append([what, step, float(t.float().min()), float(t.float().max()), expect(step)])
        verdict["ok"] &= ok
        return ok

    # 0. the same message as a strided view (rank 0) / a misaligned view (rank 1)
    #    against a dense tensor elsewhere: every rank must take the one-shot path
    for step, kind in ((900, "strided"), (901, "misaligned")):
        ref_t = reference(world, n, step)
        dense = inputs(rank, n, step).to(dev)
        if rank == 0 and kind == "strided":
            big = torch.zeros(n, 2, dtype=torch.bfloat16, device=dev)
            big[:, 0] = dense
            t = big[:, 0]
        elif rank == 1 and kind == "misaligned":
            raw = torch.zeros(n + 1, dtype=torch.bfloat16, device=dev)
            t = raw[1:]
            t.copy_(dense)
        else:
            t = dense
        before = ar.calls_custom
        ar(t)
        ok = torch.equal(t.cpu(), ref_t) and ar.calls_custom == before + 1
        if not ok:
            verdict["msgs"].append(["layout", kind])
        verdict["ok"] &= bool(ok)
    ar.check()
    # 1. skewed launch
    x.fill_(skew_value(rank, 1))
    dist.barrier()
    time.sleep(0.025 * rank)
    ar(x)
    torch.cuda.synchronize()
    check(x, 1, "skewed launch")
    # 2. skewed, values change every step
    for step in range(2, 12):
        x.fill_(skew_value(rank, step))
        dist.barrier()
        time.sleep(0.01 * ((rank + step) % world))
        ar(x)
        torch.cuda.synchronize()
        check(x, step, "skewed changing values")
    # 3. 200 calls, random skew, no host barrier; a full random message every 10th
    rng = random.Random(1234 + rank)
    bad = 0
    for step in range(12, 212):
        if step % 10 == 0:
            t = inputs(rank, n, step).to(dev)
            if rng.random() < 0.3:
                time.sleep(rng.random() * 0.005)
            ar(t)
            if not torch.equal(t.cpu(), reference(world, n, step)):
                bad += 1
            continue
        x.fill_(skew_value(rank, step))
        if rng.random() < 0.1:
            time.sleep(rng.random() * 0.005)
        ar(x)
        torch.cuda.synchronize()
        if not bool(torch.all(x == expect(step)).item()):
            bad += 1
    if bad:
        verdict["ok"] = False
        verdict["msgs"].append(["long skewed run: wrong steps", bad])
    verdict["skew_long_steps"] = 200
    ar.check()
    # 4. one graph, 20 replays, new values each time, skewed replays
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    x.fill_(skew_value(rank, 0))
    torch.cuda.synchronize()
    dist.barrier()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            ar(x)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    dist.barrier()
    for rep in range(20):
        step = 300 + rep
        x.fill_(skew_value(rank, step))
        torch.cuda.synchronize()
        time.sleep(0.005 * ((rank + rep) % world))
        g.replay()
        torch.cuda.synchronize()
        check(x, step, "graph replay")
    del g
    ar.check()
    # 5. 24 graphs of different sizes alive, replayed in order
    sizes = [16 * (i + 1) for i in range(4)] + [512, 1024, 2048, 2560, 5120]
    sizes = (sizes * 3)[:24]
    bufs, graphs = [], []
    for m in sizes:
        b = torch.full((m,), skew_value(rank, 0), dtype=torch.bfloat16, device=dev)
        ar(b)                                   # warm the size before capturing it
        torch.cuda.synchronize()
        dist.barrier()
        gi = torch.cuda.CUDAGraph()
        si = torch.cuda.Stream()
        si.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(si):
            with torch.cuda.graph(gi, stream=si):
                ar(b)
        torch.cuda.current_stream().wait_stream(si)
        bufs.append(b)                          # a graph replays against the captured address
        graphs.append(gi)
    torch.cuda.synchronize()
    for rnd in range(2):
        for i, (b, gi) in enumerate(zip(bufs, graphs)):
            step = 400 + 30 * rnd + i
            b.fill_(skew_value(rank, step))
            torch.cuda.synchronize()
            dist.barrier()
            gi.replay()
            torch.cuda.synchronize()
            check(b, step, f"graph {i} of {len(graphs)} alive")
    del graphs
    ar.check()
    verdict["calls_custom"], verdict["calls_fallback"] = ar.calls_custom, ar.calls_fallback


def fused_gates(ar, rank, world, dev, verdict):
    """Row-parallel shards of one seeded layer (each rank holds K/world columns):
    the fused linear + all-reduce against the linear followed by the one-shot
    all-reduce, bit for bit, for plain and SwiGLU inputs, several M (one beyond
    the message limit, NCCL), and replays of a captured graph with new inputs;
    with the epilogue storing into its own slot (peers read it, the default)
    and into every rank's slot (W4A8_OPT_AR_PUSH)."""
    from w4a8_b200 import _lib
    for opt in (0, _lib.OPT_AR_PUSH):
        old = _lib.lib().w4a8_set_options(opt)
        try:
            _fused_cases(ar, rank, world, dev, verdict, "push" if opt else "pull")
        finally:
            _lib.lib().w4a8_set_options(old)
    verdict["calls_fused"] = ar.calls_fused


def _fused_cases(ar, rank, world, dev, verdict, variant):
    from w4a8_b200 import ops, tp
    from w4a8_b200 import synthetic as syn
    gk = 128
    cases = [(5120, 5120, None), (5120, 27648, "swiglu")]      # (N, full K, act): o_proj, down
    ok = True
    for N, Kf, act in cases:
        g = torch.Generator(device=dev).manual_seed(1234 + N + Kf)
        codes = torch.randint(-8, 8, (N, Kf), generator=g, device=dev, dtype=torch.int16).to(torch.int8)
        scale = torch.exp(torch.randn(Kf // gk, N, generator=g, device=dev) * 0.5 - 6.0)
        c, sc = tp.row_shard(codes, scale, rank, world, gk)
        K = Kf // world
        pw = ops.prepare_weights(ops.pack_int4_grouped(c.contiguous(), gk), sc.contiguous(), None, K, gk)
        for M in (1, 16, 64, 200):
            x = syn.activation_torch(M, 2 * K if act else K, 50 + M + 7 * rank, dev)
            y = ar.linear_prepared(x, pw, act=act)
            ref = ops.linear_prepared(x, pw, act=act)
            ar(ref)
            torch.cuda.synchronize()
            if not torch.equal(y, ref):
                ok = False
                verdict["msgs"].append(["fused != linear + all-reduce", variant, N, Kf, M, act])
        # graph: capture once, replay with new inputs
        M = 16
        x = syn.activation_torch(M, 2 * K if act else K, 90 + rank, dev)
        ar.linear_prepared(x, pw, act=act)
        torch.cuda.synchronize()
        dist.barrier()
        gr = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(gr, stream=s):
                yg = ar.linear_prepared(x, pw, act=act)
        torch.cuda.current_stream().wait_stream(s)
        for rep in range(5):
            x.copy_(syn.activation_torch(M, 2 * K if act else K, 100 + rep + 7 * rank, dev))
            torch.cuda.synchronize()
            dist.barrier()
            gr.replay()
            torch.cuda.synchronize()
            ref = ops.linear_prepared(x, pw, act=act)
            ar(ref)
            torch.cuda.synchronize()
            if not torch.equal(yg, ref):
                ok = False
                verdict["msgs"].append(["graph replay differs", variant, N, rep])
        del gr
        ar.check()
    verdict["ok"] &= ok


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
        elif mode == "skew":
            skew_gates(ar, rank, world, dev, verdict)
        elif mode == "fused":
            fused_gates(ar, rank, world, dev, verdict)
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
