"""The one-shot custom all-reduce: single-GPU checks here, two-GPU runs in
child processes (skipped with fewer than two GPUs)."""
import json
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def test_world1_is_a_copy():
    from w4a8_b200.allreduce import _Handle
    dev = _dev()
    h = _Handle(0, 1, 1 << 16)
    try:
        h.open_local([h])
        x = torch.randn(5120, device=dev).to(torch.bfloat16)
        y = torch.empty_like(x)
        h.allreduce(x, y)
        torch.cuda.synchronize()
        assert torch.equal(x, y) and h.status() == 0
        with pytest.raises(RuntimeError):          # count * 2 > max_bytes
            h.allreduce(torch.empty(1 << 16, dtype=torch.bfloat16, device=dev),
                        torch.empty(1 << 16, dtype=torch.bfloat16, device=dev))
    finally:
        h.destroy()


def test_absent_peer_times_out_and_leaves_output():
    """Rank 1's handle exists but its kernel never runs: rank 0's wait on a flag
    nothing sets must run out (1 s), be reported, and leave the output alone."""
    from w4a8_b200 import _lib
    from w4a8_b200.allreduce import _Handle
    dev = _dev()
    h0, h1 = _Handle(0, 2, 1 << 16), _Handle(1, 2, 1 << 16)
    try:
        h0.open_local([h0, h1])
        x = torch.randn(4096, device=dev).to(torch.bfloat16)
        y = torch.full_like(x, 7.0)
        h0.allreduce(x, y)
        torch.cuda.synchronize()
        assert h0.status(reset=True) == _lib.ERR_TIMEOUT
        assert torch.all(y == 7.0)
        assert h0.status() == 0                    # reset
    finally:
        torch.cuda.synchronize()
        h0.destroy()
        h1.destroy()


@pytest.mark.parametrize("M,N,K,act", [(16, 5120, 2560, None), (5, 640, 3456, "swiglu"), (64, 5120, 640, None),
                                        (1, 1024, 1024, "swiglu"), (100, 5120, 1280, None)])
def test_world1_fused_row_linear_equals_linear(M, N, K, act):
    """One rank: the fused row-parallel linear + all-reduce gives the linear's bits
    (the sum of one slot), on two calls in a row (the bank alternates)."""
    from w4a8_b200 import _lib, ops
    from w4a8_b200 import synthetic as syn
    from w4a8_b200.allreduce import _Handle
    dev = _dev()
    gk = 128
    codes, scale, _ = syn.weight_torch(N, K, gk, 7 + K, dev)
    pw = ops.prepare_weights(ops.pack_int4_grouped(codes, gk), scale, None, K, gk)
    h = _Handle(0, 1, 1 << 20)
    try:
        h.open_local([h])
        L = _lib.lib()
        for call in range(2):
            x = syn.activation_torch(M, 2 * K if act else K, 8 + call, dev)
            ref = ops.linear_prepared(x, pw, act=act)
            y = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=dev)
            ws, wsb = ops.workspace(ops._ws_bytes(M, N, K, gk), dev)
            rc = L.w4a8_linear_prepared_allreduce(
                x.data_ptr(), M, K, x.stride(0), N, gk, pw.ptr(), pw.ws_dtype, 0,
                _lib.ACT_SWIGLU if act else _lib.ACT_NONE, y.data_ptr(), ws, wsb, h.h,
                torch.cuda.current_stream().cuda_stream)
            assert rc == 0, L.w4a8_status_string(rc).decode()
            torch.cuda.synchronize()
            assert torch.equal(y, ref), call
            assert h.status() == 0 and ops.workspace_status() == 0
        with pytest.raises(RuntimeError):                 # M * N * 2 beyond the buffer
            _lib.check(L.w4a8_linear_prepared_allreduce(
                x.data_ptr(), 1024, K, x.stride(0), N, gk, pw.ptr(), pw.ws_dtype, 0, 0, y.data_ptr(), ws, wsb,
                h.h, None), "oversize")
    finally:
        torch.cuda.synchronize()
        h.destroy()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(mode, tmp_path, world, timeout=240):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    port = str(_free_port())
    procs, outs = [], []
    for r in range(world):
        out = str(tmp_path / f"ar_{mode}_{r}.json")
        outs.append(out)
        procs.append(subprocess.Popen([sys.executable, os.path.join(HERE, "ar_worker.py"), str(r), str(world), port,
                                       mode, out], env=dict(os.environ), start_new_session=True))
    try:
        for p in procs:
            p.wait(timeout=timeout)
    finally:
        for p in procs:
            if p.poll() is None:
                os.killpg(p.pid, 9)
    return [json.load(open(o)) for o in outs]


def test_two_gpus_parity_graph_and_fallback(tmp_path):
    vs = _run("parity", tmp_path, 2)
    for v in vs:
        assert v["ok"], v
        assert v["calls_custom"] >= 6 and v["calls_fallback"] == 1
    print({k: v for k, v in vs[0].items() if k.startswith("us_")})


def test_two_gpus_skewed_barrier_gates(tmp_path):
    """Ranks desynchronised on purpose: only the kernel's flags keep them together."""
    for v in _run("skew", tmp_path, 2):
        assert v["ok"], v


def test_all_gpus_skewed_barrier_gates(tmp_path):
    world = min(torch.cuda.device_count(), 8) if torch.cuda.is_available() else 0
    if world < 3:
        pytest.skip("needs three or more GPUs")
    for v in _run("skew", tmp_path, world, timeout=420):
        assert v["ok"], v


def test_two_gpus_fused_row_linear(tmp_path):
    """Row-parallel linear fused with the all-reduce on 2 ranks: the same bits as
    the linear followed by the one-shot all-reduce; eager and graph replays."""
    for v in _run("fused", tmp_path, 2):
        assert v["ok"], v
        assert v["calls_fused"] >= 8, v


def test_all_gpus_fused_row_linear(tmp_path):
    world = min(torch.cuda.device_count(), 8) if torch.cuda.is_available() else 0
    if world < 3:
        pytest.skip("needs three or more GPUs")
    for v in _run("fused", tmp_path, world):
        assert v["ok"], v


def test_two_gpus_absent_rank(tmp_path):
    vs = _run("absent", tmp_path, 2)
    assert vs[0]["ok"] and any("timed out" in m for m in vs[0]["msgs"]), vs[0]
    assert vs[1]["ok"], vs[1]


def test_all_gpus_parity(tmp_path):
    """Every GPU of the box as one group (3 to 8 ranks)."""
    world = min(torch.cuda.device_count(), 8) if torch.cuda.is_available() else 0
    if world < 3:
        pytest.skip("needs three or more GPUs")
    for v in _run("parity", tmp_path, world):
        assert v["ok"], v
        assert v["calls_custom"] >= 6 and v["calls_fallback"] == 1
