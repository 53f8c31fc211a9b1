"""Pipeline liveness under back-to-back calls.

The decode sweep (QwQ-32B qkv / o / gate_up / down x M in {1, 4, 8, 16, 32, 64},
each call quantiser + GEMM + stream-K fix-up chained by programmatic dependent
launch) is captured once in a CUDA graph and replayed 2,000 times: 48,000
calls.  Every wait inside the kernels is bounded, so a call whose pipeline
stalls ends with a timeout status (0x100 + wait site) in the workspace status
word instead of a hung GPU; the test asserts that no call recorded one.

A build that launched the dependents of each GEMM at its setup stalled about
once in 50,000 calls of exactly this sequence, so the replay count is sized to
catch a regression of that kind more often than not.

The last replay's outputs are compared with a separate eager run of the same
calls (bit-identical: the kernels are deterministic)."""
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

SHAPES = ("qkv", "o", "gate_up", "down")
MS = (1, 4, 8, 16, 32, 64)
GK = 128
REPLAYS = 2000


def test_decode_sweep_graph_replays_without_stall():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from w4a8_b200 import ops
    from w4a8_b200.synthetic import QWQ_SHAPES, activation_torch, weight_torch

    dev = torch.device("cuda", 0)
    W = {}
    for i, s in enumerate(SHAPES):
        K, N = QWQ_SHAPES[s]
        codes, scale, _ = weight_torch(N, K, GK, 11 + i, dev)
        packed = ops.pack_int4_grouped(codes, GK)
        del codes
        W[s] = (K, N, ops.prepare_weights(packed, scale.contiguous(), None, K, GK))
        del packed
    cfgs = [(s, M) for M in MS for s in SHAPES]
    xs = {(s, M): activation_torch(M, W[s][0], 200 + M, dev) for (s, M) in cfgs}
    ys = {(s, M): torch.empty(M, W[s][1], dtype=torch.bfloat16, device=dev) for (s, M) in cfgs}

    def step():
        for (s, M) in cfgs:
            ops.linear_prepared(xs[(s, M)], W[s][2], out=ys[(s, M)])

    ops.workspace_status(dev, reset=True)
    step()
    torch.cuda.synchronize()
    ref = {k: v.clone() for k, v in ys.items()}
    assert ops.workspace_status(dev) == 0

    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    bad = []
    for i in range(REPLAYS):
        g.replay()
        if i % 100 == 99:
            torch.cuda.synchronize()
            st = ops.workspace_status(dev)
            if st:
                bad.append((i, hex(st)))
    torch.cuda.synchronize()
    del g
    assert not bad, f"replays whose calls recorded a timed-out wait: {bad}"
    for k, v in ys.items():
        assert torch.equal(v, ref[k]), f"call {k} differs from the eager run"


# Configurations whose rings put one stage or TMEM buffer in front of both MMA
# issuers (128-token tiles: 3 activation stages; GK = 1024: several stages per
# unit).  Before they ran on one issuer, an issuer could match the other's
# unfinished round by parity and multiply stale activations: 3 of 11 repeated
# down-projection calls at M = 4096, GK = 256 gave a few wrong token columns in
# split tiles.  Each case repeats the call and requires identical bits.
REPEAT_CASES = [  # shape or (N, K), M, gk
    ("down", 4096, 256), ("down", 2048, 256), ("down", 4096, 128), ("gate_up", 2048, 256),
    ((1024, 8192), 130, 1024), ((2048, 4096), 48, 1024), ((1024, 8192), 20, 1024), ((2048, 6144), 64, 1024),
]


@pytest.mark.parametrize("case", REPEAT_CASES)
def test_repeated_calls_identical(case):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from w4a8_b200 import ops
    from w4a8_b200.synthetic import QWQ_SHAPES, activation_torch, weight_torch
    shape, M, gk = case
    K, N = QWQ_SHAPES[shape] if isinstance(shape, str) else (shape[1], shape[0])
    dev = torch.device("cuda", 0)
    codes, scale, _ = weight_torch(N, K, gk, 90 + gk, dev)
    packed = ops.pack_int4_grouped(codes, gk)
    del codes
    pw = ops.prepare_weights(packed, scale, None, K, gk)
    x = activation_torch(M, K, 91 + M, dev)
    ref = ops.linear_prepared(x, pw)
    for i in range(12):
        y = ops.linear_prepared(x, pw) if i % 2 else ops.linear(x, packed, scale, None, gk)
        assert torch.equal(y, ref), f"call {i + 1} of {case} differs from the first"
    assert ops.workspace_status(dev) == 0
