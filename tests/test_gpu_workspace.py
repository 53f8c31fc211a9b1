"""The per-device workspace behind the torch ops and CUDA graphs.

A graph captured with a small call holds the workspace address of that
moment.  A later eager call with a larger shape grows the workspace; the old
buffer must stay allocated, so replaying the graph still computes into memory
no other tensor owns and gives the eager result bit for bit."""
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def test_graph_survives_workspace_growth():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from w4a8_b200 import ops
    from w4a8_b200 import synthetic as syn
    dev = torch.device("cuda", 0)
    K, N, gk = 5120, 7168, 128
    codes, scale, _ = syn.weight_torch(N, K, gk, 31, dev)
    pw = ops.prepare_weights(ops.pack_int4_grouped(codes, gk), scale, None, K, gk)
    x16 = syn.activation_torch(16, K, 32, dev)
    y16 = torch.empty(16, N, dtype=torch.bfloat16, device=dev)
    # start from a workspace sized for this call (earlier tests may have grown
    # the current one; it stays allocated and is no longer handed out)
    ops._WS.pop(0, None)
    ops.linear_prepared(x16, pw, out=y16)
    small = ops._WS[0].numel()
    ref16 = y16.clone()
    torch.cuda.synchronize()

    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        ops.linear_prepared(x16, pw, out=y16)

    # grows the workspace past what the graph was captured with
    x_big = syn.activation_torch(2048, K, 33, dev)
    y_big = ops.linear_prepared(x_big, pw)
    ref_big = y_big.clone()
    assert ops._WS[0].numel() > small
    # tensors allocated after the growth would take the freed buffer's memory
    fillers = [torch.full((1 << 20,), 7, dtype=torch.int32, device=dev) for _ in range(8)]
    y16.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(y16, ref16)
    assert all(bool((f == 7).all()) for f in fillers)
    assert torch.equal(ops.linear_prepared(x_big, pw), ref_big)
    assert ops.workspace_status(dev) == 0
    del g
