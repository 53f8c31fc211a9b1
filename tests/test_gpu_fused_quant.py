"""The activation quantiser fused into the GEMM (w4a8_set_options(
W4A8_OPT_FUSED_QUANT); calls with M <= 16, group size <= 256, 16-byte aligned
rows) against the default path, the standalone quantiser kernel followed by
the GEMM: the same codes, scales and accumulation order, so the same bits; and
both against the oracle at the linear tolerance."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

CASES = [  # M, N, K, gk, asym, prepared
    (1, 7168, 5120, 128, False, True), (4, 5120, 5120, 128, False, True), (16, 5120, 27648, 128, False, True),
    (16, 1024, 1000, 128, False, False), (7, 384, 3000, 64, True, True), (16, 640, 2304, 256, True, False),
    (3, 256, 520, 64, False, True), (16, 55296, 5120, 128, False, True), (9, 768, 1024, 256, False, True),
]


def _bits(t):
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("M,N,K,gk,asym,prepared", CASES)
def test_fused_equals_standalone(orc, M, N, K, gk, asym, prepared):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from w4a8_b200 import _lib, ops
    from w4a8_b200 import synthetic as syn
    dev = torch.device("cuda", 0)
    xb = syn.activation_np(M, K, 70 + M + K)
    w = syn.weight_np(N, K, gk, 71 + N, asym=asym)
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).to(dev)
    packed = ops.pack_int4_grouped(torch.from_numpy(w.codes), gk).to(dev)
    scale = torch.from_numpy(w.scale).to(dev)
    wz = None if w.zero is None else torch.from_numpy(w.zero).to(torch.bfloat16).to(dev)
    pw = ops.prepare_weights(packed, scale, wz, K, gk) if prepared else None

    def run():
        return ops.linear_prepared(x, pw) if prepared else ops.linear(x, packed, scale, wz, gk)

    L = _lib.lib()
    standalone = run()
    old = L.w4a8_set_options(_lib.OPT_FUSED_QUANT)
    try:
        fused = run()
        assert torch.equal(run(), fused)             # repeatable
    finally:
        L.w4a8_set_options(old)
    assert torch.equal(fused, standalone)
    assert ops.workspace_status() == 0
    # the oracle on a column sample
    cols = np.unique(np.concatenate([np.arange(0, N, 128), np.arange(127, N, 128)]))
    y64, _ = orc.linear(xb, w.codes[cols], w.scale[:, cols], None if w.zero is None else w.zero[:, cols], gk,
                        exact=True)
    y = orc.bf16_to_f32(_bits(fused)[:, cols]).astype(np.float64)
    err = np.abs(y - y64).max() / np.abs(y64).max()
    cos = float((y * y64).sum() / (np.linalg.norm(y) * np.linalg.norm(y64)))
    assert err <= 1e-2 and cos >= 0.9999, (err, cos)


def test_fused_in_graph_and_strided_rows(orc):
    """A strided activation (row stride > K, 16-byte aligned) takes the fused
    path; replaying a captured graph with new activation values recomputes."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from w4a8_b200 import _lib
    old = _lib.lib().w4a8_set_options(_lib.OPT_FUSED_QUANT)
    try:
        _fused_graph_case()
    finally:
        _lib.lib().w4a8_set_options(old)


def _fused_graph_case():
    from w4a8_b200 import ops
    from w4a8_b200 import synthetic as syn
    dev = torch.device("cuda", 0)
    M, N, K, gk = 16, 7168, 5120, 128
    codes, scale, _ = syn.weight_torch(N, K, gk, 80, dev)
    pw = ops.prepare_weights(ops.pack_int4_grouped(codes, gk), scale, None, K, gk)
    big = torch.zeros(M, K + 64, dtype=torch.bfloat16, device=dev)
    x = big[:, :K]
    x.copy_(syn.activation_torch(M, K, 81, dev))
    y = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    ops.linear_prepared(x, pw, out=y)
    assert torch.equal(y, ops.linear_prepared(x.contiguous(), pw))
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        ops.linear_prepared(x, pw, out=y)
    x.copy_(syn.activation_torch(M, K, 82, dev))
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, ops.linear_prepared(x.contiguous(), pw))
    assert ops.workspace_status() == 0
    del g
