"""The tensor-parallel layer stack on the CUDA op.

* tp = 1 through the CUDA op (down projection with the in-quantiser SwiGLU)
  against the same stack with the reference arithmetic on CPU;
* tp = 2 / 4 / 8 at the full QwQ-32B dimensions, every rank's shard on one GPU
  run in lockstep with the all-reduce as an fp32 rank-order sum, against tp = 1
  on the same GPU: the sharding (column-parallel per section, row-parallel at
  group boundaries) and the per-shard linears at TP shapes;
* the SwiGLU-input linear against the oracle on the activation computed on CPU.

Each linear requantises the previous bf16 output, so stacks are compared with
the stack bound: max|y - ref| / max|ref| <= 3e-2, cosine >= 0.9995; a single
linear with the linear bound (1e-2, 0.9999)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

STACK_REL, STACK_COS = 3e-2, 0.9995


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _cmp(y, r):
    y = y.float().cpu().numpy().astype(np.float64)
    r = r.float().cpu().numpy().astype(np.float64)
    err = np.abs(y - r).max() / np.abs(r).max()
    cos = float((y * r).sum() / (np.linalg.norm(y) * np.linalg.norm(r)))
    return err, cos


def test_stack_cuda_matches_reference(orc):
    import tp_worker
    from w4a8_b200 import tp
    dev = _dev()
    d = tp.Dims(**tp_worker.SMALL)
    x = torch.randn(6, d.hidden, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
    ref = tp.stack_forward(x, tp.build_layers(1, 0, 1, "cpu", d), 1, tp_worker.oracle_linear(d.gk),
                           lambda t: None, d)
    Ls = tp.build_layers(1, 0, 1, dev, d, prepare=True, gen_device="cpu")
    y = tp.stack_forward(x.to(dev), Ls, 1, tp.cuda_linear, lambda t: None, d, tp.cuda_swiglu_linear)
    err, cos = _cmp(y, ref)
    assert err <= STACK_REL, err
    assert cos >= STACK_COS, cos


@pytest.mark.parametrize("tpn", [2, 4, 8])
def test_sharded_stack_matches_tp1(tpn):
    from w4a8_b200 import tp
    dev = _dev()
    d = tp.QWQ
    ref_layers = tp.build_layers(1, 0, 1, dev, d, prepare=True)
    ranks = [tp.build_layers(1, r, tpn, dev, d, prepare=True) for r in range(tpn)]
    for M in (16, 256):
        gen = torch.Generator(device=dev).manual_seed(99 + M)
        h = torch.randn(M, d.hidden, generator=gen, device=dev).to(torch.bfloat16)
        ref = tp.stack_forward(h, ref_layers, 1, tp.cuda_linear, lambda t: None, d, tp.cuda_swiglu_linear)
        y = tp.emulated_stack_forward(h, ranks, tp.cuda_linear, d, tp.cuda_swiglu_linear)
        err, cos = _cmp(y, ref)
        assert err <= STACK_REL and cos >= STACK_COS, (tpn, M, err, cos)


@pytest.mark.parametrize("M,K,N", [(16, 3456, 5120), (5, 1000, 256), (64, 27648, 640)])
def test_swiglu_linear(orc, M, K, N):
    """y = bf16(silu(gate) * up) @ W^T from gu = [gate | up] in one op."""
    from w4a8_b200 import ops, tp
    from w4a8_b200 import synthetic as syn
    dev = _dev()
    gk = 128
    gu = syn.activation_torch(M, 2 * K, 40 + M, dev)
    w = syn.weight_np(N, K, gk, 41 + K)
    packed = ops.pack_int4_grouped(torch.from_numpy(w.codes), gk).to(dev)
    scale = torch.from_numpy(w.scale).to(dev)
    pw = ops.prepare_weights(packed, scale, None, K, gk)
    y = ops.linear_prepared(gu, pw, act="swiglu")
    assert torch.equal(y, ops.linear(gu, packed, scale, None, gk, act="swiglu"))
    act = tp.swiglu(gu.cpu())                        # the activation, computed on the CPU
    xb = act.contiguous().view(torch.int16).numpy().view(np.uint16)
    y64, _ = orc.linear(xb, w.codes, w.scale, None, gk, exact=True)
    yv = y.float().cpu().numpy().astype(np.float64)
    err = np.abs(yv - y64).max() / np.abs(y64).max()
    cos = float((yv * y64).sum() / (np.linalg.norm(yv) * np.linalg.norm(y64)))
    assert err <= 1e-2 and cos >= 0.9999, (err, cos)
    # a strided [gate | up] (ldx > 2K) gives the same result
    big = torch.zeros(M, 2 * K + 64, dtype=torch.bfloat16, device=dev)
    big[:, :2 * K] = gu
    assert torch.equal(ops.linear_prepared(big[:, :2 * K], pw, act="swiglu"), y)
    with pytest.raises(RuntimeError):
        ops.linear_prepared(gu[:, :K], pw, act="swiglu")
