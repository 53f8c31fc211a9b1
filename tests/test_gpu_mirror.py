"""The reference-facing ops on the GPU: torch.ops.npu.* and torch.ops.w4a8.*
give the same bits as the library calls, and the vLLM quant method
(create_weights -> load a checkpoint-layout tensor set -> process_weights_after_loading
-> apply) gives the same bits as the reference-layout linear and stays within
the linear tolerance: max|y - ref| / max|ref| <= 1e-2 and cosine >= 0.9999
against the float64 exact-integer reference."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _bits(t):
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def _check(y, y64):
    yf = y.float().cpu().numpy().astype(np.float64)
    err = np.abs(yf - y64).max() / np.abs(y64).max()
    cos = (yf * y64).sum() / (np.linalg.norm(yf) * np.linalg.norm(y64))
    assert err <= 1e-2 and cos >= 0.9999, (err, cos)


def test_npu_ops_match_library(orc):
    from w4a8_b200 import ops, w4a8_ops
    from w4a8_b200 import synthetic as syn
    dev = _dev()
    w4a8_ops.load()
    M, K, N = 20, 2048, 256
    x = syn.activation_torch(M, K, 31, dev)
    w = torch.randn(N, K, generator=torch.Generator().manual_seed(32)).mul(0.02).to(torch.bfloat16)
    wq, ws, wk, wz = (t.to(dev) for t in w4a8_ops.quantize_weight(w, 1024))
    outs_npu = torch.ops.npu.midgroup_quant_a(x)
    outs_lib = ops.midgroup_quant_a(x, 1024)
    for a, b in zip(outs_npu, outs_lib):
        assert torch.equal(a, b)
    y_npu = torch.ops.npu.midgroup_w4a8_gemm(*outs_npu, wq, ws, wk, wz, K)
    y_lib = ops.midgroup_w4a8_gemm(*outs_lib, wq, ws, wk, wz, K, 1024)
    assert torch.equal(y_npu, y_lib)
    y_lin = w4a8_ops.linear(x, wq, ws, wk, wz)
    assert torch.equal(y_lin, torch.ops.w4a8.linear(x, wq, ws, wz, 1024))
    codes = ops.unpack_int4_grouped(wq.cpu(), K, 1024).numpy()
    y64, _ = orc.linear(_bits(x), codes, ws.float().cpu().numpy(), wz.float().cpu().numpy(), 1024, exact=True)
    _check(y_npu[:M], y64)
    _check(y_lin, y64)


@pytest.mark.parametrize("gk,K", [(128, 1024), (1024, 2048)])
def test_quant_method_end_to_end(orc, gk, K):
    pytest.importorskip("vllm")
    from w4a8_b200 import midgroup_quant as mq
    from w4a8_b200 import ops, w4a8_ops
    from w4a8_b200 import synthetic as syn
    dev = _dev()
    N, M = 384, 9
    meth = mq.MidGroupW4A8LinearMethod(mq.MidGroupW4A8Config(group_size=gk), "layer")
    layer = torch.nn.Module()
    meth.create_weights(layer, K, [N], K, N, torch.bfloat16)
    w = torch.randn(N, K, generator=torch.Generator().manual_seed(40 + gk)).mul(0.02).to(torch.bfloat16)
    wq, ws, wk, wz = w4a8_ops.quantize_weight(w, gk)
    with torch.no_grad():          # the checkpoint stores the scale-like tensors [N, G]
        layer.weight_packed.copy_(wq)
        layer.weight_scale.copy_(ws.t())
        layer.weight_zero.copy_(wz.t())
        layer.weight_ksum.copy_(wk.t())
    layer.to(dev)
    meth.process_weights_after_loading(layer)
    x = syn.activation_torch(M, K, 41, dev).reshape(3, 3, K)
    bias = torch.randn(N, device=dev).to(torch.bfloat16)
    y = meth.apply(layer, x, bias)
    assert y.shape == (3, 3, N)
    assert torch.equal(y, ops.linear(x, wq.to(dev), ws.to(dev), wz.to(dev), gk) + bias)
    codes = ops.unpack_int4_grouped(wq, K, gk).numpy()
    y64, _ = orc.linear(_bits(x.reshape(M, K)), codes, ws.float().numpy(), wz.float().numpy(), gk, exact=True)
    _check(meth.apply(layer, x).reshape(M, N), y64)
