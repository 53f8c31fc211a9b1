"""Vendor W4A8_DYNAMIC projections converted at load and run on the CUDA kernel."""
import numpy as np
import pytest
import torch

from test_vendor_cpu import vendor_projection

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K,gs,offsets", [(16, 512, 1280, 128, False), (5, 256, 640, 64, True),
                                               (130, 384, 1024, 128, True)])
def test_vendor_projection_on_kernel(orc, M, N, K, gs, offsets):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from w4a8_b200 import ops
    from w4a8_b200 import vendor as V
    dev = torch.device("cuda", 0)
    t, codes = vendor_projection(N, K, gs, 40 + M, offsets)
    conv = V.convert_projection(t, gs)
    pw = V.prepare(conv, dev)
    x = torch.randn(M, K, generator=torch.Generator().manual_seed(M)).to(torch.bfloat16)
    y = ops.linear_prepared(x.to(dev), pw).float().cpu().numpy().astype(np.float64)
    assert ops.workspace_status() == 0
    # W4A8 reference: the same codes, combined fp32 scales and zero points
    xbits = x.view(torch.int16).numpy().view(np.uint16)
    zero = None if conv["w_zero"] is None else conv["w_zero"].float().numpy()
    y64, _ = orc.linear(xbits, codes.numpy(), conv["w_scale"].numpy(), zero, gs, exact=True)
    err = np.abs(y - y64).max() / np.abs(y64).max()
    cos = float((y * y64).sum() / (np.linalg.norm(y) * np.linalg.norm(y64)))
    assert err <= 1e-2 and cos >= 0.9999, (err, cos)
    # the vendor's own semantics (bf16 activations, dequantised weights): only the
    # activation quantisation separates the two
    w16 = V.dequantize(conv).double().numpy()
    ya = x.double().numpy() @ w16.T
    cos_a = float((y * ya).sum() / (np.linalg.norm(y) * np.linalg.norm(ya)))
    assert cos_a >= 0.999, cos_a
