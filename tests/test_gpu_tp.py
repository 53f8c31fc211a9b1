"""The tensor-parallel layer stack through the CUDA op (tp = 1 on one GPU)
against the same stack with the reference arithmetic on CPU.

Each linear requantises the previous bf16 output, so the two stacks are
compared with the stack bound: max|y - ref| / max|ref| <= 3e-2, cosine >= 0.9995."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def test_stack_cuda_matches_reference(orc):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import tp_worker
    from w4a8_b200 import tp
    dev = torch.device("cuda", 0)
    d = tp.Dims(**tp_worker.SMALL)
    x = torch.randn(6, d.hidden, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
    ref = tp.stack_forward(x, tp.build_layers(1, 0, 1, "cpu", d), 1, tp_worker.oracle_linear(d.gk),
                           lambda t: None, d)
    Ls = tp.build_layers(1, 0, 1, dev, d, prepare=True, gen_device="cpu")
    y = tp.stack_forward(x.to(dev), Ls, 1, tp.cuda_linear, lambda t: None, d).float().cpu().numpy()
    r = ref.float().numpy()
    err = np.abs(y - r).max() / np.abs(r).max()
    cos = float((y.astype(np.float64) * r).sum() / (np.linalg.norm(y) * np.linalg.norm(r)))
    assert err <= 3e-2, err
    assert cos >= 0.9995, cos
