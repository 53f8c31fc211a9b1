"""w4a8_linear_fixed_scratch: the workspace-free linear entry point.

Compared with w4a8_linear (same inputs, caller-provided workspace) on two
calls in a row; both must satisfy the linear tolerance against each other:

    max|y - y_ref| / max|y_ref| <= 1e-2   and   cosine(y, y_ref) >= 0.9999

The file is named to be collected last and does not depend on any other test
having run before it."""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

MAX_REL = 1e-2
MIN_COS = 0.9999


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _close(y, ref):
    y = y.float().cpu().numpy().astype(np.float64)
    ref = ref.float().cpu().numpy().astype(np.float64)
    err = np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30)
    cos = float((y * ref).sum() / (np.linalg.norm(y) * np.linalg.norm(ref) + 1e-300))
    assert err <= MAX_REL, f"max rel {err}"
    assert cos >= MIN_COS, f"cosine {cos}"


def _call(L, x, w_packed, w_scale, w_zero, gk, y):
    M, K = x.shape
    N = w_packed.shape[0]
    sd = 1 if w_scale.dtype == torch.float32 else 0
    return L.w4a8_linear_fixed_scratch(
        x.data_ptr(), M, K, x.stride(0), N, gk, w_packed.data_ptr(), w_scale.data_ptr(), sd,
        None if w_zero is None else w_zero.data_ptr(), y.data_ptr(), y.stride(0),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("M,N,K,gk,asym", [(16, 7168, 5120, 128, False), (5, 384, 1057, 1024, True),
                                           (64, 1024, 2048, 64, False)])
def test_fixed_scratch_matches_linear(M, N, K, gk, asym):
    from w4a8_b200 import _lib, ops
    from w4a8_b200 import synthetic as syn
    dev = _dev()
    L = _lib.lib()
    x = syn.activation_torch(M, K, 11 + M, dev)
    codes, scale, zero = syn.weight_torch(N, K, gk, 12 + N, dev, asym=asym)
    packed = ops.pack_int4_grouped(codes, gk)
    wz = None if zero is None else zero.to(torch.bfloat16).contiguous()
    ref = ops.linear(x, packed, scale, wz, gk)
    for _ in range(2):          # two calls in a row on the same fixed scratch
        y = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=dev)
        rc = _call(L, x, packed, scale, wz, gk, y)
        assert rc == 0, L.w4a8_status_string(rc).decode()
        torch.cuda.synchronize()
        _close(y, ref)


def test_fixed_scratch_rejects_oversize():
    from w4a8_b200 import _lib, ops
    dev = _dev()
    L = _lib.lib()
    M, N, K, gk = 2048, 7168, 5120, 128
    assert L.w4a8_linear_workspace_size(M, N, K, gk) > _lib.FIXED_SCRATCH_BYTES
    x = torch.zeros(M, K, dtype=torch.bfloat16, device=dev)
    packed = torch.zeros(N, ops.k_pad_elems(K, gk) // 2, dtype=torch.int8, device=dev)
    scale = torch.ones(ops.num_groups(K, gk), N, dtype=torch.float32, device=dev)
    y = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    assert _call(L, x, packed, scale, None, gk, y) == _lib.ERR_WORKSPACE
