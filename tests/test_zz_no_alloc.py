"""w4a8_linear_fixed_scratch: the workspace-free linear entry point.

Some callers cannot allocate device memory where they call the linear layer:
a foreign-language host that binds the C ABI but holds no device allocator,
or a serving loop whose allocator must not be entered mid-step.  This entry
point keeps its scratch in one fixed array inside the library instead.

It launches the same kernels as w4a8_linear on the same inputs, so its output
must equal w4a8_linear's bit for bit, on two calls in a row; both are also
held to the linear tolerance against the float64 exact-integer oracle:

    max|y - y_ref| / max|y_ref| <= 1e-2   and   cosine(y, y_ref) >= 0.9999

After every call the array's status word (a kernel wait that ran out) must
read 0.  The file is named to be collected last and does not depend on any
other test having run before it."""
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


def _bits(t) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def _close(y_bits, ref64, orc):
    y = orc.bf16_to_f32(y_bits).astype(np.float64)
    err = np.abs(y - ref64).max() / max(np.abs(ref64).max(), 1e-30)
    cos = float((y * ref64).sum() / (np.linalg.norm(y) * np.linalg.norm(ref64) + 1e-300))
    assert err <= MAX_REL, f"max rel {err}"
    assert cos >= MIN_COS, f"cosine {cos}"


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _call(L, x, w_packed, w_scale, w_zero, gk, y):
    M, K = x.shape
    N = w_packed.shape[0]
    sd = 1 if w_scale.dtype == torch.float32 else 0
    return L.w4a8_linear_fixed_scratch(
        x.data_ptr(), M, K, x.stride(0), N, gk, w_packed.data_ptr(), w_scale.data_ptr(), sd,
        None if w_zero is None else w_zero.data_ptr(), y.data_ptr(), y.stride(0), _stream())


def _call_linear(L, x, w_packed, w_scale, w_zero, gk, y, ws, ws_bytes):
    M, K = x.shape
    N = w_packed.shape[0]
    sd = 1 if w_scale.dtype == torch.float32 else 0
    return L.w4a8_linear(
        x.data_ptr(), M, K, x.stride(0), N, gk, w_packed.data_ptr(), w_scale.data_ptr(), sd,
        None if w_zero is None else w_zero.data_ptr(), y.data_ptr(), y.stride(0), ws, ws_bytes, _stream())


@pytest.mark.parametrize("M,N,K,gk,asym", [(16, 7168, 5120, 128, False), (5, 384, 1057, 1024, True),
                                           (64, 1024, 2048, 64, False)])
def test_fixed_scratch_matches_linear(orc, M, N, K, gk, asym):
    from w4a8_b200 import _lib, ops
    from w4a8_b200 import synthetic as syn
    dev = _dev()
    L = _lib.lib()
    xb = syn.activation_np(M, K, 11 + M)
    w = syn.weight_np(N, K, gk, 12 + N, asym=asym)
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).to(dev)
    packed = ops.pack_int4_grouped(torch.from_numpy(w.codes), gk).to(dev)
    scale = torch.from_numpy(w.scale).to(dev)
    wz = None if w.zero is None else torch.from_numpy(w.zero).to(torch.bfloat16).to(dev)

    # the workspace entry point, through the C ABI with its own zeroed workspace
    ws_bytes = L.w4a8_linear_workspace_size(M, N, K, gk)
    ws_buf = torch.zeros(ws_bytes + 1024, dtype=torch.uint8, device=dev)
    ws = (ws_buf.data_ptr() + 1023) & ~1023
    ref = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    rc = _call_linear(L, x, packed, scale, wz, gk, ref, ws, ws_bytes)
    assert rc == 0, L.w4a8_status_string(rc).decode()
    assert L.w4a8_workspace_status(ws, 1, _stream()) == 0
    ref_bits = _bits(ref)
    y64, _ = orc.linear(xb, w.codes, w.scale, w.zero, gk, exact=True)
    _close(ref_bits, y64, orc)

    for _ in range(2):          # two calls in a row on the same fixed scratch
        y = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=dev)
        rc = _call(L, x, packed, scale, wz, gk, y)
        assert rc == 0, L.w4a8_status_string(rc).decode()
        assert L.w4a8_fixed_scratch_status(1, _stream()) == 0
        y_bits = _bits(y)
        assert np.array_equal(y_bits, ref_bits), "fixed-scratch output differs from w4a8_linear"
        _close(y_bits, y64, orc)


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
