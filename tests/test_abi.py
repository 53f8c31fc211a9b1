"""The C-ABI library loads and exports every symbol include/w4a8_b200.h
declares (no compute calls: this runs without a GPU)."""
import ctypes
import os
import re

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(REPO, "include", "w4a8_b200.h")).read()
    return sorted(set(re.findall(r"W4A8_API\s+[\w\s\*]+?\b(w4a8_\w+)\s*\(", src)))


def test_header_declares_symbols():
    names = _declared()
    assert "w4a8_linear" in names and "w4a8_midgroup_w4a8_gemm" in names
    assert len(names) >= 15


def test_library_exports_every_declared_symbol():
    from w4a8_b200 import _lib
    path = _lib.lib_path()
    if not os.path.exists(path):
        pytest.skip("libw4a8_b200.so not built")
    L = ctypes.CDLL(path)
    for name in _declared():
        assert hasattr(L, name), name
    # the Python binding covers exactly the declared surface
    assert sorted(n for n, _, _ in _lib.SIGNATURES) == _declared()


def test_host_only_entry_points():
    """Geometry helpers are pure host code: callable without a GPU."""
    from w4a8_b200 import _lib, ops
    if not os.path.exists(_lib.lib_path()):
        pytest.skip("libw4a8_b200.so not built")
    L = _lib.lib()
    for K, gk in [(5120, 128), (1057, 1024), (1, 1024), (33, 64), (27648, 128), (3456, 128), (100, 256)]:
        assert L.w4a8_num_groups(K, gk) == ops.num_groups(K, gk)
        assert L.w4a8_k_pad_elems(K, gk) == ops.k_pad_elems(K, gk)
    for M in [1, 16, 17, 64, 65, 128, 129, 1000]:
        assert L.w4a8_pad_rows(M) == ops.pad_rows(M)
    assert L.w4a8_build_arch() == 100
    assert L.w4a8_status_string(-2) == b"unsupported group size or dtype"


def test_linear_argument_contract_before_device_work():
    """w4a8_linear validates its arguments before touching the device or any
    memory (the include/w4a8_b200.h error contract); the pointer values here
    are never dereferenced.  A call whose arguments are all valid then fails
    on this machine's missing device, or, on a GPU machine, on the missing
    workspace -- in both cases before any kernel launch."""
    from w4a8_b200 import _lib
    if not os.path.exists(_lib.lib_path()):
        pytest.skip("libw4a8_b200.so not built")
    L = _lib.lib()
    A = 1 << 20                       # 1024-byte aligned fake device addresses
    x, w, s, y = A, 2 * A, 3 * A, 4 * A

    def call(M=16, K=5120, ldx=5120, N=7168, gk=128, x=x, w=w, s=s, sd=_lib.DTYPE_F32, z=None, y=y, ldy=7168):
        return L.w4a8_linear(x, M, K, ldx, N, gk, w, s, sd, z, y, ldy, None, 0, None)

    inv, uns = _lib.ERR_INVALID, _lib.ERR_UNSUPPORTED
    assert call(M=-1) == inv
    assert call(N=7160 + 4) == inv                      # N % 8 != 0
    assert call(gk=100) == uns                          # group size not in {64, 128, 256, 1024}
    assert call(M=0) == _lib.OK                         # empty input: nothing to do
    assert call(x=None) == inv
    assert call(ldx=5119) == inv                        # row stride shorter than K
    assert call(x=x + 1) == inv                         # bf16 rows need 2-byte alignment
    assert call(w=None) == inv
    assert call(s=s + 8) == inv                         # scales need 16-byte alignment
    assert call(sd=7) == uns                            # scale dtype neither bf16 nor fp32
    assert call(y=None) == inv
    assert call(ldy=7167) == inv
    assert call() in (_lib.ERR_CUDA, _lib.ERR_DEVICE, _lib.ERR_WORKSPACE)


def test_fixed_scratch_argument_contract():
    """w4a8_linear_fixed_scratch (no workspace argument) applies the same
    checks first.  Only invalid calls are made here: a valid one would go on to
    launch kernels on the fake addresses if a GPU were present."""
    from w4a8_b200 import _lib
    if not os.path.exists(_lib.lib_path()):
        pytest.skip("libw4a8_b200.so not built")
    L = _lib.lib()
    A = 1 << 20
    x, w, s, y = A, 2 * A, 3 * A, 4 * A

    def call(M=16, K=5120, ldx=5120, N=7168, gk=128, x=x, w=w, s=s, sd=_lib.DTYPE_F32, y=y, ldy=7168):
        return L.w4a8_linear_fixed_scratch(x, M, K, ldx, N, gk, w, s, sd, None, y, ldy, None)

    inv, uns = _lib.ERR_INVALID, _lib.ERR_UNSUPPORTED
    assert call(M=0) == _lib.OK
    assert call(N=12) == inv
    assert call(gk=32) == uns
    assert call(x=None) == inv
    assert call(ldx=100) == inv
    assert call(w=w + 4) == inv
    assert call(sd=2) == uns
    assert call(y=y + 1) == inv
    assert call(ldy=0) == inv
