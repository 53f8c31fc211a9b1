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
