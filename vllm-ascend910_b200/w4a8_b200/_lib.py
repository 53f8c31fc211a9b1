"""ctypes binding of libw4a8_b200.so (the C ABI in include/w4a8_b200.h).

The library is built in-tree (``make -C vllm-ascend910_b200/csrc``) and lives
next to this file; ``W4A8_B200_LIB`` overrides the path.  There is no fallback:
if the library is missing every op raises.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_NAME = "libw4a8_b200.so"

OK = 0
ERR_INVALID = -1
ERR_UNSUPPORTED = -2
ERR_CUDA = -3
ERR_WORKSPACE = -4
ERR_DEVICE = -5
ERR_TIMEOUT = -6
DTYPE_BF16 = 0
DTYPE_F32 = 1
FIXED_SCRATCH_BYTES = 16 << 20   # W4A8_FIXED_SCRATCH_BYTES
OPT_FUSED_QUANT = 1              # W4A8_OPT_FUSED_QUANT
OPT_AR_PUSH = 2                  # W4A8_OPT_AR_PUSH
ACT_NONE = 0                     # W4A8_ACT_NONE
ACT_SWIGLU = 1                   # W4A8_ACT_SWIGLU

_L = None

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_sz = ctypes.c_size_t

# (name, restype, argtypes) of every exported symbol, in header order.
SIGNATURES = [
    ("w4a8_num_groups", _i64, [_i64, _i32]),
    ("w4a8_k_pad_elems", _i64, [_i64, _i32]),
    ("w4a8_pad_rows", _i64, [_i64]),
    ("w4a8_linear_workspace_size", _sz, [_i64, _i64, _i64, _i32]),
    ("w4a8_linear", ctypes.c_int,
     [_p, _i64, _i64, _i64, _i64, _i32, _p, _p, _i32, _p, _p, _i64, _p, _sz, _p]),
    ("w4a8_linear_swiglu", ctypes.c_int,
     [_p, _i64, _i64, _i64, _i64, _i32, _p, _p, _i32, _p, _p, _i64, _p, _sz, _p]),
    ("w4a8_linear_quant", ctypes.c_int, [_p, _i64, _i64, _i64, _i64, _i32, _p, _sz, _p]),
    ("w4a8_linear_gemm", ctypes.c_int,
     [_i64, _i64, _i64, _i32, _p, _p, _i32, _p, _p, _i64, _p, _sz, _p]),
    ("w4a8_prepared_weights_size", _sz, [_i64, _i64, _i32, _i32, _i32]),
    ("w4a8_prepare_weights", ctypes.c_int, [_p, _p, _i32, _p, _i64, _i64, _i32, _p, _sz, _p]),
    ("w4a8_linear_prepared", ctypes.c_int,
     [_p, _i64, _i64, _i64, _i64, _i32, _p, _i32, _i32, _p, _i64, _p, _sz, _p]),
    ("w4a8_linear_prepared_swiglu", ctypes.c_int,
     [_p, _i64, _i64, _i64, _i64, _i32, _p, _i32, _i32, _p, _i64, _p, _sz, _p]),
    ("w4a8_linear_gemm_prepared", ctypes.c_int,
     [_i64, _i64, _i64, _i32, _p, _i32, _i32, _p, _i64, _p, _sz, _p]),
    ("w4a8_linear_fixed_scratch", ctypes.c_int,
     [_p, _i64, _i64, _i64, _i64, _i32, _p, _p, _i32, _p, _p, _i64, _p]),
    ("w4a8_fixed_scratch_status", ctypes.c_int, [_i32, _p]),
    ("w4a8_quant_act", ctypes.c_int, [_p, _i64, _i64, _i64, _i32, _p, _p, _i32, _p, _p]),
    ("w4a8_midgroup_quant_a", ctypes.c_int, [_p, _i64, _i64, _i32, _i64, _p, _p, _p, _p, _p]),
    ("w4a8_midgroup_gemm_workspace_size", _sz, [_i64, _i64, _i64, _i32]),
    ("w4a8_midgroup_w4a8_gemm", ctypes.c_int,
     [_p, _p, _p, _p, _i64, _p, _p, _p, _p, _i64, _i64, _i32, _p, _p, _sz, _p]),
    ("w4a8_group_partials", ctypes.c_int,
     [_p, _i64, _i64, _i64, _i64, _i32, _p, _p, _p, _p, _sz, _p]),
    ("w4a8_ar_ipc_handle_size", _sz, []),
    ("w4a8_ar_create", ctypes.c_int, [_i32, _i32, _sz, ctypes.POINTER(_p)]),
    ("w4a8_ar_ipc_handle", ctypes.c_int, [_p, _p]),
    ("w4a8_ar_open_peers", ctypes.c_int, [_p, _p]),
    ("w4a8_ar_open_local", ctypes.c_int, [_p, _p]),
    ("w4a8_ar_max_bytes", _sz, [_p]),
    ("w4a8_ar_allreduce_bf16", ctypes.c_int, [_p, _p, _p, _i64, _p]),
    ("w4a8_ar_status", ctypes.c_int, [_p, _i32]),
    ("w4a8_ar_destroy", ctypes.c_int, [_p]),
    ("w4a8_linear_prepared_allreduce", ctypes.c_int,
     [_p, _i64, _i64, _i64, _i64, _i32, _p, _i32, _i32, _i32, _p, _p, _sz, _p, _p]),
    ("w4a8_workspace_status", ctypes.c_int, [_p, _i32, _p]),
    ("w4a8_status_string", ctypes.c_char_p, [ctypes.c_int]),
    ("w4a8_last_cuda_error", ctypes.c_int, []),
    ("w4a8_build_arch", ctypes.c_int, []),
    ("w4a8_set_options", ctypes.c_int, [_i32]),
]


def lib_path() -> str:
    return os.environ.get("W4A8_B200_LIB") or os.path.join(_HERE, LIB_NAME)


def lib() -> ctypes.CDLL:
    """Load the library once.  Raises if it was not built."""
    global _L
    if _L is None:
        path = lib_path()
        if not os.path.exists(path):
            raise RuntimeError(
                f"{path} not found: build it with `make -C vllm-ascend910_b200/csrc` "
                "(the B200 W4A8 ops have no CPU implementation)")
        L = ctypes.CDLL(path)
        for name, res, args in SIGNATURES:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _L = L
    return _L


class W4A8Error(RuntimeError):
    pass


def check(rc: int, what: str) -> None:
    if rc != OK:
        msg = lib().w4a8_status_string(rc).decode()
        if rc == ERR_CUDA:
            msg += f" (cudaError {lib().w4a8_last_cuda_error()})"
        raise W4A8Error(f"{what}: {msg}")
