"""CPU checker for the W4A8 mid-group path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import this package, and only to check or time the reference algorithm.
The shipped library never imports it and has no CPU fallback.

Two independent implementations sit behind this module:

* ``libw4a8_oracle.so`` -- a C restatement of the reference's CPU path
  (``oracle/w4a8_oracle.c``; each function cites the reference file:line it
  follows).  Built by ``make -C oracle``.
* ``_ref/libw4a8_ref.so`` -- the reference's own C++ CPU GEMM
  (``int4_cube_lab/host/gemm_ref.cpp``) compiled from the reference source tree
  by ``make -C oracle ref``; optional (``ref_available()``).

All arrays are numpy.  bf16 values travel as their ``uint16`` bit patterns.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional, Tuple

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB: Optional[ctypes.CDLL] = None
_REF: Optional[ctypes.CDLL] = None

_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_u32 = ctypes.c_uint32
_p = ctypes.c_void_p


def _ptr(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data_as(_p)


def lib() -> ctypes.CDLL:
    """Load the C restatement (building it is ``make -C oracle``)."""
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "libw4a8_oracle.so")
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle`")
        L = ctypes.CDLL(path)
        L.orc_num_groups.restype = _i64
        L.orc_num_groups.argtypes = [_i64, _i32]
        L.orc_k_pad_elems.restype = _i64
        L.orc_k_pad_elems.argtypes = [_i64, _i32]
        L.orc_group_real.restype = _i64
        L.orc_group_real.argtypes = [_i64, _i64, _i32]
        L.orc_f32_to_bf16.restype = ctypes.c_uint16
        L.orc_f32_to_bf16.argtypes = [ctypes.c_float]
        L.orc_quant_act.argtypes = [_p, _i64, _i64, _i64, _i32, _p, _p, _p]
        L.orc_midgroup_quant_a.argtypes = [_p, _i64, _i64, _i64, _i32, _p, _p, _p, _p]
        L.orc_pack_int4_grouped.argtypes = [_p, _i64, _i64, _i32, _p]
        L.orc_unpack_int4_grouped.argtypes = [_p, _i64, _i64, _i32, _p]
        L.orc_msd_recombine.argtypes = [_p, _p, _i64, _i64, _i32, _p]
        L.orc_group_partials.argtypes = [_p, _p, _p, _i64, _i64, _i64, _i32, _p]
        L.orc_gemm_kernel_order.argtypes = [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i32, _p]
        L.orc_gemm_f64.argtypes = [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i32, _p]
        L.orc_f32_to_bf16_array.argtypes = [_p, _i64, _p]
        L.orc_set_threads.argtypes = [_i32]
        _LIB = L
    return _LIB


def set_threads(n: int) -> None:
    """OpenMP threads for the oracle's and the reference C++ GEMM's loops (one
    process-wide setting; independent of OMP_NUM_THREADS in the environment)."""
    lib().orc_set_threads(int(n))


def ref_available() -> bool:
    return os.path.exists(os.path.join(_HERE, "_ref", "libw4a8_ref.so"))


def ref() -> ctypes.CDLL:
    """The reference's own C++ CPU GEMM, compiled from its sources."""
    global _REF
    if _REF is None:
        path = os.path.join(_HERE, "_ref", "libw4a8_ref.so")
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle ref`")
        R = ctypes.CDLL(path)
        R.ref_midgroup_gemm.argtypes = [_p, _p, _p, _p, _p, _p, _u32, _u32, _u32, _u32, _u32]
        R.ref_pack_int4_grouped.argtypes = [_p, _u32, _u32, _u32, _p]
        R.ref_split_planes_grouped.argtypes = [_p, _u32, _u32, _u32, _p, _p]
        R.ref_weight_ksum_per_group.argtypes = [_p, _u32, _u32, _u32, _p]
        R.ref_act_ksum_neg_per_group.argtypes = [_p, _u32, _u32, _u32, _p]
        _REF = R
    return _REF


# ---------------------------------------------------------------- helpers

def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bits (NaN kept quiet)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().orc_f32_to_bf16_array(_ptr(x), x.size, _ptr(out))
    return out


def num_groups(K: int, gk: int) -> int:
    return int(lib().orc_num_groups(K, gk))


def k_pad_elems(K: int, gk: int) -> int:
    return int(lib().orc_k_pad_elems(K, gk))


def group_real(g: int, K: int, gk: int) -> int:
    return int(lib().orc_group_real(g, K, gk))


# ---------------------------------------------------------------- quantiser

def quant_act(x_bits: np.ndarray, gk: int) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """bf16 bits [M,K] -> (q int8 [M,K], scale bf16 bits [G,M], ksum_neg int32 [G,M])."""
    x = np.ascontiguousarray(x_bits, dtype=np.uint16)
    M, K = x.shape
    G = num_groups(K, gk)
    q = np.zeros((M, K), np.int8)
    s = np.zeros((G, M), np.uint16)
    ks = np.zeros((G, M), np.int32)
    lib().orc_quant_act(_ptr(x), M, K, K, gk, _ptr(q), _ptr(s), _ptr(ks))
    return q, s, ks


def midgroup_quant_a(x_bits: np.ndarray, Mp: int, gk: int):
    """The four tensors of the reference's ``midgroup_quant_a`` op."""
    x = np.ascontiguousarray(x_bits, dtype=np.uint16)
    M, K = x.shape
    G, Kp = num_groups(K, gk), k_pad_elems(K, gk)
    hi = np.zeros((Mp, Kp // 2), np.int8)
    lo = np.zeros((Mp, Kp // 2), np.int8)
    s = np.zeros((G, Mp), np.uint16)
    ks = np.zeros((G, Mp), np.int32)
    lib().orc_midgroup_quant_a(_ptr(x), M, Mp, K, gk, _ptr(hi), _ptr(lo), _ptr(s), _ptr(ks))
    return hi, lo, s, ks


def msd_recombine(hi: np.ndarray, lo: np.ndarray, K: int, gk: int) -> np.ndarray:
    hi = np.ascontiguousarray(hi, np.int8)
    lo = np.ascontiguousarray(lo, np.int8)
    q = np.zeros((hi.shape[0], K), np.int8)
    lib().orc_msd_recombine(_ptr(hi), _ptr(lo), hi.shape[0], K, gk, _ptr(q))
    return q


# ---------------------------------------------------------------- weights

def pack_int4_grouped(codes: np.ndarray, gk: int) -> np.ndarray:
    c = np.ascontiguousarray(codes, np.int8)
    rows, K = c.shape
    out = np.zeros((rows, k_pad_elems(K, gk) // 2), np.int8)
    lib().orc_pack_int4_grouped(_ptr(c), rows, K, gk, _ptr(out))
    return out


def unpack_int4_grouped(packed: np.ndarray, K: int, gk: int) -> np.ndarray:
    p = np.ascontiguousarray(packed, np.int8)
    out = np.zeros((p.shape[0], K), np.int8)
    lib().orc_unpack_int4_grouped(_ptr(p), p.shape[0], K, gk, _ptr(out))
    return out


# ---------------------------------------------------------------- GEMM

def _f32(a):
    return None if a is None else np.ascontiguousarray(a, np.float32)


def group_partials(qa: np.ndarray, qw: np.ndarray, wz: Optional[np.ndarray], gk: int) -> np.ndarray:
    """int32 P[G,M,N] = sum_{k in g} A*(W - wz)."""
    qa = np.ascontiguousarray(qa, np.int8)
    qw = np.ascontiguousarray(qw, np.int8)
    M, K = qa.shape
    N = qw.shape[0]
    G = num_groups(K, gk)
    wzf = _f32(wz)
    P = np.zeros((G, M, N), np.int32)
    lib().orc_group_partials(_ptr(qa), _ptr(qw), _ptr(wzf), M, N, K, gk, _ptr(P))
    return P


def gemm_kernel_order(qa, as_f32, qw, ws_f32, wz, gk) -> np.ndarray:
    """fp32 y [M,N] in fake_linear's accumulation order."""
    qa = np.ascontiguousarray(qa, np.int8)
    qw = np.ascontiguousarray(qw, np.int8)
    M, K = qa.shape
    N = qw.shape[0]
    y = np.zeros((M, N), np.float32)
    asf, wsf, wzf = _f32(as_f32), _f32(ws_f32), _f32(wz)
    lib().orc_gemm_kernel_order(_ptr(qa), _ptr(asf), _ptr(qw), _ptr(wsf), _ptr(wzf), M, N, K, gk, _ptr(y))
    return y


def gemm_f64(qa, as_f32, qw, ws_f32, wz, gk) -> np.ndarray:
    """float64 y [M,N]: exact integer partials, float64 rescale."""
    qa = np.ascontiguousarray(qa, np.int8)
    qw = np.ascontiguousarray(qw, np.int8)
    M, K = qa.shape
    N = qw.shape[0]
    y = np.zeros((M, N), np.float64)
    asf, wsf, wzf = _f32(as_f32), _f32(ws_f32), _f32(wz)
    lib().orc_gemm_f64(_ptr(qa), _ptr(asf), _ptr(qw), _ptr(wsf), _ptr(wzf), M, N, K, gk, _ptr(y))
    return y


def linear(x_bits: np.ndarray, w_codes: np.ndarray, ws_f32: np.ndarray,
           wz: Optional[np.ndarray], gk: int, exact: bool = False):
    """The whole reference path: quantise x per (row, group), then the GEMM.

    Returns ``(y, parts)`` where ``y`` is fp32 (kernel order) or float64
    (``exact=True``) and ``parts = (q, a_scale_bits, ksum_neg)``.
    """
    q, s, ks = quant_act(x_bits, gk)
    as_f32 = bf16_to_f32(s)
    f = gemm_f64 if exact else gemm_kernel_order
    return f(q, as_f32, w_codes, ws_f32, wz, gk), (q, s, ks)


# ---------------------------------------------------------------- reference C++

def ref_midgroup_gemm(qa, as_bits, qw, ws_bits, wz_bits, gk, mp: int = 0) -> np.ndarray:
    """bf16 bits y [M,N] from the reference's ReferenceMidGroupGemm."""
    qa = np.ascontiguousarray(qa, np.int8)
    qw = np.ascontiguousarray(qw, np.int8)
    M, K = qa.shape
    N = qw.shape[0]
    y = np.zeros((M, N), np.uint16)
    asb = np.ascontiguousarray(as_bits, np.uint16)
    wsb = np.ascontiguousarray(ws_bits, np.uint16)
    wzb = None if wz_bits is None else np.ascontiguousarray(wz_bits, np.uint16)
    ref().ref_midgroup_gemm(_ptr(qa), _ptr(asb), _ptr(qw), _ptr(wsb), _ptr(wzb), _ptr(y),
                            M, N, K, gk, mp)
    return y


def ref_pack_int4_grouped(codes, gk) -> np.ndarray:
    c = np.ascontiguousarray(codes, np.int8)
    rows, K = c.shape
    out = np.zeros((rows, k_pad_elems(K, gk) // 2), np.int8)
    ref().ref_pack_int4_grouped(_ptr(c), rows, K, gk, _ptr(out))
    return out


def ref_split_planes_grouped(q, gk):
    a = np.ascontiguousarray(q, np.int8)
    rows, K = a.shape
    kp = k_pad_elems(K, gk) // 2
    hi = np.zeros((rows, kp), np.int8)
    lo = np.zeros((rows, kp), np.int8)
    ref().ref_split_planes_grouped(_ptr(a), rows, K, gk, _ptr(hi), _ptr(lo))
    return hi, lo


def ref_act_ksum_neg(q, gk) -> np.ndarray:
    a = np.ascontiguousarray(q, np.int8)
    rows, K = a.shape
    out = np.zeros((num_groups(K, gk), rows), np.int32)
    ref().ref_act_ksum_neg_per_group(_ptr(a), rows, K, gk, _ptr(out))
    return out


def ref_weight_ksum(w, gk) -> np.ndarray:
    a = np.ascontiguousarray(w, np.int8)
    rows, K = a.shape
    out = np.zeros((num_groups(K, gk), rows), np.int32)
    ref().ref_weight_ksum_per_group(_ptr(a), rows, K, gk, _ptr(out))
    return out
