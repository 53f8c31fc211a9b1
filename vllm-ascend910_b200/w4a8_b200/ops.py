"""Torch-facing W4A8 ops over the C ABI (CUDA tensors in, CUDA tensors out).

Argument checks mirror the reference host ops' TORCH_CHECKs
(npu_ops/host/midgroup_quant_a.cpp:42-43, midgroup_w4a8_gemm.cpp:149-183) and
raise ``RuntimeError`` with a message.  Kernels run on the current CUDA stream;
nothing here synchronises, so every op is CUDA-graph capturable once its
workspace exists.

Workspaces: each device keeps one zero-initialised scratch buffer, grown on
demand outside graph capture (the kernels leave it reusable).  A buffer that
is outgrown stays allocated for the life of the process: a CUDA graph captured
while it was current keeps writing to it on every replay.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Tuple

import torch

from . import _lib

GROUP = 1024          # the reference op's compile-time group size (w4a8_ops.py:60)
_WS: Dict[int, torch.Tensor] = {}
# Every buffer ever handed out per device, current one last.  Graphs captured
# earlier hold the addresses of outgrown buffers; freeing those would let the
# caching allocator give their memory to other tensors that the replays then
# overwrite.
_WS_ALL: Dict[int, List[torch.Tensor]] = {}


def num_groups(K: int, group_size: int = GROUP) -> int:
    return -(-K // group_size)


def group_real(g: int, K: int, group_size: int = GROUP) -> int:
    G = num_groups(K, group_size)
    return group_size if g + 1 < G else K - (G - 1) * group_size


def k_pad_elems(K: int, group_size: int = GROUP) -> int:
    """Group-padded row length: each group rounded up to 64 elements (mg_kgeom.h:97-101)."""
    G = num_groups(K, group_size)
    stride = -(-group_size // 64) * 64
    last = -(-group_real(G - 1, K, group_size) // 64) * 64
    return (G - 1) * stride + last


def tile_m_for(m: int) -> int:
    """The reference's TileMFor (npu_ops/host/midgroup_quant_a.cpp:37)."""
    return 16 if m <= 16 else (64 if m <= 64 else 128)


def pad_rows(m: int) -> int:
    t = tile_m_for(m)
    return (m + t - 1) // t * t


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream_of(t: torch.Tensor) -> int:
    """The current stream of t's device, as a cudaStream_t value (the raw lookup
    skips the Python Stream object that current_stream() builds per call)."""
    if _raw_stream is not None:
        return _raw_stream(t.get_device())
    return _stream(t.device)


# workspace bytes per (M, N, K, group size): a pure function of the shape and
# the device's SM count (one process drives one kind of GPU)
_WS_BYTES: Dict[Tuple[int, int, int, int], int] = {}


def _ws_bytes(M: int, N: int, K: int, group_size: int) -> int:
    key = (M, N, K, group_size)
    n = _WS_BYTES.get(key)
    if n is None:
        n = _lib.lib().w4a8_linear_workspace_size(M, N, K, group_size)
        _WS_BYTES[key] = n
    return n


def _act_k(x: torch.Tensor, act: Optional[str]) -> int:
    """The linear's K for input x: its last dimension, or half of it for
    act="swiglu" (x = [gate | up])."""
    if act is None:
        return x.shape[-1]
    _check(act == "swiglu", f"w4a8 linear: unknown activation {act!r} (None or 'swiglu')")
    _check(x.shape[-1] % 2 == 0, "w4a8 linear: act='swiglu' needs x = [gate | up] with an even last dimension")
    return x.shape[-1] // 2


def workspace(nbytes: int, device: torch.device) -> Tuple[int, int]:
    """(aligned pointer, usable bytes) of this device's scratch buffer.

    One buffer per device: ops on one device are expected to run in stream
    order (CUDA-graph capture included).  Callers that run W4A8 ops
    concurrently on several streams of one device must give each stream its
    own buffer through the C ABI."""
    key = device.index if device.index is not None else torch.cuda.current_device()
    buf = _WS.get(key)
    need = nbytes + 1024
    if buf is None or buf.numel() < need:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError(
                f"w4a8 workspace of {nbytes} bytes must exist before CUDA graph capture; "
                "run the op once eagerly with the largest shape first")
        buf = torch.zeros(max(need, 1 << 20), dtype=torch.uint8, device=device)
        _WS[key] = buf
        _WS_ALL.setdefault(key, []).append(buf)
    base = buf.data_ptr()
    aligned = (base + 1023) & ~1023
    return aligned, buf.numel() - (aligned - base)


def workspace_status(device: Optional[torch.device] = None, reset: bool = True) -> int:
    """Device status word of this device's workspaces (0 = no kernel reported a
    failure): the first non-zero word among the current buffer and every
    outgrown one (graphs captured earlier still write to those)."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    workspace(0, device)
    key = device.index if device.index is not None else torch.cuda.current_device()
    status = 0
    for buf in _WS_ALL.get(key, []):
        ptr = (buf.data_ptr() + 1023) & ~1023
        v = _lib.lib().w4a8_workspace_status(ptr, 1 if reset else 0, _stream(device))
        status = status or v
    return status


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _check_cuda(*ts: Optional[torch.Tensor]) -> None:
    dev = None
    for t in ts:
        if t is None:
            continue
        _check(t.is_cuda, "w4a8 ops need CUDA tensors (there is no CPU implementation)")
        dev = dev or t.device
        _check(t.device == dev, "w4a8 ops: all tensors must be on one device")


# ---------------------------------------------------------------- quantiser

def quant_act(x: torch.Tensor, group_size: int, scale_dtype: torch.dtype = torch.bfloat16,
              with_ksum: bool = True):
    """x bf16 [M, K] -> (q int8 [M, K], scale [G, M], ksum int32 [G, M] negated or None)."""
    _check(x.dim() == 2, "quant_act: x must be [M, K]")
    _check(x.dtype == torch.bfloat16, "quant_act: x must be bfloat16")
    _check_cuda(x)
    x = x.contiguous()
    M, K = x.shape
    G = num_groups(K, group_size)
    q = torch.empty((M, K), dtype=torch.int8, device=x.device)
    s = torch.empty((G, M), dtype=scale_dtype, device=x.device)
    ks = torch.empty((G, M), dtype=torch.int32, device=x.device) if with_ksum else None
    sd = _lib.DTYPE_F32 if scale_dtype == torch.float32 else _lib.DTYPE_BF16
    _check(scale_dtype in (torch.float32, torch.bfloat16), "quant_act: scale dtype must be bf16 or f32")
    rc = _lib.lib().w4a8_quant_act(x.data_ptr(), M, K, K, group_size, q.data_ptr(), s.data_ptr(), sd,
                                   _ptr(ks), _stream(x.device))
    _lib.check(rc, "w4a8_quant_act")
    return q, s, ks


def midgroup_quant_a(x: torch.Tensor, group_size: int = GROUP) -> List[torch.Tensor]:
    """The reference op ``midgroup_quant_a(Tensor x) -> Tensor[]``
    (npu_ops/host/midgroup_quant_a.cpp:40-78): [a_hi, a_lo, a_scale, a_ksum]
    with M padded to the reference's TILE_M."""
    _check(x.dim() == 2, "midgroup_quant_a: x must be [M, K]")
    _check(x.dtype == torch.bfloat16, "midgroup_quant_a: x must be bfloat16")
    _check_cuda(x)
    x = x.contiguous()
    M, K = x.shape
    G, Kp, Mp = num_groups(K, group_size), k_pad_elems(K, group_size), pad_rows(M)
    dev = x.device
    a_hi = torch.empty((Mp, Kp // 2), dtype=torch.int8, device=dev)
    a_lo = torch.empty((Mp, Kp // 2), dtype=torch.int8, device=dev)
    a_scale = torch.empty((G, Mp), dtype=torch.bfloat16, device=dev)
    a_ksum = torch.empty((G, Mp), dtype=torch.int32, device=dev)
    rc = _lib.lib().w4a8_midgroup_quant_a(x.data_ptr(), M, K, group_size, Mp, a_hi.data_ptr(),
                                          a_lo.data_ptr(), a_scale.data_ptr(), a_ksum.data_ptr(),
                                          _stream(dev))
    _lib.check(rc, "w4a8_midgroup_quant_a")
    return [a_hi, a_lo, a_scale, a_ksum]


# ---------------------------------------------------------------- GEMMs

def midgroup_w4a8_gemm(a_hi, a_lo, a_scale, a_ksum, w_q, w_scale, w_ksum, w_zero, K: int,
                       group_size: int = GROUP) -> torch.Tensor:
    """The reference op ``midgroup_w4a8_gemm`` (npu_ops/host/midgroup_w4a8_gemm.cpp:143-238):
    y bf16 [a_hi.rows, N]."""
    _check(a_hi.dim() == 2 and a_lo.dim() == 2 and w_q.dim() == 2,
           "midgroup_w4a8_gemm: a_hi/a_lo [M,K/2] and w_q [N,K/2] must be 2-D")
    _check(a_hi.dtype == torch.int8 and a_lo.dtype == torch.int8 and w_q.dtype == torch.int8,
           "midgroup_w4a8_gemm: packed int4 planes must be int8 tensors")
    _check(a_scale.dtype == torch.bfloat16 and w_scale.dtype == torch.bfloat16 and
           (w_zero is None or w_zero.dtype == torch.bfloat16),
           "midgroup_w4a8_gemm: a_scale/w_scale/w_zero must be bfloat16")
    _check((a_ksum is None or a_ksum.dtype == torch.int32) and (w_ksum is None or w_ksum.dtype == torch.int32),
           "midgroup_w4a8_gemm: a_ksum/w_ksum must be int32")
    _check_cuda(a_hi, a_lo, a_scale, a_ksum, w_q, w_scale, w_ksum, w_zero)
    M, N = a_hi.shape[0], w_q.shape[0]
    Kb = k_pad_elems(K, group_size) // 2
    _check(a_hi.shape[1] == Kb and a_lo.shape[1] == Kb and w_q.shape[1] == Kb,
           f"midgroup_w4a8_gemm: packed row length must be Kpad/2 = {Kb} for K={K} "
           f"(group-padded layout); got a_hi {a_hi.shape[1]} w_q {w_q.shape[1]}")
    _check(N % 8 == 0, f"midgroup_w4a8_gemm: N must be a multiple of 8; got {N}")
    G = num_groups(K, group_size)
    _check(tuple(a_scale.shape) == (G, M), "midgroup_w4a8_gemm: a_scale must be group-major [K/group, M]")
    _check(tuple(w_scale.shape) == (G, N), "midgroup_w4a8_gemm: w_scale must be group-major [K/group, N]")
    _check(w_zero is None or tuple(w_zero.shape) == (G, N), "midgroup_w4a8_gemm: w_zero must be [K/group, N]")
    a_hi, a_lo, a_scale, w_q, w_scale = (t.contiguous() for t in (a_hi, a_lo, a_scale, w_q, w_scale))
    w_zero = None if w_zero is None else w_zero.contiguous()
    y = torch.empty((M, N), dtype=torch.bfloat16, device=a_hi.device)
    L = _lib.lib()
    ws, wsb = workspace(L.w4a8_midgroup_gemm_workspace_size(M, N, K, group_size), a_hi.device)
    rc = L.w4a8_midgroup_w4a8_gemm(a_hi.data_ptr(), a_lo.data_ptr(), a_scale.data_ptr(), _ptr(a_ksum), M,
                                   w_q.data_ptr(), w_scale.data_ptr(), _ptr(w_ksum), _ptr(w_zero), N, K,
                                   group_size, y.data_ptr(), ws, wsb, _stream(a_hi.device))
    _lib.check(rc, "w4a8_midgroup_w4a8_gemm")
    return y


def _check_weight(w_packed, w_scale, w_zero, K, group_size):
    N = w_packed.shape[0]
    G, Kb = num_groups(K, group_size), k_pad_elems(K, group_size) // 2
    _check(w_packed.dtype == torch.int8 and w_packed.dim() == 2 and w_packed.shape[1] == Kb,
           f"w4a8 linear: w_packed must be int8 [N, {Kb}] for K={K}, group {group_size}")
    _check(w_scale.dtype in (torch.bfloat16, torch.float32) and tuple(w_scale.shape) == (G, N),
           f"w4a8 linear: w_scale must be bf16/f32 [{G}, {N}] (group-major)")
    _check(w_zero is None or (w_zero.dtype == torch.bfloat16 and tuple(w_zero.shape) == (G, N)),
           f"w4a8 linear: w_zero must be bf16 [{G}, {N}]")
    _check(N % 8 == 0, f"w4a8 linear: N must be a multiple of 8; got {N}")
    return N


def linear(x: torch.Tensor, w_packed: torch.Tensor, w_scale: torch.Tensor,
           w_zero: Optional[torch.Tensor], group_size: int, out: Optional[torch.Tensor] = None,
           act: Optional[str] = None) -> torch.Tensor:
    """y = x @ W^T for packed int4 W with per-group scales (and zero points):
    the activation is quantised per (token, group) inside the op.  With
    act="swiglu", x = [gate | up] and the op computes bf16(silu(gate) * up) @ W^T
    (the activation is applied by the quantiser as it reads x)."""
    _check(x.dtype == torch.bfloat16, "w4a8 linear: x must be bfloat16")
    _check_cuda(x, w_packed, w_scale, w_zero)
    K = _act_k(x, act)
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    M = x2.shape[0]
    N = _check_weight(w_packed, w_scale, w_zero, K, group_size)
    y = out if out is not None else torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    if M == 0:
        return y.reshape(*lead, N)
    L = _lib.lib()
    ws, wsb = workspace(_ws_bytes(M, N, K, group_size), x.device)
    sd = _lib.DTYPE_F32 if w_scale.dtype == torch.float32 else _lib.DTYPE_BF16
    fn = L.w4a8_linear if act is None else L.w4a8_linear_swiglu
    rc = fn(x2.data_ptr(), M, K, x2.stride(0), N, group_size, w_packed.data_ptr(),
            w_scale.data_ptr(), sd, _ptr(w_zero), y.data_ptr(), y.stride(0), ws, wsb, _stream_of(x2))
    _lib.check(rc, "w4a8_linear" if act is None else "w4a8_linear_swiglu")
    return y.reshape(*lead, N)


def linear_quant(x2: torch.Tensor, N: int, group_size: int) -> None:
    """First half of ``linear``: quantise x into this stream's workspace."""
    M, K = x2.shape
    L = _lib.lib()
    ws, wsb = workspace(_ws_bytes(M, N, K, group_size), x2.device)
    rc = L.w4a8_linear_quant(x2.data_ptr(), M, K, x2.stride(0), N, group_size, ws, wsb, _stream(x2.device))
    _lib.check(rc, "w4a8_linear_quant")


def linear_gemm(M: int, K: int, w_packed, w_scale, w_zero, group_size: int, y: torch.Tensor) -> None:
    """Second half of ``linear``: the GEMM on the activation ``linear_quant`` left behind."""
    N = w_packed.shape[0]
    L = _lib.lib()
    ws, wsb = workspace(L.w4a8_linear_workspace_size(M, N, K, group_size), y.device)
    sd = _lib.DTYPE_F32 if w_scale.dtype == torch.float32 else _lib.DTYPE_BF16
    rc = L.w4a8_linear_gemm(M, K, N, group_size, w_packed.data_ptr(), w_scale.data_ptr(), sd, _ptr(w_zero),
                            y.data_ptr(), y.stride(0), ws, wsb, _stream(y.device))
    _lib.check(rc, "w4a8_linear_gemm")


class PreparedWeight:
    """A linear layer's weights regrouped once into the GEMM's tile order
    (``w4a8_prepare_weights``): the same values as (w_packed, w_scale, w_zero),
    read by the kernel with one bulk copy per pipeline stage."""

    __slots__ = ("buf", "N", "K", "group_size", "ws_dtype", "has_zero")

    def __init__(self, buf: torch.Tensor, N: int, K: int, group_size: int, ws_dtype: int, has_zero: bool):
        self.buf, self.N, self.K, self.group_size = buf, N, K, group_size
        self.ws_dtype, self.has_zero = ws_dtype, has_zero

    def ptr(self) -> int:
        return (self.buf.data_ptr() + 255) & ~255


def prepare_weights(w_packed: torch.Tensor, w_scale: torch.Tensor, w_zero: Optional[torch.Tensor],
                    K: int, group_size: int) -> PreparedWeight:
    """Regroup reference-layout weights for the bulk-copy GEMM path (one-time, like
    ``process_weights_after_loading`` in npu_ops/python/midgroup_quant.py:148-161)."""
    _check_cuda(w_packed, w_scale, w_zero)
    N = _check_weight(w_packed, w_scale, w_zero, K, group_size)
    w_packed, w_scale = w_packed.contiguous(), w_scale.contiguous()
    w_zero = None if w_zero is None else w_zero.contiguous()
    sd = _lib.DTYPE_F32 if w_scale.dtype == torch.float32 else _lib.DTYPE_BF16
    L = _lib.lib()
    nbytes = L.w4a8_prepared_weights_size(N, K, group_size, sd, 1 if w_zero is not None else 0)
    _check(nbytes > 0, "prepare_weights: unsupported shape")
    buf = torch.empty(nbytes + 256, dtype=torch.uint8, device=w_packed.device)
    pw = PreparedWeight(buf, N, K, group_size, sd, w_zero is not None)
    rc = L.w4a8_prepare_weights(w_packed.data_ptr(), w_scale.data_ptr(), sd, _ptr(w_zero), N, K, group_size,
                                pw.ptr(), nbytes, _stream(w_packed.device))
    _lib.check(rc, "w4a8_prepare_weights")
    return pw


def linear_prepared(x: torch.Tensor, pw: PreparedWeight, out: Optional[torch.Tensor] = None,
                    act: Optional[str] = None) -> torch.Tensor:
    """``linear`` on prepared weights (bit-identical results).  The per-call
    host work is kept to the checks the kernels need, one cached workspace
    lookup and one C call: decode steps make many small calls."""
    if x.dtype != torch.bfloat16:
        raise RuntimeError("w4a8 linear: x must be bfloat16")
    if not x.is_cuda or x.device != pw.buf.device:
        raise RuntimeError("w4a8 ops need CUDA tensors on the weights' device (there is no CPU implementation)")
    K = pw.K
    if x.shape[-1] != (K if act is None else 2 * K):
        _act_k(x, act)
        raise RuntimeError(f"w4a8 linear: x has last dimension {x.shape[-1]}, weights were prepared for K={K}"
                           + (" (act='swiglu' takes [gate | up] = 2K)" if act else ""))
    x2 = x if x.dim() == 2 else x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    M, N = x2.shape[0], pw.N
    y = out if out is not None else torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    if M == 0:
        return y.reshape(*x.shape[:-1], N)
    ws, wsb = workspace(_ws_bytes(M, N, K, pw.group_size), x.device)
    L = _lib.lib()
    fn = L.w4a8_linear_prepared if act is None else L.w4a8_linear_prepared_swiglu
    rc = fn(x2.data_ptr(), M, K, x2.stride(0), N, pw.group_size, pw.ptr(), pw.ws_dtype,
            1 if pw.has_zero else 0, y.data_ptr(), y.stride(0), ws, wsb, _stream_of(x2))
    if rc != 0:
        _lib.check(rc, "w4a8_linear_prepared" if act is None else "w4a8_linear_prepared_swiglu")
    return y if x.dim() == 2 else y.reshape(*x.shape[:-1], N)


def linear_gemm_prepared(M: int, pw: PreparedWeight, y: torch.Tensor) -> None:
    """Second half of ``linear_prepared`` after ``linear_quant(x2, pw.N, pw.group_size)``."""
    L = _lib.lib()
    ws, wsb = workspace(_ws_bytes(M, pw.N, pw.K, pw.group_size), y.device)
    rc = L.w4a8_linear_gemm_prepared(M, pw.K, pw.N, pw.group_size, pw.ptr(), pw.ws_dtype,
                                     1 if pw.has_zero else 0, y.data_ptr(), y.stride(0), ws, wsb,
                                     _stream(y.device))
    _lib.check(rc, "w4a8_linear_gemm_prepared")


def group_partials(x: torch.Tensor, w_packed: torch.Tensor, w_zero: Optional[torch.Tensor],
                   group_size: int) -> torch.Tensor:
    """int32 P[G, M, N] = sum_{k in g} A_q * (W - wz), from the tensor-core path."""
    _check(x.dim() == 2 and x.dtype == torch.bfloat16, "group_partials: x must be bf16 [M, K]")
    _check_cuda(x, w_packed, w_zero)
    x = x.contiguous()
    M, K = x.shape
    N = w_packed.shape[0]
    G = num_groups(K, group_size)
    P = torch.empty((G, M, N), dtype=torch.int32, device=x.device)
    L = _lib.lib()
    ws, wsb = workspace(L.w4a8_linear_workspace_size(M, N, K, group_size), x.device)
    rc = L.w4a8_group_partials(x.data_ptr(), M, K, K, N, group_size, w_packed.data_ptr(), _ptr(w_zero),
                               P.data_ptr(), ws, wsb, _stream(x.device))
    _lib.check(rc, "w4a8_group_partials")
    return P


# ---------------------------------------------------------------- weight packing (device-agnostic torch)

def pack_int4(v: torch.Tensor) -> torch.Tensor:
    """[..., K] int8 codes in [-8,7] -> [..., K/2], even index in the LOW nibble
    (npu_ops/python/w4a8_ops.py:142-148)."""
    _check(v.shape[-1] % 2 == 0, "K must be even to pack int4")
    lo = v[..., 0::2].to(torch.int16) & 0xF
    hi = v[..., 1::2].to(torch.int16) & 0xF
    return (lo | (hi << 4)).to(torch.uint8).view(torch.int8)


def pack_int4_grouped(codes: torch.Tensor, group_size: int) -> torch.Tensor:
    """codes [N, K] -> packed [N, Kpad/2] in the group-padded layout (w4a8_ops.py:231-239)."""
    N, K = codes.shape
    G = num_groups(K, group_size)
    kpad = k_pad_elems(K, group_size)
    stride = -(-group_size // 64) * 64
    if kpad == K and stride == group_size:
        return pack_int4(codes.to(torch.int8))
    padded = codes.new_zeros((N, kpad), dtype=torch.int8)
    for g in range(G):
        real = group_real(g, K, group_size)
        padded[:, g * stride:g * stride + real] = codes[:, g * group_size:g * group_size + real]
    return pack_int4(padded)


def unpack_int4_grouped(packed: torch.Tensor, K: int, group_size: int) -> torch.Tensor:
    """Inverse of ``pack_int4_grouped`` (export_w4a8_checkpoint.py:59-66 for the aligned case)."""
    b = packed.view(torch.uint8).to(torch.int16)
    lo = b & 0xF
    hi = (b >> 4) & 0xF
    v = torch.stack([lo, hi], dim=-1).reshape(packed.shape[0], -1)
    v = torch.where(v >= 8, v - 16, v).to(torch.int8)
    G = num_groups(K, group_size)
    stride = -(-group_size // 64) * 64
    parts = [v[:, g * stride:g * stride + group_real(g, K, group_size)] for g in range(G)]
    return torch.cat(parts, dim=1)
