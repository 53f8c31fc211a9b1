"""The reference's W4A8 op module (npu_ops/python/w4a8_ops.py) on the B200 kernels.

Same names, arguments and layouts:

    load()                                      registers the torch ops (idempotent)
    torch.ops.npu.midgroup_quant_a(x) -> [a_hi, a_lo, a_scale, a_ksum]
    torch.ops.npu.midgroup_w4a8_gemm(a_hi, a_lo, a_scale, a_ksum, w_q, w_scale, w_ksum, w_zero, K) -> y
    quantize_weight(w, group) -> (w_q, w_scale, w_ksum, w_zero)   kernel layout, [G, N] scales
    linear(x, wq, ws, wk, wz) -> y
    GROUP, tile_m_for, pad_rows, num_groups, group_real, k_pad_elems, pack_int4

The ``npu`` namespace ops keep the reference's signatures (group size 1024, the
reference's compile-time constant).  The same ops, with the group size as an
argument, are registered as ``torch.ops.w4a8.*`` together with the fused
``torch.ops.w4a8.linear``.  Every op has a fake (meta) kernel so the ops trace
under FakeTensor / torch.compile / CUDA-graph capture the way the reference's
do (w4a8_ops.py:96-128).  There is no CPU kernel: calling an op on CPU tensors
raises.
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch

from . import ops
from .ops import GROUP, group_real, k_pad_elems, num_groups, pack_int4, pad_rows, tile_m_for

__all__ = ["GROUP", "tile_m_for", "pad_rows", "load", "num_groups", "group_real", "k_pad_elems",
           "pack_int4", "quantize_weight", "linear", "QMIN", "QMAX"]

QMAX = {4: 7, 8: 127}
QMIN = {4: -8, 8: -128}

_LIBS: List[torch.library.Library] = []
_LOADED = False


def _quant_a_impl(x: torch.Tensor, group_size: int) -> List[torch.Tensor]:
    return ops.midgroup_quant_a(x, group_size)


def _quant_a_fake(x: torch.Tensor, group_size: int) -> List[torch.Tensor]:
    M, K = x.shape
    G, Kp, Mp = num_groups(K, group_size), k_pad_elems(K, group_size), pad_rows(M)
    return [x.new_empty((Mp, Kp // 2), dtype=torch.int8), x.new_empty((Mp, Kp // 2), dtype=torch.int8),
            x.new_empty((G, Mp), dtype=torch.bfloat16), x.new_empty((G, Mp), dtype=torch.int32)]


def _gemm_impl(a_hi, a_lo, a_scale, a_ksum, w_q, w_scale, w_ksum, w_zero, K: int, group_size: int):
    return ops.midgroup_w4a8_gemm(a_hi, a_lo, a_scale, a_ksum, w_q, w_scale, w_ksum, w_zero, K, group_size)


def _gemm_fake(a_hi, a_lo, a_scale, a_ksum, w_q, w_scale, w_ksum, w_zero, K: int, group_size: int):
    return a_scale.new_empty((a_hi.shape[0], w_q.shape[0]), dtype=torch.bfloat16)


def _linear_impl(x, w_packed, w_scale, w_zero, group_size: int):
    return ops.linear(x, w_packed, w_scale, w_zero, group_size)


def _linear_fake(x, w_packed, w_scale, w_zero, group_size: int):
    return x.new_empty((*x.shape[:-1], w_packed.shape[0]), dtype=torch.bfloat16)


def load() -> None:
    """Register the ops (idempotent): ``torch.ops.w4a8.*`` always, and the
    reference's ``torch.ops.npu.midgroup_*`` names when no other library owns
    them.  Checks that the CUDA library is present (there is no CPU fallback)."""
    global _LOADED
    if _LOADED:
        return
    from . import _lib
    _lib.lib()
    w = torch.library.Library("w4a8", "DEF")
    w.define("midgroup_quant_a(Tensor x, int group_size=1024) -> Tensor[]")
    w.define("midgroup_w4a8_gemm(Tensor a_hi, Tensor a_lo, Tensor a_scale, Tensor? a_ksum, Tensor w_q, "
             "Tensor w_scale, Tensor? w_ksum, Tensor? w_zero, int K, int group_size=1024) -> Tensor")
    w.define("linear(Tensor x, Tensor w_packed, Tensor w_scale, Tensor? w_zero, int group_size) -> Tensor")
    w.impl("midgroup_quant_a", _quant_a_impl, "CUDA")
    w.impl("midgroup_w4a8_gemm", _gemm_impl, "CUDA")
    w.impl("linear", _linear_impl, "CUDA")
    torch.library.register_fake("w4a8::midgroup_quant_a", _quant_a_fake, lib=w)
    torch.library.register_fake("w4a8::midgroup_w4a8_gemm", _gemm_fake, lib=w)
    torch.library.register_fake("w4a8::linear", _linear_fake, lib=w)
    _LIBS.append(w)
    if not hasattr(torch.ops.npu, "midgroup_quant_a"):
        n = torch.library.Library("npu", "FRAGMENT")
        n.define("midgroup_quant_a(Tensor x) -> Tensor[]")
        n.define("midgroup_w4a8_gemm(Tensor a_hi, Tensor a_lo, Tensor a_scale, Tensor a_ksum, Tensor w_q, "
                 "Tensor w_scale, Tensor w_ksum, Tensor w_zero, int K) -> Tensor")
        n.impl("midgroup_quant_a", lambda x: _quant_a_impl(x, GROUP), "CUDA")
        n.impl("midgroup_w4a8_gemm",
               lambda a, b, c, d, e, f, g, h, K: _gemm_impl(a, b, c, d, e, f, g, h, K, GROUP), "CUDA")
        torch.library.register_fake("npu::midgroup_quant_a", lambda x: _quant_a_fake(x, GROUP), lib=n)
        torch.library.register_fake("npu::midgroup_w4a8_gemm",
                                    lambda a, b, c, d, e, f, g, h, K: _gemm_fake(a, b, c, d, e, f, g, h, K, GROUP),
                                    lib=n)
        _LIBS.append(n)
    _LOADED = True


# ---------------------------------------------------------------- weight quantiser

def _tiny_where_zero(scale: torch.Tensor) -> torch.Tensor:
    return torch.where(scale == 0, torch.full_like(scale, torch.finfo(torch.bfloat16).tiny), scale)


def group_params_asym(xg: torch.Tensor, bits: int = 4) -> Tuple[torch.Tensor, torch.Tensor]:
    """(scale, zero) of one asymmetric group (fakequant_lab/quant.py:89-133):
    scale = bf16((max - min) / (2^bits - 1)) (bf16 tiny when 0) and
    zero = bf16(QMIN - round(min / scale)); a constant group gets
    scale = bf16(|v| / QMAX), zero = 0."""
    qmax, qmin = QMAX[bits], QMIN[bits]
    mx = xg.amax(dim=-1, keepdim=True)
    mn = xg.amin(dim=-1, keepdim=True)
    rng = mx - mn
    scale = _tiny_where_zero((rng / (qmax - qmin)).to(torch.bfloat16))
    zero = (float(qmin) - torch.round(mn / scale.float())).to(torch.bfloat16)
    const = rng == 0
    scale = torch.where(const, _tiny_where_zero((mx.abs() / qmax).to(torch.bfloat16)), scale)
    zero = torch.where(const, torch.zeros_like(zero), zero)
    return scale, zero


def _quantize_asym(x: torch.Tensor, gl: int):
    """x [N, G*gl] -> codes int8 [N, G*gl], scale bf16 [N, G], zero bf16 [N, G]
    (fakequant_lab/quant.py:143-173 with an asymmetric int4 spec)."""
    N, K = x.shape
    xg = x.float().reshape(N, K // gl, gl)
    scale, zero = group_params_asym(xg)
    q = torch.round(xg / scale.float()) + zero.float()
    q = q.clamp_(QMIN[4], QMAX[4]).to(torch.int8)
    return q.reshape(N, K), scale.squeeze(-1), zero.squeeze(-1)


def quantize_weight(w: torch.Tensor, group: int = GROUP
                    ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """bf16 [N, K] -> (w_q packed int4 [N, Kpad/2], w_scale bf16 [G, N],
    w_ksum int32 [G, N], w_zero bf16 [G, N]) in the kernel layout
    (npu_ops/python/w4a8_ops.py:181-240).

    Asymmetric int4 per group along K; a ragged last group is quantised on its
    real members only, then zero-padded to 64 elements in the packed layout.
    ``w_ksum`` is the per-group sum of the raw codes (the reference's MSD term)."""
    N, K = w.shape
    G = num_groups(K, group)
    k_full = (G - 1) * group
    parts_q, parts_s, parts_z = [], [], []
    if k_full:
        q, s, z = _quantize_asym(w[:, :k_full], group)
        parts_q.append(q)
        parts_s.append(s)
        parts_z.append(z)
    q, s, z = _quantize_asym(w[:, k_full:], K - k_full)
    parts_q.append(q)
    parts_s.append(s)
    parts_z.append(z)
    codes = torch.cat(parts_q, dim=1)
    w_scale = torch.cat(parts_s, dim=1).T.contiguous()
    w_zero = torch.cat(parts_z, dim=1).T.contiguous()
    ksum = torch.stack([codes[:, g * group:g * group + group_real(g, K, group)].to(torch.int32).sum(dim=1)
                        for g in range(G)], dim=1)
    w_ksum = ksum.to(torch.int32).T.contiguous()
    w_q = ops.pack_int4_grouped(codes, group)
    return w_q, w_scale, w_ksum, w_zero


def linear(x: torch.Tensor, wq: torch.Tensor, ws: torch.Tensor, wk: Optional[torch.Tensor],
           wz: Optional[torch.Tensor], group: int = GROUP) -> torch.Tensor:
    """y = x @ W.T with mid-group W4A8; x is bf16 [..., K] (w4a8_ops.py:243-252).

    ``wk`` (the raw-code sums) only matters to the MSD form of the reference's
    kernel and is ignored here: the B200 kernel multiplies int8 by (W - zero)
    directly."""
    load()
    lead, K = x.shape[:-1], x.shape[-1]
    y = torch.ops.w4a8.linear(x.reshape(-1, K).to(torch.bfloat16), wq, ws, wz, group)
    return y.reshape(*lead, wq.shape[0])
