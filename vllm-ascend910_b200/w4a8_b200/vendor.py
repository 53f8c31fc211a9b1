"""Vendor ``W4A8_DYNAMIC`` (group-wise int4) projections -> the mid-group kernel layout.

The vendor checkpoint stores, per projection (the reference's structural
builder, scripts/build_random_w4a8.py:102-147):

    <proj>.weight                int8  [N/2, K]  two signed int4 codes per byte along the OUTPUT axis
    <proj>.weight_scale          fp32  [N, 1]    per-channel scale
    <proj>.weight_offset         fp32  [N, 1]    per-channel offset
    <proj>.weight_scale_second   fp16  [N, K/gs] per-group scale
    <proj>.weight_offset_second  fp16  [N, K/gs] per-group offset (code units)
    <proj>.scale_bias            fp32  [N, 1]    ([N, 16] for row-parallel projections)

with gs = 64 or 128 (``quant_description.group_size``).  Converted once at load
into the layout the B200 GEMM reads, so vendor checkpoints run on the same
kernel:

    w_packed  int8  [N, Kpad/2]  two codes per byte along K, even k in the low nibble
    w_scale   fp32  [G, N]       weight_scale[n] * weight_scale_second[n, g], kept in fp32
    w_zero    bf16  [G, N]       weight_offset_second (integers), or None when all zero

Interpretation (the reference documents the tensors, not their arithmetic):
w[n, k] = weight_scale[n] * weight_scale_second[n, g(k)] * (code[n, k] -
weight_offset_second[n, g(k)]); the low nibble of byte [i, k] holds output row
2i and the high nibble row 2i + 1 (``low_first=False`` swaps them).  A
per-channel offset or a non-zero ``scale_bias`` has no place in this layout,
and the conversion refuses it rather than dropping it.
"""
from __future__ import annotations

from typing import Callable, Dict, Optional, Sequence

import torch

from . import ops

SUFFIXES = ("weight", "weight_scale", "weight_offset", "weight_scale_second", "weight_offset_second",
            "scale_bias")


def unpack_output_axis(packed: torch.Tensor, low_first: bool = True) -> torch.Tensor:
    """int8 [N/2, K] -> int8 codes [N, K] in [-8, 7] (rows interleaved 2i, 2i+1)."""
    b = packed.to(torch.int16) & 0xFF
    lo = b & 0xF
    hi = (b >> 4) & 0xF
    first, second = (lo, hi) if low_first else (hi, lo)
    codes = torch.stack([first, second], dim=1).reshape(2 * packed.shape[0], packed.shape[1])
    return torch.where(codes >= 8, codes - 16, codes).to(torch.int8)


def pack_output_axis(codes: torch.Tensor, low_first: bool = True) -> torch.Tensor:
    """int8 codes [N, K] in [-8, 7] (N even) -> int8 [N/2, K]; inverse of unpack_output_axis."""
    if codes.shape[0] % 2:
        raise ValueError("N must be even to pack along the output axis")
    c = codes.to(torch.int16) & 0xF
    even, odd = c[0::2], c[1::2]
    lo, hi = (even, odd) if low_first else (odd, even)
    return ((hi << 4) | lo).to(torch.uint8).view(torch.int8)


def convert_projection(t: Dict[str, torch.Tensor], group: int, low_first: bool = True) -> Dict[str, Optional[torch.Tensor]]:
    """One vendor projection (its six tensors, keyed by suffix) -> kernel tensors."""
    packed = t["weight"]
    if packed.dtype != torch.int8 or packed.dim() != 2:
        raise ValueError("weight must be int8 [N/2, K]")
    N, K = 2 * packed.shape[0], packed.shape[1]
    if K % group:
        raise ValueError(f"K = {K} is not a multiple of the group size {group}")
    G = K // group
    s2 = t["weight_scale_second"].float()
    o2 = t["weight_offset_second"].float()
    if tuple(s2.shape) != (N, G) or tuple(o2.shape) != (N, G):
        raise ValueError(f"per-group tensors must be [N, K/gs] = [{N}, {G}]")
    s1 = t["weight_scale"].float().reshape(N, -1)
    if s1.shape[1] != 1:
        raise ValueError("weight_scale must be per channel [N, 1]")
    if "weight_offset" in t and bool(torch.any(t["weight_offset"].float() != 0)):
        raise ValueError("a per-channel weight_offset cannot be folded into the mid-group layout")
    if "scale_bias" in t and bool(torch.any(t["scale_bias"].float() != 0)):
        raise ValueError("a non-zero scale_bias cannot be folded into the mid-group layout")
    if not bool(torch.all(o2 == torch.round(o2))):
        raise ValueError("weight_offset_second must hold integers (code units)")
    codes = unpack_output_axis(packed, low_first)
    w_packed = ops.pack_int4_grouped(codes, group)
    w_scale = (s1 * s2).t().contiguous()                       # fp32 [G, N]
    w_zero = o2.t().contiguous().to(torch.bfloat16) if bool(torch.any(o2 != 0)) else None
    return {"w_packed": w_packed, "w_scale": w_scale, "w_zero": w_zero, "K": K, "N": N, "group": group}


def load_projection(get: Callable[[str], torch.Tensor], names: Sequence[str], group: int,
                    low_first: bool = True) -> Dict[str, Optional[torch.Tensor]]:
    """Convert and concatenate (along N) the named vendor projections, e.g. the
    q/k/v or gate/up members of one fused linear."""
    parts = []
    for name in names:
        t = {}
        for suf in SUFFIXES:
            try:
                t[suf] = get(f"{name}.{suf}")
            except KeyError:
                if suf in ("weight_offset", "scale_bias"):
                    continue
                raise
        parts.append(convert_projection(t, group, low_first))
    if len(parts) == 1:
        return parts[0]
    K = parts[0]["K"]
    if any(p["K"] != K for p in parts):
        raise ValueError("fused members must share K")
    zero = None
    if any(p["w_zero"] is not None for p in parts):
        zero = torch.cat([p["w_zero"] if p["w_zero"] is not None else
                          torch.zeros(p["w_scale"].shape, dtype=torch.bfloat16) for p in parts], 1)
    return {"w_packed": torch.cat([p["w_packed"] for p in parts], 0),
            "w_scale": torch.cat([p["w_scale"] for p in parts], 1), "w_zero": zero,
            "K": K, "N": sum(p["N"] for p in parts), "group": group}


def prepare(conv: Dict[str, Optional[torch.Tensor]], device) -> "ops.PreparedWeight":
    """The converted projection regrouped into the GEMM's tile order on ``device``."""
    zero = None if conv["w_zero"] is None else conv["w_zero"].to(device)
    return ops.prepare_weights(conv["w_packed"].to(device), conv["w_scale"].to(device), zero,
                               conv["K"], conv["group"])


def dequantize(conv: Dict[str, Optional[torch.Tensor]]) -> torch.Tensor:
    """fp32 [N, K] weights the converted tensors represent (for checks)."""
    K, g = conv["K"], conv["group"]
    codes = ops.unpack_int4_grouped(conv["w_packed"], K, g).float()
    sc = conv["w_scale"].float().t().repeat_interleave(g, 1)[:, :K]
    z = conv["w_zero"].float().t().repeat_interleave(g, 1)[:, :K] if conv["w_zero"] is not None else 0.0
    return (codes - z) * sc


__all__ = ["SUFFIXES", "unpack_output_axis", "pack_output_axis", "convert_projection", "load_projection",
           "prepare", "dequantize"]
