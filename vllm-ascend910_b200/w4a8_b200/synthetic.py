"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (QwQ-32B projection shapes; no real checkpoint or
dataset is involved).

* weights: int4 codes uniform in [-8, 7] (symmetric), or uint4 codes uniform in
  [0, 15] with an integer zero point uniform in [6, 9] (asymmetric).  The
  asymmetric form is stored the reference's way: signed nibble ``q_u - 8`` and
  a signed zero point ``z_u - 8`` in code units (``q_u - z_u == q_s - z_s``),
  matching ``fakequant_lab/quant.py:106-113``.
* per-group, per-output-channel weight scales: ``exp(N(-6, 0.5))``, fp32 (or
  rounded to bf16 for the checkpoint-format variants).
* activations: bf16 ``N(0, 1)`` with 0.5 % of the K channels (the same channels
  for every row) multiplied by 20.

``numpy`` generators are bit-reproducible on any machine and feed the parity
tests; the ``torch`` generators build full-size inputs directly on a GPU for
the benchmark.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import numpy as np

# (K, N) of the four QwQ-32B projections (hidden 5120, FFN 27648, 40 q heads
# + 8 kv heads of 128).
QWQ_SHAPES = {
    "qkv": (5120, 7168),
    "o": (5120, 5120),
    "gate_up": (5120, 55296),
    "down": (27648, 5120),
}
DECODE_MS = (1, 4, 8, 16, 32, 64)
PREFILL_MS = (1024, 2048, 4096, 8192)


def _f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return r.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


@dataclass
class SynthWeight:
    codes: np.ndarray            # [N, K] int8 in [-8, 7]
    scale: np.ndarray            # [G, N] float32 (bf16-exact when scale_bf16)
    zero: Optional[np.ndarray]   # [G, N] float32 integer zero points, or None
    gk: int


def activation_np(M: int, K: int, seed: int, outlier_frac: float = 0.005,
                  outlier_mult: float = 20.0) -> np.ndarray:
    """bf16 bits [M, K]."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K), dtype=np.float32)
    n_out = max(1, int(round(outlier_frac * K)))
    ch = rng.choice(K, size=n_out, replace=False)
    x[:, ch] *= np.float32(outlier_mult)
    return _f32_to_bf16_bits(x)


def weight_np(N: int, K: int, gk: int, seed: int, asym: bool = False,
              scale_bf16: bool = False) -> SynthWeight:
    rng = np.random.default_rng(seed)
    G = -(-K // gk)
    if asym:
        qu = rng.integers(0, 16, size=(N, K), dtype=np.int16)
        zu = rng.integers(6, 10, size=(G, N), dtype=np.int16)
        codes = (qu - 8).astype(np.int8)
        zero = (zu - 8).astype(np.float32)
    else:
        codes = rng.integers(-8, 8, size=(N, K), dtype=np.int16).astype(np.int8)
        zero = None
    scale = np.exp(rng.normal(-6.0, 0.5, size=(G, N))).astype(np.float32)
    if scale_bf16:
        scale = bf16_bits_to_f32(_f32_to_bf16_bits(scale))
    return SynthWeight(codes, scale, zero, gk)


# ------------------------------------------------------------------ torch, on device

def activation_torch(M: int, K: int, seed: int, device, outlier_frac: float = 0.005,
                     outlier_mult: float = 20.0):
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(M, K, generator=g, device=device, dtype=torch.float32)
    n_out = max(1, int(round(outlier_frac * K)))
    ch = torch.randperm(K, generator=g, device=device)[:n_out]
    x[:, ch] *= outlier_mult
    return x.to(torch.bfloat16)


def weight_torch(N: int, K: int, gk: int, seed: int, device, asym: bool = False,
                 scale_dtype=None):
    """(codes int8 [N,K], scale [G,N], zero [G,N] bf16 or None) on ``device``."""
    import torch
    scale_dtype = scale_dtype or torch.float32
    g = torch.Generator(device=device).manual_seed(seed)
    G = -(-K // gk)
    if asym:
        codes = (torch.randint(0, 16, (N, K), generator=g, device=device, dtype=torch.int16) - 8).to(torch.int8)
        zero = (torch.randint(6, 10, (G, N), generator=g, device=device, dtype=torch.int16) - 8).to(torch.bfloat16)
    else:
        codes = torch.randint(-8, 8, (N, K), generator=g, device=device, dtype=torch.int16).to(torch.int8)
        zero = None
    scale = torch.exp(torch.randn(G, N, generator=g, device=device) * 0.5 - 6.0).to(scale_dtype)
    return codes, scale, zero
