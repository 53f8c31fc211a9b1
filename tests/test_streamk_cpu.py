"""Stream-K partition rules shared by the GEMM, its fix-up kernel and the host
planner, restated on the CPU and checked against each other.

- Planner (`make_plan`, csrc/w4a8_capi.cu): token tile TT by M, units per
  output tile upt (two-k-block stages for TT <= 32 and GK <= 256, one k-block
  for larger tiles, one group for GK = 1024), grid = min(SMs, units), and
  `split` = some CTA boundary falls inside an output tile.
- GEMM (`cta_range`, `cta_of_unit`, `flush_tile`, csrc/w4a8_gemm.cu): CTA c
  owns units [c*U/C, (c+1)*U/C); a CTA that holds only part of a tile writes
  its fp32 part into slot side 0 when the tile is its first tile, else side 1.
- Fix-up (`splitk_reduce_kernel`): for a split tile it sums the parts of CTAs
  cf..cl, reading side 0 for every CTA after the first and, for the first CTA,
  side 0 only when that CTA's range starts at the tile -- the rule it uses to
  do its integer divisions before waiting for the GEMM.

The last rule must pick exactly the slot flush_tile wrote, for every split
tile of every plan; a mismatch would read a stale part.
"""
import random

import pytest

SMS = 148
QWQ = {"qkv": (5120, 7168), "o": (5120, 5120), "gate_up": (5120, 55296), "down": (27648, 5120)}


def cdiv(a, b):
    return -(-a // b)


def kpad(K, gk):
    """Each group padded to a multiple of 64 elements (mg_kgeom.h)."""
    G = cdiv(K, gk)
    last = K - (G - 1) * gk
    return (G - 1) * gk + cdiv(last, 64) * 64


def plan(M, N, K, gk, sms=SMS):
    tt = 16 if M <= 16 else (32 if M <= 32 else (64 if M <= 64 else 128))
    n_wt, n_tt = cdiv(N, 128), cdiv(M, tt)
    kb_total = cdiv(kpad(K, gk), 256)
    ks = 2 if tt <= 16 else 1
    upt = cdiv(kb_total, ks) if gk <= 256 else cdiv(K, gk)
    units = n_wt * n_tt * upt
    grid = max(1, min(sms, units))
    split = any((c * units // grid) % upt != 0 for c in range(1, grid))
    return dict(tt=tt, upt=upt, units=units, grid=grid, split=split)


def cta_range(c, units, C):
    return c * units // C, (c + 1) * units // C


def cta_of_unit(u, units, C):
    return ((u + 1) * C - 1) // units


def check_plan(units, upt, C):
    """All rules for one (units, units per tile, grid); returns split tiles seen."""
    starts = [cta_range(c, units, C)[0] for c in range(C)]
    for c in range(C):
        u0, u1 = cta_range(c, units, C)
        assert u1 > u0, "empty CTA range"
        for u in (u0, u1 - 1):
            assert cta_of_unit(u, units, C) == c
    n_split = 0
    for t in range(units // upt):
        tf, tl = t * upt, t * upt + upt - 1
        cf, cl = cta_of_unit(tf, units, C), cta_of_unit(tl, units, C)
        if cf == cl:
            continue
        n_split += 1
        side_f = 0 if starts[cf] == tf else 1
        for c in range(cf, cl + 1):
            written = 0 if t == starts[c] // upt else 1          # flush_tile
            read = side_f if c == cf else 0                       # splitk_reduce_kernel
            assert written == read, (units, upt, C, t, c)
    return n_split


@pytest.mark.parametrize("shape", sorted(QWQ))
@pytest.mark.parametrize("M", [1, 16, 32, 64, 2048, 4096])
def test_sweep_and_prefill_plans(shape, M):
    K, N = QWQ[shape]
    p = plan(M, N, K, 128)
    n_split = check_plan(p["units"], p["upt"], p["grid"])
    assert (n_split > 0) == p["split"]


def test_random_plans():
    rng = random.Random(7)
    for _ in range(3000):
        upt = rng.randint(1, 120)
        tiles = rng.randint(1, 600)
        units = upt * tiles
        C = min(rng.randint(1, 160), units)
        n_split = check_plan(units, upt, C)
        split = any((c * units // C) % upt != 0 for c in range(1, C))
        assert (n_split > 0) == split


def test_negative_control_naive_side_rule_is_caught():
    """Reading side 0 for the first CTA too (skipping its range check) must
    pick a slot flush_tile did not write for some split tile of the sweep."""
    mismatches = 0
    for shape, (K, N) in QWQ.items():
        for M in (1, 16, 32, 64):
            p = plan(M, N, K, 128)
            units, upt, C = p["units"], p["upt"], p["grid"]
            starts = [cta_range(c, units, C)[0] for c in range(C)]
            for t in range(units // upt):
                cf = cta_of_unit(t * upt, units, C)
                cl = cta_of_unit(t * upt + upt - 1, units, C)
                if cf != cl and (0 if t == starts[cf] // upt else 1) != 0:
                    mismatches += 1
    assert mismatches > 0
