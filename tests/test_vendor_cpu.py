"""Vendor W4A8_DYNAMIC (group-wise int4) -> mid-group layout conversion, on CPU.

The vendor tensors are the ones the reference's structural builder writes
(scripts/build_random_w4a8.py:102-147); the conversion must reproduce the codes,
the combined per-group scale and the zero points exactly, and refuse what the
mid-group layout cannot hold.
"""
import pytest
import torch

from w4a8_b200 import ops
from w4a8_b200 import vendor as V


def vendor_projection(N, K, gs, seed, offsets=False, low_first=True):
    g = torch.Generator().manual_seed(seed)
    codes = torch.randint(-8, 8, (N, K), generator=g, dtype=torch.int16).to(torch.int8)
    s1 = torch.exp(torch.randn(N, 1, generator=g) * 0.2)
    s2 = (torch.exp(torch.randn(N, K // gs, generator=g) * 0.5 - 6.0)).to(torch.float16)
    o2 = (torch.randint(-2, 3, (N, K // gs), generator=g).float() if offsets
          else torch.zeros(N, K // gs)).to(torch.float16)
    t = {"weight": V.pack_output_axis(codes, low_first), "weight_scale": s1, "weight_offset": torch.zeros(N, 1),
         "weight_scale_second": s2, "weight_offset_second": o2, "scale_bias": torch.zeros(N, 1)}
    return t, codes


@pytest.mark.parametrize("low_first", [True, False])
def test_output_axis_pack_roundtrip(low_first):
    codes = torch.randint(-8, 8, (6, 10), dtype=torch.int16).to(torch.int8)
    p = V.pack_output_axis(codes, low_first)
    assert p.shape == (3, 10) and p.dtype == torch.int8
    assert torch.equal(V.unpack_output_axis(p, low_first), codes)
    # the byte holds rows 2i / 2i+1 in the low / high nibble
    b = int(p[1, 4]) & 0xFF
    lo, hi = b & 0xF, b >> 4
    sx = lambda v: v - 16 if v >= 8 else v
    assert (sx(lo), sx(hi)) == ((int(codes[2, 4]), int(codes[3, 4])) if low_first else
                                (int(codes[3, 4]), int(codes[2, 4])))
    with pytest.raises(ValueError):
        V.pack_output_axis(codes[:5])


@pytest.mark.parametrize("gs,offsets", [(128, False), (128, True), (64, True)])
def test_convert_exact(gs, offsets):
    N, K = 256, 640
    t, codes = vendor_projection(N, K, gs, 1, offsets)
    c = V.convert_projection(t, gs)
    assert c["w_packed"].shape == (N, K // 2) and c["N"] == N and c["K"] == K
    assert torch.equal(ops.unpack_int4_grouped(c["w_packed"], K, gs), codes)
    assert c["w_scale"].dtype == torch.float32
    assert torch.equal(c["w_scale"], (t["weight_scale"] * t["weight_scale_second"].float()).t())
    if offsets:
        assert torch.equal(c["w_zero"].float(), t["weight_offset_second"].float().t())
    else:
        assert c["w_zero"] is None
    ref = (t["weight_scale"] * t["weight_scale_second"].float().repeat_interleave(gs, 1)) * \
        (codes.float() - t["weight_offset_second"].float().repeat_interleave(gs, 1))
    torch.testing.assert_close(V.dequantize(c), ref, rtol=1e-6, atol=0)


def test_structural_builder_tensors_convert():
    """The exact tensors the reference's random builder writes (ones / zeros / 0.001)."""
    g = torch.Generator().manual_seed(5)
    N, K, gs = 128, 512, 128
    for width in (1, 16):                                     # column- / row-parallel scale_bias
        t = {"weight": torch.randint(-128, 128, (N // 2, K), dtype=torch.int8, generator=g),
             "weight_scale": torch.ones(N, 1), "weight_offset": torch.zeros(N, 1),
             "weight_scale_second": torch.full((N, K // gs), 0.001, dtype=torch.float16),
             "weight_offset_second": torch.zeros(N, K // gs, dtype=torch.float16),
             "scale_bias": torch.zeros(N, width)}
        c = V.convert_projection(t, gs)
        assert c["w_zero"] is None
        assert torch.all(c["w_scale"] == torch.tensor(0.001, dtype=torch.float16).float())
        assert torch.equal(ops.unpack_int4_grouped(c["w_packed"], K, gs), V.unpack_output_axis(t["weight"]))


def test_convert_refuses_what_the_layout_cannot_hold():
    t, _ = vendor_projection(128, 256, 128, 2)
    for key, val in (("weight_offset", torch.ones(128, 1)), ("scale_bias", torch.full((128, 1), 0.5)),
                     ("weight_offset_second", torch.full((128, 2), 0.5, dtype=torch.float16))):
        bad = dict(t)
        bad[key] = val
        with pytest.raises(ValueError):
            V.convert_projection(bad, 128)
    with pytest.raises(ValueError):
        V.convert_projection(t, 96)                            # K not a multiple of the group


def test_fused_members_concatenate_along_n():
    parts = {}
    codes = []
    for i, (name, n) in enumerate((("q", 256), ("k", 64), ("v", 64))):
        t, c = vendor_projection(n, 384, 128, 10 + i, offsets=(name == "k"))
        for suf, v in t.items():
            parts[f"l.{name}.{suf}"] = v
        codes.append(c)
    c = V.load_projection(parts.__getitem__, ["l.q", "l.k", "l.v"], 128)
    assert c["N"] == 384 and c["w_scale"].shape == (3, 384) and c["w_zero"].shape == (3, 384)
    assert torch.equal(ops.unpack_int4_grouped(c["w_packed"], 384, 128), torch.cat(codes, 0))
    assert torch.all(c["w_zero"][:, :256] == 0) and torch.all(c["w_zero"][:, 320:] == 0)
