"""The CPU oracle pinned against the reference's own outputs (golden.npz was
written by tests/golden/make_golden.py from fakequant_lab and the reference's
compiled C++), and against the reference C++ run live when it was built."""
import numpy as np
import pytest


QUANT_CASES = ["q0_", "q1_", "q2_", "q3_", "q4_", "qr_"]


@pytest.mark.parametrize("p", QUANT_CASES)
def test_quant_matches_fakequant(golden, orc, p):
    # quant.py:89-141: bf16 scale from amax/127, true division, half-even, clamp.
    q, s, ks = orc.quant_act(golden[p + "x"], int(golden[p + "gk"]))
    assert np.array_equal(q, golden[p + "q"])
    assert np.array_equal(s.T, golden[p + "scale"])
    # the negated row sum the kernel consumes (midgroup_quant_a.inc:11)
    gk = int(golden[p + "gk"])
    K = q.shape[1]
    for g in range(s.shape[0]):
        assert np.array_equal(ks[g], -q[:, g * gk:min(K, (g + 1) * gk)].astype(np.int32).sum(1))


def test_crafted_quant_edges(golden, orc):
    q, s, _ = orc.quant_act(golden["q0_x"], 128)
    assert np.all(q[1] == 0) and np.all(s[:, 1] == 0x0080)          # zero row -> bf16 tiny
    assert s[0, 2] == orc.f32_to_bf16(np.float32(0.125))             # exact 2^-3 scale
    # exact half quotients round to even
    xs = orc.bf16_to_f32(golden["q0_x"][2, 1:128]) / np.float32(0.125)
    assert np.array_equal(q[2, 1:128], np.rint(xs).astype(np.int8))
    assert np.any(np.abs(xs - np.trunc(xs)) == 0.5)


@pytest.mark.parametrize("i", range(5))
def test_gemm_matches_fakequant_kernel_mode(golden, orc, i):
    p = f"g{i}_"
    M, N, K, gk, asym, sbf = (int(v) for v in golden[p + "meta"])
    wz = golden[p + "wz"] if asym else None
    y, (q, s, ks) = orc.linear(golden[p + "x"], golden[p + "codes"], golden[p + "ws"], wz, gk)
    # int32 group partials: bit-exact (run_selftest.py T4 exact-integer reference)
    assert np.array_equal(orc.group_partials(q, golden[p + "codes"], wz, gk), golden[p + "P"])
    # fp32 rescale: T4's bound (rel < 1e-6) against FakeQuantLinear._kernel_gemm
    ref = golden[p + "y"]
    assert np.abs(y - ref).max() / np.abs(ref).max() < 1e-6
    y64, _ = orc.linear(golden[p + "x"], golden[p + "codes"], golden[p + "ws"], wz, gk, exact=True)
    assert np.abs(y64 - golden[p + "y64"]).max() <= 1e-12 * np.abs(golden[p + "y64"]).max()


@pytest.mark.parametrize("i", range(4))
def test_layouts_and_gemm_match_reference_cpp(golden, orc, i):
    p = f"r{i}_"
    if p + "meta" not in golden:
        pytest.skip("fixtures generated without the reference C++")
    M, N, K, gk, asym = (int(v) for v in golden[p + "meta"])
    qa, qw = golden[p + "qa"], golden[p + "qw"]
    # PackInt4Grouped / SplitInt8ToInt4PlanesGrouped byte layouts (ragged K)
    assert np.array_equal(orc.pack_int4_grouped(qw, gk), golden[p + "wpack"])
    assert np.array_equal(orc.unpack_int4_grouped(golden[p + "wpack"], K, gk), qw)
    assert np.array_equal(orc.msd_recombine(golden[p + "a_hi"], golden[p + "a_lo"], K, gk), qa)
    wz = orc.bf16_to_f32(golden[p + "wz"]) if asym else None
    y = orc.gemm_kernel_order(qa, orc.bf16_to_f32(golden[p + "as"]), qw,
                              orc.bf16_to_f32(golden[p + "ws"]), wz, gk)
    assert np.array_equal(orc.f32_to_bf16(y), golden[p + "y"])     # ReferenceMidGroupGemm, bf16


def test_msd_planes_match_reference_packer(golden, orc):
    """midgroup_quant_a planes of the oracle == the reference packer on the same codes."""
    x = golden["q4_x"][:5]
    hi, lo, s, ks = orc.midgroup_quant_a(x, 16, 128)
    q, s2, ks2 = orc.quant_act(x, 128)
    if orc.ref_available():
        rh, rl = orc.ref_split_planes_grouped(q, 128)
        assert np.array_equal(hi[:5], rh) and np.array_equal(lo[:5], rl)
    assert np.all(hi[5:] == 0) and np.all(lo[5:] == np.int8(-120))   # 0x88 pad rows
    assert np.all(s[:, 5:] == 0x0080) and np.all(ks[:, 5:] == 0)
    assert np.array_equal(s[:, :5], s2) and np.array_equal(ks[:, :5], ks2)
    assert np.array_equal(orc.msd_recombine(hi, lo, 5120, 128)[:5], q)


def test_reference_cpp_live(orc):
    """Run the reference's compiled ReferenceMidGroupGemm against the oracle on fresh data."""
    if not orc.ref_available():
        pytest.skip("oracle/_ref not built")
    rng = np.random.default_rng(7)
    for (M, N, K, gk, asym) in [(5, 128, 1025, 1024, True), (9, 256, 640, 64, False), (2, 128, 33, 128, True)]:
        G = -(-K // gk)
        qa = rng.integers(-128, 128, size=(M, K)).astype(np.int8)
        qw = rng.integers(-8, 8, size=(N, K)).astype(np.int8)
        asb = orc.f32_to_bf16(rng.uniform(1e-3, 2e-3, (G, M)).astype(np.float32))
        wsb = orc.f32_to_bf16(rng.uniform(1e-3, 2e-3, (G, N)).astype(np.float32))
        wzb = orc.f32_to_bf16(rng.integers(-8, 8, (G, N)).astype(np.float32)) if asym else None
        yref = orc.ref_midgroup_gemm(qa, asb, qw, wsb, wzb, gk)
        y = orc.gemm_kernel_order(qa, orc.bf16_to_f32(asb), qw, orc.bf16_to_f32(wsb),
                                  None if wzb is None else orc.bf16_to_f32(wzb), gk)
        assert np.array_equal(orc.f32_to_bf16(y), yref)


def test_ragged_layout_gate(orc):
    """The reference's own host-only ragged-K gate (ragged_layout_test.cpp), if built."""
    import os, subprocess
    exe = os.path.join(os.path.dirname(orc.__file__), "_ref", "ragged_layout_test")
    if not os.path.exists(exe):
        pytest.skip("oracle/_ref not built")
    out = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0 and "ALL PASS" in out.stdout


def test_negative_control_flipped_a_ksum_fails(golden, orc):
    """The quantiser's negated group sums a_ksum carry the zero-point term of the
    reference's kernel form, P = A_q.W_q + a_ksum * wz (fake_linear.py:170-178):
    with the quantiser's a_ksum the golden partials come out exactly, with its
    sign flipped they do not."""
    p = "g2_"
    M, N, K, gk, asym, _ = (int(v) for v in golden[p + "meta"])
    assert asym
    q, s, ks = orc.quant_act(golden[p + "x"], gk)               # ks: int32 [G, M]
    P_aw = orc.group_partials(q, golden[p + "codes"], None, gk).astype(np.int64)   # sum A_q * W_q
    wz = golden[p + "wz"].astype(np.int64)                        # [G, N], integers
    good = P_aw + ks.astype(np.int64)[:, :, None] * wz[:, None, :]
    bad = P_aw - ks.astype(np.int64)[:, :, None] * wz[:, None, :]
    assert np.array_equal(good, golden[p + "P"])
    assert not np.array_equal(bad, golden[p + "P"])


def test_negative_control_asym_data_on_sym_path_fails(golden, orc):
    """Asymmetric weights run as if symmetric (zero points dropped) must not
    reproduce the asymmetric reference: partials or y."""
    p = "g2_"
    M, N, K, gk, asym, _ = (int(v) for v in golden[p + "meta"])
    q, s, ks = orc.quant_act(golden[p + "x"], gk)
    P_sym = orc.group_partials(q, golden[p + "codes"], None, gk)
    assert not np.array_equal(P_sym, golden[p + "P"])
    y_sym, _ = orc.linear(golden[p + "x"], golden[p + "codes"], golden[p + "ws"], None, gk, exact=True)
    ref = golden[p + "y64"]
    assert np.abs(y_sym - ref).max() / np.abs(ref).max() > 1e-2


def test_negative_control_flipped_ksum_fails(golden, orc):
    """A planted mistake in the oracle (flipped zero-point sign) must break parity."""
    p = "g2_"
    M, N, K, gk, asym, _ = (int(v) for v in golden[p + "meta"])
    q, s, ks = orc.quant_act(golden[p + "x"], gk)
    bad = orc.group_partials(q, golden[p + "codes"], -golden[p + "wz"], gk)
    assert not np.array_equal(bad, golden[p + "P"])
