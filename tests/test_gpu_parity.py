"""GPU parity: the sm_100a kernels against the CPU oracle on the same seeded
inputs.  Integer work (codes, MSD planes, int32 group partials) must be
bit-exact; bf16 outputs must satisfy the stated tolerance:

    max|y - ref| / max|ref| <= 1e-2   and   cosine(y, ref) >= 0.9999

against the float64 exact-integer reference (``oracle.gemm_f64``), and be
within a few bf16 ulps of the oracle's fp32 kernel-order result."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

MAX_REL = 1e-2
MIN_COS = 0.9999


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _bf16_cuda(bits: np.ndarray):
    return torch.from_numpy(np.ascontiguousarray(bits, np.uint16).view(np.int16)).view(torch.bfloat16).cuda()


def _bits(t) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def _weights(w, gk, dev, scale_dtype=torch.float32):
    from w4a8_b200 import ops
    codes = torch.from_numpy(w.codes)
    packed = ops.pack_int4_grouped(codes, gk).to(dev)
    ws = torch.from_numpy(w.scale).to(dev, scale_dtype)
    wz = None if w.zero is None else torch.from_numpy(w.zero).to(torch.bfloat16).to(dev)
    return packed, ws, wz


def _close(y, ref64, yk=None):
    y = np.asarray(y, np.float64)
    err = np.abs(y - ref64).max() / max(np.abs(ref64).max(), 1e-30)
    cos = float((y * ref64).sum() / (np.linalg.norm(y) * np.linalg.norm(ref64) + 1e-300))
    assert err <= MAX_REL, f"max rel {err}"
    assert cos >= MIN_COS, f"cosine {cos}"
    if yk is not None:
        # y differs from the oracle's fp32 kernel-order result only in fp32
        # accumulation order before the bf16 rounding: at most 2 bf16 ulps.
        yk = yk.astype(np.float64)
        d = np.abs(y - yk)
        tol = 2 * 2.0 ** -7 * np.abs(yk) + 1e-6 * np.abs(yk).max()
        assert np.all(d <= tol), f"worst {np.max(d / tol)} of the 2-ulp bound"


# ------------------------------------------------------------------ quantiser

QUANT_SHAPES = [(1, 128, 128), (4, 1024, 128), (3, 512, 64), (2, 2048, 1024), (5, 768, 256),
                (7, 1057, 1024), (3, 777, 128), (2, 33, 64), (16, 5120, 128), (1, 27648, 128),
                (130, 640, 64)]


@pytest.mark.parametrize("M,K,gk", QUANT_SHAPES)
def test_quant_act_bitexact(orc, M, K, gk):
    from w4a8_b200 import ops
    from w4a8_b200 import synthetic as syn
    _dev()
    xb = syn.activation_np(M, K, 1000 + M + K)
    q, s, ks = ops.quant_act(_bf16_cuda(xb), gk)
    oq, os_, oks = orc.quant_act(xb, gk)
    assert np.array_equal(q.cpu().numpy(), oq)
    assert np.array_equal(_bits(s), os_)
    assert np.array_equal(ks.cpu().numpy(), oks)


def test_quant_act_golden(golden):
    from w4a8_b200 import ops
    _dev()
    for p in ["q0_", "q1_", "q2_", "q3_", "q4_", "qr_"]:
        q, s, _ = ops.quant_act(_bf16_cuda(golden[p + "x"]), int(golden[p + "gk"]))
        assert np.array_equal(q.cpu().numpy(), golden[p + "q"]), p
        assert np.array_equal(_bits(s).T, golden[p + "scale"]), p


def test_quant_act_f32_scale(orc):
    from w4a8_b200 import ops
    from w4a8_b200 import synthetic as syn
    _dev()
    xb = syn.activation_np(9, 1280, 77)
    q, s, _ = ops.quant_act(_bf16_cuda(xb), 128, scale_dtype=torch.float32, with_ksum=False)
    oq, os_, _ = orc.quant_act(xb, 128)
    assert np.array_equal(q.cpu().numpy(), oq)
    assert np.array_equal(s.cpu().numpy(), orc.bf16_to_f32(os_))


@pytest.mark.parametrize("M,K,gk", [(1, 5120, 1024), (16, 5120, 128), (17, 1057, 1024), (64, 640, 64),
                                    (65, 777, 256), (130, 2048, 128)])
def test_midgroup_quant_a_bitexact(orc, M, K, gk):
    from w4a8_b200 import ops
    from w4a8_b200 import synthetic as syn
    _dev()
    xb = syn.activation_np(M, K, 2000 + M)
    hi, lo, s, ks = ops.midgroup_quant_a(_bf16_cuda(xb), gk)
    Mp = ops.pad_rows(M)
    ohi, olo, os_, oks = orc.midgroup_quant_a(xb, Mp, gk)
    assert hi.shape == (Mp, ohi.shape[1])
    assert np.array_equal(hi.cpu().numpy(), ohi)
    assert np.array_equal(lo.cpu().numpy(), olo)
    assert np.array_equal(_bits(s), os_)
    assert np.array_equal(ks.cpu().numpy(), oks)


# ------------------------------------------------------------------ group partials (bit-exact)

PARTIAL_CASES = [  # M, N, K, gk, asym
    (1, 128, 256, 128, False), (16, 256, 1024, 128, False), (16, 256, 1024, 128, True),
    (5, 128, 640, 64, False), (7, 256, 1280, 256, True), (3, 128, 2048, 1024, True),
    (3, 128, 2048, 1024, False), (33, 384, 768, 128, False), (64, 128, 512, 64, True),
    (100, 256, 1024, 256, False), (200, 256, 640, 128, True), (3, 128, 1057, 1024, True),
    (2, 128, 777, 128, False), (4, 128, 3456, 128, True), (1, 1024, 5120, 128, False),
]


@pytest.mark.parametrize("M,N,K,gk,asym", PARTIAL_CASES)
def test_group_partials_bitexact(orc, M, N, K, gk, asym):
    from w4a8_b200 import ops
    from w4a8_b200 import synthetic as syn
    dev = _dev()
    xb = syn.activation_np(M, K, 3000 + M + K)
    w = syn.weight_np(N, K, gk, 4000 + N + K, asym=asym)
    packed, _, wz = _weights(w, gk, dev)
    P = ops.group_partials(_bf16_cuda(xb), packed, wz, gk).cpu().numpy()
    q, _, _ = orc.quant_act(xb, gk)
    ref = orc.group_partials(q, w.codes, w.zero, gk)
    assert np.array_equal(P, ref), f"{np.sum(P != ref)} of {P.size} partials differ"
    assert ops.workspace_status() == 0


def test_group_partials_golden(golden):
    """Against the int64 partials of the reference's own T4 reference."""
    from w4a8_b200 import ops
    dev = _dev()
    for i in range(5):
        p = f"g{i}_"
        M, N, K, gk, asym, sbf = (int(v) for v in golden[p + "meta"])
        packed = ops.pack_int4_grouped(torch.from_numpy(golden[p + "codes"]), gk).to(dev)
        wz = torch.from_numpy(golden[p + "wz"]).to(torch.bfloat16).to(dev) if asym else None
        P = ops.group_partials(_bf16_cuda(golden[p + "x"]), packed, wz, gk).cpu().numpy()
        assert np.array_equal(P, golden[p + "P"]), p


# ------------------------------------------------------------------ fused linear (tolerance)

LINEAR_CASES = [  # M, N, K, gk, asym, scale_dtype
    (1, 128, 256, 128, False, "f32"), (16, 512, 1024, 128, False, "f32"), (16, 512, 1024, 128, True, "bf16"),
    (9, 256, 640, 64, False, "bf16"), (31, 256, 1280, 256, True, "f32"), (48, 128, 2048, 1024, True, "bf16"),
    (64, 384, 1024, 128, False, "f32"), (65, 256, 1024, 128, True, "f32"), (256, 512, 1024, 128, False, "bf16"),
    (300, 256, 1057, 1024, False, "f32"), (4, 128, 3456, 128, True, "bf16"), (128, 896, 640, 128, False, "f32"),
]


@pytest.mark.parametrize("M,N,K,gk,asym,sd", LINEAR_CASES)
def test_linear_tolerance(orc, M, N, K, gk, asym, sd):
    from w4a8_b200 import ops
    from w4a8_b200 import synthetic as syn
    dev = _dev()
    xb = syn.activation_np(M, K, 5000 + M + K)
    w = syn.weight_np(N, K, gk, 6000 + N + K, asym=asym, scale_bf16=(sd == "bf16"))
    packed, ws, wz = _weights(w, gk, dev, torch.bfloat16 if sd == "bf16" else torch.float32)
    y = ops.linear(_bf16_cuda(xb), packed, ws, wz, gk)
    yf = orc.bf16_to_f32(_bits(y))
    y64, _ = orc.linear(xb, w.codes, w.scale, w.zero, gk, exact=True)
    yk, _ = orc.linear(xb, w.codes, w.scale, w.zero, gk)
    _close(yf, y64, orc.bf16_to_f32(orc.f32_to_bf16(yk)))
    assert ops.workspace_status() == 0


def test_negative_controls_cuda(orc):
    """Negative controls on the CUDA path, each of which must fail parity.

    (a) a_ksum: the quantiser's negated group sums carry the zero-point term of
    the reference's kernel form, P = A_q.W_q + a_ksum * wz (fake_linear.py:170-178).
    With the GPU quantiser's a_ksum the tensor-core partials of asymmetric weights
    come out exactly; with its sign flipped they do not.
    (b) asymmetric weights run on the symmetric path (zero points dropped) must
    not meet the tolerance against the asymmetric reference, while matching the
    reference evaluated the same way (the kernel computed what it was given)."""
    from w4a8_b200 import ops
    from w4a8_b200 import synthetic as syn
    dev = _dev()
    M, N, K, gk = 16, 256, 1280, 128
    xb = syn.activation_np(M, K, 9100)
    w = syn.weight_np(N, K, gk, 9200, asym=True)
    packed, ws, wz = _weights(w, gk, dev)
    x = _bf16_cuda(xb)
    _, _, ks = ops.quant_act(x, gk)
    P_aw = ops.group_partials(x, packed, None, gk).cpu().numpy().astype(np.int64)
    P = ops.group_partials(x, packed, wz, gk).cpu().numpy().astype(np.int64)
    term = ks.cpu().numpy().astype(np.int64)[:, :, None] * w.zero.astype(np.int64)[:, None, :]
    assert np.array_equal(P_aw + term, P)
    assert not np.array_equal(P_aw - term, P)
    y_sym = orc.bf16_to_f32(_bits(ops.linear(x, packed, ws, None, gk))).astype(np.float64)
    y_asym64, _ = orc.linear(xb, w.codes, w.scale, w.zero, gk, exact=True)
    assert np.abs(y_sym - y_asym64).max() / np.abs(y_asym64).max() > 1e-2
    y_sym64, _ = orc.linear(xb, w.codes, w.scale, None, gk, exact=True)
    _close(y_sym, y_sym64)
    assert ops.workspace_status() == 0


# Shapes where every CTA runs four or more K-units, so the accumulator-slot
# ring wraps many times and both MMA issuers run ahead of the epilogue (with
# GK = 64 a unit fills 4 slots, as many as or more than the ring holds).
MANY_UNIT_CASES = [  # M, N, K, gk, asym, scale_dtype
    (130, 2048, 5120, 64, False, "f32"), (64, 4096, 5120, 64, True, "bf16"), (32, 8192, 5120, 64, False, "f32"),
    (16, 8192, 5120, 64, False, "bf16"), (256, 2048, 5120, 128, False, "f32"), (100, 2048, 5120, 256, True, "f32"),
]


@pytest.mark.parametrize("M,N,K,gk,asym,sd", MANY_UNIT_CASES)
def test_linear_many_units_per_cta(orc, M, N, K, gk, asym, sd):
    from w4a8_b200 import ops
    from w4a8_b200 import synthetic as syn
    dev = _dev()
    xb = syn.activation_np(M, K, 7000 + M + gk)
    w = syn.weight_np(N, K, gk, 8000 + N + gk, asym=asym, scale_bf16=(sd == "bf16"))
    packed, ws, wz = _weights(w, gk, dev, torch.bfloat16 if sd == "bf16" else torch.float32)
    x = _bf16_cuda(xb)
    y = ops.linear(x, packed, ws, wz, gk)
    assert ops.workspace_status() == 0
    y64, _ = orc.linear(xb, w.codes, w.scale, w.zero, gk, exact=True)
    _close(orc.bf16_to_f32(_bits(y)), y64)
    # repeated calls give the same bits (no dependence on timing)
    for _ in range(3):
        assert np.array_equal(_bits(ops.linear(x, packed, ws, wz, gk)), _bits(y))
    assert ops.workspace_status() == 0


@pytest.mark.parametrize("M,N,K,gk,asym,sd", LINEAR_CASES)
def test_linear_prepared_matches_raw(orc, M, N, K, gk, asym, sd):
    """Prepared (tile-order) weights give the same bits as the reference layout."""
    from w4a8_b200 import ops
    from w4a8_b200 import synthetic as syn
    dev = _dev()
    xb = syn.activation_np(M, K, 5000 + M + K)
    w = syn.weight_np(N, K, gk, 6000 + N + K, asym=asym, scale_bf16=(sd == "bf16"))
    packed, ws, wz = _weights(w, gk, dev, torch.bfloat16 if sd == "bf16" else torch.float32)
    x = _bf16_cuda(xb)
    pw = ops.prepare_weights(packed, ws, wz, K, gk)
    y_raw = _bits(ops.linear(x, packed, ws, wz, gk))
    y_pre = _bits(ops.linear_prepared(x, pw))
    assert np.array_equal(y_raw, y_pre)
    y64, _ = orc.linear(xb, w.codes, w.scale, w.zero, gk, exact=True)
    _close(orc.bf16_to_f32(y_pre), y64)
    assert ops.workspace_status() == 0


def test_linear_prepared_split_and_leading_dims(orc):
    """linear_quant + linear_gemm_prepared equals linear_prepared; 3-D input."""
    from w4a8_b200 import ops
    from w4a8_b200 import synthetic as syn
    dev = _dev()
    M, N, K, gk = 12, 640, 5120, 128
    xb = syn.activation_np(M, K, 41)
    w = syn.weight_np(N, K, gk, 42)
    packed, ws, _ = _weights(w, gk, dev)
    pw = ops.prepare_weights(packed, ws, None, K, gk)
    x = _bf16_cuda(xb)
    y1 = ops.linear_prepared(x.view(3, 4, K), pw)
    assert y1.shape == (3, 4, N)
    y2 = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    ops.linear_quant(x, N, gk)
    ops.linear_gemm_prepared(M, pw, y2)
    assert np.array_equal(_bits(y1.view(M, N)), _bits(y2))
    with pytest.raises(RuntimeError):
        ops.linear_prepared(x[:, :1024].contiguous(), pw)          # K mismatch


def test_linear_golden(golden, orc):
    """Against FakeQuantLinear._kernel_gemm output stored by make_golden.py."""
    from w4a8_b200 import ops
    dev = _dev()
    for i in range(5):
        p = f"g{i}_"
        M, N, K, gk, asym, sbf = (int(v) for v in golden[p + "meta"])
        packed = ops.pack_int4_grouped(torch.from_numpy(golden[p + "codes"]), gk).to(dev)
        ws = torch.from_numpy(golden[p + "ws"]).to(dev)
        wz = torch.from_numpy(golden[p + "wz"]).to(torch.bfloat16).to(dev) if asym else None
        y = ops.linear(_bf16_cuda(golden[p + "x"]), packed, ws, wz, gk)
        _close(orc.bf16_to_f32(_bits(y)), golden[p + "y64"])


def test_linear_deterministic_and_repeatable(orc):
    """Stream-K reduction order is fixed: repeated calls give identical bits."""
    from w4a8_b200 import ops
    from w4a8_b200 import synthetic as syn
    dev = _dev()
    M, N, K, gk = 16, 1024, 5120, 128
    xb = syn.activation_np(M, K, 7)
    w = syn.weight_np(N, K, gk, 8)
    packed, ws, _ = _weights(w, gk, dev)
    x = _bf16_cuda(xb)
    ys = [_bits(ops.linear(x, packed, ws, None, gk)) for _ in range(3)]
    assert all(np.array_equal(ys[0], y) for y in ys[1:])


def test_config0_full_size(orc):
    """The reference's CPU-runnable case: M=16 K=5120 N=7168 GK=128, fp32 lognormal scales."""
    from w4a8_b200 import ops
    from w4a8_b200 import synthetic as syn
    dev = _dev()
    M, K, N, gk = 16, 5120, 7168, 128
    xb = syn.activation_np(M, K, 0)
    w = syn.weight_np(N, K, gk, 1)
    packed, ws, _ = _weights(w, gk, dev)
    x = _bf16_cuda(xb)
    P = ops.group_partials(x, packed, None, gk).cpu().numpy()
    q, _, _ = orc.quant_act(xb, gk)
    assert np.array_equal(P, orc.group_partials(q, w.codes, None, gk))
    y = ops.linear(x, packed, ws, None, gk)
    y64, _ = orc.linear(xb, w.codes, w.scale, None, gk, exact=True)
    _close(orc.bf16_to_f32(_bits(y)), y64)


@pytest.mark.parametrize("shape,M", [("gate_up", 8192), ("down", 4096), ("qkv", 8192), ("o", 2048)])
def test_config2_full_size_sampled_rows(orc, shape, M):
    """The prefill configuration at its largest sizes.  Activation quantisation is per
    row, so the oracle evaluated on a subset of rows is exact for those rows:
    sampled rows from every token tile region (first, middle, last) are checked
    against the float64 reference, and repeated calls must be bit-identical."""
    from w4a8_b200 import ops
    from w4a8_b200 import synthetic as syn
    from w4a8_b200.synthetic import QWQ_SHAPES
    dev = _dev()
    K, N = QWQ_SHAPES[shape]
    gk = 128
    codes, scale, _ = syn.weight_torch(N, K, gk, 21, dev)
    pw = ops.prepare_weights(ops.pack_int4_grouped(codes, gk), scale, None, K, gk)
    x = syn.activation_torch(M, K, 22, dev)
    y = ops.linear_prepared(x, pw)
    y2 = ops.linear_prepared(x, pw)
    assert torch.equal(y, y2)
    assert ops.workspace_status() == 0
    rows = sorted({0, 1, 127, 128, M // 2 - 1, M // 2, M // 2 + 77, M - 129, M - 2, M - 1})
    xb = _bits(x[rows])
    y64, _ = orc.linear(xb, codes.cpu().numpy(), scale.cpu().numpy(), None, gk, exact=True)
    _close(orc.bf16_to_f32(_bits(y[rows])), y64)


# ------------------------------------------------------------------ reference-compatible GEMM

@pytest.mark.parametrize("M,N,K,gk", [(1, 128, 1024, 1024), (16, 256, 5120, 1024), (20, 128, 1057, 1024),
                                      (64, 256, 1280, 128), (130, 128, 2048, 256)])
def test_midgroup_gemm_compat(orc, M, N, K, gk):
    """quant_a -> gemm, the reference op pair, against ReferenceMidGroupGemm semantics."""
    from w4a8_b200 import ops
    from w4a8_b200 import synthetic as syn
    dev = _dev()
    xb = syn.activation_np(M, K, 9000 + M)
    w = syn.weight_np(N, K, gk, 9100 + N, asym=True, scale_bf16=True)
    packed, ws, wz = _weights(w, gk, dev, torch.bfloat16)
    a_hi, a_lo, a_s, a_k = ops.midgroup_quant_a(_bf16_cuda(xb), gk)
    y = ops.midgroup_w4a8_gemm(a_hi, a_lo, a_s, a_k, packed, ws, None, wz, K, gk)
    assert y.shape == (ops.pad_rows(M), N)
    y = y[:M]
    y64, _ = orc.linear(xb, w.codes, w.scale, w.zero, gk, exact=True)
    _close(orc.bf16_to_f32(_bits(y)), y64)
    if orc.ref_available():
        q, s, _ = orc.quant_act(xb, gk)
        yref = orc.ref_midgroup_gemm(q, s, w.codes, orc.f32_to_bf16(w.scale), orc.f32_to_bf16(w.zero), gk)
        d = np.abs(orc.bf16_to_f32(_bits(y)).astype(np.float64) - orc.bf16_to_f32(yref))
        assert d.max() <= 2 * 2.0 ** -7 * np.abs(orc.bf16_to_f32(yref)).max()


def test_errors_raise():
    from w4a8_b200 import ops
    dev = _dev()
    x = torch.zeros(4, 256, dtype=torch.bfloat16, device=dev)
    w = torch.zeros(128, 128, dtype=torch.int8, device=dev)
    s = torch.zeros(2, 128, dtype=torch.float32, device=dev)
    with pytest.raises(RuntimeError):
        ops.linear(x.float(), w, s, None, 128)                      # dtype
    with pytest.raises(RuntimeError):
        ops.linear(x, w[:, :64], s, None, 128)                      # packed row length
    with pytest.raises(RuntimeError):
        ops.linear(x, w, s, None, 96)                               # unsupported group size
    y = ops.linear(x, w, s, None, 128)
    assert torch.count_nonzero(y) == 0
