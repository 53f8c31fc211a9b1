"""Parity at the benchmark configurations' full sizes.

Config 1 (decode): the four QwQ-32B projections at M in {1, 4, 8, 16, 32, 64};
config 3: gate_up and down at M in {16, 4096} x group size {64, 128, 256} x
{symmetric int4, asymmetric uint4 with an integer zero point in [6, 9]}.

The CUDA path runs at full size (prepared weights, the benchmark's product
path).  The oracle is evaluated on a sample of output columns that touches
every 128-row weight tile (first row, last row, one row in between, plus
random ones), on every row for decode sizes and on rows from every token-tile
region at M = 4096 (activation quantisation is per row, so a row subset is
exact).  Bars, as everywhere:
  * int32 group partials bit-exact (sampled columns, all rows, M <= 64);
  * y: max|y - ref| / max|ref| <= 1e-2 and cosine >= 0.9999 against the
    float64 exact-integer reference, and within 2 bf16 ulps of the oracle's
    fp32 kernel-order result."""
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


def _bits(t) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def _cols(N: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    n_wt = -(-N // 128)
    base = np.arange(n_wt) * 128
    cols = np.concatenate([base, base + 127, base + 1 + rng.integers(0, 126, n_wt), rng.integers(0, N, 128)])
    cols = np.unique(cols)
    return cols[cols < N]


def _close(y_bits, ref64, yk, orc, what):
    y = orc.bf16_to_f32(y_bits).astype(np.float64)
    err = np.abs(y - ref64).max() / max(np.abs(ref64).max(), 1e-30)
    cos = float((y * ref64).sum() / (np.linalg.norm(y) * np.linalg.norm(ref64) + 1e-300))
    assert err <= MAX_REL, f"{what}: max rel {err}"
    assert cos >= MIN_COS, f"{what}: cosine {cos}"
    yk = yk.astype(np.float64)
    tol = 2 * 2.0 ** -7 * np.abs(yk) + 1e-6 * np.abs(yk).max()
    d = np.abs(y - yk)
    assert np.all(d <= tol), f"{what}: worst {np.max(d / tol)} of the 2-ulp bound"


class _Weights:
    """One projection's weights at full size on the device, plus the sampled
    columns on the host for the oracle."""

    def __init__(self, N, K, gk, seed, dev, asym):
        from w4a8_b200 import ops
        from w4a8_b200 import synthetic as syn
        codes, scale, zero = syn.weight_torch(N, K, gk, seed, dev, asym=asym)
        self.N, self.K, self.gk = N, K, gk
        self.packed = ops.pack_int4_grouped(codes, gk)
        self.scale = scale.contiguous()
        self.zero = None if zero is None else zero.contiguous()
        self.pw = ops.prepare_weights(self.packed, self.scale, self.zero, K, gk)
        self.cols = _cols(N, seed)
        ct = torch.from_numpy(self.cols).to(dev)
        self.codes_s = codes[ct].cpu().numpy()
        self.scale_s = np.ascontiguousarray(self.scale[:, ct].cpu().numpy())
        self.zero_s = None if zero is None else np.ascontiguousarray(zero[:, ct].float().cpu().numpy())
        del codes


def _check_rows(orc, W, x, y, rows, what):
    xb = _bits(x[rows])
    y64, _ = orc.linear(xb, W.codes_s, W.scale_s, W.zero_s, W.gk, exact=True)
    yk, _ = orc.linear(xb, W.codes_s, W.scale_s, W.zero_s, W.gk)
    _close(_bits(y[rows][:, torch.from_numpy(W.cols).to(y.device)]), y64, yk, orc, what)


def _check_decode(orc, W, M, seed, dev, what, raw_too=False):
    from w4a8_b200 import ops
    from w4a8_b200 import synthetic as syn
    x = syn.activation_torch(M, W.K, seed, dev)
    y = ops.linear_prepared(x, W.pw)
    if raw_too:
        assert torch.equal(y, ops.linear(x, W.packed, W.scale, W.zero, W.gk)), f"{what}: raw != prepared"
    P = ops.group_partials(x, W.packed, W.zero, W.gk)
    P = P[:, :, torch.from_numpy(W.cols).to(dev)].cpu().numpy()
    q, _, _ = orc.quant_act(_bits(x), W.gk)
    assert np.array_equal(P, orc.group_partials(q, W.codes_s, W.zero_s, W.gk)), f"{what}: partials"
    _check_rows(orc, W, x, y, list(range(M)), what)
    assert ops.workspace_status() == 0


@pytest.mark.parametrize("shape", ["qkv", "o", "gate_up", "down"])
def test_config1_full_size(orc, shape):
    from w4a8_b200.synthetic import QWQ_SHAPES
    dev = _dev()
    K, N = QWQ_SHAPES[shape]
    W = _Weights(N, K, 128, 40 + len(shape), dev, asym=False)
    for M in (1, 4, 8, 16, 32, 64):
        _check_decode(orc, W, M, 500 + M, dev, f"{shape} M={M}", raw_too=(M == 16))


@pytest.mark.parametrize("gk", [64, 128, 256])
@pytest.mark.parametrize("asym", [False, True])
@pytest.mark.parametrize("shape", ["gate_up", "down"])
def test_config3_full_size(orc, shape, gk, asym):
    from w4a8_b200 import ops
    from w4a8_b200 import synthetic as syn
    from w4a8_b200.synthetic import QWQ_SHAPES
    dev = _dev()
    K, N = QWQ_SHAPES[shape]
    W = _Weights(N, K, gk, 60 + gk + int(asym), dev, asym=asym)
    what = f"{shape} gk={gk} {'asym' if asym else 'sym'}"
    _check_decode(orc, W, 16, 700 + gk, dev, what + " M=16", raw_too=True)
    M = 4096
    x = syn.activation_torch(M, K, 800 + gk, dev)
    y = ops.linear_prepared(x, W.pw)
    rows = sorted({0, 1, 127, 128, 1000, M // 2 - 1, M // 2, M - 129, M - 2, M - 1})
    _check_rows(orc, W, x, y, rows, what + " M=4096")
    assert torch.equal(y, ops.linear_prepared(x, W.pw)), what + ": repeat differs"
    assert ops.workspace_status() == 0
