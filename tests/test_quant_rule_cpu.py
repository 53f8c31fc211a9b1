"""The division-free activation quantisation rule, checked exhaustively in
IEEE fp32 arithmetic on the CPU (numpy float32 multiply, divide and rint
round to nearest even, as the GPU's __fmul_rn, __frcp_rn, __fdiv_rn and
rintf do).

The reference quantises q = clamp(rint(x / s), -128, 127) with a true
division (fakequant_lab/quant.py:89-141), x and s both bf16 values.  The
kernels compute y = x * (1/s) instead and fall back to the true division
only when y lies within 2^-11 of a half-integer.  Why that is exact: with
s normal, x / s is either a half-integer or at least 1/1020 away from every
half-integer (x = X 2^a, s = S 2^b with 8-bit integer significands), while
|y - x/s| <= 128 * 2^-23; so rint(y) = rint(x / s) away from ties, and every
tie lands in the fallback window.  A group whose scale is a bf16 subnormal
takes the division for every element.  The clamp never binds on the fast
path: |x| <= amax and s = bf16(amax / 127) >= amax / 127.4985."""
import numpy as np

THRESH = np.float32(0.49951171875)          # 0.5 - 2^-11


def _bf16_values():
    return (np.arange(0, 1 << 16, dtype=np.uint32) << 16).view(np.float32)


def _bf16_rne(v):
    u = np.ascontiguousarray(v, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint32)
    return (r << 16).view(np.float32)


def test_fast_path_equals_true_division():
    vals = _bf16_values()
    vals = vals[np.isfinite(vals)]
    mismatches = ties = slow = 0
    for se in (-126, -125, -60, -1, 0, 1, 7, 60, 100):
        for sm in range(128):
            s = np.float32(np.ldexp(1 + sm / 128.0, se))
            x = vals[np.abs(vals) <= np.float32(127.4985) * s]
            exact = np.rint(x / s)
            y = x * (np.float32(1) / s)
            n = np.rint(y)
            near = np.abs(y - n) > THRESH
            q = np.where(near, exact, n)
            mismatches += int(np.sum(q != exact))
            ties += int(np.sum(np.abs((x / s) - np.floor(x / s) - np.float32(0.5)) == 0))
            slow += int(near.sum())
    assert mismatches == 0
    assert ties > 0 and slow == ties      # the window catches the exact ties and nothing else


def test_scale_bounds_the_quotient():
    """For every positive normal bf16 amax: amax / s < 127.5, so no element of
    the group rounds beyond +-127 and the fast path needs no clamp."""
    a = _bf16_values()[1:0x7F80]          # positive finite bf16
    a = a[a >= np.float32(2.0 ** -126) * 127]
    s = _bf16_rne(a / np.float32(127))
    assert np.all(a / s < np.float32(127.5))
