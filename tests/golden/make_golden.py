"""Generate the golden fixtures from the reference's OWN code.

Run in a checkout where the reference project is available (it is imported,
never copied):

    python tests/golden/make_golden.py [--reference /path/to/reference]

Writes ``tests/golden/golden.npz``.  Sources of truth:

* ``fakequant_lab.quant.quantize`` (activation quantiser, quant.py:153-173)
  for the (row, group) int8 codes and bf16 scales, including crafted groups
  that hit exact half-integer quotients, clamping and all-zero groups;
* ``fakequant_lab.fake_linear.FakeQuantLinear(mode="kernel", w_qt=...)``
  (fake_linear.py:103-179) for the GEMM output, with synthetic integer weights
  injected through ``QTensor`` exactly as the survey's config 0 describes;
* an int64/float64 restatement of ``run_selftest._exact_reference``
  (run_selftest.py:104-121) for the int32 group partials;
* ``npu_ops/python/w4a8_ops.quantize_weight`` (w4a8_ops.py:181-240) for the
  asymmetric int4 weight layout (codes, bf16 scales and zero points, raw-code sums);
* when ``oracle/_ref`` was built (``make -C oracle ref``), the reference's C++
  ``PackInt4Grouped`` / ``SplitInt8ToInt4PlanesGrouped`` /
  ``ReferenceMidGroupGemm`` for ragged-K byte layouts and bf16 outputs.

The fixture stores inputs and outputs, so the tests never need the reference
checkout at run time.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "vllm-ascend910_b200"))


def _bits(t):
    import torch
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _bf16(bits):
    import torch
    return torch.from_numpy(np.ascontiguousarray(bits, np.uint16).view(np.int16)).view(torch.bfloat16)


def quant_cases(quant, out):
    """Activation quantiser golden: q codes and bf16 scale bits per (row, group)."""
    import torch
    from w4a8_b200 import synthetic as syn
    cases = [(4, 1024, 128, 11), (3, 512, 64, 12), (2, 2048, 1024, 13), (5, 768, 256, 14),
             (16, 5120, 128, 15)]
    for i, (M, K, gk, seed) in enumerate(cases):
        xb = syn.activation_np(M, K, seed)
        if i == 0:
            # Crafted rows: row 1 is all zero; row 2 group 0 has amax = 127*2^-3 so
            # the bf16 scale is exactly 2^-3 and every other element sits on an
            # exact half quotient (round-half-to-even); row 3 group 1 is constant.
            xf = syn.bf16_bits_to_f32(xb).copy()
            xf[1, :] = 0.0
            s = 0.125
            halves = (np.arange(-60, 60, dtype=np.float32) + 0.5) * s
            xf[2, :gk] = np.resize(halves, gk)
            xf[2, 0] = 127 * s
            xf[3, gk:2 * gk] = -1.5
            xb = syn._f32_to_bf16_bits(xf)
        x = _bf16(xb)
        qt = quant.quantize(x.float(), quant.QuantSpec(8, gk, "A"))
        out[f"q{i}_x"] = xb
        out[f"q{i}_gk"] = np.int32(gk)
        out[f"q{i}_q"] = qt.q.numpy().astype(np.int8)
        out[f"q{i}_scale"] = _bits(qt.scale.to(torch.bfloat16))        # [M, G]
    # Ragged K: the final group is quantised on its real members only, as its
    # own group (the kernel contract of mg_kgeom.h and midgroup_quant_a.inc).
    M, K, gk = 3, 1057, 1024
    xb = syn.activation_np(M, K, 21)
    x = _bf16(xb).float()
    full = quant.quantize(x[:, :1024], quant.QuantSpec(8, 1024, "A"))
    tail = quant.quantize(x[:, 1024:], quant.QuantSpec(8, K - 1024, "A"))
    out["qr_x"] = xb
    out["qr_gk"] = np.int32(gk)
    out["qr_q"] = np.concatenate([full.q.numpy(), tail.q.numpy()], axis=1).astype(np.int8)
    out["qr_scale"] = np.concatenate([_bits(full.scale.to(torch.bfloat16)),
                                      _bits(tail.scale.to(torch.bfloat16))], axis=1)


def exact_partials(qa, qw, wz, gk):
    """int64 per-group partials, the T4 exact-integer reference (run_selftest.py:104-121)."""
    M, K = qa.shape
    N = qw.shape[0]
    G = -(-K // gk)
    P = np.zeros((G, M, N), np.int64)
    for g in range(G):
        a = qa[:, g * gk:(g + 1) * gk].astype(np.int64)
        w = qw[:, g * gk:(g + 1) * gk].astype(np.int64)
        p = a @ w.T
        if wz is not None:
            p -= a.sum(1, keepdims=True) * wz[g].astype(np.int64)[None, :]
        P[g] = p
    assert np.abs(P).max() < 2 ** 31
    return P.astype(np.int32)


def gemm_cases(quant, fl, out):
    import torch
    import torch.nn as nn
    from w4a8_b200 import synthetic as syn
    cases = [  # (M, N, K, gk, asym, scale_bf16, seed)
        (16, 256, 1024, 128, False, False, 31),   # config-0 distribution, fp32 scales
        (5, 128, 640, 64, False, True, 32),
        (7, 256, 1280, 256, True, False, 33),     # uint4 + zp [6,9]
        (3, 128, 2048, 1024, True, True, 34),
        (1, 128, 512, 128, True, False, 35),
    ]
    for i, (M, N, K, gk, asym, sbf, seed) in enumerate(cases):
        xb = syn.activation_np(M, K, seed)
        w = syn.weight_np(N, K, gk, seed + 100, asym=asym, scale_bf16=sbf)
        spec_w = quant.QuantSpec(4, gk, "W", sym=not asym)
        spec_a = quant.QuantSpec(8, gk, "A")
        qt = quant.QTensor(
            torch.from_numpy(w.codes.copy()),
            torch.from_numpy(w.scale.T.copy()),                          # [N, G]
            None if w.zero is None else torch.from_numpy(w.zero.T.copy()).to(torch.bfloat16),
            spec_w)
        base = nn.Linear(K, N, bias=False)
        fq = fl.FakeQuantLinear(base, fl.Config("golden", spec_w, spec_a), mode="kernel", w_qt=qt)
        x = _bf16(xb)
        with torch.no_grad():
            y = fq._kernel_gemm(x).numpy().astype(np.float32)             # fp32 acc
            qa = quant.quantize(x, spec_a)
        qa_q = qa.q.numpy().astype(np.int8)
        P = exact_partials(qa_q, w.codes, w.zero, gk)
        as64 = qa.scale.float().numpy().astype(np.float64).T               # [G, M]
        y64 = np.zeros((M, N), np.float64)
        for g in range(P.shape[0]):
            y64 += P[g].astype(np.float64) * (as64[g][:, None] * w.scale[g].astype(np.float64)[None, :])
        pfx = f"g{i}_"
        out[pfx + "meta"] = np.array([M, N, K, gk, int(asym), int(sbf)], np.int64)
        out[pfx + "x"] = xb
        out[pfx + "codes"] = w.codes
        out[pfx + "ws"] = w.scale
        if w.zero is not None:
            out[pfx + "wz"] = w.zero
        out[pfx + "y"] = y
        out[pfx + "y64"] = y64
        out[pfx + "P"] = P


def ref_cpp_cases(out):
    import oracle
    if not oracle.ref_available():
        print("oracle/_ref not built: skipping the C++ reference fixtures")
        return
    rng = np.random.default_rng(41)
    for i, (M, N, K, gk, asym) in enumerate([(3, 128, 1057, 1024, True), (2, 128, 777, 128, False),
                                             (4, 128, 5120 // 8, 128, True), (3, 128, 3456, 128, True)]):
        G = -(-K // gk)
        qa = rng.integers(-128, 128, size=(M, K), dtype=np.int16).astype(np.int8)
        qw = rng.integers(-8, 8, size=(N, K), dtype=np.int16).astype(np.int8)
        as_bits = oracle.f32_to_bf16(np.float32(0.0005) + np.float32(0.0015) * rng.random((G, M), np.float32))
        ws_bits = oracle.f32_to_bf16(np.float32(0.0005) + np.float32(0.0015) * rng.random((G, N), np.float32))
        wz_bits = oracle.f32_to_bf16(rng.integers(-8, 8, size=(G, N)).astype(np.float32)) if asym else None
        pfx = f"r{i}_"
        out[pfx + "meta"] = np.array([M, N, K, gk, int(asym)], np.int64)
        out[pfx + "qa"] = qa
        out[pfx + "qw"] = qw
        out[pfx + "as"] = as_bits
        out[pfx + "ws"] = ws_bits
        if asym:
            out[pfx + "wz"] = wz_bits
        out[pfx + "wpack"] = oracle.ref_pack_int4_grouped(qw, gk)
        hi, lo = oracle.ref_split_planes_grouped(qa, gk)
        out[pfx + "a_hi"] = hi
        out[pfx + "a_lo"] = lo
        out[pfx + "aks"] = oracle.ref_act_ksum_neg(qa, gk)
        out[pfx + "wks"] = oracle.ref_weight_ksum(qw, gk)
        out[pfx + "y"] = oracle.ref_midgroup_gemm(qa, as_bits, qw, ws_bits, wz_bits, gk)


def weight_cases(reference, out):
    """Weight quantiser golden: the reference's quantize_weight
    (npu_ops/python/w4a8_ops.py:181-240) on seeded bf16 weights, including a
    constant group, an all-positive group and a ragged last group."""
    import torch
    sys.path.insert(0, os.path.join(reference, "npu_ops", "python"))
    import w4a8_ops as ref_ops
    cases = [(256, 2048, 1024, 21), (128, 1057, 1024, 22), (128, 640, 128, 23)]
    for i, (N, K, gk, seed) in enumerate(cases):
        g = torch.Generator().manual_seed(seed)
        w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
        w[0, :gk] = 0.0125                                   # constant group
        w[1, :gk] = w[1, :gk].abs() + 0.01                   # all-positive group
        w_q, w_scale, w_ksum, w_zero = ref_ops.quantize_weight(w, gk)
        p = f"w{i}_"
        out[p + "meta"] = np.array([N, K, gk], np.int64)
        out[p + "w"] = _bits(w)
        out[p + "wq"] = w_q.numpy()
        out[p + "ws"] = _bits(w_scale)
        out[p + "wk"] = w_ksum.numpy()
        out[p + "wz"] = _bits(w_zero)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("W4A8_REFERENCE"),
                    help="the reference checkout (default: $W4A8_REFERENCE)")
    ap.add_argument("--out", default=os.path.join(HERE, "golden.npz"))
    args = ap.parse_args()
    if not args.reference or not os.path.isdir(args.reference):
        ap.error("name the reference checkout with --reference or $W4A8_REFERENCE")
    sys.path.insert(0, args.reference)
    from fakequant_lab import fake_linear as fl
    from fakequant_lab import quant
    import torch
    torch.manual_seed(0)
    out = {}
    quant_cases(quant, out)
    gemm_cases(quant, fl, out)
    ref_cpp_cases(out)
    weight_cases(args.reference, out)
    np.savez_compressed(args.out, **out)
    print(f"wrote {args.out}: {len(out)} arrays, {os.path.getsize(args.out) / 1024:.0f} KiB")


if __name__ == "__main__":
    main()
