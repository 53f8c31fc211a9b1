"""Checkpoint exporter / loader parity on CPU (synthetic bf16 checkpoints).

The design follows the reference's bitwise seam test
(npu_ops/python/test_w4a8_ckpt_seam.py:58-97): exported tensors must equal
runtime quantisation bit for bit, and quantising per projection must equal
quantising the fused q/k/v and gate/up matrices.  On top of that: a tampered
checkpoint must fail the seam, tensor-parallel shards cut the way vLLM's
loaders cut them must equal quantising the bf16 shard itself, and the shards
must fit the parameters the quant method creates.
"""
import json
import os
import shutil

import pytest
import torch

from w4a8_b200 import checkpoint as C
from w4a8_b200 import w4a8_ops as W

HIDDEN, KV, FFN, LAYERS = 256, 64, 512, 2


def _w(gen, n, k):
    w = torch.randn(n, k, generator=gen) * 0.02
    # a few large input channels, as real projections have
    idx = torch.randint(0, k, (max(1, k // 64),), generator=gen)
    w[:, idx] *= 8
    return w.to(torch.bfloat16)


def make_src(path, layers=LAYERS, seed=0):
    from safetensors.torch import save_file
    os.makedirs(path, exist_ok=True)
    gen = torch.Generator().manual_seed(seed)
    t = {"model.embed_tokens.weight": _w(gen, 64, HIDDEN), "model.norm.weight": torch.ones(HIDDEN, dtype=torch.bfloat16),
         "lm_head.weight": _w(gen, 64, HIDDEN)}
    for li in range(layers):
        p = f"model.layers.{li}"
        t[f"{p}.self_attn.q_proj.weight"] = _w(gen, HIDDEN, HIDDEN)
        t[f"{p}.self_attn.k_proj.weight"] = _w(gen, KV, HIDDEN)
        t[f"{p}.self_attn.v_proj.weight"] = _w(gen, KV, HIDDEN)
        for b, n in (("q", HIDDEN), ("k", KV), ("v", KV)):
            t[f"{p}.self_attn.{b}_proj.bias"] = (torch.randn(n, generator=gen) * 0.1).to(torch.bfloat16)
        t[f"{p}.self_attn.o_proj.weight"] = _w(gen, HIDDEN, HIDDEN)
        t[f"{p}.mlp.gate_proj.weight"] = _w(gen, FFN, HIDDEN)
        t[f"{p}.mlp.up_proj.weight"] = _w(gen, FFN, HIDDEN)
        t[f"{p}.mlp.down_proj.weight"] = _w(gen, HIDDEN, FFN)
        t[f"{p}.input_layernorm.weight"] = torch.ones(HIDDEN, dtype=torch.bfloat16)
    keys = sorted(t)
    files = {"model-00001-of-00002.safetensors": keys[: len(keys) // 2],
             "model-00002-of-00002.safetensors": keys[len(keys) // 2:]}
    wm = {}
    for f, ks in files.items():
        save_file({k: t[k].contiguous() for k in ks}, os.path.join(path, f), metadata={"format": "pt"})
        wm.update({k: f for k in ks})
    json.dump({"metadata": {}, "weight_map": wm}, open(os.path.join(path, C.INDEX), "w"))
    json.dump({"num_hidden_layers": layers, "hidden_size": HIDDEN, "intermediate_size": FFN},
              open(os.path.join(path, "config.json"), "w"))
    open(os.path.join(path, "tokenizer.json"), "w").write("{}")
    return t


@pytest.fixture(scope="module")
def src(tmp_path_factory):
    p = str(tmp_path_factory.mktemp("bf16"))
    return p, make_src(p)


@pytest.fixture(scope="module", params=[128, 1024])
def exported(src, tmp_path_factory, request):
    gk = request.param
    dst = str(tmp_path_factory.mktemp(f"w4a8_{gk}"))
    stats = C.export(src[0], dst, group=gk, shard_bytes=200_000, log=lambda s: None)
    return gk, dst, stats


def test_seam_bitwise(src, exported):
    gk, dst, stats = exported
    _, sget = C.open_checkpoint(src[0])
    _, cget = C.open_checkpoint(dst)
    checks, fails = C.seam(sget, cget, range(LAYERS), gk)
    assert checks == LAYERS * (7 * 4 + 2 * 4)
    assert fails == []
    assert stats["quantised"] == 7 * LAYERS and stats["shards"] >= 2


def test_export_format(src, exported):
    gk, dst, _ = exported
    tensors = src[1]
    wm, cget = C.open_checkpoint(dst)
    cfg = json.load(open(os.path.join(dst, "config.json")))
    assert cfg["quantization_config"] == C.quant_config_block(gk)
    assert cfg["num_hidden_layers"] == LAYERS and os.path.exists(os.path.join(dst, "tokenizer.json"))
    for k, v in tensors.items():
        if C.is_quant_target(k):
            base = k[: -len(".weight")]
            assert k not in wm
            N, K = v.shape
            G = W.num_groups(K, gk)
            assert tuple(cget(base + ".weight_packed").shape) == (N, W.k_pad_elems(K, gk) // 2)
            for suf, dt in (("weight_scale", torch.bfloat16), ("weight_zero", torch.bfloat16),
                            ("weight_ksum", torch.int32)):
                t = cget(f"{base}.{suf}")
                assert tuple(t.shape) == (N, G) and t.dtype == dt
        else:
            assert torch.equal(cget(k), v)                      # passed through unchanged


def test_export_first_layers_only(src, tmp_path):
    dst = str(tmp_path / "l1")
    C.export(src[0], dst, group=128, layers=1, log=lambda s: None)
    wm, _ = C.open_checkpoint(dst)
    assert not any(k.startswith("model.layers.1.") for k in wm)
    assert any(k.startswith("model.layers.0.") for k in wm) and "lm_head.weight" in wm
    assert json.load(open(os.path.join(dst, "config.json")))["num_hidden_layers"] == 1


def test_seam_detects_tampering(src, exported, tmp_path):
    """Negative control: one changed scale, or a swapped fused member, must fail."""
    from safetensors.torch import load_file, save_file
    gk, dst, _ = exported
    bad = str(tmp_path / "bad")
    shutil.copytree(dst, bad)
    wm, _ = C.open_checkpoint(bad)
    key = "model.layers.1.mlp.up_proj.weight_scale"
    f = os.path.join(bad, wm[key])
    d = load_file(f)
    d[key] = d[key].clone()
    d[key][3, 0] = d[key][3, 0] * 2
    save_file(d, f, metadata={"format": "pt"})
    _, sget = C.open_checkpoint(src[0])
    _, cget = C.open_checkpoint(bad)
    checks, fails = C.seam(sget, cget, range(LAYERS), gk)
    assert "model.layers.1.mlp.up_proj.weight_scale" in fails
    assert "model.layers.1.mlp.gate_up (fused).weight_scale" in fails

    def swapped(k):                                            # k and v exchanged on disk
        if ".self_attn.k_proj." in k:
            return C.open_checkpoint(dst)[1](k.replace(".k_proj.", ".v_proj."))
        if ".self_attn.v_proj." in k:
            return C.open_checkpoint(dst)[1](k.replace(".v_proj.", ".k_proj."))
        return C.open_checkpoint(dst)[1](k)
    _, fails = C.seam(sget, swapped, [0], gk)
    assert any("k_proj" in f for f in fails)


@pytest.mark.parametrize("tp", [1, 2])
def test_tp_shards_equal_shard_quantisation(src, exported, tp):
    """vLLM-style shards of the checkpoint == quantising the bf16 shard itself."""
    gk, dst, _ = exported
    tensors = src[1]
    _, cget = C.open_checkpoint(dst)
    for li in range(LAYERS):
        p = f"model.layers.{li}"
        for rank in range(tp):
            # column-parallel, fused sections: per-member row slices, member order
            names = [f"{p}.self_attn.{m}_proj" for m in ("q", "k", "v")]
            got = C.load_projection(cget, names, rank, tp)
            parts = []
            for n in names:
                w = tensors[n + ".weight"]
                s = w.shape[0] // tp
                parts.append(w[rank * s:(rank + 1) * s])
            ref = C.quantize_projection(torch.cat(parts, 0), gk)
            for suf in C.TENSOR_SUFFIXES:
                assert torch.equal(got[suf], ref[suf]), (li, rank, suf)
            # row-parallel down (K = FFN): only group-aligned shards
            if tp > 1 and FFN % (tp * gk):
                with pytest.raises(ValueError):
                    C.load_projection(cget, [f"{p}.mlp.down_proj"], rank, tp, True, FFN, gk)
                continue
            got = C.load_projection(cget, [f"{p}.mlp.down_proj"], rank, tp, True, FFN, gk)
            w = tensors[f"{p}.mlp.down_proj.weight"]
            s = FFN // tp
            ref = C.quantize_projection(w[:, rank * s:(rank + 1) * s], gk)
            for suf in C.TENSOR_SUFFIXES:
                assert torch.equal(got[suf], ref[suf]), (li, rank, suf)


@pytest.mark.parametrize("tp", [1, 2])
def test_shards_fit_quant_method_parameters(exported, tp):
    """create_weights of the quant method accepts every shard (shapes and dtypes)."""
    from w4a8_b200.midgroup_quant import MidGroupW4A8Config, MidGroupW4A8LinearMethod
    gk, dst, _ = exported
    _, cget = C.open_checkpoint(dst)
    cfg = MidGroupW4A8Config(group_size=gk)
    p = "model.layers.0"
    cases = [([f"{p}.self_attn.{m}_proj" for m in "qkv"], False, HIDDEN, [HIDDEN // tp, KV // tp, KV // tp]),
             ([f"{p}.mlp.gate_proj", f"{p}.mlp.up_proj"], False, HIDDEN, [FFN // tp, FFN // tp]),
             ([f"{p}.self_attn.o_proj"], True, HIDDEN, [HIDDEN]),
             ([f"{p}.mlp.down_proj"], True, FFN, [HIDDEN])]
    for rank in range(tp):
        for names, row, K, outs in cases:
            k_part = K // tp if row else K
            layer = torch.nn.Module()
            meth = MidGroupW4A8LinearMethod(cfg, names[0])
            if row and tp > 1 and K % (tp * gk):
                with pytest.raises(ValueError):
                    meth.create_weights(layer, k_part, outs, K, sum(outs), torch.bfloat16)
                continue
            if sum(outs) % 128:
                continue                                       # the kernel needs N % 128 == 0
            meth.create_weights(layer, k_part, outs, K, sum(outs), torch.bfloat16)
            C.load_into_layer(layer, C.load_projection(cget, names, rank, tp, row, K, gk))
            assert layer.mg_k == k_part and layer.mg_n == sum(outs)
