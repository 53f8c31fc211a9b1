"""Checkpoint -> quant method -> CUDA op, end to end on the GPU.

An exported checkpoint, loaded through ``MidGroupW4A8LinearMethod`` (create_weights,
copy, process_weights_after_loading), must give bit-for-bit the output of the op
on runtime-quantised weights (TP = 1); row-parallel shards summed over two
ranks must match the float64 reference within the parity tolerance.
"""
import numpy as np
import pytest
import torch

from test_checkpoint_cpu import FFN, HIDDEN, KV, make_src

pytestmark = pytest.mark.gpu


def _layer(cfg, names, row, K, outs, rank, tp, cget, gk):
    from w4a8_b200 import checkpoint as C
    from w4a8_b200.midgroup_quant import MidGroupW4A8LinearMethod
    layer = torch.nn.Module()
    meth = MidGroupW4A8LinearMethod(cfg, names[0])
    meth.create_weights(layer, K // tp if row else K, outs, K, sum(outs), torch.bfloat16)
    C.load_into_layer(layer, C.load_projection(cget, names, rank, tp, row, K, gk))
    layer.to("cuda")
    meth.process_weights_after_loading(layer)
    return meth, layer


@pytest.mark.parametrize("gk", [128, 1024])
def test_checkpoint_load_apply_bitwise(tmp_path, gk):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from w4a8_b200 import checkpoint as C
    from w4a8_b200 import ops
    from w4a8_b200 import w4a8_ops as W
    from w4a8_b200.midgroup_quant import MidGroupW4A8Config
    tensors = make_src(str(tmp_path / "bf16"), layers=1, seed=3)
    C.export(str(tmp_path / "bf16"), str(tmp_path / "ck"), group=gk, log=lambda s: None)
    _, cget = C.open_checkpoint(str(tmp_path / "ck"))
    cfg = MidGroupW4A8Config(group_size=gk)
    p = "model.layers.0"
    gen = torch.Generator().manual_seed(7)
    for names, K, bias in (([f"{p}.self_attn.{m}_proj" for m in "qkv"], HIDDEN, True),
                           ([f"{p}.mlp.gate_proj", f"{p}.mlp.up_proj"], HIDDEN, False),
                           ([f"{p}.mlp.down_proj"], FFN, False)):
        outs = [tensors[n + ".weight"].shape[0] for n in names]
        meth, layer = _layer(cfg, names, False, K, outs, 0, 1, cget, gk)
        x = torch.randn(5, K, generator=gen).to(torch.bfloat16).cuda()
        b = torch.cat([tensors[n + ".bias"] for n in names]).cuda() if bias else None
        y = meth.apply(layer, x, b)
        wq, ws, _, wz = W.quantize_weight(torch.cat([tensors[n + ".weight"] for n in names], 0), gk)
        ref = ops.linear(x, wq.cuda(), ws.cuda(), wz.cuda(), gk)
        if b is not None:
            ref = ref + b
        assert torch.equal(y, ref), names[0]
    assert ops.workspace_status() == 0


def test_checkpoint_row_parallel_two_ranks(tmp_path, orc):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from w4a8_b200 import checkpoint as C
    from w4a8_b200 import ops
    from w4a8_b200.midgroup_quant import MidGroupW4A8Config
    gk, tp = 128, 2
    tensors = make_src(str(tmp_path / "bf16"), layers=1, seed=4)
    C.export(str(tmp_path / "bf16"), str(tmp_path / "ck"), group=gk, log=lambda s: None)
    _, cget = C.open_checkpoint(str(tmp_path / "ck"))
    cfg = MidGroupW4A8Config(group_size=gk)
    name = "model.layers.0.mlp.down_proj"
    xb = (torch.randn(9, FFN, generator=torch.Generator().manual_seed(11))).to(torch.bfloat16)
    acc = torch.zeros(9, HIDDEN, dtype=torch.float32, device="cuda")
    for rank in range(tp):
        meth, layer = _layer(cfg, [name], True, FFN, [HIDDEN], rank, tp, cget, gk)
        s = FFN // tp
        acc += meth.apply(layer, xb[:, rank * s:(rank + 1) * s].cuda()).float()
    full = C.load_projection(cget, [name])
    codes = orc.unpack_int4_grouped(full["weight_packed"].numpy(), FFN, gk)
    ws = full["weight_scale"].t().float().numpy()
    wz = full["weight_zero"].t().float().numpy()
    xbits = xb.view(torch.int16).numpy().view(np.uint16)
    y64, _ = orc.linear(xbits, codes, ws, wz, gk, exact=True)
    y = acc.cpu().numpy().astype(np.float64)
    err = np.abs(y - y64).max() / np.abs(y64).max()
    cos = float((y * y64).sum() / (np.linalg.norm(y) * np.linalg.norm(y64)))
    assert err <= 1e-2 and cos >= 0.9999, (err, cos)
    assert ops.workspace_status() == 0
