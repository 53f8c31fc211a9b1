"""Tensor-parallel layer stack on CPU, with the reference arithmetic (oracle).

Exact checks of the sharding: row-parallel K shards are group-aligned, so the
ranks' exact (float64) partial outputs sum to the unsharded output; column
shards concatenate to it bit for bit.  End to end, 2 gloo ranks run one
layer; each rank rounds its partial to bf16 before the all-reduce and the next
linear requantises the sum, so the stack is compared with a looser bound:
max|y - y1| / max|y1| <= 3e-2 and cosine >= 0.9995."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_check_dims_rejects_unaligned_shards():
    from w4a8_b200 import tp
    tp.check_dims(tp.QWQ, 8)
    with pytest.raises(ValueError):
        tp.check_dims(tp.Dims(hidden=5120, qkv=7168, ffn=27648, gk=1024), 8)


def test_shards_partition_the_layer():
    from w4a8_b200 import tp
    d = tp.Dims(hidden=256, qkv=384, ffn=512, gk=128)
    full = tp.build_layers(1, 0, 1, "cpu", d)[0]
    parts = [tp.build_layers(1, r, 2, "cpu", d)[0] for r in range(2)]
    h, kv = d.hidden // 2, (d.qkv - d.hidden) // 4
    for sec, (a, n) in enumerate(((0, h), (h, kv), (h + kv, kv))):
        full_rows = torch.cat([p.qkv.codes[a:a + n] for p in parts], 0)
        lo = (0, d.hidden, d.hidden + 2 * kv)[sec]
        assert torch.equal(full_rows, full.qkv.codes[lo:lo + 2 * n])
    assert torch.equal(torch.cat([p.o.codes for p in parts], 1), full.o.codes)
    assert torch.equal(torch.cat([p.o.scale for p in parts], 0), full.o.scale)
    f = d.ffn // 2
    gate = torch.cat([p.gate_up.codes[:f] for p in parts], 0)
    up = torch.cat([p.gate_up.codes[f:] for p in parts], 0)
    assert torch.equal(torch.cat([gate, up], 0), full.gate_up.codes)
    assert torch.equal(torch.cat([p.down.scale for p in parts], 0), full.down.scale)


def _bits(x):
    return x.contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("tp_", [2, 4])
def test_row_parallel_partials_sum_exactly(orc, tp_):
    from w4a8_b200 import tp
    d = tp.Dims(hidden=512, qkv=768, ffn=1024, gk=128)
    full = tp.build_layers(1, 0, 1, "cpu", d)[0]
    x = torch.randn(5, d.ffn, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16)
    y_full, _ = orc.linear(_bits(x), full.down.codes.numpy(), full.down.scale.numpy(), None, d.gk, exact=True)
    acc = np.zeros_like(y_full)
    k = d.ffn // tp_
    for r in range(tp_):
        w = tp.build_layers(1, r, tp_, "cpu", d)[0].down
        y_r, _ = orc.linear(_bits(x[:, r * k:(r + 1) * k]), w.codes.numpy(), w.scale.numpy(), None, d.gk, exact=True)
        acc += y_r
    np.testing.assert_allclose(acc, y_full, rtol=1e-12, atol=1e-12 * np.abs(y_full).max())


def test_column_parallel_concatenates(orc):
    from w4a8_b200 import tp
    d = tp.Dims(hidden=256, qkv=384, ffn=512, gk=128)
    full = tp.build_layers(1, 0, 1, "cpu", d)[0]
    x = torch.randn(3, d.hidden, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16)
    y_full, _ = orc.linear(_bits(x), full.gate_up.codes.numpy(), full.gate_up.scale.numpy(), None, d.gk)
    parts = []
    for r in range(2):
        w = tp.build_layers(1, r, 2, "cpu", d)[0].gate_up
        parts.append(orc.linear(_bits(x), w.codes.numpy(), w.scale.numpy(), None, d.gk)[0])
    f = d.ffn // 2
    gate = np.concatenate([p[:, :f] for p in parts], 1)
    up = np.concatenate([p[:, f:] for p in parts], 1)
    assert np.array_equal(np.concatenate([gate, up], 1), y_full)


def test_tp2_matches_tp1(orc, tmp_path):
    import torch.multiprocessing as mp

    import tp_worker
    mp.spawn(tp_worker.run, args=(2, _free_port(), str(tmp_path), 1), nprocs=2, join=True)
    outs = [np.load(os.path.join(tmp_path, f"rank{r}.npz")) for r in range(2)]
    assert np.array_equal(outs[0]["y"], outs[1]["y"]), "ranks disagree after the all-reduce"
    y, y1 = outs[0]["y"].astype(np.float64), outs[0]["y1"].astype(np.float64)
    err = np.abs(y - y1).max() / np.abs(y1).max()
    cos = float((y * y1).sum() / (np.linalg.norm(y) * np.linalg.norm(y1)))
    assert err <= 3e-2, err
    assert cos >= 0.9995, cos
