"""Mid-group W4A8 checkpoints: exporter, bitwise seam check, shard-aware loader.

On-disk format (the reference's, npu_ops/python/export_w4a8_checkpoint.py:125-186),
kept alike on purpose so checkpoints move between the two stacks unchanged:

    <proj>.weight_packed  int8  [N, k_pad_elems(K) // 2]  two int4 codes per byte, even k low
    <proj>.weight_scale   bf16  [N, G]
    <proj>.weight_zero    bf16  [N, G]
    <proj>.weight_ksum    int32 [N, G]   sum of raw codes per group

for the seven projections of every decoder layer (q, k, v, o, gate, up, down);
every other tensor passes through.  Scale-like tensors are stored [N, G] so
they concatenate along dim 0 exactly like the weight (fused q/k/v and gate/up
loaders work unchanged) and a row-parallel K shard is a dim-1 slice; the
quant method transposes them to the kernel's [G, N] once at load.
``config.json`` gets the ``quantization_config`` block the loader dispatches on.

Quantisation is per projection, not on the fused matrices.  That is exact:
groups run along K and every scale and zero point belongs to one output row,
so concatenating along N cannot move a group boundary.  ``seam`` checks it
bitwise, together with export == runtime quantisation (the reference's seam
test design, npu_ops/python/test_w4a8_ckpt_seam.py:58-97).

CLI::

    python -m w4a8_b200.checkpoint export --src BF16_DIR --dst W4A8_DIR [--group 1024]
    python -m w4a8_b200.checkpoint seam --src BF16_DIR --ckpt W4A8_DIR [--layers 0 1]
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
import sys
from typing import Callable, Dict, Iterable, List, Optional, Sequence, Tuple

import torch

from . import w4a8_ops as W

PROJ_SUFFIXES = (".self_attn.q_proj.weight", ".self_attn.k_proj.weight", ".self_attn.v_proj.weight",
                 ".self_attn.o_proj.weight", ".mlp.gate_proj.weight", ".mlp.up_proj.weight",
                 ".mlp.down_proj.weight")
TENSOR_SUFFIXES = ("weight_packed", "weight_scale", "weight_zero", "weight_ksum")
AUX_FILES = ("tokenizer.json", "tokenizer_config.json", "vocab.json", "merges.txt", "added_tokens.json",
             "special_tokens_map.json", "generation_config.json", "configuration.json")
INDEX = "model.safetensors.index.json"

Getter = Callable[[str], torch.Tensor]


def is_quant_target(key: str) -> bool:
    """The projections the W4A8 kernel takes over; everything else stays as it is."""
    return key.startswith("model.layers.") and key.endswith(PROJ_SUFFIXES)


def quant_config_block(group: int) -> dict:
    return {"quant_method": "midgroup_w4a8", "group_size": group, "weight_bits": 4, "activation_bits": 8,
            "sym": False, "packed_layout": "mg_kgeom_v1", "ignored_layers": ["lm_head"]}


def quantize_projection(w: torch.Tensor, group: int) -> Dict[str, torch.Tensor]:
    """One projection's four on-disk tensors (scale-likes [N, G])."""
    wq, ws, wk, wz = W.quantize_weight(w.to(torch.bfloat16), group)
    return {"weight_packed": wq.contiguous(), "weight_scale": ws.t().contiguous(),
            "weight_zero": wz.t().contiguous(), "weight_ksum": wk.t().contiguous()}


def open_checkpoint(path: str) -> Tuple[Dict[str, str], Getter]:
    """(weight_map, get) over a sharded safetensors directory; files open lazily."""
    from safetensors import safe_open
    weight_map = json.load(open(os.path.join(path, INDEX)))["weight_map"]
    handles: Dict[str, object] = {}

    def get(key: str) -> torch.Tensor:
        f = weight_map[key]
        if f not in handles:
            handles[f] = safe_open(os.path.join(path, f), framework="pt")
        return handles[f].get_tensor(key)
    return weight_map, get


def _layer_of(key: str) -> Optional[int]:
    return int(key.split(".")[2]) if key.startswith("model.layers.") else None


def export(src: str, dst: str, group: int = W.GROUP, shard_bytes: float = 4e9, layers: int = 0,
           log: Callable[[str], None] = print) -> Dict[str, int]:
    """Write the mid-group W4A8 checkpoint of the bf16 checkpoint in ``src`` to ``dst``.

    ``layers`` > 0 keeps only the first that many decoder layers (and sets
    ``num_hidden_layers``).  Shards hold about ``shard_bytes`` each; source files
    are read one at a time."""
    from safetensors import safe_open
    from safetensors.torch import save_file
    os.makedirs(dst, exist_ok=True)
    weight_map = json.load(open(os.path.join(src, INDEX)))["weight_map"]
    by_file: Dict[str, List[str]] = {}
    for k, f in weight_map.items():
        if layers and _layer_of(k) is not None and _layer_of(k) >= layers:
            continue
        by_file.setdefault(f, []).append(k)
    index: Dict[str, str] = {}
    pending: Dict[str, torch.Tensor] = {}
    state = {"bytes": 0, "shards": 0, "quantised": 0, "passed": 0}

    def flush(final: bool) -> None:
        if not pending or (not final and state["bytes"] < shard_bytes):
            return
        state["shards"] += 1
        name = f"model-{state['shards']:05d}.safetensors"
        save_file(dict(pending), os.path.join(dst, name), metadata={"format": "pt"})
        for k in pending:
            index[k] = name
        log(f"[export] {name}: {len(pending)} tensors, {state['bytes'] / 1e9:.2f} GB")
        pending.clear()
        state["bytes"] = 0

    for fname in sorted(by_file):
        with safe_open(os.path.join(src, fname), framework="pt") as f:
            for key in sorted(by_file[fname]):
                t = f.get_tensor(key)
                if is_quant_target(key):
                    base = key[: -len(".weight")]
                    for suf, v in quantize_projection(t, group).items():
                        pending[f"{base}.{suf}"] = v
                        state["bytes"] += v.numel() * v.element_size()
                    state["quantised"] += 1
                else:
                    pending[key] = t.contiguous()
                    state["bytes"] += t.numel() * t.element_size()
                    state["passed"] += 1
                flush(False)
    flush(True)
    total = sum(os.path.getsize(os.path.join(dst, n)) for n in set(index.values()))
    json.dump({"metadata": {"total_size": total}, "weight_map": dict(sorted(index.items()))},
              open(os.path.join(dst, INDEX), "w"), indent=1)
    cfg_path = os.path.join(src, "config.json")
    cfg = json.load(open(cfg_path)) if os.path.exists(cfg_path) else {}
    if layers:
        cfg["num_hidden_layers"] = layers
    cfg["quantization_config"] = quant_config_block(group)
    json.dump(cfg, open(os.path.join(dst, "config.json"), "w"), indent=2)
    for aux in AUX_FILES:
        if os.path.exists(os.path.join(src, aux)):
            shutil.copy2(os.path.join(src, aux), os.path.join(dst, aux))
    log(f"[export] {state['quantised']} projections quantised, {state['passed']} tensors passed through, "
        f"{state['shards']} shards, {total / 1e9:.3f} GB")
    return {"quantised": state["quantised"], "passed": state["passed"], "shards": state["shards"], "bytes": total}


# ---------------------------------------------------------------- seam check

FUSED = (("self_attn", "qkv", ("q", "k", "v")), ("mlp", "gate_up", ("gate", "up")))


def _same(a: torch.Tensor, b: torch.Tensor) -> bool:
    return a.shape == b.shape and a.dtype == b.dtype and torch.equal(a, b)


def seam(src_get: Getter, ck_get: Getter, layers: Iterable[int], group: int) -> Tuple[int, List[str]]:
    """Bitwise seam between the exported checkpoint and runtime quantisation.

    1. per projection: the four exported tensors == quantize_weight(bf16 weight);
    2. fusion: the exported q/k/v (gate/up) tensors concatenated along N ==
       quantize_weight of the concatenated bf16 weight.
    Returns (number of checks, failure messages)."""
    checks, fails = 0, []
    for li in layers:
        pfx = f"model.layers.{li}"
        for block, _, members in FUSED + (("self_attn", "o", ("o",)), ("mlp", "down", ("down",))):
            for m in members:
                name = f"{pfx}.{block}.{m}_proj"
                ref = quantize_projection(src_get(f"{name}.weight"), group)
                for suf in TENSOR_SUFFIXES:
                    checks += 1
                    if not _same(ref[suf], ck_get(f"{name}.{suf}")):
                        fails.append(f"{name}.{suf}")
        for block, fused, members in FUSED:
            base = f"{pfx}.{block}"
            ref = quantize_projection(torch.cat([src_get(f"{base}.{m}_proj.weight") for m in members], 0), group)
            for suf in TENSOR_SUFFIXES:
                checks += 1
                got = torch.cat([ck_get(f"{base}.{m}_proj.{suf}") for m in members], 0)
                if not _same(ref[suf], got):
                    fails.append(f"{base}.{fused} (fused).{suf}")
    return checks, fails


# ---------------------------------------------------------------- loading

def load_projection(ck_get: Getter, names: Sequence[str], rank: int = 0, tp: int = 1,
                    row_parallel: bool = False, k: Optional[int] = None,
                    group: Optional[int] = None) -> Dict[str, torch.Tensor]:
    """The on-disk tensors of one (possibly fused) linear as rank ``rank`` of
    ``tp`` holds them, the way vLLM's loaders cut them.

    Column-parallel (default): each member projection is split along N and the
    rank's pieces are concatenated in member order (QKVParallelLinear /
    MergedColumnParallelLinear).  Row-parallel: one projection, split along K
    (dim 1 of every tensor); ``k`` and ``group`` are required and the shard must
    land on group boundaries (K a multiple of tp * group, group a multiple of
    64), so every group's codes are a whole, equal number of packed bytes."""
    if row_parallel and tp > 1:
        if k is None or group is None or k % (tp * group) or group % 64:
            raise ValueError(f"row-parallel K = {k} does not split {tp} ways on groups of {group}")
    out: Dict[str, torch.Tensor] = {}
    for suf in TENSOR_SUFFIXES:
        parts = []
        for name in names:
            t = ck_get(f"{name}.{suf}")
            if row_parallel:
                if t.shape[1] % tp:
                    raise ValueError(f"{name}.{suf}: dim 1 = {t.shape[1]} does not split {tp} ways")
                s = t.shape[1] // tp
                parts.append(t[:, rank * s:(rank + 1) * s])
            else:
                if t.shape[0] % tp:
                    raise ValueError(f"{name}.{suf}: N = {t.shape[0]} does not split {tp} ways")
                s = t.shape[0] // tp
                parts.append(t[rank * s:(rank + 1) * s])
        out[suf] = torch.cat(parts, 0).contiguous()
    return out


def load_into_layer(layer: torch.nn.Module, tensors: Dict[str, torch.Tensor]) -> None:
    """Copy loaded on-disk tensors into the parameters ``create_weights`` made."""
    for suf in TENSOR_SUFFIXES:
        p = getattr(layer, suf)
        src = tensors[suf]
        if tuple(p.shape) != tuple(src.shape) or p.dtype != src.dtype:
            raise ValueError(f"{suf}: parameter {tuple(p.shape)} {p.dtype} vs checkpoint "
                             f"{tuple(src.shape)} {src.dtype}")
        p.data.copy_(src)


# ---------------------------------------------------------------- CLI

def main(argv: Optional[Sequence[str]] = None) -> int:
    ap = argparse.ArgumentParser(prog="python -m w4a8_b200.checkpoint")
    sub = ap.add_subparsers(dest="cmd", required=True)
    e = sub.add_parser("export", help="bf16 HF checkpoint -> mid-group W4A8 checkpoint")
    e.add_argument("--src", required=True)
    e.add_argument("--dst", required=True)
    e.add_argument("--group", type=int, default=W.GROUP)
    e.add_argument("--shard-gb", type=float, default=4.0)
    e.add_argument("--layers", type=int, default=0, help="export only the first N layers; 0 = all")
    s = sub.add_parser("seam", help="bitwise check: exported == runtime quantisation, fused == concat")
    s.add_argument("--src", required=True)
    s.add_argument("--ckpt", required=True)
    s.add_argument("--layers", type=int, nargs="+", default=[0])
    args = ap.parse_args(argv)
    if args.cmd == "export":
        export(args.src, args.dst, args.group, args.shard_gb * 1e9, args.layers)
        return 0
    group = json.load(open(os.path.join(args.ckpt, "config.json")))["quantization_config"]["group_size"]
    _, sget = open_checkpoint(args.src)
    _, cget = open_checkpoint(args.ckpt)
    checks, fails = seam(sget, cget, args.layers, group)
    for f in fails:
        print(f"FAIL {f}")
    print(f"[seam] {checks - len(fails)}/{checks} bitwise checks passed")
    return 1 if fails else 0


if __name__ == "__main__":
    sys.exit(main())
