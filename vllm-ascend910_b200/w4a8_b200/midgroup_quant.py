"""vLLM quantization method ``midgroup_w4a8`` on the B200 kernels.

Mirrors npu_ops/python/midgroup_quant.py: the same config name and class names,
the same checkpoint tensors and the same ``apply(layer, x, bias)``.

Checkpoint tensors per projection (export_w4a8_checkpoint.py:125-186):

    <proj>.weight_packed  [N, k_pad_elems(K)//2]  int8   two int4 codes per byte, even k low
    <proj>.weight_scale   [N, G]                  bf16
    <proj>.weight_zero    [N, G]                  bf16
    <proj>.weight_ksum    [N, G]                  int32  sum of raw codes (unused by this kernel)

All four carry ``output_dim=0`` so vLLM's fused (qkv, gate_up) and column-parallel
loaders concatenate along N.  After loading, the scale-like tensors are
transposed to the kernel's [G, N] (midgroup_quant.py:148-161), and the weights are
regrouped once into the GEMM's tile order (``w4a8_prepare_weights``); the raw
packed copy is then released.

Row-parallel shards: the reference refuses any K shard.  Here a K shard is
accepted when it lands on group boundaries (K_shard and K both multiples of the
group size, which is a multiple of 64, so the packed bytes, scales and zero
points split into whole groups); the parameters then carry ``input_dim=1`` and
vLLM's row-parallel loader narrows them.  Other shards raise.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import ops
from . import w4a8_ops as W

try:                                                     # vLLM is optional for the kernels
    from vllm.model_executor.layers.linear import LinearBase, LinearMethodBase
    from vllm.model_executor.layers.quantization.base_config import QuantizationConfig
    HAVE_VLLM = True
except Exception:                                        # pragma: no cover - exercised without vLLM
    HAVE_VLLM = False

    class LinearBase(torch.nn.Module):                   # type: ignore[no-redef]
        pass

    class LinearMethodBase:                              # type: ignore[no-redef]
        pass

    class QuantizationConfig:                            # type: ignore[no-redef]
        def __init__(self):
            pass

TILE_N = 128
# The GEMM folds the zero point into its int8 operand: W - zero must fit int8,
# so zero points must be integers in [ZERO_MIN, ZERO_MAX] (the quantiser's
# QMIN - round(min/scale) lies in [-8, 7] whenever a group spans both signs).
ZERO_MIN, ZERO_MAX = -23, 7


class MidGroupW4A8Config(QuantizationConfig):
    """Config block written into config.json by the exporter (midgroup_quant.py:47-98)."""

    def __init__(self, group_size: int = 1024, sym: bool = False, ignored_layers: Optional[list] = None):
        super().__init__()
        self.group_size = group_size
        self.sym = sym
        self.ignored_layers = ignored_layers or ["lm_head"]
        self.quant_description: dict = {}

    def __repr__(self) -> str:
        return f"MidGroupW4A8Config(group_size={self.group_size}, sym={self.sym})"

    @classmethod
    def get_name(cls) -> str:
        return "midgroup_w4a8"

    @classmethod
    def get_supported_act_dtypes(cls) -> list:
        return [torch.bfloat16]

    @classmethod
    def get_min_capability(cls) -> int:
        return 100          # sm_100

    @classmethod
    def get_config_filenames(cls) -> list:
        return []

    @classmethod
    def from_config(cls, config: dict) -> "MidGroupW4A8Config":
        return cls(group_size=config.get("group_size", 1024), sym=config.get("sym", False),
                   ignored_layers=config.get("ignored_layers", ["lm_head"]))

    def get_quant_method(self, layer: torch.nn.Module, prefix: str):
        if not isinstance(layer, LinearBase):
            return None
        if any(ig in prefix for ig in self.ignored_layers):
            from vllm.model_executor.layers.linear import UnquantizedLinearMethod
            return UnquantizedLinearMethod()
        return MidGroupW4A8LinearMethod(self, prefix)


class MidGroupW4A8LinearMethod(LinearMethodBase):
    """create_weights / process_weights_after_loading / apply (midgroup_quant.py:101-178)."""

    def __init__(self, quant_config: MidGroupW4A8Config, prefix: str = ""):
        self.quant_config = quant_config
        self.prefix = prefix

    def create_weights(self, layer: torch.nn.Module, input_size_per_partition: int, output_partition_sizes: list,
                       input_size: int, output_size: int, params_dtype: torch.dtype, **extra_weight_attrs) -> None:
        gk = self.quant_config.group_size
        k = input_size_per_partition
        n = sum(output_partition_sizes)
        sharded_k = k != input_size
        if sharded_k and (k % gk or input_size % gk or gk % 64):
            raise ValueError(
                f"{self.prefix}: row-parallel shard K={k} of {input_size} does not land on group "
                f"boundaries of {gk}; export the checkpoint for this TP degree or run TP=1")
        if n % TILE_N:
            raise ValueError(f"{self.prefix}: N={n} not a multiple of {TILE_N}")
        g = W.num_groups(k, gk)
        kpad = W.k_pad_elems(k, gk)
        loader = extra_weight_attrs.get("weight_loader")

        def add(name: str, t: torch.Tensor) -> None:
            p = torch.nn.Parameter(t, requires_grad=False)
            setattr(p, "output_dim", 0)
            if sharded_k:
                setattr(p, "input_dim", 1)
            if loader is not None:
                setattr(p, "weight_loader", loader)
            layer.register_parameter(name, p)

        add("weight_packed", torch.empty(n, kpad // 2, dtype=torch.int8))
        add("weight_scale", torch.empty(n, g, dtype=torch.bfloat16))
        add("weight_zero", torch.empty(n, g, dtype=torch.bfloat16))
        add("weight_ksum", torch.empty(n, g, dtype=torch.int32))
        layer.mg_k = k
        layer.mg_n = n
        layer.mg_gk = gk

    def process_weights_after_loading(self, layer: torch.nn.Module) -> None:
        """[N, G] -> [G, N], then the one-time regrouping into the GEMM's tile order."""
        W.load()
        for name in ("weight_scale", "weight_zero", "weight_ksum"):
            t = getattr(layer, name).data.t().contiguous()
            delattr(layer, name)
            layer.register_parameter(name, torch.nn.Parameter(t, requires_grad=False))
        zero = None if self.quant_config.sym else layer.weight_zero.data
        if zero is not None:
            zf = zero.float()
            if not bool(torch.all((zf == torch.round(zf)) & (zf >= ZERO_MIN) & (zf <= ZERO_MAX))):
                raise ValueError(f"{self.prefix}: zero points must be integers in [{ZERO_MIN}, {ZERO_MAX}]")
        packed = layer.weight_packed.data.contiguous()
        layer.w4a8_prepared = ops.prepare_weights(packed, layer.weight_scale.data, zero, layer.mg_k, layer.mg_gk)
        # the prepared buffer holds the same weights, scales and zero points
        layer.weight_packed = torch.nn.Parameter(packed.new_empty((0, packed.shape[1])), requires_grad=False)

    def apply(self, layer: torch.nn.Module, x: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Straight-line and graph-capturable, like the reference's apply."""
        y = ops.linear_prepared(x.to(torch.bfloat16), layer.w4a8_prepared)
        if bias is not None:
            y = y + bias
        return y


def register() -> None:
    """Make ``quant_method: midgroup_w4a8`` resolvable by vLLM (midgroup_quant.py:181-206):
    register the config class and add the name to the platform's allow-list."""
    from vllm.model_executor.layers.quantization import register_quantization_config
    try:
        register_quantization_config("midgroup_w4a8")(MidGroupW4A8Config)
    except ValueError:
        pass
    from vllm.platforms import current_platform
    allow = getattr(type(current_platform), "supported_quantization", None)
    if allow is not None and "midgroup_w4a8" not in allow:
        allow.append("midgroup_w4a8")
