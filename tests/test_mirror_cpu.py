"""The reference-facing Python surface without a GPU: the weight quantiser
against the reference's own outputs (bit-exact), the torch op schemas and fake
kernels, and the vLLM quant method's parameter contract."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")


def _bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits, np.uint16).view(np.int16)).view(torch.bfloat16)


@pytest.mark.parametrize("case", [0, 1, 2])
def test_quantize_weight_matches_reference(golden, case):
    from w4a8_b200 import w4a8_ops
    p = f"w{case}_"
    N, K, gk = (int(v) for v in golden[p + "meta"])
    w_q, w_scale, w_ksum, w_zero = w4a8_ops.quantize_weight(_bf16(golden[p + "w"]), gk)
    assert np.array_equal(w_q.numpy(), golden[p + "wq"])
    assert np.array_equal(_bits(w_scale), golden[p + "ws"])
    assert np.array_equal(w_ksum.numpy(), golden[p + "wk"])
    assert np.array_equal(_bits(w_zero), golden[p + "wz"])


def test_torch_ops_registered_with_fake_kernels():
    from torch._subclasses.fake_tensor import FakeTensorMode

    from w4a8_b200 import w4a8_ops
    w4a8_ops.load()
    M, K, N, gk = 20, 2048, 256, 128
    with FakeTensorMode():
        x = torch.empty(M, K, dtype=torch.bfloat16, device="meta")
        a_hi, a_lo, a_s, a_k = torch.ops.npu.midgroup_quant_a(x)
        assert a_hi.shape == (64, 1024) and a_s.shape == (2, 64) and a_k.dtype == torch.int32
        wq = torch.empty(N, 1024, dtype=torch.int8, device="meta")
        ws = torch.empty(2, N, dtype=torch.bfloat16, device="meta")
        y = torch.ops.npu.midgroup_w4a8_gemm(a_hi, a_lo, a_s, a_k, wq, ws, a_k, ws, K)
        assert y.shape == (64, N) and y.dtype == torch.bfloat16
        ws2 = torch.empty(16, N, dtype=torch.float32, device="meta")
        y2 = torch.ops.w4a8.linear(x, wq, ws2, None, gk)
        assert y2.shape == (M, N)


def test_ops_refuse_cpu_tensors():
    from w4a8_b200 import w4a8_ops
    w4a8_ops.load()
    x = torch.zeros(4, 256, dtype=torch.bfloat16)
    with pytest.raises((RuntimeError, NotImplementedError)):
        torch.ops.w4a8.linear(x, torch.zeros(128, 128, dtype=torch.int8), torch.ones(2, 128), None, 128)


def test_quant_method_parameter_contract():
    pytest.importorskip("vllm")
    from w4a8_b200 import midgroup_quant as mq
    cfg = mq.MidGroupW4A8Config.from_config({"group_size": 128, "sym": False})
    assert cfg.get_name() == "midgroup_w4a8"
    meth = mq.MidGroupW4A8LinearMethod(cfg, "model.layers.0.mlp.down_proj")
    layer = torch.nn.Module()
    meth.create_weights(layer, 1024, [512], 1024, 512, torch.bfloat16)
    assert layer.weight_packed.shape == (512, 512) and layer.weight_scale.shape == (512, 8)
    assert layer.weight_zero.dtype == torch.bfloat16 and layer.weight_ksum.dtype == torch.int32
    assert getattr(layer.weight_scale, "output_dim") == 0 and not hasattr(layer.weight_scale, "input_dim")
    # a group-aligned row-parallel shard is accepted and marked for narrowing
    shard = torch.nn.Module()
    meth.create_weights(shard, 512, [512], 1024, 512, torch.bfloat16)
    assert shard.weight_packed.shape == (512, 256) and getattr(shard.weight_packed, "input_dim") == 1
    # a shard that cuts a group is refused, as is N not a multiple of 128
    cfg1024 = mq.MidGroupW4A8Config(group_size=1024)
    with pytest.raises(ValueError):
        mq.MidGroupW4A8LinearMethod(cfg1024).create_weights(torch.nn.Module(), 2560, [512], 5120, 512, torch.bfloat16)
    with pytest.raises(ValueError):
        meth.create_weights(torch.nn.Module(), 1024, [500], 1024, 500, torch.bfloat16)
