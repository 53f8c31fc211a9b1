"""Host-side logic of the custom all-reduce: which tensors take the one-shot path."""
import torch

from w4a8_b200.allreduce import DEFAULT_MAX_BYTES, eligible


def test_eligibility():
    mb = DEFAULT_MAX_BYTES
    assert eligible(16 * 5120, torch.bfloat16, True, 1 << 20, mb)
    assert eligible(64 * 5120, torch.bfloat16, True, 256, mb)            # 640 KB: M <= 64 at hidden 5120
    assert not eligible(128 * 5120, torch.bfloat16, True, 256, mb)       # too large: NCCL
    assert not eligible(16 * 5120, torch.float32, True, 256, mb)         # dtype
    assert not eligible(16 * 5120, torch.bfloat16, False, 256, mb)       # strided
    assert not eligible(12, torch.bfloat16, True, 256, mb)               # count % 8
    assert not eligible(16, torch.bfloat16, True, 8, mb)                 # 16-byte alignment
    assert not eligible(0, torch.bfloat16, True, 256, mb)
