"""Host-side logic of the custom all-reduce: which tensors take the one-shot
path, and that the choice depends only on values every rank shares."""
import torch

from w4a8_b200.allreduce import DEFAULT_MAX_BYTES, direct, eligible


def test_eligibility():
    mb = DEFAULT_MAX_BYTES
    assert eligible(16 * 5120, torch.bfloat16, mb)
    assert eligible(64 * 5120, torch.bfloat16, mb)            # 640 KB: M <= 64 at hidden 5120
    assert not eligible(128 * 5120, torch.bfloat16, mb)       # too large: NCCL
    assert not eligible(16 * 5120, torch.float32, mb)         # dtype
    assert not eligible(12, torch.bfloat16, mb)               # count % 8
    assert not eligible(0, torch.bfloat16, mb)


def test_layout_never_decides_the_path():
    """Two ranks holding the same message as differently laid-out tensors
    (a strided view on one, a dense tensor on the other; an address off the
    16-byte grid on one) must both choose the one-shot path: the layout only
    selects the in-place or the staged form of it."""
    mb = DEFAULT_MAX_BYTES
    dense = torch.zeros(16, 5120, dtype=torch.bfloat16)
    strided = torch.zeros(16, 10240, dtype=torch.bfloat16)[:, ::2]
    offset = torch.zeros(16 * 5120 + 1, dtype=torch.bfloat16)[1:]
    for t in (dense, strided, offset):
        assert eligible(t.numel(), t.dtype, mb)
    assert direct(dense)
    assert not direct(strided)
    assert not direct(offset)
