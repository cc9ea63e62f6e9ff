"""Host-side mirror of QLin without a GPU: shape checks fail with the
reference's messages before any device work (qwen35.rs:405-411,
6854-6884), and the benchmark's torch quantiser equals the oracle's."""
import numpy as np
import pytest
import torch

import q4oracle as O
import thq4
from thq4 import synth


def test_qlin_linear_rejects_in_dim_mismatch():
    """qlin_linear_rejects_in_dim_mismatch (qwen35.rs:6860-6876)."""
    out, inp = 64, 4096
    q = thq4.QLin(torch.zeros((out, inp // 8), dtype=torch.int32), torch.zeros((out, 2 * inp // 64),
                  dtype=torch.bfloat16), out, inp, 64)
    bad = torch.zeros((1, 8, 32, 128), dtype=torch.bfloat16)
    with pytest.raises(thq4.Thq4Error) as e:
        q.linear(bad)
    assert "x last dim 128 != weight inp 4096" in str(e.value)


def test_qlin_rejects_bad_scale_dtype():
    with pytest.raises(thq4.Thq4Error):
        thq4.QLin(torch.zeros((16, 8), dtype=torch.int32), torch.zeros((16, 2), dtype=torch.float32), 16, 64, 64)


@pytest.mark.parametrize("dt,sbd", [(torch.float16, O.SB_F16), (torch.bfloat16, O.SB_BF16)])
def test_torch_quantiser_equals_oracle(dt, sbd):
    w = torch.randn(300, 512, generator=torch.Generator().manual_seed(3)) * 0.02
    a, b = synth.quantize(w, dt)
    wq, sb = O.quantize(w.numpy(), sbd)
    assert np.array_equal(a.numpy().view(np.uint32), wq)
    assert np.array_equal(b.view(torch.int16).numpy().view(np.uint16), sb)
