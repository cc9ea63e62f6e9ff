"""thq4_linear_noalloc -- thq4_linear without a caller workspace -- against
thq4_linear on the same weight and activation, through the C ABI, two
consecutive calls each.  The file is collected last so that it runs after
every other test has used the library on the device; it passes alone too."""
import ctypes

import numpy as np
import pytest
import torch

import q4oracle as O
import thq4
from helpers import assert_close_ref, dev

pytestmark = pytest.mark.gpu

P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("out,inp,m", [(6144, 2048, 1), (1000, 1088, 1), (2560, 9728, 4), (520, 448, 8)])
def test_noalloc_matches_workspace_entry(out, inp, m):
    wq, sb = O.rand_qlin(out, inp, out + m)
    q = thq4.QLin(dev(wq), dev(sb), out, inp, 64).tiled()
    x = dev(np.stack([O.rand_x(inp, 40 + t) for t in range(m)]))
    L = thq4.lib()
    desc = ctypes.byref(q.packed.desc)
    ws = thq4.qlin.workspace(q.packed.desc, x.device)
    want = torch.empty((m, out), dtype=torch.float32, device="cuda")
    thq4.check(L.thq4_linear(desc, P(x), thq4.BF16, m, P(want), thq4.F32, P(ws), ws.numel(), _stream()))
    want_h = want.cpu().numpy()
    for call in range(2):
        got = torch.full((m, out), float("nan"), dtype=torch.float32, device="cuda")
        thq4.check(L.thq4_linear_noalloc(desc, P(x), thq4.BF16, m, P(got), thq4.F32, _stream()))
        got_h = got.cpu().numpy()
        for t in range(m):
            assert_close_ref(f"noalloc call {call} token {t} {out}x{inp}", got_h[t], want_h[t])


def test_noalloc_rejects_weights_above_its_scratch():
    x = torch.zeros((1, 64), dtype=torch.bfloat16, device="cuda")
    y = torch.zeros((1, 8), dtype=torch.bfloat16, device="cuda")
    w = thq4._lib.thq4_weight()
    # a descriptor is only checked, never launched: 8 million rows exceed the buffer
    w.out, w.in_, w.gs, w.sb_dtype = 8_000_000, 64, 64, thq4.BF16
    w.qw = w.sb = ctypes.c_void_p(x.data_ptr())
    st = thq4.lib().thq4_linear_noalloc(ctypes.byref(w), P(x), thq4.BF16, 1, P(y), thq4.BF16, _stream())
    assert st == thq4._lib.ERR_UNSUPPORTED
    assert "use thq4_linear" in thq4.last_error()
