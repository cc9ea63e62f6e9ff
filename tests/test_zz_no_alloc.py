"""thq4_linear_noalloc -- thq4_linear without a caller workspace -- against
thq4_linear on the same weight and activation, through the C ABI, two
consecutive calls each.

It exists for callers that cannot allocate device memory where they run a
projection (a host binding that only receives tensors and has no device
allocator of its own, or a serving loop whose memory is fixed before the
first request), so it takes its scratch from one fixed buffer inside the
library.  The file is collected last so that it runs after every other test
has used the library on the device; it passes alone too."""
import ctypes

import numpy as np
import pytest
import torch

import q4oracle as O
import thq4
from helpers import assert_close_ref, assert_rms_close, dev

pytestmark = pytest.mark.gpu

P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
SCRATCH = 6 << 20  # the built-in buffer's bytes


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _both(desc, x, x_dtype, m, out):
    """thq4_linear (own workspace) once, then thq4_linear_noalloc twice."""
    L = thq4.lib()
    ws = thq4.qlin.workspace(desc, x.device)
    want = torch.empty((m, out), dtype=torch.float32, device="cuda")
    thq4.check(L.thq4_linear(ctypes.byref(desc), P(x), x_dtype, m, P(want), thq4.F32, P(ws), ws.numel(), _stream()))
    got = []
    for _ in range(2):
        y = torch.full((m, out), float("nan"), dtype=torch.float32, device="cuda")
        thq4.check(L.thq4_linear_noalloc(ctypes.byref(desc), P(x), x_dtype, m, P(y), thq4.F32, _stream()))
        got.append(y.cpu().numpy())
    return want.cpu().numpy(), got


@pytest.mark.parametrize("out,inp,m", [(6144, 2048, 1), (1000, 1088, 1), (2560, 9728, 4), (520, 448, 8),
                                       (1000, 1088, 16), (2048, 1024, 512)])
def test_noalloc_matches_workspace_entry(out, inp, m):
    """m <= 8 runs the decode/verify kernel on the built-in scratch; m > 8
    (bf16 x) runs the prefill kernel, as thq4_linear does."""
    wq, sb = O.rand_qlin(out, inp, out + m)
    q = thq4.QLin(dev(wq), dev(sb), out, inp, 64).tiled()
    x = dev(np.stack([O.rand_x(inp, 40 + t) for t in range(m)]))
    want, got = _both(q.packed.desc, x, thq4.BF16, m, out)
    for call, g in enumerate(got):
        assert np.array_equal(g, want), f"noalloc call {call}: differs from thq4_linear"
    xf = O.bf16_to_f32(x.view(torch.int16).cpu().numpy().view(np.uint16))
    if m <= 8:  # the decode/verify kernel: per-group arithmetic
        ref = O.linear_group(wq, sb, O.SB_BF16, xf)
        for t in range(m):
            assert_close_ref(f"noalloc token {t} {out}x{inp}", got[1][t], ref[t])
    else:  # the prefill kernel: bf16-dequantised weights, f32 accumulate
        assert_rms_close(f"noalloc prefill {m}x{out}x{inp}", got[1], O.linear_dequant(wq, sb, O.SB_BF16, xf))


def test_noalloc_f32_activation():
    """f32 x: the decode/verify kernel for any m (passes of 4 tokens)."""
    out, inp, m = 600, 2048, 9
    wq, sb = O.synthetic_weight(out, inp, 1, O.SB_F16)
    q = thq4.QLin(dev(wq), torch.from_numpy(sb.view(np.int16)).cuda().view(torch.float16), out, inp, 64).tiled()
    xh = np.random.default_rng(2).standard_normal((m, inp)).astype(np.float32)
    want, got = _both(q.packed.desc, torch.from_numpy(xh).cuda(), thq4.F32, m, out)
    for g in got:
        assert np.array_equal(g, want)
    assert_rms_close("noalloc f32 x", got[1], O.linear_group(wq, sb, O.SB_F16, xh))


def _limit_rows():
    """The largest row count whose decode/verify scratch fits the buffer
    (it depends on the SM count)."""
    L = thq4.lib()
    w = thq4._lib.thq4_weight()
    w.in_, w.gs, w.sb_dtype = 64, 64, thq4.BF16
    lo, hi = 128, 1 << 24
    while hi - lo > 128:  # scratch grows by whole 128-row slabs
        mid = (lo + hi) // 2 // 128 * 128
        w.out = mid
        if L.thq4_linear_workspace_bytes(ctypes.byref(w), 1) <= SCRATCH:
            lo = mid
        else:
            hi = mid
    return lo


def test_noalloc_size_limit():
    """A weight just under the buffer's limit runs and matches thq4_linear; one
    slab more is rejected before anything is launched.  Both weights are real
    device buffers of their full size, so even a launch would stay in bounds."""
    rows = _limit_rows()
    assert 1_000_000 < rows < 20_000_000
    L = thq4.lib()
    for r, ok in ((rows, True), (rows + 128, False)):
        qb, sbb = ctypes.c_size_t(), ctypes.c_size_t()
        L.thq4_weight_bytes(r, 64, 64, ctypes.byref(qb), ctypes.byref(sbb))
        g = torch.Generator(device="cuda")
        g.manual_seed(r)
        qw = torch.randint(0, 256, (qb.value,), dtype=torch.uint8, device="cuda", generator=g)
        sb = (torch.rand((sbb.value // 2,), device="cuda", generator=g) * 0.01).to(torch.bfloat16)
        w = thq4._lib.thq4_weight()
        thq4.check(L.thq4_weight_init(ctypes.byref(w), r, 64, 64, thq4.BF16, P(qw), P(sb)))
        x = torch.randn((1, 64), device="cuda").to(torch.bfloat16)
        if ok:
            want, got = _both(w, x, thq4.BF16, 1, r)
            for gt in got:
                assert np.array_equal(gt, want)
        else:
            y = torch.zeros((1, r), dtype=torch.float32, device="cuda")
            st = L.thq4_linear_noalloc(ctypes.byref(w), P(x), thq4.BF16, 1, P(y), thq4.F32, _stream())
            assert st == thq4._lib.ERR_UNSUPPORTED
            assert "use thq4_linear" in thq4.last_error()
        del qw, sb
        torch.cuda.empty_cache()
