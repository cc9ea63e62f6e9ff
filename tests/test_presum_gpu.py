"""Presum blocks on the device (the reference's K45 machinery,
engine/src/quant_kernel.rs:265-318, 3642-3657): the two producers
(Q4AttachSums and AddRmsNorm { sums }, gdn_kernel.rs:1851-1866, 1919-1962)
bit for bit against the oracle, and decode / verify projections reading a
block against the same projections on plain x."""
import ctypes

import numpy as np
import pytest
import torch

import q4oracle as O
import thq4
from helpers import assert_close_ref, assert_gate_up_close, assert_rms_close, dev, host_bits, to_f32

pytestmark = pytest.mark.gpu


def _bf(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda().view(torch.bfloat16)


def _split(block, inp):
    b = block.cpu().numpy()
    rows = b[:8 * inp * 2].view(np.uint16).reshape(8, inp)
    sums = b[8 * inp * 2:].view(np.float32).reshape(inp // 64, 8)
    return rows, sums


@pytest.mark.parametrize("m,inp", [(1, 5120), (3, 1024), (8, 2560), (8, 64)])
def test_presum_attach_bit_exact(m, inp):
    x = O.f32_to_bf16(np.random.default_rng(m + inp).standard_normal((m, inp)).astype(np.float32))
    block, view = thq4.presum_block(_bf(x))
    torch.cuda.synchronize()
    assert block.numel() == 8 * inp * 2 + inp // 64 * 32 == thq4.presum_block_bytes(inp)
    rows, sums = _split(block, inp)
    want_rows, want_sums = O.presum_block(x)
    assert np.array_equal(rows, want_rows)
    assert np.array_equal(sums, want_sums)
    assert np.array_equal(host_bits(view), x)


@pytest.mark.parametrize("T,C", [(1, 5120), (3, 1024), (8, 2048)])
def test_add_rms_norm_bit_exact(T, C):
    rng = np.random.default_rng(T * C)
    x = O.f32_to_bf16(rng.standard_normal((T, C)).astype(np.float32))
    r = O.f32_to_bf16(rng.standard_normal((T, C)).astype(np.float32))
    w = O.f32_to_bf16((1 + 0.1 * rng.standard_normal(C)).astype(np.float32))
    res, block, view = thq4.add_rms_norm(_bf(x), _bf(r), _bf(w), 1e-6)
    torch.cuda.synchronize()
    want_res, want_rows, want_sums = O.add_rms_norm(x, r, w, 1e-6)
    assert np.array_equal(host_bits(res), want_res)
    rows, sums = _split(block, C)
    assert np.array_equal(rows, want_rows), f"{(rows != want_rows).sum()} normed values differ"
    assert np.array_equal(sums, want_sums)
    assert view.shape == (T, C)


@pytest.mark.parametrize("m", [1, 4, 8])
def test_projection_on_a_presum_block(m):
    """thq4_linear / thq4_gate_up with x given as a presum block take each
    group's bias-term sum from the block; against the same call on plain x
    (one bf16 step, the per-element rule) and the oracle."""
    out, inp = 1000, 17 * 64
    wq, sb = O.rand_qlin(out, inp, 50 + m)
    q = thq4.QLin(dev(wq), dev(sb), out, inp, 64).tiled()
    xs = np.stack([O.rand_x(inp, 60 + t) for t in range(m)])
    block, view = thq4.presum_block(_bf(xs))
    got = to_f32(q.linear_ps(view, presum=True))
    plain = to_f32(q.linear_ps(_bf(xs)))
    want = O.linear_group(wq, sb, O.SB_BF16, O.bf16_to_f32(xs))
    for t in range(m):
        assert_close_ref(f"presum t{t}", got[t], want[t])
        assert_close_ref(f"presum vs plain t{t}", got[t], plain[t])
    got32 = to_f32(q.linear_ps(view, presum=True, out_dtype=torch.float32))
    assert_rms_close("presum f32", got32, want)
    half = 264
    wq2, sb2 = O.rand_qlin(2 * half, inp, 70 + m)
    g2 = thq4.QLin(dev(wq2), dev(sb2), 2 * half, inp, 64)
    h = to_f32(g2.gate_up_act_ps(view, presum=True)[0])
    gu = O.linear_group(wq2, sb2, O.SB_BF16, O.bf16_to_f32(xs))
    for t in range(m):
        assert_gate_up_close(f"presum gate_up t{t}", h[t], gu[t, :half], gu[t, half:], inp)


def test_presum_validation():
    inp = 1024
    wq, sb = O.rand_qlin(256, inp, 5)
    q = thq4.QLin(dev(wq), dev(sb), 256, inp, 64).tiled()
    x = torch.zeros((2, inp), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(thq4.Thq4Error, match="presum block missing"):
        q.linear_ps(x, presum=True)  # a plain tensor: no sums behind its rows
    L = thq4.lib()
    y = torch.empty((9, 256), dtype=torch.bfloat16, device="cuda")
    block = torch.zeros(thq4.presum_block_bytes(inp) + 64, dtype=torch.uint8, device="cuda")
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    ws = thq4.qlin.workspace(q.packed.desc, x.device)
    st = L.thq4_linear(ctypes.byref(q.packed.desc), P(block), thq4._lib.PRESUM, 9, P(y), thq4.BF16, P(ws),
                       ws.numel(), None)
    assert st == thq4._lib.ERR_INVALID_ARGUMENT and "at most 8 rows" in thq4.last_error()
    st = L.thq4_linear(ctypes.byref(q.packed.desc), ctypes.c_void_p(block.data_ptr() + 8), thq4._lib.PRESUM, 1,
                       P(y), thq4.BF16, P(ws), ws.numel(), None)
    assert st == thq4._lib.ERR_INVALID_ARGUMENT and "16-byte" in thq4.last_error()
    assert L.thq4_presum_attach(P(x), 9, inp, P(block), None) == thq4._lib.ERR_INVALID_ARGUMENT
    assert L.thq4_add_rms_norm(P(x), P(x), P(x), 2, 100, ctypes.c_float(1e-6), P(x), P(block), None) == \
        thq4._lib.ERR_INVALID_ARGUMENT
    assert L.thq4_presum_block_bytes(100) == 0
