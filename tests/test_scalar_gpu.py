"""thq4_linear_scalar -- the scalar GPU reference product (the reference's
AffineQmv / AffineQmm, engine/src/quant_kernel.rs:1026-1147, 1634-1740) --
against the CPU oracle, and the tuned decode/verify kernel against it on the
device, as the reference's qmvt tests check every tile config against
scalar_ref (engine/src/qwen35.rs:6928-6989)."""
import ctypes

import numpy as np
import pytest
import torch

import q4oracle as O
import thq4
from helpers import assert_close_ref, assert_rms_close, dev, dev_sb, to_f32

pytestmark = pytest.mark.gpu

P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
SPLITS = [(0, 0, 0), (4, 2, 0), (8, 3, 0), (4, 3, 7), (4, 6, 0), (8, 2, 3), (4, 4, 1), (4, 3, 296)]


@pytest.fixture(autouse=True)
def _reset_split():
    yield
    thq4.lib().thq4_debug_set_gemv(0, 0, 0, 0)


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _scalar(desc, x, x_dtype, m, out, y_dtype=thq4.F32):
    y = torch.full((m, out), float("nan"), dtype=torch.float32 if y_dtype == thq4.F32 else torch.bfloat16,
                   device="cuda")
    thq4.check(thq4.lib().thq4_linear_scalar(ctypes.byref(desc), P(x), x_dtype, m, P(y), y_dtype, _stream()))
    return to_f32(y)


@pytest.mark.parametrize("case", range(4))
def test_scalar_matches_oracle(case):
    """f32 dequant + f32 accumulate against the oracle's f64 per-group form:
    the two differ only by f32 rounding (far below 1e-4 of the RMS)."""
    out, ng = O.QMVT_PLAIN_CASES[case]
    inp = ng * 64
    wq, sb = O.rand_qlin(out, inp, 11 + case)
    xb = O.rand_x(inp, 97 + case)
    q = thq4.QLin(dev(wq), dev(sb), out, inp, 64).tiled()
    got = _scalar(q.packed.desc, dev(xb), thq4.BF16, 1, out)
    want = O.linear_group(wq, sb, O.SB_BF16, O.bf16_to_f32(xb)[None, :])
    assert_rms_close(f"scalar {out}x{inp}", got, want, rel=1e-4)
    again = _scalar(q.packed.desc, dev(xb), thq4.BF16, 1, out)
    assert np.array_equal(got, again), "scalar kernel is not deterministic"


@pytest.mark.parametrize("m", [1, 3, 8, 11])
def test_scalar_tokens_and_f32(m):
    """Several tokens (passes of 8 beyond 8), bf16 and f32 x, f16 scales."""
    out, inp = 300, 1024
    wq, sb = O.synthetic_weight(out, inp, 5, O.SB_F16)
    q = thq4.QLin(dev(wq), dev_sb(sb, O.SB_F16), out, inp, 64).tiled()
    xh = np.random.default_rng(m).standard_normal((m, inp)).astype(np.float32)
    want = O.linear_group(wq, sb, O.SB_F16, xh)
    got = _scalar(q.packed.desc, torch.from_numpy(xh).cuda(), thq4.F32, m, out)
    assert_rms_close(f"scalar f32 x m={m}", got, want, rel=1e-4)
    xb = O.f32_to_bf16(xh)
    want_b = O.linear_group(wq, sb, O.SB_F16, O.bf16_to_f32(xb))
    got_b = _scalar(q.packed.desc, dev(xb), thq4.BF16, m, out, thq4.BF16)
    for t in range(m):
        assert_close_ref(f"scalar bf16 y m={m} t={t}", got_b[t], want_b[t])


@pytest.mark.parametrize("case", range(4))
def test_gemv_every_split_matches_scalar(case):
    """The reference's qmvt_plain_matches_scalar (qwen35.rs:6963-6989): every
    launch shape of the tuned kernel against the scalar kernel on the same
    GPU, bf16 outputs within one bf16 rounding step (qwen35.rs:6946-6961)."""
    out, ng = O.QMVT_PLAIN_CASES[case]
    inp = ng * 64
    wq, sb = O.rand_qlin(out, inp, 11 + case)
    xb = dev(O.rand_x(inp, 97 + case))
    q = thq4.QLin(dev(wq), dev(sb), out, inp, 64).tiled()
    want = _scalar(q.packed.desc, xb, thq4.BF16, 1, out, thq4.BF16)[0]
    L = thq4.lib()
    for split in SPLITS:
        thq4.check(L.thq4_debug_set_gemv(*split, 0))
        got = to_f32(q.linear(xb.reshape(1, inp))).ravel()
        assert_close_ref(f"gemv {out}x{inp} split {split} vs scalar", got, want)


def test_scalar_rejects_bad_arguments():
    L = thq4.lib()
    wq, sb = O.rand_qlin(64, 128, 1)
    q = thq4.QLin(dev(wq), dev(sb), 64, 128, 64).tiled()
    x = torch.zeros((1, 128), dtype=torch.bfloat16, device="cuda")
    y = torch.zeros((1, 64), dtype=torch.float32, device="cuda")
    assert L.thq4_linear_scalar(ctypes.byref(q.packed.desc), P(x), thq4.BF16, 0, P(y), thq4.F32,
                                _stream()) == thq4._lib.ERR_INVALID_ARGUMENT
    bad = ctypes.c_void_p(x.data_ptr() + 2)  # not 16-byte aligned
    assert L.thq4_linear_scalar(ctypes.byref(q.packed.desc), bad, thq4.BF16, 1, P(y), thq4.F32,
                                _stream()) == thq4._lib.ERR_INVALID_ARGUMENT
