"""Decode (m = 1) and verify (m <= 8) projections through the C ABI against
the CPU oracle.  Mirrors the reference's qmvt tests (engine/src/qwen35.rs:
6886-7049): the same LCG weights and activations, every split config, ragged
row counts, empty K slices, the gate/up epilogue with tile-aligned and
unaligned up streams, determinism and the misaligned-input rejection."""
import ctypes

import numpy as np
import pytest
import torch

import q4oracle as O
import thq4
from helpers import assert_close_ref, assert_rms_close, dev, dev_sb, host_bits, to_f32

pytestmark = pytest.mark.gpu

SPLITS = [(1, 8), (2, 8), (4, 8), (8, 8), (16, 16), (1, 4), (4, 16)]


@pytest.fixture(autouse=True)
def _reset_split():
    yield
    thq4.lib().thq4_debug_set_gemv(0, 0)


def _qlin(wq, sb, sb_dtype=O.SB_BF16):
    out, inp = wq.shape[0], wq.shape[1] * 8
    return thq4.QLin(dev(wq), dev_sb(sb, sb_dtype), out, inp, 64).tiled()


def _x_bf16(bits):
    return dev(bits)


@pytest.mark.parametrize("case", range(4))
def test_repack_matches_oracle_frag16(case):
    out, ng = O.QMVT_PLAIN_CASES[case]
    inp = ng * 64
    wq, sb = O.rand_qlin(out, inp, 11 + case)
    fq, fsb = O.mlx_to_frag16(wq, sb)
    q = _qlin(wq, sb)
    assert np.array_equal(host_bits(q.packed.qw).view(np.uint32), fq)
    assert np.array_equal(host_bits(q.packed.sb).view(np.uint16), fsb)
    # the reference's tiled layout and (out % 256 == 0) Splash slab give the same bytes
    tw, tsb = O.mlx_to_tiled(wq, sb)
    qt = thq4.QLin.from_layout(thq4.SRC_TILED, dev(tw), dev(tsb), out, inp, thq4.BF16)
    assert np.array_equal(host_bits(qt.packed.qw).view(np.uint32), fq)
    assert np.array_equal(host_bits(qt.packed.sb).view(np.uint16), fsb)
    if out % 256 == 0:
        slab = O.mlx_to_slab(wq, sb)
        qs = thq4.QLin.from_layout(thq4.SRC_SLAB, dev(slab), None, out, inp, thq4.BF16)
        assert np.array_equal(host_bits(qs.packed.qw).view(np.uint32), fq)
        assert np.array_equal(host_bits(qs.packed.sb).view(np.uint16), fsb)


def test_repack_row_range():
    wq, sb = O.rand_qlin(520, 448, 3)
    q = thq4.PackedWeight.repack(thq4.SRC_MLX, dev(wq), dev(sb), 520, 448, thq4.BF16, 136, 264)
    fq, fsb = O.mlx_to_frag16(wq[136:400], sb[136:400])
    assert np.array_equal(host_bits(q.qw).view(np.uint32), fq)
    assert np.array_equal(host_bits(q.sb).view(np.uint16), fsb)


@pytest.mark.parametrize("sb_dtype", [O.SB_BF16, O.SB_F16])
def test_dequant_matches_oracle(sb_dtype):
    wq, sb = O.synthetic_weight(200, 512, 7, sb_dtype)
    q = _qlin(wq, sb, sb_dtype)
    got = host_bits(q.dequant())
    want = O.dequant_bf16(wq, sb, sb_dtype)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("case", range(4))
def test_qmvt_plain_matches_oracle(case):
    out, ng = O.QMVT_PLAIN_CASES[case]
    inp = ng * 64
    wq, sb = O.rand_qlin(out, inp, 11 + case)
    xb = O.rand_x(inp, 97 + case)
    want = O.linear_group(wq, sb, O.SB_BF16, O.bf16_to_f32(xb))[0]
    q = _qlin(wq, sb)
    x = _x_bf16(xb)
    for ks, warps in SPLITS:
        thq4.check(thq4.lib().thq4_debug_set_gemv(ks, warps))
        y = q.linear(x.reshape(1, 1, inp))
        assert tuple(y.shape) == (1, 1, out)
        got = to_f32(y).ravel()
        assert_close_ref(f"plain {out}x{inp} ks{ks} w{warps}", got, want)
        again = to_f32(q.linear(x.reshape(1, 1, inp))).ravel()
        assert np.array_equal(got, again), "not deterministic"


@pytest.mark.parametrize("case", range(4))
def test_qmvt_gate_up_matches_oracle(case):
    half, ng = O.QMVT_GATE_UP_CASES[case]
    inp, out = ng * 64, 2 * half
    wq, sb = O.rand_qlin(out, inp, 211 + case)
    xb = O.rand_x(inp, 307 + case)
    want = O.bf16_to_f32(O.gate_up(wq, sb, O.SB_BF16, half, half, O.bf16_to_f32(xb)))[0]
    q = thq4.QLin(dev(wq), dev(sb), out, inp, 64)
    x = _x_bf16(xb)
    for ks, warps in SPLITS:
        thq4.check(thq4.lib().thq4_debug_set_gemv(ks, warps))
        y = q.gate_up_act(x.reshape(1, 1, inp))
        assert tuple(y.shape) == (1, 1, half)
        got = to_f32(y).ravel()
        assert_close_ref(f"gate_up {half}x{inp} ks{ks}", got, want)
        again = to_f32(q.gate_up_act(x.reshape(1, 1, inp))).ravel()
        assert np.array_equal(got, again)


@pytest.mark.parametrize("m", [2, 3, 4, 5, 8])
def test_verify_small_m_matches_oracle(m):
    out, inp = 1000, 17 * 64
    wq, sb = O.rand_qlin(out, inp, 5 + m)
    xs = np.stack([O.rand_x(inp, 400 + m * 10 + t) for t in range(m)])
    want = O.linear_group(wq, sb, O.SB_BF16, O.bf16_to_f32(xs))
    q = _qlin(wq, sb)
    y = q.linear(dev(xs))
    got = to_f32(y)
    for t in range(m):
        assert_close_ref(f"m={m} t={t}", got[t], want[t])
    # gate/up at the same m
    half = 264
    wq2, sb2 = O.rand_qlin(2 * half, inp, 77 + m)
    want2 = O.bf16_to_f32(O.gate_up(wq2, sb2, O.SB_BF16, half, half, O.bf16_to_f32(xs)))
    q2 = thq4.QLin(dev(wq2), dev(sb2), 2 * half, inp, 64)
    got2 = to_f32(q2.gate_up_act(dev(xs)))
    for t in range(m):
        assert_close_ref(f"gate_up m={m} t={t}", got2[t], want2[t])


def test_x_f32_y_f32():
    """The GEMV of the single-GEMV configuration: f32 in, f32 out."""
    out, inp = 600, 2048
    wq, sb = O.synthetic_weight(out, inp, 1, O.SB_F16)
    x = np.random.default_rng(2).standard_normal((3, inp)).astype(np.float32)
    want = O.linear_group(wq, sb, O.SB_F16, x)
    q = _qlin(wq, sb, O.SB_F16)
    y = q.linear(torch.from_numpy(x).cuda())
    assert y.dtype == torch.float32
    got = to_f32(y)
    # hi/lo split keeps ~16 bits of x: far inside one bf16 step
    rms = np.sqrt((want ** 2).mean())
    assert np.abs(got - want).max() <= 2e-4 * rms
    assert_rms_close("f32 vs reference CPU path", got, O.linear_dequant(wq, sb, O.SB_F16, x))


def test_rejects_misaligned_input():
    """qmvt_rejects_misaligned_input (qwen35.rs:7027-7049)."""
    out, inp = 256, 1024
    wq, sb = O.rand_qlin(out, inp, 5)
    q = _qlin(wq, sb)
    x = dev(O.rand_x(inp + 1, 6))[1:]
    y = torch.empty((1, out), dtype=torch.bfloat16, device="cuda")
    st = thq4.lib().thq4_linear(ctypes.byref(q.packed.desc), ctypes.c_void_p(x.data_ptr()), thq4.BF16, 1,
                                ctypes.c_void_p(y.data_ptr()), thq4.BF16, None, 0, None)
    assert st == thq4._lib.ERR_INVALID_ARGUMENT
    assert "16-byte aligned" in thq4.last_error()
    # through QLin the copy made by contiguous() is aligned again: same result as an aligned x
    xa = x.clone()
    want = O.linear_group(wq, sb, O.SB_BF16, O.bf16_to_f32(host_bits(xa)))[0]
    assert_close_ref("aligned copy", to_f32(q.linear(xa.reshape(1, inp))).ravel(), want)


def test_routing_m1_equals_direct_call():
    out, inp = 520, 448
    wq, sb = O.rand_qlin(out, inp, 11)
    q = _qlin(wq, sb)
    x = _x_bf16(O.rand_x(inp, 97))
    direct = torch.empty((1, out), dtype=torch.bfloat16, device="cuda")
    thq4.check(thq4.lib().thq4_linear(ctypes.byref(q.packed.desc), ctypes.c_void_p(x.data_ptr()), thq4.BF16, 1,
                                      ctypes.c_void_p(direct.data_ptr()), thq4.BF16, None, 0,
                                      ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    routed = q.linear(x.reshape(1, 1, inp))
    assert torch.equal(routed.reshape(-1), direct.reshape(-1))


@pytest.mark.parametrize("m", [1, 2, 4, 8])
def test_verify_config_shapes(m):
    """The spec-verify configuration: gate/up 2x9728x2560 and down
    2560x9728 at M in {1,2,4,8}, f16 scales, x ~ N(0,1) bf16."""
    rng = np.random.default_rng(100 + m)
    gu_wq, gu_sb = O.synthetic_weight(2 * 9728, 2560, 31, O.SB_F16)
    dn_wq, dn_sb = O.synthetic_weight(2560, 9728, 32, O.SB_F16)
    x = O.f32_to_bf16(rng.standard_normal((m, 2560)).astype(np.float32))
    gu = thq4.QLin(dev(gu_wq), dev_sb(gu_sb, O.SB_F16), 2 * 9728, 2560, 64)
    h = gu.gate_up_act(dev(x))
    want_h = O.bf16_to_f32(O.gate_up(gu_wq, gu_sb, O.SB_F16, 9728, 9728, O.bf16_to_f32(x)))
    got_h = to_f32(h)
    assert_rms_close("gate_up", got_h, want_h, 1e-2)
    for t in range(m):
        assert_close_ref(f"gate_up t{t}", got_h[t], want_h[t])
    dn = _qlin(dn_wq, dn_sb, O.SB_F16)
    y = to_f32(dn.linear(h))
    want_y = O.linear_group(dn_wq, dn_sb, O.SB_F16, got_h)
    for t in range(m):
        assert_close_ref(f"down t{t}", y[t], want_y[t])
    assert_rms_close("down vs reference CPU path", y, O.linear_dequant(dn_wq, dn_sb, O.SB_F16, got_h))
