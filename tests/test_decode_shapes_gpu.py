"""The headline shapes at full size through the C ABI against the CPU oracle.

BASELINE configs[3] (the decode layer of hidden 5120 the bench streams): the
fused q/k/v projection 7168 x 5120, o 5120 x 5120, the fused gate/up 2 x
17408 x 5120 with its SwiGLU epilogue, and down 5120 x 17408; and
configs[0], the single 6144 x 2048 GEMV with f32 x and f32 y.  Each call is
the one the bench makes (thq4_linear / thq4_gate_up with the default launch
policy: clusters of CTAs splitting each slab for q/k/v, o and down, one whole
slab per CTA for gate/up), on weights made by the bench's quantiser and seeds.

Bars: the north star, max|err| <= 1e-2 * RMS(y_ref) on f32 outputs, against
both the reference CPU path (every weight dequantised to bf16, f32
accumulate; qwen35.rs:110-134, 616) and the oracle's per-group arithmetic
(quant_kernel.rs:1994-2001); bf16 outputs against the reference qmvt tests'
per-element rule (qwen35.rs:6946-6961) and the gate/up split tolerance
(LinearNumerics.hpp:112-126)."""
import ctypes

import numpy as np
import pytest
import torch

import q4oracle as O
import thq4
from helpers import assert_close_ref, assert_gate_up_close, assert_rms_close, to_f32
from thq4 import synth

pytestmark = pytest.mark.gpu

P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _weight(out, inp, seed):
    """Quantised N(0, 0.02) weight (f16 scale/bias) made on the GPU as the
    bench makes it; returns the packed weight and the MLX arrays on the host."""
    wq, sb = synth.normal_weight(out, inp, seed, torch.device("cuda"))
    p = thq4.PackedWeight.repack(thq4.SRC_MLX, wq, sb, out, inp, thq4.F16)
    host = (wq.cpu().numpy().view(np.uint32), sb.cpu().view(torch.int16).numpy().view(np.uint16))
    return p, host


def _linear(p, x, x_dtype, y_dtype):
    m = x.shape[0]
    y = torch.full((m, p.desc.out), float("nan"), dtype=torch.float32 if y_dtype == thq4.F32 else torch.bfloat16,
                   device="cuda")
    ws = thq4.qlin.workspace(p.desc, x.device)
    thq4.check(thq4.lib().thq4_linear(ctypes.byref(p.desc), P(x), x_dtype, m, P(y), y_dtype, P(ws), ws.numel(),
                                      _stream()))
    return y


# (name, out, in, seed) -- the seeds of the bench's first layer
C4 = [("qkv", 7168, 5120, 1001), ("o", 5120, 5120, 1004), ("down", 5120, 17408, 1007)]


@pytest.mark.parametrize("name,out,inp,seed", C4, ids=[c[0] for c in C4])
def test_decode_layer_projection_full_size(name, out, inp, seed):
    p, (wq, sb) = _weight(out, inp, seed)
    rng = np.random.default_rng(seed)
    xb = O.f32_to_bf16(rng.standard_normal((1, inp)).astype(np.float32))
    xf = O.bf16_to_f32(xb)
    x = torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16)
    y32 = to_f32(_linear(p, x, thq4.BF16, thq4.F32))[0]
    y16 = to_f32(_linear(p, x, thq4.BF16, thq4.BF16))[0]
    want_group = O.linear_group(wq, sb, O.SB_F16, xf)[0]
    want_cpu = O.linear_dequant(wq, sb, O.SB_F16, xf)[0]
    assert np.all(np.isfinite(y32)) and np.all(np.isfinite(y16))
    assert_rms_close(f"{name} f32 vs reference CPU path", y32, want_cpu)
    assert_rms_close(f"{name} f32 vs oracle", y32, want_group)
    assert_close_ref(f"{name} bf16 vs oracle", y16, want_group)


def test_decode_layer_gate_up_full_size():
    """The fused gate/up of the intermediate-17408 MLP (2 x 17408 x 5120)."""
    inp, half = 5120, 17408
    gate, (gq, gs) = _weight(half, inp, 1005)
    up, (uq, us) = _weight(half, inp, 1006)
    rng = np.random.default_rng(1005)
    xb = O.f32_to_bf16(rng.standard_normal((1, inp)).astype(np.float32))
    xf = O.bf16_to_f32(xb)
    x = torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16)
    h = torch.full((1, half), float("nan"), dtype=torch.bfloat16, device="cuda")
    ws = thq4.qlin.workspace(gate.desc, x.device)
    thq4.check(thq4.lib().thq4_gate_up(ctypes.byref(gate.desc), ctypes.byref(up.desc), P(x), thq4.BF16, 1, P(h),
                                       thq4.BF16, P(ws), ws.numel(), _stream()))
    g = O.linear_group(gq, gs, O.SB_F16, xf)[0]
    u = O.linear_group(uq, us, O.SB_F16, xf)[0]
    assert_gate_up_close("gate_up 2x17408x5120", to_f32(h)[0], g, u, inp)
    # the two halves alone, f32 out, at the north-star bar
    for name, p, q, s in (("gate", gate, gq, gs), ("up", up, uq, us)):
        got = to_f32(_linear(p, x, thq4.BF16, thq4.F32))[0]
        assert_rms_close(f"{name} f32 vs reference CPU path", got, O.linear_dequant(q, s, O.SB_F16, xf)[0])


def test_single_gemv_config_full_size():
    """x [1 x 2048] f32 ~ N(0, 1), W [6144 x 2048] ~ N(0, 0.02)
    with f16 scale/bias, y f32."""
    out, inp = 6144, 2048
    p, (wq, sb) = _weight(out, inp, 6144)
    x = np.random.default_rng(2048).standard_normal((1, inp)).astype(np.float32)
    got = to_f32(_linear(p, torch.from_numpy(x).cuda(), thq4.F32, thq4.F32))[0]
    want = O.linear_group(wq, sb, O.SB_F16, x)[0]
    rms = float(np.sqrt((want.astype(np.float64) ** 2).mean()))
    # the f32 activation is split into fp16 hi + lo parts (22 significant bits)
    assert np.abs(got - want).max() <= 2e-4 * rms
    assert_rms_close("C1 f32 vs reference CPU path", got, O.linear_dequant(wq, sb, O.SB_F16, x)[0])
