"""thq4_linear_chain -- dependent projections in one persistent launch --
through the C ABI against the CPU oracle and against the same projections
run as separate thq4_linear / thq4_gate_up calls.

Each op must give what its single call gives (the reference qmvt tests'
per-element rule, qwen35.rs:6946-6961, and the gate/up split tolerance,
LinearNumerics.hpp:112-126, against the oracle on the op's own inputs), an
op must see every earlier op's output (not only its predecessor's), and the
chain must leave its workspace zeroed for the next call."""
import ctypes

import numpy as np
import pytest
import torch

import q4oracle as O
import thq4
from helpers import assert_close_ref, assert_gate_up_close, assert_rms_close, host_bits, to_f32
from thq4 import synth

pytestmark = pytest.mark.gpu


def _w(out, inp, seed):
    wq, sb = synth.normal_weight(out, inp, seed, torch.device("cuda"))
    p = thq4.PackedWeight.repack(thq4.SRC_MLX, wq, sb, out, inp, thq4.F16)
    return p, (wq.cpu().numpy().view(np.uint32), sb.cpu().view(torch.int16).numpy().view(np.uint16))


def _bf(t):
    return O.bf16_to_f32(host_bits(t))


def _empty(m, n, dtype=torch.bfloat16):
    return torch.full((m, n), float("nan"), dtype=dtype, device="cuda")


@pytest.mark.parametrize("m", [1, 3, 8])
def test_chain_of_two_layers_matches_oracle(m):
    """Per layer: q/k/v and q (both from the layer input), o from q, gate/up
    from o, down from the gate/up output; the second layer's input is the
    first layer's down output, so its q reads an output two ops back.  The
    last down writes f32."""
    H, KV, I = 1024, 256, 2816
    torch.manual_seed(m)
    x = torch.randn((m, H), device="cuda").to(torch.bfloat16)
    ops, checks, src = [], [], x
    for l in range(2):
        qkv, qkv_h = _w(H + 2 * KV, H, 10 * l + 1)
        q, q_h = _w(H, H, 10 * l + 6)
        o, o_h = _w(H, H, 10 * l + 2)
        g, g_h = _w(I, H, 10 * l + 3)
        u, u_h = _w(I, H, 10 * l + 4)
        d, d_h = _w(H, I, 10 * l + 5)
        t_qkv, t_q, t_o, t_h = _empty(m, H + 2 * KV), _empty(m, H), _empty(m, H), _empty(m, I)
        t_d = _empty(m, H, torch.float32 if l == 1 else torch.bfloat16)
        ops += [(qkv, None, src, t_qkv), (q, None, src, t_q), (o, None, t_q, t_o), (g, u, t_o, t_h), (d, None, t_h, t_d)]
        checks += [("qkv", qkv_h, None, src, t_qkv), ("q", q_h, None, src, t_q), ("o", o_h, None, t_q, t_o),
                   ("gate_up", g_h, u_h, t_o, t_h), ("down", d_h, None, t_h, t_d)]
        src = t_d
    chain = thq4.LinearChain(ops, m=m)
    chain()
    torch.cuda.synchronize()
    for i, (name, wh, uh, xin, yout) in enumerate(checks):
        xf = _bf(xin)
        if uh is not None:
            gg = O.linear_group(*wh, O.SB_F16, xf)
            uu = O.linear_group(*uh, O.SB_F16, xf)
            got = _bf(yout)
            for t in range(m):
                assert_gate_up_close(f"op {i} {name} t{t}", got[t], gg[t], uu[t], xf.shape[1])
            continue
        want = O.linear_group(*wh, O.SB_F16, xf)
        got = to_f32(yout) if yout.dtype == torch.float32 else _bf(yout)
        assert np.all(np.isfinite(got)), f"op {i} {name}: not every output was written"
        for t in range(m):
            assert_close_ref(f"op {i} {name} t{t}", got[t], want[t])
        if yout.dtype == torch.float32:
            assert_rms_close(f"op {i} {name} f32", got, want, 1e-4)
    # the arrival counters and the barrier words at the end of the workspace
    # are back at zero (the split-K partials before them may hold anything),
    # and a second call gives the same bits
    rows = max(op[0].desc.out for op in ops)
    counters = ((rows + 127) // 128 * 8 * 4 + 255) // 256 * 256 + 256
    assert int(chain.ws[-counters:].count_nonzero()) == 0, "the chain must leave its counters at zero"
    before = [host_bits(c[4]).copy() for c in checks]
    chain()
    torch.cuda.synchronize()
    assert all(np.array_equal(a, host_bits(c[4])) for a, c in zip(before, checks)), "not deterministic"
    st = ctypes.c_uint32()
    thq4.check(thq4.lib().thq4_device_status(ctypes.byref(st), None))
    assert st.value == 0


def test_chain_matches_separate_calls_on_the_bench_layer():
    """The bench's layer (hidden 5120, intermediate 17408) as a 4-op chain
    against the same four projections as separate calls on the chain's own
    inputs: within the per-element rule (their summation orders differ).
    The gate/up op's bf16(silu(bf16 g) * bf16 u) is held, in both forms, to
    the reference's split tolerance around the oracle's g and u: a bf16
    step of g can move a strongly negative g's output by several steps."""
    H, KV, I = 5120, 1024, 17408
    qkv, _ = _w(H + 2 * KV, H, 1001)
    o, _ = _w(H, H, 1004)
    g, (gq, gsb) = _w(I, H, 1005)
    u, (uq, usb) = _w(I, H, 1006)
    d, _ = _w(H, I, 1007)
    x = torch.randn((1, H), device="cuda").to(torch.bfloat16)
    outs = [_empty(1, n) for n in (H + 2 * KV, H, I, H)]
    chain = thq4.LinearChain([(qkv, None, x, outs[0]), (o, None, outs[0], outs[1]), (g, u, outs[1], outs[2]),
                              (d, None, outs[2], outs[3])])
    chain()
    torch.cuda.synchronize()
    L = thq4.lib()
    ws = torch.zeros(max(L.thq4_linear_workspace_bytes(ctypes.byref(p.desc), 1) for p in (qkv, o, g, d)),
                     dtype=torch.uint8, device="cuda")
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    ref = [torch.empty_like(t) for t in outs]
    thq4.check(L.thq4_linear(ctypes.byref(qkv.desc), P(x), thq4.BF16, 1, P(ref[0]), thq4.BF16, P(ws), ws.numel(), s))
    thq4.check(L.thq4_linear(ctypes.byref(o.desc), P(outs[0]), thq4.BF16, 1, P(ref[1]), thq4.BF16, P(ws), ws.numel(),
                             s))
    thq4.check(L.thq4_gate_up(ctypes.byref(g.desc), ctypes.byref(u.desc), P(outs[1]), thq4.BF16, 1, P(ref[2]),
                              thq4.BF16, P(ws), ws.numel(), s))
    thq4.check(L.thq4_linear(ctypes.byref(d.desc), P(outs[2]), thq4.BF16, 1, P(ref[3]), thq4.BF16, P(ws), ws.numel(),
                             s))
    torch.cuda.synchronize()
    for i, name in enumerate(("qkv", "o", "gate_up", "down")):
        if name == "gate_up":
            xo = _bf(outs[1])
            gate = O.linear_group(gq, gsb, O.SB_F16, xo)[0]
            up = O.linear_group(uq, usb, O.SB_F16, xo)[0]
            assert_gate_up_close("gate_up chain", _bf(outs[2])[0], gate, up, H)
            assert_gate_up_close("gate_up call", _bf(ref[2])[0], gate, up, H)
        else:
            assert_close_ref(f"{name} chain vs call", _bf(outs[i])[0], _bf(ref[i])[0])


def test_chain_validation():
    L = thq4.lib()
    p, _ = _w(256, 512, 3)
    x = torch.zeros((1, 512), dtype=torch.bfloat16, device="cuda")
    y = torch.zeros((1, 256), dtype=torch.bfloat16, device="cuda")
    arr = (thq4._lib.thq4_chain_op * 2)()
    arr[0].w, arr[0].x, arr[0].y, arr[0].y_dtype = ctypes.addressof(p.desc), x.data_ptr(), y.data_ptr(), thq4.BF16
    need = L.thq4_linear_chain_workspace_bytes(arr, 1)
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert L.thq4_linear_chain(arr, 0, thq4.BF16, 1, P(ws), need, s) == thq4._lib.ERR_INVALID_ARGUMENT
    assert L.thq4_linear_chain(arr, 113, thq4.BF16, 1, P(ws), need, s) == thq4._lib.ERR_INVALID_ARGUMENT
    assert L.thq4_linear_chain(arr, 1, thq4.BF16, 9, P(ws), need, s) == thq4._lib.ERR_UNSUPPORTED
    assert L.thq4_linear_chain(arr, 1, thq4.F32, 5, P(ws), need, s) == thq4._lib.ERR_UNSUPPORTED
    assert L.thq4_linear_chain(arr, 1, thq4.BF16, 1, P(ws), need - 1, s) == thq4._lib.ERR_WORKSPACE
    arr[0].y = x.data_ptr()
    assert L.thq4_linear_chain(arr, 1, thq4.BF16, 1, P(ws), need, s) == thq4._lib.ERR_INVALID_ARGUMENT
    assert "aliases" in thq4.last_error()
    arr[0].y, arr[0].reserved = y.data_ptr(), 1
    assert L.thq4_linear_chain(arr, 1, thq4.BF16, 1, P(ws), need, s) == thq4._lib.ERR_INVALID_ARGUMENT
    arr[0].reserved = 0
    q2 = thq4.PackedWeight(256, 512, thq4.BF16, torch.device("cuda"))  # a bf16-scaled op after an f16 one
    arr[1].w, arr[1].x, arr[1].y, arr[1].y_dtype = ctypes.addressof(q2.desc), x.data_ptr(), y.data_ptr(), thq4.BF16
    assert L.thq4_linear_chain(arr, 2, thq4.BF16, 1, P(ws), need, s) == thq4._lib.ERR_INVALID_ARGUMENT
    assert "scale dtype" in thq4.last_error()
    assert L.thq4_linear_chain(arr, 1, thq4.BF16, 1, P(ws), need, s) == thq4._lib.OK
    torch.cuda.synchronize()
