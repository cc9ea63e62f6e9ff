"""The prefill GEMM (m > 8 tokens, tcgen05) through the C ABI against the CPU
oracle.  The cases are the reference's prefill tests (quant_kernel.rs:
5428-5466, pf_vec_matches_legacy_bitwise): one LCG stream generates the tiled
weights and activations of every case in order; gate/up cases are a fused
[gate | up] weight of 2 x out rows.  The reference compares its kernel
families with each other; here every output is held to the reference CPU
path (bf16-dequantised weight, f32 accumulate)."""
import numpy as np
import pytest
import torch

import q4oracle as O
import thq4
from helpers import assert_close_ref, assert_gate_up_close, assert_rms_close, dev, dev_sb, to_f32

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def pf_cases():
    st = O.PfStream()
    cases = []
    for out, inp, gu, m in O.PF_CASES:
        total = 2 * out if gu else out
        tw, tsb, x = st.case(total, inp, m)
        wq, sb = O.tiled_to_mlx(tw, tsb, total, inp)
        cases.append((out, inp, gu, m, tw, tsb, wq, sb, x))
    return cases


@pytest.mark.parametrize("idx", range(len(O.PF_CASES)))
def test_prefill_matches_reference_cpu_path(pf_cases, idx):
    out, inp, gu, m, tw, tsb, wq, sb, x = pf_cases[idx]
    xd = dev(x)
    xf = O.bf16_to_f32(x)
    if not gu:
        q = thq4.QLin.from_layout(thq4.SRC_TILED, dev(tw), dev(tsb), out, inp, thq4.BF16)
        want = O.linear_dequant(wq, sb, O.SB_BF16, xf)
        got32 = to_f32(q.linear_ps(xd, out_dtype=torch.float32))
        assert got32.shape == (m, out)
        assert_rms_close(f"prefill f32 {out}x{inp} m{m}", got32, want, rel=1e-3)
        got = to_f32(q.linear(xd))
        for t in range(m):
            assert_close_ref(f"prefill bf16 {out}x{inp} m{m} t{t}", got[t], want[t])
        again = to_f32(q.linear(xd))
        assert np.array_equal(got, again), "not deterministic"
    else:
        q = thq4.QLin(dev(wq), dev(sb), 2 * out, inp, 64)
        got = to_f32(q.gate_up_act(xd))
        assert got.shape == (m, out)
        g = O.linear_dequant(wq, sb, O.SB_BF16, xf)
        for t in range(m):
            assert_gate_up_close(f"prefill gate_up {out}x{inp} m{m} t{t}", got[t], g[t, :out], g[t, out:], inp)


@pytest.mark.parametrize("m", [9, 16, 127, 300])
def test_prefill_token_counts(m):
    """Token counts around the decode/prefill boundary and tile edges."""
    out, inp = 392, 640
    wq, sb = O.synthetic_weight(out, inp, 900 + m, O.SB_F16)
    rng = np.random.default_rng(m)
    x = O.f32_to_bf16(rng.standard_normal((m, inp)).astype(np.float32))
    q = thq4.QLin(dev(wq), dev_sb(sb, O.SB_F16), out, inp, 64).tiled()
    got = to_f32(q.linear_ps(dev(x), out_dtype=torch.float32))
    assert_rms_close(f"prefill m{m}", got, O.linear_dequant(wq, sb, O.SB_F16, O.bf16_to_f32(x)), rel=1e-3)


@pytest.mark.parametrize("m", [512, 2048])
def test_prefill_baseline_config(m):
    """x [m x 4096] bf16 ~ N(0,1), W [12288 x 4096] ~
    N(0, 0.02) with f16 scale/bias.  The whole product runs on the GPU; the
    oracle checks 192 output columns (a block at each end and a seeded
    sample) on every token."""
    out, inp = 12288, 4096
    wq, sb = O.synthetic_weight(out, inp, 77, O.SB_F16)
    rng = np.random.default_rng(5 + m)
    x = O.f32_to_bf16(rng.standard_normal((m, inp)).astype(np.float32))
    q = thq4.QLin(dev(wq), dev_sb(sb, O.SB_F16), out, inp, 64).tiled()
    got = to_f32(q.linear_ps(dev(x), out_dtype=torch.float32))
    cols = np.unique(np.concatenate([np.arange(64), np.arange(out - 64, out), rng.choice(out, 64, replace=False)]))
    want = O.linear_dequant(wq[cols], sb[cols], O.SB_F16, O.bf16_to_f32(x))
    assert_rms_close(f"prefill C3 m{m}", got[:, cols], want, rel=1e-3)


@pytest.mark.parametrize("out,inp,m", [(20000, 1024, 300), (4608, 2048, 1100)])
@pytest.mark.parametrize("y_f32", [True, False])
def test_prefill_stream_k_split(out, inp, m, y_f32):
    """With a workspace of thq4_linear_workspace_bytes(w, m) bytes the
    prefill splits the k-stages of the tiles evenly over the SMs (these
    shapes have more 256-token tiles than SMs, not a whole number of waves,
    ragged rows and a ragged last token tile); a tile cut between two CTAs
    is finished by the one that claims it second.  Checked against the
    oracle on every token of 192 columns, against the whole-tile kernel (no
    workspace), for run-to-run equality, and for the claim words being zero
    again after the call."""
    import ctypes
    L = thq4.lib()
    wq, sb = O.synthetic_weight(out, inp, 31 + m, O.SB_F16)
    rng = np.random.default_rng(m)
    x = O.f32_to_bf16(rng.standard_normal((m, inp)).astype(np.float32))
    q = thq4.QLin(dev(wq), dev_sb(sb, O.SB_F16), out, inp, 64).tiled()
    desc = ctypes.byref(q.packed.desc)
    need = L.thq4_linear_workspace_bytes(desc, m)
    gemv_need = L.thq4_linear_workspace_bytes(desc, 1)
    assert need > gemv_need, "these shapes take the split"
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    xd = dev(x)
    ydt = torch.float32 if y_f32 else torch.bfloat16
    code = thq4.F32 if y_f32 else thq4.BF16
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def run(workspace):
        y = torch.full((m, out), float("nan"), dtype=ydt, device="cuda")
        wp, wn = (ctypes.c_void_p(workspace.data_ptr()), workspace.numel()) if workspace is not None else (None, 0)
        thq4.check(L.thq4_linear(desc, ctypes.c_void_p(xd.data_ptr()), thq4.BF16, m, ctypes.c_void_p(y.data_ptr()),
                                 code, wp, wn, stream))
        torch.cuda.synchronize()
        return to_f32(y)

    split = run(ws)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    sync0 = (gemv_need + 255) // 256 * 256
    assert int(ws[sync0:sync0 + 8 * sms].count_nonzero()) == 0, "claim words not zeroed"
    assert int(ws[:gemv_need].count_nonzero()) == 0, "decode region touched"
    again = run(ws)
    assert np.array_equal(split, again), "split prefill not deterministic"
    whole = run(None)
    assert not np.isnan(split).any() and not np.isnan(whole).any()
    cols = np.unique(np.concatenate([np.arange(64), np.arange(out - 64, out), rng.choice(out, 64, replace=False)]))
    want = O.linear_dequant(wq[cols], sb[cols], O.SB_F16, O.bf16_to_f32(x))
    if y_f32:
        assert_rms_close(f"split prefill {out}x{inp} m{m}", split[:, cols], want, rel=1e-3)
        assert_rms_close(f"whole prefill {out}x{inp} m{m}", whole[:, cols], want, rel=1e-3)
        assert_rms_close(f"split vs whole {out}x{inp} m{m}", split, whole, rel=1e-5)
    else:  # bf16 outputs: the reference's per-element rule (qwen35.rs:6946-6961)
        for t in range(m):
            assert_close_ref(f"split prefill bf16 {out}x{inp} m{m} t{t}", split[t, cols], want[t])
            assert_close_ref(f"whole prefill bf16 {out}x{inp} m{m} t{t}", whole[t, cols], want[t])


def test_prefill_split_needs_aligned_workspace():
    """A workspace large enough for the split but not 256-byte aligned runs
    whole tiles: the output equals the no-workspace call bit for bit."""
    import ctypes
    L = thq4.lib()
    out, inp, m = 4608, 2048, 1100
    wq, sb = O.synthetic_weight(out, inp, 5, O.SB_F16)
    x = dev(O.f32_to_bf16(np.random.default_rng(3).standard_normal((m, inp)).astype(np.float32)))
    q = thq4.QLin(dev(wq), dev_sb(sb, O.SB_F16), out, inp, 64).tiled()
    desc = ctypes.byref(q.packed.desc)
    need = L.thq4_linear_workspace_bytes(desc, m)
    ws = torch.zeros(need + 256, dtype=torch.uint8, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def run(ptr, n):
        y = torch.empty((m, out), dtype=torch.float32, device="cuda")
        thq4.check(L.thq4_linear(desc, ctypes.c_void_p(x.data_ptr()), thq4.BF16, m, ctypes.c_void_p(y.data_ptr()),
                                 thq4.F32, ptr, n, stream))
        torch.cuda.synchronize()
        return to_f32(y)

    shifted = run(ctypes.c_void_p(ws.data_ptr() + 16), need)
    whole = run(None, 0)
    assert np.array_equal(shifted, whole)
    assert int(ws.count_nonzero()) == 0, "the misaligned workspace was written"
