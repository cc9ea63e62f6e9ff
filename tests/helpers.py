"""Helpers shared by the GPU tests: device uploads and the reference's
tolerance rules."""
from __future__ import annotations

import numpy as np
import torch

import q4oracle as O


def dev(a: np.ndarray) -> torch.Tensor:
    """numpy -> CUDA tensor with the same bytes (uint32 goes through int32)."""
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        return torch.from_numpy(a.view(np.int32)).cuda()
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).cuda().view(torch.bfloat16)
    return torch.from_numpy(a).cuda()


def dev_sb(sb: np.ndarray, sb_dtype: int) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(sb).view(np.int16)).cuda()
    return t.view(torch.float16 if sb_dtype == O.SB_F16 else torch.bfloat16)


def host_bits(t: torch.Tensor) -> np.ndarray:
    """Raw bytes of a CUDA tensor as a numpy array of the matching unsigned type."""
    c = t.detach().contiguous().cpu()
    if c.element_size() == 2:
        return c.view(torch.int16).numpy().view(np.uint16)
    if c.element_size() == 4:
        return c.view(torch.int32).numpy().view(np.uint32)
    return c.view(torch.uint8).numpy()


def to_f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def assert_close_ref(tag: str, got: np.ndarray, want: np.ndarray) -> float:
    """The reference's qmvt tolerance (qwen35.rs:6946-6961): |got - want| <=
    2^-7 * max(|want|, 0.02 * max|want|) per element -- one bf16 rounding
    step apart, floored for near-zero rows.  Returns max|d| / max|want|."""
    got = np.asarray(got, dtype=np.float64).ravel()
    want = np.asarray(want, dtype=np.float64).ravel()
    assert got.shape == want.shape, f"{tag}: len"
    mag = np.abs(want).max()
    assert mag > 0, f"{tag}: degenerate reference"
    tol = 2.0 ** -7 * np.maximum(np.abs(want), 0.02 * mag)
    d = np.abs(got - want)
    bad = np.nonzero(d > tol)[0]
    assert bad.size == 0, (f"{tag}: {bad.size} elements off, first row {bad[0]}: got {got[bad[0]]} "
                           f"want {want[bad[0]]} (|d| {d[bad[0]]} > {tol[bad[0]]})")
    return float(d.max() / mag)


def assert_rms_close(tag: str, got: np.ndarray, want: np.ndarray, rel: float = 1e-2) -> float:
    """The north-star bar: max|got - want| <= rel * RMS(want)."""
    got = np.asarray(got, dtype=np.float64).ravel()
    want = np.asarray(want, dtype=np.float64).ravel()
    rms = float(np.sqrt(np.mean(want ** 2)))
    err = float(np.abs(got - want).max())
    assert err <= rel * rms, f"{tag}: max|err| {err:.3e} > {rel} * RMS {rms:.3e}"
    return err / rms


def assert_gate_up_close(tag: str, got: np.ndarray, gate: np.ndarray, up: np.ndarray, inp: int) -> None:
    """The reference's split-K tolerance for the gate/up epilogue
    (LinearNumerics.hpp:112-126, pinned by tests/test_oracle.py): the output
    bf16(silu(bf16 g) * bf16 u) may move by one ulp of the output plus what one
    ulp (plus fp32 reassociation slack) of g and of u propagates to."""
    from helpers_tol import split_tolerance
    got = np.asarray(got, dtype=np.float64).ravel()
    gate = np.asarray(gate, dtype=np.float64).ravel()
    up = np.asarray(up, dtype=np.float64).ravel()
    import q4oracle as O
    want = O.bf16_to_f32(O.silu_mul_bf16(gate.astype(np.float32), up.astype(np.float32))).astype(np.float64)
    slack = (inp // 64) * 2.0 ** -24 * max(np.abs(gate).max(), np.abs(up).max())
    for i in range(got.size):
        tol = split_tolerance(2, want[i], 0.0, gate[i], up[i], slack)
        assert abs(got[i] - want[i]) <= tol, (f"{tag}: element {i}: got {got[i]} want {want[i]} "
                                              f"(g {gate[i]}, u {up[i]}, tol {tol})")


def moe_combine_f32(residual_bf16, weights_bf16, d_bf16, T: int, H: int) -> np.ndarray:
    """The MoE combine before its bf16 rounding (moe.metal:642-664): per
    token, the residual (or 0) then + w * d over the route slots in order,
    each product and each sum rounded to f32 (no fused multiply-add), from
    the oracle's per-route bf16 expert outputs d [T * slots][H]."""
    w = O.bf16_to_f32(np.asarray(weights_bf16)).astype(np.float32).reshape(T, -1)
    slots = w.shape[1]
    d = O.bf16_to_f32(np.asarray(d_bf16)).astype(np.float32).reshape(T, slots, H)
    acc = np.zeros((T, H), dtype=np.float32) if residual_bf16 is None else \
        O.bf16_to_f32(np.asarray(residual_bf16)).astype(np.float32).reshape(T, H)
    for s in range(slots):
        prod = (w[:, s:s + 1] * d[:, s, :]).astype(np.float32)
        acc = (acc + prod).astype(np.float32)
    return acc


def ulp_bf16_array(v) -> np.ndarray:
    """One bf16 step at each |v| (LinearNumerics.hpp ulpBf16, restated in
    tests/helpers_tol.py and pinned there): 2^(e - 8) for |v| in [2^(e-1), 2^e),
    2^-133 below the normal range."""
    a = np.abs(np.asarray(v, dtype=np.float64))
    out = np.full(a.shape, 2.0 ** -133)
    ok = a >= 2.0 ** -126
    _, e = np.frexp(a[ok])
    out[ok] = np.ldexp(1.0, e - 8)
    return out


def assert_moe_close(tag: str, got32, want32, weights_bf16, d_bf16, T: int, H: int, rel: float = 1e-2,
                     max_beyond: float = 1e-3) -> dict:
    """The MoE layer's f32 output (the combine before its bf16 rounding)
    against the oracle's.  The reference stores every route's expert output d
    in bf16 (moe.metal:642-664 reads expert_output as bfloat), so two correct
    implementations whose f32 sums differ in order round a few d elements to
    neighbouring bf16 values; one such step at |d| ~ 0.5 alone moves an output
    by ~2e-3, above 1e-2 RMS of this layer.  The bar is therefore, per
    element: |got - want| <= rel * RMS(want) + sum over the token's routes of
    |w| * one bf16 step of d (one rounding flip per route), and at most
    `max_beyond` of the elements may exceed rel * RMS at all (flips are rare)."""
    got = np.asarray(got32, dtype=np.float64).reshape(T, H)
    want = np.asarray(want32, dtype=np.float64).reshape(T, H)
    w = np.abs(O.bf16_to_f32(np.asarray(weights_bf16)).astype(np.float64)).reshape(T, -1)
    slots = w.shape[1]
    d = O.bf16_to_f32(np.asarray(d_bf16)).astype(np.float64).reshape(T, slots, H)
    flip = (w[:, :, None] * ulp_bf16_array(d)).sum(axis=1)
    rms = float(np.sqrt(np.mean(want ** 2)))
    err = np.abs(got - want)
    bad = err > rel * rms + flip
    assert not bad.any(), (f"{tag}: {int(bad.sum())} outputs beyond 1e-2 RMS + one bf16 step per route; "
                           f"worst {float(err[bad].max()):.3e} (RMS {rms:.3e})")
    beyond = float((err > rel * rms).mean())
    assert beyond <= max_beyond, f"{tag}: {beyond:.2e} of the outputs exceed {rel} RMS (flips should be rare)"
    return {"max_err_over_rms": float(err.max()) / rms, "beyond_rel": beyond}
