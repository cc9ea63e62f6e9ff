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
