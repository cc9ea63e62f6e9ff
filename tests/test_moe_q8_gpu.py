"""The Splash MoE block on the GPU (thq4_moe_add and its parts) against the
CPU oracle: the Q8 router's scores bit for bit, the routing (expert ids, the
shared route, the grouping permutation) bit for bit, routing weights within
one bf16 step (exp differs between libraries by an ulp), and the layer with
the reference MoE test's own fixture and tolerance
(docs/splash/dev/tests/engine/moe_metal_test.mm:392-469:
|y - ref| <= 0.02 + 0.01 * the magnitude of the contributions)."""
import ctypes

import numpy as np
import pytest
import torch

import q4oracle as O
import thq4
from helpers import assert_moe_close, moe_combine_f32
from thq4 import _lib
from test_moe_q8_cpu import (E, H, I, K, configure_routing, fixture_router, fixture_shared_gate, mlx_experts,
                             rand_q8)

pytestmark = pytest.mark.gpu


def q8(parts, inp):
    q, sc, bi = parts
    return thq4.Q8Projection(torch.from_numpy(q).cuda(), torch.from_numpy(sc.view(np.int16)).cuda().view(torch.bfloat16),
                             torch.from_numpy(bi.view(np.int16)).cuda().view(torch.bfloat16), inp)


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def dev_bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda().view(torch.bfloat16)


def status() -> int:
    st = ctypes.c_uint32()
    thq4.check(thq4.lib().thq4_device_status(ctypes.byref(st), None))
    return st.value


@pytest.mark.parametrize("T,H_,ncols", [(1, 2048, 128), (8, 2048, 256), (37, 1024, 40), (256, 2048, 128),
                                        (70, 256, 64)])
def test_router_scores_bit_exact(T, H_, ncols):
    parts = rand_q8(H_, T + H_)
    x = O.f32_to_bf16(np.random.default_rng(T).standard_normal((T, H_)).astype(np.float32))
    got = bits(thq4.moe_scores_q8(dev_bf16(x), q8(parts, H_), ncols))
    want = O.moe_scores_q8(x, *parts, ncols)
    assert np.array_equal(got, want), f"{(got != want).sum()} of {want.size} scores differ"


@pytest.mark.parametrize("T,H_,E_,k,shared", [(1, 2048, 128, 8, True), (8, 2048, 128, 8, False),
                                              (256, 2048, 128, 8, True), (520, 1024, 8, 2, True),
                                              (100, 512, 256, 32, True)])
def test_route_q8_matches_oracle(T, H_, E_, k, shared):
    rp = rand_q8(H_, 7 + T)
    sp = rand_q8(H_, 8 + T) if shared else None
    x = O.f32_to_bf16(np.random.default_rng(T + 1).standard_normal((T, H_)).astype(np.float32))
    status()
    ids, w, tiles, grouped, rows = thq4.moe_route_q8(dev_bf16(x), q8(rp, H_), E_, k, q8(sp, H_) if shared else None)
    torch.cuda.synchronize()
    assert status() == 0
    want_ids, want_w, _ = O.moe_route_q8(x, E_, k, rp, sp)
    got_ids = ids.cpu().numpy().view(np.uint32)
    assert np.array_equal(got_ids, want_ids), "expert selection differs"
    dw = np.abs(bits(w).astype(np.int32) - want_w.astype(np.int32))
    assert dw.max() <= 1, "routing weights differ by more than one bf16 step"
    t_want, n_want, g_want, rr_want = O.moe_group_shared(want_ids, k, E_, 32)
    n = tiles.shape[0]
    assert n == n_want
    assert np.array_equal(tiles.cpu().numpy().view(np.uint32), t_want[:n])
    assert np.array_equal(grouped.cpu().numpy().view(np.uint32), g_want[:n * 32])
    assert np.array_equal(rows.cpu().numpy().view(np.uint32), rr_want)


@pytest.fixture(scope="module")
def fixture():
    return O.splash_moe_fixture(H, I, E, 520)


def _weights(fixture, shared=True, e0=0, e1=E, run_shared=None):
    slabs = lambda name, lo=0, hi=None: torch.from_numpy(fixture[name][lo:hi]).cuda()  # noqa: E731
    gate = thq4.PackedExperts.from_slabs(slabs("gate", e0, e1), I, H, thq4.BF16)
    up = thq4.PackedExperts.from_slabs(slabs("up", e0, e1), I, H, thq4.BF16)
    down = thq4.PackedExperts.from_slabs(slabs("down", e0, e1), H, I, thq4.BF16)
    run_shared = shared if run_shared is None else run_shared
    sg = su = sd = None
    if run_shared:
        sg = thq4.PackedExperts.from_slabs(slabs("shared_gate"), I, H, thq4.BF16)
        su = thq4.PackedExperts.from_slabs(slabs("shared_up"), I, H, thq4.BF16)
        sd = thq4.PackedExperts.from_slabs(slabs("shared_down"), H, I, thq4.BF16)
    return thq4.MoeWeights(q8(fixture_router(H, E), H), gate, up, down, sg, su, sd,
                           q8(fixture_shared_gate(H), H) if shared else None)


@pytest.mark.parametrize("distribution", ["dispersed", "concentrated", "skewed"])
@pytest.mark.parametrize("rows", [1, 8, 37, 520])
def test_reference_fixture_moe_add(fixture, distribution, rows):
    """moe_metal_test.mm's fixture and checks, through thq4_moe_add."""
    x = configure_routing(fixture["x"], distribution)[:rows]
    res = fixture["residual"][:rows]
    w = _weights(fixture)
    status()
    y = thq4.moe_add(dev_bf16(x), w, K, residual=dev_bf16(res))
    ids, wt, tiles, grouped, route_rows = thq4.moe_route_q8(dev_bf16(x), w.router, E, K, w.shared_expert_gate)
    torch.cuda.synchronize()
    assert status() == 0
    want_ids, want_w, _ = O.moe_route_q8(x, E, K, fixture_router(H, E), fixture_shared_gate(H))
    assert np.array_equal(ids.cpu().numpy().view(np.uint32), want_ids)
    assert np.abs(bits(wt).astype(np.int32) - want_w.astype(np.int32)).max() <= 1
    assert tiles.shape[0] >= K + 1
    gu_q, gu_s, dq, ds, shared = mlx_experts(fixture)
    want_y, _, d = O.moe_forward(x, res, want_ids, want_w, gu_q, gu_s, dq, ds, O.SB_BF16, I, shared=shared)
    wf = O.bf16_to_f32(want_w).astype(np.float64)
    mag = np.abs(O.bf16_to_f32(res).astype(np.float64))
    dd = O.bf16_to_f32(d).astype(np.float64).reshape(rows, K + 1, H)
    mag += np.abs(wf[:, :, None] * dd).sum(axis=1)
    got = O.bf16_to_f32(bits(y)).astype(np.float64)
    ref = O.bf16_to_f32(want_y).astype(np.float64)
    assert np.all(np.isfinite(got))
    bad = np.abs(got - ref) > 0.02 + 0.01 * mag
    assert not bad.any(), f"{bad.sum()} outputs differ from the oracle's layer"


@pytest.mark.parametrize("distribution", ["dispersed", "concentrated", "skewed"])
def test_reference_fixture_f32_at_north_star_bar(fixture, distribution):
    """The whole block (all 520 rows, shared expert included) in f32: the
    f32 output of thq4_moe_add_partial over every expert, with the residual,
    is the combine before its one bf16 rounding; against the oracle's f32
    combine of its own per-route expert outputs, max|err| <= 1e-2 * RMS plus
    one bf16 step of each route's bf16 expert output (assert_moe_close; the
    reference test's 0.02 + 0.01 magnitude above is the weaker check)."""
    rows = 520
    x = configure_routing(fixture["x"], distribution)[:rows]
    res = fixture["residual"][:rows]
    w = _weights(fixture)
    y32 = thq4.moe_add_partial(dev_bf16(x), w, K, 0, E, residual=dev_bf16(res))
    y = thq4.moe_add(dev_bf16(x), w, K, residual=dev_bf16(res))
    torch.cuda.synchronize()
    assert status() == 0
    want_ids, want_w, _ = O.moe_route_q8(x, E, K, fixture_router(H, E), fixture_shared_gate(H))
    gu_q, gu_s, dq, ds, shared = mlx_experts(fixture)
    _, _, d = O.moe_forward(x, res, want_ids, want_w, gu_q, gu_s, dq, ds, O.SB_BF16, I, shared=shared)
    # the device's routing weights may differ from the host's by one bf16 step
    # (exp); the oracle's combine uses the device's weights
    _, wt, _, _, _ = thq4.moe_route_q8(dev_bf16(x), w.router, E, K, w.shared_expert_gate)
    want = moe_combine_f32(res, bits(wt), d, rows, H)
    got = y32.cpu().numpy()
    assert np.all(np.isfinite(got))
    assert_moe_close(f"block f32 {distribution}", got, want, bits(wt), d, rows, H)
    assert torch.equal(y32.to(torch.bfloat16).view(torch.int16), y.view(torch.int16)), "bf16 block != rounded f32"


def test_without_shared_expert_equals_logits_path(fixture):
    """With no shared expert, thq4_moe_add is thq4_moe on the router's scores:
    the same routing and the same kernels, bit for bit."""
    rows = 64
    x = configure_routing(fixture["x"], "skewed")[:rows]
    w = _weights(fixture, shared=False)
    y = thq4.moe_add(dev_bf16(x), w, K)
    scores = thq4.moe_scores_q8(dev_bf16(x), w.router, E)
    y2 = thq4.moe(dev_bf16(x), scores, K, w.gate, w.up, w.down)
    torch.cuda.synchronize()
    assert torch.equal(y.view(torch.int16), y2.view(torch.int16))


def test_expert_shards_sum_to_the_block(fixture):
    """Two shards on one GPU: experts [0, 4) with the shared expert and
    [4, 8) without; their f32 partials sum to the whole block's output up to
    the f32 summation order."""
    rows = 40
    x = configure_routing(fixture["x"], "dispersed")[:rows]
    res = dev_bf16(fixture["residual"][:rows])
    full = thq4.moe_add(dev_bf16(x), _weights(fixture), K, residual=res)
    p0 = thq4.moe_add_partial(dev_bf16(x), _weights(fixture, e0=0, e1=4, run_shared=True), K, 0, E, residual=res)
    p1 = thq4.moe_add_partial(dev_bf16(x), _weights(fixture, e0=4, e1=8, run_shared=False), K, 4, E)
    torch.cuda.synchronize()
    got = (p0 + p1).bfloat16().float()
    diff = (got - full.float()).abs()
    assert float(diff.max()) <= 0.02 + 0.01 * float(full.float().abs().max())
    assert float((diff > 0).float().mean()) < 0.05, "most outputs agree bit for bit"


def test_moe_add_validation(fixture):
    L = thq4.lib()
    w = _weights(fixture)
    x = torch.zeros((4, H), dtype=torch.bfloat16, device="cuda")
    y = torch.empty_like(x)
    ws = torch.empty(1 << 20, dtype=torch.uint8, device="cuda")
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    # I not a multiple of 256 (MoeShape::valid, MoE.hpp:21-26)
    st = L.thq4_moe_add(P(x), None, 4, H, 320, E, K, ctypes.byref(w.desc), P(y), P(ws), ws.numel(), s)
    assert st == _lib.ERR_INVALID_ARGUMENT and "execution shape" in thq4.last_error()
    # a router of the wrong input size
    d = _lib.thq4_moe_weights.from_buffer_copy(w.desc)
    d.router.in_ = 512
    st = L.thq4_moe_add(P(x), None, 4, H, I, E, K, ctypes.byref(d), P(y), P(ws), ws.numel(), s)
    assert st == _lib.ERR_INVALID_ARGUMENT and "router" in thq4.last_error()
    # the shared expert without its gate
    d = _lib.thq4_moe_weights.from_buffer_copy(w.desc)
    d.shared_expert_gate.q = None
    st = L.thq4_moe_add(P(x), None, 4, H, I, E, K, ctypes.byref(d), P(y), P(ws), ws.numel(), s)
    assert st == _lib.ERR_INVALID_ARGUMENT
    # scratch below the bound
    need = L.thq4_moe_add_workspace_bytes(4, H, I, E, K, 1)
    st = L.thq4_moe_add(P(x), None, 4, H, I, E, K, ctypes.byref(w.desc), P(y), P(ws), need - 1, s)
    assert st == _lib.ERR_WORKSPACE and "smaller than its bound" in thq4.last_error()
