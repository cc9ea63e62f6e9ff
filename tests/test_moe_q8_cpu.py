"""The Q8 router, the shared expert's gate, grouping with the shared expert
and the layer with it, in the CPU oracle (no GPU): the C oracle against the
independent numpy restatement, and against the reference MoE test's own
fixture and expectations (docs/splash/dev/tests/engine/moe_metal_test.mm:
46-470: Random(0x0e5) expert slabs and rows, a router whose expert e reads
input column e at scale 4, a bias-only shared gate of 0.003 per group)."""
import numpy as np
import pytest

import q4_numpy as N
import q4oracle as O

H, I, E, K = 1024, 512, 8, 2  # moe_metal_test.mm:48-53
ROWS = 520  # kMaximumRows (moe_metal_test.mm:56)


def rand_q8(H_, seed):
    """A random Q8 projection in StorageN = 256 order."""
    rng = np.random.default_rng(seed)
    G = H_ // 64
    q = rng.integers(0, 256, G * 256 * 64, dtype=np.uint8)
    sc = O.f32_to_bf16(rng.uniform(0.0005, 0.004, G * 256).astype(np.float32))
    bi = O.f32_to_bf16((rng.standard_normal(G * 256) * 0.05).astype(np.float32))
    return q, sc, bi


def fixture_router(H_, E_):
    """fixtureRouter(backend, false) (moe_metal_test.mm:172-186)."""
    G = H_ // 64
    q = np.zeros(G * 256 * 64, np.uint8)
    sc = np.zeros(G * 256, np.uint16)
    bi = np.zeros(G * 256, np.uint16)
    for e in range(E_):
        q[e * 64 + e] = 1
        sc[e] = O.f32_to_bf16(np.float32([4.0]))[0]
    return q, sc, bi


def fixture_shared_gate(H_):
    """fixtureRouter(backend, true) (moe_metal_test.mm:187-196): row 0's
    bias 0.003 in every group, nothing else."""
    G = H_ // 64
    bi = np.zeros(G * 256, np.uint16)
    bi[np.arange(G) * 256] = O.f32_to_bf16(np.float32([0.003]))[0]
    return np.zeros(G * 256 * 64, np.uint8), np.zeros(G * 256, np.uint16), bi


def configure_routing(x, distribution):
    """configureRouting (moe_metal_test.mm:276-300): columns 0..E-1 of each
    row steer the router to a first and a second expert."""
    x = x.copy()
    for row in range(x.shape[0]):
        first = 0 if (distribution == "concentrated" or (distribution == "skewed" and row % 8 < 6)) else row % E
        second = (first + 1) % E
        vals = [1.0 if e == first else 0.5 if e == second else 0.01 * e for e in range(E)]
        x[row, :E] = O.f32_to_bf16(np.float32(vals))
    return x


@pytest.fixture(scope="module")
def fixture():
    return O.splash_moe_fixture(H, I, E, ROWS)


def test_router_scores_c_matches_numpy():
    T, H_, ncols = 37, 1024, 40
    q, sc, bi = rand_q8(H_, 3)
    x = O.f32_to_bf16(np.random.default_rng(4).standard_normal((T, H_)).astype(np.float32))
    c = O.moe_scores_q8(x, q, sc, bi, ncols)
    n = N.moe_scores_q8(x, q, sc, bi, ncols)
    assert np.array_equal(c, n)


@pytest.mark.parametrize("H_", [256, 384, 2048])
def test_router_scores_small_and_ragged_slices(H_):
    # H = 256 and 384 leave some of the eight K slices empty
    T = 5
    q, sc, bi = rand_q8(H_, H_)
    x = O.f32_to_bf16(np.random.default_rng(H_).standard_normal((T, H_)).astype(np.float32))
    assert np.array_equal(O.moe_scores_q8(x, q, sc, bi, 256), N.moe_scores_q8(x, q, sc, bi, 256))


def test_shared_gate_c_matches_numpy():
    T, H_ = 23, 2048
    q, sc, bi = rand_q8(H_, 8)
    x = O.f32_to_bf16(np.random.default_rng(9).standard_normal((T, H_)).astype(np.float32))
    w, logit = O.moe_shared_gate(x, q, sc, bi)
    w2, logit2 = N.moe_shared_gate(x, q, sc, bi)
    assert np.array_equal(logit, logit2)
    # exp differs between libraries by an ulp at most: one bf16 step apart at most
    assert np.abs(w.astype(np.int32) - w2.astype(np.int32)).max() <= 1


def test_fixture_generator_is_deterministic(fixture):
    f2 = O.splash_moe_fixture(H, I, E, 8)
    for name in ("gate", "up", "down", "shared_gate", "shared_up", "shared_down"):
        assert np.array_equal(fixture[name], f2[name]), name
    assert np.array_equal(fixture["x"][:8], f2["x"]) and np.array_equal(fixture["residual"][:8], f2["residual"])
    x = O.bf16_to_f32(fixture["x"])
    # inputs sign * (0.55 + 0.45 unit), negative on every third row (moe_metal_test.mm:259-268)
    assert np.all(x[0::3] < 0) and np.all(x[1::3] > 0) and np.all(np.abs(x) >= 0.099)
    assert np.all(np.abs(O.bf16_to_f32(fixture["residual"])) <= 0.1005)  # bf16 of 0.1 rounds up
    # scales in [0.01, 0.03), biases in [-0.25, -0.15) (moe_metal_test.mm:119-123)
    n = I * H
    sc = O.bf16_to_f32(fixture["gate"][0, n // 2:n // 2 + n // 32].view(np.uint16))
    bi = O.bf16_to_f32(fixture["gate"][0, n // 2 + n // 32:].view(np.uint16))
    assert sc.min() >= 0.0099 and sc.max() <= 0.0301 and bi.min() >= -0.2501 and bi.max() <= -0.1499


@pytest.mark.parametrize("distribution", ["dispersed", "concentrated", "skewed"])
def test_reference_fixture_routing_and_grouping(fixture, distribution):
    """The routing and grouping expectations of moe_metal_test.mm check()
    (:302-390), on the oracle."""
    x = configure_routing(fixture["x"], distribution)
    ids, w, scores = O.moe_route_q8(x, E, K, fixture_router(H, E), fixture_shared_gate(H))
    xf = O.bf16_to_f32(x)
    four = O.bf16_to_f32(O.f32_to_bf16((np.float32(4.0) * xf[:, :E]).astype(np.float32)))
    assert np.array_equal(O.bf16_to_f32(scores), four), "router scores are bf16(4 x_e)"
    wf = O.bf16_to_f32(w)
    for row in range(ROWS):
        ordered = sorted(range(E), key=lambda e: (-float(four[row, e]), e))
        assert list(ids[row, :K]) == ordered[:K], f"row {row}"
        a, b = float(four[row, ordered[0]]), float(four[row, ordered[1]])
        e0 = float(O.bf16_round(np.float32([1.0 / (1.0 + np.exp(np.float32(b - a)))]))[0])
        e1 = float(O.bf16_round(np.float32([1.0 / (1.0 + np.exp(np.float32(a - b)))]))[0])
        assert abs(wf[row, 0] + wf[row, 1] - 1.0) < 0.01
        assert abs(wf[row, 0] - e0) < 0.004 and abs(wf[row, 1] - e1) < 0.004
        s = np.float32(0)
        for v in xf[row]:
            s = np.float32(s + v)
        expect = 1.0 / (1.0 + np.exp(-float(s) * float(O.bf16_to_f32(O.f32_to_bf16(np.float32([0.003])))[0])))
        assert ids[row, K] == E and abs(wf[row, K] - expect) < 0.01, f"shared route, row {row}"

    for tile_rows in (8, 32):
        tiles, n, grouped, route_rows = O.moe_group_shared(ids, K, E, tile_rows)
        rows_ = ROWS
        assert K + 1 <= n <= rows_ * K + (rows_ + tile_rows - 1) // tile_rows
        counts = np.bincount(ids.ravel(), minlength=E + 1)
        assert n == sum((c + tile_rows - 1) // tile_rows for c in counts)
        for r in range(rows_ * (K + 1)):
            g = route_rows[r]
            assert g < n * tile_rows and grouped[g] == r and tiles[g // tile_rows, 0] == ids.ravel()[r]
        for t in range(n):
            live = tiles[t, 1]
            assert 0 < live <= tile_rows
            assert np.all(grouped[t * tile_rows + live:(t + 1) * tile_rows] == 0xFFFFFFFF)
        # the shared expert's tiles come last and hold every row in order
        nst = (rows_ + tile_rows - 1) // tile_rows
        assert np.all(tiles[n - nst:n, 0] == E)
        assert np.array_equal(grouped[(n - nst) * tile_rows:(n - nst) * tile_rows + rows_],
                              np.arange(rows_, dtype=np.uint32) * (K + 1) + K)
        assert n <= O.moe_max_tiles_shared(rows_, E, K, tile_rows, True)


def _mlx(fixture_part, out, inp):
    wq, sb = zip(*(O.slab_to_mlx(s, out, inp) for s in fixture_part))
    return np.stack(wq), np.stack(sb)


def mlx_experts(fixture):
    """The fixture's experts as MLX row-major weights: [gate | up] fused per
    expert, and down."""
    gq, gs = _mlx(fixture["gate"], I, H)
    uq, us = _mlx(fixture["up"], I, H)
    dq, ds = _mlx(fixture["down"], H, I)
    sgq, sgs = _mlx(fixture["shared_gate"], I, H)
    suq, sus = _mlx(fixture["shared_up"], I, H)
    sdq, sds = _mlx(fixture["shared_down"], H, I)
    gu_q, gu_s = np.concatenate([gq, uq], axis=1), np.concatenate([gs, us], axis=1)
    shared = (np.concatenate([sgq, suq], axis=1)[0], np.concatenate([sgs, sus], axis=1)[0], sdq[0], sds[0])
    return gu_q, gu_s, dq, ds, shared


def test_reference_fixture_layer_matches_project(fixture):
    """The layer with the shared expert against the reference test's
    expected output (moe_metal_test.mm:392-469) restated with the numpy
    projection, on a few rows: |y - ref| <= 0.02 + 0.01 * magnitude."""
    rows = 6
    x = configure_routing(fixture["x"], "dispersed")[:rows]
    res = fixture["residual"][:rows]
    ids, w, _ = O.moe_route_q8(x, E, K, fixture_router(H, E), fixture_shared_gate(H))
    gu_q, gu_s, dq, ds, shared = mlx_experts(fixture)
    y, h, d = O.moe_forward(x, res, ids, w, gu_q, gu_s, dq, ds, O.SB_BF16, I, want_h=True, shared=shared)
    xf = O.bf16_to_f32(x)
    wf = O.bf16_to_f32(w)
    for row in range(rows):
        expected = O.bf16_to_f32(res[row]).astype(np.float64)
        magnitude = np.abs(expected)
        for slot in range(K + 1):
            e = ids[row, slot]
            gq_, gs_ = (shared[0], shared[1]) if e == E else (gu_q[e], gu_s[e])
            dq_, ds_ = (shared[2], shared[3]) if e == E else (dq[e], ds[e])
            g = N.linear_group(gq_, gs_, 0, xf[row])[0]
            inter = O.bf16_to_f32(O.silu_mul_bf16(g[:I], g[I:]))
            got_h = O.bf16_to_f32(h[row * (K + 1) + slot])
            assert np.all(np.abs(got_h - inter) <= 0.02 + 0.01 * np.abs(inter)), "gate/up differs"
            down = O.bf16_round(N.linear_group(dq_, ds_, 0, got_h)[0]).astype(np.float64)
            expected += wf[row, slot] * down
            magnitude += np.abs(wf[row, slot] * down)
        yf = O.bf16_to_f32(y[row]).astype(np.float64)
        assert np.all(np.abs(yf - expected) <= 0.02 + 0.01 * magnitude), f"row {row}"


@pytest.mark.parametrize("T,E_,k,shared,tile_rows", [(37, 16, 4, True, 32), (100, 8, 2, True, 8),
                                                      (64, 32, 8, False, 32), (1, 4, 2, True, 32)])
def test_group_shared_c_matches_numpy(T, E_, k, shared, tile_rows):
    rng = np.random.default_rng(T * E_ + k)
    ids = np.stack([rng.permutation(E_)[:k] for _ in range(T)]).astype(np.uint32)
    if shared:
        ids = np.concatenate([ids, np.full((T, 1), E_, np.uint32)], axis=1)
    tiles, n, grouped, rr = O.moe_group_shared(ids, k, E_, tile_rows)
    t2, g2, rr2 = N.moe_group_shared(ids, k, E_, tile_rows)
    assert n == len(t2) and [tuple(t) for t in tiles[:n]] == t2
    assert np.array_equal(grouped[:n * tile_rows], g2) and np.array_equal(rr, rr2)


def _py_fixture(H_, I_, E_, rows, seed=0x0E5):
    """moe_metal_test.mm's Random and makeFixture (:69-75, :108-145, :217-271)
    restated in plain Python, as an independent check of the C generator:
    nibbles n-major, then per parameter a scale and a bias, slabs packed in
    StorageN = 256 order; then per row and column an input and a residual."""
    state = [seed]
    M = (1 << 64) - 1

    def nxt():
        state[0] = (state[0] * 6364136223846793005 + 1442695040888963407) & M
        return state[0] >> 33

    def unit():
        return np.float32(np.float32(nxt() & 0xFFFFFF) / np.float32(8388608.0)) - np.float32(1.0)

    def fma32(a, b, c):  # the contracted multiply-add of the reference build, rounded once
        return np.float32(np.float64(np.float32(a)) * np.float64(np.float32(b)) + np.float64(np.float32(c)))

    def slab(out, inp):
        n_el = out * inp
        nib = np.array([nxt() & 15 for _ in range(n_el)], dtype=np.uint8).reshape(out, inp)
        sc, bi = np.empty(n_el // 64, np.uint16), np.empty(n_el // 64, np.uint16)
        for i in range(n_el // 64):
            sc[i] = O.f32_to_bf16(np.float32([fma32(0.01, unit() + np.float32(1.0), 0.01)]))[0]
            bi[i] = O.f32_to_bf16(np.float32([fma32(0.05, unit(), -0.2)]))[0]
        groups = inp // 64
        packed = np.zeros(n_el // 2, np.uint8)
        for n in range(out):
            prm = ((n // 256) * groups + np.arange(groups)) * 256 + n % 256
            idx = (prm[:, None] * 64 + np.arange(64)[None, :]).ravel()
            vals = nib[n].reshape(groups, 64).ravel()
            lo, hi = idx[idx % 2 == 0], idx[idx % 2 == 1]
            packed[lo // 2] |= vals[idx % 2 == 0]
            packed[hi // 2] |= (vals[idx % 2 == 1] << 4).astype(np.uint8)
        return np.concatenate([packed, sc.view(np.uint8), bi.view(np.uint8)])

    f = {}
    for name, (o, i_, cnt) in [("gate", (I_, H_, E_)), ("up", (I_, H_, E_)), ("down", (H_, I_, E_)),
                               ("shared_gate", (I_, H_, 1)), ("shared_up", (I_, H_, 1)),
                               ("shared_down", (H_, I_, 1))]:
        f[name] = np.stack([slab(o, i_) for _ in range(cnt)])
    x, res = np.empty((rows, H_), np.uint16), np.empty((rows, H_), np.uint16)
    for r in range(rows):
        sign = np.float32(-1.0 if r % 3 == 0 else 1.0)
        for c in range(H_):
            x[r, c] = O.f32_to_bf16(np.float32([sign * fma32(0.45, unit(), 0.55)]))[0]
            res[r, c] = O.f32_to_bf16(np.float32([np.float32(0.1) * unit()]))[0]
    f["x"], f["residual"] = x, res
    return f


def test_fixture_generator_matches_a_python_restatement():
    got = O.splash_moe_fixture(256, 256, 1, 3)
    want = _py_fixture(256, 256, 1, 3)
    for name in want:
        assert np.array_equal(got[name], want[name]), name
