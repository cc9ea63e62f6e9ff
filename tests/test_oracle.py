"""The CPU oracle: cross-checked against an independent numpy restatement,
pinned against the reference's own compiled C++ helpers where those exist, and
against the committed golden fixtures.  No GPU."""
import os

import numpy as np
import pytest

import q4_numpy as N
import q4oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden_oracle.npz")


def test_lcg_matches_reference_sequence():
    # q4o_lcg is the reference tests' LCG (qwen35.rs:6889-6892)
    s = 11
    got = []
    import ctypes
    st = ctypes.c_uint64(s)
    for _ in range(4):
        got.append(O.lib().q4o_lcg(ctypes.byref(st)))
    want, x = [], s
    for _ in range(4):
        x = (x * 6364136223846793005 + 1442695040888963407) % (1 << 64)
        want.append(x >> 33)
    assert got == want


@pytest.mark.parametrize("out,ng", O.QMVT_PLAIN_CASES)
def test_linear_group_matches_numpy(out, ng):
    inp = ng * 64
    wq, sb = O.rand_qlin(out, inp, 3)
    x = O.bf16_to_f32(np.stack([O.rand_x(inp, 5), O.rand_x(inp, 6)]))
    a = O.linear_group(wq, sb, O.SB_BF16, x)
    b = N.linear_group(wq, sb, O.SB_BF16, x)
    assert np.allclose(a, b, rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("sb_dtype", [O.SB_BF16, O.SB_F16])
def test_layouts_round_trip_and_match_numpy(sb_dtype):
    wq, sb = O.synthetic_weight(520, 448, 1, sb_dtype)
    for ts in (1, 2, 8):
        fq, fsb = O.mlx_to_frag(wq, sb, ts)
        fq2, fsb2 = N.frag_from_mlx(wq, sb, 520, 448, ts)
        assert np.array_equal(fq, fq2) and np.array_equal(fsb, fsb2)
        w2, s2 = O.frag_to_mlx(fq, fsb, 520, 448, ts)
        assert np.array_equal(w2, wq) and np.array_equal(s2, sb)
    tw, tsb = O.mlx_to_tiled(wq, sb)
    tw2, tsb2 = N.tiled_from_mlx(wq, sb, 520, 448)
    assert np.array_equal(tw, tw2) and np.array_equal(tsb, tsb2)
    w3, s3 = O.tiled_to_mlx(tw, tsb, 520, 448)
    assert np.array_equal(w3, wq) and np.array_equal(s3, sb)


def test_slab_is_tiled_byte_for_byte():
    # moe_metal_test.mm:126-145 packs nibble (n, k) at parameter(n, g)*64 + k%64
    wq, sb = O.rand_qlin(512, 256, 9)
    slab = O.mlx_to_slab(wq, sb)
    assert slab.size == 512 * 256 // 16 * 9  # q4PackedBytes, WeightStore.cpp:57-60
    tw, tsb = O.mlx_to_tiled(wq, sb)
    assert np.array_equal(slab[: 512 * 256 // 2], tw.view(np.uint8))
    q = N.unpack_mlx(wq)
    nib = np.frombuffer(slab[: 512 * 256 // 2].tobytes(), dtype=np.uint8)
    for n, k in [(0, 0), (3, 65), (300, 255), (511, 130)]:
        prm = ((n // 256) * 4 + k // 64) * 256 + n % 256
        idx = prm * 64 + k % 64
        byte = nib[idx // 2]
        assert ((byte >> 4) if idx & 1 else (byte & 15)) == q[n, k]
    w2, s2 = O.slab_to_mlx(slab, 512, 256)
    assert np.array_equal(w2, wq) and np.array_equal(s2, sb)


def test_quantiser_bounds():
    rng = np.random.default_rng(0)
    w = rng.standard_normal((64, 512)).astype(np.float32) * 0.02
    for sbd in (O.SB_BF16, O.SB_F16):
        wq, sb = O.quantize(w, sbd)
        deq = N.unpack_mlx(wq) * N.sb_values(sb, sbd)[:, :8].repeat(64, 1) + N.sb_values(sb, sbd)[:, 8:].repeat(64, 1)
        step = (w.reshape(64, 8, 64).max(2) - w.reshape(64, 8, 64).min(2)) / 15
        assert np.all(np.abs(deq - w) <= 0.51 * step.repeat(64, 1) + 2e-4)


def test_dequant_path_vs_group_path_within_north_star_bar():
    wq, sb = O.synthetic_weight(256, 1024, 4, O.SB_F16)
    x = np.random.default_rng(1).standard_normal((2, 1024)).astype(np.float32)
    a = O.linear_group(wq, sb, O.SB_F16, x)
    b = O.linear_dequant(wq, sb, O.SB_F16, x)
    assert np.abs(a - b).max() <= 1e-2 * np.sqrt((a ** 2).mean())


def test_moe_select_tie_break_and_weights():
    rng = np.random.default_rng(3)
    logits = O.f32_to_bf16(rng.standard_normal((40, 64)).astype(np.float32))
    logits[0, :] = O.f32_to_bf16(np.zeros(64, np.float32))  # all tied: ids 0..k-1
    logits[1, 10] = logits[1, 5] = O.f32_to_bf16(np.float32([9.0]))[0]
    ids, w = O.moe_select(logits, 8)
    ids2, w2 = N.moe_select(logits, 8)
    assert np.array_equal(ids, ids2) and np.array_equal(w, w2)
    assert list(ids[0]) == list(range(8))
    assert ids[1, 0] == 5 and ids[1, 1] == 10
    assert np.allclose(O.bf16_to_f32(w).sum(1), 1.0, atol=0.02)


@pytest.mark.parametrize("tile_rows", [8, 16, 32])
def test_moe_group_is_stable_counting_sort(tile_rows):
    rng = np.random.default_rng(tile_rows)
    ids = rng.integers(0, 32, size=(100, 4)).astype(np.uint32)
    ids[:, 1] = 3  # a hot expert spanning several tiles
    tiles, n, grouped, rr = O.moe_group(ids, 32, tile_rows)
    t2, g2, rr2 = N.moe_group(ids, 32, tile_rows)
    assert n == len(t2) and np.array_equal(tiles[:n], np.array(t2, np.uint32))
    assert np.array_equal(grouped[: n * tile_rows], g2) and np.array_equal(rr, rr2)
    # round trip and padding (moe_metal_test.mm:330-360)
    flat = ids.ravel()
    for r in range(flat.size):
        assert grouped[rr[r]] == r and tiles[rr[r] // tile_rows, 0] == flat[r]
    for t in range(n):
        live = tiles[t, 1]
        assert 0 < live <= tile_rows
        assert np.all(grouped[t * tile_rows + live:(t + 1) * tile_rows] == 0xFFFFFFFF)
    assert n <= O.moe_max_tiles(100, 32, 4, tile_rows)


def test_moe_forward_small_matches_project_semantics():
    T, H, I, E, k = 6, 128, 128, 4, 2
    rng = np.random.default_rng(5)
    x = O.f32_to_bf16(rng.standard_normal((T, H)).astype(np.float32))
    logits = O.f32_to_bf16(rng.standard_normal((T, E)).astype(np.float32))
    ids, w = O.moe_select(logits, k)
    gu = [O.synthetic_weight(2 * I, H, 10 + e, O.SB_BF16) for e in range(E)]
    dn = [O.synthetic_weight(H, I, 20 + e, O.SB_BF16) for e in range(E)]
    gu_wq = np.stack([a for a, _ in gu]); gu_sb = np.stack([b for _, b in gu])
    dn_wq = np.stack([a for a, _ in dn]); dn_sb = np.stack([b for _, b in dn])
    y, h, d = O.moe_forward(x, None, ids, w, gu_wq, gu_sb, dn_wq, dn_sb, O.SB_BF16, I, want_h=True)
    for t in range(T):
        acc = np.zeros(H, np.float32)
        for s in range(k):
            e = ids[t, s]
            g = N.linear_group(gu_wq[e], gu_sb[e], 0, O.bf16_to_f32(x[t]))[0]
            hh = O.bf16_to_f32(O.silu_mul_bf16(g[:I], g[I:]))
            assert np.abs(hh - O.bf16_to_f32(h[t * k + s])).max() <= 0.02 + 0.01 * np.abs(hh).max()
            dd = O.bf16_round(N.linear_group(dn_wq[e], dn_sb[e], 0, O.bf16_to_f32(h[t * k + s]))[0])
            acc += O.bf16_to_f32(w[t, s : s + 1])[0] * dd
        assert np.abs(O.bf16_to_f32(y[t]) - acc).max() <= 0.02 + 0.01 * np.abs(acc).max()


# ---- pins against the reference's own compiled C++ ------------------------------

ref = O.ref_pins()
needs_ref = pytest.mark.skipif(ref is None, reason="oracle/_ref not built (reference not mounted when built)")


@needs_ref
def test_bf16_rounding_pinned_to_reference():
    rng = np.random.default_rng(11)
    vals = (rng.standard_normal(20000) * 10.0 ** rng.uniform(-38, 38, 20000)).astype(np.float32)
    # ties: values exactly half-way between bf16 neighbours
    ties = (np.arange(1, 2001, dtype=np.uint32) << 16 | 0x8000).view(np.float32)
    vals = np.concatenate([vals, ties, -ties, np.float32([0.0, -0.0, 1e-40, -1e-40])])
    ours = O.f32_to_bf16(vals)
    theirs = np.array([ref.ref_float_to_bf16(float(v)) for v in vals], dtype=np.uint16)
    assert np.array_equal(ours, theirs)
    back = np.array([ref.ref_bf16_to_float(int(b)) for b in ours[:500]], dtype=np.float32)
    assert np.array_equal(back, O.bf16_to_f32(ours[:500]))


@needs_ref
def test_moe_bounds_pinned_to_reference():
    assert ref.ref_moe_tile_descriptor_bytes() == 8
    for T, E, k, tr in [(256, 128, 8, 8), (256, 128, 8, 16), (7, 8, 2, 32), (520, 8, 2, 8)]:
        # the reference adds ceil(T/tr) tiles for its shared expert
        assert ref.ref_moe_maximum_tiles(T, 2048, E, k, 768, tr) == O.moe_max_tiles(T, E, k, tr) + (T + tr - 1) // tr


@needs_ref
def test_split_tolerance_pinned_to_reference():
    import ctypes  # noqa: F401
    from helpers_tol import split_tolerance, ulp_bf16
    rng = np.random.default_rng(4)
    for v in rng.standard_normal(300).astype(np.float32) * 10:
        assert ulp_bf16(float(v)) == ref.ref_ulp_bf16(float(v))
        for epi in (0, 2):
            g, u = float(v) * 0.5, float(v) * 0.25
            assert np.isclose(split_tolerance(epi, float(v), 0.0, g, u, 1e-6),
                              ref.ref_split_tolerance(epi, float(v), 0.0, g, u, 1e-6), rtol=1e-6)


# ---- golden fixtures -------------------------------------------------------------

def test_golden_fixtures_reproduce():
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(os.path.dirname(GOLDEN), "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    want = np.load(GOLDEN)
    got = mg.compute()
    assert set(got) == set(want.files)
    for k in want.files:
        assert np.array_equal(np.asarray(got[k]), want[k]), k


def test_presum_sums_follow_the_lane_pattern():
    """The presum sums (q4_store_input_sums, quant_kernel.rs:1864-1884) against
    a plain-Python restatement: lane l adds x[64g + l] + x[64g + 32 + l], then
    xor butterfly over the 32 lanes, every add in f32."""
    rng = np.random.default_rng(3)
    rows = O.f32_to_bf16(rng.standard_normal((8, 192)).astype(np.float32))
    got = O.presum_sums(rows)
    xf = O.bf16_to_f32(rows).astype(np.float32)
    for t in range(8):
        for g in range(3):
            v = [np.float32(xf[t, 64 * g + l] + xf[t, 64 * g + 32 + l]) for l in range(32)]
            for o in (16, 8, 4, 2, 1):
                v = [np.float32(v[l] + v[l ^ o]) for l in range(32)]
            assert got[g, t] == v[0]
    assert abs(float(got.sum()) - float(xf.astype(np.float64).sum())) < 1e-3


def test_add_rms_norm_oracle_is_rms_norm():
    rng = np.random.default_rng(4)
    T, C = 3, 512
    x = O.f32_to_bf16(rng.standard_normal((T, C)).astype(np.float32))
    r = O.f32_to_bf16(rng.standard_normal((T, C)).astype(np.float32))
    w = O.f32_to_bf16((1 + 0.1 * rng.standard_normal(C)).astype(np.float32))
    res, rows, sums = O.add_rms_norm(x, r, w, 1e-6)
    v = O.bf16_to_f32(x).astype(np.float64) + O.bf16_to_f32(r).astype(np.float64)
    want = O.bf16_to_f32(O.f32_to_bf16(v.astype(np.float32))).astype(np.float64)
    want = want / np.sqrt((v ** 2).mean(axis=1, keepdims=True) + 1e-6) * O.bf16_to_f32(w).astype(np.float64)
    got = O.bf16_to_f32(rows[:T]).astype(np.float64)
    assert np.abs(got - want).max() <= 2 ** -7 * np.abs(want).max()
    assert not rows[T:].any() and not sums[:, T:].any()
    assert np.array_equal(sums, O.presum_sums(rows))
