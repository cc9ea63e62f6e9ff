"""Regenerates tests/golden/golden_oracle.npz from the CPU oracle.

    python tests/golden/make_golden.py

The reference ships no golden vectors for this path (its numerics tests
compare GPU kernel families against each other on seeded LCG inputs), so
these fixtures record the oracle's answers on the reference tests' own LCG
inputs -- qwen35.rs:6893-6926 (qmvt plain / gate-up cases) and
quant_kernel.rs:5428-5466 (prefill cases) -- plus MoE routing on seeded
logits, the reference MoE test's fixture (moe_metal_test.mm:46-300) routed
through its Q8 router and shared gate, and a random Q8 router's scores.  They pin the oracle against drift: tests/test_oracle.py recomputes
every entry and requires bitwise equality.  Large outputs are stored as a
SHA-256 of their bf16 bits plus every 97th value.
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
import q4oracle as O  # noqa: E402


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def compute() -> dict:
    g = {}
    for case, (out, ng) in enumerate(O.QMVT_PLAIN_CASES):
        inp = ng * 64
        wq, sb = O.rand_qlin(out, inp, 11 + case)
        x = O.rand_x(inp, 97 + case)
        y = O.linear_group(wq, sb, O.SB_BF16, O.bf16_to_f32(x))[0]
        g[f"qmvt_plain_{case}"] = O.f32_to_bf16(y.astype(np.float32))
        g[f"qmvt_plain_{case}_inputs_sha"] = np.array(sha(wq) + sha(sb) + sha(x))
    for case, (half, ng) in enumerate(O.QMVT_GATE_UP_CASES):
        inp = ng * 64
        wq, sb = O.rand_qlin(2 * half, inp, 211 + case)
        x = O.rand_x(inp, 307 + case)
        g[f"qmvt_gate_up_{case}"] = O.gate_up(wq, sb, O.SB_BF16, half, half, O.bf16_to_f32(x))[0]
    pf = O.PfStream()
    for case, (out, inp, gu, m) in enumerate(O.PF_CASES):
        total = 2 * out if gu else out
        tw, tsb, x = pf.case(total, inp, m)
        wq, sb = O.tiled_to_mlx(tw, tsb, total, inp)
        xf = O.bf16_to_f32(x)
        if gu:
            y = O.gate_up(wq, sb, O.SB_BF16, out, out, xf)
        else:
            y = O.f32_to_bf16(O.linear_dequant(wq, sb, O.SB_BF16, xf).astype(np.float32))
        g[f"pf_{case}_sha"] = np.array(sha(y))
        g[f"pf_{case}_sample"] = y.ravel()[::97].copy()
    rng = np.random.default_rng(0x40E)
    logits = O.f32_to_bf16(rng.standard_normal((256, 128)).astype(np.float32))
    logits[7, 3] = logits[7, 90]  # an exact tie: lower id ranks first
    ids, w = O.moe_select(logits, 8)
    tiles, n, grouped, route_rows = O.moe_group(ids, 128, 16)
    g["moe_logits"] = logits
    g["moe_ids"] = ids
    g["moe_weights"] = w
    g["moe_tiles"] = tiles[:n]
    g["moe_grouped"] = grouped[: n * 16]
    g["moe_route_rows"] = route_rows

    # the Splash MoE block: the reference MoE test's fixture (moe_metal_test.mm:
    # 46-300, Random(0x0e5)) routed by its column-reading Q8 router and its
    # bias-only shared gate, for each routing distribution; and a random Q8
    # router's scores and a random shared gate on seeded inputs
    H, I, E, K, rows = 1024, 512, 8, 2, 520
    fx = O.splash_moe_fixture(H, I, E, rows)
    for name in ("gate", "up", "down", "shared_gate", "shared_up", "shared_down", "x", "residual"):
        g[f"splash_fixture_{name}_sha"] = np.array(sha(fx[name]))
    G = H // 64
    router_q = np.zeros(G * 256 * 64, np.uint8)
    router_s = np.zeros(G * 256, np.uint16)
    for e in range(E):
        router_q[e * 64 + e] = 1
        router_s[e] = O.f32_to_bf16(np.float32([4.0]))[0]
    zeros_b = np.zeros(G * 256, np.uint16)
    shared_b = zeros_b.copy()
    shared_b[np.arange(G) * 256] = O.f32_to_bf16(np.float32([0.003]))[0]
    for dist in ("dispersed", "concentrated", "skewed"):
        x = fx["x"].copy()
        for row in range(rows):
            first = 0 if (dist == "concentrated" or (dist == "skewed" and row % 8 < 6)) else row % E
            vals = [1.0 if e == first else 0.5 if e == (first + 1) % E else 0.01 * e for e in range(E)]
            x[row, :E] = O.f32_to_bf16(np.float32(vals))
        ids, w, _ = O.moe_route_q8(x, E, K, (router_q, router_s, zeros_b),
                                   (np.zeros_like(router_q), np.zeros_like(router_s), shared_b))
        tiles, n, grouped, route_rows = O.moe_group_shared(ids, K, E, 32)
        g[f"splash_{dist}_ids"] = ids
        g[f"splash_{dist}_weights"] = w
        g[f"splash_{dist}_tables_sha"] = np.array(sha(tiles[:n]) + sha(grouped[:n * 32]) + sha(route_rows))
    rng = np.random.default_rng(0x5E0)
    Hr, Tr = 2048, 64
    rq = rng.integers(0, 256, Hr // 64 * 256 * 64, dtype=np.uint8)
    rs = O.f32_to_bf16(rng.uniform(0.0005, 0.004, Hr // 64 * 256).astype(np.float32))
    rb = O.f32_to_bf16((rng.standard_normal(Hr // 64 * 256) * 0.05).astype(np.float32))
    xr = O.f32_to_bf16(rng.standard_normal((Tr, Hr)).astype(np.float32))
    scores = O.moe_scores_q8(xr, rq, rs, rb, 256)
    g["q8_router_scores_sha"] = np.array(sha(scores))
    g["q8_router_scores_sample"] = scores.ravel()[::97].copy()
    sw, slogit = O.moe_shared_gate(xr, rq, rs, rb)
    g["q8_shared_gate_logits"] = slogit
    return g


if __name__ == "__main__":
    out = os.path.join(HERE, "golden_oracle.npz")
    np.savez_compressed(out, **compute())
    print(out, os.path.getsize(out), "bytes")
