"""Independent numpy restatement of the oracle's arithmetic, used only to
cross-check oracle/q4_oracle.c.  TEST INFRASTRUCTURE ONLY.

Every function restates the same reference lines as its C counterpart
(q4_oracle.h) but is written array-at-a-time, so the two share no code.
"""
from __future__ import annotations

import numpy as np


def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    return (np.asarray(a, dtype=np.uint32) << 16).view(np.float32)


def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    """Round to nearest even (LinearNumerics.hpp:19-23)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = u + 0x7FFF + ((u >> 16) & 1)
    return ((u >> 16) & 0xFFFF).astype(np.uint16)


def sb_values(sb: np.ndarray, sb_dtype: int) -> np.ndarray:
    sb = np.ascontiguousarray(sb, dtype=np.uint16)
    return sb.view(np.float16).astype(np.float64) if sb_dtype == 1 else bf16_to_f32(sb).astype(np.float64)


def unpack_mlx(wq: np.ndarray) -> np.ndarray:
    """u32 [out][in/8] -> nibbles [out][in], element 8w+e = bits 4e.. of word w
    (qwen35.rs:126-128)."""
    shifts = (np.arange(8, dtype=np.uint32) * 4)[None, None, :]
    q = (np.asarray(wq, dtype=np.uint32)[:, :, None] >> shifts) & 0xF
    return q.reshape(wq.shape[0], -1).astype(np.uint8)


def pack_mlx(q: np.ndarray) -> np.ndarray:
    out, inp = q.shape
    q = q.reshape(out, inp // 8, 8).astype(np.uint32)
    return np.bitwise_or.reduce(q << (np.arange(8, dtype=np.uint32) * 4), axis=2).astype(np.uint32)


def linear_group(wq, sb, sb_dtype: int, x: np.ndarray) -> np.ndarray:
    """acc += s * sum(q*x) + b * sum(x) per group (quant_kernel.rs:1994-2001)."""
    x = np.atleast_2d(np.asarray(x, dtype=np.float64))
    q = unpack_mlx(wq).astype(np.float64)
    out, inp = q.shape
    ng = inp // 64
    s = sb_values(sb, sb_dtype)
    sc, bi = s[:, :ng], s[:, ng:]
    dots = np.einsum("ngk,mgk->mng", q.reshape(out, ng, 64), x.reshape(-1, ng, 64))
    sums = x.reshape(-1, ng, 64).sum(axis=2)  # [m][ng]
    return (dots * sc[None]).sum(axis=2) + sums @ bi.T


def frag_from_mlx(wq, sb, out: int, inp: int, ts: int = 8):
    """The frag layout (thq4_common.cuh), built with index arithmetic."""
    q = unpack_mlx(wq)
    nb, ng = (out + 16 * ts - 1) // (16 * ts), inp // 64
    qp = np.zeros((nb * 16 * ts, inp), dtype=np.uint32)
    qp[:out] = q
    lane = np.arange(32)
    r, c = lane // 4, lane % 4
    fq = np.zeros((nb, ng, ts, 32, 4), dtype=np.uint32)
    for t in range(ts):
        for j in range(4):
            word = np.zeros((nb, ng, 32), dtype=np.uint32)
            for i in range(8):
                rows = (np.arange(nb)[:, None] * ts + t) * 16 + (r + 8 * ((i >> 1) & 1))[None, :]
                kk = np.arange(ng)[:, None] * 64 + (32 * (j >> 1) + 8 * (j & 1) + 16 * (i & 1) + 2 * c + (i >> 2))[None, :]
                vals = qp[rows[:, None, :], kk[None, :, :]]
                word |= vals << np.uint32(4 * i)
            fq[:, :, t, :, j] = word
    sbp = np.zeros((nb * 16 * ts, 2 * ng), dtype=np.uint16)
    sbp[:out] = sb
    fsb = np.zeros((nb, ng, ts, 8, 4), dtype=np.uint16)
    for t in range(ts):
        for rr in range(8):
            for half in range(2):
                rows = (np.arange(nb) * ts + t) * 16 + rr + 8 * half
                fsb[:, :, t, rr, 2 * half] = sbp[rows, :ng]
                fsb[:, :, t, rr, 2 * half + 1] = sbp[rows, ng:]
    return fq.reshape(-1), fsb.reshape(-1)


def tiled_from_mlx(wq, sb, out: int, inp: int):
    """QLin::tiled (qwen35.rs:629-697)."""
    ng, tiles = inp // 64, (out + 255) // 256
    padded = tiles * 256
    w = np.zeros((padded, ng, 8), dtype=np.uint32)
    w[:out] = np.asarray(wq).reshape(out, ng, 8)
    tw = w.reshape(tiles, 256, ng, 8).transpose(0, 2, 1, 3).reshape(-1)
    s = np.zeros((padded, 2 * ng), dtype=np.uint16)
    s[:out] = sb
    sc = s[:, :ng].reshape(tiles, 256, ng).transpose(0, 2, 1).reshape(-1)
    bi = s[:, ng:].reshape(tiles, 256, ng).transpose(0, 2, 1).reshape(-1)
    return tw, np.concatenate([sc, bi])


def moe_select(logits_bf16: np.ndarray, k: int):
    """Stable sort on (-score, id) (moe_metal_test.mm:366-372)."""
    s = bf16_to_f32(logits_bf16)
    T, E = s.shape
    ids = np.empty((T, k), dtype=np.uint32)
    w = np.empty((T, k), dtype=np.uint16)
    for t in range(T):
        order = sorted(range(E), key=lambda e: (-float(s[t, e]), e))[:k]
        ids[t] = order
        top = s[t, order].astype(np.float32)
        ex = np.exp((top - top[0]).astype(np.float32)).astype(np.float32)
        den = np.float32(0)
        for v in ex:
            den = np.float32(den + v)
        w[t] = f32_to_bf16((ex / den).astype(np.float32))
    return ids, w


def moe_group(ids: np.ndarray, E: int, tile_rows: int):
    """Stable counting sort by expert; returns (tiles list, grouped, route_rows)."""
    flat = np.asarray(ids, dtype=np.int64).ravel()
    order = np.argsort(flat, kind="stable")
    counts = np.bincount(flat, minlength=E)
    tiles, grouped, route_rows = [], [], np.empty(flat.size, dtype=np.uint32)
    pos = 0
    for e in range(E):
        routes = order[pos:pos + counts[e]]
        pos += counts[e]
        for t0 in range(0, counts[e], tile_rows):
            chunk = routes[t0:t0 + tile_rows]
            tiles.append((e, len(chunk)))
            for i, r in enumerate(chunk):
                route_rows[r] = len(grouped) + i
            grouped.extend(int(r) for r in chunk)
            grouped.extend([0xFFFFFFFF] * (tile_rows - len(chunk)))
    return tiles, np.array(grouped, dtype=np.uint32), route_rows


# ---- the Q8 router and the shared expert's gate (moe.metal:1-361) -------------

def _fma32(a, b, c):
    """f32 fma of f32 arrays whose product a*b is exact in f64 (it is for the
    router's bf16/u8/f32 operands); the f64 sum then rounds once to f32
    except in the rare double-rounding case."""
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)


def _butterfly32(v: np.ndarray) -> np.ndarray:
    """Xor-butterfly sum over the last axis (32 lanes), partners 16 .. 1."""
    for o in (16, 8, 4, 2, 1):
        v = (v + v[..., np.arange(32) ^ o]).astype(np.float32)
    return v[..., 0]


def moe_scores_q8(x_bf16, q, scales, biases, ncols: int) -> np.ndarray:
    """Router scores bf16 [T][ncols], array at a time over (token, column)."""
    x = bf16_to_f32(np.asarray(x_bf16, dtype=np.uint16))
    T, H = x.shape
    G = H // 64
    pairs = (x.reshape(T, G, 64)[:, :, :32] + x.reshape(T, G, 64)[:, :, 32:]).astype(np.float32)
    sums = _butterfly32(pairs)  # [T][G]
    qv = np.asarray(q, dtype=np.uint8).reshape(G, 256, 64)[:, :ncols, :].astype(np.float32)
    sc = bf16_to_f32(np.asarray(scales, dtype=np.uint16).reshape(G, 256)[:, :ncols])
    bi = bf16_to_f32(np.asarray(biases, dtype=np.uint16).reshape(G, 256)[:, :ncols])
    total = np.zeros((T, ncols), np.float32)
    for s in range(8):
        sl = np.zeros((T, ncols), np.float32)
        for g in range(s * G // 8, (s + 1) * G // 8):
            dot = np.zeros((T, ncols), np.float32)
            for j in range(64):
                dot = (dot + x[:, 64 * g + j, None] * qv[g, None, :, j]).astype(np.float32)
            c = (sums[:, g, None] * bi[g][None, :]).astype(np.float32)
            sl = (sl + _fma32(dot, np.broadcast_to(sc[g], dot.shape), c)).astype(np.float32)
        total = (total + sl).astype(np.float32)
    return f32_to_bf16(total)


def moe_shared_gate(x_bf16, q, scales, biases):
    """(weights bf16 [T], logits f32 [T]) of the shared expert's scalar gate."""
    x = bf16_to_f32(np.asarray(x_bf16, dtype=np.uint16))
    T, H = x.shape
    G = H // 64
    qv = np.asarray(q, dtype=np.uint8).reshape(G, 256, 64)[:, 0, :].astype(np.float32).reshape(H)
    sc = np.repeat(bf16_to_f32(np.asarray(scales, dtype=np.uint16).reshape(G, 256)[:, 0]), 64)
    bi = np.repeat(bf16_to_f32(np.asarray(biases, dtype=np.uint16).reshape(G, 256)[:, 0]), 64)
    deq = _fma32(qv, sc, bi)
    acc = np.zeros((T, 256), np.float32)
    for base in range(0, H, 256):
        n = min(256, H - base)
        acc[:, :n] = _fma32(x[:, base:base + n], np.broadcast_to(deq[base:base + n], (T, n)), acc[:, :n])
    warps = _butterfly32(acc.reshape(T, 8, 32))  # [T][8]
    total = np.zeros(T, np.float32)
    for w in range(8):
        total = (total + warps[:, w]).astype(np.float32)
    return f32_to_bf16((np.float32(1) / (np.float32(1) + np.exp(-total))).astype(np.float32)), total


def moe_group_shared(ids: np.ndarray, k: int, E: int, tile_rows: int):
    """Grouping with a shared slot last in each token's routes: the routed
    slots sorted stably by expert, then the shared routes in token order as
    expert E.  Returns (tiles list, grouped, route_rows)."""
    ids = np.asarray(ids, dtype=np.int64)
    T, rpr = ids.shape
    routed = [(int(ids[t, s]), t * rpr + s) for t in range(T) for s in range(min(k, rpr))]
    tiles, grouped = [], []
    route_rows = np.full(T * rpr, 0xFFFFFFFF, dtype=np.uint32)
    for e in range(E):
        mine = [r for (ee, r) in routed if ee == e]  # routes ascend: stable
        for t0 in range(0, len(mine), tile_rows):
            chunk = mine[t0:t0 + tile_rows]
            tiles.append((e, len(chunk)))
            for i, r in enumerate(chunk):
                route_rows[r] = len(grouped) + i
            grouped.extend(chunk)
            grouped.extend([0xFFFFFFFF] * (tile_rows - len(chunk)))
    if rpr > k:
        for t0 in range(0, T, tile_rows):
            chunk = [t * rpr + k for t in range(t0, min(T, t0 + tile_rows))]
            tiles.append((E, len(chunk)))
            for i, r in enumerate(chunk):
                route_rows[r] = len(grouped) + i
            grouped.extend(chunk)
            grouped.extend([0xFFFFFFFF] * (tile_rows - len(chunk)))
    return tiles, np.array(grouped, dtype=np.uint32), route_rows
