"""numpy/ctypes front end of the CPU oracle (oracle/q4_oracle.c).

TEST INFRASTRUCTURE ONLY.  This module is the checker the CUDA path is compared
against; only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline and
reference legs import it.  The product library never loads it.

Parity status: partially pinned -- see q4_oracle.h.  ``ref_pins()`` returns the
reference's own compiled helpers (oracle/_ref/libq4ref.so) when they were built
here; they travel to the GPU box with the rest of the tree, but nothing on the
box rebuilds them.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from ctypes import POINTER, c_double, c_float, c_int, c_size_t, c_uint16, c_uint32, c_uint64, c_void_p

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = os.path.join(_HERE, "libq4oracle.so")
_REF = os.path.join(_HERE, "_ref", "libq4ref.so")
_lib = None
_ref = None

SB_BF16 = 0
SB_F16 = 1


def reference_root():
    """The reference checkout whose headers the pins compile: $REF_ROOT, else
    BASELINE.json's reference_path; None when neither names a directory (the
    GPU box has no reference)."""
    root = os.environ.get("REF_ROOT")
    if not root:
        try:
            import json
            with open(os.path.join(_HERE, "..", "BASELINE.json")) as f:
                root = json.load(f).get("reference_path")
        except (OSError, ValueError):
            root = None
    return root if root and os.path.isdir(root) else None


def build(force: bool = False) -> None:
    """Compile the oracle (and the reference pins when the reference exists)."""
    if force or not os.path.exists(_LIB):
        subprocess.check_call(["make", "-s", "-C", _HERE, "oracle"])
    root = reference_root()
    if root and (force or not os.path.exists(_REF)):
        subprocess.check_call(["make", "-s", "-C", _HERE, "ref", "REF_ROOT=" + root])


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB):
            build()
        _lib = ctypes.CDLL(_LIB)
        _declare(_lib)
    return _lib


def ref_pins():
    """The reference's own helpers compiled from its sources, or None."""
    global _ref
    if _ref is None and os.path.exists(_REF):
        r = ctypes.CDLL(_REF)
        r.ref_float_to_bf16.restype = c_uint16
        r.ref_float_to_bf16.argtypes = [c_float]
        r.ref_bf16_to_float.restype = c_float
        r.ref_bf16_to_float.argtypes = [c_uint16]
        r.ref_ulp_bf16.restype = c_float
        r.ref_ulp_bf16.argtypes = [c_float]
        r.ref_silu.restype = c_float
        r.ref_silu.argtypes = [c_float]
        r.ref_reassociation_slack.restype = c_float
        r.ref_reassociation_slack.argtypes = [c_uint32, c_float]
        r.ref_split_tolerance.restype = c_float
        r.ref_split_tolerance.argtypes = [c_int, c_float, c_float, c_float, c_float, c_float]
        r.ref_moe_maximum_tiles.restype = c_uint32
        r.ref_moe_maximum_tiles.argtypes = [c_uint32] * 6
        r.ref_moe_tile_descriptor_bytes.restype = c_uint32
        r.ref_moe_tile_descriptor_bytes.argtypes = []
        _ref = r
    return _ref


def _p(a: np.ndarray):
    return a.ctypes.data_as(c_void_p)


def _declare(L) -> None:
    v = c_void_p
    sig = {
        "q4o_f32_to_bf16": (c_uint16, [c_float]),
        "q4o_bf16_to_f32": (c_float, [c_uint16]),
        "q4o_f32_to_f16": (c_uint16, [c_float]),
        "q4o_f16_to_f32": (c_float, [c_uint16]),
        "q4o_f32_to_bf16_n": (None, [v, v, c_size_t]),
        "q4o_bf16_to_f32_n": (None, [v, v, c_size_t]),
        "q4o_lcg": (c_uint64, [POINTER(c_uint64)]),
        "q4o_rand_qlin": (None, [c_int, c_int, c_uint64, v, v]),
        "q4o_rand_x": (None, [c_int, c_uint64, v]),
        "q4o_rand_pf_case": (None, [c_int, c_int, c_int, POINTER(c_uint64), v, v, v]),
        "q4o_quantize": (None, [v, c_int, c_int, c_int, c_int, v, v, c_int]),
        "q4o_mlx_to_tiled": (None, [v, v, c_int, c_int, v, v]),
        "q4o_tiled_to_mlx": (None, [v, v, c_int, c_int, v, v]),
        "q4o_slab_bytes": (c_size_t, [c_int, c_int]),
        "q4o_mlx_to_slab": (None, [v, v, c_int, c_int, v]),
        "q4o_slab_to_mlx": (None, [v, c_int, c_int, v, v]),
        "q4o_frag_qw_bytes": (c_size_t, [c_int, c_int, c_int]),
        "q4o_frag_sb_bytes": (c_size_t, [c_int, c_int, c_int]),
        "q4o_mlx_to_frag": (None, [v, v, c_int, c_int, c_int, v, v]),
        "q4o_frag_to_mlx": (None, [v, v, c_int, c_int, c_int, v, v]),
        "q4o_linear_group": (None, [v, v, c_int, c_int, c_int, v, c_int, v, c_int]),
        "q4o_linear_dequant": (None, [v, v, c_int, c_int, c_int, v, c_int, v, c_int]),
        "q4o_dequant_bf16": (None, [v, v, c_int, c_int, c_int, v]),
        "q4o_silu_mul_bf16": (c_uint16, [c_float, c_float]),
        "q4o_gate_up": (None, [v, v, c_int, c_int, c_int, c_int, c_int, v, c_int, v, c_int]),
        "q4o_moe_select": (None, [v, c_int, c_int, c_int, v, v]),
        "q4o_moe_max_tiles": (c_uint32, [c_int, c_int, c_int, c_int]),
        "q4o_moe_group": (c_int, [v, c_int, c_int, c_int, c_int, c_int, v, v, v]),
        "q4o_moe_forward": (None, [v, v, c_int, c_int, c_int, c_int, c_int, v, v, v, v, v, v,
                                   c_int, v, v, v, c_int]),
        "q4o_moe_forward_shared": (None, [v, v, c_int, c_int, c_int, c_int, c_int, v, v, v, v, v, v,
                                          v, v, v, v, c_int, v, v, v, c_int]),
        "q4o_moe_scores_q8": (None, [v, c_int, c_int, v, v, v, c_int, v, c_int]),
        "q4o_moe_shared_gate": (None, [v, c_int, c_int, v, v, v, v, v]),
        "q4o_moe_group_shared": (c_int, [v, c_int, c_int, c_int, c_int, c_int, c_int, v, v, v]),
        "q4o_splash_moe_fixture": (None, [c_int, c_int, c_int, c_int, c_uint64, v, v, v, v, v, v, v, v]),
        "q4o_cpu_linear": (c_int, [v, v, c_int, c_int, c_int, v, c_int, v, c_int]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args


def threads() -> int:
    return max(1, len(os.sched_getaffinity(0)))


# ---- conversions --------------------------------------------------------------

def f32_to_bf16(a) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty(a.shape, dtype=np.uint16)
    lib().q4o_f32_to_bf16_n(_p(a), _p(out), a.size)
    return out


def bf16_to_f32(a) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.uint16)
    out = np.empty(a.shape, dtype=np.float32)
    lib().q4o_bf16_to_f32_n(_p(a), _p(out), a.size)
    return out


def bf16_round(a) -> np.ndarray:
    return bf16_to_f32(f32_to_bf16(a))


def sb_to_f32(a, sb_dtype: int) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.uint16)
    if sb_dtype == SB_F16:
        return a.view(np.float16).astype(np.float32)
    return bf16_to_f32(a)


# ---- generators -----------------------------------------------------------------

def rand_qlin(out: int, inp: int, seed: int):
    """The reference tests' random packed weight (qwen35.rs:6896-6915)."""
    wq = np.empty((out, inp // 8), dtype=np.uint32)
    sb = np.empty((out, 2 * (inp // 64)), dtype=np.uint16)
    lib().q4o_rand_qlin(out, inp, seed, _p(wq), _p(sb))
    return wq, sb


def rand_x(inp: int, seed: int) -> np.ndarray:
    """The reference tests' random activation as bf16 bits (qwen35.rs:6917-6923)."""
    x = np.empty(inp, dtype=np.uint16)
    lib().q4o_rand_x(inp, seed, _p(x))
    return x


class PfStream:
    """The prefill tests' single LCG state (quant_kernel.rs:5446)."""

    def __init__(self, seed: int = 0x5EED):
        self.state = c_uint64(seed)

    def case(self, total_out: int, inp: int, m: int):
        """(tiled words, planar sb, x bf16 [m][inp]) for the next case."""
        ng, padded = inp // 64, (total_out + 255) // 256 * 256
        tw = np.empty(padded * ng * 8, dtype=np.uint32)
        tsb = np.empty(2 * padded * ng, dtype=np.uint16)
        x = np.empty((m, inp), dtype=np.uint16)
        lib().q4o_rand_pf_case(total_out, inp, m, ctypes.byref(self.state), _p(tw), _p(tsb), _p(x))
        return tw, tsb, x


# (out per stream, inp, gate_up, m) of pf_vec_matches_legacy_bitwise
PF_CASES = [(640, 512, False, 130), (720, 256, False, 257), (384, 1024, False, 64),
            (1280, 512, False, 200), (512, 512, True, 161), (256, 1024, True, 96)]
# (out, ng) of qmvt_plain_matches_scalar and (half, ng) of qmvt_gate_up_matches_scalar
QMVT_PLAIN_CASES = [(520, 7), (256, 80), (1000, 17), (72, 96)]
QMVT_GATE_UP_CASES = [(256, 7), (264, 80), (512, 17), (1000, 6)]


def quantize(w: np.ndarray, sb_dtype: int = SB_F16, gs: int = 64):
    w = np.ascontiguousarray(w, dtype=np.float32)
    out, inp = w.shape
    wq = np.empty((out, inp // 8), dtype=np.uint32)
    sb = np.empty((out, 2 * (inp // gs)), dtype=np.uint16)
    lib().q4o_quantize(_p(w), out, inp, gs, sb_dtype, _p(wq), _p(sb), threads())
    return wq, sb


def synthetic_weight(out: int, inp: int, seed: int, sb_dtype: int = SB_F16, std: float = 0.02):
    """W ~ N(0, std) quantised by this repository's min/max group-64 quantiser."""
    rng = np.random.default_rng(seed)
    w = rng.standard_normal((out, inp), dtype=np.float32) * np.float32(std)
    return quantize(w, sb_dtype)


# ---- layouts --------------------------------------------------------------------

def mlx_to_tiled(wq, sb):
    out, inp = wq.shape[0], wq.shape[1] * 8
    ng, tiles = inp // 64, (out + 255) // 256
    tw = np.empty(tiles * ng * 2048, dtype=np.uint32)
    tsb = np.empty(2 * tiles * 256 * ng, dtype=np.uint16)
    lib().q4o_mlx_to_tiled(_p(np.ascontiguousarray(wq)), _p(np.ascontiguousarray(sb)), out, inp, _p(tw), _p(tsb))
    return tw, tsb


def tiled_to_mlx(tw, tsb, out: int, inp: int):
    wq = np.empty((out, inp // 8), dtype=np.uint32)
    sb = np.empty((out, 2 * (inp // 64)), dtype=np.uint16)
    lib().q4o_tiled_to_mlx(_p(tw), _p(tsb), out, inp, _p(wq), _p(sb))
    return wq, sb


def mlx_to_slab(wq, sb) -> np.ndarray:
    out, inp = wq.shape[0], wq.shape[1] * 8
    slab = np.empty(lib().q4o_slab_bytes(out, inp), dtype=np.uint8)
    lib().q4o_mlx_to_slab(_p(np.ascontiguousarray(wq)), _p(np.ascontiguousarray(sb)), out, inp, _p(slab))
    return slab


def slab_to_mlx(slab, out: int, inp: int):
    wq = np.empty((out, inp // 8), dtype=np.uint32)
    sb = np.empty((out, 2 * (inp // 64)), dtype=np.uint16)
    lib().q4o_slab_to_mlx(_p(slab), out, inp, _p(wq), _p(sb))
    return wq, sb


# tiles per slab of the library's layout (thq4_common.cuh)
SLAB_TILES = 8


def mlx_to_frag(wq, sb, ts: int = SLAB_TILES):
    """The B200 frag layout (nibbles as u32 words, quads as u16)."""
    out, inp = wq.shape[0], wq.shape[1] * 8
    fq = np.empty(lib().q4o_frag_qw_bytes(out, inp, ts) // 4, dtype=np.uint32)
    fsb = np.empty(lib().q4o_frag_sb_bytes(out, inp, ts) // 2, dtype=np.uint16)
    lib().q4o_mlx_to_frag(_p(np.ascontiguousarray(wq)), _p(np.ascontiguousarray(sb)), out, inp, ts, _p(fq), _p(fsb))
    return fq, fsb


def frag_to_mlx(fq, fsb, out: int, inp: int, ts: int = SLAB_TILES):
    wq = np.empty((out, inp // 8), dtype=np.uint32)
    sb = np.empty((out, 2 * (inp // 64)), dtype=np.uint16)
    lib().q4o_frag_to_mlx(_p(fq), _p(fsb), out, inp, ts, _p(wq), _p(sb))
    return wq, sb


# ---- products -------------------------------------------------------------------

def _x2d(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    return x.reshape(1, -1) if x.ndim == 1 else x


def linear_group(wq, sb, sb_dtype: int, x) -> np.ndarray:
    """Per-group kernel semantics in fp64: y [m][out] (unrounded)."""
    x = _x2d(x)
    out, inp = wq.shape[0], wq.shape[1] * 8
    y = np.empty((x.shape[0], out), dtype=np.float64)
    lib().q4o_linear_group(_p(np.ascontiguousarray(wq)), _p(np.ascontiguousarray(sb)), sb_dtype, out, inp,
                           _p(x), x.shape[0], _p(y), threads())
    return y


def linear_dequant(wq, sb, sb_dtype: int, x) -> np.ndarray:
    """Reference CPU path: bf16-dequantised weight, fp64 dot: y [m][out]."""
    x = _x2d(x)
    out, inp = wq.shape[0], wq.shape[1] * 8
    y = np.empty((x.shape[0], out), dtype=np.float64)
    lib().q4o_linear_dequant(_p(np.ascontiguousarray(wq)), _p(np.ascontiguousarray(sb)), sb_dtype, out, inp,
                             _p(x), x.shape[0], _p(y), threads())
    return y


def dequant_bf16(wq, sb, sb_dtype: int) -> np.ndarray:
    out, inp = wq.shape[0], wq.shape[1] * 8
    w = np.empty((out, inp), dtype=np.uint16)
    lib().q4o_dequant_bf16(_p(np.ascontiguousarray(wq)), _p(np.ascontiguousarray(sb)), sb_dtype, out, inp, _p(w))
    return w


def silu_mul_bf16(gate, up) -> np.ndarray:
    gate = np.asarray(gate, dtype=np.float32).ravel()
    up = np.asarray(up, dtype=np.float32).ravel()
    f = lib().q4o_silu_mul_bf16
    return np.array([f(float(g), float(u)) for g, u in zip(gate, up)], dtype=np.uint16)


def gate_up(wq, sb, sb_dtype: int, up_row: int, half: int, x) -> np.ndarray:
    """Fused [gate | up] projection with the SwiGLU epilogue -> bf16 [m][half]."""
    x = _x2d(x)
    out, inp = wq.shape[0], wq.shape[1] * 8
    y = np.empty((x.shape[0], half), dtype=np.uint16)
    lib().q4o_gate_up(_p(np.ascontiguousarray(wq)), _p(np.ascontiguousarray(sb)), sb_dtype, out, inp,
                      up_row, half, _p(x), x.shape[0], _p(y), threads())
    return y


# ---- MoE ------------------------------------------------------------------------

def moe_select(logits_bf16, k: int):
    logits_bf16 = np.ascontiguousarray(logits_bf16, dtype=np.uint16)
    T, E = logits_bf16.shape
    ids = np.empty((T, k), dtype=np.uint32)
    w = np.empty((T, k), dtype=np.uint16)
    lib().q4o_moe_select(_p(logits_bf16), T, E, k, _p(ids), _p(w))
    return ids, w


def moe_max_tiles(T: int, E: int, k: int, tile_rows: int) -> int:
    return int(lib().q4o_moe_max_tiles(T, E, k, tile_rows))


def moe_group(ids, E: int, tile_rows: int, max_tiles: int | None = None):
    ids = np.ascontiguousarray(ids, dtype=np.uint32)
    T, k = ids.shape
    if max_tiles is None:
        max_tiles = moe_max_tiles(T, E, k, tile_rows)
    tiles = np.empty((max_tiles, 2), dtype=np.uint32)
    grouped = np.empty(max_tiles * tile_rows, dtype=np.uint32)
    route_rows = np.empty(T * k, dtype=np.uint32)
    n = lib().q4o_moe_group(_p(ids), T, k, E, tile_rows, max_tiles, _p(tiles), _p(grouped), _p(route_rows))
    if n < 0:
        raise ValueError("max_tiles too small")
    return tiles, n, grouped, route_rows


def moe_forward(x_bf16, residual_bf16, ids, weights_bf16, gu_wq, gu_sb, dn_wq, dn_sb, sb_dtype: int,
                I: int, want_h: bool = False, shared=None):
    """One MoE layer on MLX row-major experts; returns (y, h, d) as bf16.
    ``shared`` = (gu_wq, gu_sb, dn_wq, dn_sb) of the shared expert (one
    expert, same shapes), which the id E selects in ``ids``."""
    x_bf16 = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    T, H = x_bf16.shape
    k = ids.shape[1]
    E = gu_wq.shape[0]
    y = np.empty((T, H), dtype=np.uint16)
    d = np.empty((T * k, H), dtype=np.uint16)
    h = np.empty((T * k, I), dtype=np.uint16) if want_h else None
    res = None if residual_bf16 is None else np.ascontiguousarray(residual_bf16, dtype=np.uint16)
    sh = [None] * 4 if shared is None else [_p(np.ascontiguousarray(a)) for a in shared]
    keep = shared
    lib().q4o_moe_forward_shared(_p(x_bf16), None if res is None else _p(res), T, H, I, E, k,
                                 _p(np.ascontiguousarray(ids, dtype=np.uint32)),
                                 _p(np.ascontiguousarray(weights_bf16, dtype=np.uint16)),
                                 _p(np.ascontiguousarray(gu_wq)), _p(np.ascontiguousarray(gu_sb)),
                                 _p(np.ascontiguousarray(dn_wq)), _p(np.ascontiguousarray(dn_sb)),
                                 sh[0], sh[1], sh[2], sh[3], sb_dtype,
                                 None if h is None else _p(h), _p(d), _p(y), threads())
    del keep
    return y, h, d


# ---- the Q8 router and the shared expert (moe.metal:1-361) ---------------------

Q8_STORAGE_N = 256


def moe_scores_q8(x_bf16, q, scales, biases, ncols: int):
    """Router scores bf16 [T][ncols] of a Q8 projection in StorageN = 256
    order (q u8 [H/64 * 256 * 64], scales and biases bf16 [H/64 * 256])."""
    x_bf16 = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    T, H = x_bf16.shape
    out = np.empty((T, ncols), dtype=np.uint16)
    lib().q4o_moe_scores_q8(_p(x_bf16), T, H, _p(np.ascontiguousarray(q, dtype=np.uint8)),
                            _p(np.ascontiguousarray(scales, dtype=np.uint16)),
                            _p(np.ascontiguousarray(biases, dtype=np.uint16)), ncols, _p(out), threads())
    return out


def moe_shared_gate(x_bf16, q, scales, biases):
    """The shared expert's routing weights bf16 [T] and gate logits f32 [T]."""
    x_bf16 = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    T, H = x_bf16.shape
    w = np.empty(T, dtype=np.uint16)
    logit = np.empty(T, dtype=np.float32)
    lib().q4o_moe_shared_gate(_p(x_bf16), T, H, _p(np.ascontiguousarray(q, dtype=np.uint8)),
                              _p(np.ascontiguousarray(scales, dtype=np.uint16)),
                              _p(np.ascontiguousarray(biases, dtype=np.uint16)), _p(w), _p(logit))
    return w, logit


def moe_route_q8(x_bf16, E: int, k: int, router, shared_gate=None):
    """The whole routing of Splash's MoE::add: scores from the Q8 router
    (a (q, scales, biases) triple), top k of the E experts, and with a shared
    expert gate a last slot per token holding expert E and its sigmoid weight.
    Returns ids [T][rpr] u32, weights [T][rpr] bf16, scores bf16 [T][E]."""
    scores = moe_scores_q8(x_bf16, *router, E)
    ids, w = moe_select(scores, k)
    if shared_gate is not None:
        sw, _ = moe_shared_gate(x_bf16, *shared_gate)
        ids = np.concatenate([ids, np.full((ids.shape[0], 1), E, dtype=np.uint32)], axis=1)
        w = np.concatenate([w, sw[:, None]], axis=1)
    return ids, w, scores


def moe_max_tiles_shared(T: int, E: int, k: int, tile_rows: int, shared: bool) -> int:
    """moeMaximumTiles (MoE.hpp:72-77): the routed bound plus the shared tiles."""
    return moe_max_tiles(T, E, k, tile_rows) + ((T + tile_rows - 1) // tile_rows if shared else 0)


def moe_group_shared(ids, k: int, E: int, tile_rows: int, max_tiles: int | None = None):
    """Grouping of ids [T][rpr] whose slots past k are the shared expert's."""
    ids = np.ascontiguousarray(ids, dtype=np.uint32)
    T, rpr = ids.shape
    if max_tiles is None:
        max_tiles = moe_max_tiles_shared(T, E, k, tile_rows, rpr > k)
    tiles = np.empty((max_tiles, 2), dtype=np.uint32)
    grouped = np.empty(max_tiles * tile_rows, dtype=np.uint32)
    route_rows = np.empty(T * rpr, dtype=np.uint32)
    n = lib().q4o_moe_group_shared(_p(ids), T, k, rpr, E, tile_rows, max_tiles, _p(tiles), _p(grouped),
                                   _p(route_rows))
    if n < 0:
        raise ValueError("max_tiles too small")
    return tiles, n, grouped, route_rows


SPLASH_MOE_SEED = 0x0E5


def splash_moe_fixture(H: int, I: int, E: int, rows: int, seed: int = SPLASH_MOE_SEED):
    """The expert slabs and rows of moe_metal_test.mm's makeFixture: a dict of
    Splash slab arrays u8 ``gate``/``up``/``down`` [E, bytes] and
    ``shared_gate``/``shared_up``/``shared_down`` [1, bytes], ``x`` and
    ``residual`` bf16 [rows][H]."""
    gs, ds = lib().q4o_slab_bytes(I, H), lib().q4o_slab_bytes(H, I)
    f = {"gate": np.empty((E, gs), np.uint8), "up": np.empty((E, gs), np.uint8), "down": np.empty((E, ds), np.uint8),
         "shared_gate": np.empty((1, gs), np.uint8), "shared_up": np.empty((1, gs), np.uint8),
         "shared_down": np.empty((1, ds), np.uint8), "x": np.empty((rows, H), np.uint16),
         "residual": np.empty((rows, H), np.uint16)}
    lib().q4o_splash_moe_fixture(H, I, E, rows, seed, *[_p(f[n]) for n in ("gate", "up", "down", "shared_gate",
                                                                             "shared_up", "shared_down", "x",
                                                                             "residual")])
    return f


# ---- CPU baseline ---------------------------------------------------------------

def cpu_linear(wq, sb, sb_dtype: int, x, nthreads: int | None = None):
    """The timed CPU baseline (f32 accumulate, threaded).  Returns (y, threads)."""
    x = _x2d(x)
    out, inp = wq.shape[0], wq.shape[1] * 8
    y = np.empty((x.shape[0], out), dtype=np.float32)
    n = lib().q4o_cpu_linear(_p(np.ascontiguousarray(wq)), _p(np.ascontiguousarray(sb)), sb_dtype, out, inp,
                             _p(x), x.shape[0], _p(y), nthreads or threads())
    if n < 0:
        raise ValueError("unsupported shape for the CPU baseline")
    return y, n


# ---- presum blocks (engine/src/quant_kernel.rs:265-318, 1864-1884;
#      engine/src/gdn_kernel.rs:1851-1866, 1919-1962) --------------------------

def _lane_butterfly(v: np.ndarray) -> np.ndarray:
    """32 lanes on the last axis combined by xor butterfly (partners 16, 8, 4,
    2, 1), each step an f32 add; returns lane 0's value."""
    lanes = np.arange(32)
    v = np.asarray(v, dtype=np.float32)
    for o in (16, 8, 4, 2, 1):
        v = (v + v[..., lanes ^ o]).astype(np.float32)
    return v[..., 0]


def presum_sums(rows_bf16) -> np.ndarray:
    """f32 sums [in/64][8] of a presum block's 8 bf16 rows [8][in]: lane l of
    group g adds x[64g + l] + x[64g + 32 + l] (q4_store_input_sums,
    quant_kernel.rs:1864-1884), the lanes combine by the butterfly."""
    x = bf16_to_f32(np.asarray(rows_bf16, dtype=np.uint16)).astype(np.float32)
    rows, inp = x.shape
    g = x.reshape(rows, inp // 64, 64)
    v = (g[:, :, :32] + g[:, :, 32:]).astype(np.float32)
    return np.ascontiguousarray(_lane_butterfly(v).T)


def presum_block(x_bf16) -> tuple:
    """Q4AttachSums: (rows [8][in] bf16 with rows >= m zero, sums [in/64][8])."""
    x = np.asarray(x_bf16, dtype=np.uint16)
    m, inp = x.shape
    rows = np.zeros((8, inp), dtype=np.uint16)
    rows[:m] = x
    return rows, presum_sums(rows)


def add_rms_norm(x_bf16, r_bf16, w_bf16, eps: float) -> tuple:
    """AddRmsNorm { sums } (gdn_kernel.rs:1919-1962, per-row form :1964-2004):
    v = x + r in f32, res = bf16(v); lane l accumulates ss += v * v over
    columns l, l + 32, ... in order (f32 multiply, then f32 add), the lanes
    combine by the butterfly; inv = 1 / sqrt(ss / C + eps), each step f32 and
    correctly rounded; nrm = bf16((bf16(v) * inv) * w).  Returns (res [T][C],
    block rows [8][C] with rows >= T zero, sums [C/64][8])."""
    xf = bf16_to_f32(np.asarray(x_bf16, dtype=np.uint16)).astype(np.float32)
    rf = bf16_to_f32(np.asarray(r_bf16, dtype=np.uint16)).astype(np.float32)
    wf = bf16_to_f32(np.asarray(w_bf16, dtype=np.uint16)).astype(np.float32)
    T, C = xf.shape
    v = (xf + rf).astype(np.float32)
    res = f32_to_bf16(v)
    ss = np.zeros((T, 32), dtype=np.float32)
    for j in range(C // 32):
        c = v[:, j * 32:(j + 1) * 32]
        ss = (ss + (c * c).astype(np.float32)).astype(np.float32)
    tot = _lane_butterfly(ss)
    inv = (np.float32(1.0) / np.sqrt((tot / np.float32(C)).astype(np.float32) + np.float32(eps))).astype(np.float32)
    nrm = f32_to_bf16(((bf16_to_f32(res).astype(np.float32) * inv[:, None]).astype(np.float32) * wf).astype(np.float32))
    rows = np.zeros((8, C), dtype=np.uint16)
    rows[:T] = nrm
    return res, rows, presum_sums(rows)
