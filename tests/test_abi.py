"""The C-ABI library without a GPU: it loads, exports every symbol
include/thq4.h declares, and its host-side validation rejects bad arguments
before touching the device (the reference bails before encoding,
quant_kernel.rs:2671-2684)."""
import ctypes
import os
import re

import pytest

import thq4
from thq4 import _lib

HEADER = os.path.join(os.path.dirname(__file__), "..", "include", "thq4.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(thq4_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    L = thq4.lib()
    names = declared_functions()
    assert len(names) >= 10
    for n in names:
        assert hasattr(L, n), f"libthq4.so does not export {n}"
        assert n in _lib.SIGNATURES, f"ctypes binding lacks {n}"


def test_version():
    assert thq4.version().startswith("thq4 ") and "sm_100a" in thq4.version()


def test_weight_bytes_match_q4_package_size():
    q, s = ctypes.c_size_t(), ctypes.c_size_t()
    tot = thq4.lib().thq4_weight_bytes(6144, 2048, 64, ctypes.byref(q), ctypes.byref(s))
    assert tot == 6144 * 2048 * 9 // 16 == 7077888  # 0.5625 B/weight, same as q4PackedBytes
    assert q.value == 6144 * 2048 // 2
    # ragged rows pad to the 16-row tile
    assert thq4.lib().thq4_weight_bytes(520, 448, 64, None, None) == 640 * 448 * 9 // 16  # 128-row slabs
    assert thq4.lib().thq4_weight_bytes(64, 100, 64, None, None) == 0


def _w(out=256, inp=1024, gs=64, sbd=thq4.BF16, qw=0x1000, sb=0x2000):
    return _lib.thq4_weight(out, inp, gs, sbd, qw, sb)


@pytest.mark.parametrize("w,msg", [
    (_w(inp=1000), "not a multiple of 64"),
    (_w(gs=32), "group size"),
    (_w(sbd=thq4.F32), "scale dtype"),
    (_w(qw=0x1008), "16-byte aligned"),
    (_w(out=0), "weight has out"),
])
def test_linear_rejects_bad_weights(w, msg):
    st = thq4.lib().thq4_linear(ctypes.byref(w), ctypes.c_void_p(0x3000), thq4.BF16, 1, ctypes.c_void_p(0x4000),
                                thq4.BF16, None, 0, None)
    assert st in (_lib.ERR_INVALID_ARGUMENT, _lib.ERR_UNSUPPORTED)
    assert msg in thq4.last_error()


@pytest.mark.parametrize("x,m,xd,yd,msg", [
    (0x3008, 1, thq4.BF16, thq4.BF16, "16-byte aligned"),
    (0x3000, 0, thq4.BF16, thq4.BF16, "m must be"),
    (0x3000, 1, thq4.F16, thq4.BF16, "x dtype"),
    (0x3000, 1, thq4.BF16, thq4.F16, "y dtype"),
    (0, 1, thq4.BF16, thq4.BF16, "non-NULL"),
])
def test_linear_rejects_bad_io(x, m, xd, yd, msg):
    w = _w()
    st = thq4.lib().thq4_linear(ctypes.byref(w), ctypes.c_void_p(x), xd, m, ctypes.c_void_p(0x4000), yd, None, 0,
                                None)
    assert st == _lib.ERR_INVALID_ARGUMENT
    assert msg in thq4.last_error()


def test_gate_up_rejects_mismatched_halves():
    g, u = _w(out=256), _w(out=264)
    st = thq4.lib().thq4_gate_up(ctypes.byref(g), ctypes.byref(u), ctypes.c_void_p(0x3000), thq4.BF16, 1,
                                 ctypes.c_void_p(0x4000), thq4.BF16, None, 0, None)
    assert st == _lib.ERR_INVALID_ARGUMENT and "differ" in thq4.last_error()


def test_repack_validation():
    L = thq4.lib()
    st = L.thq4_repack(thq4.SRC_SLAB, ctypes.c_void_p(0x1000), None, 520, 256, 64, thq4.BF16, 0, 520,
                       ctypes.c_void_p(0x2000), 1 << 20, ctypes.c_void_p(0x3000), 1 << 20, None)
    assert st == _lib.ERR_INVALID_ARGUMENT and "StorageN=256" in thq4.last_error()
    st = L.thq4_repack(thq4.SRC_MLX, ctypes.c_void_p(0x1000), ctypes.c_void_p(0x1800), 520, 256, 64, thq4.BF16,
                       500, 40, ctypes.c_void_p(0x2000), 1 << 20, ctypes.c_void_p(0x3000), 1 << 20, None)
    assert st == _lib.ERR_INVALID_ARGUMENT and "row range" in thq4.last_error()
    st = L.thq4_repack(thq4.SRC_MLX, ctypes.c_void_p(0x1000), ctypes.c_void_p(0x1800), 520, 256, 64, thq4.BF16,
                       0, 520, ctypes.c_void_p(0x2000), 10, ctypes.c_void_p(0x3000), 10, None)
    assert st == _lib.ERR_INVALID_ARGUMENT and "too small" in thq4.last_error()


def test_linear_requires_workspace():
    w = _w()
    st = thq4.lib().thq4_linear(ctypes.byref(w), ctypes.c_void_p(0x3000), thq4.BF16, 1, ctypes.c_void_p(0x4000),
                                thq4.BF16, None, 0, None)
    assert st == _lib.ERR_WORKSPACE and "zero-filled workspace" in thq4.last_error()
    assert thq4.lib().thq4_linear_workspace_bytes(ctypes.byref(w), 1) > 0


def test_debug_hook_validation():
    assert thq4.lib().thq4_debug_set_gemv(3, 0, 0, 0) == _lib.ERR_INVALID_ARGUMENT
    assert thq4.lib().thq4_debug_set_gemv(1, 0, 0, 0) == _lib.ERR_INVALID_ARGUMENT
    assert thq4.lib().thq4_debug_set_gemv(2, 0, 0, 0) == _lib.ERR_INVALID_ARGUMENT
    assert thq4.lib().thq4_debug_set_gemv(0, 9, 0, 0) == _lib.ERR_INVALID_ARGUMENT
    assert thq4.lib().thq4_debug_set_gemv(0, 0, 0, 1) == _lib.ERR_INVALID_ARGUMENT
    assert thq4.lib().thq4_debug_set_gemv(0, 0, 0, 0) == _lib.OK


def test_error_messages_are_per_thread():
    import threading
    w = _w(inp=1000)
    seen = {}

    def other():
        seen["msg"] = thq4.last_error()

    thq4.lib().thq4_linear(ctypes.byref(w), ctypes.c_void_p(0x3000), thq4.BF16, 1, ctypes.c_void_p(0x4000),
                           thq4.BF16, None, 0, None)
    t = threading.Thread(target=other)
    t.start()
    t.join()
    assert seen["msg"] == "" and "multiple of 64" in thq4.last_error()


# ---- the MoE block and the multi-GPU exchange: host-side validation ---------------

def _experts(E, out, inp, qw=0x10000, sb=0x20000, sbd=thq4.BF16):
    q, s = ctypes.c_size_t(), ctypes.c_size_t()
    thq4.lib().thq4_weight_bytes(out, inp, 64, ctypes.byref(q), ctypes.byref(s))
    return _lib.thq4_experts(E, out, inp, 64, sbd, 0, qw, sb, q.value, s.value)


def _moe_weights(H=1024, I=512, E=8, shared=True):
    w = _lib.thq4_moe_weights()
    w.router = _lib.thq4_q8_weight(256, H, 0x30000, 0x40000, 0x50000)
    w.gate, w.up, w.down = _experts(E, I, H), _experts(E, I, H), _experts(E, H, I)
    if shared:
        w.shared_gate, w.shared_up, w.shared_down = _experts(1, I, H), _experts(1, I, H), _experts(1, H, I)
        w.shared_expert_gate = _lib.thq4_q8_weight(256, H, 0x60000, 0x70000, 0x80000)
    return w


def _moe_add(w, T=16, H=1024, I=512, E=8, k=2, ws_bytes=1 << 30):
    return thq4.lib().thq4_moe_add(ctypes.c_void_p(0x90000), None, T, H, I, E, k, ctypes.byref(w),
                                   ctypes.c_void_p(0xA0000), ctypes.c_void_p(0x100000), ws_bytes, None)


def test_moe_add_tile_bound_pinned_to_reference():
    from test_oracle import ref
    for T, E, k in [(256, 128, 8), (520, 8, 2), (1, 256, 8), (33, 64, 4)]:
        with_shared = thq4.lib().thq4_moe_add_max_tiles(T, E, k, 1)
        without = thq4.lib().thq4_moe_add_max_tiles(T, E, k, 0)
        assert with_shared == without + (T + 31) // 32
        if ref is not None:  # moeMaximumTiles (MoE.hpp:72-77) with 32-row tiles
            assert with_shared == ref.ref_moe_maximum_tiles(T, 2048, E, k, 768, 32)


def test_moe_add_workspace_sizes():
    L = thq4.lib()
    full = L.thq4_moe_add_workspace_bytes(256, 2048, 768, 128, 8, 1)
    assert full > L.thq4_moe_add_workspace_bytes(256, 2048, 768, 128, 8, 0) > 0
    # a shard holds fewer experts' tiles; without the shared expert it needs less still
    half = L.thq4_moe_add_partial_workspace_bytes(256, 2048, 768, 128, 8, 0, 64, 1, 1)
    assert 0 < L.thq4_moe_add_partial_workspace_bytes(256, 2048, 768, 128, 8, 64, 128, 1, 0) < half < full
    assert L.thq4_moe_add_partial_workspace_bytes(256, 2048, 768, 128, 8, 64, 200, 1, 0) == 0
    assert L.thq4_moe_scores_workspace_bytes(256, 128) == 8 * 256 * 128 * 4


@pytest.mark.parametrize("change,msg", [
    (dict(I=320), "execution shape"),
    (dict(H=1000), "execution shape"),
    (dict(E=300), "execution shape"),
    (dict(k=9, E=8), "execution shape"),
])
def test_moe_add_rejects_bad_shapes(change, msg):
    args = dict(T=16, H=1024, I=512, E=8, k=2)
    args.update(change)
    st = _moe_add(_moe_weights(), **args)
    assert st == _lib.ERR_INVALID_ARGUMENT and msg in thq4.last_error()


def test_moe_add_rejects_bad_weights():
    w = _moe_weights()
    w.router.in_ = 512
    assert _moe_add(w) == _lib.ERR_INVALID_ARGUMENT and "router" in thq4.last_error()
    w = _moe_weights()
    w.down = _experts(8, 512, 512)
    assert _moe_add(w) == _lib.ERR_INVALID_ARGUMENT and "down" in thq4.last_error()
    w = _moe_weights()
    w.shared_expert_gate.q = None  # a shared expert without its gate
    assert _moe_add(w) == _lib.ERR_INVALID_ARGUMENT
    w = _moe_weights()
    w.up = _experts(8, 512, 1024, sbd=thq4.F16)
    assert _moe_add(w) == _lib.ERR_INVALID_ARGUMENT and "dtype" in thq4.last_error()
    w = _moe_weights()
    w.router.q = 0x30008  # the router's bytes are read as 16-byte vectors
    assert _moe_add(w) == _lib.ERR_INVALID_ARGUMENT and "16-byte" in thq4.last_error()
    assert _moe_add(_moe_weights(), ws_bytes=1024) == _lib.ERR_WORKSPACE
    assert "smaller than its bound" in thq4.last_error()


def test_peer_exchange_rejects_bad_descriptors():
    L = thq4.lib()
    w = _w(out=256, inp=512)
    g = _lib.thq4_peer_gather()
    g.world, g.rank, g.rows, g.stride = 2, 0, 256, 512
    g.dst = g.flags = g.count = g.arrive = 0x5000
    call = lambda y=0x4000, xd=thq4.BF16: L.thq4_linear_peer(  # noqa: E731
        ctypes.byref(w), None, ctypes.c_void_p(0x3000), xd, 1, ctypes.c_void_p(y) if y else None,
        ctypes.c_void_p(0x100000), 1 << 20, ctypes.byref(g), None)
    g.world = 9
    assert call() == _lib.ERR_INVALID_ARGUMENT and "world" in thq4.last_error()
    g.world, g.out_mode = 2, 4
    assert call() == _lib.ERR_INVALID_ARGUMENT and "out_mode" in thq4.last_error()
    g.out_mode, g.x_parts = 1, 9
    assert call() == _lib.ERR_INVALID_ARGUMENT and "x_parts" in thq4.last_error()
    g.x_parts, g.slot = 0, 100  # reduce slots hold m * stride floats
    assert call(y=0) == _lib.ERR_INVALID_ARGUMENT and "slot" in thq4.last_error()
    g.out_mode, g.x_parts, g.x_slot = 2, 2, 512
    assert call(xd=thq4.BF16) == _lib.ERR_INVALID_ARGUMENT and "partials are f32" in thq4.last_error()
    g.x_slot = 100
    assert call(xd=thq4.F32) == _lib.ERR_INVALID_ARGUMENT and "x_slot" in thq4.last_error()


# ---- the decode/verify planner's policy table (host only) ------------------------
# The reference pins its dispatch tables per decode shape (plain_tile_table,
# qmvt_policy_table, quant_kernel.rs:5914-5973); this is the same check of
# this library's planner for the BASELINE shapes on a 148-SM B200.  Cluster
# capacity depends on how the SMs group into GPCs; the table below stands for
# eight GPCs of 18 SMs (clusters of j: 8 * floor(18 / j)).
GPC_FIT = [0, 0] + [8 * (18 // j) for j in range(2, 9)]


def _plan(out, inp, m=1, x_f32=0, gate_up=0, sms=148, fit=GPC_FIT):
    p = (ctypes.c_int64 * 8)()
    f = (ctypes.c_int * 9)(*fit) if fit is not None else None
    assert thq4.lib().thq4_debug_gemv_plan(out, inp, m, x_f32, gate_up, sms, f, p) == 0, thq4.last_error()
    return tuple(p)[:7]  # planned, CTAs, cluster size, stages, tokens per launch, chunks per slab, groups per chunk


@pytest.mark.parametrize("shape,want", [
    # hidden-5120 decode layer, m = 1
    ((17408, 5120, 1, 0, 1), (1, 136, 1, 2, 1, 10, 8)),  # fused gate/up: one whole slab per CTA, no split
    ((7168, 5120), (1, 112, 2, 5, 1, 10, 8)),  # q/k/v: 56 slabs x clusters of 2
    ((5120, 5120), (1, 120, 3, 5, 1, 10, 8)),  # o: 40 slabs x 3
    ((5120, 17408), (1, 120, 3, 5, 1, 34, 8)),  # down: 40 slabs x 3
    # 6144 x 2048, f32 x and y
    ((6144, 2048, 1, 1, 0), (1, 144, 3, 5, 1, 4, 8)),
    # configs[1] verify: gate/up 2 x 9728 x 2560 (76 slabs: split-K over every SM), down 2560 x 9728
    ((9728, 2560, 8, 0, 1), (1, 148, 1, 2, 8, 5, 8)),
    ((2560, 9728, 4), (1, 120, 6, 5, 4, 19, 8)),  # 20 slabs: clusters of 6
    ((9728, 2560, 8, 1, 1), (1, 148, 1, 2, 4, 5, 8)),  # f32 x: 4 tokens per launch (hi + lo columns)
    # column shards at two and eight GPUs
    ((2560, 5120), (1, 120, 6, 5, 1, 10, 8)),  # o at N = 2: clusters of 7 do not all fit, 6 do
    ((896, 5120), (1, 56, 8, 5, 1, 10, 8)),  # q/k/v at N = 8: 7 slabs; a flat split cannot fill the SMs either,
                                              # so clusters of 8 combine in DSMEM
    ((5120, 640), (1, 80, 2, 5, 1, 2, 8)),    # o at N = 8 (row shard): 40 slabs of 2 chunks, clusters of 2
])
def test_planner_policy_table(shape, want):
    assert _plan(*shape) == want


def test_planner_without_clusters_and_on_fewer_sms():
    # no cluster fits: split-K over every SM
    assert _plan(7168, 5120, fit=None) == (1, 148, 1, 5, 1, 10, 8)
    # a 132-SM part: the 136-slab gate/up no longer fits one slab per SM
    assert _plan(17408, 5120, 1, 0, 1, sms=132)[:3] == (1, 132, 1)


def test_planner_follows_the_testing_hook():
    L = thq4.lib()
    try:
        assert L.thq4_debug_set_gemv(4, 3, 64, 0) == 0
        planned, ctas, cl, stages, _, cps, ch = _plan(5120, 5120)
        assert (planned, ctas, cl, ch, cps) == (1, 64, 1, 4, 20) and stages <= 3
    finally:
        assert L.thq4_debug_set_gemv(0, 0, 0, 0) == 0
    assert _plan(5120, 5120) == (1, 120, 3, 5, 1, 10, 8)
    assert L.thq4_debug_gemv_plan(5120, 100, 1, 0, 0, 148, None, (ctypes.c_int64 * 8)()) == _lib.ERR_INVALID_ARGUMENT


@pytest.mark.parametrize("env,want", [
    ("4,3,64", (1, 64, 1, None, 1, 20, 4)),   # every field taken
    ("8,0,0", (1, 120, 3, 5, 1, 10, 8)),      # zeros leave the policy
    ("5,9,-1", (1, 120, 3, 5, 1, 10, 8)),     # out-of-range fields are ignored one by one
    ("r2s4", (1, 120, 3, 5, 1, 10, 8)),       # not a THQ4_GEMV value: ignored
    ("", (1, 120, 3, 5, 1, 10, 8)),
])
def test_environment_override_is_parsed_once_and_validated(env, want):
    """THQ4_GEMV="chunk,stages,grid,pre" is read once per process (as the
    reference reads its TH_QMVT / TH_Q4_POLICY switches, quant_kernel.rs:
    41-78, 367-432, and rejects values that name no instantiated config)."""
    import json
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    code = (
        "import ctypes, json, sys; sys.path.insert(0, %r); sys.path.insert(0, %r)\n"
        "from test_abi import _plan\n"
        "print(json.dumps(_plan(5120, 5120)))\n" % (os.path.join(here, "..", "token-horizon_b200"), here))
    out = subprocess.run([sys.executable, "-c", code], env=dict(os.environ, THQ4_GEMV=env), capture_output=True,
                         text=True, timeout=120, check=True).stdout
    got = tuple(json.loads(out.strip().splitlines()[-1]))
    assert got[:3] == want[:3] and got[4:] == want[4:]
    assert (got[3] <= 3) if want[3] is None else got[3] == want[3]


@pytest.mark.parametrize("out,inp,m,split", [
    (12288, 4096, 512, True),     # configs[2] M = 512: 192 tiles of 256 tokens fill 1.3 waves -> stream-K
    (12288, 4096, 1024, False),   # 384 tiles, waves 86% full: whole tiles
    (12288, 4096, 2048, False),   # 768 tiles, 86%: whole tiles
    (12288, 4096, 9, False),      # 96 tiles, fewer than the SMs: whole tiles
    (20000, 1024, 300, True),     # 314 tiles (ragged rows and tokens), 71%
    (4608, 2048, 1100, True),     # 180 tiles, 61%
])
def test_prefill_split_plan_and_workspace(out, inp, m, split):
    """Host-only: thq4_linear_workspace_bytes(w, m) is the decode kernel's
    figure unless the prefill splits its k-stages (stream-K), which it does
    when 256-token tiles outnumber the SMs but fill the waves to less than
    80%; the split region is 256-aligned after the decode region: one claim
    word pair and one 128-row x 256-token f32 part per SM (148 here, the
    library's SM count without a device)."""
    w = _w(out=out, inp=inp, sbd=thq4.F16)
    L = thq4.lib()
    base = L.thq4_linear_workspace_bytes(ctypes.byref(w), 1)
    got = L.thq4_linear_workspace_bytes(ctypes.byref(w), m)
    if not split:
        assert got == base
        return
    sms = 148
    r256 = lambda v: (v + 255) // 256 * 256
    assert got == r256(base) + r256(sms * 8) + sms * 256 * 128 * 4


def _pf_plan(out, inp, m, gate_up=0, sms=148):
    p = (ctypes.c_int64 * 5)()
    assert thq4.lib().thq4_debug_prefill_plan(out, inp, m, gate_up, sms, p) == 0, thq4.last_error()
    return tuple(p)


@pytest.mark.parametrize("shape,want", [
    # configs[2] at M = 512: 256-token tiles fill 1.3 waves -> stream-K over 148 CTAs
    ((12288, 4096, 512), (256, 1, 192, 148, None)),
    ((12288, 4096, 1024), (256, 0, 384, 148, 0)),   # waves 86% full: whole 256-token tiles
    ((12288, 4096, 2048), (256, 0, 768, 148, 0)),
    ((12288, 4096, 300), (256, 1, 192, 148, None)), # 2 x 96 tiles fill 65% of two waves: split too
    ((12288, 4096, 40), (192, 0, 96, 96, 0)),       # one token tile: the widest least-cost width
    ((12288, 4096, 512, 1), (128, 0, 384, 148, 0)), # the gate/up form: 128-token tiles, whole
])
def test_prefill_policy_table(shape, want):
    """Host only: the prefill planner's launch shape for the BASELINE prefill
    shape and its neighbours on 148 SMs (as test_planner_policy_table pins
    the decode kernel's)."""
    got = _pf_plan(*shape)
    assert got[:4] == want[:4]
    if want[4] is None:
        assert got[4] > 148 * 256 * 128 * 4  # the parts, after the decode region
    else:
        assert got[4] == want[4]


def test_prefill_plan_rejects_decode_rows():
    assert thq4.lib().thq4_debug_prefill_plan(12288, 4096, 8, 0, 148, (ctypes.c_int64 * 5)()) == \
        _lib.ERR_INVALID_ARGUMENT
    assert "m > 8" in thq4.last_error()
