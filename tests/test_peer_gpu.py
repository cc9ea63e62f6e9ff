"""The all-gather fused into the projection (thq4_linear_peer) on one GPU:
world 1 through a real PeerGroup, and the epilogue of a world-2 rank with
both ranks' buffers on this GPU (the peer never runs, so nothing waits on
it): the shard's rows land in every rank's full vector, the rank's slot of
the peer's flags receives the gather count, a wait on flags already raised
passes, and a wait on a flag nothing raises ends with the timeout bit set
instead of hanging."""
import ctypes
import time

import numpy as np
import pytest
import torch

import q4oracle as O
import thq4
from thq4 import _lib
from thq4.shard import PeerGroup
from helpers import dev, host_bits

pytestmark = pytest.mark.gpu

P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
S = lambda: ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)  # noqa: E731
TIMEOUT_BIT = 1 << 2


def _weight(out, inp, seed):
    wq, sb = O.rand_qlin(out, inp, seed)
    return wq, sb, thq4.QLin(dev(wq), dev(sb), out, inp, 64).tiled()


def _status():
    st = ctypes.c_uint32()
    thq4.check(thq4.lib().thq4_device_status(ctypes.byref(st), None))
    return st.value


def _workspace(desc):
    return thq4.qlin.workspace(desc, torch.device("cuda"))


@pytest.mark.parametrize("gate_up", [False, True])
def test_world1_matches_plain_call(gate_up):
    out, inp, m = 1024, 1536, 2
    wq, sb = O.rand_qlin(2 * out if gate_up else out, inp, 5)
    q = thq4.QLin(dev(wq), dev(sb), 2 * out if gate_up else out, inp, 64).tiled(out if gate_up else 0)
    L = thq4.lib()
    x = dev(np.stack([O.rand_x(inp, 60 + t) for t in range(m)]))
    grp = PeerGroup(m * out * 2, torch.device("cuda"))
    try:
        off = grp.buffer(m * out * 2)
        first = q.packed_gate if gate_up else q.packed
        ws = _workspace(first.desc)
        y_ref = torch.empty((m, out), dtype=torch.bfloat16, device="cuda")
        y = torch.full((m, out), float("nan"), dtype=torch.bfloat16, device="cuda")
        wd = ctypes.byref(first.desc)
        ud = ctypes.byref(q.packed_up.desc) if gate_up else None
        if gate_up:
            thq4.check(L.thq4_gate_up(wd, ud, P(x), thq4.BF16, m, P(y_ref), thq4.BF16, P(ws), ws.numel(), S()))
        else:
            thq4.check(L.thq4_linear(wd, P(x), thq4.BF16, m, P(y_ref), thq4.BF16, P(ws), ws.numel(), S()))
        for call in range(2):
            desc = grp.gather(off, out, 0, out, wait=True)
            thq4.check(L.thq4_linear_peer(wd, ud, P(x), thq4.BF16, m, P(y), P(ws), ws.numel(), ctypes.byref(desc), S()))
            torch.cuda.synchronize()
            assert torch.equal(y.view(torch.int16), y_ref.view(torch.int16)), "local rows differ from the plain call"
            full = torch.empty((m, out), dtype=torch.bfloat16, device="cuda")
            thq4.check(L.thq4_copy(P(full), ctypes.c_void_p(grp.ptr(off)), full.numel() * 2, S()))
            torch.cuda.synchronize()
            assert torch.equal(full.view(torch.int16), y_ref.view(torch.int16)), "gathered vector differs"
        cnt = torch.empty(1, dtype=torch.int32, device="cuda")
        thq4.check(L.thq4_copy(P(cnt), ctypes.c_void_p(grp.count), 4, S()))
        torch.cuda.synchronize()
        assert int(cnt.item()) == 2, "one gather count per call"
        assert _status() & TIMEOUT_BIT == 0
    finally:
        grp.close()


def _emulated_rank0(region_a, region_b, out, stride, wait):
    """thq4_peer_gather of rank 0 of 2 whose peer (rank 1) lives in region_b
    of this GPU.  Regions: flags [2] u32 at 0, count at 64, arrive at 128,
    the full vector at 256."""
    ptrs = lambda *ts: torch.tensor([t for t in ts], dtype=torch.int64, device="cuda")  # noqa: E731
    dst = ptrs(region_a.data_ptr() + 256, region_b.data_ptr() + 256)
    flags = ptrs(region_a.data_ptr(), region_b.data_ptr())
    g = _lib.thq4_peer_gather()
    g.world, g.rank, g.rows, g.offset, g.stride, g.wait = 2, 0, out, 0, stride, int(wait)
    g.dst, g.flags = dst.data_ptr(), flags.data_ptr()
    g.count, g.arrive = region_a.data_ptr() + 64, region_a.data_ptr() + 128
    return g, (dst, flags)


def test_world2_epilogue_and_flags_on_one_gpu():
    out, inp = 512, 1024
    wq, sb, q = _weight(out, inp, 9)
    L = thq4.lib()
    x = dev(O.rand_x(inp, 77).reshape(1, inp))
    ws = _workspace(q.packed.desc)
    y_ref = torch.empty((1, out), dtype=torch.bfloat16, device="cuda")
    thq4.check(L.thq4_linear(ctypes.byref(q.packed.desc), P(x), thq4.BF16, 1, P(y_ref), thq4.BF16, P(ws), ws.numel(),
                             S()))
    nbytes = 256 + 2 * out * 2
    ra = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    rb = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    y = torch.empty((1, out), dtype=torch.bfloat16, device="cuda")
    g, keep = _emulated_rank0(ra, rb, out, 2 * out, wait=False)
    thq4.check(L.thq4_linear_peer(ctypes.byref(q.packed.desc), None, P(x), thq4.BF16, 1, P(y), P(ws), ws.numel(),
                                  ctypes.byref(g), S()))
    torch.cuda.synchronize()
    want = host_bits(y_ref).ravel()
    for region in (ra, rb):
        full = host_bits(region[256:256 + 2 * out * 2].view(torch.bfloat16)).ravel()
        assert np.array_equal(full[:out], want), "rank 0's rows missing from a rank's full vector"
        assert not full[out:].any(), "rank 1's half was written"
    fa = ra[:8].view(torch.int32).cpu().numpy()
    fb = rb[:8].view(torch.int32).cpu().numpy()
    assert fb[0] == 1 and fb[1] == 0, "rank 0's slot of the peer's flags holds its gather count"
    assert not fa.any(), "a rank raises no flag of its own"
    assert int(ra[64:68].view(torch.int32).item()) == 1
    assert int(ra[128:132].view(torch.int32).item()) == 0, "the arrival counter is left at 0"

    # rank 1 "has" completed one gather: rank 0's wait passes at once
    ra[4:8].view(torch.int32).fill_(1)
    g2, keep2 = _emulated_rank0(ra, rb, out, 2 * out, wait=True)
    _status()
    thq4.check(L.thq4_linear_peer(ctypes.byref(q.packed.desc), None, P(x), thq4.BF16, 1, P(y), P(ws), ws.numel(),
                                  ctypes.byref(g2), S()))
    torch.cuda.synchronize()
    assert _status() & TIMEOUT_BIT == 0
    assert int(rb[:4].view(torch.int32).item()) == 2


def test_wait_on_a_flag_nothing_raises_times_out():
    """Failure detection: the peer never completes its gather.  The wait gives
    up after its 2 s bound, the call returns and the status word says so; the
    context stays usable."""
    out, inp = 256, 512
    wq, sb, q = _weight(out, inp, 13)
    L = thq4.lib()
    x = dev(O.rand_x(inp, 5).reshape(1, inp))
    ws = _workspace(q.packed.desc)
    nbytes = 256 + 2 * out * 2
    ra = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    rb = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    ra[64:68].view(torch.int32).fill_(3)  # this rank has completed 3 gathers, the peer none
    y = torch.empty((1, out), dtype=torch.bfloat16, device="cuda")
    g, keep = _emulated_rank0(ra, rb, out, 2 * out, wait=True)
    _status()
    t0 = time.time()
    thq4.check(L.thq4_linear_peer(ctypes.byref(q.packed.desc), None, P(x), thq4.BF16, 1, P(y), P(ws), ws.numel(),
                                  ctypes.byref(g), S()))
    torch.cuda.synchronize()
    assert time.time() - t0 < 30
    assert _status() & TIMEOUT_BIT, "the bounded wait reports its timeout"
    # the context is still usable
    thq4.check(L.thq4_linear(ctypes.byref(q.packed.desc), P(x), thq4.BF16, 1, P(y), thq4.BF16, P(ws), ws.numel(), S()))
    torch.cuda.synchronize()
    assert _status() == 0


def test_peer_call_validation():
    L = thq4.lib()
    w = _lib.thq4_weight()
    w.out, w.in_, w.gs, w.sb_dtype = 256, 512, 64, thq4.BF16
    x = torch.zeros((16, 512), dtype=torch.bfloat16, device="cuda")
    y = torch.zeros((16, 256), dtype=torch.bfloat16, device="cuda")
    w.qw = w.sb = ctypes.c_void_p(x.data_ptr())
    g = _lib.thq4_peer_gather()
    g.world, g.rank, g.rows, g.offset, g.stride = 2, 2, 256, 0, 512
    g.dst = g.flags = g.count = g.arrive = x.data_ptr()
    st = L.thq4_linear_peer(ctypes.byref(w), None, P(x), thq4.BF16, 1, P(y), P(x), 1 << 20, ctypes.byref(g), S())
    assert st == _lib.ERR_INVALID_ARGUMENT and "rank" in thq4.last_error()
    g.rank = 1
    st = L.thq4_linear_peer(ctypes.byref(w), None, P(x), thq4.BF16, 16, P(y), P(x), 1 << 20, ctypes.byref(g), S())
    assert st == _lib.ERR_UNSUPPORTED
    g.offset = 300
    st = L.thq4_linear_peer(ctypes.byref(w), None, P(x), thq4.BF16, 1, P(y), P(x), 1 << 20, ctypes.byref(g), S())
    assert st == _lib.ERR_INVALID_ARGUMENT and "stride" in thq4.last_error()


# ---- row-parallel shards: the reduce epilogue and partials read back --------------

def _f32_out(q, x, m=1):
    ws = _workspace(q.packed.desc)
    y = torch.empty((m, q.packed.desc.out), dtype=torch.float32, device="cuda")
    thq4.check(thq4.lib().thq4_linear(ctypes.byref(q.packed.desc), P(x), thq4.BF16, m, P(y), thq4.F32, P(ws),
                                      ws.numel(), S()))
    return y


def test_world1_reduce_then_partials_equal_the_plain_chain():
    """World 1: a projection in reduce mode writes its f32 output into slot 0;
    the next projection reads it as one partial (rounded to bf16 as staged):
    the pair equals the plain chain bit for bit."""
    n1, k1, n2, m = 512, 768, 256, 2
    _, _, q1 = _weight(n1, k1, 71)
    _, _, q2 = _weight(n2, n1, 72)
    L = thq4.lib()
    x = dev(np.stack([O.rand_x(k1, 80 + t) for t in range(m)]))
    ws1, ws2 = _workspace(q1.packed.desc), _workspace(q2.packed.desc)
    y1 = torch.empty((m, n1), dtype=torch.bfloat16, device="cuda")
    y2 = torch.empty((m, n2), dtype=torch.bfloat16, device="cuda")
    thq4.check(L.thq4_linear(ctypes.byref(q1.packed.desc), P(x), thq4.BF16, m, P(y1), thq4.BF16, P(ws1), ws1.numel(),
                             S()))
    thq4.check(L.thq4_linear(ctypes.byref(q2.packed.desc), P(y1), thq4.BF16, m, P(y2), thq4.BF16, P(ws2), ws2.numel(),
                             S()))
    grp = PeerGroup(4 * m * n1 + 256, torch.device("cuda"))
    try:
        off = grp.buffer(grp.reduction_bytes(n1, m))
        g1 = grp.reduce(off, n1, m, wait=False)
        g2 = grp.local_out(wait=True, x_parts=1, x_slot=m * n1)
        z2 = torch.empty_like(y2)
        for _ in range(2):
            thq4.check(L.thq4_linear_peer(ctypes.byref(q1.packed.desc), None, P(x), thq4.BF16, m, None, P(ws1),
                                          ws1.numel(), ctypes.byref(g1), S()))
            thq4.check(L.thq4_linear_peer(ctypes.byref(q2.packed.desc), None, ctypes.c_void_p(grp.ptr(off)),
                                          thq4.F32, m, P(z2), P(ws2), ws2.numel(), ctypes.byref(g2), S()))
            torch.cuda.synchronize()
            assert torch.equal(z2.view(torch.int16), y2.view(torch.int16)), "reduce + partials differ from the chain"
        part = torch.empty((m, n1), dtype=torch.float32, device="cuda")
        thq4.check(L.thq4_copy(P(part), ctypes.c_void_p(grp.ptr(off)), part.numel() * 4, S()))
        torch.cuda.synchronize()
        assert torch.equal(part, _f32_out(q1, x, m)), "slot 0 holds the f32 output"
        assert _status() & TIMEOUT_BIT == 0
    finally:
        grp.close()


def test_world2_reduce_epilogue_on_one_gpu():
    """Rank 0 of 2 (the peer's region also on this GPU, the peer never runs):
    its f32 partial lands in slot 0 of both ranks' reduction buffers, slot 1
    stays untouched, and rank 0's flag on the peer counts the exchange."""
    out, inp, m = 384, 512, 1
    _, _, q = _weight(out, inp, 73)
    L = thq4.lib()
    x = dev(O.rand_x(inp, 74).reshape(1, inp))
    ws = _workspace(q.packed.desc)
    nbytes = 256 + 2 * m * out * 4
    ra = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    rb = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    g, keep = _emulated_rank0(ra, rb, out, out, wait=False)
    g.out_mode, g.slot = 1, m * out
    thq4.check(L.thq4_linear_peer(ctypes.byref(q.packed.desc), None, P(x), thq4.BF16, m, None, P(ws), ws.numel(),
                                  ctypes.byref(g), S()))
    torch.cuda.synchronize()
    want = _f32_out(q, x).cpu()
    for region in (ra, rb):
        slots = region[256:].view(torch.float32).cpu().reshape(2, out)
        assert torch.equal(slots[0], want[0]), "rank 0's partial missing from a rank's buffer"
        assert not slots[1].any(), "rank 1's slot was written"
    assert int(rb[:4].view(torch.int32).item()) == 1 and not ra[:8].any()


@pytest.mark.parametrize("parts,gate_up", [(2, False), (3, True), (8, False)])
def test_partials_are_summed_in_rank_order(parts, gate_up):
    """x given as `parts` f32 partials is staged as bf16(p0 + p1 + ...): the
    call equals the plain call on that x, bit for bit."""
    n, inp, m = 256, 1024, 3
    wq, sb = O.rand_qlin(2 * n if gate_up else n, inp, 75)
    q = thq4.QLin(dev(wq), dev(sb), 2 * n if gate_up else n, inp, 64).tiled(n if gate_up else 0)
    first = q.packed_gate if gate_up else q.packed
    L = thq4.lib()
    rng = np.random.default_rng(parts)
    p = torch.from_numpy(rng.standard_normal((parts, m, inp)).astype(np.float32)).cuda()
    total = torch.zeros((m, inp), dtype=torch.float32, device="cuda")
    for r in range(parts):
        total += p[r]
    xb = total.to(torch.bfloat16)  # round to nearest even, as the staging does
    ws = _workspace(first.desc)
    ud = ctypes.byref(q.packed_up.desc) if gate_up else None
    y_ref = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    if gate_up:
        thq4.check(L.thq4_gate_up(ctypes.byref(first.desc), ud, P(xb), thq4.BF16, m, P(y_ref), thq4.BF16, P(ws),
                                  ws.numel(), S()))
    else:
        thq4.check(L.thq4_linear(ctypes.byref(first.desc), P(xb), thq4.BF16, m, P(y_ref), thq4.BF16, P(ws),
                                 ws.numel(), S()))
    flags = torch.zeros(64, dtype=torch.int32, device="cuda")
    g = _lib.thq4_peer_gather()
    g.world, g.rank, g.wait, g.out_mode = 1, 0, 0, 2
    keep = torch.tensor([flags.data_ptr()], dtype=torch.int64, device="cuda")
    g.flags, g.count = keep.data_ptr(), flags.data_ptr() + 64
    g.x_parts, g.x_slot = parts, m * inp
    y = torch.empty_like(y_ref)
    thq4.check(L.thq4_linear_peer(ctypes.byref(first.desc), ud, P(p), thq4.F32, m, P(y), P(ws), ws.numel(),
                                  ctypes.byref(g), S()))
    torch.cuda.synchronize()
    assert torch.equal(y.view(torch.int16), y_ref.view(torch.int16))


def test_reduce_validation():
    L = thq4.lib()
    w = _lib.thq4_weight()
    w.out, w.in_, w.gs, w.sb_dtype = 256, 512, 64, thq4.BF16
    x = torch.zeros((16, 512), dtype=torch.float32, device="cuda")
    w.qw = w.sb = ctypes.c_void_p(x.data_ptr())
    g = _lib.thq4_peer_gather()
    g.world, g.rank, g.rows, g.offset, g.stride, g.out_mode, g.slot = 2, 0, 256, 0, 256, 1, 256
    g.dst = g.flags = g.count = g.arrive = x.data_ptr()
    g.rows = 128
    st = L.thq4_linear_peer(ctypes.byref(w), None, P(x), thq4.BF16, 1, None, P(x), 1 << 20, ctypes.byref(g), S())
    assert st == _lib.ERR_INVALID_ARGUMENT and "reduce needs rows == out" in thq4.last_error()
    g.rows = 256
    st = L.thq4_linear_peer(ctypes.byref(w), ctypes.byref(w), P(x), thq4.BF16, 1, None, P(x), 1 << 20,
                            ctypes.byref(g), S())
    assert st == _lib.ERR_UNSUPPORTED
    g.out_mode, g.x_parts, g.x_slot = 2, 2, 512
    st = L.thq4_linear_peer(ctypes.byref(w), None, P(x), thq4.BF16, 1, P(x), P(x), 1 << 20, ctypes.byref(g), S())
    assert st == _lib.ERR_INVALID_ARGUMENT and "partials are f32" in thq4.last_error()
    g.out_mode = 4
    st = L.thq4_linear_peer(ctypes.byref(w), None, P(x), thq4.F32, 1, P(x), P(x), 1 << 20, ctypes.byref(g), S())
    assert st == _lib.ERR_INVALID_ARGUMENT and "out_mode" in thq4.last_error()
    g.out_mode, g.x_ll, g.wait = 2, 1, 1  # the low-latency words are polled: no flag wait with them
    st = L.thq4_linear_peer(ctypes.byref(w), None, P(x), thq4.F32, 1, P(x), P(x), 1 << 20, ctypes.byref(g), S())
    assert st == _lib.ERR_INVALID_ARGUMENT and "x_ll" in thq4.last_error()


# ---- the low-latency reduce: 8-byte words {value, exchange number}, polled ----------

def test_world1_low_latency_reduce_equals_the_plain_chain():
    """World 1, out_mode 3: the projection's f32 output lands in slot 0 as
    words {value, exchange number}; the next projection polls them (x_ll)
    and equals the plain chain bit for bit, call after call (the exchange
    number goes up by one per exchange)."""
    n1, k1, n2, m = 512, 768, 256, 2
    _, _, q1 = _weight(n1, k1, 91)
    _, _, q2 = _weight(n2, n1, 92)
    L = thq4.lib()
    x = dev(np.stack([O.rand_x(k1, 93 + t) for t in range(m)]))
    ws1, ws2 = _workspace(q1.packed.desc), _workspace(q2.packed.desc)
    y1 = torch.empty((m, n1), dtype=torch.bfloat16, device="cuda")
    y2 = torch.empty((m, n2), dtype=torch.bfloat16, device="cuda")
    thq4.check(L.thq4_linear(ctypes.byref(q1.packed.desc), P(x), thq4.BF16, m, P(y1), thq4.BF16, P(ws1), ws1.numel(),
                             S()))
    thq4.check(L.thq4_linear(ctypes.byref(q2.packed.desc), P(y1), thq4.BF16, m, P(y2), thq4.BF16, P(ws2), ws2.numel(),
                             S()))
    grp = PeerGroup(8 * m * n1 + 256, torch.device("cuda"))
    try:
        off = grp.buffer(grp.reduction_bytes(n1, m, ll=True))
        g1 = grp.reduce(off, n1, m, wait=False, ll=True)
        g2 = grp.local_out(wait=True, x_parts=1, x_slot=m * n1, x_ll=True)
        assert g2.wait == 0
        z2 = torch.empty_like(y2)
        for call in range(1, 4):
            thq4.check(L.thq4_linear_peer(ctypes.byref(q1.packed.desc), None, P(x), thq4.BF16, m, None, P(ws1),
                                          ws1.numel(), ctypes.byref(g1), S()))
            thq4.check(L.thq4_linear_peer(ctypes.byref(q2.packed.desc), None, ctypes.c_void_p(grp.ptr(off)),
                                          thq4.F32, m, P(z2), P(ws2), ws2.numel(), ctypes.byref(g2), S()))
            torch.cuda.synchronize()
            assert torch.equal(z2.view(torch.int16), y2.view(torch.int16)), "low-latency reduce differs from the chain"
            words = torch.empty((m, n1, 2), dtype=torch.int32, device="cuda")
            thq4.check(L.thq4_copy(P(words), ctypes.c_void_p(grp.ptr(off)), words.numel() * 4, S()))
            torch.cuda.synchronize()
            assert torch.equal(words[..., 0].view(torch.float32), _f32_out(q1, x, m)), "slot 0 holds the f32 output"
            assert bool((words[..., 1] == call).all()), "every word carries this exchange's number"
        assert _status() & TIMEOUT_BIT == 0
    finally:
        grp.close()


def _ll_regions(out, m, parts):
    ra = torch.zeros(256 + parts * m * out * 8, dtype=torch.uint8, device="cuda")
    rb = torch.zeros_like(ra)
    return ra, rb


def test_world2_low_latency_writer_and_reader_on_one_gpu():
    """Rank 0 of 2 on one GPU (the peer never runs): its out_mode 3 words land
    in slot 0 of both ranks' buffers with exchange number count + 1, no flag is
    raised and the count goes up; a reader whose slot 1 words the test has
    written (the peer's share) equals the plain call on bf16(p0 + p1)."""
    out, inp, m = 384, 512, 1
    _, _, q = _weight(out, inp, 94)
    _, _, q2 = _weight(256, out, 95)
    L = thq4.lib()
    x = dev(O.rand_x(inp, 96).reshape(1, inp))
    ws, ws2 = _workspace(q.packed.desc), _workspace(q2.packed.desc)
    ra, rb = _ll_regions(out, m, 2)
    ra[64:68].view(torch.int32).fill_(6)  # this rank has completed 6 exchanges
    g, keep = _emulated_rank0(ra, rb, out, out, wait=False)
    g.out_mode, g.slot = 3, m * out
    thq4.check(L.thq4_linear_peer(ctypes.byref(q.packed.desc), None, P(x), thq4.BF16, m, None, P(ws), ws.numel(),
                                  ctypes.byref(g), S()))
    torch.cuda.synchronize()
    want = _f32_out(q, x).cpu()
    for region in (ra, rb):
        words = region[256:].view(torch.int32).cpu().reshape(2, out, 2)
        assert torch.equal(words[0, :, 0].view(torch.float32), want[0])
        assert bool((words[0, :, 1] == 7).all()), "words carry exchange number count + 1"
        assert not words[1].any(), "rank 1's slot was written"
    assert not ra[:8].any() and not rb[:8].any(), "no flags for low-latency words"
    assert int(ra[64:68].view(torch.int32).item()) == 7 and int(ra[128:132].view(torch.int32).item()) == 0
    # the peer's share arrives in slot 1 of this rank's buffer; the reader sums both
    peer = torch.from_numpy(np.random.default_rng(3).standard_normal(out).astype(np.float32)).cuda()
    w1 = ra[256 + m * out * 8:].view(torch.int32).view(out, 2)
    w1[:, 0] = peer.view(torch.int32)
    w1[:, 1] = 7
    g2, keep2 = _emulated_rank0(ra, rb, out, out, wait=False)
    g2.out_mode, g2.x_parts, g2.x_slot, g2.x_ll = 2, 2, m * out, 1
    y = torch.empty((1, 256), dtype=torch.bfloat16, device="cuda")
    _status()
    thq4.check(L.thq4_linear_peer(ctypes.byref(q2.packed.desc), None, ctypes.c_void_p(ra.data_ptr() + 256), thq4.F32,
                                  1, P(y), P(ws2), ws2.numel(), ctypes.byref(g2), S()))
    xb = (want[0].cuda() + peer).to(torch.bfloat16).reshape(1, out)
    y_ref = torch.empty_like(y)
    thq4.check(L.thq4_linear(ctypes.byref(q2.packed.desc), P(xb), thq4.BF16, 1, P(y_ref), thq4.BF16, P(ws2),
                             ws2.numel(), S()))
    torch.cuda.synchronize()
    assert _status() & TIMEOUT_BIT == 0
    assert torch.equal(y.view(torch.int16), y_ref.view(torch.int16))


def test_low_latency_words_that_never_arrive_time_out():
    """Failure detection for the low-latency exchange: the peer's words never
    carry this exchange's number.  Every poll shares one 2 s deadline, the
    call returns with the timeout bit set and the context stays usable."""
    out, inp, m = 256, 512, 1
    _, _, q = _weight(out, inp, 97)
    L = thq4.lib()
    ws = _workspace(q.packed.desc)
    ra, rb = _ll_regions(inp, m, 2)
    ra[64:68].view(torch.int32).fill_(5)  # expects exchange 5; the words say 4
    ra[256:].view(torch.int32).view(-1, 2)[:, 1] = 4
    g, keep = _emulated_rank0(ra, rb, inp, inp, wait=False)
    g.out_mode, g.x_parts, g.x_slot, g.x_ll = 2, 2, m * inp, 1
    y = torch.empty((1, out), dtype=torch.bfloat16, device="cuda")
    _status()
    t0 = time.time()
    thq4.check(L.thq4_linear_peer(ctypes.byref(q.packed.desc), None, ctypes.c_void_p(ra.data_ptr() + 256), thq4.F32, 1,
                                  P(y), P(ws), ws.numel(), ctypes.byref(g), S()))
    torch.cuda.synchronize()
    assert time.time() - t0 < 30
    assert _status() & TIMEOUT_BIT, "the bounded poll reports its timeout"
    x = dev(O.rand_x(inp, 5).reshape(1, inp))
    thq4.check(L.thq4_linear(ctypes.byref(q.packed.desc), P(x), thq4.BF16, 1, P(y), thq4.BF16, P(ws), ws.numel(), S()))
    torch.cuda.synchronize()
    assert _status() == 0
