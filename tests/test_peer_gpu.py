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
