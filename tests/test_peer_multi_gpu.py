"""Column shards over two GPUs with the all-gather fused into the projection:
two ranks (one process per GPU) each own half the rows of two chained
projections; the first gathers its output into both ranks' full vectors over
NVLink, the second reads that vector (after waiting for the peer's flag) and
gathers again.  Both ranks' full outputs must match the CPU oracle's
unsharded chain.  The MoE layer with its experts split over the two ranks
(each rank's f32 partial, one NCCL all-reduce) must match the oracle's
layer.  Skipped with fewer than two GPUs."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, ret):
    import ctypes
    import datetime

    import torch.distributed as dist

    import q4oracle as O
    import thq4
    from helpers import dev
    from thq4.shard import PeerGroup, shard_rows

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    d = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=d,
                            timeout=datetime.timedelta(seconds=120))
    try:
        n1, k1, n2 = 1024, 768, 512  # y1 = W1 x (1024 x 768), y2 = W2 y1 (512 x 1024)
        w1q, w1s = O.rand_qlin(n1, k1, 31)
        w2q, w2s = O.rand_qlin(n2, n1, 32)
        x = O.rand_x(k1, 33)
        b1, r1 = shard_rows(n1, world, rank)
        b2, r2 = shard_rows(n2, world, rank)
        q1 = thq4.QLin(dev(w1q[b1:b1 + r1]).to(d), dev(w1s[b1:b1 + r1]).to(d), r1, k1, 64).tiled()
        q2 = thq4.QLin(dev(w2q[b2:b2 + r2]).to(d), dev(w2s[b2:b2 + r2]).to(d), r2, n1, 64).tiled()
        L = thq4.lib()
        grp = PeerGroup((n1 + n2) * 2 + 512, d)
        o1, o2 = grp.buffer(n1 * 2), grp.buffer(n2 * 2)
        g1 = grp.gather(o1, r1, b1, n1, wait=True)
        g2 = grp.gather(o2, r2, b2, n2, wait=True)
        ws = thq4.qlin.workspace(q1.packed.desc, d)
        ws2 = torch.zeros_like(ws)
        xt = dev(x.reshape(1, k1)).to(d)
        y1 = torch.empty((1, r1), dtype=torch.bfloat16, device=d)
        y2 = torch.empty((1, r2), dtype=torch.bfloat16, device=d)
        P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        for _ in range(3):  # the flags count up across repeated chains
            thq4.check(L.thq4_linear_peer(ctypes.byref(q1.packed.desc), None, P(xt), thq4.BF16, 1, P(y1), P(ws),
                                          ws.numel(), ctypes.byref(g1), s))
            thq4.check(L.thq4_linear_peer(ctypes.byref(q2.packed.desc), None, ctypes.c_void_p(grp.ptr(o1)),
                                          thq4.BF16, 1, P(y2), P(ws2), ws2.numel(), ctypes.byref(g2), s))
        thq4.check(L.thq4_peer_wait(ctypes.byref(g2), s))  # the peer's last slice has landed
        full1 = torch.empty((1, n1), dtype=torch.bfloat16, device=d)
        full2 = torch.empty((1, n2), dtype=torch.bfloat16, device=d)
        thq4.check(L.thq4_copy(P(full1), ctypes.c_void_p(grp.ptr(o1)), n1 * 2, s))
        thq4.check(L.thq4_copy(P(full2), ctypes.c_void_p(grp.ptr(o2)), n2 * 2, s))
        torch.cuda.synchronize()
        st = ctypes.c_uint32()
        thq4.check(L.thq4_device_status(ctypes.byref(st), None))
        out = (full1.float().cpu().numpy().ravel(), full2.float().cpu().numpy().ravel(), int(st.value))
        grp.close()
        ret.put((rank, out))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_chain_matches_oracle():
    import torch.multiprocessing as mp

    import q4oracle as O
    from helpers import assert_close_ref

    paths = [HERE, ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "token-horizon_b200")]
    os.environ["PYTHONPATH"] = os.pathsep.join(paths + [os.environ.get("PYTHONPATH", "")])
    ctx = mp.get_context("spawn")
    ret = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, ret)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(ret.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    n1, k1, n2 = 1024, 768, 512
    w1q, w1s = O.rand_qlin(n1, k1, 31)
    w2q, w2s = O.rand_qlin(n2, n1, 32)
    x = O.bf16_to_f32(O.rand_x(k1, 33))
    y1 = O.linear_group(w1q, w1s, O.SB_BF16, x.reshape(1, k1))
    y1b = O.bf16_to_f32(O.f32_to_bf16(y1))
    y2 = O.linear_group(w2q, w2s, O.SB_BF16, y1b)
    for rank in range(2):
        f1, f2, status = got[rank]
        assert status == 0, f"rank {rank}: device status {status:#x}"
        assert_close_ref(f"rank {rank} gathered y1", f1, y1[0])
        assert_close_ref(f"rank {rank} gathered y2", f2, y2[0])
    assert np.array_equal(got[0][0], got[1][0]) and np.array_equal(got[0][1], got[1][1]), "ranks disagree"


def _moe_rank(rank, world, port, ret):
    import datetime

    import torch.distributed as dist

    import q4oracle as O
    import thq4
    from helpers import dev
    from thq4.shard import expert_range, moe_sharded

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    d = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=d,
                            timeout=datetime.timedelta(seconds=120))
    try:
        T, H, I, E, k = 64, 256, 128, 8, 2
        gu = [O.synthetic_weight(2 * I, H, 900 + e, O.SB_BF16) for e in range(E)]
        dn = [O.synthetic_weight(H, I, 950 + e, O.SB_BF16) for e in range(E)]
        gq, gs = np.stack([a for a, _ in gu]), np.stack([b for _, b in gu])
        dq, ds = np.stack([a for a, _ in dn]), np.stack([b for _, b in dn])
        e0, n = expert_range(E, world, rank)
        gate = thq4.PackedExperts.from_mlx(dev(gq[e0:e0 + n]).to(d), dev(gs[e0:e0 + n]).to(d), thq4.BF16, 0, I)
        up = thq4.PackedExperts.from_mlx(dev(gq[e0:e0 + n]).to(d), dev(gs[e0:e0 + n]).to(d), thq4.BF16, I, I)
        down = thq4.PackedExperts.from_mlx(dev(dq[e0:e0 + n]).to(d), dev(ds[e0:e0 + n]).to(d), thq4.BF16)
        rng = np.random.default_rng(3)
        x = O.f32_to_bf16(rng.standard_normal((T, H)).astype(np.float32))
        res = O.f32_to_bf16(rng.standard_normal((T, H)).astype(np.float32))
        lg = O.f32_to_bf16(rng.standard_normal((T, E)).astype(np.float32))
        y = moe_sharded(dev(x).to(d), dev(lg).to(d), k, e0, gate, up, down, residual=dev(res).to(d))
        torch.cuda.synchronize()
        ret.put((rank, y.cpu().view(torch.int16).numpy().view(np.uint16)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_expert_shards_match_oracle():
    import torch.multiprocessing as mp

    import q4oracle as O

    paths = [HERE, ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "token-horizon_b200")]
    os.environ["PYTHONPATH"] = os.pathsep.join(paths + [os.environ.get("PYTHONPATH", "")])
    ctx = mp.get_context("spawn")
    ret = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_moe_rank, args=(r, 2, port, ret)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(ret.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    T, H, I, E, k = 64, 256, 128, 8, 2
    gu = [O.synthetic_weight(2 * I, H, 900 + e, O.SB_BF16) for e in range(E)]
    dn = [O.synthetic_weight(H, I, 950 + e, O.SB_BF16) for e in range(E)]
    gq, gs = np.stack([a for a, _ in gu]), np.stack([b for _, b in gu])
    dq, ds = np.stack([a for a, _ in dn]), np.stack([b for _, b in dn])
    rng = np.random.default_rng(3)
    x = O.f32_to_bf16(rng.standard_normal((T, H)).astype(np.float32))
    res = O.f32_to_bf16(rng.standard_normal((T, H)).astype(np.float32))
    lg = O.f32_to_bf16(rng.standard_normal((T, E)).astype(np.float32))
    ids, w = O.moe_select(lg, k)
    want = O.bf16_to_f32(O.moe_forward(x, res, ids, w, gq, gs, dq, ds, O.SB_BF16, I)[0]).astype(np.float64)
    assert np.array_equal(got[0], got[1]), "ranks disagree after the all-reduce"
    y = O.bf16_to_f32(got[0]).astype(np.float64)
    assert np.all(np.abs(y - want) <= 0.02 + 0.01 * np.abs(want)), "sharded MoE differs from the oracle"


def _row_rank(rank, world, port, ret, ll=False):
    """y1 = W1 x on this rank's rows (kept local), y2 = W2 y1 row-parallel
    (this rank's input columns = its y1 rows; f32 partial into slot `rank`
    of every rank's reduction buffer), y3 = W3 bf16(sum of the partials)
    column-sharded and gathered."""
    import ctypes
    import datetime

    import torch.distributed as dist

    import q4oracle as O
    import thq4
    from helpers import dev
    from thq4.shard import PeerGroup, shard_cols, shard_rows, slice_cols_mlx

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    d = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=d,
                            timeout=datetime.timedelta(seconds=120))
    try:
        n1, k1, n2, n3 = 1024, 768, 768, 512
        w1q, w1s = O.rand_qlin(n1, k1, 41)
        w2q, w2s = O.rand_qlin(n2, n1, 42)
        w3q, w3s = O.rand_qlin(n3, n2, 43)
        x = O.rand_x(k1, 44)
        b1, r1 = shard_rows(n1, world, rank, align=64)
        k0, kk = shard_cols(n1, world, rank)
        b3, r3 = shard_rows(n3, world, rank)
        q1 = thq4.QLin(dev(w1q[b1:b1 + r1]).to(d), dev(w1s[b1:b1 + r1]).to(d), r1, k1, 64).tiled()
        w2r, s2r = slice_cols_mlx(dev(w2q).to(d), dev(w2s).to(d), k0, kk)
        q2 = thq4.QLin(w2r, s2r, n2, kk, 64).tiled()
        q3 = thq4.QLin(dev(w3q[b3:b3 + r3]).to(d), dev(w3s[b3:b3 + r3]).to(d), r3, n2, 64).tiled()
        L = thq4.lib()
        grp = PeerGroup(world * n2 * 8 + n3 * 2 + 1024, d)
        red = grp.buffer(grp.reduction_bytes(n2, 1, ll=ll))
        full3 = grp.buffer(n3 * 2)
        g2 = grp.reduce(red, n2, 1, wait=False, ll=ll)
        g3 = grp.gather(full3, r3, b3, n3, wait=True, x_parts=world, x_slot=n2, x_ll=ll)
        ws = [thq4.qlin.workspace(q.packed.desc, d) for q in (q1, q2, q3)]
        xt = dev(x.reshape(1, k1)).to(d)
        y1 = torch.empty((1, r1), dtype=torch.bfloat16, device=d)
        y3 = torch.empty((1, r3), dtype=torch.bfloat16, device=d)
        P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        for _ in range(3):
            thq4.check(L.thq4_linear(ctypes.byref(q1.packed.desc), P(xt), thq4.BF16, 1, P(y1), thq4.BF16, P(ws[0]),
                                     ws[0].numel(), s))
            thq4.check(L.thq4_linear_peer(ctypes.byref(q2.packed.desc), None, P(y1), thq4.BF16, 1, None, P(ws[1]),
                                          ws[1].numel(), ctypes.byref(g2), s))
            thq4.check(L.thq4_linear_peer(ctypes.byref(q3.packed.desc), None, ctypes.c_void_p(grp.ptr(red)), thq4.F32,
                                          1, P(y3), P(ws[2]), ws[2].numel(), ctypes.byref(g3), s))
            # one reduction buffer serves every iteration: a rank may write it
            # again only once every peer's reader of it is done
            torch.cuda.synchronize()
            dist.barrier(device_ids=[rank])
        thq4.check(L.thq4_peer_wait(ctypes.byref(g3), s))
        out = torch.empty((1, n3), dtype=torch.bfloat16, device=d)
        thq4.check(L.thq4_copy(P(out), ctypes.c_void_p(grp.ptr(full3)), n3 * 2, s))
        torch.cuda.synchronize()
        st = ctypes.c_uint32()
        thq4.check(L.thq4_device_status(ctypes.byref(st), None))
        ret.put((rank, (out.float().cpu().numpy().ravel(), int(st.value))))
        grp.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("ll", [False, True], ids=["flags", "low-latency"])
def test_two_gpu_row_parallel_reduce_matches_oracle(ll):
    import torch.multiprocessing as mp

    import q4oracle as O
    from helpers import assert_close_ref

    paths = [HERE, ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "token-horizon_b200")]
    os.environ["PYTHONPATH"] = os.pathsep.join(paths + [os.environ.get("PYTHONPATH", "")])
    ctx = mp.get_context("spawn")
    ret = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_row_rank, args=(r, 2, port, ret, ll)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(ret.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    n1, k1, n2, n3 = 1024, 768, 768, 512
    w1q, w1s = O.rand_qlin(n1, k1, 41)
    w2q, w2s = O.rand_qlin(n2, n1, 42)
    w3q, w3s = O.rand_qlin(n3, n2, 43)
    x = O.bf16_to_f32(O.rand_x(k1, 44)).reshape(1, k1)
    y1 = O.bf16_round(O.linear_group(w1q, w1s, O.SB_BF16, x))
    y2 = O.bf16_round(O.linear_group(w2q, w2s, O.SB_BF16, y1))
    y3 = O.linear_group(w3q, w3s, O.SB_BF16, y2)
    for rank in range(2):
        f3, status = got[rank]
        assert status == 0, f"rank {rank}: device status {status:#x}"
        assert_close_ref(f"rank {rank} row-parallel chain", f3, y3[0])
    assert np.array_equal(got[0][0], got[1][0]), "ranks disagree"


def _block_rank(rank, world, port, ret):
    """The Splash MoE block (Q8 router, shared expert) with the routed experts
    split over two ranks and the shared expert on the last rank
    (thq4.shard.moe_add_sharded: partials, one NCCL all-reduce)."""
    import datetime

    import torch.distributed as dist

    import q4oracle as O
    import thq4
    from test_moe_q8_cpu import E, H, I, K, configure_routing, fixture_router, fixture_shared_gate
    from thq4.shard import expert_range, moe_add_sharded

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    d = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=d,
                            timeout=datetime.timedelta(seconds=120))
    try:
        rows = 48
        fx = O.splash_moe_fixture(H, I, E, rows)
        x = configure_routing(fx["x"], "dispersed")
        e0, n = expert_range(E, world, rank)
        sl = lambda name, lo=0, hi=None: torch.from_numpy(fx[name][lo:hi]).to(d)  # noqa: E731
        bf = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(d).view(torch.bfloat16)  # noqa
        q8 = lambda p: thq4.Q8Projection(torch.from_numpy(p[0]).to(d), bf(p[1]), bf(p[2]), H)  # noqa: E731
        last = rank == world - 1
        w = thq4.MoeWeights(q8(fixture_router(H, E)),
                            thq4.PackedExperts.from_slabs(sl("gate", e0, e0 + n), I, H, thq4.BF16),
                            thq4.PackedExperts.from_slabs(sl("up", e0, e0 + n), I, H, thq4.BF16),
                            thq4.PackedExperts.from_slabs(sl("down", e0, e0 + n), H, I, thq4.BF16),
                            thq4.PackedExperts.from_slabs(sl("shared_gate"), I, H, thq4.BF16) if last else None,
                            thq4.PackedExperts.from_slabs(sl("shared_up"), I, H, thq4.BF16) if last else None,
                            thq4.PackedExperts.from_slabs(sl("shared_down"), H, I, thq4.BF16) if last else None,
                            q8(fixture_shared_gate(H)))
        y = moe_add_sharded(bf(x), w, K, e0, E, residual=bf(fx["residual"]))
        torch.cuda.synchronize()
        ret.put((rank, y.cpu().view(torch.int16).numpy().view(np.uint16)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_moe_block_with_shared_expert():
    import torch.multiprocessing as mp

    import q4oracle as O
    from test_moe_q8_cpu import E, H, I, K, configure_routing, fixture_router, fixture_shared_gate, mlx_experts

    paths = [HERE, ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "token-horizon_b200")]
    os.environ["PYTHONPATH"] = os.pathsep.join(paths + [os.environ.get("PYTHONPATH", "")])
    ctx = mp.get_context("spawn")
    ret = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_block_rank, args=(r, 2, port, ret)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(ret.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert np.array_equal(got[0], got[1]), "ranks disagree after the all-reduce"
    rows = 48
    fx = O.splash_moe_fixture(H, I, E, rows)
    x = configure_routing(fx["x"], "dispersed")
    ids, w, _ = O.moe_route_q8(x, E, K, fixture_router(H, E), fixture_shared_gate(H))
    gu_q, gu_s, dq, ds, shared = mlx_experts(fx)
    want, _, dd = O.moe_forward(x, fx["residual"], ids, w, gu_q, gu_s, dq, ds, O.SB_BF16, I, shared=shared)
    mag = np.abs(O.bf16_to_f32(fx["residual"])).astype(np.float64) + (
        np.abs(O.bf16_to_f32(w)[:, :, None] * O.bf16_to_f32(dd).reshape(rows, K + 1, H))).sum(axis=1)
    diff = np.abs(O.bf16_to_f32(got[0]).astype(np.float64) - O.bf16_to_f32(want))
    assert np.all(diff <= 0.02 + 0.01 * mag), "sharded MoE block differs from the oracle"
