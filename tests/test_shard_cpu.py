"""Multi-rank host logic on CPU: the column shards cover every output row
once, and two gloo ranks that each compute their slice of y (with the CPU
oracle standing in for the kernel) reassemble exactly the single-rank y."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import q4oracle as O
from thq4.shard import gather_rows, shard_rows


@pytest.mark.parametrize("total,world", [(5120, 2), (5120, 8), (17408, 4), (1024, 8), (7168, 2)])
def test_shards_partition_the_rows(total, world):
    seen = np.zeros(total, dtype=np.int32)
    for r in range(world):
        b, n = shard_rows(total, world, r)
        assert n % 16 == 0 and n == total // world
        seen[b:b + n] += 1
    assert (seen == 1).all()


def test_shard_rejects_ragged_splits():
    with pytest.raises(ValueError):
        shard_rows(1000, 3, 0)
    with pytest.raises(ValueError):
        shard_rows(5120, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out, inp, m, ret):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    wq, sb = O.rand_qlin(out, inp, 21)
    x = O.bf16_to_f32(np.stack([O.rand_x(inp, 50 + t) for t in range(m)]))
    b, n = shard_rows(out, world, rank)
    local = torch.from_numpy(O.linear_group(wq[b:b + n], sb[b:b + n], O.SB_BF16, x).astype(np.float32))
    full = gather_rows(local)
    if rank == 0:
        ret.put(full.numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_reassemble_y():
    out, inp, m, world = 256, 448, 3, 2
    # spawned ranks re-import this module: hand them the test import paths
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    paths = [here, root, os.path.join(root, "oracle"), os.path.join(root, "token-horizon_b200")]
    os.environ["PYTHONPATH"] = os.pathsep.join(paths + [os.environ.get("PYTHONPATH", "")])
    ctx = mp.get_context("spawn")
    ret = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, out, inp, m, ret)) for r in range(world)]
    for p in procs:
        p.start()
    got = ret.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    wq, sb = O.rand_qlin(out, inp, 21)
    x = O.bf16_to_f32(np.stack([O.rand_x(inp, 50 + t) for t in range(m)]))
    want = O.linear_group(wq, sb, O.SB_BF16, x).astype(np.float32)
    assert np.array_equal(got, want)


def test_expert_ranges_partition_the_experts():
    from thq4.shard import expert_range
    for E, world in [(128, 2), (128, 8), (8, 4), (64, 1)]:
        seen = np.zeros(E, dtype=np.int32)
        for r in range(world):
            e0, n = expert_range(E, world, r)
            seen[e0:e0 + n] += 1
        assert (seen == 1).all()
    with pytest.raises(ValueError):
        expert_range(10, 4, 0)
