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


# ---- row-parallel shards (input columns) and the reduce ------------------------

def test_column_shards_are_whole_groups():
    from thq4.shard import shard_cols
    for K, world in [(5120, 2), (5120, 8), (17408, 4), (1024, 8)]:
        seen = np.zeros(K, dtype=np.int32)
        for r in range(world):
            k0, k = shard_cols(K, world, r)
            assert k0 % 64 == 0 and k % 64 == 0
            seen[k0:k0 + k] += 1
        assert (seen == 1).all()
    with pytest.raises(ValueError):
        shard_cols(5120, 3, 0)


def test_sliced_columns_are_the_weight_restricted_to_them():
    from thq4.shard import slice_cols_mlx
    out, inp, world = 128, 512, 4
    wq, sb = O.rand_qlin(out, inp, 8)
    x = O.bf16_to_f32(O.rand_x(inp, 9)).reshape(1, inp)
    full = O.linear_group(wq, sb, O.SB_BF16, x)[0].astype(np.float64)
    parts = np.zeros(out)
    for r in range(world):
        k0, k = r * inp // world, inp // world
        w_r, s_r = slice_cols_mlx(torch.from_numpy(wq.view(np.int32)), torch.from_numpy(sb.view(np.int16)), k0, k)
        assert w_r.shape == (out, k // 8) and s_r.shape == (out, 2 * k // 64)
        # the shard is the full weight's nibbles, scales and biases of its groups
        y_r = O.linear_group(w_r.numpy().view(np.uint32), s_r.numpy().view(np.uint16), O.SB_BF16, x[:, k0:k0 + k])
        parts += y_r[0]
    # the partials sum to the full product up to the f32 summation order
    assert np.abs(parts - full).max() <= 1e-5 * np.abs(full).max() + 1e-6


def _mlp_rank(rank, world, port, ret):
    """A column-then-row-parallel pair on gloo: y1 = W1 x on this rank's rows
    (local), y2_r = W2[:, rows] y1_r (f32 partial), all-reduced in rank order
    and rounded once, as the fused reduce does on the GPU."""
    from thq4.shard import shard_cols, slice_cols_mlx
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    n1, k1, n2 = 256, 384, 192
    w1, s1 = O.rand_qlin(n1, k1, 61)
    w2, s2 = O.rand_qlin(n2, n1, 62)
    x = O.bf16_to_f32(O.rand_x(k1, 63)).reshape(1, k1)
    b, n = shard_rows(n1, world, rank, align=64)
    y1 = O.bf16_round(O.linear_group(w1[b:b + n], s1[b:b + n], O.SB_BF16, x))
    k0, k = shard_cols(n1, world, rank)
    assert (k0, k) == (b, n)
    w2r, s2r = slice_cols_mlx(torch.from_numpy(w2.view(np.int32)), torch.from_numpy(s2.view(np.int16)), k0, k)
    part = torch.from_numpy(O.linear_group(w2r.numpy().view(np.uint32), s2r.numpy().view(np.uint16), O.SB_BF16,
                                           y1).astype(np.float32))
    parts = [torch.empty_like(part) for _ in range(world)]
    dist.all_gather(parts, part)
    total = torch.zeros_like(part)
    for p in parts:  # rank order, as the consumer's staging sums them
        total += p
    if rank == 0:
        ret.put(O.bf16_round(total.numpy()))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_row_parallel_pair():
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    paths = [here, root, os.path.join(root, "oracle"), os.path.join(root, "token-horizon_b200")]
    os.environ["PYTHONPATH"] = os.pathsep.join(paths + [os.environ.get("PYTHONPATH", "")])
    ctx = mp.get_context("spawn")
    ret = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_mlp_rank, args=(r, 2, port, ret)) for r in range(2)]
    for p in procs:
        p.start()
    got = ret.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    n1, k1, n2 = 256, 384, 192
    w1, s1 = O.rand_qlin(n1, k1, 61)
    w2, s2 = O.rand_qlin(n2, n1, 62)
    x = O.bf16_to_f32(O.rand_x(k1, 63)).reshape(1, k1)
    want = O.linear_group(w2, s2, O.SB_BF16, O.bf16_round(O.linear_group(w1, s1, O.SB_BF16, x)))
    from helpers import assert_close_ref
    assert_close_ref("row-parallel pair", got[0], want[0])
