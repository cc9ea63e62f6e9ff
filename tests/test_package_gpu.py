"""Splash package sections repacked on the device: a Q4 projection and an
expert projection loaded from a package file become the same frag bytes as
the MLX arrays they were made from, and the loaded projection matches the
CPU oracle."""
import ctypes
import os

import numpy as np
import pytest
import torch

import q4oracle as O
import thq4
from thq4 import package as pk
from helpers import assert_close_ref, dev

pytestmark = pytest.mark.gpu
MAGIC = b"THQ4TEST"


def test_package_projection_and_experts(tmp_path):
    out, inp = 512, 448
    wq, sb = O.rand_qlin(out, inp, 41)
    slab = O.mlx_to_slab(wq, sb)
    ex = [O.rand_qlin(256, 192, 50 + e) for e in range(3)]
    ex_slabs = np.stack([O.mlx_to_slab(a, b) for a, b in ex])
    path = os.path.join(tmp_path, "layer0.bin")
    pk.write_weight_file(path, MAGIC, 0, 3, [slab.tobytes(), ex_slabs.tobytes()])
    d = torch.device("cuda")
    with pk.WeightFile(path, MAGIC, 0, 3) as f:
        p = pk.load_q4_projection(f.q4_projection(out, inp, "proj"), out, inp, d)
        e = pk.load_expert_q4_projection(f.expert_q4_projection(3, 256, 192, "experts"), 256, 192, d)
        f.finish()
    ref = thq4.PackedWeight.repack(thq4.SRC_MLX, dev(wq), dev(sb), out, inp, thq4.BF16)
    assert torch.equal(p.qw, ref.qw) and torch.equal(p.sb, ref.sb), "package projection != MLX repack"
    ref_e = thq4.PackedExperts.from_mlx(dev(np.stack([a for a, _ in ex])), dev(np.stack([b for _, b in ex])),
                                        thq4.BF16)
    assert torch.equal(e.qw, ref_e.qw) and torch.equal(e.sb, ref_e.sb), "package experts != MLX repack"
    x = O.rand_x(inp, 9)
    y = torch.empty((1, out), dtype=torch.float32, device=d)
    ws = thq4.qlin.workspace(p.desc, d)
    L = thq4.lib()
    thq4.check(L.thq4_linear(ctypes.byref(p.desc), ctypes.c_void_p(dev(x.reshape(1, inp)).data_ptr()), thq4.BF16, 1,
                             ctypes.c_void_p(y.data_ptr()), thq4.F32, ctypes.c_void_p(ws.data_ptr()), ws.numel(),
                             ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    want = O.linear_group(wq, sb, O.SB_BF16, O.bf16_to_f32(x).reshape(1, inp))[0]
    assert_close_ref("package projection", y.cpu().numpy().ravel(), want)


def test_package_q8_router_scores(tmp_path):
    """A Q8 section loaded from a package is the router the library reads
    as stored: its scores equal the oracle's bit for bit."""
    out, inp, T = 256, 1024, 12
    rng = np.random.default_rng(3)
    q = rng.integers(0, 256, out * inp, dtype=np.uint8)
    sc = O.f32_to_bf16(rng.uniform(0.0005, 0.004, out * inp // 64).astype(np.float32))
    bi = O.f32_to_bf16((rng.standard_normal(out * inp // 64) * 0.05).astype(np.float32))
    path = os.path.join(tmp_path, "router.bin")
    pk.write_weight_file(path, MAGIC, 0, 5, [np.concatenate([q, sc.view(np.uint8), bi.view(np.uint8)]).tobytes()])
    with pk.WeightFile(path, MAGIC, 0, 5) as f:
        r = pk.load_q8_projection(f.q8_projection(out, inp, "router"), out, inp, torch.device("cuda"))
        f.finish()
    x = O.f32_to_bf16(rng.standard_normal((T, inp)).astype(np.float32))
    got = thq4.moe_scores_q8(dev(x).view(torch.bfloat16), r, 256)
    want = O.moe_scores_q8(x, q, sc, bi, 256)
    assert np.array_equal(got.cpu().view(torch.int16).numpy().view(np.uint16), want)
