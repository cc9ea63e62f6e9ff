"""Splash packed weight files (docs/splash/runtime/model/WeightStore.cpp) on
the host: a package written from oracle-made slabs reads back byte for byte,
its Q4 sections convert back to the MLX arrays they came from, and every
malformed file is rejected with the reference's message."""
import os

import numpy as np
import pytest

import q4oracle as O
from thq4 import package as pk

MAGIC = b"THQ4TEST"


def _proj(out, inp, seed):
    wq, sb = O.rand_qlin(out, inp, seed)
    return wq, sb, O.mlx_to_slab(wq, sb)


def test_round_trip(tmp_path):
    wq, sb, slab = _proj(512, 320, 3)
    experts = [_proj(256, 128, 10 + e) for e in range(3)]
    ex = np.concatenate([s for _, _, s in experts])
    path = os.path.join(tmp_path, "layer.bin")
    pk.write_weight_file(path, MAGIC, 7, 2, [slab.tobytes(), ex.tobytes()])
    assert os.path.getsize(path) % pk.ALIGNMENT == 0
    with pk.WeightFile(path, MAGIC, 7, 2) as f:
        got = f.q4_projection(512, 320, "attn")
        assert np.array_equal(got, slab)
        w2, s2 = O.slab_to_mlx(got, 512, 320)
        assert np.array_equal(w2, wq) and np.array_equal(s2, sb)
        gx = f.expert_q4_projection(3, 256, 128, "experts")
        for e, (ew, es, eslab) in enumerate(experts):
            assert np.array_equal(gx[e], eslab)
        f.finish()


def test_sizes_follow_the_reference():
    assert pk.q4_packed_bytes(256, 64) == 256 * 64 // 16 * 9
    assert pk.q4_packed_bytes(12288, 4096) == 28311552  # 9/16 byte per element
    with pytest.raises(pk.WeightFileError, match="StorageN=256"):
        pk.validate_q4_layout(300, 64)
    with pytest.raises(pk.WeightFileError, match="input-aligned"):
        pk.validate_q4_layout(256, 100)


@pytest.mark.parametrize("case,msg", [
    ("magic", "header mismatch"), ("layer", "header mismatch"), ("unaligned", "16 KiB-aligned"),
    ("truncated", "truncated at section"), ("unconsumed", "unconsumed or missing"),
    ("after_finish", "after packed file finish"), ("empty", "must not be empty"),
])
def test_malformed_files_are_rejected(tmp_path, case, msg):
    _, _, slab = _proj(256, 64, 5)
    path = os.path.join(tmp_path, "bad.bin")
    pk.write_weight_file(path, MAGIC, 1, 1, [slab.tobytes()])
    if case == "unaligned":
        with open(path, "ab") as f:
            f.write(b"\0" * 100)
    with pytest.raises(pk.WeightFileError, match=msg):
        f = pk.WeightFile(path, b"OTHERMAG" if case == "magic" else MAGIC, 2 if case == "layer" else 1, 1)
        if case == "truncated":
            f.q4_projection(256, 64, "a")
            f.q4_projection(256 * 64, 64, "b")
        elif case == "unconsumed":
            f.finish()
        elif case == "after_finish":
            f.q4_projection(256, 64, "a")
            f.finish()
            f.section(16, "late")
        elif case == "empty":
            f.section(0, "nothing")


def test_q8_section_round_trip(tmp_path):
    # readQ8Projection (WeightStore.cpp:264-282): weights, scales, biases in one section
    out, inp = 256, 512
    rng = np.random.default_rng(2)
    q = rng.integers(0, 256, out * inp, dtype=np.uint8)
    sc = rng.integers(0, 1 << 16, out * inp // 64, dtype=np.uint16)
    bi = rng.integers(0, 1 << 16, out * inp // 64, dtype=np.uint16)
    sec = np.concatenate([q, sc.view(np.uint8), bi.view(np.uint8)])
    assert sec.size == pk.q8_packed_bytes(out, inp) == out * inp + out * inp // 32 * 2
    _, _, slab = _proj(256, 64, 5)
    path = os.path.join(tmp_path, "moe.bin")
    pk.write_weight_file(path, MAGIC, 3, 4, [sec.tobytes(), slab.tobytes()])
    with pk.WeightFile(path, MAGIC, 3, 4) as f:
        got = f.q8_projection(out, inp, "router")
        assert np.array_equal(got, sec)
        f.q4_projection(256, 64, "next")
        f.finish()
    with pytest.raises(pk.WeightFileError, match="input-aligned"):
        pk.q8_packed_bytes(256, 100)
