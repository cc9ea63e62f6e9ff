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
