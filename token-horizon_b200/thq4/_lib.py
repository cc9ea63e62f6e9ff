"""ctypes binding of libthq4.so, the C ABI declared in include/thq4.h.

The library is built in-tree by token-horizon_b200/build.py.  Loading fails
loudly when it is missing: there is no CPU fallback for any operator.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_int, c_size_t, c_uint32, c_void_p

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libthq4.so")

# thq4_status
OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_UNSUPPORTED = 2
ERR_WORKSPACE = 3
ERR_CUDA = 4
ERR_NCCL = 5

# thq4_dtype
BF16 = 0
F16 = 1
F32 = 2
PRESUM = 3

# thq4_src_layout
SRC_MLX = 0
SRC_TILED = 1
SRC_SLAB = 2
SRC_FRAG = 3


class Thq4Error(RuntimeError):
    """A thq4 call returned a non-OK status; `status` holds the code."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class thq4_weight(ctypes.Structure):
    _fields_ = [("out", ctypes.c_int32), ("in_", ctypes.c_int32), ("gs", ctypes.c_int32),
                ("sb_dtype", ctypes.c_int32), ("qw", c_void_p), ("sb", c_void_p)]


class thq4_experts(ctypes.Structure):
    _fields_ = [("experts", ctypes.c_int32), ("out", ctypes.c_int32), ("in_", ctypes.c_int32),
                ("gs", ctypes.c_int32), ("sb_dtype", ctypes.c_int32), ("reserved", ctypes.c_int32),
                ("qw", c_void_p), ("sb", c_void_p), ("qw_stride", ctypes.c_uint64),
                ("sb_stride", ctypes.c_uint64)]


class thq4_q8_weight(ctypes.Structure):
    _fields_ = [("out", ctypes.c_int32), ("in_", ctypes.c_int32), ("q", c_void_p), ("scales", c_void_p),
                ("biases", c_void_p)]


class thq4_moe_weights(ctypes.Structure):
    _fields_ = [("router", thq4_q8_weight), ("gate", thq4_experts), ("up", thq4_experts), ("down", thq4_experts),
                ("shared_gate", thq4_experts), ("shared_up", thq4_experts), ("shared_down", thq4_experts),
                ("shared_expert_gate", thq4_q8_weight)]


class thq4_peer_gather(ctypes.Structure):
    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32), ("rows", ctypes.c_int32),
                ("offset", ctypes.c_int32), ("stride", ctypes.c_int32), ("wait", ctypes.c_int32),
                ("dst", c_void_p), ("flags", c_void_p), ("count", c_void_p), ("arrive", c_void_p),
                ("out_mode", ctypes.c_int32), ("x_parts", ctypes.c_int32), ("slot", ctypes.c_int64),
                ("x_slot", ctypes.c_int64), ("x_ll", ctypes.c_int32), ("reserved", ctypes.c_int32)]


class thq4_chain_op(ctypes.Structure):
    _fields_ = [("w", c_void_p), ("up", c_void_p), ("x", c_void_p), ("y", c_void_p), ("y_dtype", ctypes.c_int32),
                ("reserved", ctypes.c_int32)]


IPC_HANDLE_BYTES = 64

_lib = None

# name -> (restype, argtypes); every symbol include/thq4.h declares
SIGNATURES = {
    "thq4_version": (c_char_p, []),
    "thq4_last_error": (c_size_t, [c_void_p, c_size_t]),
    "thq4_device_status": (c_int, [POINTER(c_uint32), c_void_p]),
    "thq4_weight_bytes": (c_size_t, [c_int, c_int, c_int, POINTER(c_size_t), POINTER(c_size_t)]),
    "thq4_repack": (c_int, [c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int,
                            c_void_p, c_size_t, c_void_p, c_size_t, c_void_p]),
    "thq4_weight_init": (c_int, [POINTER(thq4_weight), c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
    "thq4_linear": (c_int, [POINTER(thq4_weight), c_void_p, c_int, c_int, c_void_p, c_int, c_void_p,
                            c_size_t, c_void_p]),
    "thq4_linear_noalloc": (c_int, [POINTER(thq4_weight), c_void_p, c_int, c_int, c_void_p, c_int, c_void_p]),
    "thq4_gate_up": (c_int, [POINTER(thq4_weight), POINTER(thq4_weight), c_void_p, c_int, c_int, c_void_p,
                             c_int, c_void_p, c_size_t, c_void_p]),
    "thq4_linear_workspace_bytes": (c_size_t, [POINTER(thq4_weight), c_int]),
    "thq4_linear_scalar": (c_int, [POINTER(thq4_weight), c_void_p, c_int, c_int, c_void_p, c_int, c_void_p]),
    "thq4_dequant": (c_int, [POINTER(thq4_weight), c_void_p, c_void_p]),
    "thq4_moe_max_tiles": (c_uint32, [c_int, c_int, c_int]),
    "thq4_moe_route": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                               c_void_p, c_int, c_void_p]),
    "thq4_moe_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int]),
    "thq4_moe": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, POINTER(thq4_experts),
                         POINTER(thq4_experts), POINTER(thq4_experts), c_void_p, c_void_p, c_size_t, c_void_p]),
    "thq4_moe_partial": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                                 POINTER(thq4_experts), POINTER(thq4_experts), POINTER(thq4_experts), c_void_p,
                                 c_void_p, c_size_t, c_void_p]),
    "thq4_moe_scores_workspace_bytes": (c_size_t, [c_int, c_int]),
    "thq4_moe_scores_q8": (c_int, [c_void_p, c_int, POINTER(thq4_q8_weight), c_int, c_void_p, c_int, c_void_p,
                                   c_size_t, c_void_p]),
    "thq4_moe_add_max_tiles": (c_uint32, [c_int, c_int, c_int, c_int]),
    "thq4_moe_route_q8": (c_int, [c_void_p, c_int, c_int, c_int, POINTER(thq4_q8_weight), POINTER(thq4_q8_weight),
                                  c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p,
                                  c_size_t, c_void_p]),
    "thq4_moe_add_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int, c_int]),
    "thq4_moe_add_partial_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                                                        c_int]),
    "thq4_moe_add": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, POINTER(thq4_moe_weights),
                             c_void_p, c_void_p, c_size_t, c_void_p]),
    "thq4_moe_add_partial": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                                     POINTER(thq4_moe_weights), c_void_p, c_void_p, c_size_t, c_void_p]),
    "thq4_linear_peer": (c_int, [POINTER(thq4_weight), POINTER(thq4_weight), c_void_p, c_int, c_int, c_void_p,
                                 c_void_p, c_size_t, POINTER(thq4_peer_gather), c_void_p]),
    "thq4_peer_wait": (c_int, [POINTER(thq4_peer_gather), c_void_p]),
    "thq4_ipc_alloc": (c_int, [c_size_t, POINTER(c_void_p), c_void_p]),
    "thq4_ipc_open": (c_int, [c_void_p, POINTER(c_void_p)]),
    "thq4_ipc_close": (c_int, [c_void_p]),
    "thq4_ipc_free": (c_int, [c_void_p]),
    "thq4_copy": (c_int, [c_void_p, c_void_p, c_size_t, c_void_p]),
    "thq4_linear_chain_workspace_bytes": (c_size_t, [c_void_p, c_int]),
    "thq4_linear_chain": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "thq4_presum_block_bytes": (c_size_t, [c_int]),
    "thq4_presum_attach": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p]),
    "thq4_add_rms_norm": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, ctypes.c_float, c_void_p, c_void_p,
                                  c_void_p]),
    "thq4_debug_set_gemv": (c_int, [c_int, c_int, c_int, c_int]),
    "thq4_debug_set_trace": (c_int, [c_void_p, c_size_t]),
    "thq4_debug_gemv_plan": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
    "thq4_debug_prefill_plan": (c_int, [c_int, c_int, c_int, c_int, c_int, c_void_p]),
}


def lib():
    """The loaded library; raises if libthq4.so was not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise Thq4Error(ERR_UNSUPPORTED,
                            f"{LIB_PATH} is missing: build it with `python token-horizon_b200/build.py`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name, None)
            if f is None:
                continue
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    L = lib()
    n = L.thq4_last_error(None, 0)
    buf = ctypes.create_string_buffer(n + 1)
    L.thq4_last_error(buf, n + 1)
    return buf.value.decode(errors="replace")


def check(status: int) -> None:
    if status != OK:
        raise Thq4Error(status, last_error())


def version() -> str:
    return lib().thq4_version().decode()
