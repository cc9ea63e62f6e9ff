"""Host-side mirror of th-engine's quant-linear operator (QLin) over the C ABI.

The reference's operator surface is ``QLin`` in engine/src/qwen35.rs:303-923:
``QLin::new`` (:320), ``tiled`` (:629-697), ``linear`` / ``linear_ps``
(:389-617), ``gate_up_act`` / ``gate_up_act_ps`` (:704-884), ``fuse_lins``
(:1581-1610), ``maybe_tiled`` (:890-898) and ``lin_apply`` / ``lin_apply_ps``
(:912-923).  This module keeps those names, argument meanings and error
messages; the arithmetic runs in libthq4.so (include/thq4.h).  torch provides
device memory and the current stream only.

Shapes follow the reference: ``wq`` u32 [out, in/8] (MLX nibbles, LSB first)
and ``sb`` [out, 2*ng] (a row's scales then its biases), bf16 or f16.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Sequence

import torch

from . import _lib
from ._lib import BF16, F16, F32, SRC_MLX, SRC_SLAB, SRC_TILED, Thq4Error, check, thq4_weight

_SB_DTYPE = {torch.bfloat16: BF16, torch.float16: F16}
_X_DTYPE = {torch.bfloat16: BF16, torch.float32: F32}


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


_WORKSPACES: dict = {}


def workspace(desc, device: torch.device, m: int = 1) -> torch.Tensor:
    """A zero-filled workspace big enough for `desc` at `m` rows, cached per
    device and stream (the kernels leave its counters zeroed after every
    call; at m > 8 it also holds the prefill's stream-K parts)."""
    need = _lib.lib().thq4_linear_workspace_bytes(ctypes.byref(desc), m)
    key = (device.index if device.index is not None else torch.cuda.current_device(),
           torch.cuda.current_stream(device).cuda_stream)
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.zeros(max(need, 1 << 20), dtype=torch.uint8, device=device)
        _WORKSPACES[key] = ws
    return ws


class PackedWeight:
    """One frag weight (rows x in) resident on the device."""

    def __init__(self, rows: int, inp: int, sb_dtype: int, device: torch.device):
        qb, sbb = ctypes.c_size_t(), ctypes.c_size_t()
        _lib.lib().thq4_weight_bytes(rows, inp, 64, ctypes.byref(qb), ctypes.byref(sbb))
        self.rows, self.inp, self.sb_dtype = rows, inp, sb_dtype
        self.qw = torch.empty(qb.value, dtype=torch.uint8, device=device)
        self.sb = torch.empty(sbb.value, dtype=torch.uint8, device=device)
        self.desc = thq4_weight()
        check(_lib.lib().thq4_weight_init(ctypes.byref(self.desc), rows, inp, 64, sb_dtype,
                                          _ptr(self.qw), _ptr(self.sb)))

    @property
    def nbytes(self) -> int:
        return self.qw.numel() + self.sb.numel()

    @classmethod
    def repack(cls, layout: int, w: torch.Tensor, sb: Optional[torch.Tensor], src_out: int, inp: int,
               sb_dtype: int, row_begin: int = 0, rows: Optional[int] = None) -> "PackedWeight":
        rows = src_out - row_begin if rows is None else rows
        p = cls(rows, inp, sb_dtype, w.device)
        check(_lib.lib().thq4_repack(layout, _ptr(w), _ptr(sb), src_out, inp, 64, sb_dtype, row_begin, rows,
                                     _ptr(p.qw), p.qw.numel(), _ptr(p.sb), p.sb.numel(), _stream()))
        return p


class QLin:
    """Packed Q4 projection; mirror of ``QLin`` (qwen35.rs:303-325).

    ``tiled`` is True once the weight is packed in the kernels' layout (the
    reference's Splash tile layout becomes this library's frag layout).
    """

    def __init__(self, wq: torch.Tensor, sb: torch.Tensor, out: int, inp: int, gs: int = 64):
        # QLin::new (qwen35.rs:320-324)
        self.wq, self.sb = wq, sb
        self.out, self.inp, self.gs = out, inp, gs
        self.tiled_flag = False
        self.sb_dtype = _SB_DTYPE.get(sb.dtype)
        if self.sb_dtype is None:
            raise Thq4Error(_lib.ERR_INVALID_ARGUMENT, f"QLin: scale/bias dtype {sb.dtype} is not bf16 or f16")
        self.packed: Optional[PackedWeight] = None
        # fused [gate | up]: the two halves packed separately (see tiled)
        self.up_row = 0
        self.packed_gate: Optional[PackedWeight] = None
        self.packed_up: Optional[PackedWeight] = None

    new = classmethod(lambda cls, wq, sb, out, inp, gs: cls(wq, sb, out, inp, gs))

    @classmethod
    def from_layout(cls, layout: int, w: torch.Tensor, sb: Optional[torch.Tensor], out: int, inp: int,
                    sb_dtype: int) -> "QLin":
        """A QLin straight from a reference layout (SRC_TILED / SRC_SLAB)."""
        q = cls.__new__(cls)
        q.wq, q.sb, q.out, q.inp, q.gs = None, None, out, inp, 64
        q.sb_dtype, q.up_row = sb_dtype, 0
        q.packed = PackedWeight.repack(layout, w, sb, out, inp, sb_dtype)
        q.packed_gate = q.packed_up = None
        q.tiled_flag = True
        return q

    def tiled(self, up_row: int = 0) -> "QLin":
        """Repack for the kernels (QLin::tiled, qwen35.rs:629-697).  With
        ``up_row`` > 0 the weight is a fused [gate | up] and the halves
        [0, up_row) and [up_row, out) are packed as separate weights so that
        the up stream may start anywhere (the reference allows any up_row)."""
        if self.tiled_flag and (up_row == 0 or self.packed_gate is not None):
            return self
        if self.gs != 64 or self.inp % 64 != 0:
            raise Thq4Error(_lib.ERR_UNSUPPORTED, f"QLin::tiled: group size {self.gs}, inp {self.inp}")
        wq = self.wq.contiguous()
        sb = self.sb.contiguous()
        self.packed = PackedWeight.repack(SRC_MLX, wq, sb, self.out, self.inp, self.sb_dtype)
        if up_row > 0:
            half = self.out - up_row
            self.packed_gate = PackedWeight.repack(SRC_MLX, wq, sb, self.out, self.inp, self.sb_dtype, 0, up_row)
            self.packed_up = PackedWeight.repack(SRC_MLX, wq, sb, self.out, self.inp, self.sb_dtype, up_row, half)
            self.up_row = up_row
        self.tiled_flag = True
        return self

    # -- QLin::linear_ps (qwen35.rs:398-617) -----------------------------------
    def linear(self, x: torch.Tensor) -> torch.Tensor:
        return self.linear_ps(x, False)

    def linear_ps(self, x: torch.Tensor, presum: bool = False, out_dtype: Optional[torch.dtype] = None,
                  out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """x [..., in] -> y [..., out].  With ``presum`` x is the live [m, in]
        view of a presum block (presum_block / add_rms_norm, m <= 8): the
        kernel takes each group's sum for the bias term from the block."""
        if presum:
            _check_presum_view(x, self.inp, "affine-qmpp")
        dims = list(x.shape)
        in_d = dims[-1]
        rows = 1
        for d in dims[:-1]:
            rows *= d
        if in_d != self.inp:
            raise Thq4Error(_lib.ERR_INVALID_ARGUMENT,
                            f"QLin::linear: x last dim {in_d} != weight inp {self.inp} (x {dims})")
        if not self.tiled_flag:
            self.tiled()
        x_dtype = _lib.PRESUM if presum else _X_DTYPE.get(x.dtype)
        if x_dtype is None:
            raise Thq4Error(_lib.ERR_INVALID_ARGUMENT, f"QLin::linear: x dtype {x.dtype} is not bf16 or f32")
        xv = x if presum else x.reshape(rows, in_d).contiguous()
        ydt = out_dtype or (torch.float32 if x.dtype == torch.float32 else torch.bfloat16)
        y = out if out is not None else torch.empty((rows, self.out), dtype=ydt, device=x.device)
        ws = workspace(self.packed.desc, x.device, rows)
        check(_lib.lib().thq4_linear(ctypes.byref(self.packed.desc), _ptr(xv), x_dtype, rows, _ptr(y),
                                     F32 if y.dtype == torch.float32 else BF16, _ptr(ws), ws.numel(), _stream()))
        return y.reshape(dims[:-1] + [self.out])

    # -- QLin::gate_up_act_ps (qwen35.rs:711-884) -------------------------------
    def gate_up_act(self, x: torch.Tensor) -> Optional[torch.Tensor]:
        r = self.gate_up_act_ps(x, False)
        return None if r is None else r[0]

    def gate_up_act_ps(self, x: torch.Tensor, presum: bool = False, up_row: Optional[int] = None,
                       out: Optional[torch.Tensor] = None):
        """Fused [gate | up] -> silu(bf16 g) * bf16 u, [..., half].  Returns
        (tensor, emitted_presum) like the reference; the flag is always False
        (the down projection's block comes from presum_block when wanted).
        With ``presum`` x is the live view of a presum block."""
        if presum:
            _check_presum_view(x, self.inp, "affine-qmpp gate_up")
        if self.out % 2 != 0 and up_row is None:
            return None
        half = self.out // 2 if up_row is None else self.out - up_row
        up_row = self.out - half
        dims = list(x.shape)
        rows = 1
        for d in dims[:-1]:
            rows *= d
        if dims[-1] != self.inp:
            raise Thq4Error(_lib.ERR_INVALID_ARGUMENT,
                            f"QLin::gate_up_act: x last dim {dims[-1]} != weight inp {self.inp} (x {dims})")
        if self.packed_gate is None or self.up_row != up_row:
            if self.wq is None:
                raise Thq4Error(_lib.ERR_UNSUPPORTED, "QLin::gate_up_act: weight was not built from MLX tensors")
            self.tiled_flag = False
            self.tiled(up_row)
        x_dtype = _lib.PRESUM if presum else _X_DTYPE.get(x.dtype)
        if x_dtype is None:
            raise Thq4Error(_lib.ERR_INVALID_ARGUMENT, f"QLin::gate_up_act: x dtype {x.dtype}")
        xv = x if presum else x.reshape(rows, dims[-1]).contiguous()
        y = out if out is not None else torch.empty((rows, half), dtype=torch.bfloat16, device=x.device)
        ws = workspace(self.packed_gate.desc, x.device)
        check(_lib.lib().thq4_gate_up(ctypes.byref(self.packed_gate.desc), ctypes.byref(self.packed_up.desc),
                                      _ptr(xv), x_dtype, rows, _ptr(y),
                                      F32 if y.dtype == torch.float32 else BF16, _ptr(ws), ws.numel(), _stream()))
        return y.reshape(dims[:-1] + [half]), False

    def dequant(self) -> torch.Tensor:
        """bf16 [out, in] (AffineDequant, quant_kernel.rs:1765-1781)."""
        if not self.tiled_flag:
            self.tiled()
        y = torch.empty((self.out, self.inp), dtype=torch.bfloat16, device=self.packed.qw.device)
        check(_lib.lib().thq4_dequant(ctypes.byref(self.packed.desc), _ptr(y), _stream()))
        return y


# -- presum blocks (quant_kernel.rs:265-318, 3642-3657) ---------------------------

def presum_block_bytes(inp: int) -> int:
    return int(_lib.lib().thq4_presum_block_bytes(inp))


def _check_presum_view(x: torch.Tensor, inp: int, who: str) -> None:
    """The reference's check that x is the live [m, in] view of a whole presum
    block (quant_kernel.rs:3642-3657)."""
    need = x.storage_offset() * 2 + presum_block_bytes(inp)
    have = x.untyped_storage().nbytes()
    m = x.numel() // inp if inp else 0
    if (x.dtype != torch.bfloat16 or not x.is_contiguous() or (x.storage_offset() * 2) % 16 != 0 or have < need
            or x.numel() != m * inp or not 1 <= m <= 8):
        raise Thq4Error(_lib.ERR_INVALID_ARGUMENT,
                        f"{who}: presum block missing (x_off {x.storage_offset() * 2}, buffer {have} < {need}, "
                        f"x {list(x.shape)}, m {m})")


def presum_block(x: torch.Tensor):
    """Q4AttachSums: x [m, in] bf16 (m <= 8) as a presum block.  Returns the
    block (uint8, presum_block_bytes(in)) and the [m, in] view of its rows."""
    m, inp = x.shape
    block = torch.empty(presum_block_bytes(inp), dtype=torch.uint8, device=x.device)
    xc = x.contiguous()
    check(_lib.lib().thq4_presum_attach(_ptr(xc), m, inp, _ptr(block), _stream()))
    return block, block[:m * inp * 2].view(torch.bfloat16).view(m, inp)


def add_rms_norm(x: torch.Tensor, r: torch.Tensor, w: torch.Tensor, eps: float):
    """AddRmsNorm { sums } (gdn_kernel.rs:1851-1866): res = bf16(x + r) and the
    normed rows as a presum block.  Returns (res [T, C], block, the [T, C]
    view of the block's normed rows)."""
    T, C = x.shape
    res = torch.empty_like(x)
    block = torch.empty(presum_block_bytes(C), dtype=torch.uint8, device=x.device)
    check(_lib.lib().thq4_add_rms_norm(_ptr(x.contiguous()), _ptr(r.contiguous()), _ptr(w.contiguous()), T, C,
                                       ctypes.c_float(eps), _ptr(res), _ptr(block), _stream()))
    return res, block, block[:T * C * 2].view(torch.bfloat16).view(T, C)


def fuse_lins(lins: Sequence[QLin]) -> QLin:
    """Concatenate packed projections along out (qwen35.rs:1581-1610)."""
    wq = torch.cat([l.wq for l in lins], 0)
    sb = torch.cat([l.sb for l in lins], 0)
    return QLin(wq, sb, sum(l.out for l in lins), lins[0].inp, lins[0].gs)


def maybe_tiled(l: QLin) -> QLin:
    """The reference tiles by default (qwen35.rs:890-898)."""
    return l.tiled()


def lin_apply_ps(x: torch.Tensor, l: QLin, presum: bool = False) -> torch.Tensor:
    return l.linear_ps(x, presum)


def lin_apply(x: torch.Tensor, l: QLin) -> torch.Tensor:
    return lin_apply_ps(x, l, False)


# -- MoE (Splash MoE::add, docs/splash/runtime/ops/MoE.cpp:119-231) ------------

class LinearChain:
    """Dependent projections in one persistent launch (thq4_linear_chain).

    ``ops`` is a list of (w, up, x, y): a PackedWeight (the gate half of a
    gate/up op), the up half or None, and the op's input and output tensors
    ([m, w.in] of the chain's x dtype, [m, w.out] bf16 or f32).  An op may
    read any earlier op's output.  The descriptors and the workspace are built
    once, so calling the chain again (or capturing it in a CUDA graph) reuses
    them."""

    def __init__(self, ops, m: int = 1, x_dtype: int = _lib.BF16, device: Optional[torch.device] = None):
        self.n = len(ops)
        self.m = m
        self.x_dtype = x_dtype
        self._keep = list(ops)
        self._arr = (_lib.thq4_chain_op * max(self.n, 1))()
        for i, (w, up, x, y) in enumerate(ops):
            o = self._arr[i]
            o.w = ctypes.addressof(w.desc)
            o.up = ctypes.addressof(up.desc) if up is not None else None
            o.x = x.data_ptr()
            o.y = y.data_ptr()
            o.y_dtype = _lib.F32 if y.dtype == torch.float32 else _lib.BF16
            o.reserved = 0
        need = _lib.lib().thq4_linear_chain_workspace_bytes(self._arr, self.n)
        dev = device if device is not None else ops[0][2].device
        self.ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=dev)

    def __call__(self) -> None:
        check(_lib.lib().thq4_linear_chain(self._arr, self.n, self.x_dtype, self.m, _ptr(self.ws), self.ws.numel(),
                                           _stream()))


class PackedExperts:
    """E experts of one shape (rows x inp), packed back to back in the frag
    layout; the host mirror of Splash's ExpertQ4Projection
    (docs/splash/runtime/ops/Linear.hpp:37-43)."""

    def __init__(self, experts: int, rows: int, inp: int, sb_dtype: int, device: torch.device):
        qb, sbb = ctypes.c_size_t(), ctypes.c_size_t()
        _lib.lib().thq4_weight_bytes(rows, inp, 64, ctypes.byref(qb), ctypes.byref(sbb))
        self.experts, self.rows, self.inp, self.sb_dtype = experts, rows, inp, sb_dtype
        self.qw_stride, self.sb_stride = qb.value, sbb.value
        self.qw = torch.empty(experts * qb.value, dtype=torch.uint8, device=device)
        self.sb = torch.empty(experts * sbb.value, dtype=torch.uint8, device=device)
        self.desc = _lib.thq4_experts()
        self.desc.experts, self.desc.out, self.desc.in_, self.desc.gs = experts, rows, inp, 64
        self.desc.sb_dtype, self.desc.reserved = sb_dtype, 0
        self.desc.qw, self.desc.sb = self.qw.data_ptr(), self.sb.data_ptr()
        self.desc.qw_stride, self.desc.sb_stride = qb.value, sbb.value

    @classmethod
    def from_mlx(cls, wq: torch.Tensor, sb: torch.Tensor, sb_dtype: int, row_begin: int = 0,
                 rows: Optional[int] = None) -> "PackedExperts":
        """wq u32 [E, src_out, inp/8], sb [E, src_out, 2*inp/64]: rows
        [row_begin, row_begin + rows) of every expert (e.g. the gate or the up
        half of a fused [gate | up] expert)."""
        E, src_out, inp = wq.shape[0], wq.shape[1], wq.shape[2] * 8
        rows = src_out - row_begin if rows is None else rows
        p = cls(E, rows, inp, sb_dtype, wq.device)
        for e in range(E):
            check(_lib.lib().thq4_repack(SRC_MLX, _ptr(wq[e].contiguous()), _ptr(sb[e].contiguous()), src_out, inp, 64,
                                         sb_dtype, row_begin, rows,
                                         ctypes.c_void_p(p.qw.data_ptr() + e * p.qw_stride), p.qw_stride,
                                         ctypes.c_void_p(p.sb.data_ptr() + e * p.sb_stride), p.sb_stride, _stream()))
        return p



def _experts_from_slabs(cls, slabs: torch.Tensor, out: int, inp: int, sb_dtype: int) -> "PackedExperts":
    """slabs u8 [E, out*inp/16*9] on the device: Splash expert slabs (a
    package's expert section, docs/splash/runtime/model/WeightStore.cpp:
    284-299), repacked expert by expert (THQ4_SRC_SLAB)."""
    E = slabs.shape[0]
    p = cls(E, out, inp, sb_dtype, slabs.device)
    for e in range(E):
        check(_lib.lib().thq4_repack(SRC_SLAB, _ptr(slabs[e].contiguous()), None, out, inp, 64, sb_dtype, 0, out,
                                     ctypes.c_void_p(p.qw.data_ptr() + e * p.qw_stride), p.qw_stride,
                                     ctypes.c_void_p(p.sb.data_ptr() + e * p.sb_stride), p.sb_stride, _stream()))
    return p


PackedExperts.from_slabs = classmethod(_experts_from_slabs)

_MOE_WS: dict = {}


def moe_route(logits: torch.Tensor, k: int):
    """Device routing (moe.metal:270-449): ids [T, k] u32, weights [T, k] bf16,
    tiles [n, 2] u32, grouped_routes [n*32] u32, route_rows [T*k] u32."""
    T, E = logits.shape
    L = _lib.lib()
    mt = L.thq4_moe_max_tiles(T, E, k)
    dev = logits.device
    ids = torch.empty((T, k), dtype=torch.int32, device=dev)
    w = torch.empty((T, k), dtype=torch.bfloat16, device=dev)
    tiles = torch.empty((mt, 2), dtype=torch.int32, device=dev)
    grouped = torch.empty(mt * 32, dtype=torch.int32, device=dev)
    rows = torch.empty(T * k, dtype=torch.int32, device=dev)
    n = torch.zeros(1, dtype=torch.int32, device=dev)
    check(L.thq4_moe_route(_ptr(logits.contiguous()), T, E, k, _ptr(ids), _ptr(w), _ptr(tiles), _ptr(grouped),
                           _ptr(rows), _ptr(n), mt, _stream()))
    nt = int(n.item())
    return ids, w, tiles[:nt], grouped[:nt * 32], rows


def moe_partial(x: torch.Tensor, logits: torch.Tensor, k: int, e0: int, gate: PackedExperts, up: PackedExperts,
                down: PackedExperts, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """An expert shard's part of one MoE layer: gate/up/down hold experts
    [e0, e0 + gate.experts) of logits.shape[1]; returns f32 [T, H] (plus the
    residual where given).  The layer's output is the ranks' sum, rounded
    once to bf16."""
    T, H = x.shape
    E = logits.shape[1]
    El, I = gate.experts, gate.rows
    L = _lib.lib()
    need = L.thq4_moe_workspace_bytes(T, H, I, El, k)
    key = ("partial", x.device.index, torch.cuda.current_stream(x.device).cuda_stream)
    ws = _MOE_WS.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.empty(need, dtype=torch.uint8, device=x.device)
        _MOE_WS[key] = ws
    y = torch.empty((T, H), dtype=torch.float32, device=x.device)
    check(L.thq4_moe_partial(_ptr(x.contiguous()), _ptr(residual), _ptr(logits.contiguous()), T, H, I, E, k, e0,
                             e0 + El, ctypes.byref(gate.desc), ctypes.byref(up.desc), ctypes.byref(down.desc), _ptr(y),
                             _ptr(ws), ws.numel(), _stream()))
    return y


def moe(x: torch.Tensor, logits: torch.Tensor, k: int, gate: PackedExperts, up: PackedExperts,
        down: PackedExperts, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One MoE layer: residual + sum_slot w * down(silu(gate x) * up x), bf16 [T, H]."""
    T, H = x.shape
    E, I = gate.experts, gate.rows
    L = _lib.lib()
    need = L.thq4_moe_workspace_bytes(T, H, I, E, k)
    key = (x.device.index, torch.cuda.current_stream(x.device).cuda_stream)
    ws = _MOE_WS.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.empty(need, dtype=torch.uint8, device=x.device)
        _MOE_WS[key] = ws
    y = torch.empty((T, H), dtype=torch.bfloat16, device=x.device)
    check(L.thq4_moe(_ptr(x.contiguous()), _ptr(residual), _ptr(logits.contiguous()), T, H, I, E, k,
                     ctypes.byref(gate.desc), ctypes.byref(up.desc), ctypes.byref(down.desc), _ptr(y), _ptr(ws),
                     ws.numel(), _stream()))
    return y


# -- the Splash MoE block: Q8 router and shared expert (MoE.hpp:15-44) ----------

class Q8Projection:
    """Splash's Q8Projection (docs/splash/runtime/ops/Linear.hpp:27-33): 8-bit
    affine weights in StorageN = 256 order -- the byte of output n and input
    k at ((k/64)*256 + n)*64 + k%64, the bf16 scale and bias at (k/64)*256 +
    n -- on the device.  Used as the MoE router and the shared expert's
    scalar gate (row 0)."""

    def __init__(self, q: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, inp: int, out: int = 256):
        self.q = q.contiguous().view(torch.uint8)
        self.scales = scales.contiguous()
        self.biases = biases.contiguous()
        self.out, self.inp = out, inp
        self.desc = _lib.thq4_q8_weight(out, inp, self.q.data_ptr(), self.scales.data_ptr(), self.biases.data_ptr())

    @classmethod
    def from_section(cls, packed: torch.Tensor, inp: int, out: int = 256) -> "Q8Projection":
        """One package section (out*inp weight bytes, then the bf16 scales,
        then the bf16 biases: WeightStore.cpp:264-282) on the device."""
        elements = out * inp
        pb = elements // 32
        packed = packed.contiguous().view(torch.uint8)
        return cls(packed[:elements], packed[elements:elements + pb].view(torch.bfloat16),
                   packed[elements + pb:elements + 2 * pb].view(torch.bfloat16), inp, out)


class MoeWeights:
    """All weights of one sparse MoE block, the host mirror of Splash's
    MoeWeights (MoE.hpp:35-44): the router, the routed experts and,
    optionally, the shared expert (one-expert gate / up / down) with its
    scalar gate.  For an expert shard, gate / up / down hold the shard's
    experts and the shared projections are given on the rank that runs the
    shared expert (the shared expert gate on every rank)."""

    def __init__(self, router: Q8Projection, gate: PackedExperts, up: PackedExperts, down: PackedExperts,
                 shared_gate: Optional[PackedExperts] = None, shared_up: Optional[PackedExperts] = None,
                 shared_down: Optional[PackedExperts] = None, shared_expert_gate: Optional[Q8Projection] = None):
        self.router, self.gate, self.up, self.down = router, gate, up, down
        self.shared_gate, self.shared_up, self.shared_down = shared_gate, shared_up, shared_down
        self.shared_expert_gate = shared_expert_gate
        d = _lib.thq4_moe_weights()
        d.router = router.desc
        d.gate, d.up, d.down = gate.desc, up.desc, down.desc
        if shared_gate is not None:
            d.shared_gate, d.shared_up, d.shared_down = shared_gate.desc, shared_up.desc, shared_down.desc
        if shared_expert_gate is not None:
            d.shared_expert_gate = shared_expert_gate.desc
        self.desc = d

    @property
    def has_shared(self) -> bool:
        return self.shared_expert_gate is not None

    @property
    def runs_shared(self) -> bool:
        return self.shared_gate is not None


def _moe_ws(key, need: int, device) -> torch.Tensor:
    ws = _MOE_WS.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.empty(need, dtype=torch.uint8, device=device)
        _MOE_WS[key] = ws
    return ws


def moe_scores_q8(x: torch.Tensor, router: Q8Projection, ncols: int = 256) -> torch.Tensor:
    """Router scores bf16 [T, ncols] (moe_route_scores_q8, moe.metal:34-262)."""
    T = x.shape[0]
    L = _lib.lib()
    ws = _moe_ws(("scores", x.device.index, torch.cuda.current_stream(x.device).cuda_stream),
                 L.thq4_moe_scores_workspace_bytes(T, ncols), x.device)
    s = torch.empty((T, ncols), dtype=torch.bfloat16, device=x.device)
    check(L.thq4_moe_scores_q8(_ptr(x.contiguous()), T, ctypes.byref(router.desc), ncols, _ptr(s), ncols, _ptr(ws),
                               ws.numel(), _stream()))
    return s


def moe_route_q8(x: torch.Tensor, router: Q8Projection, E: int, k: int,
                 shared_expert_gate: Optional[Q8Projection] = None):
    """The routing of MoE::add on the device: ids [T, rpr] u32, weights
    [T, rpr] bf16 (rpr = k, + 1 with a shared expert), tiles [n, 2],
    grouped_routes [n*32], route_rows [T*rpr]."""
    T = x.shape[0]
    L = _lib.lib()
    sh = shared_expert_gate is not None
    rpr = k + int(sh)
    mt = L.thq4_moe_add_max_tiles(T, E, k, int(sh))
    dev = x.device
    ids = torch.empty((T, rpr), dtype=torch.int32, device=dev)
    w = torch.empty((T, rpr), dtype=torch.bfloat16, device=dev)
    tiles = torch.empty((mt, 2), dtype=torch.int32, device=dev)
    grouped = torch.empty(mt * 32, dtype=torch.int32, device=dev)
    rows = torch.empty(T * rpr, dtype=torch.int32, device=dev)
    n = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = _moe_ws(("scores", dev.index, torch.cuda.current_stream(dev).cuda_stream),
                 L.thq4_moe_scores_workspace_bytes(T, E), dev)
    check(L.thq4_moe_route_q8(_ptr(x.contiguous()), T, E, k, ctypes.byref(router.desc),
                              ctypes.byref(shared_expert_gate.desc) if sh else None, _ptr(ids), _ptr(w), _ptr(tiles),
                              _ptr(grouped), _ptr(rows), _ptr(n), mt, _ptr(ws), ws.numel(), _stream()))
    nt = int(n.item())
    return ids, w, tiles[:nt], grouped[:nt * 32], rows


def moe_add(x: torch.Tensor, weights: MoeWeights, k: int, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One MoE block (MoE::add, MoE.cpp:119-231): bf16 [T, H]."""
    T, H = x.shape
    E, I = weights.gate.experts, weights.gate.rows
    L = _lib.lib()
    need = L.thq4_moe_add_workspace_bytes(T, H, I, E, k, int(weights.runs_shared))
    ws = _moe_ws(("add", x.device.index, torch.cuda.current_stream(x.device).cuda_stream), need, x.device)
    y = torch.empty((T, H), dtype=torch.bfloat16, device=x.device)
    check(L.thq4_moe_add(_ptr(x.contiguous()), _ptr(residual), T, H, I, E, k, ctypes.byref(weights.desc), _ptr(y),
                         _ptr(ws), ws.numel(), _stream()))
    return y


def moe_add_partial(x: torch.Tensor, weights: MoeWeights, k: int, e0: int, E: int,
                    residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """An expert shard's part of one MoE block: the shard holds routed
    experts [e0, e0 + weights.gate.experts) of E; f32 [T, H]."""
    T, H = x.shape
    El, I = weights.gate.experts, weights.gate.rows
    L = _lib.lib()
    need = L.thq4_moe_add_partial_workspace_bytes(T, H, I, E, k, e0, e0 + El, int(weights.has_shared),
                                                  int(weights.runs_shared))
    ws = _moe_ws(("add_partial", x.device.index, torch.cuda.current_stream(x.device).cuda_stream), need, x.device)
    y = torch.empty((T, H), dtype=torch.float32, device=x.device)
    check(L.thq4_moe_add_partial(_ptr(x.contiguous()), _ptr(residual), T, H, I, E, k, e0, e0 + El,
                                 ctypes.byref(weights.desc), _ptr(y), _ptr(ws), ws.numel(), _stream()))
    return y
