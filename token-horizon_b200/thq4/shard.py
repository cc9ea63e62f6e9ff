"""Column sharding of the projections over the GPUs of one node.

Each rank holds a contiguous range of a projection's output rows (the
columns of y) and computes that slice of y from a replicated x; an NCCL
all-gather reassembles y only where the next projection needs all of it.
The fused [gate | up] weight shards both halves with the same row range, so
the SwiGLU epilogue stays local.  Shards are multiples of 16 rows (one MMA
tile) and equal in size, the layout `all_gather_into_tensor` concatenates.

`PeerGroup` sets up the fused alternative to that all-gather
(`thq4_linear_peer`): one region of device memory per rank, mapped by every
other rank through CUDA IPC, holding the gather flags and the full-vector
buffers that the projections write into directly over NVLink.

The reference engine is single-device; this module is the host logic of the
multi-GPU extension and carries no arithmetic of its own.
"""
from __future__ import annotations

import ctypes
from typing import List, Optional

import torch


def shard_rows(total: int, world: int, rank: int, align: int = 16):
    """(first row, rows) of `rank`'s equal shard of `total` output rows."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    per, rem = divmod(total, world)
    if rem or per % align:
        raise ValueError(f"{total} rows do not split into {world} shards of a multiple of {align}")
    return rank * per, per


def shard_cols(total: int, world: int, rank: int):
    """(first input column, columns) of `rank`'s equal shard of a row-
    parallel projection's `total` inputs: whole 64-wide quant groups."""
    return shard_rows(total, world, rank, align=64)


def slice_cols_mlx(wq: torch.Tensor, sb: torch.Tensor, k0: int, k: int):
    """Input columns [k0, k0 + k) of an MLX weight (wq u32 [out][in/8], sb
    [out][2 * in/64]: a row's scales, then its biases), as an MLX weight of
    k inputs -- a row-parallel shard, before the repack."""
    if k0 % 64 or k % 64:
        raise ValueError("column shards must be whole 64-wide groups")
    ng = sb.shape[1] // 2
    g0, gk = k0 // 64, k // 64
    return (wq[:, k0 // 8:(k0 + k) // 8].contiguous(),
            torch.cat([sb[:, g0:g0 + gk], sb[:, ng + g0:ng + g0 + gk]], dim=1).contiguous())


def gather_rows(local: torch.Tensor, full: Optional[torch.Tensor] = None, group=None) -> torch.Tensor:
    """All-gather the ranks' y slices [m, rows] into y [m, world * rows] in
    rank order.  The collective concatenates the ranks' [m, rows] blocks;
    they are then reordered to [m][world * rows] (for m = 1, the decode case,
    the reorder is free)."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    m, rows = local.shape
    cat = torch.empty((world * m, rows), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(cat, local.contiguous(), group=group)
    out = cat.view(world, m, rows).permute(1, 0, 2).reshape(m, world * rows)
    if full is not None:
        full.copy_(out)
        return full
    return out


def expert_range(E: int, world: int, rank: int):
    """(first expert, experts) of `rank`'s equal share of E experts."""
    per, rem = divmod(E, world)
    if rem or not 0 <= rank < world:
        raise ValueError(f"{E} experts do not split into {world} equal shards")
    return rank * per, per


def moe_sharded(x: torch.Tensor, logits: torch.Tensor, k: int, e0: int, gate, up, down,
                residual: Optional[torch.Tensor] = None, group=None) -> torch.Tensor:
    """One MoE layer with the experts sharded over the ranks: each rank runs
    its experts' routes (thq4_moe_partial, f32 partial [T, H]; the residual is
    added on rank 0 only), one all-reduce sums the partials, and the sum is
    rounded once to bf16."""
    import torch.distributed as dist

    from .qlin import moe_partial

    rank = dist.get_rank(group) if dist.is_initialized() else 0
    part = moe_partial(x, logits, k, e0, gate, up, down, residual if rank == 0 else None)
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(part, group=group)
    return part.to(torch.bfloat16)


def moe_add_sharded(x: torch.Tensor, weights, k: int, e0: int, E: int, residual: Optional[torch.Tensor] = None,
                    group=None) -> torch.Tensor:
    """One MoE block (MoE::add) with the routed experts sharded over the
    ranks: `weights` (a MoeWeights) holds this rank's experts [e0, e0 +
    weights.gate.experts) of E, the full router and, on the rank that runs
    it, the shared expert; each rank writes its f32 partial (the residual on
    rank 0 only), one all-reduce sums them, one rounding to bf16."""
    import torch.distributed as dist

    from .qlin import moe_add_partial

    rank = dist.get_rank(group) if dist.is_initialized() else 0
    part = moe_add_partial(x, weights, k, e0, E, residual if rank == 0 else None)
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(part, group=group)
    return part.to(torch.bfloat16)


class PeerGroup:
    """One IPC-mapped region per rank: [0, 256) control words (flags[world]
    u32 at 0, the gather count at 64, the CTA arrival counter at 128), then
    full-vector buffers placed by `buffer` at the same offset on every rank
    (every rank makes the same calls in the same order)."""

    CONTROL = 256

    def __init__(self, nbytes: int, device: torch.device, group=None):
        import torch.distributed as dist

        from . import _lib

        self._lib = _lib.lib()
        self._L = _lib
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.device = device
        self.size = self.CONTROL + nbytes
        self._next = self.CONTROL
        base, handle = ctypes.c_void_p(), ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
        _lib.check(self._lib.thq4_ipc_alloc(self.size, ctypes.byref(base), handle))
        self.local = base.value
        handles: List[bytes] = [handle.raw]
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, handle.raw, group=group)
        self.bases: List[int] = []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.bases.append(self.local)
                continue
            p = ctypes.c_void_p()
            _lib.check(self._lib.thq4_ipc_open(ctypes.create_string_buffer(h, len(h)), ctypes.byref(p)))
            self.bases.append(p.value)
        self._flags = self._ptr_array([b for b in self.bases])
        self.count = self.local + 64
        self.arrive = self.local + 128
        self._keep = []

    def _ptr_array(self, ptrs) -> torch.Tensor:
        t = torch.tensor(list(ptrs), dtype=torch.int64, device=self.device)
        return t

    def buffer(self, nbytes: int) -> int:
        """Offset of a new buffer of `nbytes` (256-byte aligned) in every rank's region."""
        off = self._next
        self._next = (off + nbytes + 255) // 256 * 256
        if self._next > self.size:
            raise ValueError(f"PeerGroup region of {self.size} bytes is full")
        return off

    def ptr(self, offset: int) -> int:
        """This rank's address of the buffer at `offset`."""
        return self.local + offset

    def gather(self, offset: int, rows: int, at: int, stride: int, wait: bool, x_parts: int = 0,
               x_slot: int = 0, x_ll: bool = False):
        """A thq4_peer_gather for a projection whose first `rows` outputs go to
        full[t * stride + at + row] in the buffer at `offset` on every rank."""
        dst = self._ptr_array([b + offset for b in self.bases])
        self._keep.append(dst)
        g = self._L.thq4_peer_gather()
        g.world, g.rank, g.rows, g.offset, g.stride, g.wait = self.world, self.rank, rows, at, stride, int(wait)
        g.dst, g.flags = dst.data_ptr(), self._flags.data_ptr()
        g.count, g.arrive = self.count, self.arrive
        g.x_parts, g.x_slot, g.x_ll = x_parts, x_slot, int(x_ll)
        if x_ll:
            g.wait = 0  # the low-latency words are polled, not waited for
        return g

    def reduce(self, offset: int, out: int, m: int, wait: bool, x_parts: int = 0, x_slot: int = 0,
               ll: bool = False, x_ll: bool = False):
        """A thq4_peer_gather for a row-parallel projection of `out` outputs:
        its f32 partial goes to slot `rank` of the reduction buffer at
        `offset` on every rank (slots of m * out values; the buffer holds
        world slots, `reduction_bytes`).  Read back with x_parts = world,
        x_slot = m * out.  ll: low-latency words (out_mode 3; the reader sets
        x_ll and does not wait)."""
        g = self.gather(offset, out, 0, out, wait, x_parts, x_slot)
        g.out_mode, g.slot = (3 if ll else 1), m * out
        g.x_ll = int(x_ll)
        return g

    def local_out(self, wait: bool, x_parts: int = 0, x_slot: int = 0, x_ll: bool = False):
        """A thq4_peer_gather that only waits (for the exchange x comes from)
        and reads x as partials; the projection's output stays local.  x_ll:
        the partials are low-latency words, polled instead of waited for."""
        g = self._L.thq4_peer_gather()
        g.world, g.rank, g.wait = self.world, self.rank, int(wait and not x_ll)
        g.flags, g.count = self._flags.data_ptr(), self.count
        g.out_mode, g.x_parts, g.x_slot, g.x_ll = 2, x_parts, x_slot, int(x_ll)
        return g

    def reduction_bytes(self, out: int, m: int, ll: bool = False) -> int:
        """Bytes of a reduction buffer: world slots of m * out f32 values
        (8-byte words for the low-latency form)."""
        return self.world * m * out * (8 if ll else 4)

    def close(self) -> None:
        """Unmap the peers' regions, then free this rank's (after every rank
        has unmapped it).  Collective."""
        import torch.distributed as dist

        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        for r, b in enumerate(self.bases):
            if r != self.rank:
                self._L.check(self._lib.thq4_ipc_close(ctypes.c_void_p(b)))
        if self.world > 1:
            dist.barrier(group=self.group)
        self._L.check(self._lib.thq4_ipc_free(ctypes.c_void_p(self.local)))
        self.bases, self._keep = [], []
