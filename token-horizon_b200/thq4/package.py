"""Splash's packed Q4 weight files on the host: read (and, for tools and
tests, write) the on-disk package, then repack its Q4 projections into this
library's layout on the device.

The format follows docs/splash/runtime/model/WeightStore.{hpp,cpp}:

- a 16-byte header: an 8-byte magic, then the layer and the type as
  little-endian u32 (WeightStore.cpp:176-186);
- sections one after another, each starting at the next 16 KiB boundary
  after the header or the previous section (WeightStore.cpp:198-211);
- the file size is a multiple of 16 KiB and every byte up to it belongs to
  a section or its alignment padding (WeightStore.cpp:214-223);
- a Q4 projection of `out` x `inp` elements is one section of out*inp/16*9
  bytes: the nibbles (out*inp/2 bytes), then the bf16 scales and the bf16
  biases (out*inp/32 bytes each), in StorageN = 256 order, out a multiple of
  256 (WeightStore.cpp:57-67, 229-249) -- the Splash slab layout that
  thq4_repack reads as THQ4_SRC_SLAB;
- an expert projection is one section of `experts` such slabs back to back
  (WeightStore.cpp:284-299);
- a Q8 projection (the MoE router, the shared expert's gate) is one section
  of out*inp + 2 * out*inp/32 bytes: the weight bytes, then the bf16 scales,
  then the bf16 biases, in StorageN = 256 order (WeightStore.cpp:47-53,
  264-282), read by the library as stored.

Error messages follow the reference's WeightStoreError texts.  This module
only moves bytes; the arithmetic runs in libthq4.so.
"""
from __future__ import annotations

import mmap
import os
import struct
from typing import List, Optional

import numpy as np

ALIGNMENT = 16 * 1024
STORAGE_N = 256
GROUP = 64


class WeightFileError(ValueError):
    """A malformed or mismatched package file (WeightStoreError)."""


def q4_elements(out: int, inp: int) -> int:
    if out <= 0 or inp <= 0 or inp % GROUP:
        raise WeightFileError("Q4 projection dimensions must be positive and input-aligned")
    return out * inp


def q4_packed_bytes(out: int, inp: int) -> int:
    """Bytes of one Q4 projection section: 9/16 of a byte per element."""
    return q4_elements(out, inp) // 16 * 9


def q8_packed_bytes(out: int, inp: int) -> int:
    """Bytes of one Q8 projection section: the elements plus a bf16 scale and
    bias per 64 elements (q8PackedBytes, WeightStore.cpp:47-53)."""
    elements = q4_elements(out, inp)
    return elements + elements // 32 * 2


def validate_q4_layout(out: int, inp: int) -> None:
    q4_elements(out, inp)
    if out % STORAGE_N:
        raise WeightFileError("Q4 output dimension is incompatible with StorageN=256")


def _align(offset: int) -> int:
    return (offset + ALIGNMENT - 1) // ALIGNMENT * ALIGNMENT


class WeightFile:
    """A read-only mapping of one package file; `section` hands out its
    sections in order (host memory views)."""

    def __init__(self, path: str, magic: bytes, layer: int, type_: int):
        if len(magic) != 8:
            raise WeightFileError("packed file magic must contain eight bytes")
        self.path = path
        size = os.path.getsize(path)
        if size < 16 or size % ALIGNMENT:
            raise WeightFileError(f"packed file size is not 16 KiB-aligned: {path}")
        with open(path, "rb") as f:
            self._map = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
        head_magic = self._map[:8]
        head_layer, head_type = struct.unpack("<II", self._map[8:16])
        if head_magic != magic or head_layer != layer or head_type != type_:
            self._map.close()
            raise WeightFileError(f"packed file header mismatch: {path}")
        self.magic, self.layer, self.type = magic, layer, type_
        self.size = size
        self._offset = 16
        self._finished = False

    def section(self, nbytes: int, label: str) -> memoryview:
        if self._finished:
            raise WeightFileError("cannot add a section after packed file finish")
        if nbytes <= 0:
            raise WeightFileError("packed section must not be empty")
        start = _align(self._offset)
        end = start + nbytes
        if end > self.size:
            raise WeightFileError(f"packed file is truncated at section {label}")
        self._offset = end
        return memoryview(self._map)[start:end]

    def finish(self) -> None:
        if self._finished:
            return
        if _align(self._offset) != self.size:
            raise WeightFileError(f"packed file has unconsumed or missing bytes: {self.path}")
        self._finished = True

    def q4_projection(self, out: int, inp: int, label: str) -> np.ndarray:
        """The slab bytes (u8) of one Q4 projection section."""
        validate_q4_layout(out, inp)
        return np.frombuffer(self.section(q4_packed_bytes(out, inp), label), dtype=np.uint8)

    def expert_q4_projection(self, experts: int, out: int, inp: int, label: str) -> np.ndarray:
        """[experts, slab bytes] (u8) of one expert projection section."""
        if experts <= 0:
            raise WeightFileError("expert projection requires experts")
        validate_q4_layout(out, inp)
        stride = q4_packed_bytes(out, inp)
        raw = np.frombuffer(self.section(experts * stride, label), dtype=np.uint8)
        return raw.reshape(experts, stride)

    def q8_projection(self, out: int, inp: int, label: str) -> np.ndarray:
        """The bytes (u8) of one Q8 projection section (readQ8Projection,
        WeightStore.cpp:264-282)."""
        validate_q4_layout(out, inp)
        return np.frombuffer(self.section(q8_packed_bytes(out, inp), label), dtype=np.uint8)

    def close(self) -> None:
        try:
            self._map.close()
        except BufferError:  # sections still referenced: the mapping goes with them
            pass

    def __enter__(self) -> "WeightFile":
        return self

    def __exit__(self, *exc) -> None:
        self.close()


def write_weight_file(path: str, magic: bytes, layer: int, type_: int, sections: List[bytes]) -> None:
    """Write a package: header, then each section at the next 16 KiB
    boundary, zero padding up to a 16 KiB multiple."""
    if len(magic) != 8:
        raise WeightFileError("packed file magic must contain eight bytes")
    with open(path, "wb") as f:
        f.write(magic + struct.pack("<II", layer, type_))
        offset = 16
        for sec in sections:
            if not len(sec):
                raise WeightFileError("packed section must not be empty")
            start = _align(offset)
            f.write(b"\0" * (start - offset))
            f.write(bytes(sec))
            offset = start + len(sec)
        f.write(b"\0" * (_align(offset) - offset))


def load_q4_projection(slab: np.ndarray, out: int, inp: int, device, sb_dtype: Optional[int] = None):
    """A PackedWeight from one section's slab bytes: uploaded, then repacked
    on the device (THQ4_SRC_SLAB; the package's scales are bf16)."""
    import torch

    from ._lib import BF16, SRC_SLAB
    from .qlin import PackedWeight

    validate_q4_layout(out, inp)
    src = torch.from_numpy(np.ascontiguousarray(slab)).to(device)
    return PackedWeight.repack(SRC_SLAB, src, None, out, inp, BF16 if sb_dtype is None else sb_dtype)


def load_expert_q4_projection(slabs: np.ndarray, out: int, inp: int, device, sb_dtype: Optional[int] = None):
    """PackedExperts from an expert section ([experts, slab bytes])."""
    import torch

    from ._lib import BF16
    from .qlin import PackedExperts

    validate_q4_layout(out, inp)
    src = torch.from_numpy(np.ascontiguousarray(slabs)).to(device)
    return PackedExperts.from_slabs(src, out, inp, BF16 if sb_dtype is None else sb_dtype)


def load_q8_projection(section: np.ndarray, out: int, inp: int, device):
    """A Q8Projection from one section's bytes, uploaded as stored (the
    library reads the StorageN = 256 order directly)."""
    import torch

    from .qlin import Q8Projection

    validate_q4_layout(out, inp)
    if section.size != q8_packed_bytes(out, inp):
        raise WeightFileError("Q8 projection section has the wrong size")
    return Q8Projection.from_section(torch.from_numpy(np.ascontiguousarray(section)).to(device), inp, out)
