"""Synthetic Q4 weights for benchmarks: W ~ N(0, std) quantised group-wise.

The quantiser is the same min/max affine group-64 rule as the CPU oracle's
q4o_quantize (this repository's own; the reference loads pre-quantised
checkpoints): per (row, group) s = (max - min) / 15 and b = min, both rounded
to the 16-bit scale dtype, and q = clamp(round((w - b) / s), 0, 15) against
the rounded values, computed in f64.  It runs on whatever device `w` lives on,
so benchmark weights of several GB are made on the GPU in seconds.  Output is
the reference's MLX layout: wq int32 [out, in/8] (u32 bits, nibbles LSB first)
and sb [out, 2*ng] (scales, then biases).
"""
from __future__ import annotations

import torch


def quantize(w: torch.Tensor, sb_dtype: torch.dtype = torch.float16, gs: int = 64):
    out, inp = w.shape
    ng = inp // gs
    g = w.reshape(out, ng, gs)
    lo = g.amin(dim=2)
    hi = g.amax(dim=2)
    s16 = ((hi - lo) / 15.0).to(sb_dtype)
    b16 = lo.to(sb_dtype)
    s = s16.double().unsqueeze(2)
    b = b16.double().unsqueeze(2)
    t = torch.round((g.double() - b) / torch.where(s > 0, s, torch.ones_like(s)))
    q = torch.where(s > 0, t.clamp(0, 15), torch.zeros_like(t)).to(torch.int64)
    q = q.reshape(out, inp // 8, 8)
    shifts = torch.arange(0, 32, 4, device=w.device, dtype=torch.int64)
    words = (q << shifts).sum(dim=2)
    wq = torch.where(words >= 2 ** 31, words - 2 ** 32, words).to(torch.int32)
    sb = torch.cat([s16, b16], dim=1).contiguous()
    return wq.contiguous(), sb


def normal_weight(out: int, inp: int, seed: int, device, std: float = 0.02,
                  sb_dtype: torch.dtype = torch.float16, chunk_rows: int = 4096):
    """Quantised N(0, std) weight, generated and quantised in row chunks."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    wqs, sbs = [], []
    for r0 in range(0, out, chunk_rows):
        rows = min(chunk_rows, out - r0)
        w = torch.randn((rows, inp), generator=gen, device=device, dtype=torch.float32) * std
        a, b = quantize(w, sb_dtype)
        wqs.append(a)
        sbs.append(b)
        del w
    return torch.cat(wqs, 0), torch.cat(sbs, 0)
