#!/usr/bin/env python
"""Headline benchmark of the B200 Q4 quantized-matmul path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl thq4|reference]

Workload (the configuration the GEMV GB/s metric is
scaled on): one decode token through the projection set of a hidden-5120
transformer layer -- q/k/v/o (5120x5120, 1024x5120 x2, 5120x5120) and the MLP
gate/up/down (intermediate 17408) -- Q4 affine group-64 weights with f16
scale/bias, batch 1, bf16 activations.  A step runs `--layers` (24) distinct
layers back to back, so the 4.46 GB of weights exceed the 126 MB L2 many
times over and no flush is needed.  Per layer: the fused qkv GEMV, o, the
fused gate/up GEMV with the SwiGLU epilogue, and down; each layer starts from
the same input activation (no norms or attention exist on this path, and
chaining raw projections would overflow bf16), while every projection still
consumes the previous one's output.  On one GPU the step runs by default
as one thq4_linear / thq4_gate_up call per projection (`--launch
chain-step` runs the step's 96 projections as one persistent chain launch,
thq4_linear_chain, `--launch chain-layer` one chain per layer; the line
reports all three).  With N GPUs (the default `--tp row`) q/k/v and gate/up are
column-sharded with local outputs and o and down are row-sharded: their f32
partials go over NVLink into every rank's reduction buffer from the GEMV's
epilogue and the next projection sums them as it stages its input (no
collective inside the step); each layer then reads the previous layer's
all-reduced output.  `--tp col` column-shards every projection with the
all-gather fused into the epilogue, `--nccl-gather` uses NCCL all-gathers.

One JSON line on rank 0: `value` is algorithmic weight bytes of the whole job
per step / max-over-ranks step time (GB/s), the step captured in a CUDA graph
and timed with CUDA events; `e2e` is the same metric with the input copied
from pinned host memory and the layer output read back inside the timed
region; `roofline` is the dominant kernel; `cpu_baseline` times the CPU
restatement of the reference's CPU path on a bounded sample (N=1 only,
before any CUDA work); `prefill` reports the prefill GEMM (BASELINE
configs[2], M=512 and 2048) in TFLOP/s, `moe` the MoE layer,
`c1` the single GEMV of configs[0] and `verify` the spec-verify products of
configs[1] (N=1).  With N > 1 the line also carries `kernel_only` (the same
shards without any exchange) and `parity` (the sharded layer's output
against one GPU's unsharded recomputation).

`--impl reference` times the reference's CPU semantics (the oracle port, all
host threads) on the same workload and metric; under torchrun only rank 0
runs.
"""
from __future__ import annotations

import argparse
import ctypes
import datetime as _dt
import gc
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "token-horizon_b200"))

HIDDEN, INTER, KV = 5120, 17408, 1024
Q4_BYTES_PER_WEIGHT = 0.5625
LAYER_WEIGHTS = 2 * HIDDEN * HIDDEN + 2 * KV * HIDDEN + 3 * INTER * HIDDEN
LAYER_BYTES = int(LAYER_WEIGHTS * Q4_BYTES_PER_WEIGHT)  # 185,794,560
METRIC = "Q4 GEMV achieved HBM GB/s (% of peak); prefill GEMM TFLOP/s; at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", default="thq4", choices=["thq4", "reference"])
    p.add_argument("--layers", type=int, default=24)
    p.add_argument("--no-graph", action="store_true")
    p.add_argument("--cpu-seconds", type=float, default=10.0)
    p.add_argument("--skip-prefill", action="store_true", help="N=1: skip the prefill and MoE lines")
    p.add_argument("--skip-extras", action="store_true", help="N=1: skip the configs[0] and configs[1] lines")
    p.add_argument("--launch", default="calls", choices=["chain-step", "chain-layer", "calls"],
                   help="N=1: the step as one persistent chain launch (thq4_linear_chain), one chain per layer, or "
                        "one thq4_linear / thq4_gate_up call per projection (N > 1 always uses calls)")
    p.add_argument("--trace", default=None,
                   help="write the GEMV's per-phase %%globaltimer trace of one step made of separate calls (after "
                        "the timed runs) to this JSON file (one file per rank: .rankR appended for N > 1)")
    p.add_argument("--nccl-gather", action="store_true",
                   help="N > 1: gather each projection's output with NCCL all-gather (the baseline) instead of "
                        "the GEMV epilogue's NVLink stores")
    p.add_argument("--exchange", default="ll", choices=["ll", "flags"],
                   help="--tp row: the reduce's partials as low-latency words the reader polls (ll) or as f32 values "
                        "behind a system-scope fence and per-rank flags (flags)")
    p.add_argument("--tp", default="row", choices=["col", "row"],
                   help="N > 1: col = every projection column-sharded with a fused all-gather; row = o and down "
                        "row-sharded with a fused all-reduce (partials stored to every rank, summed as the next "
                        "projection stages them), q/k/v and gate/up column-sharded with local outputs")
    return p.parse_args()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, 1400.0, "fallback"


# ---------------------------------------------------------------------------
# clocks sampler (nvidia-smi during the timed region)
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu_ids):
        self.rows = []
        self.proc = None
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100"]
        if gpu_ids:
            cmd += ["-i", ",".join(gpu_ids)]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True, bufsize=1)
        except Exception:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                ts = _dt.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f")
                self.rows.append((ts, int(parts[1]), float(parts[2]), float(parts[3]), parts[5:9]))
            except ValueError:
                continue

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self, t0: _dt.datetime, t1: _dt.datetime):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        inwin = [r for r in self.rows if t0 <= r[0] <= t1]
        note = None
        if not inwin:  # region shorter than the sampling period: nearest samples
            inwin = sorted(self.rows, key=lambda r: abs((r[0] - t0).total_seconds()))[:4]
            note = "timed region shorter than 100 ms sampling: nearest samples"
        reasons = sorted({self.REASONS[i] for r in inwin for i, v in enumerate(r[4]) if v.lower() == "active"})
        out = {"sm_mhz": statistics.median(r[2] for r in inwin), "sm_max_mhz": max(r[3] for r in inwin),
               "reasons": reasons, "samples": len(inwin)}
        if note:
            out["note"] = note
        return out


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ---------------------------------------------------------------------------
# the thq4 arm
# ---------------------------------------------------------------------------
def run_thq4(args):
    import torch
    import torch.distributed as dist
    import thq4
    from thq4 import synth
    from thq4.shard import shard_rows, slice_cols_mlx

    world, rank, local = dist_env()
    # the CPU baseline runs first, before this process has touched CUDA, as
    # the reference arm does
    cpu = cpu_baseline(args.cpu_seconds) if rank == 0 and world == 1 else None
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=_dt.timedelta(seconds=300))
    L = args.layers
    hbm_peak, tc_peak, tc_sust, peak_kind = peaks()

    # -- weights: each rank quantises the full layer on its GPU, keeps its rows
    def packed(out_rows, inp, seed, begin, rows):
        wq, sb = synth.normal_weight(out_rows, inp, seed, dev)
        p = thq4.PackedWeight.repack(thq4.SRC_MLX, wq, sb, out_rows, inp, thq4.F16, begin, rows)
        del wq, sb
        return p

    row_tp = world > 1 and args.tp == "row" and not args.nccl_gather
    align = 64 if row_tp else 16  # row shards split o's and down's inputs into whole groups
    q0, qn = shard_rows(HIDDEN, world, rank, align)
    k0, kn = shard_rows(KV, world, rank)
    i0, inn = shard_rows(INTER, world, rank, align)

    def packed_cols(out_rows, inp, seed, c0, cols):
        """A row-parallel shard: input columns [c0, c0 + cols), every output row."""
        wq, sb = synth.normal_weight(out_rows, inp, seed, dev)
        wq_r, sb_r = slice_cols_mlx(wq, sb, c0, cols)
        del wq, sb
        return thq4.PackedWeight.repack(thq4.SRC_MLX, wq_r, sb_r, out_rows, cols, thq4.F16)

    def build_layer(l, q0, qn, k0, kn, i0, inn, rows_of_o_down):
        """Layer l's weights (seeds 1000 (l + 1) + 1..7): this rank's shards, or
        the whole layer with full ranges.  rows_of_o_down: o and down hold
        input-column shards (row-parallel) instead of output rows."""
        s = 1000 * (l + 1)
        # fused qkv shard = [q rows | k rows | v rows] of this rank, repacked as three weights then joined
        wq_q, sb_q = synth.normal_weight(HIDDEN, HIDDEN, s + 1, dev)
        wq_k, sb_k = synth.normal_weight(KV, HIDDEN, s + 2, dev)
        wq_v, sb_v = synth.normal_weight(KV, HIDDEN, s + 3, dev)
        wq_qkv = torch.cat([wq_q[q0:q0 + qn], wq_k[k0:k0 + kn], wq_v[k0:k0 + kn]], 0).contiguous()
        sb_qkv = torch.cat([sb_q[q0:q0 + qn], sb_k[k0:k0 + kn], sb_v[k0:k0 + kn]], 0).contiguous()
        del wq_q, wq_k, wq_v, sb_q, sb_k, sb_v
        qkv = thq4.PackedWeight.repack(thq4.SRC_MLX, wq_qkv, sb_qkv, qn + 2 * kn, HIDDEN, thq4.F16)
        del wq_qkv, sb_qkv
        o = packed_cols(HIDDEN, HIDDEN, s + 4, q0, qn) if rows_of_o_down else packed(HIDDEN, HIDDEN, s + 4, q0, qn)
        gate = packed(INTER, HIDDEN, s + 5, i0, inn)
        up = packed(INTER, HIDDEN, s + 6, i0, inn)
        down = packed_cols(HIDDEN, INTER, s + 7, i0, inn) if rows_of_o_down else packed(HIDDEN, INTER, s + 7, q0, qn)
        return qkv, o, gate, up, down

    layers = [build_layer(l, q0, qn, k0, kn, i0, inn, row_tp) for l in range(L)]
    torch.cuda.synchronize()
    rank_bytes = sum(p.nbytes for lay in layers for p in lay)

    lib = thq4.lib()
    BF = thq4.BF16
    # one zero-filled workspace for the chain (calls are stream-ordered)
    ws_bytes = max(lib.thq4_linear_workspace_bytes(ctypes.byref(p.desc), 1) for lay in layers for p in lay)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(7)
    x_in = (torch.randn((1, HIDDEN), generator=gen, device=dev)).to(torch.bfloat16)
    t_qkv = torch.empty((1, qn + 2 * kn), dtype=torch.bfloat16, device=dev)
    t_o = torch.empty((1, qn), dtype=torch.bfloat16, device=dev)
    t_h = torch.empty((1, inn), dtype=torch.bfloat16, device=dev)
    t_d = torch.empty((1, qn), dtype=torch.bfloat16, device=dev)
    full_q = torch.empty((1, HIDDEN), dtype=torch.bfloat16, device=dev) if world > 1 else None
    full_o = torch.empty((1, HIDDEN), dtype=torch.bfloat16, device=dev) if world > 1 else t_o
    full_h = torch.empty((1, INTER), dtype=torch.bfloat16, device=dev) if world > 1 else t_h
    y_out = torch.empty((1, HIDDEN), dtype=torch.bfloat16, device=dev) if world > 1 else t_d

    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731

    def stream():
        return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    # N > 1: each projection's epilogue stores its rows into every rank's full
    # vector over NVLink (IPC-mapped buffers) and raises this rank's flag on
    # every peer; the next projection waits for the peers' flags before it
    # reads x.  No collective runs in the step.
    peer = None
    if row_tp:
        # o and down row-sharded: each writes its f32 partial of the whole
        # output into its slot of every rank's reduction buffer; q/k/v and
        # gate/up read x as the sum of the partials (after the peers' flags)
        # and keep their column-sharded outputs local.  Two exchanges per
        # layer instead of four.
        # With --exchange ll (the default) the partials are low-latency words
        # {value, exchange number} that the readers poll (no fence, no flag);
        # the step's last down uses the flagged form into its own buffer, so
        # the result can be waited for and read back.
        from thq4.shard import PeerGroup

        ll = args.exchange == "ll"
        peer = PeerGroup(3 * world * HIDDEN * 8 + 4 * 256, dev)
        red_o = peer.buffer(peer.reduction_bytes(HIDDEN, 1, ll=ll))
        red_d = peer.buffer(peer.reduction_bytes(HIDDEN, 1, ll=ll))
        red_f = peer.buffer(peer.reduction_bytes(HIDDEN, 1))
        g_qkv = peer.local_out(wait=True, x_parts=world, x_slot=HIDDEN, x_ll=ll)
        g_o = peer.reduce(red_o, HIDDEN, 1, wait=False, ll=ll)
        g_gu = peer.local_out(wait=True, x_parts=world, x_slot=HIDDEN, x_ll=ll)
        g_dn = peer.reduce(red_d, HIDDEN, 1, wait=False, ll=ll)
        g_dn_last = peer.reduce(red_f, HIDDEN, 1, wait=False)
        g_fin = peer.local_out(wait=True)  # waits for the peers' last flagged exchange
        V = lambda off: ctypes.c_void_p(peer.ptr(off))  # noqa: E731
        F32 = thq4.F32
    elif world > 1 and not args.nccl_gather:
        from thq4.shard import PeerGroup

        peer = PeerGroup((3 * HIDDEN + INTER) * 2 + 4 * 256, dev)
        off_q, off_o = peer.buffer(HIDDEN * 2), peer.buffer(HIDDEN * 2)
        off_h, off_y = peer.buffer(INTER * 2), peer.buffer(HIDDEN * 2)
        g_qkv = peer.gather(off_q, qn, q0, HIDDEN, wait=True)
        g_o = peer.gather(off_o, qn, q0, HIDDEN, wait=True)
        g_gu = peer.gather(off_h, inn, i0, INTER, wait=True)
        g_dn = peer.gather(off_y, qn, q0, HIDDEN, wait=True)
        V = lambda off: ctypes.c_void_p(peer.ptr(off))  # noqa: E731

    def layer_peer(lay):
        qkv, o, gate, up, down = lay
        s = stream()
        thq4.check(lib.thq4_linear_peer(ctypes.byref(qkv.desc), None, P(x_in), BF, 1, P(t_qkv), P(ws), ws_bytes,
                                        ctypes.byref(g_qkv), s))
        thq4.check(lib.thq4_linear_peer(ctypes.byref(o.desc), None, V(off_q), BF, 1, P(t_o), P(ws), ws_bytes,
                                        ctypes.byref(g_o), s))
        thq4.check(lib.thq4_linear_peer(ctypes.byref(gate.desc), ctypes.byref(up.desc), V(off_o), BF, 1, P(t_h),
                                        P(ws), ws_bytes, ctypes.byref(g_gu), s))
        thq4.check(lib.thq4_linear_peer(ctypes.byref(down.desc), None, V(off_h), BF, 1, P(t_d), P(ws), ws_bytes,
                                        ctypes.byref(g_dn), s))

    def layer_row(li, lay, last=False):
        """last: the step's final down, in the flagged form into red_f."""
        qkv, o, gate, up, down = lay
        s = stream()
        if li == 0:  # the step's input
            thq4.check(lib.thq4_linear(ctypes.byref(qkv.desc), P(x_in), BF, 1, P(t_qkv), BF, P(ws), ws_bytes, s))
        else:  # the previous layer's down, all-reduced as it is staged
            thq4.check(lib.thq4_linear_peer(ctypes.byref(qkv.desc), None, V(red_d), F32, 1, P(t_qkv), P(ws),
                                            ws_bytes, ctypes.byref(g_qkv), s))
        thq4.check(lib.thq4_linear_peer(ctypes.byref(o.desc), None, P(t_qkv), BF, 1, None, P(ws), ws_bytes,
                                        ctypes.byref(g_o), s))
        thq4.check(lib.thq4_linear_peer(ctypes.byref(gate.desc), ctypes.byref(up.desc), V(red_o), F32, 1, P(t_h),
                                        P(ws), ws_bytes, ctypes.byref(g_gu), s))
        thq4.check(lib.thq4_linear_peer(ctypes.byref(down.desc), None, P(t_h), BF, 1, None, P(ws), ws_bytes,
                                        ctypes.byref(g_dn_last if last else g_dn), s))

    def layer_plain(lay):
        qkv, o, gate, up, down = lay
        s = stream()
        thq4.check(lib.thq4_linear(ctypes.byref(qkv.desc), P(x_in), BF, 1, P(t_qkv), BF, P(ws), ws_bytes, s))
        if world > 1:
            dist.all_gather_into_tensor(full_q, t_qkv[:, :qn])
            src_o = full_q
        else:
            src_o = t_qkv  # the first 5120 outputs are q; o reads in = 5120 of them
        thq4.check(lib.thq4_linear(ctypes.byref(o.desc), P(src_o), BF, 1, P(t_o), BF, P(ws), ws_bytes, s))
        if world > 1:
            dist.all_gather_into_tensor(full_o, t_o)
        thq4.check(lib.thq4_gate_up(ctypes.byref(gate.desc), ctypes.byref(up.desc), P(full_o), BF, 1, P(t_h),
                                    BF, P(ws), ws_bytes, s))
        if world > 1:
            dist.all_gather_into_tensor(full_h, t_h)
        thq4.check(lib.thq4_linear(ctypes.byref(down.desc), P(full_h), BF, 1, P(t_d), BF, P(ws), ws_bytes, s))
        if world > 1:
            dist.all_gather_into_tensor(y_out, t_d)

    def layer(li, lay, last=None):
        if row_tp:
            layer_row(li, lay, li == len(layers) - 1 if last is None else last)
        elif peer is not None:
            layer_peer(lay)
        else:
            layer_plain(lay)

    def step_calls():
        for li, lay in enumerate(layers):
            layer(li, lay)

    # N = 1: the step's projections can also run as persistent chains
    # (thq4_linear_chain): one launch per layer or one for the whole step
    chains_layer = chain_step = None
    if world == 1:
        chains_layer = [thq4.LinearChain([(qkv, None, x_in, t_qkv), (o, None, t_qkv, t_o), (gate, up, t_o, t_h),
                                          (down, None, t_h, t_d)], device=dev)
                        for (qkv, o, gate, up, down) in layers]
        chain_step = thq4.LinearChain([op for c in chains_layer for op in c._keep], device=dev)

    def step_chain_layer():
        for c in chains_layer:
            c()

    def step_chain_step():
        chain_step()

    modes = {"calls": (step_calls, 4 * L)}
    if world == 1:
        modes["chain-layer"] = (step_chain_layer, L)
        modes["chain-step"] = (step_chain_step, 1)
    launch_mode = args.launch if world == 1 else "calls"
    step, launches_per_step = modes[launch_mode]

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    # warm up eagerly (sets kernel attributes), then capture the step
    for _ in range(2):
        step()
    torch.cuda.synchronize()
    graph = None
    if not args.no_graph:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        torch.cuda.synchronize()
    run = graph.replay if graph is not None else step

    gpu_ids = []
    if rank == 0:
        try:
            gpu_ids = ["GPU-" + str(torch.cuda.get_device_properties(i).uuid) for i in range(torch.cuda.device_count())][:max(world, 1)]
        except Exception:
            gpu_ids = []
    sampler = ClockSampler(gpu_ids) if rank == 0 else None

    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    barrier()

    def timed(body, reps):
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            body()
        b.record()
        torch.cuda.synchronize()
        barrier()
        ms = a.elapsed_time(b)
        if world > 1:
            t = torch.tensor([ms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    w0 = _dt.datetime.now()
    ms = timed(run, args.steps)
    w1 = _dt.datetime.now()
    ms_step = ms / args.steps
    total_bytes = LAYER_BYTES * L
    value = total_bytes / (ms_step * 1e-3) / 1e9

    # the other launch modes of the same step, for comparison (N = 1)
    mode_results = {launch_mode: {"ms_per_step": round(ms_step, 5), "value": round(value, 2),
                                  "launches_per_step": launches_per_step}}
    for name, (fn, nl) in modes.items():
        if name == launch_mode:
            continue
        fn()
        gm = None
        if not args.no_graph:
            gm = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gm):
                fn()
        rm = gm.replay if gm is not None else fn
        for _ in range(3):
            rm()
        msm = timed(rm, args.steps) / args.steps
        mode_results[name] = {"ms_per_step": round(msm, 5), "value": round(total_bytes / (msm * 1e-3) / 1e9, 2),
                              "launches_per_step": nl}
        if gm is not None:
            gm.reset()
        rm = gm = None

    # e2e: pinned host input -> device, step, result -> pinned host
    x_host = torch.empty((1, HIDDEN), dtype=torch.bfloat16).pin_memory()
    x_host.copy_(x_in.cpu())
    y_host = torch.empty((1, HIDDEN), dtype=torch.bfloat16).pin_memory()

    if row_tp:  # the step's result: the last down's partials, summed on the device
        y_host = torch.empty((1, HIDDEN), dtype=torch.float32).pin_memory()
        red_dev = torch.empty((world, HIDDEN), dtype=torch.float32, device=dev)

    def e2e_body():
        x_in.copy_(x_host, non_blocking=True)
        run()
        if row_tp:
            thq4.check(lib.thq4_peer_wait(ctypes.byref(g_fin), stream()))
            thq4.check(lib.thq4_copy(P(red_dev), V(red_f), world * HIDDEN * 4, stream()))
            y_host.copy_(red_dev.sum(0, keepdim=True), non_blocking=True)
        elif peer is not None:
            thq4.check(lib.thq4_copy(P(y_host), V(off_y), HIDDEN * 2, stream()))
        else:
            y_host.copy_(y_out, non_blocking=True)

    for _ in range(3):
        e2e_body()
    ms_e2e = timed(e2e_body, args.steps) / args.steps
    e2e_value = total_bytes / (ms_e2e * 1e-3) / 1e9

    if args.trace:
        path = args.trace + (f".rank{rank}" if world > 1 else "")
        trace_step(torch, lib, step_calls, dev, path, barrier, world, rank)
        if launch_mode == "chain-step":
            trace_step(torch, lib, step, dev, path + ".chain", barrier, world, rank)

    kernel_only = parity = projections = None
    if world > 1:
        # the same shards and launches with no exchange and no waits: what the
        # step costs without its collectives
        k_o = torch.empty((1, layers[0][1].desc.out), dtype=torch.bfloat16, device=dev)
        k_d = torch.empty((1, layers[0][4].desc.out), dtype=torch.bfloat16, device=dev)
        o_in = t_qkv if row_tp else x_in
        d_in = t_h if row_tp else full_h

        def step_local():
            s = stream()
            for (qkv, o, gate, up, down) in layers:
                thq4.check(lib.thq4_linear(ctypes.byref(qkv.desc), P(x_in), BF, 1, P(t_qkv), BF, P(ws), ws_bytes, s))
                thq4.check(lib.thq4_linear(ctypes.byref(o.desc), P(o_in), BF, 1, P(k_o), BF, P(ws), ws_bytes, s))
                thq4.check(lib.thq4_gate_up(ctypes.byref(gate.desc), ctypes.byref(up.desc), P(x_in), BF, 1, P(t_h),
                                            BF, P(ws), ws_bytes, s))
                thq4.check(lib.thq4_linear(ctypes.byref(down.desc), P(d_in), BF, 1, P(k_d), BF, P(ws), ws_bytes, s))

        step_local()
        g_loc = None
        if not args.no_graph:
            g_loc = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g_loc):
                step_local()
        run_loc = g_loc.replay if g_loc is not None else step_local
        for _ in range(3):
            run_loc()
        ms_loc = timed(run_loc, args.steps) / args.steps
        kernel_only = {"value": round(total_bytes / (ms_loc * 1e-3) / 1e9, 2), "unit": "GB/s",
                       "ms_per_step": round(ms_loc, 5),
                       "what": "the same per-rank shards and launches with no exchange (no NVLink stores, flags or "
                               "waits): whole-job weight bytes / max-over-ranks step time"}
        if g_loc is not None:
            g_loc.reset()
        run_loc = g_loc = None

        # parity: layer 0 through the sharded chain (the step's own calls),
        # against the same layer recomputed unsharded on one GPU (rank 0)
        torch.cuda.synchronize()
        barrier()
        layer(0, layers[0], last=True)
        if row_tp:
            thq4.check(lib.thq4_peer_wait(ctypes.byref(g_fin), stream()))
            parts = torch.empty((world, HIDDEN), dtype=torch.float32, device=dev)
            thq4.check(lib.thq4_copy(P(parts), V(red_f), world * HIDDEN * 4, stream()))
            ph = parts.cpu().numpy()
            y_sh = ph[0].copy()
            for r in range(1, world):  # the rank-order sum the next projection would form
                y_sh = (y_sh + ph[r]).astype(ph.dtype)
        else:
            if peer is not None:
                thq4.check(lib.thq4_peer_wait(ctypes.byref(g_dn), stream()))
                y_dev = torch.empty((1, HIDDEN), dtype=torch.bfloat16, device=dev)
                thq4.check(lib.thq4_copy(P(y_dev), V(off_y), HIDDEN * 2, stream()))
            else:
                y_dev = y_out
            y_sh = y_dev.float().cpu().numpy()[0]
        torch.cuda.synchronize()
        if rank == 0:
            import numpy as np
            full = build_layer(0, 0, HIDDEN, 0, KV, 0, INTER, False)
            f_ws = torch.zeros(max(lib.thq4_linear_workspace_bytes(ctypes.byref(p.desc), 1) for p in full),
                               dtype=torch.uint8, device=dev)
            fb = f_ws.numel()
            f_qkv = torch.empty((1, HIDDEN + 2 * KV), dtype=torch.bfloat16, device=dev)
            f_o = torch.empty((1, HIDDEN), dtype=torch.bfloat16, device=dev)
            f_h = torch.empty((1, INTER), dtype=torch.bfloat16, device=dev)
            f_y = torch.empty((1, HIDDEN), dtype=torch.float32 if row_tp else torch.bfloat16, device=dev)
            s = stream()
            qkv, o, gate, up, down = full
            thq4.check(lib.thq4_linear(ctypes.byref(qkv.desc), P(x_in), BF, 1, P(f_qkv), BF, P(f_ws), fb, s))
            thq4.check(lib.thq4_linear(ctypes.byref(o.desc), P(f_qkv), BF, 1, P(f_o), BF, P(f_ws), fb, s))
            thq4.check(lib.thq4_gate_up(ctypes.byref(gate.desc), ctypes.byref(up.desc), P(f_o), BF, 1, P(f_h), BF,
                                        P(f_ws), fb, s))
            thq4.check(lib.thq4_linear(ctypes.byref(down.desc), P(f_h), BF, 1, P(f_y),
                                       thq4.F32 if row_tp else BF, P(f_ws), fb, s))
            y_ref = f_y.float().cpu().numpy()[0].astype(np.float64)
            rms = float(np.sqrt(np.mean(y_ref ** 2)))
            err = float(np.abs(y_sh.astype(np.float64) - y_ref).max())
            parity = {"max_err_over_rms": round(err / rms, 6), "rms": round(rms, 6), "bar": 1e-2,
                      "ok": bool(err <= 1e-2 * rms),
                      "vs": "layer 0 of the step through the sharded chain (its exchanges included) against the "
                            "same layer unsharded on one GPU (rank 0), " +
                            ("f32 outputs" if row_tp else "bf16 outputs")}
            del full, f_ws
        barrier()
    else:
        # each projection kind alone: 24 launches on the 24 layers' weights
        def kind(i):
            def body():
                s = stream()
                for lay in layers:
                    w = lay[i]
                    if i == 2:
                        thq4.check(lib.thq4_gate_up(ctypes.byref(w.desc), ctypes.byref(lay[3].desc), P(x_in), BF, 1,
                                                    P(t_h), BF, P(ws), ws_bytes, s))
                    else:
                        src = t_h if i == 4 else x_in
                        thq4.check(lib.thq4_linear(ctypes.byref(w.desc), P(src), BF, 1,
                                                   P(t_qkv if i == 0 else t_o), BF, P(ws), ws_bytes, s))
            return body

        projections = {}
        reps_k = max(5, min(100, args.steps))
        for i, name in ((0, "qkv 7168x5120"), (1, "o 5120x5120"), (2, "gate_up 2x17408x5120"),
                        (4, "down 5120x17408")):
            body = kind(i)
            body()
            gk = None
            if not args.no_graph:
                gk = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gk):
                    body()
            rk = gk.replay if gk is not None else body
            for _ in range(3):
                rk()
            us = timed(rk, reps_k) / (reps_k * L) * 1e3
            nb = layers[0][i].nbytes + (layers[0][3].nbytes if i == 2 else 0)
            projections[name] = {"us": round(us, 2), "gbs": round(nb / (us * 1e-6) / 1e9, 1),
                                 "frac": round(nb / (us * 1e-6) / 1e9 / hbm_peak, 4)}
            if gk is not None:
                gk.reset()
            rk = gk = None

    # roofline: the fused gate/up GEMV (dominant kernel) alone, one launch per layer
    g2 = None

    def gu_only():
        s = stream()
        for (_, _, gate, up, _) in layers:
            thq4.check(lib.thq4_gate_up(ctypes.byref(gate.desc), ctypes.byref(up.desc), P(full_o), BF, 1, P(t_h), BF,
                                        P(ws), ws_bytes, s))

    gu_only()
    if not args.no_graph:
        g2 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g2):
            gu_only()
    run_gu = g2.replay if g2 is not None else gu_only
    for _ in range(3):
        run_gu()
    reps = max(5, min(200, args.steps))
    ms_gu = timed(run_gu, reps) / (reps * L)
    gu_bytes = 2 * inn * HIDDEN * Q4_BYTES_PER_WEIGHT
    achieved = gu_bytes / (ms_gu * 1e-3) / 1e9
    if sampler:
        sampler.stop()
    clocks = sampler.summary(w0, w1) if sampler else None

    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "ncu_traffic.json")) as f:
            tr = json.load(f).get("gate_up_gemv_bytes_per_weight")
        if tr:
            traffic = tr * 2 * inn * HIDDEN
    except Exception:
        pass

    prefill = moe = None
    if world > 1 and not args.skip_prefill:
        # every rank: the MoE layer with its experts sharded over the GPUs
        layers = None
        torch.cuda.empty_cache()
        moe = bench_moe_sharded(torch, thq4, synth, dev, hbm_peak, world, rank, local)
    if rank == 0 and world == 1 and not args.skip_prefill:
        # the decode weights go first: these measurements have their own working sets
        layers = None
        torch.cuda.empty_cache()
        prefill = bench_prefill(torch, thq4, synth, dev, tc_peak, peak_kind)
        torch.cuda.empty_cache()
        moe = bench_moe(torch, thq4, synth, dev, hbm_peak)
        torch.cuda.empty_cache()
    c1 = verify = None
    if rank == 0 and world == 1 and not args.skip_extras:
        layers = chains_layer = chain_step = None
        torch.cuda.empty_cache()
        c1 = bench_c1(torch, thq4, synth, dev, hbm_peak, not args.no_graph)
        torch.cuda.empty_cache()
        verify = bench_verify(torch, thq4, synth, dev, hbm_peak, not args.no_graph)

    # Release the graphs (they hold NCCL work) before the process group goes
    # away, or its teardown waits for good: reset them and drop every
    # reference, the bound `replay` methods included.
    cuda_graph_used = graph is not None
    torch.cuda.synchronize()
    for gr in (graph, g2):
        if gr is not None:
            gr.reset()
    run = run_gu = None
    graph = g2 = None
    gc.collect()
    torch.cuda.synchronize()
    if peer is not None:
        peer.close()

    gate_up_alone = {"kernel": "gemv_kernel (fused gate/up, SwiGLU epilogue), one launch per layer",
                     "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / hbm_peak, 4), "bytes_per_launch": int(gu_bytes),
                     "us_per_launch": round(ms_gu * 1e3, 3)}
    if launch_mode == "chain-step":
        # the step is one launch of the chain kernel: it is the dominant (only) kernel
        chain_traffic = None
        try:
            with open(os.path.join(ROOT, "profiles", "ncu_traffic.json")) as f:
                tr = json.load(f).get("chain_bytes_per_weight")
            if tr:
                chain_traffic = tr * LAYER_WEIGHTS * L
        except Exception:
            pass
        roofline = {"bound": "hbm", "kernel": "chain_kernel (the step's 96 projections in one persistent launch)",
                    "achieved": round(value, 1), "peak": hbm_peak, "unit": "GB/s",
                    "frac": round(value / hbm_peak, 4), "peak_kind": peak_kind, "traffic": chain_traffic,
                    "bytes_per_launch": int(total_bytes), "us_per_launch": round(ms_step * 1e3, 3),
                    "gate_up_alone": gate_up_alone}
    else:
        roofline = dict(bound="hbm", peak_kind=peak_kind, traffic=traffic, **gate_up_alone,
                        step_frac=round(value / world / hbm_peak, 4))
    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_step, 5),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic: x ~ N(0,1) bf16; W ~ N(0,0.02) quantised Q4 affine group-64, f16 scale/bias",
            "config": {
                "workload": "decode-layer projection set, hidden 5120 (q/k/v/o 5120x5120, 1024x5120 x2, "
                            "5120x5120; MLP gate/up/down intermediate 17408), batch 1",
                "layers_per_step": L, "bytes_per_step": total_bytes, "batch": 1, "hidden": HIDDEN,
                "intermediate": INTER, "group": 64, "scale_dtype": "f16",
                "l2": f"inputs larger than L2: {total_bytes / 1e9:.2f} GB of weights per step "
                      f"({rank_bytes / 1e9:.2f} GB per GPU), no flush",
                "parallelism": (f"tensor-parallel x{world}: q/k/v and gate/up column-sharded, o and down row-sharded "
                                "with the all-reduce fused (f32 partials stored over NVLink into every rank's buffer "
                                + ("as low-latency words {value, exchange number} polled by" if args.exchange == "ll"
                                   else "+ flags, summed by") + " the next projection's staging)") if row_tp else (
                    f"column-shard x{world}" + (
                        "" if world == 1 else " + NCCL all-gather per projection" if args.nccl_gather else
                        ", outputs gathered by the GEMV epilogue (NVLink stores to IPC-mapped buffers + flags)")),
                "cuda_graph": cuda_graph_used,
            },
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": 2 * HIDDEN * world,
                    "d2h_bytes_per_step": (4 * HIDDEN * world) if row_tp else 2 * HIDDEN * world,
                    "ms_per_step": round(ms_e2e, 5)},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks,
            "launch_mode": launch_mode,
            "launch_modes": mode_results,
            "kernel_only": kernel_only,
            "parity": parity,
            "projections": projections,
            "prefill": prefill,
            "moe": moe,
            "c1": c1,
            "verify": verify,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


TRACE_PHASES = ("running", "predecessor complete", "peers' flags seen", "activation staged",
                "first stage landed", "stream consumed", "outputs stored", "exchange signalled",
                "stores fenced (exchange)", "flags written (exchange, last CTA)")
TRACE_STAMPS = len(TRACE_PHASES)


def _mean_or_none(v):
    v = [x for x in v if x is not None]
    return round(sum(v) / len(v), 3) if v else None


def trace_step(torch, lib, step, dev, path, barrier, world, rank):
    """One step with the GEMV's phase trace on (thq4_debug_set_trace), captured
    in its own CUDA graph and replayed (the last replay's stamps are kept).
    Writes, per launch, the CTA-median time of each phase after the launch's
    first CTA started, its span (first start to last exit) and the gap from the
    previous launch's last exit; and the same averaged per projection shape."""
    import numpy as np
    import thq4

    words = 1 << 22  # 32 MB of records
    buf = torch.zeros(words, dtype=torch.int64, device=dev)
    thq4.check(lib.thq4_debug_set_trace(ctypes.c_void_p(buf.data_ptr()), words * 8))
    g = torch.cuda.CUDAGraph()
    try:
        with torch.cuda.graph(g):
            step()
    finally:
        thq4.check(lib.thq4_debug_set_trace(None, 0))
    for _ in range(3):
        torch.cuda.synchronize()
        barrier()
        g.replay()
    torch.cuda.synchronize()
    g.reset()
    del g
    h = buf.cpu().numpy().view(np.uint64)
    if h.size and h[0] == 0x7468713463686e21:  # a chain launch: per (op, CTA) stamps
        return _trace_chain(h, path, world, rank)
    recs, off = [], 0
    while off + 8 <= h.size and h[off] == 0x7468713474726163:
        grid = int(h[off + 1])
        st = h[off + 8: off + 8 + TRACE_STAMPS * grid].reshape(grid, TRACE_STAMPS).astype(np.int64)
        flags = int(h[off + 4])
        recs.append({"out": int(h[off + 2]), "in": int(h[off + 3]), "gate_up": flags & 1,
                     "cluster": (flags >> 8) & 0xFF, "mode": (flags >> 16) & 0xFF, "wait": (flags >> 24) & 0xFF,
                     "m": int(h[off + 5]), "chunk": int(h[off + 6]) & 0xFF, "stages": int(h[off + 6]) >> 8,
                     "ctas": grid, "st": st})
        off += 8 + TRACE_STAMPS * grid
    launches, prev_end = [], None
    for r in recs:
        st = r.pop("st")
        t0 = int(st[:, 0].min())
        end = int(st[:, 7].max())
        med, mx = [], []
        for i in range(TRACE_STAMPS):
            col = st[:, i][st[:, i] > 0]  # stamps a CTA did not take stay 0
            med.append(round(float(np.median(col - t0)) / 1e3, 3) if col.size else None)
            mx.append(round(float((col - t0).max()) / 1e3, 3) if col.size else None)
        r.update({"span_us": round((end - t0) / 1e3, 3),
                  "gap_from_previous_exit_us": None if prev_end is None else round((t0 - prev_end) / 1e3, 3),
                  "phase_median_us": dict(zip(TRACE_PHASES, med)), "phase_max_us": dict(zip(TRACE_PHASES, mx)),
                  "stream_max_us": mx[5], "start_ns": t0})
        prev_end = end
        launches.append(r)
    base = launches[0]["start_ns"] if launches else 0
    for r in launches:
        r["start_us"] = round((r.pop("start_ns") - base) / 1e3, 3)
    kinds = {}
    for r in launches:
        key = f"{'gate_up 2x' if r['gate_up'] else ''}{r['out']}x{r['in']} m{r['m']}"
        kinds.setdefault(key, []).append(r)
    summary = {}
    for key, rs in kinds.items():
        gaps = [r["gap_from_previous_exit_us"] for r in rs if r["gap_from_previous_exit_us"] is not None]
        summary[key] = {
            "launches": len(rs), "ctas": rs[0]["ctas"], "cluster": rs[0]["cluster"], "chunk": rs[0]["chunk"],
            "stages": rs[0]["stages"], "mode": rs[0]["mode"], "wait": rs[0]["wait"],
            "span_us": round(float(np.mean([r["span_us"] for r in rs])), 3),
            "gap_us": round(float(np.mean(gaps)) if gaps else 0.0, 3),
            "phase_median_us": {p: _mean_or_none([r["phase_median_us"][p] for r in rs]) for p in TRACE_PHASES},
            "phase_max_us": {p: _mean_or_none([r["phase_max_us"][p] for r in rs]) for p in TRACE_PHASES}}
    step_us = max((r["start_us"] + r["span_us"] for r in launches), default=0.0)
    with open(path, "w") as f:
        json.dump({"world": world, "rank": rank, "launches": len(launches), "step_us": round(step_us, 3),
                   "per_shape": summary, "per_launch": launches}, f, indent=1)


CHAIN_PHASES = ("op begun", "activation staged", "stream consumed", "outputs stored")


def _trace_chain(h, path, world, rank):
    """The chain kernel's record: per op, the CTA medians of each phase after
    the op's first CTA began it, the longest stream, and the op's span from
    the previous op's last store to its own."""
    import numpy as np
    grid, n = int(h[1]), int(h[2])
    st = h[8: 8 + n * grid * 4].reshape(n, grid, 4).astype(np.int64)
    ops, prev_end = [], int(st[0, :, 0].min())
    base = prev_end
    for p in range(n):
        begun = st[p, :, 0]
        t0 = int(begun.min())
        act = st[p, :, 3] > 0  # CTAs with a run in this op
        end = int(st[p, act, 3].max()) if act.any() else t0
        med = {CHAIN_PHASES[i]: round(float(np.median(st[p, act, i] - t0)) / 1e3, 3) if act.any() else None
               for i in range(4)}
        ops.append({"op": p, "active": int(act.sum()), "begin_us": round((t0 - base) / 1e3, 3),
                    "span_us": round((end - prev_end) / 1e3, 3), "phase_median_us": med,
                    "stream_max_us": round(float((st[p, act, 2] - t0).max()) / 1e3, 3) if act.any() else None,
                    "store_max_us": round(float((st[p, act, 3] - t0).max()) / 1e3, 3) if act.any() else None})
        prev_end = end
    by_kind = {}
    for o in ops:
        by_kind.setdefault(o["op"] % 4, []).append(o)
    names = {0: "qkv", 1: "o", 2: "gate_up", 3: "down"}
    summary = {names[k]: {"span_us": round(float(np.mean([o["span_us"] for o in v])), 3),
                          "phase_median_us": {ph: round(float(np.mean([o["phase_median_us"][ph] for o in v
                                                                        if o["phase_median_us"][ph] is not None])), 3)
                                              for ph in CHAIN_PHASES},
                          "stream_max_us": round(float(np.mean([o["stream_max_us"] for o in v if o["stream_max_us"]])), 3),
                          "store_max_us": round(float(np.mean([o["store_max_us"] for o in v if o["store_max_us"]])), 3)}
               for k, v in by_kind.items()} if n % 4 == 0 else {}
    with open(path, "w") as f:
        json.dump({"world": world, "rank": rank, "kernel": "chain_kernel", "ops": n, "ctas": grid,
                   "stages": int(h[3]), "step_us": round((prev_end - base) / 1e3, 3), "per_kind": summary,
                   "per_op": ops}, f, indent=1)


def bench_c1(torch, thq4, synth, dev, hbm_peak, graph):
    """the single GEMV, x [1 x 2048] f32 ~ N(0, 1), W
    [6144 x 2048] Q4 ~ N(0, 0.02) with f16 scale/bias, y f32.  72 distinct
    weight copies (510 MB, > 4x L2) rotate inside one CUDA graph; GB/s =
    7,077,888 algorithmic bytes per launch / mean launch time."""
    out, inp, copies = 6144, 2048, 72
    ws = []
    for i in range(copies):
        wq, sb = synth.normal_weight(out, inp, 60_000 + i, dev)
        ws.append(thq4.PackedWeight.repack(thq4.SRC_MLX, wq, sb, out, inp, thq4.F16))
        del wq, sb
    lib = thq4.lib()
    wsb = lib.thq4_linear_workspace_bytes(ctypes.byref(ws[0].desc), 1)
    scratch = torch.zeros(wsb, dtype=torch.uint8, device=dev)
    x = torch.randn((1, inp), device=dev, dtype=torch.float32)
    y = torch.empty((1, out), dtype=torch.float32, device=dev)

    def call():
        s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        for w in ws:
            thq4.check(lib.thq4_linear(ctypes.byref(w.desc), ctypes.c_void_p(x.data_ptr()), thq4.F32, 1,
                                       ctypes.c_void_p(y.data_ptr()), thq4.F32, ctypes.c_void_p(scratch.data_ptr()),
                                       wsb, s))

    call()
    g = None
    if graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            call()
    run = g.replay if g is not None else call
    ms = _time_ms(torch, run, 20) / copies
    nbytes = out * inp * Q4_BYTES_PER_WEIGHT
    gbs = nbytes / (ms * 1e-3) / 1e9
    if g is not None:
        g.reset()
    return {"config": "x 1x2048 f32, W 6144x2048 Q4 (f16 scale/bias), y f32", "us": round(ms * 1e3, 3),
            "gbs": round(gbs, 1), "frac": round(gbs / hbm_peak, 4), "bytes": int(nbytes),
            "l2": f"{copies} weight copies ({copies * nbytes / 1e6:.0f} MB) rotate in one CUDA graph",
            "kernel": "gemv_kernel (f32 x split into fp16 hi/lo columns)"}


def bench_verify(torch, thq4, synth, dev, hbm_peak, graph):
    """spec-decode verify, x [M x 2560] bf16 ~ N(0, 1),
    M in {1, 2, 4, 8}; the fused gate/up 2 x 9728 x 2560 (SwiGLU epilogue)
    then down 2560 x 9728, Q4 f16 scale/bias.  12 distinct weight sets
    (504 MB, > 4x L2) rotate inside one CUDA graph per M; GB/s per kernel =
    its algorithmic bytes (28,016,640 and 14,008,320) / its mean launch time,
    each kernel timed in its own graph of 12 launches."""
    H, I, sets_n = 2560, 9728, 12
    sets = []
    for i in range(sets_n):
        g_wq, g_sb = synth.normal_weight(I, H, 70_000 + 3 * i, dev)
        u_wq, u_sb = synth.normal_weight(I, H, 70_001 + 3 * i, dev)
        d_wq, d_sb = synth.normal_weight(H, I, 70_002 + 3 * i, dev)
        sets.append((thq4.PackedWeight.repack(thq4.SRC_MLX, g_wq, g_sb, I, H, thq4.F16),
                     thq4.PackedWeight.repack(thq4.SRC_MLX, u_wq, u_sb, I, H, thq4.F16),
                     thq4.PackedWeight.repack(thq4.SRC_MLX, d_wq, d_sb, H, I, thq4.F16)))
        del g_wq, g_sb, u_wq, u_sb, d_wq, d_sb
    lib = thq4.lib()
    wsb = max(lib.thq4_linear_workspace_bytes(ctypes.byref(p.desc), 8) for st in sets for p in st)
    scratch = torch.zeros(wsb, dtype=torch.uint8, device=dev)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    gu_bytes, dn_bytes = 2 * I * H * Q4_BYTES_PER_WEIGHT, H * I * Q4_BYTES_PER_WEIGHT
    out = {"config": "x Mx2560 bf16; gate/up 2x9728x2560 then down 2560x9728, Q4 f16 scale/bias",
           "l2": f"{sets_n} weight sets ({sets_n * (gu_bytes + dn_bytes) / 1e6:.0f} MB) rotate in one CUDA graph",
           "kernel": "gemv_kernel with M token columns",
           "reference_m5max": "m=8 on an Apple M5 Max (other shapes): gate_up 34816x5120 530 GB/s, down 5120x17408 "
                              "400 GB/s (engine/reports/perf-2026-09/impl-th-wp2-matmul-roofline.md:142-143)"}
    for M in (1, 2, 4, 8):
        x = torch.randn((M, H), device=dev).to(torch.bfloat16)
        h = torch.empty((M, I), dtype=torch.bfloat16, device=dev)
        y = torch.empty((M, H), dtype=torch.bfloat16, device=dev)

        def gu_call():
            s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
            for g_, u_, _ in sets:
                thq4.check(lib.thq4_gate_up(ctypes.byref(g_.desc), ctypes.byref(u_.desc), P(x), thq4.BF16, M, P(h),
                                            thq4.BF16, P(scratch), wsb, s))

        def dn_call():
            s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
            for _, _, d_ in sets:
                thq4.check(lib.thq4_linear(ctypes.byref(d_.desc), P(h), thq4.BF16, M, P(y), thq4.BF16, P(scratch),
                                           wsb, s))

        res = {}
        for name, fn, nb in (("gate_up", gu_call, gu_bytes), ("down", dn_call, dn_bytes)):
            fn()
            g = None
            if graph:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    fn()
            ms = _time_ms(torch, g.replay if g is not None else fn, 20) / sets_n
            gbs = nb / (ms * 1e-3) / 1e9
            res[name] = {"us": round(ms * 1e3, 3), "gbs": round(gbs, 1), "frac": round(gbs / hbm_peak, 4)}
            if g is not None:
                g.reset()
        out[f"m{M}"] = res
    return out


def _time_ms(torch, fn, reps):
    """Mean ms per call: CUDA events on the current stream after 3 warm-up
    calls (the callers rotate operands larger than L2)."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def bench_prefill(torch, thq4, synth, dev, tc_peak, peak_kind):
    """x [M x 4096] bf16 ~ N(0,1), W [12288 x 4096] Q4
    with f16 scale/bias, M = 512 (headline) and 2048 -> TFLOP/s.  Four weight
    copies (113 MB) rotate so the weight stream is not served from L2."""
    N, K = 12288, 4096
    ws = []
    for i in range(4):
        wq, sb = synth.normal_weight(N, K, 99 + i, dev)
        ws.append(thq4.PackedWeight.repack(thq4.SRC_MLX, wq, sb, N, K, thq4.F16))
        del wq, sb
    lib = thq4.lib()
    out = {"kernel": "prefill_kernel (tcgen05.mma kind::f16, dequantised weights in TMEM, x by TMA)",
           "peak_tflops": tc_peak, "peak_kind": peak_kind}
    for M in (512, 2048):
        x = torch.randn((M, K), device=dev).to(torch.bfloat16)
        y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
        # the workspace thq4_linear asks for at M rows: room for the stream-K
        # parts, so the k-stages are split evenly over the SMs
        wsb = lib.thq4_linear_workspace_bytes(ctypes.byref(ws[0].desc), M)
        wsp = torch.zeros(max(wsb, 256), dtype=torch.uint8, device=dev)

        def call():
            s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
            for w in ws:
                thq4.check(lib.thq4_linear(ctypes.byref(w.desc), ctypes.c_void_p(x.data_ptr()), thq4.BF16, M,
                                           ctypes.c_void_p(y.data_ptr()), thq4.BF16, ctypes.c_void_p(wsp.data_ptr()),
                                           wsp.numel(), s))

        ms = _time_ms(torch, call, 10) / len(ws)
        tflops = 2.0 * M * N * K / (ms * 1e-3) / 1e12
        out[f"m{M}"] = {"config": f"x {M}x4096 bf16, W 12288x4096 Q4 (f16 scale/bias)", "tflops": round(tflops, 2),
                        "us": round(ms * 1e3, 2), "frac": round(tflops / tc_peak, 4)}
    return out


def synthetic_router(torch, H, dev, seed):
    """A random Q8 router (StorageN = 256 order) for the MoE block."""
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    G = H // 64
    q = torch.randint(0, 256, (G * 256 * 64,), dtype=torch.uint8, device=dev, generator=g)
    sc = (torch.rand((G * 256,), device=dev, generator=g) * 0.0035 + 0.0005).to(torch.bfloat16)
    bi = (torch.randn((G * 256,), device=dev, generator=g) * 0.05).to(torch.bfloat16)
    return q, sc, bi


def bench_moe(torch, thq4, synth, dev, hbm_peak):
    """T = 256 tokens, H = 2048, E = 128 experts, top-8,
    I = 768, Q4 f16 scale/bias, through thq4_moe_add (MoE::add: the Q8
    router, routing, gather, grouped gate/up and down products, combine; no
    shared expert, as the config has none) -> expert-weight GB/s (339,738,624
    algorithmic bytes, every expert touched) and us per layer.  Two expert
    sets (680 MB) rotate."""
    T, H, I, E, k = 256, 2048, 768, 128, 8
    sets = []
    for s in range(2):
        gu = [synth.normal_weight(2 * I, H, 10_000 * (s + 1) + e, dev) for e in range(E)]
        gu_wq, gu_sb = torch.stack([a for a, _ in gu]), torch.stack([b for _, b in gu])
        del gu
        dn = [synth.normal_weight(H, I, 20_000 * (s + 1) + e, dev) for e in range(E)]
        dn_wq, dn_sb = torch.stack([a for a, _ in dn]), torch.stack([b for _, b in dn])
        del dn
        sets.append((thq4.PackedExperts.from_mlx(gu_wq, gu_sb, thq4.F16, 0, I),
                     thq4.PackedExperts.from_mlx(gu_wq, gu_sb, thq4.F16, I, I),
                     thq4.PackedExperts.from_mlx(dn_wq, dn_sb, thq4.F16)))
        del gu_wq, gu_sb, dn_wq, dn_sb
    x = torch.randn((T, H), device=dev).to(torch.bfloat16)
    blocks = [thq4.MoeWeights(thq4.Q8Projection(*synthetic_router(torch, H, dev, 77 + i), H), g, u, d)
              for i, (g, u, d) in enumerate(sets)]

    def call():
        for w in blocks:
            thq4.moe_add(x, w, k)

    ms = _time_ms(torch, call, 10) / len(sets)
    nbytes = E * (2 * I * H + H * I) * Q4_BYTES_PER_WEIGHT
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"config": "T 256, H 2048, E 128, k 8, I 768, Q4 f16 scale/bias, Q8 router", "us": round(ms * 1e3, 2),
            "weight_gbs": round(gbs, 1), "frac": round(gbs / hbm_peak, 4), "bytes": int(nbytes),
            "kernel": "thq4_moe_add: route_scores_kernel (Q8 router) + select / group / gather + moe_gemv_kernel "
                      "(grouped small-tile mma.sync experts) + combine"}


def bench_moe_sharded(torch, thq4, synth, dev, hbm_peak, world, rank, local):
    """BASELINE configs[4] with the experts split E/N per GPU: every rank
    routes all 256 tokens through the same Q8 router (bit-identically), runs
    its experts' routes (thq4_moe_add_partial, f32 partial) and one NCCL
    all-reduce sums the partials; whole-job expert-weight GB/s and us per
    layer, max over ranks.  Two expert sets rotate."""
    import torch.distributed as dist

    from thq4.shard import expert_range, moe_add_sharded

    T, H, I, E, k = 256, 2048, 768, 128, 8
    e0, n = expert_range(E, world, rank)
    sets = []
    for s in range(2):
        gu = [synth.normal_weight(2 * I, H, 10_000 * (s + 1) + e0 + e, dev) for e in range(n)]
        gu_wq, gu_sb = torch.stack([a for a, _ in gu]), torch.stack([b for _, b in gu])
        del gu
        dn = [synth.normal_weight(H, I, 20_000 * (s + 1) + e0 + e, dev) for e in range(n)]
        dn_wq, dn_sb = torch.stack([a for a, _ in dn]), torch.stack([b for _, b in dn])
        del dn
        sets.append((thq4.PackedExperts.from_mlx(gu_wq, gu_sb, thq4.F16, 0, I),
                     thq4.PackedExperts.from_mlx(gu_wq, gu_sb, thq4.F16, I, I),
                     thq4.PackedExperts.from_mlx(dn_wq, dn_sb, thq4.F16)))
        del gu_wq, gu_sb, dn_wq, dn_sb
    g = torch.Generator(device=dev)
    g.manual_seed(1234)  # the same activations and logits on every rank
    x = torch.randn((T, H), device=dev, generator=g).to(torch.bfloat16)
    blocks = [thq4.MoeWeights(thq4.Q8Projection(*synthetic_router(torch, H, dev, 77 + i), H), gt, up, dn)
              for i, (gt, up, dn) in enumerate(sets)]

    def call():
        for w in blocks:
            moe_add_sharded(x, w, k, e0, E)

    for _ in range(3):
        call()
    torch.cuda.synchronize()
    dist.barrier(device_ids=[local])
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(10):
        call()
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / (10 * len(sets))], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    nbytes = E * (2 * I * H + H * I) * Q4_BYTES_PER_WEIGHT
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"config": f"T 256, H 2048, E 128 ({n} per GPU), k 8, I 768, Q4 f16 scale/bias", "us": round(ms * 1e3, 2),
            "weight_gbs": round(gbs, 1), "frac": round(gbs / (hbm_peak * world), 4), "bytes": int(nbytes),
            "kernel": "thq4_moe_add_partial per expert shard + NCCL all-reduce of the f32 partials"}


# ---------------------------------------------------------------------------
# CPU baseline (oracle port of the reference CPU semantics)
# ---------------------------------------------------------------------------
def _cpu_layer(seed: int):
    """One layer's MLX weights made on the CPU (same quantiser), as numpy."""
    import numpy as np
    import torch
    from thq4 import synth
    out = []
    for i, (rows, inp) in enumerate([(HIDDEN + 2 * KV, HIDDEN), (HIDDEN, HIDDEN), (2 * INTER, HIDDEN), (HIDDEN, INTER)]):
        wq, sb = synth.normal_weight(rows, inp, seed + i, "cpu")
        out.append((wq.numpy().view(np.uint32), sb.view(torch.int16).numpy().view(np.uint16), rows, inp))
    return out


def _cpu_step(O, layer, xs):
    for (wq, sb, rows, inp) in layer:
        O.cpu_linear(wq, sb, O.SB_F16, xs[inp])


def cpu_baseline(seconds: float):
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import q4oracle as O
    layer = _cpu_layer(5)
    rng = np.random.default_rng(0)
    xs = {HIDDEN: rng.standard_normal((1, HIDDEN)).astype(np.float32),
          INTER: rng.standard_normal((1, INTER)).astype(np.float32)}
    _cpu_step(O, layer, xs)
    n = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        _cpu_step(O, layer, xs)
        n += 1
    dt = time.perf_counter() - t0
    threads = O.threads()
    return {"value": round(LAYER_BYTES * n / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{n} passes over one decode layer's projections ({LAYER_BYTES / 1e6:.1f} MB Q4, MLX layout), "
                      f"dequantise-to-bf16 + f32 accumulate, {threads} threads, {dt:.1f} s"}


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import q4oracle as O
    layer = _cpu_layer(5)
    rng = np.random.default_rng(0)
    xs = {HIDDEN: rng.standard_normal((1, HIDDEN)).astype(np.float32),
          INTER: rng.standard_normal((1, INTER)).astype(np.float32)}
    t0 = time.perf_counter()
    _cpu_step(O, layer, xs)
    t_one = time.perf_counter() - t0
    # bound the run to ~2 minutes: sample fewer projections per step if needed
    sample = layer
    label = "one decode layer's projections"
    if t_one * (args.steps + args.warmup) > 120:
        sample = [layer[1]]
        label = "the o projection (5120x5120) of one decode layer"
    sample_bytes = sum(int(r * i * Q4_BYTES_PER_WEIGHT) for (_, _, r, i) in sample)
    for _ in range(args.warmup):
        _cpu_step(O, sample, xs)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        _cpu_step(O, sample, xs)
    dt = (time.perf_counter() - t0) / args.steps
    value = sample_bytes / dt / 1e9
    threads = O.threads()
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 3),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: x ~ N(0,1); W ~ N(0,0.02) quantised Q4 affine group-64, f16 scale/bias",
        "config": {"workload": "decode-layer projection set, hidden 5120, batch 1 (CPU sample: " + label + ")",
                   "hidden": HIDDEN, "intermediate": INTER, "group": 64, "scale_dtype": "f16"},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{label}, {sample_bytes / 1e6:.1f} MB Q4 per step, reference CPU semantics "
                                   f"(dequantise to bf16, f32 accumulate), {threads} threads"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_thq4(args)


if __name__ == "__main__":
    main()
