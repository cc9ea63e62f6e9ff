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
consumes the previous one's output.  With N GPUs every projection is
column-sharded (rows split in multiples of 16) and its output is
all-gathered over NVLink with NCCL before the next projection reads it.

One JSON line on rank 0: `value` is algorithmic weight bytes of the whole job
per step / max-over-ranks step time (GB/s), the step captured in a CUDA graph
and timed with CUDA events; `e2e` is the same metric with the input copied
from pinned host memory and the result read back inside the timed region;
`roofline` times the dominant kernel (the fused gate/up GEMV) alone;
`cpu_baseline` times the CPU restatement of the reference's CPU path on a
bounded sample (N=1 only); `prefill` reports the prefill GEMM (BASELINE
configs[2], M=512) in TFLOP/s.

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
    p.add_argument("--skip-prefill", action="store_true")
    p.add_argument("--nccl-gather", action="store_true",
                   help="N > 1: gather each projection's output with NCCL all-gather (the baseline) instead of "
                        "the GEMV epilogue's NVLink stores")
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

    layers = []
    for l in range(L):
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
        o = packed_cols(HIDDEN, HIDDEN, s + 4, q0, qn) if row_tp else packed(HIDDEN, HIDDEN, s + 4, q0, qn)
        gate = packed(INTER, HIDDEN, s + 5, i0, inn)
        up = packed(INTER, HIDDEN, s + 6, i0, inn)
        down = packed_cols(HIDDEN, INTER, s + 7, i0, inn) if row_tp else packed(HIDDEN, INTER, s + 7, q0, qn)
        layers.append((qkv, o, gate, up, down))
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
        from thq4.shard import PeerGroup

        peer = PeerGroup(2 * world * HIDDEN * 4 + 4 * 256, dev)
        red_o, red_d = peer.buffer(peer.reduction_bytes(HIDDEN, 1)), peer.buffer(peer.reduction_bytes(HIDDEN, 1))
        g_qkv = peer.local_out(wait=True, x_parts=world, x_slot=HIDDEN)
        g_o = peer.reduce(red_o, HIDDEN, 1, wait=False)
        g_gu = peer.local_out(wait=True, x_parts=world, x_slot=HIDDEN)
        g_dn = peer.reduce(red_d, HIDDEN, 1, wait=False)
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

    def step_peer():
        s = stream()
        for (qkv, o, gate, up, down) in layers:
            thq4.check(lib.thq4_linear_peer(ctypes.byref(qkv.desc), None, P(x_in), BF, 1, P(t_qkv), P(ws), ws_bytes,
                                            ctypes.byref(g_qkv), s))
            thq4.check(lib.thq4_linear_peer(ctypes.byref(o.desc), None, V(off_q), BF, 1, P(t_o), P(ws), ws_bytes,
                                            ctypes.byref(g_o), s))
            thq4.check(lib.thq4_linear_peer(ctypes.byref(gate.desc), ctypes.byref(up.desc), V(off_o), BF, 1, P(t_h),
                                            P(ws), ws_bytes, ctypes.byref(g_gu), s))
            thq4.check(lib.thq4_linear_peer(ctypes.byref(down.desc), None, V(off_h), BF, 1, P(t_d), P(ws), ws_bytes,
                                            ctypes.byref(g_dn), s))

    def step_row():
        s = stream()
        for li, (qkv, o, gate, up, down) in enumerate(layers):
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
                                            ctypes.byref(g_dn), s))

    def step():
        if row_tp:
            return step_row()
        if peer is not None:
            return step_peer()
        s = stream()
        for (qkv, o, gate, up, down) in layers:
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

    launches_per_step = 4 * L

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

    # e2e: pinned host input -> device, step, result -> pinned host
    x_host = torch.empty((1, HIDDEN), dtype=torch.bfloat16).pin_memory()
    x_host.copy_(x_in.cpu())
    y_host = torch.empty((1, HIDDEN), dtype=torch.bfloat16).pin_memory()

    if row_tp:  # the step's result is the last down's partials, one per rank
        y_host = torch.empty((world, HIDDEN), dtype=torch.float32).pin_memory()

    def e2e_body():
        x_in.copy_(x_host, non_blocking=True)
        run()
        if row_tp:
            thq4.check(lib.thq4_peer_wait(ctypes.byref(g_gu), stream()))
            thq4.check(lib.thq4_copy(P(y_host), V(red_d), world * HIDDEN * 4, stream()))
        elif peer is not None:
            thq4.check(lib.thq4_copy(P(y_host), V(off_y), HIDDEN * 2, stream()))
        else:
            y_host.copy_(y_out, non_blocking=True)

    for _ in range(3):
        e2e_body()
    ms_e2e = timed(e2e_body, args.steps) / args.steps
    e2e_value = total_bytes / (ms_e2e * 1e-3) / 1e9

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

    cpu = None
    if rank == 0 and world == 1:
        cpu = cpu_baseline(args.cpu_seconds)

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
                                "+ flags, summed by the next projection's staging)") if row_tp else (
                    f"column-shard x{world}" + (
                        "" if world == 1 else " + NCCL all-gather per projection" if args.nccl_gather else
                        ", outputs gathered by the GEMV epilogue (NVLink stores to IPC-mapped buffers + flags)")),
                "cuda_graph": cuda_graph_used,
            },
            "roofline": {"bound": "hbm", "kernel": "gemv_kernel (fused gate/up, SwiGLU epilogue)",
                         "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(achieved / hbm_peak, 4), "peak_kind": peak_kind,
                         "traffic": traffic, "bytes_per_launch": int(gu_bytes), "us_per_launch": round(ms_gu * 1e3, 3),
                         "step_frac": round(value / world / hbm_peak, 4)},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": 2 * HIDDEN * world,
                    "d2h_bytes_per_step": (4 * HIDDEN * world * world) if row_tp else 2 * HIDDEN * world,
                    "ms_per_step": round(ms_e2e, 5)},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks,
            "prefill": prefill,
            "moe": moe,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


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

        def call():
            s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
            for w in ws:
                thq4.check(lib.thq4_linear(ctypes.byref(w.desc), ctypes.c_void_p(x.data_ptr()), thq4.BF16, M,
                                           ctypes.c_void_p(y.data_ptr()), thq4.BF16, None, 0, s))

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
