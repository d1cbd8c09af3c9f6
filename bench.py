"""Benchmark of the sparse-voxel hot path on B200 (one JSON line on rank 0).

Workloads (seeded synthetic surfaces, mogecpp_b200/synth.py; C = 128, fp16
state, ggml Q8_0 weights, LayerNorm -> SiLU -> submanifold conv 3x3x3 ->
SiLU -> conv -> +skip per residual block):

* ``shell_4m`` (default) - 3,145,728 voxels, a 3-voxel-thick height shell on
  a 1024^3 grid, 8 residual blocks: the large sharded configuration, run on
  1/2/4/8 GPUs.
* ``res4_c128`` - 364,846 voxels on a 256^3 grid, 4 residual blocks.

One step = rebuild the topology (hash + 27-tap neighbour map, as the refiner
does on every refine pass) and run the residual stack (2 sparse convs per
block).  The convs gather through the neighbour map; ``--conv ordered``
(default) also builds the level's tap-order plan (voxels sorted by their
27-tap neighbourhood mask, so that each 128-row tile runs over fewer taps),
``--conv direct`` runs the tiles in (b, z, y, x) order, and ``--conv
cached`` builds the row-cache plan and runs the row-cached conv.

    value = active voxels x sparse convs per step / step time   (device-resident inputs)
    e2e   = the same, through the C ABI with host buffers: the step's coordinates and
            features are copied from pinned host memory and the result copied back
            inside the timed region.

Multi-GPU (torchrun, one process per GPU): the voxels are split into z-slabs
at voxel-count quantiles (mogecpp_b200/slab.py); each rank builds the
topology of its slab plus a two-plane halo per side and, before every block,
exchanges the boundary planes with its z-neighbours over NCCL.  Total work
is fixed ("scaling": "strong"); timing is the max over ranks.

``--impl reference`` times the reference's own CPU implementation (mogecpp
src/sparse.cpp + ggml CPU backend, compiled from the reference sources into
oracle/_ref/) on a bounded voxel sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

C_CH = 128
METRIC = "active voxels/s per sparse conv"
# block: the residual block each workload is quoted on: "ln" is the
# reference's res_block (LayerNorm -> SiLU -> conv -> SiLU -> conv -> +x),
# "gn" the GroupNorm(32) block (conv -> GroupNorm -> SiLU -> conv -> +x)
WORKLOADS = {
    "shell_4m": dict(blocks=8, coords="shell_4m_coords", grid=1024, block="ln"),
    "res4_c128": dict(blocks=4, coords="res4_c128_coords", grid=256, block="gn"),
}
GN_EPS = 1e-5
BLOCK_NAME = {"ln": "LayerNorm res_block", "gn": "GroupNorm(32) res block"}
# DRAM bytes per voxel of one sparse-conv launch, by residual-block kind:
# dram__bytes_read.sum + dram__bytes_write.sum from one ncu capture of a
# block's two convs on res4_c128, averaged (profiles/conv_traffic_res4_c128.md).
# Other workloads scale it by the voxels a launch processes.
CONV_DRAM_BYTES_PER_VOXEL = {"gn": 860.0, "ln": 646.0}
PLAN_SORT_KERNELS = 8  # cub onesweep radix sort of 55-bit keys: histogram + 7 digit passes


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p["hbm_gbs"]), "measured"
    except Exception:
        return 1590.0, 6650.0, "fallback"


def workload_inputs(name: str, rows=None):
    """Coordinates (all voxels), the fp16 features of `rows` (default: all)
    and the residual blocks' parameters."""
    from mogecpp_b200 import synth
    w = WORKLOADS[name]
    coords = getattr(synth, w["coords"])()
    n = coords.shape[0]
    x0 = synth.features_rows(2, np.arange(n) if rows is None else rows, C_CH, np.float16)
    blocks = []
    for b in range(w["blocks"]):
        rng = np.random.default_rng(1000 + b)
        blk = dict(norm_w=(1 + 0.1 * rng.standard_normal(C_CH)).astype(np.float32),
                   norm_b=(0.1 * rng.standard_normal(C_CH)).astype(np.float32),
                   w1=synth.conv_weight(2000 + 2 * b, C_CH, C_CH),
                   b1=(0.05 * rng.standard_normal(C_CH)).astype(np.float32),
                   w2=synth.conv_weight(2001 + 2 * b, C_CH, C_CH),
                   b2=(0.05 * rng.standard_normal(C_CH)).astype(np.float32))
        blk["gn_w"], blk["gn_b"] = blk["norm_w"], blk["norm_b"]  # the one affine serves either norm
        blocks.append(blk)
    return coords, x0, blocks


def cpu_stack(impl, x, nbr, blocks, block_kind):
    """One pass of the residual stack on the CPU: `impl` is the reference
    build (Reference) or the oracle (Oracle).  Returns seconds."""
    from oracle.oracle import Reference, W_Q8_0
    is_ref = isinstance(impl, Reference)
    if block_kind == "ln" and is_ref:
        return impl.res_stack(x, nbr, blocks, W_Q8_0, iters=1)[1]
    t0 = time.perf_counter()
    h = x
    sample = np.zeros(x.shape[0], np.int32)
    for b in blocks:
        if block_kind == "ln":
            h = impl.res_block(h, nbr, b, W_Q8_0)
        elif is_ref:
            h = impl.res_block_gn(h, nbr, b, W_Q8_0, 32, GN_EPS)
        else:
            h = impl.res_block_gn(h, nbr, sample, b, W_Q8_0, 32, GN_EPS)
    return time.perf_counter() - t0


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""
    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clocks_setting"}

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = os.path.join("/tmp", f"msc_clocks_{os.getpid()}.csv")

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index),
                 "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active",
                 "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, mx, reasons = [], None, set()
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 4:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
                mask = int(parts[3], 16)
            except ValueError:
                continue
            for bit, name in self.REASONS.items():
                if mask & bit and name != "gpu_idle":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def cpu_reference_sample(coords, x0, blocks, target_s: float, n_threads: int, block_kind: str):
    """Times the reference CPU res-block stack on the first voxels of the
    (b, z, y, x)-ordered set (a z-slab), sized to about target_s per run."""
    from oracle.oracle import Oracle, Reference
    try:
        R = Reference(n_threads=n_threads)
        kind = "reference"
    except FileNotFoundError:
        R = Oracle()
        kind = "port"
    ns = min(coords.shape[0], 4096)
    for _ in range(3):
        nbr = R.make_level(coords[:ns])
        sec = cpu_stack(R, x0[:ns].astype(np.float32), nbr, blocks, block_kind)
        if sec >= 0.5 * target_s or ns == coords.shape[0]:
            break
        ns = int(min(coords.shape[0], ns * max(2.0, target_s / max(sec, 1e-3))))
    return R, kind, ns, sec


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from mogecpp_b200 import synth
    coords = getattr(synth, WORKLOADS[args.workload]["coords"])()
    # the sample is the first voxels: draw only those features
    _, x0, blocks = workload_inputs(args.workload, np.arange(min(coords.shape[0], 1 << 18)))
    coords = coords[:x0.shape[0]]
    convs = 2 * len(blocks)
    threads = os.cpu_count() or 1
    per_step = min(8.0, 150.0 / max(1, args.steps + args.warmup))
    R, kind, ns, _ = cpu_reference_sample(coords, x0, blocks, per_step, threads, args.block)
    if kind == "port":
        threads = 1
    nbr = R.make_level(coords[:ns])
    times = []
    for i in range(args.warmup + args.steps):
        sec = cpu_stack(R, x0[:ns].astype(np.float32), nbr, blocks, args.block)
        if i >= args.warmup:
            times.append(sec)
    t = sum(times) / len(times)
    value = ns * convs / t
    sample = (f"first {ns} voxels of {args.workload} in (b,z,y,x) order (a z-slab), {len(blocks)} x "
              f"{BLOCK_NAME[args.block]}, Q8_0")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "voxels/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "q8_0 x fp32 (ggml CPU)", "data": "synthetic",
            "config": {"workload": args.workload, "voxels": int(ns), "channels": C_CH, "blocks": len(blocks),
                       "block": BLOCK_NAME[args.block]},
            "cpu_baseline": {"value": value, "unit": "voxels/s", "cores": threads, "kind": kind, "sample": sample},
            "e2e": {"value": value, "unit": "voxels/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ours(args):
    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    from mogecpp_b200 import slab, synth
    from mogecpp_b200.sparse import SparseCudaExecutor

    ex = SparseCudaExecutor(local)
    coords = getattr(synth, WORKLOADS[args.workload]["coords"])()
    part = slab.partition(coords, world)[rank]
    rows = part.local_rows()
    # this rank's rows only (and rank 0's CPU sample, the first voxels)
    _, lx0, blocks_np = workload_inputs(args.workload, rows)
    n = coords.shape[0]
    convs = 2 * len(blocks_np)
    lcoords = np.ascontiguousarray(coords[rows])
    nl = lcoords.shape[0]
    dev = torch.device("cuda", local)
    coords_d = torch.from_numpy(lcoords).to(dev)
    x0_d = torch.from_numpy(lx0).to(dev)
    x_d = torch.empty_like(x0_d)
    halo = slab.SlabExchange(part, world)
    blocks = []
    for b in blocks_np:
        blocks.append(dict(norm_w=torch.from_numpy(b["norm_w"]).to(dev), norm_b=torch.from_numpy(b["norm_b"]).to(dev),
                           gn_w=torch.from_numpy(b["gn_w"]).to(dev), gn_b=torch.from_numpy(b["gn_b"]).to(dev),
                           b1=torch.from_numpy(b["b1"]).to(dev), b2=torch.from_numpy(b["b2"]).to(dev),
                           w1=ex.prepare_weight(torch.from_numpy(synth.quantize_q8_0(b["w1"])).to(dev), "q8_0",
                                                C_CH, C_CH, 27),
                           w2=ex.prepare_weight(torch.from_numpy(synth.quantize_q8_0(b["w2"])).to(dev), "q8_0",
                                                C_CH, C_CH, 27)))
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    cached = args.conv == "cached"
    plan_kind = {"cached": "row_cache", "ordered": "tap_order"}.get(args.conv)

    # GroupNorm statistics are sample-wide: summed over the slabs (NCCL)
    gn_allreduce = (lambda t: dist.all_reduce(t)) if world > 1 else None

    def step(coords_t=coords_d, x_t=x_d):
        nbr = ex.make_level(coords_t)
        plan = ex.conv_plan(coords_t, nbr, plan_kind) if plan_kind else None
        for blk in blocks:
            halo.exchange(x_t)
            if args.block == "gn":
                ex.res_block_gn(x_t, None if cached else nbr, coords_t, 1, blk, eps=GN_EPS, plan=plan,
                                n_stat=part.n_owned, allreduce=gn_allreduce)
            else:
                ex.res_block(x_t, None if cached else nbr, blk, plan=plan)
        return nbr

    def barrier():
        if world > 1:
            dist.barrier()

    barrier()
    # warm-up (also validates device status once)
    for _ in range(args.warmup):
        x_d.copy_(x0_d)
        nbr = step()
    ex.check()
    e_pairs = int((nbr < nl).sum().item())
    barrier()

    # ---- device-resident timed region
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    torch.cuda.synchronize()
    barrier()
    ex.profile(True)
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            x_d.copy_(x0_d)
            flush.fill_(i & 0xff)  # L2 flush between steps (outside the events)
            barrier()
            ev[i][0].record()
            step()
            ev[i][1].record()
        torch.cuda.synchronize()
    ex.profile(False)
    prof = ex.profile_read()
    ex.check()
    step_ms = [a.elapsed_time(b) for a, b in ev]
    t_ms = sum(step_ms) / len(step_ms)
    if world > 1:
        t = torch.tensor([t_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_ms = float(t.item())
        barrier()
    value = n * convs / (t_ms * 1e-3)

    # ---- end to end through the C ABI with host buffers: a stream of steps,
    # each with the host->device copy of its inputs (pinned) and the
    # device->host copy of its result.  Inputs are double-buffered on the
    # device and the copies run on their own streams, so step i+1's input copy
    # and step i's result copy overlap step i's compute, as a serving loop
    # would run them.  Timed from the first input copy to the last result
    # copy of the K steps (pipeline fill and drain included).
    h_coords = torch.from_numpy(lcoords).pin_memory()
    h_x = torch.from_numpy(lx0).pin_memory()
    h_out = [torch.empty((part.n_owned, C_CH), dtype=x0_d.dtype).pin_memory() for _ in range(2)]
    bufs = [(coords_d, x_d), (torch.empty_like(coords_d), torch.empty_like(x_d))]
    comp = torch.cuda.current_stream()
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_comp = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def e2e_run(k):
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

        def copy_in(i):
            bi = i % 2
            if i >= 2:
                s_in.wait_event(ev_out[bi])  # step i-2's result copy has read this buffer
            with torch.cuda.stream(s_in):
                if i == 0:
                    t0.record(s_in)
                bufs[bi][0].copy_(h_coords, non_blocking=True)
                bufs[bi][1].copy_(h_x, non_blocking=True)
                ev_in[bi].record(s_in)

        torch.cuda.synchronize()
        barrier()
        copy_in(0)
        for i in range(k):
            bi = i % 2
            if i + 1 < k:
                copy_in(i + 1)
            comp.wait_event(ev_in[bi])
            flush.fill_(i & 0xff)  # L2 flush between steps
            step(*bufs[bi])
            ev_comp[bi].record(comp)
            s_out.wait_event(ev_comp[bi])
            with torch.cuda.stream(s_out):
                h_out[bi].copy_(bufs[bi][1][:part.n_owned], non_blocking=True)
                ev_out[bi].record(s_out)
                if i == k - 1:
                    t1.record(s_out)
        torch.cuda.synchronize()
        return t0.elapsed_time(t1) / k

    e2e_run(args.warmup)
    e2e_t = e2e_run(args.steps)
    ex.check()
    if world > 1:
        t = torch.tensor([e2e_t], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_t = float(t.item())

    # ---- roofline of the dominant kernel (tensor-core sparse conv)
    peak_tf, peak_hbm, peak_src = load_peaks()
    conv_family = "conv_cached" if cached else "conv_tc"
    conv_launches, conv_ms = prof.get(conv_family, (0, 0.0))
    flops_per_launch = 2.0 * C_CH * C_CH * e_pairs
    achieved = flops_per_launch / (conv_ms / max(conv_launches, 1) * 1e-3) / 1e12 if conv_launches else None
    # launches per profiled call: make_level = clear + insert + neighbour kernels;
    # plan_build = header + Morton keys + the radix sort's kernels + subtiles
    # (row-cache: + subtiles; tap order: header + mask keys + histogram, scan and 4 passes of a 27-bit sort
    # + the per-tile neighbour lists)
    plan_kernels = 3 + PLAN_SORT_KERNELS if cached else 2 + 6 + 1
    kernels_per_family = {"make_level": 3, "plan_build": plan_kernels, "conv_tc": 1, "conv_cached": 1,
                          "act_prepare": 1}
    launches = sum(kernels_per_family.get(k, 1) * v[0] for k, v in prof.items())

    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            R, kind, ns, sec = cpu_reference_sample(coords, lx0, blocks_np, 6.0, os.cpu_count() or 1, args.block)
            cpu = {"value": ns * convs / sec, "unit": "voxels/s",
                   "cores": (os.cpu_count() or 1) if kind == "reference" else 1, "kind": kind,
                   "sample": f"first {ns} voxels in (b,z,y,x) order (a z-slab), one run of {len(blocks_np)} x "
                             f"{BLOCK_NAME[args.block]}"}
        line = {
            "metric": METRIC, "value": value, "unit": "voxels/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t_ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None,
            "dtype": "q8_0 (int8 codes exact on tcgen05, per-32-block fp32 scaling as ggml)",
            "data": "synthetic",
            "config": {"workload": args.workload, "voxels": n, "channels": C_CH, "blocks": len(blocks_np),
                       "convs_per_step": convs, "grid": WORKLOADS[args.workload]["grid"],
                       "rank0_local_voxels": nl, "rank0_valid_pairs": e_pairs,
                       "block": BLOCK_NAME[args.block],
                       "step": (f"make_level + {plan_kind} plan + " if plan_kind else "make_level + ") +
                               f"{len(blocks_np)} res blocks" + (" (halo exchange before each)" if world > 1 else "") +
                               (", GroupNorm statistics all-reduced" if world > 1 and args.block == "gn" else ""),
                       "conv": args.conv, "l2": "flushed between steps (256 MiB write)",
                       "parallelism": f"z-slabs x{world}, 2-plane halo over NCCL" if world > 1 else "single GPU"},
            "e2e": {"value": n * convs / (e2e_t * 1e-3), "unit": "voxels/s",
                    "h2d_bytes_per_step": int(lcoords.nbytes + lx0.nbytes),
                    "d2h_bytes_per_step": int(part.n_owned * C_CH * lx0.itemsize), "ms_per_step": e2e_t,
                    "copies": "pinned host buffers; step i+1's input copy and step i's result copy overlap "
                              "step i's compute (two copy streams, double-buffered device inputs)"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s",
                         "frac": (achieved / peak_tf) if achieved else None,
                         "traffic": (CONV_DRAM_BYTES_PER_VOXEL[args.block] * nl
                                     if CONV_DRAM_BYTES_PER_VOXEL.get(args.block) else None),
                         "traffic_unit": "bytes per conv launch (ncu capture, scaled by voxels)",
                         "kernel": f"{conv_family} (Q8_0, C=128)", "peak_source": peak_src,
                         "flops_per_launch": flops_per_launch,
                         "avg_launch_ms": conv_ms / max(conv_launches, 1)},
            "effective_tflops_per_conv": achieved,
            "kernel_ms_per_step": {k: v[1] / args.steps for k, v in prof.items()},
            "gpu_launches": int(launches),
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="shell_4m", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--conv", default="ordered", choices=["ordered", "direct", "cached"])
    ap.add_argument("--block", default=None, choices=["ln", "gn"],
                    help="residual block (default: the one the workload is quoted on)")
    args = ap.parse_args()
    if args.block is None:
        args.block = WORKLOADS[args.workload]["block"]
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
