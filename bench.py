"""Benchmark of the sparse-voxel hot path on B200 (one JSON line on rank 0).

Workloads (seeded synthetic surfaces, mogecpp_b200/synth.py):

* ``shell_4m`` (default) - 3,145,728 voxels, a 3-voxel-thick height shell on
  a 1024^3 grid, 8 residual blocks (LayerNorm -> SiLU -> submanifold conv
  3x3x3 -> SiLU -> conv -> +skip) at C = 128, fp16 state, ggml Q8_0
  weights: the large sharded configuration, run on 1/2/4/8 GPUs.
* ``res4_c128`` - 364,846 voxels on a 256^3 grid, 4 GroupNorm(32) residual
  blocks (conv -> GroupNorm -> SiLU -> conv -> +skip), C = 128, fp16, Q8_0.
* ``topo_4m`` - topology only: hash build + 27-tap neighbour map + stride-2
  maps over the union of 8 seeded surfaces (4,026,477 voxels) on a 1024^3
  grid.
* ``conv_c64`` - one submanifold conv, C = 64, fp32 features and weights,
  77,507 voxels on a 128^3 grid.
* ``unet_c64`` - one encoder-decoder level, batch 2 (two surfaces):
  conv 64 -> pool + linear 64->128 -> conv 128 -> linear + nearest up + skip,
  bf16 activations, fp32 weights.
* ``refine_640x480`` - one whole refiner pass (SparseRefiner::refine_once):
  a five-level refiner (channels 64/64/128/128/128, F16 weights as the
  converter stores refiner tensors) on a 640 x 480 point map; two point maps
  alternate so that every pass rebuilds its topology, as the refine loop's
  passes do when log z moves.

One step = rebuild the topology (as the refiner does on every refine pass)
and run the workload's operators.  ``value`` is active voxels x sparse convs
per second (topo_4m: voxels per second) with the inputs resident in HBM;
``e2e`` the same through the C ABI with pinned host buffers, the step's
inputs copied in and its result copied out inside the timed region.

Multi-GPU (torchrun, one process per GPU; stack workloads): the voxels are
split into z-slabs whose owned + halo rows are balanced across the ranks
(mogecpp_b200/slab.py); each rank builds the topology of its slab plus a
two-plane halo per side and refreshes the halo once per block: by default
conv2's epilogue stores the boundary planes straight into the neighbours'
halo rows over CUDA IPC peer memory (``--exchange nccl``: NCCL send/recv
before every block).
Total work is fixed ("scaling": "strong"); timing is the max over ranks.
After the timed region the owned rows are gathered on rank 0 and compared
with the single-GPU stack over the whole set (``parity``).

``--impl reference`` times the reference's own CPU implementation (mogecpp
src/sparse.cpp + ggml CPU backend, compiled from the reference sources into
oracle/_ref/) on the same workload: the whole set where it finishes in
seconds, else a z-slab sample of it (the first voxels in (b, z, y, x) order).
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

METRIC = "active voxels/s per sparse conv"
GN_EPS = 1e-5
BLOCK_NAME = {"ln": "LayerNorm res_block", "gn": "GroupNorm(32) res block"}
# kind: "stack" (residual blocks), "topo" (topology only), "conv" (one conv),
# "unet" (one encoder-decoder level)
WORKLOADS = {
    "shell_4m": dict(kind="stack", blocks=8, coords="shell_4m_coords", grid=1024, block="ln", c=128),
    "res4_c128": dict(kind="stack", blocks=4, coords="res4_c128_coords", grid=256, block="gn", c=128),
    "topo_4m": dict(kind="topo", coords="topo_4m_coords", grid=1024),
    "conv_c64": dict(kind="conv", coords="conv_c64_coords", grid=128, c=64),
    "unet_c64": dict(kind="unet", coords="unet_coords", grid=256),
    # the same U-level with the octant-weighted stride-2 conv and its
    # transpose in place of pool + linear and linear + nearest up (an
    # extension: the reference has neither, so its arm is unavailable and the
    # CPU baseline is the oracle on a z-slab sample)
    "unet_octant_c64": dict(kind="unet", coords="unet_coords", grid=256, octant=True),
    "refine_640x480": dict(kind="refine", width=640, height=480, grid=None),
}
# DRAM bytes per voxel of one sparse-conv launch, by workload and residual-
# block kind: dram__bytes_read.sum + dram__bytes_write.sum from ncu captures
# of a block's two convs on that workload (profiles/conv_traffic_*.md),
# averaged; scaled by the voxels a launch processes.  shell_4m's gathers miss
# L2 more than res4_c128's (its tap-ordered tiles spread over a 450 MB
# operand), so each workload uses its own capture.
CONV_DRAM_BYTES_PER_VOXEL = {("shell_4m", "ln"): 1302.0, ("res4_c128", "gn"): 860.0, ("res4_c128", "ln"): 646.0}
# Compulsory bytes per voxel of one Q8_0 conv launch at C = 128 (each input
# row read once): activation codes + block scales (128 + 16), the plan's
# tile row and neighbour list (4 + 108), the output (fused Q8_0 codes + scales
# 144, fp16 256 or fp32 512) and, for the second conv, the fp16 residual (256).
CONV_ALG_BYTES_PER_VOXEL = {"ln": ((144 + 112 + 144) + (144 + 112 + 256 + 256)) / 2.0,
                            "gn": ((144 + 112 + 512) + (144 + 112 + 256 + 256)) / 2.0}
Q8_WEIGHT_BYTES = 27 * 128 * 128 + 27 * 4 * 128 * 4   # int8 codes + fp32 block scales per conv
# cub::DeviceRadixSort on sm_100 (its Policy1000 tuning, 4-byte keys and
# values): up to 256 x 19 items sort in one single-tile kernel; above that, a
# histogram kernel, an exclusive-sum kernel and one onesweep kernel per 8-bit
# digit
CUB_SINGLE_TILE_ITEMS = 256 * 19
PLAN_TILE_ROWS = 128


def radix_sort_kernels(items, bits):
    if items <= 0:
        return 0
    return 1 if items <= CUB_SINGLE_TILE_ITEMS else 2 + (bits + 7) // 8


def plan_kernels(n):
    """Kernels of one conv plan build over n output rows: header, mask keys,
    the row sort (27-bit keys), tile lists, the tile schedule sort (8-bit
    costs); the header alone for an empty level."""
    if n <= 0:
        return 1
    tiles = (n + PLAN_TILE_ROWS - 1) // PLAN_TILE_ROWS
    return 1 + 1 + radix_sort_kernels(n, 27) + 1 + radix_sort_kernels(tiles, 8)
# kernels per topology call: the voxel table (table clear, brick insert,
# record clear, record fill), the neighbour map (brick kernel + the three
# per-voxel fallback kernels, which return at once unless the bricks
# overflow), the stride-2 maps (brick first-child scan, block scan, pool
# fill, brick assign + six fallback kernels); make_level_downsample's
# neighbour kernel does the first-child scan, so it launches one fewer
TOPO_KERNELS = {"make_level": 8, "downsample": 14, "make_level_downsample": 17}


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p["hbm_gbs"]), "measured"
    except Exception:
        return 1590.0, 6650.0, "fallback"


def measure_int8_peak(dev):
    """Dense int8 tensor-core throughput of this GPU (cuBLAS int8 GEMM via
    torch._int_mm, 8192^3, best of 10 CUDA-event timings), TOP/s."""
    import torch
    m = 8192
    a = torch.randint(-100, 100, (m, m), dtype=torch.int8, device=dev)
    b = torch.randint(-100, 100, (m, m), dtype=torch.int8, device=dev).t().contiguous().t()
    for _ in range(3):
        torch._int_mm(a, b)
    best = float("inf")
    for _ in range(10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._int_mm(a, b)
        e1.record()
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1))
    del a, b
    return 2.0 * m ** 3 / (best * 1e-3) / 1e12


def block_params(nblocks, c):
    from mogecpp_b200 import synth
    blocks = []
    for b in range(nblocks):
        rng = np.random.default_rng(1000 + b)
        blk = dict(norm_w=(1 + 0.1 * rng.standard_normal(c)).astype(np.float32),
                   norm_b=(0.1 * rng.standard_normal(c)).astype(np.float32),
                   w1=synth.conv_weight(2000 + 2 * b, c, c),
                   b1=(0.05 * rng.standard_normal(c)).astype(np.float32),
                   w2=synth.conv_weight(2001 + 2 * b, c, c),
                   b2=(0.05 * rng.standard_normal(c)).astype(np.float32))
        blk["gn_w"], blk["gn_b"] = blk["norm_w"], blk["norm_b"]  # the one affine serves either norm
        blocks.append(blk)
    return blocks


def unet_params():
    from mogecpp_b200 import synth
    lin = lambda seed, co, ci: (np.random.default_rng(seed).standard_normal((co, ci)) / np.sqrt(ci)).astype(np.float32)
    return dict(w0=synth.conv_weight(3000, 64, 64), wl=lin(3001, 128, 64), w1=synth.conv_weight(3002, 128, 128),
                wu=lin(3003, 64, 128), b0=np.zeros(64, np.float32), bl=np.zeros(128, np.float32),
                b1=np.zeros(128, np.float32), bu=np.zeros(64, np.float32),
                wd8=lin(3004, 128, 8 * 64), wu8=lin(3005, 64, 8 * 128))   # octant weights [cout][8*cin]


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


# ------------------------------------------------------------------ CPU arms

def open_reference(threads):
    """The reference CPU build (oracle/_ref) or, where it was not built, the
    oracle port; topology threads = min(cores, 64), the reference's cap."""
    from oracle.oracle import Oracle, Reference
    os.environ["MOGE_SPARSE_TOPOLOGY_THREADS"] = str(max(1, min(threads, 64)))
    try:
        return Reference(n_threads=threads), "reference", threads
    except FileNotFoundError:
        return Oracle(), "port", 1


def cpu_stack_step(R, kind, coords, x, blocks, block_kind):
    """One CPU step of a residual stack, timed like the GPU step: make_level
    then the blocks.  Returns (seconds, output)."""
    from oracle.oracle import W_Q8_0
    t0 = time.perf_counter()
    nbr = R.make_level(coords)
    t_topo = time.perf_counter() - t0
    if block_kind == "ln" and kind == "reference":
        y, sec = R.res_stack(x, nbr, blocks, W_Q8_0, iters=1)
        return t_topo + sec, y, nbr
    t0 = time.perf_counter()
    h = x
    sample = np.zeros(x.shape[0], np.int32)
    for b in blocks:
        if block_kind == "ln":
            h = R.res_block(h, nbr, b, W_Q8_0)
        elif kind == "reference":
            h = R.res_block_gn(h, nbr, b, W_Q8_0, 32, GN_EPS)
        else:
            h = R.res_block_gn(h, nbr, sample, b, W_Q8_0, 32, GN_EPS)
    return t_topo + time.perf_counter() - t0, h, nbr


def stack_sample(coords, x0, blocks, block_kind, R, kind, target_s):
    """Times the CPU stack on the first voxels of the (b, z, y, x)-ordered set
    (a z-slab), sized to about target_s per run; returns (voxels, seconds)."""
    ns = min(coords.shape[0], 4096)
    sec = 0.0
    for _ in range(4):
        sec, _, _ = cpu_stack_step(R, kind, coords[:ns], x0[:ns].astype(np.float32), blocks, block_kind)
        if sec >= 0.5 * target_s or ns == coords.shape[0]:
            break
        ns = int(min(coords.shape[0], ns * max(2.0, target_s / max(sec, 1e-3))))
    return ns, sec


def cpu_octant_baseline(coords, extra, ns=12000):
    """The octant U-level on the oracle (single-threaded C), on the first ns
    voxels of the set (a z-slab of the first sample): the reference has no
    such operator, so this CPU restatement is the baseline."""
    from oracle.oracle import Oracle, W_F32
    q = Oracle()
    c = np.ascontiguousarray(coords[:ns])
    x = extra["x"][:ns]
    p = extra["p"]
    t0 = time.perf_counter()
    nbr = q.make_level(c)
    parent, pool, inv, up = q.downsample(c)
    down, upm = q.octant_maps(c, pool, up)
    pc = np.ascontiguousarray(parent)
    nbr_c = q.make_level(pc)
    h0 = q.sparse_conv(x, nbr, p["w0"], W_F32)
    h1 = q.conv_rect(h0, down, pc.shape[0], 8, p["wd8"], W_F32)
    h2 = q.sparse_conv(h1, nbr_c, p["w1"], W_F32)
    q.conv_rect(h2, upm, c.shape[0], 8, p["wu8"], W_F32)
    sec = time.perf_counter() - t0
    return {"value": (c.shape[0] + pc.shape[0]) / sec, "unit": "voxels/s", "cores": 1, "kind": "port",
            "sample": f"first {c.shape[0]} voxels of the set (a z-slab), the octant U-level step on the oracle"}


def cpu_other_step(R, w, coords, extra):
    """One CPU step of the topology, single-conv or U-level workloads on the
    whole set.  Returns seconds."""
    from oracle.oracle import W_F32
    t0 = time.perf_counter()
    if w["kind"] == "topo":
        a, b = R.topology_timed(coords, iters=1) if hasattr(R, "topology_timed") else (None, None)
        if a is None:
            R.make_level(coords)
            R.downsample(coords)
            return time.perf_counter() - t0
        return a + b
    if w["kind"] == "conv":
        nbr = R.make_level(coords)
        R.sparse_conv(extra["x"], nbr, extra["w"], W_F32, None)
        return time.perf_counter() - t0
    # U-level, one reference call per sample (the reference has no batch field)
    p = extra["p"]
    for b in np.unique(coords[:, 3]):
        sel = coords[:, 3] == b
        c = coords[sel].copy()
        c[:, 3] = 0
        x = extra["x"][sel]
        nbr = R.make_level(c)
        parent, pool, inv, up = R.downsample(c)
        pc = np.zeros((parent.shape[0], 4), np.int32)
        pc[:, :3] = parent[:, :3]
        nbr_c = R.make_level(pc)
        h0 = R.sparse_conv(x, nbr, p["w0"], W_F32, p["b0"])
        h1 = R.pool_down(h0, pool, inv, p["wl"], W_F32, p["bl"])
        h2 = R.sparse_conv(h1, nbr_c, p["w1"], W_F32, p["b1"])
        R.nearest_up(h2, up, p["wu"], W_F32, p["bu"])
    return time.perf_counter() - t0


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from mogecpp_b200 import synth
    w = WORKLOADS[args.workload]
    if w.get("octant"):
        print(json.dumps({"impl": "reference", "unavailable": "the reference has no octant-weighted stride-2 conv or "
                          "transposed conv (its stride-2 operators are pool + linear and linear + nearest up, "
                          "timed by --workload unet_c64)"}), flush=True)
        return
    coords = getattr(synth, w["coords"])() if "coords" in w else np.zeros((0, 4), np.int32)
    threads = os.cpu_count() or 1
    R, kind, cores = open_reference(threads)
    budget = 150.0 / max(1, args.steps + args.warmup)   # seconds per step so the run ends in minutes
    if w["kind"] == "refine":
        img, (fa, ea, ew, eh), (fb, eb, _, _) = refine_inputs(w)
        W_, H_ = w["width"], w["height"]
        if kind != "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the reference CPU build (oracle/_ref) is not built"}))
            return
        cfgs = synth.REFINER_5L
        runs = [0]

        def run():
            runs[0] += 1
            src = (fa, ea) if runs[0] % 2 else (fb, eb)
            return R.refine_once(img, src[0], W_, H_, src[1], ew, eh)[1]
        units = None
        sample = f"one refine_once pass, {W_}x{H_} point map, five-level refiner (F16 weights)"
        cfg_n = W_ * H_
    elif w["kind"] == "stack":
        blocks = block_params(w["blocks"], w["c"])
        x0 = synth.features_rows(2, np.arange(min(coords.shape[0], 1 << 18)), w["c"], np.float16)
        ns, _ = stack_sample(coords, x0, blocks, args.block, R, kind, min(8.0, budget))
        units = ns * 2 * len(blocks)
        run = lambda: cpu_stack_step(R, kind, coords[:ns], x0[:ns].astype(np.float32), blocks, args.block)[0]
        sample = (f"first {ns} voxels of {args.workload} in (b,z,y,x) order (a z-slab), make_level + "
                  f"{len(blocks)} x {BLOCK_NAME[args.block]}, Q8_0")
        cfg_n = ns
    else:
        extra = other_inputs(w, coords)
        run = lambda: cpu_other_step(R, w, coords, extra)
        units = other_units(w, coords, extra)
        sample = f"the whole {args.workload} set ({coords.shape[0]} voxels), {other_step_name(w)}"
        cfg_n = coords.shape[0]
    times = []
    for i in range(args.warmup + args.steps):
        sec = run()
        if i >= args.warmup:
            times.append(sec)
    t = sum(times) / len(times)
    if units is None:   # refine: voxel-convs of the pass, from the GPU-side level sizes when known
        units = refine_units_cpu(img, fa, W_, H_, cfgs)
    value = units / t
    unit = "voxels/s"
    line = {"impl": "reference", "metric": workload_metric(w), "value": value, "unit": unit, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": workload_ref_dtype(w), "data": "synthetic",
            "config": {"workload": args.workload, "voxels": int(cfg_n), "total_voxels": int(coords.shape[0]),
                       **({"channels": w["c"], "blocks": w["blocks"], "block": BLOCK_NAME[args.block]}
                          if w["kind"] == "stack" else {})},
            "cpu_baseline": {"value": value, "unit": unit, "cores": cores, "kind": kind, "sample": sample},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def refine_units_cpu(img, fc, width, height, cfg):
    """Voxel-convs of one refine pass: level sizes of the point map's pyramid
    (the reference's quantize_topology_z + stride-2 chain) times the convs per
    level."""
    from oracle.oracle import Oracle
    O = Oracle()
    z = O.quantize_topology_z(fc, 256.0)
    yy, xx = np.divmod(np.arange(width * height), width)
    c = np.stack([yy, xx, z, 0 * z], 1).astype(np.int32)
    L = len(cfg["model_channels"])
    sizes = [c.shape[0]]
    for _ in range(L - 1):
        c = O.downsample(c)[0]
        sizes.append(c.shape[0])
    convs = [2 * (cfg["encoder_blocks"][l] + (cfg["decoder_blocks"][L - 2 - l] if l < L - 1 else cfg["bottleneck_blocks"]))
             for l in range(L)]
    return sum(n * k for n, k in zip(sizes, convs))


def workload_metric(w):
    if w["kind"] == "topo":
        return "active voxels/s (hash build + 27-tap neighbour map + stride-2 maps)"
    return METRIC


def workload_ref_dtype(w):
    return {"stack": "q8_0 x fp32 (ggml CPU)", "topo": "int32 / int64 keys", "conv": "fp32 (ggml CPU)",
            "unet": "fp32 (ggml CPU)", "refine": "f16 weights x fp32 state (ggml CPU)"}[w["kind"]]


def other_step_name(w):
    return {"topo": "make_level + downsample", "conv": "make_level + 1 sparse conv (fp32, C=64)",
            "unet": "make_level x2 + downsample + conv 64 + pool/linear + conv 128 + linear/up"}[w["kind"]]


def other_inputs(w, coords):
    from mogecpp_b200 import synth
    n = coords.shape[0]
    if w["kind"] == "conv":
        return dict(x=synth.features(2, n, 64), w=synth.conv_weight(2100, 64, 64))
    if w["kind"] == "unet":
        x = synth.features(2, n, 64).astype(np.float32)
        import torch
        x = torch.from_numpy(x).to(torch.bfloat16).float().numpy()   # bf16 inputs
        return dict(x=x, p=unet_params())
    return {}


def other_units(w, coords, extra, n_coarse=None):
    n = coords.shape[0]
    if w["kind"] in ("topo", "conv"):
        return n
    if n_coarse is None:
        from mogecpp_b200.synth import pack_keys
        c = coords.copy()
        c[:, :3] >>= 1
        n_coarse = len(np.unique(pack_keys(c)))
    return n + n_coarse   # the two sparse convs of the level


# ------------------------------------------------------------------ GPU arm

def run_ours(args):
    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=torch.device("cuda", local))
    w = WORKLOADS[args.workload]
    if world > 1 and w["kind"] != "stack":
        raise SystemExit(f"--gpus > 1 runs the residual-stack workloads (z-slab halo); {args.workload} is 1-GPU")
    from mogecpp_b200 import slab, synth
    from mogecpp_b200.sparse import SparseCudaExecutor

    ex = SparseCudaExecutor(local)
    dev = torch.device("cuda", local)
    coords = getattr(synth, w["coords"])() if "coords" in w else np.zeros((w["width"] * w["height"], 4), np.int32)
    if args.voxels and "coords" in w:
        coords = np.ascontiguousarray(coords[:args.voxels])   # a z-slab: (b, z, y, x) order
    n = coords.shape[0]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    W = build_workload(args, w, ex, dev, coords, rank, world)
    step = W["step"]

    barrier()
    for _ in range(args.warmup):
        W["reset"]()
        step()
    ex.check()
    W["after_warmup"]()
    barrier()

    # ---- device-resident timed region
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    torch.cuda.synchronize()
    barrier()
    ex.profile(True)
    W["halo_events"].clear()
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            W["reset"]()
            flush.fill_(i & 0xff)  # L2 flush between steps (outside the events)
            barrier()
            ev[i][0].record()
            step()
            ev[i][1].record()
        torch.cuda.synchronize()
    ex.profile(False)
    prof = ex.profile_read()
    if W["halo_events"]:
        prof["halo"] = (len(W["halo_events"]), sum(a.elapsed_time(b) for a, b in W["halo_events"]))
    ex.check()
    step_ms = [a.elapsed_time(b) for a, b in ev]
    t_ms = sum(step_ms) / len(step_ms)
    if world > 1:
        t = torch.tensor([t_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_ms = float(t.item())
        barrier()
    value = W["units"] / (t_ms * 1e-3)

    # ---- end to end through the C ABI with host buffers: a stream of steps,
    # each with the host->device copy of its inputs (pinned) and the
    # device->host copy of its result.  Inputs are double-buffered on the
    # device and the copies run on their own streams, so step i+1's input copy
    # and step i's result copy overlap step i's compute, as a serving loop
    # would run them.  Timed from the first input copy to the last result
    # copy of the K steps (pipeline fill and drain included).
    e2e_t = e2e_run(W, args, flush, barrier)
    ex.check()
    if world > 1:
        t = torch.tensor([e2e_t], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_t = float(t.item())

    parity = W["parity"]() if world > 1 else None
    if world > 1:
        barrier()

    if rank == 0:
        line = {
            "metric": workload_metric(w), "value": value, "unit": "voxels/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t_ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": W["dtype"], "data": "synthetic",
            "config": {"workload": args.workload, "voxels": n, "grid": w.get("grid"), **W["config"],
                       "l2": "flushed between steps (256 MiB write)"},
            "e2e": {"value": W["units"] / (e2e_t * 1e-3), "unit": "voxels/s",
                    "h2d_bytes_per_step": W["h2d_bytes"], "d2h_bytes_per_step": W["d2h_bytes"], "ms_per_step": e2e_t,
                    "copies": ("one msc_level_stack_host call per step (C ABI, pinned host buffers in and out; "
                               "the library copies on two copy streams ordered against the compute stream by "
                               "events, two workspaces in flight)") if W.get("e2e_host_step") else
                              ("pinned host buffers; step i+1's input copy and step i's result copy overlap "
                               "step i's compute (two copy streams, double-buffered device inputs)")},
            "roofline": W["roofline"](prof),
            "kernel_ms_per_step": {k: v[1] / args.steps for k, v in prof.items()},
            "gpu_launches": int(W["launches"](prof)),
            "clocks": clk.summary(),
        }
        if W.get("tflops"):
            line["effective_tflops_per_conv"] = W["tflops"](prof)
        if parity is not None:
            line["parity"] = parity
        if world == 1 and not args.no_cpu_baseline:
            line.update(W["cpu_baseline"]())
        print(json.dumps(line), flush=True)
    if world > 1:
        barrier()
        dist.destroy_process_group()


def e2e_run(W, args, flush, barrier):
    import torch
    h_in, d_bufs, out_dev, h_out = W["e2e_buffers"]()
    h_ins = h_in if W.get("alternate_inputs") else [h_in]
    comp = torch.cuda.current_stream()
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    if W.get("e2e_host_step"):
        return e2e_run_host(W, args, flush, barrier, h_ins[0], h_out, comp, s_in, s_out)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_comp = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def once(k):
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

        def copy_in(i):
            bi = i % 2
            if i >= 2:
                s_in.wait_event(ev_out[bi])  # step i-2's result copy has read this buffer
            with torch.cuda.stream(s_in):
                if i == 0:
                    t0.record(s_in)
                for d, h in zip(d_bufs[bi], h_ins[i % len(h_ins)]):
                    d.copy_(h, non_blocking=True)
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
            W["step"](*d_bufs[bi])
            ev_comp[bi].record(comp)
            s_out.wait_event(ev_comp[bi])
            with torch.cuda.stream(s_out):
                h_out[bi].copy_(out_dev(bi), non_blocking=True)
                ev_out[bi].record(s_out)
                if i == k - 1:
                    t1.record(s_out)
        torch.cuda.synchronize()
        return t0.elapsed_time(t1) / k

    once(args.warmup)
    return once(args.steps)


def e2e_run_host(W, args, flush, barrier, h_in, h_out, comp, s_in, s_out):
    """End to end through a host-buffer C-ABI call per step (the library
    copies the inputs in and the result out on the copy streams, ordered
    against the compute stream by events); two workspaces in flight, so
    step i+1's input copy and step i's result copy overlap compute."""
    import torch
    h_coords, h_x = h_in

    def once(k):
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        barrier()
        t0.record(s_in)
        for i in range(k):
            with torch.cuda.stream(comp):
                flush.fill_(i & 0xff)  # L2 flush between steps
            W["e2e_host_step"](i, h_coords, h_x, h_out[i % 2], comp, s_in, s_out)
        t1.record(s_out)
        torch.cuda.synchronize()
        return t0.elapsed_time(t1) / k

    once(args.warmup)
    return once(args.steps)


def build_workload(args, w, ex, dev, coords, rank, world):
    if w["kind"] == "stack":
        return build_stack(args, w, ex, dev, coords, rank, world)
    if w["kind"] == "refine":
        return build_refine(args, w, ex, dev)
    return build_other(args, w, ex, dev, coords)


def refine_inputs(w):
    from mogecpp_b200 import synth
    cfg = synth.REFINER_5L
    a = synth.refiner_inputs(40, w["width"], w["height"], 16, cfg["encoder_channels"])
    b = synth.refiner_inputs(41, w["width"], w["height"], 16, cfg["encoder_channels"])
    return synth.refiner_mogg(42, cfg, "f16"), a, b


def build_refine(args, w, ex, dev):
    import torch
    from mogecpp_b200.sparse import SparseRefiner
    img, (fa, ea, ew, eh), (fb, eb, _, _) = refine_inputs(w)
    R = SparseRefiner(ex, img)
    W, H = w["width"], w["height"]
    inputs = [(torch.from_numpy(fa).to(dev), torch.from_numpy(ea).to(dev)),
              (torch.from_numpy(fb).to(dev), torch.from_numpy(eb).to(dev))]
    fc_d, enc_d = torch.empty_like(inputs[0][0]), torch.empty_like(inputs[0][1])
    state = {"i": 0}
    cfg = R.config
    L = cfg.num_levels
    convs = [2 * (cfg.encoder_blocks[l] + (cfg.decoder_blocks[L - 2 - l] if l < L - 1 else cfg.bottleneck_blocks))
             for l in range(L)]

    def reset():
        src = inputs[state["i"] % 2]
        state["i"] += 1
        fc_d.copy_(src[0])
        enc_d.copy_(src[1])

    def step(fc_t=fc_d, enc_t=enc_d):
        R.refine_once(fc_t, W, H, enc_t, ew, eh)

    reset()
    step()
    sizes = R.level_sizes()
    units = sum(n * k for n, k in zip(sizes, convs))

    def e2e_buffers():
        h_in = (torch.from_numpy(fa).pin_memory(), torch.from_numpy(ea).pin_memory())
        h_alt = (torch.from_numpy(fb).pin_memory(), torch.from_numpy(eb).pin_memory())
        bufs = [(torch.empty_like(fc_d), torch.empty_like(enc_d)), (torch.empty_like(fc_d), torch.empty_like(enc_d))]
        h_out = [torch.empty_like(h_in[0]).pin_memory() for _ in range(2)]
        # the two point maps alternate so that every pass rebuilds its topology
        return [h_in, h_alt], bufs, (lambda bi: bufs[bi][0]), h_out

    def roofline(prof):
        peak_tf, peak_hbm, peak_src = load_peaks()
        launches, ms = prof.get("conv_tc", (0, 0.0))
        # F16 weights: activations rounded to fp16, one kind::f16 MMA per product
        flops = sum(2.0 * cfg.model_channels[l] ** 2 * 27 * sizes[l] * convs[l] for l in range(L))
        t = ms * 1e-3 / max(args.steps, 1)
        ach = flops / t / 1e12 if launches else None
        return {"bound": "tensor", "achieved": ach, "peak": peak_tf, "unit": "TFLOP/s",
                "frac": ach / peak_tf if ach else None, "traffic": None,
                "kernel": "conv_tc (F16 weights, kind::f16), all convs of a pass",
                "peak_source": f"{peak_src} bf16 peak",
                "flops_note": "dense-equivalent 2*C*C*27*N per conv (the tap-skipping kernel does less)"}

    def launches(prof):
        # one plan per level and pass: the mean kernel count over the levels
        per = {**TOPO_KERNELS, "plan_build": sum(plan_kernels(s) for s in sizes) / max(len(sizes), 1)}
        # + per pass: z quantisation (3), level-0 map, input rows, input_proj,
        # encoder rows, fuse_proj.0, SiLU, out_proj, log z update, key compare
        return round(sum(per.get(k, 1) * v[0] for k, v in prof.items())) + 12 * args.steps

    def cpu_baseline():
        threads = os.cpu_count() or 1
        Rr, kind, cores = open_reference(threads)
        if kind != "reference":
            return {"cpu_baseline": None}
        Rr.refine_once(img, fa, W, H, ea, ew, eh)
        _, sec = Rr.refine_once(img, fb, W, H, eb, ew, eh)
        return {"cpu_baseline": {"value": units / sec, "unit": "voxels/s", "cores": cores, "kind": kind,
                                 "sample": f"one refine_once pass of the same model on the same {W}x{H} point map"}}

    return dict(step=step, reset=reset, after_warmup=lambda: None, e2e_buffers=e2e_buffers, roofline=roofline,
                tflops=None, launches=launches, parity=lambda: None, cpu_baseline=cpu_baseline, halo_events=[],
                units=units, h2d_bytes=int(fa.nbytes + ea.nbytes), d2h_bytes=int(fa.nbytes),
                dtype="fp32 state, F16 weights (activations rounded to fp16 as ggml does)",
                config={"pixels": W * H, "levels": sizes, "channels": list(cfg.model_channels[:L]),
                        "convs_per_level": convs, "weights": "f16",
                        "step": "refine_once: quantise log z + topology rebuild + U-Net + log z update"},
                alternate_inputs=True)


def build_stack(args, w, ex, dev, coords, rank, world):
    import torch
    import torch.distributed as dist
    from mogecpp_b200 import slab, synth
    c = w["c"]
    n = coords.shape[0]
    part = slab.partition(coords, world)[rank]
    rows = part.local_rows()
    lx0 = synth.features_rows(2, rows, c, np.float16)
    blocks_np = block_params(w["blocks"], c)
    convs = 2 * len(blocks_np)
    lcoords = np.ascontiguousarray(coords[rows])
    nl = lcoords.shape[0]
    coords_d = torch.from_numpy(lcoords).to(dev)
    x0_d = torch.from_numpy(lx0).to(dev)
    x_d = torch.empty_like(x0_d)
    halo = slab.SlabExchange(part, world)
    halo_events = []

    def dev_block(b):
        q = lambda k: ex.prepare_weight(torch.from_numpy(synth.quantize_q8_0(b[k])).to(dev), "q8_0", c, c, 27)
        return dict(norm_w=torch.from_numpy(b["norm_w"]).to(dev), norm_b=torch.from_numpy(b["norm_b"]).to(dev),
                    gn_w=torch.from_numpy(b["gn_w"]).to(dev), gn_b=torch.from_numpy(b["gn_b"]).to(dev),
                    b1=torch.from_numpy(b["b1"]).to(dev), b2=torch.from_numpy(b["b2"]).to(dev), w1=q("w1"), w2=q("w2"))

    blocks = [dev_block(b) for b in blocks_np]
    plan_kind = "tap_order" if args.conv == "ordered" else None
    gn_allreduce = (lambda t: dist.all_reduce(t)) if world > 1 else None

    def exchange(x_t):
        if world == 1:
            return
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        halo.exchange(x_t)
        b.record()
        halo_events.append((a, b))

    def run_stack(coords_t, x_t, n_stat, single=False):
        nbr = ex.make_level(coords_t)
        plan = ex.conv_plan(coords_t, nbr, plan_kind) if plan_kind else None
        if args.block == "ln" and (single or world == 1):
            ex.res_stack(x_t, nbr, blocks, plan=plan)   # the level's block loop in one call
            return nbr
        for blk in blocks:
            if not single:
                exchange(x_t)
            if args.block == "gn":
                ex.res_block_gn(x_t, nbr, coords_t, 1, blk, eps=GN_EPS, plan=plan, n_stat=n_stat,
                                allreduce=gn_allreduce)
            else:
                ex.res_block(x_t, nbr, blk, plan=plan)
        return nbr

    state = {}
    # multi-GPU LayerNorm stacks: the exchange fused into each block's second
    # conv (peer stores over NVLink); GroupNorm stacks keep the NCCL exchange
    # (their statistics need an all-reduce per block anyway)
    peer = world > 1 and args.block == "ln" and args.exchange == "peer"
    pslab = slab.PeerSlab(ex, part, world, c) if peer else None
    if peer:
        state["nbr"] = ex.make_level(coords_d)

    def step(coords_t=coords_d, x_t=x_d, out_t=None):
        if peer:
            pslab.set_level(coords_t)
            pslab.put_features(x_t)
            for blk in blocks:
                pslab.res_block(blk)
            if out_t is not None:
                pslab.get_features(out_t)   # on the compute stream: the next step reuses the buffer
            return
        state["nbr"] = run_stack(coords_t, x_t, part.n_owned)

    def reset():
        x_d.copy_(x0_d)

    def after_warmup():
        state["e_pairs"] = int((state["nbr"] < nl).sum().item())

    def e2e_buffers():
        h_coords = torch.from_numpy(lcoords).pin_memory()
        h_x = torch.from_numpy(lx0).pin_memory()
        h_out = [torch.empty((part.n_owned, c), dtype=x0_d.dtype).pin_memory() for _ in range(2)]
        bufs = [(coords_d, x_d), (torch.empty_like(coords_d), torch.empty_like(x_d))]
        if peer:
            outs = [torch.empty((part.n_owned, c), dtype=x0_d.dtype, device=dev) for _ in range(2)]
            bufs = [b + (o,) for b, o in zip(bufs, outs)]
            return (h_coords, h_x), bufs, (lambda bi: outs[bi]), h_out
        return (h_coords, h_x), bufs, (lambda bi: bufs[bi][1][:part.n_owned]), h_out

    int8_peak = {}

    def roofline(prof):
        peak_tf, peak_hbm, peak_src = load_peaks()
        if "tops" not in int8_peak:
            int8_peak["tops"] = measure_int8_peak(dev)
        i8 = int8_peak["tops"]
        launches, ms = prof.get("conv_tc", (0, 0.0))
        t = ms / max(launches, 1) * 1e-3
        flops = 2.0 * c * c * state["e_pairs"]
        alg = CONV_ALG_BYTES_PER_VOXEL[args.block] * nl + Q8_WEIGHT_BYTES
        t_tensor, t_hbm = flops / (i8 * 1e12), alg / (peak_hbm * 1e9)
        bound = "hbm" if t_hbm >= t_tensor else "tensor"
        if bound == "hbm":
            achieved, peak, unit = (alg / t / 1e9 if launches else None), peak_hbm, "GB/s"
        else:
            achieved, peak, unit = (flops / t / 1e12 if launches else None), i8, "TOP/s"
        return {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
                "frac": (achieved / peak) if achieved else None,
                "traffic": (CONV_DRAM_BYTES_PER_VOXEL[(args.workload, args.block)] * nl
                            if (args.workload, args.block) in CONV_DRAM_BYTES_PER_VOXEL else None),
                "traffic_unit": "DRAM bytes per conv launch (ncu capture on this workload, per voxel, "
                                "scaled by the launch's voxels)",
                "kernel": "conv_tc (Q8_0 x Q8_0, kind::i8, C=128)",
                "peak_source": f"{peak_src} HBM copy bandwidth; int8 peak measured in this run (cuBLAS int8 GEMM)",
                "algorithmic_bytes_per_launch": alg, "flops_per_launch": flops,
                "int8_peak_tops": i8, "bf16_peak_tflops": peak_tf,
                "t_bound_ms": max(t_tensor, t_hbm) * 1e3, "avg_launch_ms": t * 1e3,
                "tensor_frac_int8": (flops / t / 1e12 / i8) if launches else None}

    def tflops(prof):
        launches, ms = prof.get("conv_tc", (0, 0.0))
        return 2.0 * c * c * state["e_pairs"] / (ms / max(launches, 1) * 1e-3) / 1e12 if launches else None

    def launches(prof):
        # kernels per profiled family call: topology as TOPO_KERNELS;
        # plan_build over the rank's local rows (plan_kernels);
        # gn_stats/finalize/act_prepare/conv_tc = 1
        per = {**TOPO_KERNELS, "plan_build": plan_kernels(nl), "halo": 0,
               "halo_wait": 2 if peer else 1}  # wait + signal kernels per block
        return sum(per.get(k, 1) * v[0] for k, v in prof.items())

    def parity():
        """Owned rows of every rank after one step, gathered on rank 0 and
        compared with the single-GPU stack over the whole set."""
        reset()
        step()
        owned = torch.empty((part.n_owned, c), dtype=torch.float16, device=dev)
        if peer:
            pslab.get_features(owned)
        else:
            owned.copy_(x_d[:part.n_owned])
        torch.cuda.synchronize()
        parts = slab.partition(coords, world)
        res = None
        if rank == 0:
            full = torch.empty((n, c), dtype=torch.float16, device=dev)
            full[part.lo:part.hi] = owned
            for r in range(1, world):
                p = parts[r]
                buf = torch.empty((p.n_owned, c), dtype=torch.float16, device=dev)
                dist.recv(buf, src=r)
                full[p.lo:p.hi] = buf
            cf = torch.from_numpy(coords).to(dev)
            xf = torch.from_numpy(synth.features_rows(2, np.arange(n), c, np.float16)).to(dev)
            run_stack(cf, xf, n, single=True) if args.block == "ln" else run_stack_single_gn(cf, xf)
            torch.cuda.synchronize()
            d = (full.float() - xf.float())
            res = {"reference": "single-GPU stack over all voxels (same kernels)",
                   "max_abs": float(d.abs().max().item()),
                   "rel_l2": float(d.norm().item() / max(xf.float().norm().item(), 1e-30)),
                   "bit_exact": bool(torch.equal(full, xf)), "rows": int(n)}
            del full, xf, cf
        else:
            dist.send(owned, dst=0)
        return res

    def run_stack_single_gn(cf, xf):
        nbr = ex.make_level(cf)
        plan = ex.conv_plan(cf, nbr, plan_kind) if plan_kind else None
        for blk in blocks:
            ex.res_block_gn(xf, nbr, cf, 1, blk, eps=GN_EPS, plan=plan)

    def cpu_baseline():
        return stack_cpu_baseline(args, w, ex, dev, coords, blocks, blocks_np, convs)

    host_step = None
    if world == 1 and args.block == "ln" and plan_kind:
        # one GPU, LayerNorm blocks: the end-to-end run goes through the C ABI
        # with host buffers (msc_level_stack_host: copies in, make_level,
        # plan, blocks, copy out), two workspaces in flight
        wsb = ex.level_stack_host_workspace(nl, c)
        host_ws = [torch.empty(wsb, dtype=torch.uint8, device=dev) for _ in range(2)]

        def host_step(i, h_coords, h_x, h_y, comp, s_in, s_out):
            ex.level_stack_host(h_coords, h_x, blocks, h_y, ws=host_ws[i % 2], stream=comp, copy_in=s_in,
                                copy_out=s_out)

    return dict(step=step, reset=reset, after_warmup=after_warmup, e2e_buffers=e2e_buffers, roofline=roofline,
                tflops=tflops, launches=launches, parity=parity, cpu_baseline=cpu_baseline,
                halo_events=halo_events, units=n * convs, e2e_host_step=host_step,
                h2d_bytes=int(lcoords.nbytes + lx0.nbytes), d2h_bytes=int(part.n_owned * c * lx0.itemsize),
                dtype="q8_0 (int8 codes exact on tcgen05, per-32-block fp32 scaling as ggml)",
                config={"channels": c, "blocks": len(blocks_np), "convs_per_step": convs,
                        "rank0_local_voxels": nl, "block": BLOCK_NAME[args.block],
                        "step": (f"make_level + {plan_kind} plan + " if plan_kind else "make_level + ") +
                                f"{len(blocks_np)} res blocks" + (" (halo exchange before each)" if world > 1 else "") +
                                (", GroupNorm statistics all-reduced" if world > 1 and args.block == "gn" else ""),
                        "conv": args.conv,
                        "parallelism": (f"z-slabs x{world}, 2-plane halo written by each block's second conv into "
                                        f"the neighbours' buffers (peer stores over NVLink)" if peer else
                                        f"z-slabs x{world}, 2-plane halo over NCCL") if world > 1 else "single GPU"})


def stack_cpu_baseline(args, w, ex, dev, coords, blocks, blocks_np, convs):
    """The reference CPU stack on z-slab samples of two sizes (the per-voxel
    rate should not depend on the size: the reference gathers all 27 rows of
    every voxel), timed like the GPU step (make_level + blocks); and, on the
    larger sample, our GPU blocks compared with the reference block by block
    on identical inputs."""
    import torch
    from mogecpp_b200 import synth
    threads = os.cpu_count() or 1
    R, kind, cores = open_reference(threads)
    x0 = synth.features_rows(2, np.arange(min(coords.shape[0], 1 << 18)), w["c"], np.float16)
    ns, sec = stack_sample(coords, x0, blocks_np, args.block, R, kind, 6.0)
    ns2 = max(1024, ns // 2)
    sec2, _, _ = cpu_stack_step(R, kind, coords[:ns2], x0[:ns2].astype(np.float32), blocks_np, args.block)
    rate, rate2 = ns * convs / sec, ns2 * convs / sec2
    # per-block parity on the sample: our block vs the reference block, same input
    from oracle.oracle import W_Q8_0
    cs = torch.from_numpy(np.ascontiguousarray(coords[:ns])).to(dev)
    nbr_d = ex.make_level(cs)
    nbr = nbr_d.cpu().numpy()
    x = torch.from_numpy(x0[:ns]).to(dev)
    per_block = []
    for b, bn in zip(blocks, blocks_np):
        xin = x.float().cpu().numpy()
        if args.block == "ln":
            ex.res_block(x, nbr_d, b)
            ref = R.res_stack(xin, nbr, [bn], W_Q8_0, iters=1)[0] if kind == "reference" else R.res_block(xin, nbr, bn, W_Q8_0)
        else:
            ex.res_block_gn(x, nbr_d, cs, 1, b, eps=GN_EPS)
            ref = (R.res_block_gn(xin, nbr, bn, W_Q8_0, 32, GN_EPS) if kind == "reference"
                   else R.res_block_gn(xin, nbr, np.zeros(ns, np.int32), bn, W_Q8_0, 32, GN_EPS))
        y = x.float().cpu().numpy()
        per_block.append({"rel_l2": float(np.linalg.norm(y - ref) / np.linalg.norm(ref)),
                          "max_abs": float(np.abs(y - ref).max())})
    ex.check()
    return {"cpu_baseline": {"value": rate, "unit": "voxels/s", "cores": cores, "kind": kind,
                             "sample": f"first {ns} voxels in (b,z,y,x) order (a z-slab), one run of make_level + "
                                       f"{len(blocks_np)} x {BLOCK_NAME[args.block]}",
                             "size_check": {"voxels": [ns, ns2], "voxels_per_s": [rate, rate2]}},
            "parity_vs_reference": {"rows": ns, "blocks": per_block,
                                    "tolerance": "per block on identical inputs: rel-L2 1e-3, max-abs 1e-2"}}


def build_other(args, w, ex, dev, coords):
    """topo_4m, conv_c64, unet_c64 (one GPU)."""
    import torch
    n = coords.shape[0]
    coords_d = torch.from_numpy(coords).to(dev)
    extra = other_inputs(w, coords)
    state = {}
    peak_tf, peak_hbm, peak_src = load_peaks()

    if w["kind"] == "topo":
        def step(coords_t=coords_d):
            state["nbr"], state["tr"] = ex.make_level_downsample(coords_t, sync=False)

        out_dev = lambda bi: state["nbr"]
        h_out_shape, h_out_dtype = (n, 27), torch.int32
        h_in = (torch.from_numpy(coords).pin_memory(),)
        bufs = [(coords_d,), (torch.empty_like(coords_d),)]
        units = n

        def roofline(prof):
            # compulsory bytes of one level's topology: read the coords once
            # (16 B rows), write the neighbour map (108 B per voxel), the
            # parents (16 B), pool_rows (8 x 4 B per parent), inv_count (4 B
            # per parent) and up_rows (4 B per voxel); tables and records are
            # scratch that an L2-resident design need not send to HBM
            np_ = int(state["tr"].np_dev.item())
            fam = "make_level_downsample"
            alg = 16 * n + 108 * n + 16 * np_ + 4 * (8 * np_ + np_) + 4 * n
            launches, ms = prof.get(fam, (0, 0.0))
            if not launches:
                return {"bound": "hbm", "achieved": None, "peak": peak_hbm, "unit": "GB/s", "frac": None,
                        "traffic": None}
            t = ms / launches * 1e-3
            ach = alg / t / 1e9
            return {"bound": "hbm", "achieved": ach, "peak": peak_hbm, "unit": "GB/s", "frac": ach / peak_hbm,
                    "traffic": None, "kernel": f"{fam} (brick table, neighbour map, stride-2 maps)",
                    "peak_source": peak_src, "algorithmic_bytes_per_launch": alg, "parents": np_,
                    "ms_per_launch": t * 1e3}

        dtype = "int32 coords, 64-bit packed keys"
        cfg = {"step": "make_level + downsample in one call (voxel table, 27-tap map, stride-2 maps)",
               "parents": None}
        launches_per = dict(TOPO_KERNELS)
    elif w["kind"] == "conv":
        pw = ex.prepare_weight(torch.from_numpy(extra["w"]).to(dev), "f32", 64, 64, 27)
        x_d = torch.from_numpy(extra["x"]).to(dev)

        def step(coords_t=coords_d, x_t=x_d):
            nbr = ex.make_level(coords_t)
            plan = ex.conv_plan(coords_t, nbr)
            state["nbr"] = nbr
            state["y"] = ex.sparse_conv(x_t, nbr, pw, None, plan=plan)

        out_dev = lambda bi: state["y"]
        h_out_shape, h_out_dtype = (n, 64), torch.float32
        h_in = (torch.from_numpy(coords).pin_memory(), torch.from_numpy(extra["x"]).pin_memory())
        bufs = [(coords_d, x_d), (torch.empty_like(coords_d), torch.empty_like(x_d))]
        units = n

        def roofline(prof):
            return conv_roofline(prof, "conv_tc", 64, 64, state, n, 4 + 4 + 112, 0, "fp32 (hi/lo fp16, kind::f16)",
                                 peak_tf, peak_hbm, peak_src, 3)

        dtype = "fp32 (exact hi/lo fp16 split on tcgen05 kind::f16, fp32 accumulation)"
        cfg = {"step": "make_level + tap-order plan + 1 sparse conv", "channels": 64}
        launches_per = {**TOPO_KERNELS, "plan_build": plan_kernels(n)}
    elif w.get("octant"):
        p = extra["p"]
        P = lambda k, ci, co, t: ex.prepare_weight(torch.from_numpy(p[k]).to(dev), "f32", ci, co, t)
        pw0, pwd, pw1, pwu = P("w0", 64, 64, 27), P("wd8", 64, 128, 8), P("w1", 128, 128, 27), P("wu8", 128, 64, 8)
        x_d = torch.from_numpy(extra["x"]).to(dev).to(torch.bfloat16)
        n_coarse = ex.downsample(coords_d).np

        def step(coords_t=coords_d, x_t=x_d):
            nbr, tr = ex.make_level_downsample(coords_t)
            nbr_c = ex.make_level(tr.parent.contiguous())
            down, up = ex.octant_maps(coords_t, tr)
            state["nbr"] = nbr
            h0 = ex.sparse_conv(x_t, nbr, pw0, None, out_dtype=torch.bfloat16)
            h1 = ex.octant_conv(h0, down, pwd, None, out_dtype=torch.bfloat16, plan=ex.conv_plan_rect(down, n))
            h2 = ex.sparse_conv(h1, nbr_c, pw1, None, out_dtype=torch.bfloat16)
            state["y"] = ex.octant_conv(h2, up, pwu, None, out_dtype=torch.bfloat16,
                                        plan=ex.conv_plan_rect(up, tr.np), skip=h0)

        out_dev = lambda bi: state["y"]
        h_out_shape, h_out_dtype = (n, 64), torch.bfloat16
        h_in = (torch.from_numpy(coords).pin_memory(), x_d.cpu().pin_memory())
        bufs = [(coords_d, x_d), (torch.empty_like(coords_d), torch.empty_like(x_d))]
        units = n + n_coarse   # the two submanifold convs; the octant convs are counted as stride-2 operators

        def roofline(prof):
            return conv_roofline(prof, "conv_tc", 64, 64, state, n, 4 + 4 + 112, 0, "bf16 (hi/lo fp16, kind::f16)",
                                 peak_tf, peak_hbm, peak_src, 3, bytes_x=4, bytes_y=2)

        dtype = "bf16 activations, fp32 weights (exact hi/lo fp16 split on tcgen05 kind::f16)"
        cfg = {"step": "make_level x2 + downsample + octant maps + conv 64 + octant strided conv 64->128 + conv 128 "
                       "+ octant transposed conv 128->64 + skip", "samples": 2, "coarse_voxels": int(n_coarse)}
        # two rectangular plans a step: the strided conv's (coarse rows) and
        # the transposed conv's (fine rows)
        launches_per = {**TOPO_KERNELS, "plan_build": (plan_kernels(n_coarse) + plan_kernels(n)) / 2,
                        "octant_maps": 2}
    else:  # unet
        p = extra["p"]
        P = lambda k, ci, co, t: ex.prepare_weight(torch.from_numpy(p[k]).to(dev), "f32", ci, co, t)
        pw0, pwl, pw1, pwu = P("w0", 64, 64, 27), P("wl", 64, 128, 1), P("w1", 128, 128, 27), P("wu", 128, 64, 1)
        x_d = torch.from_numpy(extra["x"]).to(dev).to(torch.bfloat16)
        tr0 = ex.downsample(coords_d)
        n_coarse = tr0.np

        def step(coords_t=coords_d, x_t=x_d):
            nbr, tr = ex.make_level_downsample(coords_t)
            nbr_c = ex.make_level(tr.parent.contiguous())
            state["nbr"] = nbr
            h0 = ex.sparse_conv(x_t, nbr, pw0, None, out_dtype=torch.bfloat16)
            h1 = ex.pool_down(h0, tr, pwl, None, out_dtype=torch.bfloat16)
            h2 = ex.sparse_conv(h1, nbr_c, pw1, None, out_dtype=torch.bfloat16)
            state["y"] = ex.nearest_up(h2, tr, pwu, None, skip=h0, out_dtype=torch.bfloat16)

        out_dev = lambda bi: state["y"]
        h_out_shape, h_out_dtype = (n, 64), torch.bfloat16
        h_in = (torch.from_numpy(coords).pin_memory(), x_d.cpu().pin_memory())
        bufs = [(coords_d, x_d), (torch.empty_like(coords_d), torch.empty_like(x_d))]
        units = n + n_coarse

        def roofline(prof):
            return conv_roofline(prof, "conv_tc", 64, 64, state, n, 4 + 4 + 112, 0, "bf16 (hi/lo fp16, kind::f16)",
                                 peak_tf, peak_hbm, peak_src, 3, bytes_x=4, bytes_y=2)

        dtype = "bf16 activations, fp32 weights (exact hi/lo fp16 split on tcgen05 kind::f16)"
        cfg = {"step": "make_level x2 + downsample + conv 64 + pool/linear 64->128 + conv 128 + linear/up + skip",
               "samples": 2, "coarse_voxels": int(n_coarse)}
        launches_per = dict(TOPO_KERNELS)

    def e2e_buffers():
        h_out = [torch.empty(h_out_shape, dtype=h_out_dtype).pin_memory() for _ in range(2)]
        return h_in, bufs, out_dev, h_out

    def launches(prof):
        return round(sum(launches_per.get(k, 1) * v[0] for k, v in prof.items()))

    def cpu_baseline():
        if w.get("octant"):
            return {"cpu_baseline": cpu_octant_baseline(coords, extra)}
        threads = os.cpu_count() or 1
        R, kind, cores = open_reference(threads)
        cpu_other_step(R, w, coords, extra)  # warm-up
        sec = cpu_other_step(R, w, coords, extra)
        u = other_units(w, coords, extra, units - n if w["kind"] == "unet" else None)
        return {"cpu_baseline": {"value": u / sec, "unit": "voxels/s", "cores": cores, "kind": kind,
                                 "sample": f"the whole set ({n} voxels), {other_step_name(w)}"}}

    def tflops(prof):
        if w["kind"] == "topo":
            return None
        launches_, ms = prof.get("conv_tc", (0, 0.0))
        e = int((state["nbr"] < n).sum().item())
        return 2.0 * 64 * 64 * e / (ms / max(launches_, 1) * 1e-3) / 1e12 if launches_ and w["kind"] == "conv" else None

    h2d = int(sum(t.numel() * t.element_size() for t in h_in))
    d2h = int(np.prod(h_out_shape) * torch.empty((), dtype=h_out_dtype).element_size())
    return dict(step=step, reset=lambda: None, after_warmup=lambda: None, e2e_buffers=e2e_buffers, roofline=roofline,
                tflops=tflops, launches=launches, parity=lambda: None, cpu_baseline=cpu_baseline, halo_events=[],
                units=units, h2d_bytes=h2d, d2h_bytes=d2h, dtype=dtype, config=cfg)


def conv_roofline(prof, fam, cin, cout, state, n, map_bytes, res_bytes, kind_name, peak_tf, peak_hbm, peak_src,
                  mma_per_kstep, bytes_x=4, bytes_y=4):
    """Roofline of a float-weight conv: useful flops 2*cin*cout*E against the
    bf16 peak divided by the MMAs issued per product (exact hi/lo split), or
    the compulsory bytes against HBM, whichever bounds."""
    launches, ms = prof.get(fam, (0, 0.0))
    if not launches:
        return {"bound": None, "achieved": None, "peak": None, "unit": None, "frac": None, "traffic": None}
    e = int((state["nbr"] < n).sum().item())
    t = ms / launches * 1e-3
    flops = 2.0 * cin * cout * e
    alg = n * (cin * bytes_x + cout * bytes_y + map_bytes + res_bytes) + 27 * cin * cout * 4
    eff_peak = peak_tf / mma_per_kstep
    t_tensor, t_hbm = flops / (eff_peak * 1e12), alg / (peak_hbm * 1e9)
    if t_hbm >= t_tensor:
        return {"bound": "hbm", "achieved": alg / t / 1e9, "peak": peak_hbm, "unit": "GB/s",
                "frac": alg / t / 1e9 / peak_hbm, "traffic": None, "kernel": f"{fam} ({kind_name})",
                "peak_source": peak_src, "algorithmic_bytes_per_launch": alg, "flops_per_launch": flops}
    return {"bound": "tensor", "achieved": flops / t / 1e12, "peak": eff_peak, "unit": "TFLOP/s",
            "frac": flops / t / 1e12 / eff_peak, "traffic": None, "kernel": f"{fam} ({kind_name})",
            "peak_source": f"{peak_src} bf16 peak / {mma_per_kstep} MMAs per product",
            "algorithmic_bytes_per_launch": alg, "flops_per_launch": flops}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="shell_4m", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--conv", default="ordered", choices=["ordered", "direct"])
    ap.add_argument("--exchange", default="peer", choices=["peer", "nccl"],
                    help="multi-GPU halo exchange: fused peer stores (default) or NCCL send/recv per block")
    ap.add_argument("--voxels", type=int, default=0,
                    help="run on the first N voxels of the workload (a z-slab), for small profiling captures")
    ap.add_argument("--block", default=None, choices=["ln", "gn"],
                    help="residual block (default: the one the workload is quoted on)")
    args = ap.parse_args()
    if args.block is None:
        args.block = WORKLOADS[args.workload].get("block", "ln")
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
