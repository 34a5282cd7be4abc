#!/usr/bin/env python
"""World-state reset benchmark: batched generation + full sky/block light +
RGBA8 -> float32 NCHW observation conversion, one batch of 128 worlds per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload per GPU (per step): 128 envs of 256 x 256 x 128 voxels (fBm terrain,
per-env seed = base_seed + env_id, 1000 surface torches per env), full
generation + light, and conversion of 128 RGBA8 160x90 frames to a
(128, 3, 90, 160) float32 tensor. Multi-GPU runs are weak-scaled: every rank
owns its own 128 envs (global env ids rank*128 ...), no data-path collective.

Prints one JSON line (rank 0). ``--impl reference`` times the reference's own
CPU implementation of the path (its CUDA CPU-fallback build, compiled from the
reference sources into oracle/_ref) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "voxels lit+generated/s"
UNIT = "voxels/s"
ENVS_PER_GPU = 128
W, H, D = 256, 128, 256
TORCHES = 1000
FRAME_H, FRAME_W = 90, 160
BASE_SEED = 1
# Bounded CPU sample: a quarter env (128 x 128 x 128) with 250 torches keeps the
# reference's torch density (1000 per 256 x 256 columns).
SAMPLE_W, SAMPLE_H, SAMPLE_D, SAMPLE_TORCHES = 128, 128, 128, 250
# Our kernel launches per step: place_torches, override count/scan(3)/scatter/sort,
# fBm surface with the column summaries, tile kernel, conversion.
LAUNCHES_PER_STEP = 10


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--envs", type=int, default=None,
                    help="envs per GPU (default: the workload's; smaller batches are for profiler captures)")
    ap.add_argument("--workload", choices=["reset", "relight", "daynight", "scaleout", "render"], default="reset",
                    help="reset (default): 128 worlds 256x256x128 regenerated + lit + frames converted per step; "
                         "relight: 1024 worlds 128^3, 10k edits per step + exact relight; daynight: 4096 worlds "
                         "128x128x96, sky sweep + 84x84 frame conversion per step; scaleout: 1024 worlds 256^3 per "
                         "GPU, 5000x1024/8192 edits per GPU per step + 90x160 frames, optional NCCL gather; "
                         "render: the reset worlds rendered to 160x90 RGBA8 frames and converted each step")
    ap.add_argument("--gather", action="store_true", help="scaleout: gather observations to rank 0 every step")
    ap.add_argument("--materialize", action="store_true",
                    help="daynight: also materialise the effective light of every cell each step")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


# ---------------------------------------------------------------- clocks --
class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled during the timed
    region through NVML read-only queries (every ~2 ms in a thread), falling
    back to `nvidia-smi -lms` when NVML is unavailable."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4}

    def __init__(self, gpu_index: int) -> None:
        self.gpu = gpu_index
        self.samples = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._nvml = None

    def start(self) -> None:
        try:
            import pynvml

            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            self._nvml = (pynvml, h)
        except Exception:
            self._nvml = None
            return

        def loop():
            pynvml, h = self._nvml
            while not self._stop.is_set():
                try:
                    mhz = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                    reasons = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.samples.append((mhz, reasons))
                except Exception:
                    pass
                time.sleep(0.002)

        self._thread = threading.Thread(target=loop, daemon=True)
        self._thread.start()

    def stop(self) -> dict:
        if self._nvml is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"], "samples": 0}
        self._stop.set()
        self._thread.join(timeout=2)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["no samples"], "samples": 0}
        mhz = [m for m, _ in self.samples]
        active = sorted({name for _, r in self.samples for name, bit in self.REASONS.items() if r & bit})
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.max_mhz, "reasons": active,
                "samples": len(self.samples), "source": "nvml"}


def workload_config(world: int) -> dict:
    return {"workload": "world reset: generation + full sky/block light + RGBA8->NCHW conversion",
            "envs_per_gpu": ENVS_PER_GPU, "world": [W, H, D], "torches_per_env": TORCHES,
            "terrain": "fBm 40+round(50*fbm)", "frames": [ENVS_PER_GPU, 3, FRAME_H, FRAME_W],
            "l2": f"outputs {2 * ENVS_PER_GPU * W * H * D / 1e9:.2f} GB per step per GPU rewritten every step "
                  f"(> 126 MB L2)",
            "parallelism": f"env shards x{world}"}


# ------------------------------------------------------------ CPU samples --
def cpu_sample(kind_pref: str = "reference"):
    """Times one bounded sample of the workload on the host cores.

    Returns (seconds, voxels, kind, cores, description)."""
    from oracle.oracle import TERRAIN_FBM, TERRAIN_REFERENCE, Oracle, Reference, WorldSpec, ref_available
    import numpy as np

    O = Oracle()
    if kind_pref == "reference" and ref_available("cpu"):
        R = Reference("cpu")
        spec = WorldSpec(BASE_SEED, SAMPLE_W, SAMPLE_H, SAMPLE_D, terrain=TERRAIN_REFERENCE)
        torches = O.place_torches(spec, SAMPLE_TORCHES, 0x5EED)
        timing = []
        R.generate(BASE_SEED, (0, 0, 0), (SAMPLE_W, SAMPLE_H, SAMPLE_D), torches,
                   np.full(len(torches), 4, np.uint8), runs=2, timing=timing)
        desc = (f"reference WorldGenerator::generate (CUDA CPU-fallback build) on one {SAMPLE_W}x{SAMPLE_H}x{SAMPLE_D} "
                f"region with {len(torches)} surface torches, reference terrain formula; converged second "
                f"generation timed (block cache + light + render list + cache readback)")
        return timing[-1] / 1e3, SAMPLE_W * SAMPLE_H * SAMPLE_D, "reference", os.cpu_count() or 1, desc
    spec = WorldSpec(BASE_SEED, SAMPLE_W, SAMPLE_H, SAMPLE_D, terrain=TERRAIN_FBM)
    torches = O.place_torches(spec, SAMPLE_TORCHES, 0x5EED)
    t0 = time.perf_counter()
    O.generate(spec, torches, np.full(len(torches), 4, np.uint8), method="per_source")
    dt = time.perf_counter() - t0
    desc = (f"oracle restatement (single thread) on one {SAMPLE_W}x{SAMPLE_H}x{SAMPLE_D} fBm region with "
            f"{len(torches)} torches")
    return dt, SAMPLE_W * SAMPLE_H * SAMPLE_D, "port", 1, desc


def gpu_reference_sample():
    """Times the reference's own CUDA kernels (its src/world/WorldGenerator.cu
    built for sm_100a under oracle/_ref) on one region of the benchmark's size,
    driven one region per call as its renderer drives them. Returns
    (seconds, voxels, description), or None when that build is absent."""
    from oracle.oracle import TERRAIN_REFERENCE, Oracle, Reference, WorldSpec, ref_available
    import numpy as np

    if not ref_available("cuda"):
        return None
    R = Reference("cuda")
    spec = WorldSpec(BASE_SEED, W, H, D, terrain=TERRAIN_REFERENCE)
    torches = Oracle().place_torches(spec, TORCHES, 0x5EED)
    timing = []
    R.generate(BASE_SEED, (0, 0, 0), (W, H, D), torches, np.full(len(torches), 4, np.uint8), runs=3, timing=timing)
    desc = (f"reference WorldGenerator::generate, its CUDA kernels built for sm_100a, on this GPU: one {W}x{H}x{D} "
            f"region with {len(torches)} surface torches, reference terrain formula; converged third generation "
            f"timed by wall clock (block cache + light + render list + its readback of the block cache)")
    return timing[-1] / 1e3, W * H * D, desc


def run_reference(args) -> None:
    rank, world, _ = dist_env()
    if rank != 0:
        return
    times = []
    vox = 0
    info = None
    for i in range(args.warmup + args.steps):
        dt, vox, kind, cores, desc = cpu_sample("reference")
        info = (kind, cores, desc)
        if i >= args.warmup:
            times.append(dt)
    total = sum(times)
    value = vox * len(times) / total
    kind, cores, desc = info
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / len(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": workload_config(args.gpus),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": kind, "sample": desc},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------- ours --
def load_traffic():
    """DRAM read+write bytes of one benchmark launch of the tile kernel, from
    the committed ncu summary (a 16-env capture scaled to the launch)."""
    path = os.path.join(ROOT, "profiles", "tile_kernel_reset_16envs_256x128x256.md")
    if os.path.exists(path):
        with open(path) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch_scaled:"):
                    return int(line.split(":", 1)[1])
    return None


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f), "measured"
    return {"hbm_gbs": 6650.0}, "fallback"


def run_ours(args) -> None:
    import numpy as np
    import torch

    global ENVS_PER_GPU
    ENVS_PER_GPU = args.envs or ENVS_PER_GPU

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist

    import blocklab_b200 as B

    cfg = B.WorldConfig(num_envs=ENVS_PER_GPU, width=W, height=H, depth=D, max_overrides=ENVS_PER_GPU * TORCHES)
    wb = B.WorldBatch(cfg, device=local)
    stream = torch.cuda.current_stream(dev)
    seeds_host = (BASE_SEED + rank * ENVS_PER_GPU + np.arange(ENVS_PER_GPU)).astype(np.uint32)
    seeds = torch.from_numpy(seeds_host.view(np.int32)).to(dev)
    gen = torch.Generator().manual_seed(1234 + rank)
    frames_host = torch.randint(0, 256, (ENVS_PER_GPU, FRAME_H, FRAME_W, 4), dtype=torch.uint8,
                                generator=gen).pin_memory()
    frames = frames_host.to(dev)
    obs = torch.empty((ENVS_PER_GPU, 3, FRAME_H, FRAME_W), dtype=torch.float32, device=dev)

    def step():
        torches = wb.place_torches(seeds, TORCHES)
        wb.generate(seeds, torches)
        B.convert_rgba8_to_float_nchw(frames, out=obs)

    def barrier():
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        step()
    wb.sync()
    barrier()

    clocks = ClockSampler(local)
    clocks.start()
    wb.profile(True)
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    clock_info = clocks.stop()
    wb.profile(False)
    prof = wb.profile_read()
    wb.sync()
    ms = ev0.elapsed_time(ev1)
    tile_ms = prof["generate_tiles_ms"] / max(prof["generate_calls"], 1)

    # End to end through the public API with host buffers: every step copies
    # its seeds and frames from pinned host memory and reads its height maps
    # back to pinned host memory. The copies run on a second stream with double
    # buffers, so that one step's transfers overlap its neighbours' kernels;
    # every step's own transfers lie inside the timed region.
    seeds_pinned = torch.from_numpy(seeds_host.view(np.int32)).pin_memory()
    copy_stream = torch.cuda.Stream(dev)
    hm_host = [torch.empty((ENVS_PER_GPU, D, W), dtype=torch.int16, pin_memory=True) for _ in range(2)]
    hm_dev = [torch.empty((ENVS_PER_GPU, D, W), dtype=torch.int16, device=dev) for _ in range(2)]
    seeds_dev = [torch.empty_like(seeds) for _ in range(2)]
    frames_dev = [torch.empty_like(frames) for _ in range(2)]
    ev = {name: [torch.cuda.Event() for _ in range(2)] for name in ("in_ready", "used", "hm_ready", "hm_read")}
    for b in range(2):  # all buffers start free
        ev["used"][b].record(stream)
        ev["hm_read"][b].record(stream)

    def issue_inputs(b):
        copy_stream.wait_event(ev["used"][b])
        with torch.cuda.stream(copy_stream):
            seeds_dev[b].copy_(seeds_pinned, non_blocking=True)
            frames_dev[b].copy_(frames_host, non_blocking=True)
        ev["in_ready"][b].record(copy_stream)

    def e2e_run(n):
        issue_inputs(0)
        for k in range(n):
            b = k % 2
            stream.wait_event(ev["in_ready"][b])
            torches = wb.place_torches(seeds_dev[b], TORCHES)
            wb.generate(seeds_dev[b], torches)
            B.convert_rgba8_to_float_nchw(frames_dev[b], out=obs)
            stream.wait_event(ev["hm_read"][b])
            hm_dev[b].copy_(wb.height_map, non_blocking=True)
            ev["used"][b].record(stream)
            ev["hm_ready"][b].record(stream)
            if k + 1 < n:
                issue_inputs(1 - b)
            copy_stream.wait_event(ev["hm_ready"][b])
            with torch.cuda.stream(copy_stream):
                hm_host[b].copy_(hm_dev[b], non_blocking=True)
            ev["hm_read"][b].record(copy_stream)
        for b in range(2):
            stream.wait_event(ev["hm_read"][b])

    e2e_run(args.warmup)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    copy_stream.wait_event(e0)
    e2e_run(args.steps)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    e2e_ms = e0.elapsed_time(e1)

    times = torch.tensor([ms, e2e_ms, tile_ms], dtype=torch.float64, device=dev)
    if pg is not None:
        pg.all_reduce(times, op=pg.ReduceOp.MAX)
    ms, e2e_ms, tile_ms = (float(v) for v in times.tolist())

    vox_step = ENVS_PER_GPU * W * H * D
    total_vox = vox_step * world * args.steps
    value = total_vox / (ms / 1e3)
    e2e_value = total_vox / (e2e_ms / 1e3)
    peaks, peak_kind = measured_peaks()
    algo_bytes = 2 * vox_step
    achieved = algo_bytes / (tile_ms / 1e3) / 1e9
    traffic = load_traffic()
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": workload_config(world),
        "env_resets_per_s": ENVS_PER_GPU * world * args.steps / (ms / 1e3),
        "roofline": {"bound": "hbm", "kernel": "tile_kernel", "achieved": achieved, "peak": peaks["hbm_gbs"],
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                     "algorithmic_bytes_per_launch": algo_bytes, "kernel_ms": tile_ms,
                     "traffic": traffic if ENVS_PER_GPU == 128 else None},
        "e2e": {"value": e2e_value, "unit": UNIT,
                "h2d_bytes_per_step": seeds.numel() * 4 + frames.numel(),
                "d2h_bytes_per_step": hm_host[0].numel() * 2},
        "gpu_launches": LAUNCHES_PER_STEP * args.steps,
        "clocks": clock_info,
        "profile": {"generate_prep_ms": prof["generate_prep_ms"] / max(prof["generate_calls"], 1),
                    "generate_tiles_ms": tile_ms},
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        dt, vox, kind, cores, desc = cpu_sample("reference")
        line["cpu_baseline"] = {"value": vox / dt, "unit": UNIT, "cores": cores, "kind": kind, "sample": desc}
        ref_gpu = gpu_reference_sample()
        if ref_gpu is not None:
            dt, vox, desc = ref_gpu
            line["reference_gpu"] = {"value": vox / dt, "unit": UNIT, "sample": desc}
    wb.close()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()


# --------------------------------------------------- secondary workloads --
# The relight, day/night and scale-out configurations. Each prints its own
# JSON line; the default invocation (reset) is the headline.
RELIGHT = dict(envs=1024, W=128, H=128, D=128, torches=200, edits=10000)
DAYNIGHT = dict(envs=4096, W=128, H=96, D=128, torches=300, frame=84, steps_per_sweep=256)
SCALEOUT = dict(envs=1024, W=256, H=256, D=256, torches=2000, amplitude=120.0, edits_total=5000, envs_total=8192)


def init_dist():
    import datetime

    import torch

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist
    return rank, world, local, dev, pg


def time_steps(fn, steps, warmup, dev, pg, clock_gpu):
    """Runs warmup untimed steps, then times `steps` calls of fn(k) with CUDA
    events on the current stream between barriers; returns (ms, clocks)."""
    import torch

    def barrier():
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize(dev)

    for k in range(warmup):
        fn(k)
    barrier()
    clocks = ClockSampler(clock_gpu)
    clocks.start()
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for k in range(steps):
        fn(warmup + k)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    info = clocks.stop()
    ms = e0.elapsed_time(e1)
    if pg is not None:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms = float(t.item())
    return ms, info


def surface_edits(rng, hm, envs, n, W, D, torch_xyz):
    """n edits over `envs` worlds: 45% dig, 45% place stone, 5% torch, 5%
    remove an existing torch; cells uniform within 8 voxels of the surface."""
    import numpy as np

    import blocklab_b200 as B

    env = rng.integers(0, envs, n)
    x, z = rng.integers(0, W, n), rng.integers(0, D, n)
    y = hm[env, z, x].astype(np.int64) + rng.integers(-8, 9, n)
    r = rng.random(n)
    blk = np.where(r < 0.45, B.AIR, np.where(r < 0.9, B.STONE, B.TORCH)).astype(np.uint8)
    kind = np.zeros(n, np.uint8)
    rm = r >= 0.95
    if rm.any() and torch_xyz is not None:
        pick = rng.integers(0, torch_xyz.shape[1], int(rm.sum()))
        t = torch_xyz[env[rm], pick]
        x[rm], y[rm], z[rm] = t[:, 0], t[:, 1], t[:, 2]
        blk[rm] = B.AIR
        kind[rm] = 1
    return B.make_overrides(np.stack([x, y, z], 1), blk, env=env, kind=kind)


def dirty_voxels(before, after, W, H, D):
    """Voxels within L-inf distance 14 (clipped to the world) of a cell whose
    light class changed (opaque / open / torch), summed over envs: the cells
    whose light an exact relight must revisit. An opaque block replaced by
    another opaque block changes no light, and neither does an air <-> opaque
    change of a cell that ends the step enclosed (below its column's top before
    and after the step, six opaque neighbours, no torch before or after). Also returns the number of
    cells whose block id changed and the number of light-class changes."""
    import numpy as np
    import torch
    import torch.nn.functional as F

    def light_class(ids):  # 0 opaque, 1 air, 2 torch (ids: Air 0, Torch 4)
        return (ids == 0).to(torch.uint8) + 2 * (ids == 4).to(torch.uint8)

    n_changed = int((before != after).sum().item())
    rows = []
    n_light = 0
    for e0 in range(0, before.shape[0], 64):  # ids [env][z][x][y], 64 envs at a time
        b, a = before[e0:e0 + 64], after[e0:e0 + 64]
        moved = light_class(b) != light_class(a)
        n_light += int(moved.sum().item())
        opaque = ((a != 0) & (a != 4)).to(torch.uint8)
        y = torch.arange(H, device=a.device, dtype=torch.int32)
        top = torch.where(opaque.bool(), y, torch.full_like(y, -1)).amax(dim=3, keepdim=True)
        top_before = torch.where((b != 0) & (b != 4), y, torch.full_like(y, -1)).amax(dim=3, keepdim=True)
        p = F.pad(opaque, (1, 1, 1, 1, 1, 1), value=1)
        nb = (p[:, :-2, 1:-1, 1:-1] & p[:, 2:, 1:-1, 1:-1] & p[:, 1:-1, :-2, 1:-1] & p[:, 1:-1, 2:, 1:-1]
              & p[:, 1:-1, 1:-1, :-2] & p[:, 1:-1, 1:-1, 2:]).bool()
        enclosed = nb & (y < top) & (y < top_before) & (b != 4) & (a != 4)
        idx = (moved & ~enclosed).nonzero()
        idx[:, 0] += e0
        rows.append(idx.cpu().numpy())
    changed = np.concatenate(rows) if rows else np.zeros((0, 4), np.int64)  # (env, z, x, y)
    total = 0
    for e in np.unique(changed[:, 0]):
        m = np.zeros((D, W, H), bool)
        for _, z, x, y in changed[changed[:, 0] == e]:
            m[max(z - 14, 0):z + 15, max(x - 14, 0):x + 15, max(y - 14, 0):y + 15] = True
        total += int(m.sum())
    return total, n_changed, n_light, len(changed)


def run_workload(args) -> None:
    import numpy as np
    import torch

    if args.impl == "reference":
        run_workload_reference(args)
        return
    import blocklab_b200 as B

    rank, world, local, dev, pg = init_dist()
    peaks, peak_kind = measured_peaks()
    line = {"n_gpus": world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "data": "synthetic"}
    rng = np.random.default_rng(4242 + rank)

    if args.workload == "relight":
        c = dict(RELIGHT)
        c["envs"] = args.envs or c["envs"]
        E, Wd, Hd, Dd = c["envs"], c["W"], c["H"], c["D"]
        n_edits = c["edits"] * E // RELIGHT["envs"]
        cfg = B.WorldConfig(num_envs=E, width=Wd, height=Hd, depth=Dd, max_overrides=E * c["torches"],
                            max_edits=n_edits)
        wb = B.WorldBatch(cfg, device=local)
        seeds = (BASE_SEED + rank * E + np.arange(E)).astype(np.uint32)
        torches = wb.place_torches(seeds, c["torches"])
        wb.generate(seeds, torches)
        wb.sync()
        hm = wb.height_map.cpu().numpy()
        tl = torches.cpu().numpy().view(B.OVERRIDE_DTYPE).reshape(E, c["torches"])
        txyz = np.stack([tl["x"], tl["y"], tl["z"]], 2)
        batches = [surface_edits(rng, hm, E, n_edits, Wd, Dd, txyz) for _ in range(args.warmup + args.steps)]
        dev_batches = [torch.from_numpy(b.view(np.uint8).copy()).to(dev) for b in batches]
        # Dirty volume of the first timed step, measured outside the timed region.
        for k in range(args.warmup):
            wb.apply_edits(dev_batches[k])
        before = wb.ids.clone()
        wb.apply_edits(dev_batches[args.warmup])
        dirty, n_changed, n_light, n_relit = dirty_voxels(before, wb.ids, Wd, Hd, Dd)
        del before
        # Timed run on a fresh copy of the same worlds and edit sequence.
        wb.generate(seeds, torches)
        wb.profile(True)
        ms, clocks = time_steps(lambda k: wb.apply_edits(dev_batches[k]), args.steps, args.warmup, dev, pg, local)
        prof = wb.profile_read()
        wb.profile(False)
        relight_ms = prof["relight_ms"] / max(prof["edit_calls"], 1)
        pinned = [torch.from_numpy(b.view(np.uint8).copy()).pin_memory() for b in batches]
        stage = torch.empty_like(dev_batches[0])
        wb.generate(seeds, torches)

        def e2e(k):
            stage.copy_(pinned[k], non_blocking=True)
            wb.apply_edits(stage)

        e2e_ms, _ = time_steps(e2e, args.steps, args.warmup, dev, pg, local)
        env_steps = E * world * args.steps
        algo = 3 * dirty
        line.update({
            "metric": "env-steps/s (incremental relight)", "value": env_steps / (ms / 1e3), "unit": "env-steps/s",
            "ms_per_step": ms / args.steps, "dtype": "u8",
            "config": {"workload": "relight: edits with World::setBlock semantics + exact incremental relight",
                       "envs_per_gpu": E, "world": [Wd, Hd, Dd], "torches_per_env": c["torches"],
                       "edits_per_step_per_gpu": n_edits, "mix": "45% dig, 45% stone, 5% torch, 5% remove torch",
                       "l2": "edits touch scattered tiles of a 4.3 GB world; no flush needed (L2 126 MB)",
                       "parallelism": f"env shards x{world}"},
            "roofline": {"bound": "hbm", "kernel": "tile_kernel (relight) + apply_edits",
                         "achieved": algo / (relight_ms / 1e3) / 1e9 if relight_ms > 0 else None,
                         "peak": peaks["hbm_gbs"], "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": (algo / (relight_ms / 1e3) / 1e9) / peaks["hbm_gbs"] if relight_ms > 0 else None,
                         "algorithmic_bytes_per_step": algo, "dirty_voxels_per_step": dirty,
                         "changed_cells_per_step": n_changed, "light_class_changes_per_step": n_light,
                         "relit_changes_per_step": n_relit,
                         "relight_ms": relight_ms, "traffic": None},
            "e2e": {"value": env_steps / (e2e_ms / 1e3), "unit": "env-steps/s",
                    "h2d_bytes_per_step": int(dev_batches[0].numel()), "d2h_bytes_per_step": 0},
            "gpu_launches": None, "clocks": clocks})
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            # The reference regenerates and relights a region for every edit
            # (src/graphics/Renderer.cpp:1121-1141): its own CUDA kernels on
            # this GPU, one region per env-step.
            from oracle.oracle import TERRAIN_REFERENCE, Oracle, Reference, WorldSpec, ref_available

            if ref_available("cuda"):
                R = Reference("cuda")
                rspec = WorldSpec(BASE_SEED, Wd, Hd, Dd, terrain=TERRAIN_REFERENCE)
                rt = Oracle().place_torches(rspec, c["torches"], 0x5EED)
                times = []
                for _ in range(5):
                    timing = []
                    R.generate(BASE_SEED, (0, 0, 0), (Wd, Hd, Dd), rt, np.full(len(rt), 4, np.uint8), runs=2,
                               timing=timing)
                    times.append(timing[-1] / 1e3)
                line["reference_gpu"] = {
                    "value": len(times) / sum(times), "unit": "env-steps/s",
                    "sample": f"reference WorldGenerator::generate, its CUDA kernels built for sm_100a, on this GPU: "
                              f"one {Wd}x{Hd}x{Dd} region with {len(rt)} torches regenerated per env-step (reference "
                              f"terrain; converged generation by wall clock, including its block-cache readback)"}
        wb.close()
    elif args.workload == "daynight":
        c = dict(DAYNIGHT)
        c["envs"] = args.envs or c["envs"]
        E, Wd, Hd, Dd, F = c["envs"], c["W"], c["H"], c["D"], c["frame"]
        cfg = B.WorldConfig(num_envs=E, width=Wd, height=Hd, depth=Dd, max_overrides=E * c["torches"])
        wb = B.WorldBatch(cfg, device=local)
        seeds = (BASE_SEED + rank * E + np.arange(E)).astype(np.uint32)
        wb.generate(seeds, wb.place_torches(seeds, c["torches"]))
        gen = torch.Generator().manual_seed(99 + rank)
        frames = torch.randint(0, 256, (E, F, F, 4), dtype=torch.uint8, generator=gen).to(dev)
        obs = torch.empty((E, 3, F, F), dtype=torch.float32, device=dev)
        eff = torch.empty_like(wb.light) if args.materialize else None
        half = c["steps_per_sweep"] // 2
        # Tick of sweep step k: across the sunset ramp, then the sunrise ramp.
        ticks = [12000 + (13702 - 12000) * k // (half - 1) for k in range(half)] + \
                [22300 + (23961 - 22300) * k // (half - 1) for k in range(half)]
        dims = torch.tensor([[B.sky_light_dimming(t)] * E for t in ticks], dtype=torch.uint8).pin_memory()
        dim_dev = torch.empty(E, dtype=torch.uint8, device=dev)

        def step(k):
            dim_dev.copy_(dims[k % len(ticks)], non_blocking=True)
            B.convert_rgba8_to_float_nchw(frames, out=obs)
            if eff is not None:
                wb.effective_light(dim_dev, out=eff)

        ms, clocks = time_steps(step, args.steps, args.warmup, dev, pg, local)
        env_steps = E * world * args.steps
        conv_bytes = 16 * E * F * F + (2 * wb.light.numel() if eff is not None else 0)
        achieved = conv_bytes * args.steps / (ms / 1e3) / 1e9
        line.update({
            "metric": "env-steps/s (day/night sweep)", "value": env_steps / (ms / 1e3), "unit": "env-steps/s",
            "ms_per_step": ms / args.steps, "dtype": "u8 -> f32",
            "config": {"workload": "daynight: sky level by tick (sunset then sunrise ramps), dimming upload, "
                                   "RGBA8 84x84 -> float32 NCHW" + (", effective light of every cell"
                                                                     if eff is not None else ""),
                       "envs_per_gpu": E, "world": [Wd, Hd, Dd], "torches_per_env": c["torches"],
                       "frames": [E, 3, F, F], "l2": f"{conv_bytes / 1e9:.2f} GB moved per step (> 126 MB L2)",
                       "parallelism": f"env shards x{world}"},
            "roofline": {"bound": "hbm", "kernel": "rgba_to_nchw_vec_kernel" + (
                " + effective_light_kernel" if eff is not None else ""), "achieved": achieved,
                "peak": peaks["hbm_gbs"], "peak_kind": peak_kind, "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"], "algorithmic_bytes_per_step": conv_bytes, "traffic": None},
            "gpu_launches": (2 if eff is not None else 1) * args.steps, "clocks": clocks})
        wb.close()
    elif args.workload == "render":
        E = args.envs or ENVS_PER_GPU
        cfg = B.WorldConfig(num_envs=E, width=W, height=H, depth=D, max_overrides=E * TORCHES)
        wb = B.WorldBatch(cfg, device=local)
        seeds = (BASE_SEED + rank * E + np.arange(E)).astype(np.uint32)
        wb.generate(seeds, wb.place_torches(seeds, TORCHES))
        hm = wb.height_map.cpu().numpy()
        # Agents at the world centre on the surface, looking around, at several day times.
        params = np.array([B.render_params_at((W / 2, hm[e, D // 2, W // 2] + 1, D / 2), 0.7 * e, -0.25,
                                              (6000 + 997 * e) % 24000) for e in range(E)], B.RENDER_PARAMS_DTYPE)
        params_dev = torch.from_numpy(params.view(np.uint8).copy()).to(dev)
        frames = torch.empty((E, FRAME_H, FRAME_W, 4), dtype=torch.uint8, device=dev)
        obs = torch.empty((E, 3, FRAME_H, FRAME_W), dtype=torch.float32, device=dev)
        from blocklab_b200 import _native as N

        def step(k):
            # Frames rendered straight into the observation tensor (RGBA8 kept too).
            N.check(N.lib.blk_render_observations(wb._ctx, params_dev.data_ptr(), FRAME_W, FRAME_H, obs.data_ptr(),
                                                  frames.data_ptr(), torch.cuda.current_stream(dev).cuda_stream))

        ms, clocks = time_steps(step, args.steps, args.warmup, dev, pg, local)
        line.update({
            "metric": "frames/s (render to observations)", "value": E * world * args.steps / (ms / 1e3),
            "unit": "frames/s", "ms_per_step": ms / args.steps, "dtype": "u8 -> f32",
            "config": {"workload": "render: ray-cast 160x90 frames of the reset worlds into RGBA8 and float NCHW",
                       "envs_per_gpu": E, "world": [W, H, D], "frames": [E, 3, FRAME_H, FRAME_W],
                       "parallelism": f"env shards x{world}"},
            "gpu_launches": args.steps, "clocks": clocks})
        wb.close()
    else:  # scaleout
        c = dict(SCALEOUT)
        c["envs"] = args.envs or c["envs"]
        E, Wd, Hd, Dd = c["envs"], c["W"], c["H"], c["D"]
        n_edits = c["edits_total"] * E // c["envs_total"]
        cfg = B.WorldConfig(num_envs=E, width=Wd, height=Hd, depth=Dd, amplitude=c["amplitude"],
                            max_overrides=E * c["torches"], max_edits=max(n_edits, 1))
        wb = B.WorldBatch(cfg, device=local)
        seeds = (BASE_SEED + rank * E + np.arange(E)).astype(np.uint32)
        seeds_dev = torch.from_numpy(seeds.view(np.int32)).to(dev)
        reset_torches = {}

        def reset(k):
            reset_torches["t"] = wb.place_torches(seeds_dev, c["torches"])
            wb.generate(seeds_dev, reset_torches["t"])

        reset_ms, reset_clocks = time_steps(reset, 1, 1, dev, pg, local)
        hm = wb.height_map.cpu().numpy()
        tl = reset_torches["t"].cpu().numpy().view(B.OVERRIDE_DTYPE).reshape(E, c["torches"])
        txyz = np.stack([tl["x"], tl["y"], tl["z"]], 2)
        batches = [torch.from_numpy(surface_edits(rng, hm, E, n_edits, Wd, Dd, txyz).view(np.uint8).copy()).to(dev)
                   for _ in range(args.warmup + args.steps)]
        gen = torch.Generator().manual_seed(7 + rank)
        frames = torch.randint(0, 256, (E, FRAME_H, FRAME_W, 4), dtype=torch.uint8, generator=gen).to(dev)
        obs = torch.empty((E, 3, FRAME_H, FRAME_W), dtype=torch.float32, device=dev)
        gathered = None
        if args.gather and pg is not None and rank == 0:
            gathered = [torch.empty_like(obs) for _ in range(world)]

        def step(k):
            wb.apply_edits(batches[k])
            B.convert_rgba8_to_float_nchw(frames, out=obs)
            if args.gather and pg is not None:
                pg.gather(obs, gathered if rank == 0 else None, dst=0)

        ms, clocks = time_steps(step, args.steps, args.warmup, dev, pg, local)
        env_steps = E * world * args.steps
        line.update({
            "metric": "env-steps/s (scale-out)", "value": env_steps / (ms / 1e3), "unit": "env-steps/s",
            "ms_per_step": ms / args.steps, "dtype": "u8",
            "config": {"workload": "scaleout: per step edits + exact relight + 90x160 frame conversion"
                                   + (" + NCCL gather of observations to rank 0" if args.gather else ""),
                       "envs_per_gpu": E, "world": [Wd, Hd, Dd], "terrain": "fBm 40+round(120*fbm)",
                       "torches_per_env": c["torches"], "edits_per_step_per_gpu": n_edits,
                       "l2": "34 GB of world per GPU", "parallelism": f"env shards x{world}"},
            "reset": {"ms": reset_ms, "voxels_per_s": E * world * Wd * Hd * Dd / (reset_ms / 1e3),
                      "clocks": reset_clocks},
            "gpu_launches": None, "clocks": clocks})
        wb.close()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()


def run_workload_reference(args) -> None:
    """The reference regenerates a region for every edit
    (src/graphics/Renderer.cpp:1121-1141): one env-step of relight costs one
    WorldGenerator::generate of the region, timed on the host cores."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    if args.workload != "relight":
        print(json.dumps({"impl": "reference", "workload": args.workload,
                          "unavailable": "the reference has no batched CPU path for this workload"}), flush=True)
        return
    import numpy as np

    from oracle.oracle import TERRAIN_REFERENCE, Oracle, Reference, WorldSpec, ref_available

    if not ref_available("cpu"):
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libref_cpu.so not built"}), flush=True)
        return
    O, R = Oracle(), Reference("cpu")
    c = RELIGHT
    spec = WorldSpec(BASE_SEED, c["W"], c["H"], c["D"], terrain=TERRAIN_REFERENCE)
    torches = O.place_torches(spec, c["torches"], 0x5EED)
    times = []
    for i in range(args.warmup + args.steps):
        timing = []
        R.generate(BASE_SEED, (0, 0, 0), (c["W"], c["H"], c["D"]), torches, np.full(len(torches), 4, np.uint8),
                   runs=1, timing=timing)
        if i >= args.warmup:
            times.append(timing[-1] / 1e3)
    value = len(times) / sum(times)
    print(json.dumps({"impl": "reference", "metric": "env-steps/s (incremental relight)", "value": value,
                      "unit": "env-steps/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                      "higher_is_better": True,
                      "cpu_baseline": {"value": value, "unit": "env-steps/s", "cores": os.cpu_count() or 1,
                                       "kind": "reference",
                                       "sample": f"one WorldGenerator::generate of a {c['W']}x{c['H']}x{c['D']} region "
                                                 f"with {len(torches)} torches per env-step (reference terrain)"}}),
          flush=True)


def main() -> None:
    args = parse_args()
    if args.workload != "reset":
        run_workload(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
