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
# terrain surface, tile kernel, conversion.
LAUNCHES_PER_STEP = 10


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--envs", type=int, default=ENVS_PER_GPU,
                    help="envs per GPU (default 128; smaller batches are for profiler captures)")
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
    ENVS_PER_GPU = args.envs

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

    # End to end through the public API with host buffers: pinned H2D of the
    # step's seeds and frames, D2H of the step's height maps.
    seeds_pinned = torch.from_numpy(seeds_host.view(np.int32)).pin_memory()
    hm_host = torch.empty((ENVS_PER_GPU, D, W), dtype=torch.int16, pin_memory=True)
    seeds_dev = torch.empty_like(seeds)
    frames_dev = torch.empty_like(frames)

    def e2e_step():
        seeds_dev.copy_(seeds_pinned, non_blocking=True)
        frames_dev.copy_(frames_host, non_blocking=True)
        torches = wb.place_torches(seeds_dev, TORCHES)
        wb.generate(seeds_dev, torches)
        B.convert_rgba8_to_float_nchw(frames_dev, out=obs)
        hm_host.copy_(wb.height_map, non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
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
                "d2h_bytes_per_step": hm_host.numel() * 2},
        "gpu_launches": LAUNCHES_PER_STEP * args.steps,
        "clocks": clock_info,
        "profile": {"generate_prep_ms": prof["generate_prep_ms"] / max(prof["generate_calls"], 1),
                    "generate_tiles_ms": tile_ms},
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        dt, vox, kind, cores, desc = cpu_sample("reference")
        line["cpu_baseline"] = {"value": vox / dt, "unit": UNIT, "cores": cores, "kind": kind, "sample": desc}
    wb.close()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
