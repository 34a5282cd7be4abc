#!/usr/bin/env python
"""World-state benchmark of the B200 world library.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload reset|relight|daynight|scaleout|render]

Default (one JSON line, rank 0): the reset workload, whose metric is the
headline. Per GPU and step: 128 envs of 256 x 256 x 128 voxels (fBm terrain,
per-env seed = base seed + global env id, 1000 surface torches per env), full
generation + sky/block light, and conversion of 128 RGBA8 160x90 frames to a
(128, 3, 90, 160) float32 tensor. K steps are timed exactly; a `sustained`
record repeats the step for at least half a second. The line also carries one
record per other configuration (`configs`: relight, daynight, scaleout), each
timed for at least half a second with its own clocks, roofline and end-to-end
figure. Multi-GPU runs are weak-scaled: every rank owns its own envs (global
env ids rank * envs ...), with no data-path collective.

`--workload X` prints only configuration X's record as the line. `--impl
reference` times the reference's own CPU implementation of the path (its CUDA
CPU-fallback build, compiled from the reference sources into oracle/_ref) on a
bounded sample of the benchmark's own world, given to it as a dense override
list (its generator has no fBm terrain).
"""
from __future__ import annotations

import argparse
import csv
import json
import math
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

BASE_SEED = 1
RESET = dict(envs=128, W=256, H=128, D=256, torches=1000, frame=(90, 160))
RELIGHT = dict(envs=1024, W=128, H=128, D=128, torches=200, edits=10000)
DAYNIGHT = dict(envs=4096, W=128, H=96, D=128, torches=300, frame=84, steps_per_sweep=256)
SCALEOUT = dict(envs=1024, W=256, H=256, D=256, torches=2000, amplitude=120.0, edits_total=5000, envs_total=8192)
# Bounded sample of the reset world for the reference's CPU build: a 128^3
# corner of env 0 keeps the benchmark's torch density (1000 per 256 x 256).
SAMPLE = dict(W=128, H=128, D=128)
SUSTAINED_S = 0.5  # every configuration is timed for at least this long
# This library's kernel launches per step (from the launch lists in profiles/):
# reset: torch placement, override count / scan (3) / scatter / sort, fBm
# surface with the column summaries, surface kernel, tile kernel over the
# tiles the surface kernel left, conversion; relight: edit
# count / scan (3) / scatter, setBlock application, change marking, region
# build, dirty-tile compaction, four region kernels, tile kernel.
LAUNCHES = dict(reset=11, relight=14, daynight=1, scaleout=15, render=1)
TRAFFIC_CSV = os.path.join(ROOT, "profiles", "generation_reset_traffic.csv")


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="reset line without the other configurations")
    ap.add_argument("--envs", type=int, default=None,
                    help="envs per GPU (default: the workload's; smaller batches are for profiler captures)")
    ap.add_argument("--workload", choices=["reset", "relight", "daynight", "scaleout", "render"], default="reset")
    ap.add_argument("--gather", action="store_true", help="scaleout: gather observations to rank 0 every step")
    ap.add_argument("--materialize", action="store_true",
                    help="daynight: also materialise the effective light of every cell each step")
    return ap.parse_args()


# ------------------------------------------------------------ plumbing --
def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


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


def barrier(dev, pg):
    import torch

    if pg is not None:
        pg.barrier()
    torch.cuda.synchronize(dev)


def max_over_ranks(values, dev, pg):
    import torch

    if pg is None:
        return [float(v) for v in values]
    t = torch.tensor(values, dtype=torch.float64, device=dev)
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return [float(v) for v in t.tolist()]


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled during a timed
    region through NVML read-only queries (every ~2 ms in a thread)."""

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


def time_steps(fn, steps, warmup, dev, pg, clock_gpu, stream=None):
    """W untimed calls of fn(k), then `steps` calls timed with CUDA events on
    the current stream between barrier + synchronize, clocks sampled meanwhile;
    returns (ms, clocks) with ms the max over ranks."""
    import torch

    for k in range(warmup):
        fn(k)
    barrier(dev, pg)
    clocks = ClockSampler(clock_gpu)
    clocks.start()
    st = stream if stream is not None else torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for k in range(steps):
        fn(warmup + k)
    e1.record(st)
    torch.cuda.synchronize(dev)
    barrier(dev, pg)
    info = clocks.stop()
    (ms,) = max_over_ranks([e0.elapsed_time(e1)], dev, pg)
    return ms, info


def sustained_steps(ms_per_step, minimum, dev, pg):
    """Steps that fill SUSTAINED_S at the measured step time (same on every rank)."""
    (ms,) = max_over_ranks([ms_per_step], dev, pg)
    return max(minimum, int(math.ceil(SUSTAINED_S * 1e3 / max(ms, 1e-3))))


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f), "measured"
    return {"hbm_gbs": 6650.0}, "fallback"


def load_traffic():
    """DRAM bytes read + written by one benchmark generation (the surface
    kernel and the tile kernel's launch over the tiles it left): ncu's own CSV
    of those two launches (profiles/generation_reset_traffic.csv, written by the
    command in the summary beside it), or None when absent."""
    if not os.path.exists(TRAFFIC_CSV):
        return None
    got = {}
    with open(TRAFFIC_CSV) as f:
        rows = [r for r in csv.reader(f) if r]
    hdr = next((r for r in rows if "Metric Name" in r), None)
    if hdr is None:
        return None
    i_name, i_val, i_kernel = hdr.index("Metric Name"), hdr.index("Metric Value"), hdr.index("Kernel Name")
    i_unit = hdr.index("Metric Unit") if "Metric Unit" in hdr else None
    scale = {"byte": 1, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9}
    for r in rows:
        if r is hdr or len(r) <= i_val or not ("tile_kernel" in r[i_kernel] or "surface_kernel" in r[i_kernel]):
            continue
        unit = r[i_unit] if i_unit is not None else "byte"
        if r[i_name] in ("dram__bytes_read.sum", "dram__bytes_write.sum"):
            got[r[i_name]] = got.get(r[i_name], 0.0) + float(r[i_val].replace(",", "")) * scale.get(unit, 1)
    if len(got) != 2:
        return None
    return int(sum(got.values()))


# ---------------------------------------------------- reference samples --
def fbm_world(seed, W, H, D, torches, amplitude=50.0):
    """The benchmark's world of one env (fBm terrain + surface torches at the
    library's torch columns) as a reference-layout block volume (D, H, W),
    built by the oracle restatement (input construction, not timed)."""
    import numpy as np

    import blocklab_b200 as B
    from oracle.oracle import Oracle, WorldSpec

    O = Oracle()
    spec = WorldSpec(seed, W, H, D, amplitude=amplitude)
    t = O.place_torches(spec, torches, B.torch_key(seed))
    blocks, _ = O.build_blocks(spec, t, np.full(len(t), 4, np.uint8))
    return blocks, len(t)


def reference_cpu_times(n_generations):
    """Wall times (s) of n consecutive generations of the reference's own CPU
    build on the bounded sample: the 128^3 corner of the reset benchmark's env
    0 (fBm world, its torches), given as a dense override list; the first
    generation converges the reference's light-source capacity and is not
    returned. Also returns (voxels, cores, description)."""
    from oracle.oracle import Reference

    blocks, n_t = fbm_world(BASE_SEED, RESET["W"], RESET["H"], RESET["D"], RESET["torches"])
    sub = blocks[:SAMPLE["D"], :SAMPLE["H"], :SAMPLE["W"]].copy()
    n_sub = int((sub == 4).sum())
    R = Reference("cpu")
    timing = []
    R.light_blocks(sub, runs=n_generations + 1, timing=timing)
    desc = (f"reference WorldGenerator::generate (its CUDA CPU-fallback build) on the {SAMPLE['W']}x{SAMPLE['H']}x"
            f"{SAMPLE['D']} corner of the reset benchmark's env 0 (fBm terrain, {n_sub} of its torches), the world "
            f"given as a dense override list (its generator has no fBm terrain: the sort of 2.1 M overrides and a "
            f"binary search per voxel are part of its time); converged generations timed by wall clock (block "
            f"cache + light + render list + cache readback)")
    return [t / 1e3 for t in timing[1:]], sub.size, os.cpu_count() or 1, desc


def reference_gpu_record(W, H, D, torches, unit, per_unit, amplitude=50.0, what="the reset benchmark's env 0"):
    """The reference's own CUDA kernels (its WorldGenerator.cu built for
    sm_100a under oracle/_ref) on one env of the configuration's world (dense
    override list): device time of its kernels per generation by CUDA events
    (one captured generation's kernels, without its host work and its 12 B per
    voxel block-cache readback), and the wall time of an ordinary generation."""
    from oracle.oracle import Reference, ref_available

    if not ref_available("cuda"):
        return None
    blocks, n_t = fbm_world(BASE_SEED, W, H, D, torches, amplitude)
    k_ms, w_ms = Reference("cuda").kernel_time(blocks, runs=2, reps=5)
    return {"value": per_unit / (k_ms / 1e3), "unit": unit, "kernel_ms": k_ms, "wall_ms": w_ms,
            "wall_value": per_unit / (w_ms / 1e3),
            "sample": f"reference WorldGenerator::generate, its CUDA kernels built for sm_100a, on this GPU: {what} "
                      f"({W}x{H}x{D}, fBm, {n_t} torches) given as a dense override list; value = its kernels' "
                      f"device time per generation (CUDA events around a graph of one converged generation's kernels, "
                      f"without its override sort and copies); wall_value = an ordinary generation by wall clock, "
                      f"including its block-cache readback"}


# ------------------------------------------------------------- records --
def reset_record(args, rank, world, local, dev, pg, peaks, peak_kind):
    import numpy as np
    import torch

    import blocklab_b200 as B

    E = args.envs or RESET["envs"]
    W, H, D, T = RESET["W"], RESET["H"], RESET["D"], RESET["torches"]
    FH, FW = RESET["frame"]
    cfg = B.WorldConfig(num_envs=E, width=W, height=H, depth=D, max_overrides=E * T)
    wb = B.WorldBatch(cfg, device=local)
    stream = torch.cuda.current_stream(dev)
    seeds_host = (BASE_SEED + rank * E + np.arange(E)).astype(np.uint32)
    seeds = torch.from_numpy(seeds_host.view(np.int32)).to(dev)
    gen = torch.Generator().manual_seed(1234 + rank)
    frames_host = torch.randint(0, 256, (E, FH, FW, 4), dtype=torch.uint8, generator=gen).pin_memory()
    frames = frames_host.to(dev)
    obs = torch.empty((E, 3, FH, FW), dtype=torch.float32, device=dev)

    def step(_k):
        torches = wb.place_torches(seeds, T)
        wb.generate(seeds, torches)
        B.convert_rgba8_to_float_nchw(frames, out=obs)

    wb.profile(True)
    ms, clocks = time_steps(step, args.steps, args.warmup, dev, pg, local)
    prof = wb.profile_read()
    wb.profile(False)
    wb.sync()
    tile_ms = prof["generate_tiles_ms"] / max(prof["generate_calls"], 1)
    prep_ms = prof["generate_prep_ms"] / max(prof["generate_calls"], 1)
    fallback = wb.generation_fallback_tiles()
    n_sus = sustained_steps(ms / args.steps, args.steps, dev, pg)
    sus_ms, sus_clocks = time_steps(step, n_sus, 1, dev, pg, local)

    # End to end through the public API with host buffers: every step copies
    # its seeds and frames from pinned host memory and reads its height maps
    # back to pinned host memory. The copies run on a second stream with double
    # buffers, so that one step's transfers overlap its neighbours' kernels;
    # every step's own transfers lie inside the timed region. Timed over the
    # sustained loop's step count (at least SUSTAINED_S), so that the first
    # step's input copy and the last step's read-back, which nothing overlaps,
    # are a small part of it.
    seeds_pinned = torch.from_numpy(seeds_host.view(np.int32)).pin_memory()
    copy_stream = torch.cuda.Stream(dev)
    hm_host = [torch.empty((E, D, W), dtype=torch.int16, pin_memory=True) for _ in range(2)]
    hm_dev = [torch.empty((E, D, W), dtype=torch.int16, device=dev) for _ in range(2)]
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
            torches = wb.place_torches(seeds_dev[b], T)
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
    barrier(dev, pg)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    copy_stream.wait_event(e0)
    e2e_run(n_sus)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(dev, pg)
    (e2e_ms,) = max_over_ranks([e0.elapsed_time(e1)], dev, pg)
    tile_ms, prep_ms = max_over_ranks([tile_ms, prep_ms], dev, pg)
    wb.close()

    vox_step = E * W * H * D
    total_vox = vox_step * world * args.steps
    algo_bytes = 2 * vox_step
    achieved = algo_bytes / (tile_ms / 1e3) / 1e9
    traffic = load_traffic() if E == RESET["envs"] else None
    return {
        "metric": "voxels lit+generated/s", "value": total_vox / (ms / 1e3), "unit": "voxels/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u8",
        "data": "synthetic: fBm terrain 40+round(50*fbm) of the library's own specification (the benchmark names "
                "fBm without its constants), seeds base+env, uniform random RGBA8 frames",
        "config": {"workload": "world reset: generation + full sky/block light + RGBA8->NCHW conversion",
                   "envs_per_gpu": E, "world": [W, H, D], "torches_per_env": T, "frames": [E, 3, FH, FW],
                   "l2": f"outputs {2 * vox_step / 1e9:.2f} GB per step per GPU rewritten every step (> 126 MB L2)",
                   "parallelism": f"env shards x{world}"},
        "env_resets_per_s": E * world * args.steps / (ms / 1e3),
        "roofline": {"bound": "hbm", "kernel": "surface_kernel<4> + tile_kernel<4, 0> over the tiles it left",
                     "achieved": achieved, "peak": peaks["hbm_gbs"],
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                     "algorithmic_bytes_per_launch": algo_bytes, "kernel_ms": tile_ms, "traffic": traffic,
                     "traffic_source": "profiles/generation_reset_traffic.csv (ncu, one full-size generation)"
                     if traffic is not None else None},
        "e2e": {"value": vox_step * world * n_sus / (e2e_ms / 1e3), "unit": "voxels/s", "steps": n_sus,
                "h2d_bytes_per_step": seeds.numel() * 4 + frames.numel(),
                "d2h_bytes_per_step": hm_host[0].numel() * 2},
        "gpu_launches": LAUNCHES["reset"] * args.steps,
        "clocks": clocks,
        "sustained": {"steps": n_sus, "ms_per_step": sus_ms / n_sus,
                      "value": vox_step * world * n_sus / (sus_ms / 1e3), "clocks": sus_clocks},
        "profile": {"generate_prep_ms": prep_ms, "generate_tiles_ms": tile_ms,
                    "fallback_tiles_per_generation": fallback, "tiles_per_generation": E * (W // 32) * (D // 32)},
    }


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


def dirty_voxels(before, after, hm_before, hm_after, origin_y=0):
    """Voxels an exact relight must revisit, summed over envs: the union of the
    prisms (clipped to the world) of every cell whose light class changed
    (opaque / open / torch) and of every cell of the column span its top moved
    over; the prism of a cell is the columns within L1 distance 14 of its
    column times the rows within 14 of it (light falls by one per step, so a
    change reaches no farther). An opaque block replaced by another opaque block changes no
    light, and neither does an air <-> opaque change of a cell that lay below
    its column's top before and after the step and ends it enclosed (six
    opaque neighbours, no torch before or after). Also returns the number of
    cells whose block id changed and the number of light-class changes.
    ids are (envs, D, W, H) tensors, height maps (envs, D, W) in world y."""
    import torch
    import torch.nn.functional as F

    def light_class(ids):  # 0 opaque, 1 air, 2 torch (ids: Air 0, Torch 4)
        return (ids == 0).to(torch.uint8) + 2 * (ids == 4).to(torch.uint8)

    n_changed = int((before != after).sum().item())
    n_light = 0
    total = 0
    H = before.shape[3]
    y = torch.arange(H, device=after.device, dtype=torch.int32)
    for e0 in range(0, before.shape[0], 32):
        b, a = before[e0:e0 + 32], after[e0:e0 + 32]
        tb = (hm_before[e0:e0 + 32].to(torch.int32) - origin_y).unsqueeze(3)
        ta = (hm_after[e0:e0 + 32].to(torch.int32) - origin_y).unsqueeze(3)
        moved = light_class(b) != light_class(a)
        n_light += int(moved.sum().item())
        opaque = ((a != 0) & (a != 4)).to(torch.uint8)
        p = F.pad(opaque, (1, 1, 1, 1, 1, 1), value=1)
        nb = (p[:, :-2, 1:-1, 1:-1] & p[:, 2:, 1:-1, 1:-1] & p[:, 1:-1, :-2, 1:-1] & p[:, 1:-1, 2:, 1:-1]
              & p[:, 1:-1, 1:-1, :-2] & p[:, 1:-1, 1:-1, 2:]).bool()
        enclosed = nb & (y < ta) & (y < tb) & (b != 4) & (a != 4)
        seed = moved & ~enclosed
        # the span of every moved top, in its column
        span = (y > torch.minimum(ta, tb)) & (y <= torch.maximum(ta, tb))
        seed = seed | span
        # rows within 14 (a 29-wide max pool along y), then columns within L1
        # distance 14 (14 steps of a cross-shaped dilation over z and x)
        dil = F.max_pool3d(seed.to(torch.float16), kernel_size=(1, 1, 29), stride=1, padding=(0, 0, 14))
        for _ in range(14):
            dil = torch.maximum(F.max_pool3d(dil, kernel_size=(3, 1, 1), stride=1, padding=(1, 0, 0)),
                                F.max_pool3d(dil, kernel_size=(1, 3, 1), stride=1, padding=(0, 1, 0)))
        total += int((dil > 0).sum().item())
    return total, n_changed, n_light


def relight_record(args, rank, world, local, dev, pg, peaks, peak_kind, standalone):
    import numpy as np
    import torch

    import blocklab_b200 as B

    c = dict(RELIGHT)
    E = (args.envs if standalone and args.envs else c["envs"])
    Wd, Hd, Dd = c["W"], c["H"], c["D"]
    n_edits = c["edits"] * E // RELIGHT["envs"]
    cfg = B.WorldConfig(num_envs=E, width=Wd, height=Hd, depth=Dd, max_overrides=E * c["torches"],
                        max_edits=n_edits)
    wb = B.WorldBatch(cfg, device=local)
    rng = np.random.default_rng(4242 + rank)
    seeds = (BASE_SEED + rank * E + np.arange(E)).astype(np.uint32)
    torches = wb.place_torches(seeds, c["torches"])
    wb.generate(seeds, torches)
    wb.sync()
    hm = wb.height_map.cpu().numpy()
    tl = torches.cpu().numpy().view(B.OVERRIDE_DTYPE).reshape(E, c["torches"])
    txyz = np.stack([tl["x"], tl["y"], tl["z"]], 2)

    def batches(n):
        return [torch.from_numpy(surface_edits(rng, hm, E, n_edits, Wd, Dd, txyz).view(np.uint8).copy()).to(dev)
                for _ in range(n)]

    # Step time from a short run, then as many steps as fill SUSTAINED_S.
    probe = batches(args.warmup + 3)
    ms_probe, _ = time_steps(lambda k: wb.apply_edits(probe[k]), 3, args.warmup, dev, pg, local)
    n = sustained_steps(ms_probe / 3, args.steps, dev, pg)
    dev_batches = batches(args.warmup + n)
    # Dirty volume per step, counted outside the timed region on the same edit
    # sequence: at the first timed step and at the last.
    wb.generate(seeds, torches)
    for k in range(args.warmup):
        wb.apply_edits(dev_batches[k])
    counts = []
    for k in (args.warmup, args.warmup + n - 1):
        if k != args.warmup:
            for j in range(args.warmup + 1, k):
                wb.apply_edits(dev_batches[j])
        before, hb = wb.ids.clone(), wb.height_map.clone()
        wb.apply_edits(dev_batches[k])
        counts.append(dirty_voxels(before, wb.ids, hb, wb.height_map))
        del before, hb
    dirty = sum(cn[0] for cn in counts) / len(counts)
    # Timed run on a fresh copy of the same worlds and edit sequence.
    wb.generate(seeds, torches)
    wb.profile(True)
    ms, clocks = time_steps(lambda k: wb.apply_edits(dev_batches[k]), n, args.warmup, dev, pg, local)
    prof = wb.profile_read()
    wb.profile(False)
    wb.sync()
    relight_ms = prof["relight_ms"] / max(prof["edit_calls"], 1)
    # End to end: each step's edits copied from pinned host memory.
    pinned = [b.cpu().pin_memory() for b in dev_batches]
    stage = torch.empty_like(dev_batches[0])
    wb.generate(seeds, torches)

    def e2e(k):
        stage.copy_(pinned[k], non_blocking=True)
        wb.apply_edits(stage)

    e2e_ms, _ = time_steps(e2e, n, args.warmup, dev, pg, local)
    (relight_ms,) = max_over_ranks([relight_ms], dev, pg)
    env_steps = E * world * n
    algo = 3 * dirty
    achieved = algo / (relight_ms / 1e3) / 1e9
    rec = {
        "metric": "env-steps/s (incremental relight)", "value": env_steps / (ms / 1e3), "unit": "env-steps/s",
        "n_gpus": world, "steps": n, "warmup": args.warmup, "ms_per_step": ms / n, "higher_is_better": True,
        "scaling": "weak", "dtype": "u8",
        "config": {"workload": "relight: edits with World::setBlock semantics + exact incremental relight",
                   "envs_per_gpu": E, "world": [Wd, Hd, Dd], "torches_per_env": c["torches"],
                   "edits_per_step_per_gpu": n_edits, "mix": "45% dig, 45% stone, 5% torch, 5% remove torch, "
                   "within 8 of the surface", "l2": "edits touch scattered regions of a 4.3 GB world",
                   "parallelism": f"env shards x{world}"},
        "roofline": {"bound": "hbm", "kernel": "relight (region kernels + tile path)", "achieved": achieved,
                     "peak": peaks["hbm_gbs"], "peak_kind": peak_kind, "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"], "algorithmic_bytes_per_step": algo,
                     "dirty_voxels_per_step": dirty, "dirty_voxels_first_last": [cn[0] for cn in counts],
                     "changed_cells_per_step": counts[0][1], "light_class_changes_per_step": counts[0][2],
                     "relight_ms": relight_ms, "edits_prep_ms": prof["edits_prep_ms"] / max(prof["edit_calls"], 1),
                     "traffic": None},
        "e2e": {"value": env_steps / (e2e_ms / 1e3), "unit": "env-steps/s",
                "h2d_bytes_per_step": int(dev_batches[0].numel()), "d2h_bytes_per_step": 0},
        "gpu_launches": LAUNCHES["relight"] * n, "clocks": clocks,
    }
    wb.close()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # The reference regenerates and relights the region for every edit
        # (src/graphics/Renderer.cpp:1121-1141): one generation per env-step.
        ref = reference_gpu_record(Wd, Hd, Dd, c["torches"], "env-steps/s", 1,
                                   what="one env of this configuration, regenerated per env-step")
        if ref is not None:
            rec["reference_gpu"] = ref
    return rec


def daynight_record(args, rank, world, local, dev, pg, peaks, peak_kind, standalone):
    import numpy as np
    import torch

    import blocklab_b200 as B

    c = dict(DAYNIGHT)
    E = (args.envs if standalone and args.envs else c["envs"])
    Wd, Hd, Dd, Fr = c["W"], c["H"], c["D"], c["frame"]
    cfg = B.WorldConfig(num_envs=E, width=Wd, height=Hd, depth=Dd, max_overrides=E * c["torches"])
    wb = B.WorldBatch(cfg, device=local)
    seeds = (BASE_SEED + rank * E + np.arange(E)).astype(np.uint32)
    wb.generate(seeds, wb.place_torches(seeds, c["torches"]))
    gen = torch.Generator().manual_seed(99 + rank)
    frames_host = torch.randint(0, 256, (E, Fr, Fr, 4), dtype=torch.uint8, generator=gen).pin_memory()
    frames = frames_host.to(dev)
    obs = torch.empty((E, 3, Fr, Fr), dtype=torch.float32, device=dev)
    eff = torch.empty_like(wb.light) if args.materialize else None
    half = c["steps_per_sweep"] // 2
    # Tick of sweep step k: across the sunset ramp, then the sunrise ramp.
    ticks = [12000 + (13702 - 12000) * k // (half - 1) for k in range(half)] + \
            [22300 + (23961 - 22300) * k // (half - 1) for k in range(half)]
    dims = torch.tensor([[B.sky_light_dimming(t)] * E for t in ticks], dtype=torch.uint8).pin_memory()
    dim_dev = torch.empty(E, dtype=torch.uint8, device=dev)

    def step(k, src=frames):
        dim_dev.copy_(dims[k % len(ticks)], non_blocking=True)
        B.convert_rgba8_to_float_nchw(src, out=obs)
        if eff is not None:
            wb.effective_light(dim_dev, out=eff)

    ms_probe, _ = time_steps(step, 3, args.warmup, dev, pg, local)
    n = sustained_steps(ms_probe / 3, args.steps, dev, pg)
    ms, clocks = time_steps(step, n, args.warmup, dev, pg, local)
    stage = torch.empty_like(frames)

    def e2e(k):
        stage.copy_(frames_host, non_blocking=True)
        step(k, stage)

    ms_probe, _ = time_steps(e2e, 2, 1, dev, pg, local)
    n_e2e = sustained_steps(ms_probe / 2, args.steps, dev, pg)
    e2e_ms, _ = time_steps(e2e, n_e2e, 1, dev, pg, local)
    env_steps = E * world * n
    conv_bytes = 16 * E * Fr * Fr + (2 * wb.light.numel() if eff is not None else 0)
    achieved = conv_bytes * n / (ms / 1e3) / 1e9
    rec = {
        "metric": "env-steps/s (day/night sweep)", "value": env_steps / (ms / 1e3), "unit": "env-steps/s",
        "n_gpus": world, "steps": n, "warmup": args.warmup, "ms_per_step": ms / n, "higher_is_better": True,
        "scaling": "weak", "dtype": "u8 -> f32",
        "config": {"workload": "daynight: sky level by tick (sunset then sunrise ramps), dimming upload, RGBA8 "
                               "84x84 -> float32 NCHW" + (", effective light of every cell" if eff is not None else ""),
                   "envs_per_gpu": E, "world": [Wd, Hd, Dd], "torches_per_env": c["torches"],
                   "frames": [E, 3, Fr, Fr], "l2": f"{conv_bytes / 1e9:.2f} GB moved per step (> 126 MB L2)",
                   "parallelism": f"env shards x{world}"},
        "roofline": {"bound": "hbm", "kernel": "rgba_to_nchw_vec_kernel" + (
            " + effective_light_kernel" if eff is not None else ""), "achieved": achieved,
            "peak": peaks["hbm_gbs"], "peak_kind": peak_kind, "unit": "GB/s",
            "frac": achieved / peaks["hbm_gbs"], "algorithmic_bytes_per_step": conv_bytes, "traffic": None},
        "e2e": {"value": E * world * n_e2e / (e2e_ms / 1e3), "unit": "env-steps/s", "steps": n_e2e,
                "h2d_bytes_per_step": frames.numel() + E, "d2h_bytes_per_step": 0},
        "gpu_launches": (2 if eff is not None else 1) * n, "clocks": clocks,
    }
    wb.close()
    return rec


def scaleout_record(args, rank, world, local, dev, pg, peaks, peak_kind, standalone):
    import numpy as np
    import torch

    import blocklab_b200 as B

    c = dict(SCALEOUT)
    E = (args.envs if standalone and args.envs else c["envs"])
    Wd, Hd, Dd = c["W"], c["H"], c["D"]
    n_edits = max(c["edits_total"] * E // c["envs_total"], 1)
    FH, FW = RESET["frame"]
    cfg = B.WorldConfig(num_envs=E, width=Wd, height=Hd, depth=Dd, amplitude=c["amplitude"],
                        max_overrides=E * c["torches"], max_edits=n_edits)
    wb = B.WorldBatch(cfg, device=local)
    seeds = (BASE_SEED + rank * E + np.arange(E)).astype(np.uint32)
    seeds_dev = torch.from_numpy(seeds.view(np.int32)).to(dev)
    reset_torches = {}

    def reset(_k):
        reset_torches["t"] = wb.place_torches(seeds_dev, c["torches"])
        wb.generate(seeds_dev, reset_torches["t"])

    ms_probe, _ = time_steps(reset, 1, 1, dev, pg, local)
    n_reset = sustained_steps(ms_probe, 1, dev, pg)
    reset_ms, reset_clocks = time_steps(reset, n_reset, 1, dev, pg, local)
    hm = wb.height_map.cpu().numpy()
    tl = reset_torches["t"].cpu().numpy().view(B.OVERRIDE_DTYPE).reshape(E, c["torches"])
    txyz = np.stack([tl["x"], tl["y"], tl["z"]], 2)
    rng = np.random.default_rng(7 + rank)
    gen = torch.Generator().manual_seed(7 + rank)
    frames_host = torch.randint(0, 256, (E, FH, FW, 4), dtype=torch.uint8, generator=gen).pin_memory()
    frames = frames_host.to(dev)
    obs = torch.empty((E, 3, FH, FW), dtype=torch.float32, device=dev)
    gathered = [torch.empty_like(obs) for _ in range(world)] if args.gather and pg is not None and rank == 0 else None

    def make(n):
        return [torch.from_numpy(surface_edits(rng, hm, E, n_edits, Wd, Dd, txyz).view(np.uint8).copy()).to(dev)
                for _ in range(n)]

    probe = make(args.warmup + 3)

    def step_with(batches, src=frames):
        def step(k):
            wb.apply_edits(batches[k])
            B.convert_rgba8_to_float_nchw(src, out=obs)
            if args.gather and pg is not None:
                pg.gather(obs, gathered if rank == 0 else None, dst=0)
        return step

    ms_probe, _ = time_steps(step_with(probe), 3, args.warmup, dev, pg, local)
    n = sustained_steps(ms_probe / 3, args.steps, dev, pg)
    batches = make(args.warmup + n)
    ms, clocks = time_steps(step_with(batches), n, args.warmup, dev, pg, local)
    # End to end: edits and frames copied from pinned host memory every step.
    pinned = [b.cpu().pin_memory() for b in batches]
    stage_e, stage_f = torch.empty_like(batches[0]), torch.empty_like(frames)

    def e2e(k):
        stage_e.copy_(pinned[k], non_blocking=True)
        stage_f.copy_(frames_host, non_blocking=True)
        wb.apply_edits(stage_e)
        B.convert_rgba8_to_float_nchw(stage_f, out=obs)

    ms_probe, _ = time_steps(e2e, 2, 1, dev, pg, local)
    n_e2e = min(sustained_steps(ms_probe / 2, args.steps, dev, pg), n)
    e2e_ms, _ = time_steps(e2e, n_e2e, args.warmup, dev, pg, local)
    env_steps = E * world * n
    vox = E * Wd * Hd * Dd
    reset_step_ms = reset_ms / n_reset
    rec = {
        "metric": "env-steps/s (scale-out)", "value": env_steps / (ms / 1e3), "unit": "env-steps/s",
        "n_gpus": world, "steps": n, "warmup": args.warmup, "ms_per_step": ms / n, "higher_is_better": True,
        "scaling": "weak", "dtype": "u8",
        "config": {"workload": "scaleout: per step edits + exact relight + 90x160 frame conversion"
                               + (" + NCCL gather of observations to rank 0" if args.gather else ""),
                   "envs_per_gpu": E, "world": [Wd, Hd, Dd], "terrain": "fBm 40+round(120*fbm)",
                   "torches_per_env": c["torches"], "edits_per_step_per_gpu": n_edits,
                   "edits_reading": "5,000 edits per step over the whole 8192-env batch (not 5,000 per env)",
                   "l2": f"{2 * vox / 1e9:.1f} GB of world per GPU", "parallelism": f"env shards x{world}"},
        "reset": {"steps": n_reset, "ms": reset_step_ms, "voxels_per_s": vox * world / (reset_step_ms / 1e3),
                  "clocks": reset_clocks},
        "roofline": {"bound": "hbm", "kernel": "reset step (2 B per voxel written)",
                     "achieved": 2 * vox / (reset_step_ms / 1e3) / 1e9, "peak": peaks["hbm_gbs"],
                     "peak_kind": peak_kind, "unit": "GB/s",
                     "frac": 2 * vox / (reset_step_ms / 1e3) / 1e9 / peaks["hbm_gbs"],
                     "algorithmic_bytes_per_reset": 2 * vox, "traffic": None},
        "e2e": {"value": E * world * n_e2e / (e2e_ms / 1e3), "unit": "env-steps/s", "steps": n_e2e,
                "h2d_bytes_per_step": int(batches[0].numel() + frames.numel()), "d2h_bytes_per_step": 0},
        "gpu_launches": LAUNCHES["scaleout"] * n, "clocks": clocks,
    }
    wb.close()
    return rec


def render_record(args, rank, world, local, dev, pg, peaks, peak_kind, standalone):
    import numpy as np
    import torch

    import blocklab_b200 as B
    from blocklab_b200 import _native as N

    E = args.envs or RESET["envs"]
    W, H, D, T = RESET["W"], RESET["H"], RESET["D"], RESET["torches"]
    FH, FW = RESET["frame"]
    wb = B.WorldBatch(B.WorldConfig(num_envs=E, width=W, height=H, depth=D, max_overrides=E * T), device=local)
    seeds = (BASE_SEED + rank * E + np.arange(E)).astype(np.uint32)
    wb.generate(seeds, wb.place_torches(seeds, T))
    hm = wb.height_map.cpu().numpy()
    # Agents at the world centre on the surface, looking around, at several day times.
    params = np.array([B.render_params_at((W / 2, hm[e, D // 2, W // 2] + 1, D / 2), 0.7 * e, -0.25,
                                          (6000 + 997 * e) % 24000) for e in range(E)], B.RENDER_PARAMS_DTYPE)
    params_dev = torch.from_numpy(params.view(np.uint8).copy()).to(dev)
    frames = torch.empty((E, FH, FW, 4), dtype=torch.uint8, device=dev)
    obs = torch.empty((E, 3, FH, FW), dtype=torch.float32, device=dev)

    def step(_k):
        # Frames rendered straight into the observation tensor (RGBA8 kept too).
        N.check(N.lib.blk_render_observations(wb._ctx, params_dev.data_ptr(), FW, FH, obs.data_ptr(),
                                              frames.data_ptr(), torch.cuda.current_stream(dev).cuda_stream))

    ms_probe, _ = time_steps(step, 3, args.warmup, dev, pg, local)
    n = sustained_steps(ms_probe / 3, args.steps, dev, pg)
    ms, clocks = time_steps(step, n, args.warmup, dev, pg, local)
    wb.close()
    return {"metric": "frames/s (render to observations)", "value": E * world * n / (ms / 1e3), "unit": "frames/s",
            "n_gpus": world, "steps": n, "warmup": args.warmup, "ms_per_step": ms / n, "higher_is_better": True,
            "scaling": "weak", "dtype": "u8 -> f32",
            "config": {"workload": "render: ray-cast 160x90 frames of the reset worlds into RGBA8 and float NCHW",
                       "envs_per_gpu": E, "world": [W, H, D], "frames": [E, 3, FH, FW],
                       "parallelism": f"env shards x{world}"},
            "gpu_launches": LAUNCHES["render"] * n, "clocks": clocks}


RECORDS = {"relight": relight_record, "daynight": daynight_record, "scaleout": scaleout_record,
           "render": render_record}


def run_ours(args) -> None:
    rank, world, local, dev, pg = init_dist()
    peaks, peak_kind = measured_peaks()
    common = (args, rank, world, local, dev, pg, peaks, peak_kind)
    if args.workload == "reset":
        line = reset_record(*common)
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            times, vox, cores, desc = reference_cpu_times(1)
            line["cpu_baseline"] = {"value": vox / times[-1], "unit": "voxels/s", "cores": cores,
                                    "kind": "reference", "sample": desc}
            ref = reference_gpu_record(RESET["W"], RESET["H"], RESET["D"], RESET["torches"], "voxels/s",
                                       RESET["W"] * RESET["H"] * RESET["D"])
            if ref is not None:
                line["reference_gpu"] = ref
        if not args.no_configs:
            line["configs"] = {name: RECORDS[name](*common, False) for name in ("relight", "daynight", "scaleout")}
    else:
        line = {"n_gpus": world, "vs_baseline": None, "data": "synthetic"}
        line.update(RECORDS[args.workload](*common, True))
    if rank == 0:
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()


# ------------------------------------------------------------ reference --
def run_reference(args) -> None:
    """The reference's own CPU implementation of the path on the box's host
    cores: `--warmup` + `--steps` consecutive generations of the bounded
    sample of the reset world (one generator, converged first). Rank 0 only."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    if args.workload != "reset":
        print(json.dumps({"impl": "reference", "workload": args.workload,
                          "unavailable": "the reference arm is timed on the reset workload, the metric's "
                                         "configuration; per-configuration reference figures are the "
                                         "reference_gpu records of the default line"}), flush=True)
        return
    from oracle.oracle import ref_available

    if not ref_available("cpu"):
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libref_cpu.so not built"}), flush=True)
        return
    times, vox, cores, desc = reference_cpu_times(args.warmup + args.steps)
    timed = times[args.warmup:]
    total = sum(timed)
    value = vox * len(timed) / total
    cfg = {"workload": "world reset: generation + full sky/block light (bounded sample of the reset world)",
           "world": [SAMPLE["W"], SAMPLE["H"], SAMPLE["D"]], "sample_of": [RESET["W"], RESET["H"], RESET["D"]],
           "envs_per_step": 1, "terrain": "fBm 40+round(50*fbm) as a dense override list",
           "parallelism": "host threads"}
    print(json.dumps({
        "impl": "reference", "metric": "voxels lit+generated/s", "value": value, "unit": "voxels/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / len(timed),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": cfg,
        "cpu_baseline": {"value": value, "unit": "voxels/s", "cores": cores, "kind": "reference", "sample": desc},
        "e2e": {"value": value, "unit": "voxels/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
        flush=True)


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
