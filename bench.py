#!/usr/bin/env python
"""Benchmark of the B200 Gaussian-splatting renderer.

One step = one frame of the hot path (projection, binning, sort, bin ranges, splatting) of
the 1,000,000-Gaussian SH3 scene at 1920x1080 with 16x16-pixel bins. Rank r renders, at step
s, view (s * N + r) mod 64 of a 64-view orbit (radius 1.5, elevations -30..30 degrees, 60
degree FOV): one view per GPU with the scene replicated, no data-path collective (weak
scaling). Inputs are larger than L2: 240 MB of scene planes and ~390 MB of key buffers per
frame, so no L2 flush is needed between frames.

Frames are kept in flight as klartraum's engine keeps its paths: frame s renders on path
s mod 3 with its own stream, so consecutive frames overlap on the GPU. A timed window is
exactly `--steps` frames between a barrier + synchronize on both sides (CUDA events, max over
ranks); windows repeat until about a second of device time has passed and the median window
gives `value` and `ms_per_step`. `e2e` is the same through kt_gs_render_host_clear (camera up,
image cleared on the device as the reference's render pass clears it, frame copied to pinned
host memory); `e2e.image_in` copies a host image in as well (kt_gs_render_host).

The same line also carries, measured the same way at the same N:
  multiview_3m   the 3,000,000-Gaussian SH3 scene over the 64-view orbit at 1920x1080 (weak)
  bands_6m       the 6,000,000-Gaussian SH3 4K frame split into bin-row bands, one per rank,
                 balanced on measured time, strips all-gathered over NCCL every step (strong)

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python bench.py --workload stress_2m --paths 1          # another scene as the main workload
    python bench.py --mode bands [--workload large_6m]      # the banded frame as the main line

``--launch`` (default graph) replays each frame as a captured CUDA graph; ``--sorted-keys`` bins
through the reference-structured path. ``--impl reference`` times the CPU restatement of the
reference algorithm (the oracle, C + OpenMP on all host cores) on the same workload; under
torchrun only rank 0 runs it. Prints one JSON line (rank 0).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "frames/s and Gaussians/s, 1M-splat SH3 1080p; multi-view fps at 1/2/4/8 B200"
WORKLOAD = "single_1m"
N_VIEWS = 64
PATHS = 3  # frames in flight, each on its own path and stream, as klartraum's engine (3 paths)


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--paths", type=int, default=PATHS,
                   help="frames in flight, each on its own path and stream (default 3, as klartraum's engine)")
    p.add_argument("--e2e-steps", type=int, default=None, help="steps of a host-buffer window (default: steps)")
    p.add_argument("--min-window-ms", type=float, default=1000.0,
                   help="repeat the timed window of `steps` frames until this much device time has passed")
    p.add_argument("--no-multiview", dest="multiview", action="store_false",
                   help="skip the 3M-Gaussian multi-view batch measured after the main workload")
    p.add_argument("--no-bands", dest="bands", action="store_false",
                   help="skip the 6M-Gaussian 4K frame split into bands measured after the main workload")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--small", action="store_true", help="tiny frame for profiler captures")
    p.add_argument("--mode", choices=["views", "bands"], default="views",
                   help="views: one view per GPU per step (default); bands: one frame split into bin-row bands "
                        "over the GPUs, strips all-gathered every step")
    p.add_argument("--launch", choices=["graph", "stream"], default="graph",
                   help="graph (default): each path's frame is captured once as a CUDA graph and replayed with new "
                        "cameras (KT_GS_FLAG_GRAPH), as the reference re-submits recorded command buffers; stage "
                        "times then come from a separate stream-launched pass. stream: every kernel launched per frame")
    p.add_argument("--sorted-keys", action="store_true",
                   help="bin through the reference-structured path (scan, key emission, radix sort of the "
                        "pairs, boundary search) instead of placing the pairs in bin order")
    p.add_argument("--workload", default=None, help="scene of scenes.WORKLOADS (default: single_1m for views, "
                                                    "large_6m for bands)")
    p.add_argument("--n", type=int, default=None,
                   help="Gaussians drawn from the workload's distributions instead of its full count (reduced cases "
                        "for profiler captures)")
    return p.parse_args()


def workload_config(w) -> dict:
    return {
        "workload": f"{w.name}: {w.n:,} Gaussians SH{w.sh_degree} {w.width}x{w.height}, 16x16-px bins, "
                    f"{N_VIEWS}-view orbit r={w.distance} elev -30..30 deg, {w.fovy_deg:.0f} deg FOV",
        "n_gaussians": w.n, "sh_degree": w.sh_degree, "width": w.width, "height": w.height, "bin_px": 16,
        "views": N_VIEWS, "parallelism": "multi-view: one view per GPU per step, scene replicated",
        "l2": "inputs larger than L2 (scene planes 240 MB, key buffers ~390 MB per frame); no flush",
        "seed": w.seed,
    }


# ----------------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clock / throttle-reason samples of one GPU while running."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.samples: list[tuple[float, list[str]]] = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-i", str(self.index), "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.time(), [x.strip() for x in line.split(",")]))

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)

    def summary(self, t0: float, t1: float) -> dict:
        inside = [s for t, s in self.samples if t0 <= t <= t1]
        note = None
        if not inside and self.samples:
            # the timed window was shorter than the sampling period: nearest samples
            mid = 0.5 * (t0 + t1)
            inside = [min(self.samples, key=lambda ts: abs(ts[0] - mid))[1]]
            note = "timed window shorter than the 100 ms sampling period; nearest sample"
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [num(s[1]) for s in inside if num(s[1]) is not None]
        smax = [num(s[2]) for s in inside if num(s[2]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in inside for i in range(4) if len(s) > 5 + i and s[5 + i] == "Active"})
        out = {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
               "reasons": reasons, "samples": len(inside)}
        if note:
            out["note"] = note
        return out


# --------------------------------------------------------------- reference arm

def run_reference(args, w, cfg_block):
    """Time the CPU restatement of the reference algorithm (oracle) on the same workload."""
    import oracle
    from klartraum_b200 import make_scene, orbit_views

    g3d = make_scene(w)
    cams = orbit_views(N_VIEWS, w.distance, w.width, w.height, fovy_deg=w.fovy_deg)
    cfg = oracle.config(w.width, w.height, bin_size=16, sh_degree=w.sh_degree)
    bg = np.zeros((w.height, w.width, 4), np.uint8)
    bg[..., 3] = 255
    # all host cores: launchers such as torchrun set OMP_NUM_THREADS=1 for their ranks
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    oracle.set_threads(threads)
    threads = oracle.lib().ko_get_threads()
    for s in range(args.warmup):
        oracle.render_frame_fast(cfg, cams[s % N_VIEWS], g3d, bg)
    t0 = time.perf_counter()
    for s in range(args.steps):
        oracle.render_frame_fast(cfg, cams[s % N_VIEWS], g3d, bg)
    dt = time.perf_counter() - t0
    fps = args.steps / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": fps, "unit": "frames/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * dt / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": cfg_block, "gaussians_per_s": fps * w.n,
        "cpu_baseline": {"value": fps, "unit": "frames/s", "cores": threads, "kind": "port",
                         "sample": f"{args.steps} full frames of the workload on the host CPU: the C "
                                   f"restatement of the reference shaders (oracle/kt_oracle.c), OpenMP"},
        "e2e": {"value": fps, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference's own path is Vulkan GLSL; no graphics stack exists on this machine, "
                "so its CPU restatement is timed",
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------- our arm

# DRAM bytes (read + write) per launch of a stage's kernel, from the ncu captures summarised in
# profiles/ (1M SH3 1080p workload): profiles/k_project_count_single_1m.md.
NCU_TRAFFIC = {"single_1m": {"project_count": 240.03e6 + 46.08e6}}
# stages whose time is set by HBM traffic (the others: dependency chains or instruction issue)
HBM_BOUND = ("project_count",)


def stage_report(w, cnt, st, stage_ms, timed_frames, nplanes, stage_names=None):
    """Per-stage time, algorithmic bytes and HBM fraction over a timed region, and the roofline
    entry of the dominant HBM-bound stage."""
    from klartraum_b200 import native as N

    stage_names = stage_names or N.STAGE_NAMES

    peak, peak_kind = load_peaks()
    frames = max(timed_frames, 1)
    K_avg = cnt["keys"] / max(cnt["frames"], 1)
    passes_avg = cnt["key_passes"] / max(cnt["keys"], 1)
    nf = max(cnt["frames"], 1)
    tiles = st["tiles_x"] * st["tiles_y"]
    ncoarse = ((st["tiles_x"] + 3) // 4) * ((st["tiles_y"] + 3) // 4)
    table = st["place_chunks"] * ncoarse * 4  # entries per (chunk, coarse bin), u32
    # bytes the placement writes: 8 per (Gaussian, coarse bin) entry, 4 per pair
    placed = cnt["sort_bytes"] / nf
    entries = max(placed - 4 * K_avg, 0.0) / 8
    per_frame_bytes = {
        # geometry and SH planes read; record 48 + count 4 + rect 8 + depth 4 written
        "project_count": w.n * (16 * 3 + 64 + 16 * nplanes),
        # depth keys (counts + depths read, 8-B keys written) and the depth sort passes (16 B per
        # Gaussian per pass)
        "depth_sort": w.n * (4 + 4 + 8) + cnt["depth_sort_bytes"] / nf,
        # rectangles gathered into depth order (order, count, rectangle read; 8 B written); the
        # (chunk, coarse bin) table written, read and rewritten as its prefix over chunks
        "coarse_count": w.n * (8 + 4 + 8 + 8) + 3 * table + ncoarse * 16,
        # depth order and rectangle per Gaussian and the table read; 8 B per entry written
        "coarse_place": w.n * (8 + 8) + table + ncoarse * 16 + entries * 8,
        # entries read twice (count, place); 4 B per pair written; bin ranges
        "fine_place": entries * 8 * 2 + K_avg * 4 + tiles * 16,
        # reference-structured path: counts, rectangles and depths read, offsets written; 12 B
        # (key + value) per pair written
        "scan_emit": w.n * (4 + 8 + 4 + 8) + K_avg * 12,
        # executed passes of the pair sort: 24 B per pair and pass
        "key_sort": cnt["sort_bytes"] / nf,
    }
    if stage_names is not N.STAGE_NAMES:
        per_frame_bytes["bin_ranges"] = K_avg * 8 + tiles * 8  # boundary search over the sorted keys
    stages = {}
    for name in stage_names[:-1]:
        avg = stage_ms[name] / frames
        d = {"ms": avg, "share": stage_ms[name] / max(stage_ms["frame"], 1e-12)}
        if name in per_frame_bytes:
            gbs = per_frame_bytes[name] / (avg / 1000.0) / 1e9 if avg > 0 else 0.0
            d.update({"bytes": per_frame_bytes[name], "gbs": gbs, "frac": gbs / peak})
        stages[name] = d
    dominant = max(stages, key=lambda k: stages[k]["ms"])
    dom = stages[dominant]
    if dominant in HBM_BOUND:
        roofline = {"kernel": dominant, "bound": "hbm", "achieved": dom["gbs"], "peak": peak, "unit": "GB/s",
                    "frac": dom["frac"], "traffic": NCU_TRAFFIC.get(w.name, {}).get(dominant),
                    "peak_source": peak_kind, "bytes_per_launch": dom["bytes"]}
    else:
        hb = max((k for k in stages if k in HBM_BOUND), key=lambda k: stages[k]["ms"])
        roofline = {"kernel": hb, "bound": "hbm", "achieved": stages[hb]["gbs"], "peak": peak, "unit": "GB/s",
                    "frac": stages[hb]["frac"], "traffic": NCU_TRAFFIC.get(w.name, {}).get(hb),
                    "peak_source": peak_kind,
                    "bytes_per_launch": stages[hb]["bytes"],
                    "note": (f"{dominant} takes the most time and is bound by "
                             + ("FP32/MUFU issue (per (pixel, Gaussian) evaluation, not by bytes; ncu issue "
                                "fraction in profiles/)" if dominant == "rasterize" else "its dependency chain")
                             + "; this entry is the HBM-bound stage")}
    return stages, roofline, K_avg, passes_avg


def load_peaks() -> tuple[float, str]:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def timed_windows(window, world, dev, dist, local_rank, min_ms=1000.0, min_windows=5, max_windows=2000):
    """Repeat a timed window of exactly `steps` frames until about `min_ms` of device time has
    passed. `window()` enqueues one window and returns its (start, end) CUDA events. Every
    window is bracketed by a barrier and a device synchronize; the window count is fixed from a
    first window timed as the max over ranks, so every rank runs the same collectives. Returns the
    per-window milliseconds (each the max over ranks) and the wall-clock span of all windows."""
    import torch

    def one():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()
        e0, e1 = window()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1)

    def max_over_ranks(vals):
        t = torch.tensor(vals, dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()

    first = max_over_ranks([one()])[0]
    count = int(min(max(math.ceil(min_ms / max(first, 1e-3)), min_windows), max_windows))
    t0 = time.time()
    ms = [one() for _ in range(count)]
    t1 = time.time()
    if world > 1:
        dist.barrier(device_ids=[local_rank])
    return max_over_ranks(ms), (t0, t1)


def window_stats(ms: list, steps: int) -> dict:
    """Median and spread of per-window times."""
    q = sorted(ms)
    med = statistics.median(q)
    return {"windows": len(q), "ms_per_window_median": med, "ms_per_step_median": med / steps,
            "ms_per_window_min": q[0], "ms_per_window_max": q[-1],
            "spread_pct": 100.0 * (q[-1] - q[0]) / med if med > 0 else 0.0,
            "iqr_pct": 100.0 * (q[(3 * len(q)) // 4] - q[len(q) // 4]) / med if med > 0 else 0.0,
            "device_ms_total": sum(q)}


def measure_views(args, w, rank, world, local_rank, dev, dist, cams, scene, stage_pass=True) -> dict:
    """Frames/s of the multi-view protocol on one workload: rank r renders view (s * N + r) mod 64
    at step s, `paths` frames in flight on their own paths and streams. Device-resident windows of
    exactly `steps` frames are repeated for about a second (median reported); then the same
    through kt_gs_render_host with pinned host images (e2e). `scene` is host records or a
    (device pointer, count) pair from the broadcast."""
    import torch

    from klartraum_b200 import Renderer, native as N

    paths = max(1, args.paths)

    def view_of(s):
        return (s * world + rank) % N_VIEWS

    base_flags = N.FLAG_SORTED_KEYS if args.sorted_keys else 0
    r = Renderer(w.width, w.height, bin_size=16, sh_degree=w.sh_degree, device=local_rank,
                 flags=N.FLAG_TIMING | base_flags, num_paths=paths)
    if isinstance(scene, tuple):
        r.set_gaussians_device(*scene)
        torch.cuda.synchronize()
    else:
        r.set_gaussians(scene)
    nplanes = (3 * (w.sh_degree + 1) ** 2 + 3) // 4
    bg = torch.zeros((w.height, w.width, 4), dtype=torch.uint8, device=dev)
    bg[..., 3] = 255
    img = bg.clone()
    sptr = torch.cuda.current_stream(dev).cuda_stream

    e2e_steps = args.e2e_steps or args.steps
    # warm-up: checked frames over every view each path renders (sizes its buffers; frames in
    # flight are async and cannot grow them)
    views = sorted({view_of(s) for s in range(max(args.steps, e2e_steps + 2 * paths, args.warmup))})
    for s in range(max(args.warmup, 3)):
        r.render(cams[view_of(s)], img, stream=sptr)
    for p in range(paths):
        for v in views:
            r.render(cams[v], img, path=p, stream=sptr)
    torch.cuda.synchronize()
    r.stage_times_total()
    for p in range(paths):
        r.counters(p)
    stage_ms, timed_frames = {}, 0
    if stage_pass:
        # stage times: a stream-launched pass on one path, frames back to back (graph replays
        # record no stage timers, and frames in flight would overlap the stages of different frames)
        r.set_flags(N.FLAG_TIMING | N.FLAG_ASYNC | base_flags)
        for s in range(min(max(args.steps, 50), 200)):
            r.render(cams[view_of(s)], img, stream=sptr)
        r.sync()
        stage_ms, timed_frames = r.stage_times_total()
        r.counters()
    graph = args.launch == "graph"
    run_flags = (N.FLAG_GRAPH if graph else 0) | N.FLAG_ASYNC | base_flags
    streams = [torch.cuda.Stream(dev) for _ in range(paths)]
    imgs = [img] + [bg.clone() for _ in range(paths - 1)]
    if graph:  # one capture per path, outside the timed region
        r.set_flags(N.FLAG_GRAPH | base_flags)
        for p in range(paths):
            r.render(cams[view_of(p)], imgs[p], path=p, stream=streams[p].cuda_stream)
        torch.cuda.synchronize()
        for p in range(paths):
            r.counters(p)

    def join_streams():
        for strm in streams[1:]:
            ev = torch.cuda.Event()
            ev.record(strm)
            streams[0].wait_event(ev)

    # ---- device-resident windows: `paths` frames in flight, frame s on path s % paths and its
    # stream, no host sync inside a window
    r.set_flags(run_flags)

    def window():
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(streams[0])
        for strm in streams[1:]:
            strm.wait_event(ev0)
        for s in range(args.steps):
            p = s % paths
            r.render(cams[view_of(s)], imgs[p], path=p, stream=streams[p].cuda_stream)
        join_streams()
        ev1.record(streams[0])
        return ev0, ev1

    clock = ClockSampler(local_rank)
    clock.start()
    time.sleep(0.3)
    ms_list, (tw0, tw1) = timed_windows(window, world, dev, dist, local_rank, args.min_window_ms)
    clocks = clock.summary(tw0, tw1)
    for p in range(paths):
        r.sync(p)  # raises if any timed frame overflowed or timed out
    cnt = {}
    for p in range(paths):
        for k, v in r.counters(p).items():
            cnt[k] = cnt.get(k, 0) + v
    wins = window_stats(ms_list, args.steps)
    assert cnt["frames"] == args.steps * (wins["windows"] + 1), cnt
    st = r.stats()
    ms_step = wins["ms_per_step_median"]
    fps = world / (ms_step / 1000.0)

    stages = roofline = None
    K_avg = cnt["keys"] / max(cnt["frames"], 1)
    passes_avg = cnt["key_passes"] / max(cnt["keys"], 1)
    if stage_pass:
        stages, roofline, _, _ = stage_report(w, cnt, st, stage_ms, timed_frames, nplanes, r.stage_names)

    # ---- end to end through the public API with host buffers: paths frames in flight
    # (klartraum's paths), each path on its own stream; a path's host image is reused only after
    # kt_gs_sync(path) says its previous frame, copies included, is done
    hosts = [torch.empty((w.height, w.width, 4), dtype=torch.uint8, pin_memory=True) for _ in range(paths)]
    for h in hosts:
        h.copy_(bg.cpu())
    r.set_flags(run_flags)

    def frame_host(s, first_of_window, clear):
        p = s % paths
        if not first_of_window or s >= paths:
            r.sync(p)
        if clear:  # the render pass's clear colour, set on the device; only the camera goes up
            r.render_host_clear(cams[view_of(s)], hosts[p].data_ptr(), clear=(0, 0, 0, 255), path=p,
                                stream=streams[p].cuda_stream)
        else:  # the host image copied in, blended into, copied out
            r.render_host(cams[view_of(s)], hosts[p].data_ptr(), path=p, stream=streams[p].cuda_stream)

    def e2e_pass(clear):
        for s in range(2 * paths):
            frame_host(s, False, clear)
        for p in range(paths):
            r.sync(p)

        def window_host():
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(streams[0])
            for strm in streams[1:]:
                strm.wait_event(e0)
            for s in range(e2e_steps):
                frame_host(s, True, clear)
            for p in range(paths):
                r.sync(p)
            join_streams()
            e1.record(streams[0])
            return e0, e1

        ems, _ = timed_windows(window_host, world, dev, dist, local_rank, args.min_window_ms)
        return window_stats(ems, e2e_steps)

    ewins = e2e_pass(True)
    iwins = e2e_pass(False)
    clock.stop()
    e2e_fps = world / (ewins["ms_per_step_median"] / 1000.0)
    img_bytes = w.width * w.height * 4
    view0 = None
    if rank == 0:
        # the image of view 0, for the divergence check of the CPU baseline
        r.set_flags(base_flags)
        img0 = bg.clone()
        r.render(cams[0], img0, stream=sptr)
        torch.cuda.synchronize()
        view0 = img0.cpu().numpy()
    out = {
        "value": fps, "ms_per_step": ms_step, "windows": wins, "st": st, "K_avg": K_avg, "passes_avg": passes_avg,
        "stages": stages, "roofline": roofline, "clocks": clocks, "view0": view0,
        "e2e": {"value": e2e_fps, "unit": "frames/s", "h2d_bytes_per_step": 192,
                "d2h_bytes_per_step": img_bytes + st["status_bytes"], "steps": e2e_steps, "windows": ewins,
                "api": f"kt_gs_render_host_clear (camera from host, image cleared to (0,0,0,1) on the device as "
                       f"the reference's render pass clears it, rendered image copied to pinned host memory) "
                       f"with {paths} frames in flight on their own paths and streams; kt_gs_sync(path) before a "
                       "host image is reused",
                "image_in": {"value": world / (iwins["ms_per_step_median"] / 1000.0), "unit": "frames/s",
                             "h2d_bytes_per_step": img_bytes + 192,
                             "d2h_bytes_per_step": img_bytes + st["status_bytes"], "windows": iwins,
                             "api": "kt_gs_render_host: the host image copied in, blended into, copied out"}},
        "gpu_launches": st["launches"] * args.steps * world * wins["windows"],
    }
    r.close()
    return out


def run_ours(args, w, cfg_block, rank, world, local_rank):
    import datetime

    import torch
    import torch.distributed as dist

    from klartraum_b200 import make_scene, orbit_views
    from klartraum_b200.scenes import WORKLOADS

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    if args.small:
        w = type(w)(**{**w.__dict__, "n": 20000, "width": 640, "height": 360})

    def scene_of(wl):
        if world > 1:
            # the scene is made once (rank 0) and broadcast over NCCL; records land in device memory
            from klartraum_b200.multigpu import broadcast_scene

            scene_dev, n_rec = broadcast_scene(make_scene(wl) if rank == 0 else None, dist, rank, dev)
            torch.cuda.synchronize()
            return scene_dev, (scene_dev.data_ptr(), n_rec)
        return None, make_scene(wl)

    cams = orbit_views(N_VIEWS, w.distance, w.width, w.height, fovy_deg=w.fovy_deg)
    keep, scene = scene_of(w)
    m = measure_views(args, w, rank, world, local_rank, dev, dist, cams, scene)
    del keep, scene
    torch.cuda.synchronize()

    # the multi-view batch workload (3M SH3, 64 views), measured the same way at every N
    mv = None
    if args.multiview and not args.small and w.name != "multiview_3m":
        wm = WORKLOADS["multiview_3m"]
        cams_m = orbit_views(N_VIEWS, wm.distance, wm.width, wm.height, fovy_deg=wm.fovy_deg)
        keep, scene = scene_of(wm)
        mm = measure_views(args, wm, rank, world, local_rank, dev, dist, cams_m, scene, stage_pass=False)
        del keep, scene
        mv = {"workload": workload_config(wm)["workload"], "value": mm["value"], "unit": "frames/s",
              "gaussians_per_s": mm["value"] * wm.n, "ms_per_step": mm["ms_per_step"], "steps": args.steps,
              "windows": mm["windows"], "keys_per_frame": mm["K_avg"], "e2e": mm["e2e"], "clocks": mm["clocks"],
              "scaling": "weak", "n_gpus": world}

    # the 6M-Gaussian 4K frame split into bin-row bands over the ranks (strong scaling), at every N
    bd = None
    if args.bands and not args.small:
        wb = WORKLOADS["large_6m"]
        cams_b = orbit_views(N_VIEWS, wb.distance, wb.width, wb.height, fovy_deg=wb.fovy_deg)
        keep, scene = scene_of(wb)
        mb = measure_bands(args, wb, rank, world, local_rank, dev, dist, cams_b, scene)
        del keep, scene
        bd = {"workload": f"{wb.name}: {wb.n:,} Gaussians SH{wb.sh_degree} {wb.width}x{wb.height}, one frame per "
                          f"step split into {world} bin-row bands (time-balanced), strips all-gathered over NCCL",
              "value": mb["value"], "unit": "frames/s", "gaussians_per_s": mb["value"] * wb.n,
              "ms_per_step": mb["ms_per_step"], "steps": args.steps, "windows": mb["windows"], "scaling": "strong",
              "n_gpus": world, "bands": mb["bands"], "band_frame_ms": mb["band_frame_ms"],
              "band_history": mb["band_history"], "gather_bytes_per_step": mb["gather_bytes_per_step"],
              "stages_rank0": mb["stages_rank0"], "e2e": mb["e2e"], "clocks": mb["clocks"]}

    st = m["st"]
    launches_per_frame = st["launches"]
    line = {
        "metric": METRIC, "value": m["value"], "unit": "frames/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": m["ms_per_step"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": cfg_block,
        "gaussians_per_s": m["value"] * w.n, "keys_per_frame": m["K_avg"], "sort_passes_per_frame": m["passes_avg"],
        "timing": {"protocol": f"windows of exactly {args.steps} frames repeated for >= {args.min_window_ms:.0f} ms "
                               "of device time, each bracketed by barrier + synchronize and timed with CUDA events "
                               "(max over ranks); value and ms_per_step from the median window",
                   **m["windows"]},
        "sort_layout": ("reference-structured: index-order scan, (bin << depth_bits | depth, index) pairs, "
                        "LSD radix sort of the pairs, boundary search" if args.sorted_keys else
                        "Gaussians radix-sorted by depth; pairs placed in bin order by a two-level counting sort "
                        "(coarse lists of 4x4 bins filled by chunk of depth order, then bins of each coarse list by "
                        "segment); a pair is stored as its u32 Gaussian index"),
        "stages": m["stages"], "roofline": m["roofline"],
        "e2e": m["e2e"],
        "gpu_launches": launches_per_frame * args.steps * world, "gpu_launches_per_step": launches_per_frame,
        "gpu_launches_all_windows": m["gpu_launches"],
        "clocks": m["clocks"],
    }
    if mv is not None:
        line["multiview_3m"] = mv
    if bd is not None:
        line["bands_6m"] = bd
    if world == 1 and rank == 0 and not args.no_cpu_baseline and not args.small:
        line["cpu_baseline"] = cpu_baseline(w, cams, m["view0"])
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def measure_bands(args, w, rank, world, local_rank, dev, dist, cams, scene) -> dict:
    """One frame split into bin-row bands over the ranks (strong scaling). Every rank projects
    the whole scene but sorts, places and draws only the Gaussians that meet its band; the strips
    are all-gathered over NCCL every step, so every rank ends the step holding the full frame.

    Bands start balanced on the pairs per bin row of view 0 (each rank's rows summed with one
    all_reduce) and are then rebalanced twice on measured time: every rank times its own band's
    frames (CUDA events, no gather), the times are all-gathered, and each band's rows are weighted
    by its measured time per pair, so the cuts follow time rather than pair counts."""
    import torch

    from klartraum_b200 import Renderer, native as N
    from klartraum_b200.multigpu import StripGather, band_pixel_rows, band_rows, rebalance_bands, row_pair_counts

    tx, ty = (w.width + 15) // 16, (w.height + 15) // 16
    base_flags = N.FLAG_SORTED_KEYS if args.sorted_keys else 0

    def renderer(band):
        r = Renderer(w.width, w.height, bin_size=16, sh_degree=w.sh_degree, device=local_rank,
                     flags=N.FLAG_TIMING | base_flags, tile_rows=band)
        if isinstance(scene, tuple):
            r.set_gaussians_device(*scene)
            torch.cuda.synchronize()
        else:
            r.set_gaussians(scene)
        return r

    bg = torch.zeros((w.height, w.width, 4), dtype=torch.uint8, device=dev)
    bg[..., 3] = 255
    img = bg.clone()
    stream = torch.cuda.current_stream(dev)
    sptr = stream.cuda_stream

    def all_ranks(vals):
        t = torch.tensor(vals, dtype=torch.float64, device=dev)
        if world > 1:
            out = torch.empty((world, len(vals)), dtype=torch.float64, device=dev)
            dist.all_gather_into_tensor(out, t)
            return out.cpu().numpy()
        return t.cpu().numpy()[None, :]

    # pairs per bin row of view 0 (equal bands, summed over the ranks)
    bands = band_rows(ty, world)
    r = renderer(bands[rank])
    r.render(cams[0], img, stream=sptr)
    torch.cuda.synchronize()
    rows = torch.from_numpy(row_pair_counts(r.dump(N.STAGE_TILE_RANGES), tx, ty).astype(np.float64)).to(dev)
    r.close()
    if world > 1:
        dist.all_reduce(rows)
    rows = rows.cpu().numpy() + 1.0
    bands = band_rows(ty, world, rows)
    history = [{"bands": bands}]
    calib = 24
    for it in range(2 if world > 1 else 0):
        r = renderer(bands[rank])
        for v in range(calib):  # checked frames size the buffers
            r.render(cams[v % N_VIEWS], img, stream=sptr)
        torch.cuda.synchronize()
        r.set_flags(base_flags | N.FLAG_ASYNC)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for v in range(calib):
            r.render(cams[v % N_VIEWS], img, stream=sptr)
        e1.record(stream)
        torch.cuda.synchronize()
        r.sync()
        r.close()
        t = all_ranks([e0.elapsed_time(e1) / calib])[:, 0]
        history[-1]["ms_per_band"] = [float(x) for x in t]
        bands = rebalance_bands(rows, bands, t)
        history.append({"bands": bands})
    r = renderer(bands[rank])
    px = [band_pixel_rows(b, 16, w.height) for b in bands]
    gather = StripGather(px, w.width, w.height, dist, rank, dev) if world > 1 else (lambda x: x)

    def frame(s):
        img.copy_(bg)
        r.render(cams[s % N_VIEWS], img, stream=sptr)
        return gather(img)

    for s in range(max(args.warmup, 3)):
        frame(s)
    for v in sorted({s % N_VIEWS for s in range(max(args.steps, 64))}):
        r.render(cams[v], img, stream=sptr)  # checked frames size the key buffers for every view
    torch.cuda.synchronize()
    r.stage_times_total()
    r.counters()

    r.set_flags(N.FLAG_TIMING | N.FLAG_ASYNC | base_flags)
    clock = ClockSampler(local_rank)
    clock.start()
    time.sleep(0.3)

    def window():
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for s in range(args.steps):
            frame(s)
        ev1.record(stream)
        return ev0, ev1

    ms_list, (tw0, tw1) = timed_windows(window, world, dev, dist, local_rank, args.min_window_ms)
    r.sync()
    clocks = clock.summary(tw0, tw1)
    wins = window_stats(ms_list, args.steps)
    ms_step = wins["ms_per_step_median"]
    stage_ms, timed_frames = r.stage_times_total()
    cnt = r.counters()
    st = r.stats()
    nplanes = (3 * (w.sh_degree + 1) ** 2 + 3) // 4
    stages, roofline, K_avg, passes_avg = stage_report(w, cnt, st, stage_ms, timed_frames, nplanes, r.stage_names)
    band_ms = all_ranks([stage_ms["frame"] / max(timed_frames, 1)])[:, 0]

    # end to end: camera from host through the API, band render, strip gather, frame to host
    r.set_flags(base_flags)
    e2e_steps = args.e2e_steps or args.steps
    host = torch.empty((w.height, w.width, 4), dtype=torch.uint8, pin_memory=True)
    for s in range(3):
        host.copy_(frame(s), non_blocking=True)
    torch.cuda.synchronize()

    def window_host():
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for s in range(e2e_steps):
            out = frame(s)
            if rank == 0:
                host.copy_(out, non_blocking=True)
            stream.synchronize()
        e1.record(stream)
        return e0, e1

    ems, _ = timed_windows(window_host, world, dev, dist, local_rank, args.min_window_ms)
    clock.stop()
    ewins = window_stats(ems, e2e_steps)
    img_bytes = w.width * w.height * 4
    r.close()
    return {
        "value": 1000.0 / ms_step, "ms_per_step": ms_step, "windows": wins, "clocks": clocks,
        "bands": bands, "band_history": history, "band_frame_ms": [float(x) for x in band_ms],
        "keys_per_frame_this_rank": K_avg, "sort_passes_per_frame": passes_avg, "stages_rank0": stages,
        "roofline": roofline, "gather_bytes_per_step": gather.bytes_per_frame if world > 1 else 0,
        "e2e": {"value": 1000.0 / ewins["ms_per_step_median"], "unit": "frames/s", "h2d_bytes_per_step": 192 * world,
                "d2h_bytes_per_step": img_bytes, "steps": e2e_steps, "windows": ewins,
                "api": "kt_gs_render (camera from host) + strip all_gather + frame copied to pinned host on rank 0"},
        "launches_per_step": st["launches"] * world,
    }


def run_bands(args, w, rank, world, local_rank):
    import datetime

    import torch
    import torch.distributed as dist

    from klartraum_b200 import make_scene, orbit_views
    from klartraum_b200.multigpu import broadcast_scene

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    if args.small:
        w = type(w)(**{**w.__dict__, "n": 20000, "width": 640, "height": 360})
    cams = orbit_views(N_VIEWS, w.distance, w.width, w.height, fovy_deg=w.fovy_deg)
    keep = None
    if world > 1:
        keep, n_rec = broadcast_scene(make_scene(w) if rank == 0 else None, dist, rank, dev)
        torch.cuda.synchronize()
        scene = (keep.data_ptr(), n_rec)
    else:
        scene = make_scene(w)
    m = measure_bands(args, w, rank, world, local_rank, dev, dist, cams, scene)
    del keep
    line = {
        "metric": f"frames/s, {w.n:,}-splat SH{w.sh_degree} {w.width}x{w.height} split into bin-row bands",
        "value": m["value"], "unit": "frames/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": m["ms_per_step"], "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{w.name}: {w.n:,} Gaussians SH{w.sh_degree} {w.width}x{w.height}, 16x16-px bins, "
                               f"{N_VIEWS}-view orbit, one frame per step split into {world} bin-row bands",
                   "bands": m["bands"], "parallelism": f"bands{world}: projection replicated, depth sort, placement "
                                                       "and splatting of the Gaussians that meet each band, strips "
                                                       "all-gathered (NCCL) every step",
                   "l2": "inputs larger than L2; no flush", "seed": w.seed},
        "timing": {"protocol": f"windows of exactly {args.steps} frames repeated for >= {args.min_window_ms:.0f} ms "
                               "of device time (max over ranks), median window", **m["windows"]},
        **{k: m[k] for k in ("band_history", "band_frame_ms", "keys_per_frame_this_rank", "sort_passes_per_frame",
                             "stages_rank0", "roofline", "gather_bytes_per_step", "e2e")},
        "gpu_launches": m["launches_per_step"] * args.steps, "gpu_launches_per_step": m["launches_per_step"],
        "clocks": m["clocks"],
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def cpu_baseline(w, cams, gpu_view0=None) -> dict:
    """The oracle (C restatement of the reference shaders, OpenMP) on full frames of the workload,
    and, for view 0, how far the GPU's and the float32 oracle's images are from the
    double-precision oracle."""
    import oracle
    from klartraum_b200 import make_scene

    g3d = make_scene(w)
    cfg = oracle.config(w.width, w.height, bin_size=16, sh_degree=w.sh_degree)
    bg = np.zeros((w.height, w.width, 4), np.uint8)
    bg[..., 3] = 255
    oracle.set_threads(len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1))
    img0, _ = oracle.render_frame_fast(cfg, cams[0], g3d, bg)  # also warms caches / pages in
    frames = 0
    t0 = time.perf_counter()
    while True:
        oracle.render_frame_fast(cfg, cams[frames % N_VIEWS], g3d, bg)
        frames += 1
        if time.perf_counter() - t0 > 10.0 or frames >= 8:
            break
    dt = time.perf_counter() - t0
    out = {"value": frames / dt, "unit": "frames/s", "cores": oracle.lib().ko_get_threads(), "kind": "port",
           "sample": f"{frames} full frames of the same workload (views 0..{frames - 1}) through the C "
                     f"restatement of the reference shaders (oracle/kt_oracle.c), OpenMP"}
    if gpu_view0 is not None:
        f64, _ = oracle.render_frame_f64(cfg, cams[0], g3d, bg)
        d = np.abs(gpu_view0.astype(np.int16) - img0.astype(np.int16))
        out["divergence_view0"] = {
            "units": "1/255 per channel, against the double-precision oracle (oracle/kt_oracle.c "
                     "ko_render_frame_f64)",
            "gpu": oracle.divergence(gpu_view0, f64), "float32_oracle": oracle.divergence(img0, f64),
            "gpu_vs_float32_oracle_max_abs": int(d.max())}
    return out


def main():
    args = parse()
    from klartraum_b200.scenes import WORKLOADS

    w = WORKLOADS[args.workload or (WORKLOAD if args.mode == "views" else "large_6m")]
    if args.n is not None:
        w = type(w)(**{**w.__dict__, "n": args.n})
    cfg_block = workload_config(w)
    cfg_block["binning"] = "sorted_keys" if args.sorted_keys else "placed"
    cfg_block["launch"] = "cuda_graph" if (args.launch == 'graph') else "stream"
    cfg_block["frames_in_flight"] = args.paths
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank == 0:
            run_reference(args, w, cfg_block)
        return
    if args.mode == "bands":
        run_bands(args, w, rank, world, local_rank)
    else:
        run_ours(args, w, cfg_block, rank, world, local_rank)


if __name__ == "__main__":
    main()
