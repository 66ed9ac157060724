#!/usr/bin/env python3
"""Benchmark of the 3DGS training hot path (render + L1/DSSIM loss + backward + Adam) on
BASELINE.json's headline workload: 3M Gaussians at 1920x1080.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl gs3d|reference]
                    [--views-per-gpu V | --global-batch B] [--no-extra] [--no-e2e]

Workload (synthetic, seeded; the BASELINE config 4 scene): 3,000,000 Gaussians, means
~ N(0, 2^2 I), log-scales ~ N(-5.5, 0.6), opacity logits ~ N(1, 1.5), SH degree 3 (48
coefficients, DC ~ N(0, 0.3), rest ~ N(0, 0.05)); 256 pinhole cameras at 1920x1080 (50 deg
horizontal FOV) on a Fibonacci hemisphere of radius 5 looking at the origin; uniform [0, 1]
target images. A step is one training iteration of the reference's training_step!
(training.jl:173-244) per GPU: render!, loss, backward!, ADC statistics, learning-rate annealing
and the Adam update, at iterations 3001.. (SH degree 3, between densify steps). By default one
view per GPU per step: at N = 1 the reference's iteration with its sparse Adam; at N > 1
multi-view data parallelism (gradient rows reduce-scattered over NCCL, each rank updates its 1/N
of the Gaussians, parameters all-gathered), so the per-GPU work is fixed ("weak" scaling).
--views-per-gpu / --global-batch train V views per GPU per step (config 4's batches of 8/16/32).
Inputs are larger than L2 (2.1 GB of parameters and moments), so no L2 flush is needed.

Beside the timed steps the line carries, measured outside the timed region: the rasterisers'
FP32-issue rooflines from exact work counts, render-only frames/s of the same scene, config 3's
4K render-only frames/s (6M Gaussians), the cost of one densify step, the drop-in sort against the
reference's CUB build, and the CPU baselines (--no-extra skips the 4K and densify legs).

`--impl reference` times the CPU restatement of the same training step (the reference has no
runnable implementation here: it is Julia/CUDA.jl and Julia is not installed) on all host
threads, rank 0 only, a time-bounded number of full steps.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
for _p in (str(REPO / "threedgaussiansplatting.jl_b200"), str(REPO)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "train iters/s and render frames/s, 3M Gaussians @1920x1080, 1/2/4/8 B200"
UNIT = "train views/s"
CONFIG_ID = 4
START_ITERATION = 3000
WORKLOAD = ("3M Gaussians (BASELINE config 4 scene), 1920x1080, 1 view per GPU per step: "
            "render + L1/DSSIM + backward + ADC stats + Adam")
POOL = 8  # distinct target images (one per camera index modulo POOL)
FALLBACK_HBM_GBS = 6650.0

# kernels per profiled stage (for gpu_launches)
KERNELS_PER_STAGE = {"keep_compact": 3, "project": 1, "dup_scan": 3, "dup_keys": 1, "tiles_end": 1,
                     "raster": 1, "zero_2d": 1, "bwd_raster": 1, "bwd_project": 1, "loss": 3,
                     "adc_stats": 1, "scatter_dense": 1, "adam_dense": 2, "adam": 2,
                     "zero_dense": 0, "tile_count": 3, "sort": 2}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["gs3d", "reference"], default="gs3d")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the config-3 render-only and densify-step legs")
    ap.add_argument("--ref-seconds", type=float, default=120.0)
    ap.add_argument("--n-gaussians", type=int, default=None,
                    help="override the Gaussian count (same distributions); for small profiling cases")
    ap.add_argument("--dp-sh", choices=["auto", "gather", "shard"], default="auto",
                    help="data-parallel factored steps: all-gather the SH coefficients after each "
                         "update, or keep them with their owners and send the next views' colours "
                         "(auto: shard with N > 1)")
    ap.add_argument("--dp-exchange", choices=["factored", "dense"], default="factored",
                    help="N > 1: gradient rows exchanged as factored rows (16 floats per Gaussian) "
                         "or dense rows (60)")
    ap.add_argument("--dp-chunks", type=int, default=None, help="N > 1: pipeline depth")
    ap.add_argument("--views-per-gpu", type=int, default=None,
                    help="views rendered and back-propagated per GPU per step (default 1: the "
                         "reference's one view per iteration on one GPU)")
    ap.add_argument("--global-batch", type=int, default=None,
                    help="views per step over all GPUs (BASELINE config 4: 8, 16 or 32); sets "
                         "--views-per-gpu to global-batch / N")
    return ap.parse_args()


def measured_peaks() -> tuple[float, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def fp32_peak() -> tuple[float, float, str]:
    """(FP32 lane-op peak per second, MUFU peak per second, source): 148 SMs x 128 FP32 lanes
    (16 MUFU lanes) x the maximum SM clock of MEASURED_PEAKS.json (sm_max_mhz; else the B200's
    nominal 1965 MHz). Derived, not measured: the measured peaks hold no FP32 figure."""
    mhz, src = 1965.0, "derived from the nominal 1965 MHz"
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            mhz = float(json.loads(p.read_text())["sm_max_mhz"])
            src = "derived: 148 SMs x 128 lanes x MEASURED_PEAKS.json sm_max_mhz"
        except Exception:
            pass
    return 148 * 128 * mhz * 1e6, 148 * 16 * mhz * 1e6, src


# FP32 operations per unit of the rasterisers' work (the hot-path analysis' per-unit costs):
# a forward blend (one (pixel, Gaussian) evaluation of the reference's loop) is ~13 FP32
# operations + 1 MUFU exponential; a contributing (pixel, Gaussian) pair of the backward blend
# is ~45 FP32 operations (+ its atomics).
FWD_OPS_PER_BLEND = 13.0
BWD_OPS_PER_PAIR = 45.0


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.idx = device_index
        self.proc = None
        self.file = None

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.idx)], stdout=self.file, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.file.flush()
        self.file.seek(0)
        sms, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.file.read().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sms.append(float(parts[1]))
                maxes.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        os.unlink(self.file.name)
        return {"sm_mhz": statistics.median(sms) if sms else None,
                "sm_max_mhz": max(maxes) if maxes else None, "samples": len(sms),
                "reasons": sorted(reasons)}


def build_workload(device, seed_offset=0, n_override=None):
    import numpy as np
    import torch
    from gs3d import RenderOptions, Tiling
    from gs3d.scene import CONFIGS, scene_radius, synthetic_gaussians
    import dataclasses
    cfg = CONFIGS[CONFIG_ID]
    spec = cfg["spec"] if not n_override else dataclasses.replace(cfg["spec"], n=int(n_override))
    gv = synthetic_gaussians(spec, cfg["seed"])
    cams = cfg["cameras"]()
    w, h = cams[0].width, cams[0].height
    gen = torch.Generator(device="cpu").manual_seed(1000 + seed_offset)
    pool_host = [torch.rand((w, h, 3), generator=gen, dtype=torch.float32) for _ in range(POOL)]
    ro = RenderOptions.for_camera(cams[0], 3)
    til = Tiling.for_camera(cams[0])
    return gv, cams, pool_host, ro, til, scene_radius(cams)


def stage_bytes(stage: str, F: int, D: int, n: int, w: int, h: int, passes: int,
                world: int = 1, factored: bool = True, tiles: int = 0) -> float | None:
    """Algorithmic bytes of one step of a stage on one rank: the hot-path analysis' minimum
    traffic per unit in the reference's data layouts (a stage that moves less than the
    reference layout needs is still credited with these bytes): keep + scan + compact 31 B per
    Gaussian; projection 300 B per filtered Gaussian; duplication 28 B read per filtered
    Gaussian (the tile counts here) and 12 B written per duplicate, the sort at the reference's
    key width (`passes` = ceil(key bits / 8) passes x 24 B per duplicate: 6 at 1080p) and the
    tile ranges 8 B per duplicate + 4 B per
    tile (the scatter + segment sort here); backward projection 548 B and Adam 1656 B per
    filtered Gaussian (data parallel: per Gaussian of the rank's n / world); blends as
    documented per rasteriser."""
    sort_bytes_per_dup = 24.0 * passes
    return {
        "project": 300.0 * F,
        "tile_count": 28.0 * F + 4.0 * tiles,
        "sort": (12.0 + sort_bytes_per_dup + 8.0) * D,
        "adam": 1656.0 * F,
        "adam_dense": 1656.0 * n / world,
        "bwd_project": 548.0 * F,
        "keep_compact": 31.0 * n,
        "dup_keys": 28.0 * F + 12.0 * D,
        "raster": 40.0 * D + 20.0 * w * h,
        "bwd_raster": 40.0 * D + 24.0 * w * h + 36.0 * F,
        "loss": 12.0 * 3 * w * h + 4.0 * 9 * 3 * w * h * 2,
    }.get(stage)


# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of one launch, from ncu captures of
# the 1M-Gaussian case of this workload (profiles/k_*_1M_1080p.md), as a fraction of that
# launch's algorithmic bytes; the full-size traffic is that fraction of the full-size bytes
# (traffic grows with the same units).
NCU_TRAFFIC_FRACTION = {
    # k_bwd_raster_masks<2>: 115.94 MB read + 5.59 MB write at F = 992,004, D = 943,223,
    # 1920x1080 (the contribution masks it reads are one 32-bit word per warp of 32 pixels and
    # 32-entry chunk, ~2 B per duplicate)
    "bwd_raster": 121.53e6 / (40.0 * 943_223 + 24.0 * 2_073_600 + 36.0 * 992_004),
    # k_raster<16, true>: 39.51 MB read + 7.75 MB write (images and the masks it writes)
    "raster": 47.26e6 / (40.0 * 943_223 + 20.0 * 2_073_600),
}


def run_reference(args, rank: int, world: int) -> None:
    """The CPU restatement of the training step on all host threads (rank 0 only)."""
    if rank != 0:
        return
    import numpy as np
    from gs3d.optimizer import bias_corrections
    from gs3d import _abi
    from gs3d.scene import CONFIGS, synthetic_gaussians
    from gs3d.training import TrainingOptions
    from gs3d import RenderOptions, Tiling
    from gs3d.scene import scene_radius
    from oracle import oracle as O
    gv, cams, pool_host, ro, til, radius = build_workload("cpu", n_override=args.n_gaussians)
    threads = os.cpu_count() or 1
    O.lib().oracle_set_threads(threads)
    g = O.NpGaussians.from_vector(gv)
    n = g.n
    m = O.NpMoments(np.zeros((n, 3, 2)), np.zeros((n, 2)), np.zeros((n, 3, 2)), np.zeros((n, 4, 2)),
                    np.zeros((n, 3, 16, 2)))
    opts = TrainingOptions(scene_radius=radius)
    acc = np.zeros(n, np.float32)
    cnt = np.zeros(n, np.int32)
    rng = np.random.default_rng(0)
    perm = rng.permutation(len(cams))
    done = 0

    def one_step():
        nonlocal done
        cam_i = int(perm[done % len(cams)])
        cam = cams[cam_i]
        target = pool_host[cam_i % POOL].numpy()
        f = O.render(g, cam, til, ro)
        (_, _, _), grad = O.loss(f["rgb"], target, opts.loss_dssim_vs_L1_weight)
        b = O.backward(g, cam, til, ro, f, grad)
        O.adc_stats(acc, cnt, b["mean2d"], f["fgidx_to_gidx"], cam.width, cam.height)
        p = _abi.AdamParamsC()
        lrs = opts.learning_rates()
        p.lr_means, p.lr_opacity_features, p.lr_scaling_features = lrs.means, lrs.opacity_features, lrs.scaling_features
        p.lr_rotation_features, p.lr_sh_dc, p.lr_sh_rest = lrs.rotation_features, lrs.sh_coeffs_dc, lrs.sh_coeffs_rest
        p.beta1, p.beta2, p.epsilon, p.update_count, p.sh_degree = 0.9, 0.999, 1e-15, done, 3
        bc1, bc2 = bias_corrections(0.9, 0.999, done)
        O.adam(g, m, b, f["fgidx_to_gidx"], p, bc1, bc2)
        done += 1

    # warm-up steps as asked, each a full step; capped at half the time cap in all
    warm = 0
    tw = time.perf_counter()
    while warm < args.warmup and (warm == 0 or time.perf_counter() - tw < args.ref_seconds / 2):
        one_step()
        warm += 1
    steps = 0
    t0 = time.perf_counter()
    while True:
        one_step()
        steps += 1
        el = time.perf_counter() - t0
        if steps >= args.steps or el >= args.ref_seconds:
            break
    value = steps / el
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": steps,
            "warmup": warm, "ms_per_step": 1000 * el / steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": workload_config(world, cams[0].width, cams[0].height, n),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"{steps} full training step(s) of the workload after {warm} "
                                       f"warm-up step(s) (time-bounded {args.ref_seconds:.0f} s), CPU "
                                       f"restatement of the reference's GPU-path arithmetic (render, loss, "
                                       f"backward, ADC statistics, Adam), {threads} threads"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def cpu_baseline_leg(gv_cpu, cams, pool_host, ro, til, opts) -> dict:
    """One full training step of the same workload through the CPU oracle (all host threads)."""
    import numpy as np
    from gs3d import _abi
    from gs3d.optimizer import bias_corrections
    from oracle import oracle as O
    threads = os.cpu_count() or 1
    O.lib().oracle_set_threads(threads)
    g = O.NpGaussians.from_vector(gv_cpu)
    n = g.n
    m = O.NpMoments(np.zeros((n, 3, 2)), np.zeros((n, 2)), np.zeros((n, 3, 2)), np.zeros((n, 4, 2)),
                    np.zeros((n, 3, 16, 2)))
    p = _abi.AdamParamsC()
    lrs = opts.learning_rates()
    p.lr_means, p.lr_opacity_features, p.lr_scaling_features = lrs.means, lrs.opacity_features, lrs.scaling_features
    p.lr_rotation_features, p.lr_sh_dc, p.lr_sh_rest = lrs.rotation_features, lrs.sh_coeffs_dc, lrs.sh_coeffs_rest
    p.beta1, p.beta2, p.epsilon, p.sh_degree = 0.9, 0.999, 1e-15, 3
    t0 = time.perf_counter()
    steps = 0
    while steps < 6 and (steps == 0 or time.perf_counter() - t0 < 10.0):  # about 10 s of work
        cam = cams[steps % len(cams)]
        f = O.render(g, cam, til, ro)
        (_, _, _), grad = O.loss(f["rgb"], pool_host[steps % len(pool_host)].numpy(),
                                 opts.loss_dssim_vs_L1_weight)
        b = O.backward(g, cam, til, ro, f, grad)
        p.update_count = steps
        bc1, bc2 = bias_corrections(0.9, 0.999, steps)
        O.adam(g, m, b, f["fgidx_to_gidx"], p, bc1, bc2)
        steps += 1
    el = time.perf_counter() - t0
    return {"value": steps / el, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{steps} full training steps (render+loss+backward+Adam) of the same workload, "
                      f"cameras 0..{steps - 1}, CPU restatement of the reference's GPU-path arithmetic, "
                      f"{threads} threads, {el:.1f} s"}


def cpu_render_leg(gv_cpu, cams, ro) -> dict:
    """The reference's own CPU renderer (forward_core.jl:25-177, restated in
    oracle/cpu_render.cpp): one frame of the render workload on all host threads and one on a
    single thread, as the reference runs it."""
    from oracle import oracle as O
    g = O.NpGaussians.from_vector(gv_cpu)
    threads = os.cpu_count() or 1
    out = {}
    for th in (threads, 1):
        t0 = time.perf_counter()
        O.cpu_render(g, cams[0], ro, th)
        out[th] = 1.0 / (time.perf_counter() - t0)
    return {"value": out[threads], "unit": "frames/s", "cores": threads, "kind": "port",
            "single_thread_value": out[1],
            "sample": f"one frame (camera 0) through the restated reference CPU renderer on "
                      f"{threads} threads, and one on 1 thread"}


def count_work(gaussians, cams, cam_indices, til, ro, buf, outputs) -> tuple[int, int]:
    """Sum over renders of the given cameras of (blends, contributions): the rasterisers'
    algorithmic work as the reference's blend loop performs it (gs3d_render_work_counts)."""
    from gs3d import _abi
    from gs3d import render as gs_render
    from gs3d.render import work_counts
    tb = tc = 0
    for i in cam_indices:
        gs_render(outputs, gaussians, cams[i], til, ro, buf, host_sync=False)
        b, c = work_counts(cams[i], til, ro, buf)
        if int(buf.device_counts[2].item()) & _abi.GS3D_STATUS_DUP_OVERFLOW:
            raise RuntimeError("duplicate-key capacity overflow while counting work")
        tb += b
        tc += c
    return tb, tc


def raster_rates(blends: float, contrib: float, fwd_ms: float | None, bwd_ms: float | None) -> dict:
    """FP32 / MUFU rates of the rasterisers from per-launch work counts and kernel times."""
    fp32, mufu, src = fp32_peak()
    out = {"fp32_peak_Tops": round(fp32 / 1e12, 2), "mufu_peak_Tops": round(mufu / 1e12, 3),
           "peak_source": src, "blends_per_launch": int(blends), "contributing_pairs_per_launch": int(contrib)}
    if fwd_ms:
        bps = blends / (fwd_ms / 1e3)
        out["forward"] = {"kernel": "k_raster", "avg_ms": round(fwd_ms, 4), "blends_per_s": bps,
                          "fp32_Tops": round(FWD_OPS_PER_BLEND * bps / 1e12, 3),
                          "fp32_frac": round(FWD_OPS_PER_BLEND * bps / fp32, 4),
                          "mufu_frac": round(bps / mufu, 4)}
    if bwd_ms:
        pps = contrib / (bwd_ms / 1e3)
        out["backward"] = {"kernel": "k_bwd_raster", "avg_ms": round(bwd_ms, 4), "pairs_per_s": pps,
                           "fp32_Tops": round(BWD_OPS_PER_PAIR * pps / 1e12, 3),
                           "fp32_frac": round(BWD_OPS_PER_PAIR * pps / fp32, 4)}
    return out


def flush_l2(device) -> None:
    import torch
    global _FLUSH
    try:
        _FLUSH
    except NameError:
        _FLUSH = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    _FLUSH.fill_(1)


def sort_baseline_leg(buf, device, bits: int, reps: int = 20) -> dict:
    """The duplicated keys of the last reference-order render (in filtered order: the input the
    reference's render! passes to its CUB sort) sorted by (a) the reference's own CUB wrapper,
    compiled from its source (oracle/_ref/cub_sort_pairs_wrapper.so), and (b) libgs3d.so's
    drop-in sort_pairs with the same signature, each timed per call with CUDA events on the
    legacy default stream (both run there), L2 flushed before every call; outputs compared."""
    import ctypes as C
    import torch
    from gs3d import _abi
    from oracle import build as obuild
    D = int(buf.device_counts[1].item())
    keys = buf.df2dgs_codes[:D].clone()
    vals = buf.dfgidx_to_fgidx[:D].clone()
    out = {"D": D, "key_bits": bits, "reps": reps, "l2": "flushed before every call"}
    libs = {"gs3d_sort_pairs": _abi.lib()}
    ref = obuild.REF_LIB
    if ref.exists():
        libs["reference_cub_sort_pairs"] = C.CDLL(str(ref))
    else:
        out["reference_cub_sort_pairs"] = "unavailable: oracle/_ref/cub_sort_pairs_wrapper.so not built"
    results = {}
    stream0 = torch.cuda.default_stream(device)
    for name, lib in libs.items():
        lib.determine_sort_pairs_temp_storage.restype = C.c_size_t
        lib.determine_sort_pairs_temp_storage.argtypes = [C.c_void_p] * 4 + [C.c_int, C.c_int]
        lib.sort_pairs.restype = None
        lib.sort_pairs.argtypes = [C.c_void_p, C.c_size_t] + [C.c_void_p] * 4 + [C.c_int, C.c_int]
        nbytes = int(lib.determine_sort_pairs_temp_storage(None, None, None, None, D, bits))
        tmp = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device)
        ko, vo = torch.empty_like(keys), torch.empty_like(vals)
        args = (C.c_void_p(tmp.data_ptr()), nbytes, C.c_void_p(keys.data_ptr()), C.c_void_p(ko.data_ptr()),
                C.c_void_p(vals.data_ptr()), C.c_void_p(vo.data_ptr()), D, bits)
        times = []
        with torch.cuda.stream(stream0):
            for r in range(reps + 3):
                flush_l2(device)
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream0)
                lib.sort_pairs(*args)
                b.record(stream0)
                torch.cuda.synchronize()
                if r >= 3:
                    times.append(a.elapsed_time(b))
        results[name] = (ko, vo)
        ms = statistics.median(times)
        out[name] = {"median_ms": round(ms, 4), "min_ms": round(min(times), 4), "temp_bytes": nbytes,
                     "keys_per_s": D / (ms / 1e3),
                     "hbm_GBps_at_reference_passes": round(24.0 * math.ceil(bits / 8) * D / (ms / 1e3) / 1e9, 1)}
    if len(results) == 2:
        (k1, v1), (k2, v2) = results.values()
        out["outputs_equal"] = bool(torch.equal(k1, k2) and torch.equal(v1, v2))
    return out


def render_only_leg(cfg_id: int, frames: int, world: int, rank: int, device, with_sort: bool) -> dict:
    """Render-only throughput of a BASELINE config (config 3: 6M Gaussians, 3840x2160, 64-frame
    orbit): device-timed frames/s, max over ranks, each rank rendering frames k * world + rank of
    the orbit; blends/s of the forward blend from its stage time and the blends the reference's
    loop performs on those frames."""
    import torch
    import torch.distributed as dist
    from gs3d import RenderBuffers, RenderOptions, RenderOutputs, Tiling, _abi
    from gs3d import render as gs_render
    from gs3d.scene import CONFIGS, synthetic_gaussians
    cfg = CONFIGS[cfg_id]
    g = synthetic_gaussians(cfg["spec"], cfg["seed"]).to(device)
    cams = cfg["cameras"]()
    ro = RenderOptions.for_camera(cams[0], 3)
    til = Tiling.for_camera(cams[0])
    outs = RenderOutputs.create(cams[0].width, cams[0].height, device)
    buf = RenderBuffers.create(g.n, til.nb_tiles, device, capacity_dup=8 * g.n, mask_dup=None)
    order = [(k * world + rank) % len(cams) for k in range(frames)]
    for k in range(3):
        gs_render(outs, g, cams[order[k % len(order)]], til, ro, buf, host_sync=False,
                  contrib_masks=False)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _abi.profile_enable(True)
    e0.record(stream)
    for i in order:
        gs_render(outs, g, cams[i], til, ro, buf, host_sync=False, contrib_masks=False)
    e1.record(stream)
    torch.cuda.synchronize()
    prof = _abi.profile_report()
    _abi.profile_enable(False)
    if int(buf.device_counts[2].item()) & _abi.GS3D_STATUS_DUP_OVERFLOW:
        raise RuntimeError("duplicate-key capacity overflow during the render-only timing")
    ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item())
    blends, contrib = count_work(g, cams, order, til, ro, buf, outs)
    fwd_ms = prof["raster"][1] / max(prof["raster"][0], 1)
    rates = raster_rates(blends / frames, contrib / frames, fwd_ms, None)
    res = {"config": cfg_id, "n_gaussians": g.n, "resolution": [cams[0].width, cams[0].height],
           "tiles": [til.tile_width, til.tile_height], "frames_per_rank": frames,
           "value": world * frames / (ms / 1e3), "unit": "frames/s", "ms_per_frame": ms / frames,
           "blends_per_frame": blends / frames, "blends_per_s_whole_frame": world * blends / (ms / 1e3),
           "forward_blend": rates.get("forward"),
           "stages_ms_per_frame": {k: round(t / frames, 4) for k, (c, t) in prof.items()}}
    if with_sort and rank == 0:
        gs_render(outs, g, cams[0], til, ro, buf, reference_order=True)
        res["sort_vs_reference_cub"] = sort_baseline_leg(buf, device, til.highest_key_bit)
    del g, buf, outs
    torch.cuda.empty_cache()
    return res


def densify_leg(trainer, world: int, steady_ms: float, device) -> dict:
    """Cost of one densify/prune step (the reference's maybe_densify_and_prune! every 100
    iterations, training.jl:313-444) at the bench's model size: the whole training step at a
    densify iteration, device-timed (max over ranks), against the steady-state step; the ADC
    statistics are the ones accumulated over the bench's earlier steps."""
    import torch
    import torch.distributed as dist
    o = trainer.options
    o.adc_interval = 100
    nxt = (trainer.iteration_nb // 100 + 1) * 100
    while nxt % o.opacity_reset_interval == 0 or not (o.adc_start_iteration_nb <= nxt <= o.adc_final_iteration_nb):
        nxt += 100
    trainer.iteration_nb = nxt - 1
    n0 = trainer.gaussians.n
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    trainer.training_step()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item())
    n1 = trainer.gaussians.n
    # a second densify step 100 iterations later: the allocations of the first one are cached
    for _ in range(3):
        trainer.training_step()
    trainer.iteration_nb = nxt + 99 if (nxt + 100) % o.opacity_reset_interval else nxt + 199
    second_it = trainer.iteration_nb + 1
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    trainer.training_step()
    e1.record(stream)
    torch.cuda.synchronize()
    ms2 = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(ms2, op=dist.ReduceOp.MAX)
    ms2 = float(ms2.item())
    # steady state after the densify steps, with the changed model
    for _ in range(3):
        trainer.training_step()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(10):
        trainer.training_step()
    e1.record(stream)
    torch.cuda.synchronize()
    after = torch.tensor([e0.elapsed_time(e1) / 10], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(after, op=dist.ReduceOp.MAX)
    return {"iteration": nxt, "densify_step_ms": round(ms, 3), "steady_step_ms": round(steady_ms, 3),
            "densify_extra_ms": round(ms - steady_ms, 3), "n_before": n0, "n_after": n1,
            "second_iteration": second_it, "second_densify_step_ms": round(ms2, 3),
            "second_densify_extra_ms": round(ms2 - steady_ms, 3),
            "step_ms_after": round(float(after.item()), 3),
            "amortised_extra_ms_per_step": round((ms2 - steady_ms) / 100, 4),
            "note": "one densify step every 100 iterations within the densify window; the first one "
                    "also pays the allocation of the new arrays, later ones reuse cached memory"}


def main() -> None:
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    assert args.warmup >= 3, "at least 3 warm-up steps"
    import numpy as np
    import torch
    import torch.distributed as dist
    import datetime
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        # NCCL on high-priority streams: its blocks are scheduled ahead of the compute kernels'
        # as SM slots free up, so the chunked reduce-scatters overlap the projection backward
        opts = dist.ProcessGroupNCCL.Options()
        opts.is_high_priority_stream = True
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=device, pg_options=opts)
    import gs3d
    from gs3d import _abi
    from gs3d.dp import DataParallelTrainer
    from gs3d.training import Trainer, TrainingOptions
    gs3d.lib()

    V = args.views_per_gpu or 1
    if args.global_batch:
        if args.global_batch % world:
            raise SystemExit(f"--global-batch {args.global_batch} is not a multiple of {world} GPUs")
        V = args.global_batch // world
    gv_cpu, cams, pool_host, ro, til, radius = build_workload(device, n_override=args.n_gaussians)
    opts = TrainingOptions(scene_radius=radius)
    if START_ITERATION + args.warmup + 2 * args.steps + 8 + 11 >= START_ITERATION + 100:
        opts.adc_interval = 10 ** 9  # keep densify steps out of every measured window
    gv = gv_cpu.to(device)
    pool_dev = [t.to(device) for t in pool_host]
    targets_dev = [pool_dev[i % POOL] for i in range(len(cams))]
    pool_pinned = [t.pin_memory() for t in pool_host]
    targets_host = [pool_pinned[i % POOL] for i in range(len(cams))]
    if world > 1 or V > 1:
        trainer = DataParallelTrainer(gv, cams, targets_dev, ro, til, opts, seed=0,
                                      capacity_dup=8 * gv.n, chunks=args.dp_chunks,
                                      factored=args.dp_exchange == "factored", views_per_rank=V,
                                      shard_sh=None if args.dp_sh == "auto" else args.dp_sh == "shard")
    else:
        trainer = Trainer(gv, cams, targets_dev, ro, til, opts, seed=0, capacity_dup=8 * gv.n)
    trainer.iteration_nb = START_ITERATION
    stream = torch.cuda.current_stream()

    for _ in range(args.warmup):
        trainer.training_step()
    torch.cuda.synchronize()
    trainer.render_host_sync = False
    F, D = (int(x) for x in trainer.render_buffers.device_counts[:2].cpu())
    # cameras of the timed steps (for the rasterisers' work counts afterwards)
    first = 0 if isinstance(trainer, DataParallelTrainer) else 1
    timed_cams = [trainer.peek_camera_index(first + k) for k in range(args.steps * V)]

    # ---- device-timed throughput, inputs resident in HBM ------------------------------
    # nvidia-smi numbers GPUs physically: map this rank's device through CUDA_VISIBLE_DEVICES
    visible = [v.strip() for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
    smi_index = visible[local] if local < len(visible) and visible[local].isdigit() else str(local)
    clocks = ClockSampler(smi_index)
    _abi.profile_enable(True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        trainer.training_step()
    if hasattr(trainer, "sync_parameters"):
        trainer.sync_parameters()  # the last step's parameter all-gathers belong to the timed work
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    if world > 1:
        dist.barrier()
    ms = e0.elapsed_time(e1)
    prof = _abi.profile_report()
    _abi.profile_enable(False)
    status = int(trainer.render_buffers.device_counts[2].item())
    if status & _abi.GS3D_STATUS_DUP_OVERFLOW:
        raise RuntimeError("duplicate-key capacity overflow during the timed region")
    ms_t = torch.tensor([ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())
    value = world * V * args.steps / (ms_max / 1000.0)

    # ---- where a data-parallel step's time goes (untimed extra steps, every rank alike) ----
    dp_phases = None
    if isinstance(trainer, DataParallelTrainer):
        trainer.training_step()  # its gathers in flight, as before every timed step
        trainer.phase_events = []
        k = min(args.steps, 10)
        t0 = time.perf_counter()
        for _ in range(k):
            trainer.training_step()
        # the host's time to issue a step: at or above the device's step time, the host paces it
        host_ms = (time.perf_counter() - t0) * 1000.0 / k
        dp_phases = trainer.phase_times()
        dp_phases["host_issue_ms_per_step"] = round(host_ms, 4)
        trainer.phase_events = None
        trainer.sync_parameters()

    # ---- end to end through the public API: pinned host targets in, loss out ----------
    e2e = None
    if not args.no_e2e:
        trainer.targets = targets_host
        loss_host = torch.empty(4, dtype=torch.float32, pin_memory=True)
        for _ in range(2):
            loss_host.copy_(trainer.training_step(), non_blocking=True)
            stream.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            loss_host.copy_(trainer.training_step(), non_blocking=True)
            stream.synchronize()
            float(loss_host[0])
        if hasattr(trainer, "sync_parameters"):
            trainer.sync_parameters()
        e1.record(stream)
        torch.cuda.synchronize()
        ms2 = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(ms2, op=dist.ReduceOp.MAX)
        w, h = cams[0].width, cams[0].height
        e2e = {"value": world * V * args.steps / (float(ms2.item()) / 1000.0), "unit": UNIT,
               "h2d_bytes_per_step": 3 * w * h * 4 * world * V, "d2h_bytes_per_step": 16 * world}

    if hasattr(trainer, "sync_parameters"):
        trainer.sync_parameters()
    # ---- render-only throughput (the metric's "render frames/s"): same scene and cameras,
    # each rank renders its own frames, device-timed, max over ranks --------------------------
    from gs3d import render as gs_render
    rb = trainer.render_buffers
    render_cams = [(k * world + rank) % len(cams) for k in range(args.steps)]
    for k in range(3):
        gs_render(trainer.render_outputs, trainer.gaussians, cams[k % len(cams)], trainer.tiling,
                  trainer.render_options, rb, host_sync=False, contrib_masks=False)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    _abi.profile_enable(True)
    e0.record(stream)
    for k in render_cams:
        gs_render(trainer.render_outputs, trainer.gaussians, cams[k], trainer.tiling,
                  trainer.render_options, rb, host_sync=False, contrib_masks=False)
    e1.record(stream)
    torch.cuda.synchronize()
    rprof = _abi.profile_report()
    _abi.profile_enable(False)
    if int(rb.device_counts[2].item()) & _abi.GS3D_STATUS_DUP_OVERFLOW:
        raise RuntimeError("duplicate-key capacity overflow during the render timing")
    ms3 = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(ms3, op=dist.ReduceOp.MAX)
    render_fps = {"value": world * args.steps / (float(ms3.item()) / 1000.0), "unit": "frames/s",
                  "ms_per_frame": float(ms3.item()) / args.steps,
                  "workload": "forward render only, same scene, 1920x1080, one frame per GPU per step"}

    # ---- the rasterisers' algorithmic work (outside every timed region) ------------------
    # the reference's blend loop on the cameras of the timed training steps and of the render
    # timing, with the parameters as they are now (a few hundred small Adam steps later)
    tb, tc = count_work(trainer.gaussians, cams, timed_cams, trainer.tiling, trainer.render_options,
                        rb, trainer.render_outputs)
    rbl, rco = count_work(trainer.gaussians, cams, render_cams, trainer.tiling, trainer.render_options,
                          rb, trainer.render_outputs)
    avg = lambda pr, k: pr[k][1] / max(pr[k][0], 1) if k in pr else None
    train_rates = raster_rates(tb / (args.steps * V), tc / (args.steps * V), avg(prof, "raster"),
                               avg(prof, "bwd_raster"))
    render_rates = raster_rates(rbl / args.steps, rco / args.steps, avg(rprof, "raster"), None)
    render_fps["forward_blend"] = render_rates.get("forward")
    render_fps["blends_per_frame"] = rbl / args.steps
    render_fps["blends_per_s_whole_frame"] = world * rbl / (float(ms3.item()) / 1000.0)

    # ---- roofline of the dominant kernel ---------------------------------------------
    peak, peak_kind = measured_peaks()
    w, h = cams[0].width, cams[0].height
    passes = math.ceil(til.highest_key_bit / 8)
    stages = {}
    factored = world > 1 and args.dp_exchange == "factored"
    for name, (cnt, tot) in prof.items():
        av = tot / max(cnt, 1)
        b = stage_bytes(name, F, D, gv.n, w, h, passes, world, factored, til.nb_tiles)
        if b and name not in ("adam", "adam_dense"):
            b *= V  # every view of a step runs the render and backward stages
        b = b * args.steps / cnt if b and cnt else b  # per launch (chunked stages: a share)
        stages[name] = {"launches": cnt, "avg_ms": round(av, 4),
                        "share": round(tot / max(sum(t for _, t in prof.values()), 1e-9), 4),
                        "alg_GBps": round(b / (av / 1000) / 1e9, 1) if b else None}
    dominant = max(prof.items(), key=lambda kv: kv[1][1])[0]
    dom = stages[dominant]
    dom_bytes = stage_bytes(dominant, F, D, gv.n, w, h, passes, world, factored, til.nb_tiles)
    if dom_bytes and dominant not in ("adam", "adam_dense"):
        dom_bytes *= V
    dom_bytes = dom_bytes * args.steps / prof[dominant][0] if dom_bytes else dom_bytes
    traffic = (round(NCU_TRAFFIC_FRACTION[dominant] * dom_bytes / 1e9, 4)
               if dominant in NCU_TRAFFIC_FRACTION and dom_bytes else None)
    if dominant in ("bwd_raster", "raster"):
        part = train_rates["backward" if dominant == "bwd_raster" else "forward"]
        fp32, _, fp32_src = fp32_peak()
        roofline = {"bound": "fp32-issue", "kernel": part["kernel"], "achieved": part["fp32_Tops"],
                    "peak": round(fp32 / 1e12, 2), "peak_source": fp32_src, "unit": "TFLOP/s",
                    "frac": part["fp32_frac"],
                    "work": (f"{BWD_OPS_PER_PAIR:.0f} FP32 ops x {tc / (args.steps * V):.0f} contributing "
                             f"(pixel, Gaussian) pairs per launch" if dominant == "bwd_raster" else
                             f"{FWD_OPS_PER_BLEND:.0f} FP32 ops x {tb / (args.steps * V):.0f} blends per launch"),
                    "avg_ms": dom["avg_ms"], "traffic": traffic, "traffic_unit": "GB per launch",
                    "hbm_frac": round(dom["alg_GBps"] / peak, 4) if dom["alg_GBps"] else None,
                    "hbm_peak": peak, "hbm_peak_source": peak_kind}
    else:
        roofline = {"bound": "hbm", "kernel": dominant, "achieved": dom["alg_GBps"], "peak": peak,
                    "peak_source": peak_kind, "unit": "GB/s",
                    "frac": round(dom["alg_GBps"] / peak, 4) if dom["alg_GBps"] else None,
                    "traffic": traffic, "traffic_unit": "GB per launch"}
    gpu_launches = 0
    for name, (cnt, _) in prof.items():
        k = KERNELS_PER_STAGE.get(name, 1)
        gpu_launches += cnt * k

    # ---- config 3: render-only 6M Gaussians at 3840x2160 ----------------------------------
    render_4k = None
    if not args.no_extra:
        render_4k = render_only_leg(3, 64, world, rank, device,
                                    with_sort=(world == 1 and not args.no_cpu_baseline))

    # ---- reference baselines (rank 0, one GPU): CPU oracle step, CPU renderer, CUB sort ----
    cpu = None
    sort_1080 = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        gs_render(trainer.render_outputs, trainer.gaussians, cams[timed_cams[-1]], trainer.tiling,
                  trainer.render_options, rb, reference_order=True)
        sort_1080 = sort_baseline_leg(rb, device, til.highest_key_bit)
        sort_1080["gs3d_tile_bucket_pipeline"] = {
            "avg_ms": round((avg(prof, "tile_count") or 0) + (avg(prof, "sort") or 0), 4),
            "stages": "tile_count + sort (counts, scan, scatter, per-tile sort: the render's default "
                      "F4-F7, which also yields tile ends)", "D_of_training_step": D}
        cpu = cpu_baseline_leg(gv_cpu, cams, pool_host, ro, til, opts)
        render_fps["cpu_baseline"] = cpu_render_leg(gv_cpu, cams, ro)

    # ---- one densify step at the bench's size (all ranks: it is collective) ---------------
    densify = None
    if not args.no_extra:
        densify = densify_leg(trainer, world, ms_max / args.steps, device)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "strong" if args.global_batch else "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": workload_config(world, w, h, gv.n, V),
            "workload_stats": {"filtered_F": F, "duplicates_D": D, "tiles": [til.tile_width, til.tile_height],
                               **({"dp_exchange": args.dp_exchange, "dp_chunks": trainer.chunks,
                                   "dp_sh": "shard" if trainer.shard_sh else "gather"}
                                  if world > 1 else {})},
            "e2e": e2e, "render": render_fps, "roofline": roofline, "rasterisers": train_rates,
            "cpu_baseline": cpu, "clocks": clk, "gpu_launches": gpu_launches, "stages": stages,
            "dp_phases": dp_phases,
            "render_config3_4k": render_4k, "densify": densify, "sort_vs_reference_cub": sort_1080,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def workload_config(world: int, w: int, h: int, n: int, views: int = 1) -> dict:
    """The workload's config, identical in both arms (the reference arm times the same one)."""
    return {"workload": WORKLOAD if views == 1 else WORKLOAD.replace("1 view per GPU", f"{views} views per GPU"),
            "global_batch": world * views, "views_per_gpu": views, "resolution": [w, h],
            "n_gaussians": n, "parallelism": f"dp{world}" if world > 1 else "single",
            "l2": "inputs larger than L2 (2.1 GB params+moments), no flush"}


if __name__ == "__main__":
    main()
