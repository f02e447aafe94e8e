#!/usr/bin/env python
"""bench.py — audio-seconds/sec of MelBandRoformer separation on B200.

Workload (N=1): the "Standard" configuration — random-init MelBandRoformer
dim 384, depth 6, 8 heads x 64, FFN x4, 60 mel bands, mask-estimator depth 2,
1 stem, fp16 — separating a 30 s stereo 44.1 kHz seeded pink-noise track
(1/f, -18 dBFS RMS, 16-bit quantised) in 8 s chunks with overlap 4,
chunk-batch 1.  One step = one separation of the whole track.  With
--gpus N (one process per GPU under torchrun) every rank separates its own
30 s track (weak scaling: tracks are independent, so no data moves between
ranks).  `--scaling strong` instead splits one track's chunk list into
contiguous ranges, one per rank, and moves only the overlap-add boundaries
between neighbours (one batched NCCL send/receive).

The default run also carries `long_track`: the two-stem bf16 model on one
3-minute track with its chunk ranges sharded over all N ranks (strong
scaling, the same timing rules), with rank 0's check of the assembled stems
against a one-GPU separation.

Prints one JSON line (rank 0).  `value` times device-resident input; `e2e`
times the host entry point (mbr_separate: pinned host track in, stems out).
`--impl reference` times the reference path's CPU restatement (the reference
has no CPU implementation of its own) on a bounded excerpt per step; under
torchrun only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "mbr-cuda-tile_b200")
sys.path.insert(0, PKG)

SR = 44100
WORKLOADS = {
    "std": dict(preset="std", dtype="fp16", seconds=30.0, overlap=4.0, chunk_batch=1,
                desc="std: dim 384, depth 6, 8x64 heads, 1 stem; 30 s stereo track, 8 s chunks, overlap 4, "
                     "chunk-batch 1"),
    "two_stem": dict(preset="two_stem", dtype="bf16", seconds=180.0, overlap=4.0, chunk_batch=4,
                     desc="two_stem: dim 384, depth 12, 8x64 heads, 2 stems; 3 min track, 8 s chunks, overlap 4, "
                          "chunk-batch 4"),
    "large": dict(preset="large", dtype="fp16", seconds=600.0, overlap=2.0, chunk_batch=8,
                  desc="large: dim 512, depth 12, 16x64 heads, 2 stems; 10 min track, 11 s chunks, overlap 2, "
                       "chunk-batch 8"),
    "pr1": dict(preset="pr1", dtype="fp32", seconds=8.0, overlap=1.0, chunk_batch=1, signal="uniform16",
                desc="pr1: dim 192, depth 1, 8x32 heads, 1 stem, fp32; one 8 s chunk of 16-bit uniform noise "
                     "(single-chunk path)"),
    "r0": dict(preset="r0", dtype="bf16", seconds=30.0, overlap=2.0, chunk_batch=1,
               desc="r0 (the reference's own shape): dim 256, depth 12, 8x64 heads, 2 stems, bf16; 30 s track, "
                    "13 s chunks (T = 1301), overlap 2, chunk-batch 1"),
}


def workload_track(wl: dict, seconds: float, seed: int) -> np.ndarray:
    """The workload's synthetic stereo track: seeded pink noise, or 16-bit
    uniform noise in [-0.5, 0.5] for PR1."""
    import csm_tool

    if wl.get("signal") == "uniform16":
        return csm_tool.uniform_noise16(int(round(seconds * SR)), seed)
    return pink_noise(seconds, seed)


def pink_noise(seconds: float, seed: int, channels: int = 2) -> np.ndarray:
    """Seeded 1/f noise, RMS -18 dBFS, quantised to 16-bit levels (k / 32768)."""
    import csm_tool

    return csm_tool.pink_noise(seconds, seed, channels, SR)


def model_flops(cfg: dict, T: int, B: int, bd: list) -> dict:
    """Algorithmic FLOPs of one forward over B chunks of T frames, per kernel class."""
    D, H, dh = cfg["dim"], cfg["heads"], cfg["dim_head"]
    DI, hid, NB = H * dh, cfg["dim"] * cfg["mlp_expansion_factor"], cfg["num_bands"]
    MT = B * T
    M = MT * NB
    L = cfg["depth"] * (cfg["time_transformer_depth"] + cfg["freq_transformer_depth"])
    Lt = cfg["depth"] * cfg["time_transformer_depth"]
    Lf = cfg["depth"] * cfg["freq_transformer_depth"]
    S, md = cfg["num_stems"], cfg["mask_estimator_depth"]
    f = {
        "gemm_bandsplit": 2.0 * MT * D * sum(bd),
        "gemm_qkv": L * 2.0 * M * D * 3 * DI,
        "gemm_out": L * 2.0 * M * DI * D,
        "gemm_ffn1": L * 2.0 * M * D * hid,
        "gemm_ffn2": L * 2.0 * M * hid * D,
        "attn_time": Lt * 4.0 * T * T * dh * H * B * NB,
        "attn_freq": Lf * 4.0 * NB * NB * dh * H * MT,
        "gemm_mask_hidden": S * 2.0 * MT * NB * (D * hid + (md - 1) * hid * hid),
        "gemm_mask_out": S * 2.0 * MT * hid * 2 * sum(bd),
    }
    return f


def band_dims(cfg: dict) -> list:
    import csm_tool

    _, nfpb, _ = csm_tool.mel_band_map(cfg["sample_rate"], cfg["stft_n_fft"], cfg["num_bands"], cfg["stereo"])
    C = 2 if cfg["stereo"] else 1
    return [int(2 * n * C) for n in nfpb]


def load_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return dict(hbm_gbs=d["hbm_gbs"], tflops=d["bf16_tflops"], tflops_sustained=d["bf16_tflops_sustained"],
                    source="measured")
    return dict(hbm_gbs=6650.0, tflops=1590.0, tflops_sustained=1400.0, source="fallback")


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            p = [x.strip() for x in l.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx = float(p[2])
            except ValueError:
                continue
            for n, v in zip(names, p[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def cpu_sample(csm: str, cfg: dict, step_flops: float, seconds_audio: float, excerpt_s: float, reps: int = 1,
               wl: dict | None = None, n_chunks: int = 0):
    """Times the CPU oracle (all host threads) on one forward of the same model.
    excerpt_s <= 0: one full chunk, and the step time is that time x the
    track's chunk count (every chunk is the same work); otherwise an excerpt of
    excerpt_s seconds scaled by algorithmic FLOPs to the step."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    m = oracle.Model(csm, 1 if cfg.get("_dtype") == "fp16" else 3 if cfg.get("_dtype") == "bf16" else 0)
    full = excerpt_s <= 0
    L = cfg["chunk_size"] if full else int(excerpt_s * SR)
    x = workload_track(wl or {}, L / SR, 7)[None]
    T = L // cfg["stft_hop_length"] + 1
    fl = sum(model_flops(cfg, T, 1, band_dims(cfg)).values())
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        m.forward(x)
        ts.append(time.perf_counter() - t0)
    t = float(np.median(ts))
    if full and n_chunks > 0:
        step_s = t * n_chunks
        how = (f"CPU oracle forward of one full {L / SR:g} s chunk ({T} frames, {fl / 1e12:.3f} TFLOP) in "
               f"{t:.2f} s, times the track's {n_chunks} chunks")
    else:
        step_s = t * step_flops / fl
        how = (f"CPU oracle forward of a {L / SR:g} s stereo excerpt ({T} frames, {fl / 1e12:.3f} TFLOP) "
               f"in {t:.2f} s, scaled by algorithmic FLOPs to the {step_flops / 1e12:.2f} TFLOP step")
    return dict(value=seconds_audio / step_s, unit="audio-s/s", cores=oracle.threads(), kind="port",
                sample=how, sample_seconds=t)


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def run_reference(args, wl):
    """The reference arm: the CPU restatement of the reference path, all host threads."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return 0
    import csm_tool

    cfg = csm_tool.base_config(**csm_tool.PRESETS[wl["preset"]])
    cfg["_dtype"] = wl["dtype"]
    with tempfile.TemporaryDirectory() as d:
        csm = os.path.join(d, "model.csm")
        csm_tool.write_csm(csm, {k: v for k, v in cfg.items() if not k.startswith("_")},
                           csm_tool.random_weights({k: v for k, v in cfg.items() if not k.startswith("_")}, 0))
        # the GPU arm's step: N independent tracks (weak) or one track (strong)
        ntracks = args.gpus if args.scaling == "weak" else 1
        seconds = wl["seconds"] * ntracks
        step_flops = step_model_flops(cfg, wl["seconds"], wl) * ntracks
        vals = []
        for i in range(args.warmup + args.steps):
            r = cpu_sample(csm, cfg, step_flops, seconds, args.cpu_excerpt, wl=wl)
            if i >= args.warmup:
                vals.append(r)
        v = float(np.mean([r["value"] for r in vals]))
        ms = float(np.mean([r["sample_seconds"] for r in vals])) * 1e3
        base = vals[-1]
        line = {
            "impl": "reference", "metric": "audio-seconds/sec", "value": v, "unit": "audio-s/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": args.scaling if args.gpus > 1 else "weak", "vs_baseline": None,
            "dtype": "f32 (fp64 reductions)", "data": "synthetic: seeded pink noise, random-init weights",
            "config": {"workload": wl["desc"] + (f"; {ntracks} tracks" if ntracks > 1 else "")},
            "cpu_baseline": {"value": v, "unit": "audio-s/s", "cores": base["cores"], "kind": "port",
                             "sample": base["sample"]},
            "e2e": {"value": v, "unit": "audio-s/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "the reference has no CPU implementation of this path; this arm times the CPU restatement "
                    "(oracle/) of the reference's forward with all host threads",
        }
        print(json.dumps(line), flush=True)
    return 0


def track_chunks(cfg, seconds, wl) -> int:
    """Chunk count of one whole-track separation (process_chunked's plan)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    N = int(round(seconds * SR))
    if N <= cfg["chunk_size"]:
        return 1
    starts, _, _, _ = oracle.chunk_plan(N, cfg["chunk_size"], -1.0 if wl["overlap"] <= 0 else wl["overlap"],
                                        cfg["num_overlap"])
    return len(starts)


def step_model_flops(cfg, seconds, wl):
    """Algorithmic FLOPs of one whole-track separation (all chunks)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    T = cfg["chunk_size"] // cfg["stft_hop_length"] + 1
    per_chunk = sum(model_flops(cfg, T, 1, band_dims(cfg)).values())
    return per_chunk * track_chunks(cfg, seconds, wl)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="mbr_b200", choices=["mbr_b200", "reference"])
    ap.add_argument("--workload", default="std", choices=sorted(WORKLOADS))
    ap.add_argument("--scaling", default="weak", choices=["weak", "strong"],
                    help="N > 1: weak = every rank separates its own track of the workload's length; strong = one "
                         "track of the workload's length, its chunk ranges split over the ranks")
    ap.add_argument("--cpu-excerpt", type=float, default=1.0,
                    help="seconds of audio per reference-arm step (the reference arm times one excerpt per step)")
    ap.add_argument("--cpu-chunk", type=float, default=0.0,
                    help="cpu_baseline of the main line: 0 = one full chunk x the chunk count, >0 = an excerpt of "
                         "this many seconds scaled by FLOPs")
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline sample")
    ap.add_argument("--no-long-track", action="store_true",
                    help="skip the long-track (two-stem, 3 min, chunk ranges over all ranks) strong-scaling "
                         "measurement that the default std run adds as `long_track`")
    ap.add_argument("--op-sweep", action="store_true",
                    help="tensor-op sweep: achieved HBM GB/s of every stand-alone op over [B*801*60, D] activations "
                         "(one JSON line per case, then a summary line)")
    ap.add_argument("--ops", default="", help="op sweep: comma-separated ops to run (default all)")
    ap.add_argument("--dtypes", default="fp32,fp16,bf16", help="op sweep: comma-separated dtypes")
    ap.add_argument("--batches", default="1,4,8", help="op sweep: comma-separated B values")
    ap.add_argument("--tensor-sweep", action="store_true",
                    help="Tensor API op sweep: achieved HBM GB/s of the Tensor class's elementwise, broadcast, "
                         "conversion and reduction kernels over the same activations (runs the native "
                         "tensor_bench; one JSON line per case, then a summary line)")
    ap.add_argument("--single-chunk", action="store_true",
                    help="profiling aid: run exactly warmup+steps forwards of one chunk batch and print their time "
                         "(not the benchmark line)")
    args = ap.parse_args()
    wl = WORKLOADS[args.workload]
    if args.impl == "reference":
        return run_reference(args, wl)
    if args.single_chunk:
        return run_single_chunk(args, wl)
    if args.op_sweep:
        return run_op_sweep(args)
    if args.tensor_sweep:
        return run_tensor_sweep(args)

    import torch

    world, rank, local = dist_env()
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE {world}"
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    dev = torch.device("cuda", local)
    # a dedicated stream (the legacy default stream cannot be graph-captured);
    # made current so that torch's copies and NCCL calls order with our work
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    ctx = dict(dev=dev, stream=stream, rank=rank, world=world, dist=dist, local=local)

    m, cfg, csm, tmpdir = make_model(wl, local)
    sharded = world > 1 and args.scaling == "strong"
    if sharded:
        seconds = wl["seconds"]
        track = workload_track(wl, seconds, 1234)
    else:
        # weak: every rank separates its own track of the workload's length
        seconds = wl["seconds"] * world
        track = workload_track(wl, wl["seconds"], 1234 + rank)
    run = TrackRun(m, cfg, wl, track, ctx, sharded)
    with ClockSampler(local) as clk:
        ms, launches = time_steps(run, args.warmup, args.steps, ctx)
    value = seconds / (ms / 1e3)
    e2e_ms, h2d, d2h = run.e2e(args.steps)
    check = run.check() if sharded else None
    e2e = {"value": seconds / (e2e_ms / 1e3), "unit": "audio-s/s", "h2d_bytes_per_step": int(h2d),
           "d2h_bytes_per_step": int(d2h), "ms_per_step": e2e_ms, "path": run.e2e_path}

    # ---- roofline of the dominant kernel class (one profiled step) ----
    peaks = load_peaks()
    m.profile(True)
    run.step()
    torch.cuda.synchronize(dev)
    prof = m.profile_read()
    m.profile(False)
    T = cfg["chunk_size"] // cfg["stft_hop_length"] + 1
    flops_fwd = model_flops(cfg, T, wl["chunk_batch"], band_dims(cfg))
    flops_fwd["ffn"] = flops_fwd["gemm_ffn1"] + flops_fwd["gemm_ffn2"]  # the fused FFN block: both contractions
    kind = max(prof, key=lambda k: prof[k][0])
    kms, kn = prof[kind]
    roof = None
    traffic = read_traffic(kind)
    if kind in flops_fwd and kn > 0:
        # launches of this class per forward
        per_fwd = {"gemm_bandsplit": 1, "gemm_mask_out": cfg["num_stems"],
                   "gemm_mask_hidden": cfg["num_stems"] * cfg["mask_estimator_depth"],
                   "attn_time": cfg["depth"] * cfg["time_transformer_depth"],
                   "attn_freq": cfg["depth"] * cfg["freq_transformer_depth"]}.get(
            kind, cfg["depth"] * (cfg["time_transformer_depth"] + cfg["freq_transformer_depth"]))
        per_launch = flops_fwd[kind] / per_fwd
        achieved = per_launch / (kms / kn / 1e3) / 1e12
        if wl["dtype"] == "fp32":
            # fp32 compute runs on the CUDA cores: nominal FMA peak
            peak, bound = 148 * 128 * 2 * 1.965e9 / 1e12, "fp32-simt"
            src = "nominal fp32 CUDA-core peak (148 SMs x 128 FMA/clk x 1965 MHz); no measured figure exists"
        else:
            peak, bound = peaks["tflops_sustained"], "tensor"
            src = f"{peaks['source']} bf16_tflops_sustained (kernel timed inside a long step)"
        roof = {"kernel": kind, "bound": bound, "achieved": achieved, "peak": peak,
                "unit": "TFLOP/s", "frac": achieved / peak, "traffic": traffic, "peak_source": src,
                "avg_launch_ms": kms / kn, "launches_profiled": kn,
                "algorithmic_flop_per_launch": per_launch}
    breakdown = {k: {"ms": round(v[0], 3), "launches": v[1]} for k, v in prof.items() if v[1] > 0}
    m.close()

    chunks_one = track_chunks(cfg, wl["seconds"], wl)
    if world == 1:
        desc = wl["desc"]
    elif sharded:
        desc = wl["desc"] + f"; one {wl['seconds']:g} s track over {world} ranks (strong scaling)"
    else:
        desc = wl["desc"] + (f"; {world} ranks, each separating its own {wl['seconds']:g} s track "
                             "(weak scaling: independent tracks, no exchange)")
    line = {
        "metric": "audio-seconds/sec", "value": value, "unit": "audio-s/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "vs_baseline": None, "dtype": "f16" if wl["dtype"] == "fp16" else wl["dtype"].replace("fp", "f"),
        "data": "synthetic: seeded pink noise (1/f, -18 dBFS RMS, 16-bit levels), random-init weights "
                "N(0,0.02), gamma=1",
        "config": {"workload": desc, "track_seconds": seconds,
                   "parallelism": (f"chunk-range shards x{world}" if sharded else
                                   f"one track per rank x{world}" if world > 1 else "single GPU"),
                   "chunks": run.chunks_total if sharded else chunks_one * world,
                   "max_chunks_per_rank": run.max_chunks_per_rank if sharded else chunks_one,
                   "l2": "no flush: the per-step working set (activations ~1 GB, mask-estimator weights "
                         "~400 MB) exceeds the 126 MB L2"},
        "roofline": roof, "profile_ms_per_step": breakdown, "e2e": e2e, "gpu_launches": int(launches),
        "scaling": args.scaling if world > 1 else "weak",
        "multi_gpu_check": check,
        "clocks": clk.summary(),
    }
    if not args.no_long_track and args.workload == "std":
        line["long_track"] = long_track(args, ctx)
    if rank == 0 and world == 1 and not args.no_cpu:
        cfg["_dtype"] = wl["dtype"]
        line["cpu_baseline"] = cpu_sample(csm, cfg, step_model_flops(cfg, seconds, wl), seconds, args.cpu_chunk,
                                          wl=wl, n_chunks=track_chunks(cfg, seconds, wl))
        line["cpu_baseline"].pop("sample_seconds", None)
    remove_model(csm, tmpdir)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def make_model(wl: dict, local: int, seed: int = 0):
    """A random-init .csm of the workload's preset in a temporary directory,
    loaded on GPU `local` in the workload's compute dtype."""
    import csm_tool
    import cudasep

    cfg = csm_tool.base_config(**csm_tool.PRESETS[wl["preset"]])
    tmpdir = tempfile.mkdtemp(prefix="mbr_bench_")
    csm = os.path.join(tmpdir, "model.csm")
    csm_tool.write_csm(csm, cfg, csm_tool.random_weights(cfg, seed))
    return cudasep.Model(csm, local, wl["dtype"]), cfg, csm, tmpdir


def remove_model(csm: str, tmpdir: str) -> None:
    try:
        os.remove(csm)
        os.rmdir(tmpdir)
    except OSError:
        pass


class TrackRun:
    """One timed separation path on this rank.

    sharded False: the rank's own whole track through mbr_separate_device
    (device-resident track in, stems out).  sharded True: the rank's
    contiguous chunk range of one track shared by all ranks — its input window
    on the device, mbr_shard_run_window, both overlap-add boundaries moved in
    one batched NCCL send/receive, mbr_shard_add_boundary, and
    mbr_shard_finalize into a buffer of its own output range."""

    def __init__(self, m, cfg, wl, track, ctx, sharded):
        import torch

        self.m, self.cfg, self.wl, self.track, self.ctx, self.sharded = m, cfg, wl, track, ctx, sharded
        dev, stream, rank, world = ctx["dev"], ctx["stream"], ctx["rank"], ctx["world"]
        self.S, self.C = m.info("num_stems"), m.info("channels")
        S, C = self.S, self.C
        N = self.N = track.shape[1]
        ov, cb = wl["overlap"], wl["chunk_batch"]
        if not sharded:
            self.d_track = torch.from_numpy(track).to(dev)
            self.d_out = torch.empty((S, C, N), dtype=torch.float32, device=dev)
            self.e2e_path = "mbr_separate (host track in, stems out; copies overlapped with the chunks)"
            return
        info = self.info = m.shard_info(N, ov, rank, world)
        self.w_lo, self.w_hi = m.shard_window(N, ov, rank, world)
        self.d_win = torch.from_numpy(track[:, self.w_lo:self.w_hi].copy()).to(dev)
        span = info["hi"] - info["lo"]
        self.acc = torch.empty((S * C, span), dtype=torch.float32, device=dev)
        self.wsum = torch.empty((span,), dtype=torch.float32, device=dev)
        prev = m.shard_info(N, ov, rank - 1, world) if rank > 0 else None
        self.rlen = prev["hi"] - prev["send_lo"] if prev else 0
        self.racc = torch.empty((S * C, max(self.rlen, 1)), dtype=torch.float32, device=dev)
        self.rws = torch.empty((max(self.rlen, 1),), dtype=torch.float32, device=dev)
        self.soff = info["send_lo"] - info["lo"]
        self.sacc = torch.empty((S * C, span - self.soff), dtype=torch.float32, device=dev)
        self.sws = torch.empty((span - self.soff,), dtype=torch.float32, device=dev)
        # the tail a rank sends is disjoint from the head it receives when every
        # rank holds at least chunk/step chunks: then all boundaries move at once
        self.plans = [m.shard_info(N, ov, r, world) for r in range(world)]
        assert all(self.plans[r - 1]["hi"] <= self.plans[r]["send_lo"] for r in range(1, world - 1)), \
            "too few chunks per rank for a concurrent boundary exchange"
        self.chunks_total = self.plans[-1]["c1"] - self.plans[0]["c0"]
        self.max_chunks_per_rank = max(pr["c1"] - pr["c0"] for pr in self.plans)
        self.wout = info["out_hi"] - info["out_lo"]
        self.d_own = torch.empty((S * C, max(self.wout, 1)), dtype=torch.float32, device=dev)
        self.e2e_path = "H2D of the rank's track window + mbr_shard_* + NCCL boundary exchange + D2H of the own range"

    def step(self):
        m, wl, ctx = self.m, self.wl, self.ctx
        stream, rank, world, dist = ctx["stream"], ctx["rank"], ctx["world"], ctx["dist"]
        ov, cb = wl["overlap"], wl["chunk_batch"]
        if not self.sharded:
            m.separate_device(self.d_track, ov, cb, out=self.d_out, stream=stream)
            return
        N, info = self.N, self.info
        m.shard_run_window(self.d_win, self.w_lo, N, ov, cb, rank, world, self.acc, self.wsum, stream=stream)
        ops = []
        if rank > 0:
            ops += [dist.P2POp(dist.irecv, self.racc, rank - 1), dist.P2POp(dist.irecv, self.rws, rank - 1)]
        if rank < world - 1:
            self.sacc.copy_(self.acc[:, self.soff:])
            self.sws.copy_(self.wsum[self.soff:])
            ops += [dist.P2POp(dist.isend, self.sacc, rank + 1), dist.P2POp(dist.isend, self.sws, rank + 1)]
        for req in dist.batch_isend_irecv(ops):
            req.wait()
        if rank > 0:
            m.shard_add_boundary(N, ov, rank, world, self.acc, self.wsum, self.racc, self.rws, self.rlen,
                                 stream=stream)
        if self.wout > 0:
            m.shard_finalize(N, ov, rank, world, self.acc, self.wsum, self.d_own, self.wout, stream=stream,
                             out_col0=info["out_lo"])

    def e2e(self, steps):
        """(ms per step, H2D bytes, D2H bytes) through the host entry points
        with pinned host buffers, max over ranks."""
        import torch

        dev, dist, world = self.ctx["dev"], self.ctx["dist"], self.ctx["world"]
        S, C, N, wl = self.S, self.C, self.N, self.wl
        h_in = torch.from_numpy(self.track).pin_memory()
        if not self.sharded:
            h_out = torch.empty((S, C, N), dtype=torch.float32).pin_memory()
            h_in_np, h_out_np = h_in.numpy(), h_out.numpy()

            def e2e_step():
                self.m.separate(h_in_np, wl["overlap"], wl["chunk_batch"], out=h_out_np)
            h2d, d2h = C * N * 4, S * C * N * 4
        else:
            h_win = h_in[:, self.w_lo:self.w_hi].contiguous().pin_memory()  # the rank's input window
            h_own = torch.empty((S * C, max(self.wout, 1)), dtype=torch.float32).pin_memory()

            def e2e_step():
                self.d_win.copy_(h_win, non_blocking=True)
                self.step()
                h_own.copy_(self.d_own, non_blocking=False)
            h2d, d2h = C * (self.w_hi - self.w_lo) * 4, S * C * self.wout * 4
        e2e_step()
        if dist:
            dist.barrier()
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        for _ in range(steps):
            e2e_step()
        torch.cuda.synchronize(dev)
        ms = (time.perf_counter() - t0) * 1e3 / steps
        if dist:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms, h2d, d2h

    def check(self):
        """Rank 0 assembles every rank's own output range and compares it with
        a one-GPU separation of the same track (collective: every rank calls)."""
        import torch

        dev, dist, rank, world, stream = (self.ctx[k] for k in ("dev", "dist", "rank", "world", "stream"))
        S, C, N, wl = self.S, self.C, self.N, self.wl
        wmax = torch.tensor([self.wout], device=dev)
        dist.all_reduce(wmax, op=dist.ReduceOp.MAX)
        pad = torch.zeros((S * C, int(wmax.item())), dtype=torch.float32, device=dev)
        pad[:, :self.wout] = self.d_own[:, :self.wout]
        parts = [torch.empty_like(pad) for _ in range(world)]
        dist.all_gather(parts, pad)
        out = None
        if rank == 0:
            one = self.m.separate_device(torch.from_numpy(self.track).to(dev), wl["overlap"], wl["chunk_batch"],
                                         stream=stream).view(S * C, N)
            torch.cuda.synchronize(dev)
            err = 0.0
            for r, pr in enumerate(self.plans):
                w = pr["out_hi"] - pr["out_lo"]
                err = max(err, float((parts[r][:, :w] - one[:, pr["out_lo"]:pr["out_hi"]]).abs().max()))
            out = {"max_abs_err_vs_one_gpu": err, "max_abs_one_gpu": float(one.abs().max())}
            del one
        dist.barrier()
        return out


def time_steps(run: TrackRun, warmup: int, steps: int, ctx: dict):
    """W untimed steps, then K steps bracketed by a barrier and a device sync
    on both sides, timed with CUDA events on the launching stream; returns
    (ms per step, max over ranks; kernel launches of one step)."""
    import torch

    dev, stream, dist = ctx["dev"], ctx["stream"], ctx["dist"]
    for _ in range(warmup):
        run.step()
    torch.cuda.synchronize(dev)
    run.m.sync_check()
    launches = run.m.last_launches()
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        run.step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    if dist:
        dist.barrier()
    ms = e0.elapsed_time(e1) / steps
    if dist:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    run.m.sync_check()
    return ms, launches


def long_track(args, ctx: dict) -> dict:
    """The long-track strong-scaling measurement that rides along every
    default run: the two-stem bf16 model on one 3-minute track, its chunk
    ranges sharded over all ranks (one GPU: the whole track), timed like the
    main line."""
    wl = WORKLOADS["two_stem"]
    m, cfg, csm, tmpdir = make_model(wl, ctx["local"])
    track = workload_track(wl, wl["seconds"], 1234)
    world = ctx["world"]
    run = TrackRun(m, cfg, wl, track, ctx, sharded=world > 1)
    steps = max(1, min(args.steps, 3))
    ms, _ = time_steps(run, 2, steps, ctx)
    e2e_ms, h2d, d2h = run.e2e(steps)
    check = run.check() if world > 1 else None
    chunks = track_chunks(cfg, wl["seconds"], wl)
    m.close()
    remove_model(csm, tmpdir)
    return {"workload": wl["desc"], "scaling": "strong", "n_gpus": world, "track_seconds": wl["seconds"],
            "value": wl["seconds"] / (ms / 1e3), "unit": "audio-s/s", "ms_per_step": ms, "steps": steps,
            "warmup": 2, "chunks": chunks,
            "max_chunks_per_rank": run.max_chunks_per_rank if world > 1 else chunks,
            "e2e": {"value": wl["seconds"] / (e2e_ms / 1e3), "unit": "audio-s/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "path": run.e2e_path},
            "multi_gpu_check": check}


def run_tensor_sweep(args):
    """Tensor API sweep (the reference tensor library's kernels): runs the
    native tensor_bench, which times every op alone after an L2 flush with CUDA
    events on the legacy stream the Tensor API uses, and summarises the
    fraction of the measured HBM copy peak per op."""
    peak = load_peaks()["hbm_gbs"]
    exe = os.path.join(PKG, "tensor_bench")
    if not os.path.exists(exe):
        raise SystemExit("tensor_bench missing: build with make -C mbr-cuda-tile_b200")
    out = subprocess.run([exe, str(max(args.steps, 1)), str(peak)], capture_output=True, text=True, check=True)
    rows = [json.loads(l) for l in out.stdout.splitlines() if l.startswith("{")]
    for r in rows:
        print(json.dumps(r), flush=True)
    summ = {}
    for r in rows:
        summ.setdefault(r["op"], []).append(r["frac"])
    print(json.dumps({"summary": "tensor_sweep", "peak_gbs": peak, "peak_source": load_peaks()["source"],
                      "per_op": {k: {"median": float(np.median(v)), "min": float(np.min(v)), "n": len(v)}
                                 for k, v in summ.items()}}), flush=True)
    return 0


def run_op_sweep(args):
    """Tensor-op sweep (the benchmark's op-sweep configuration): activations [B*801*60, D] seeded
    N(0, 1), D in {192, 384, 512}, B in {1, 4, 8}, fp32 / fp16 / bf16.  Each op
    is timed with CUDA events around one launch after an L2 flush (a 256 MiB
    write followed by a 256 MiB read, so the launch meets a cold L2 and none of
    the flush's dirty lines), averaged over `--steps` launches after `--warmup`; GB/s counts the
    algorithmic bytes (every input read once, every output written once)."""
    import torch

    import csm_tool
    import cudasep

    torch.cuda.set_device(0)
    peak = load_peaks()["hbm_gbs"]
    T, NB, J2 = 801, 60, 2 * 3958  # frames, bands, band-freq values (7916) of the 60-band split
    # L2 flush between launches: write a 256 MiB buffer, then read another one, so that the timed launch
    # starts with a cold L2 holding clean lines (the flush's own dirty lines are written back before it)
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
    flush_rd = torch.ones(64 << 20, dtype=torch.float32, device="cuda")
    flush_sum = torch.empty((), dtype=torch.float32, device="cuda")
    gen = torch.Generator(device="cuda").manual_seed(0)
    tdt = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}
    reps, warm = max(args.steps, 3), max(args.warmup, 1)
    # spin the GPU up (clocks leave their idle state) before the first timed case
    for _ in range(2000):
        flush.zero_()
    torch.cuda.synchronize()

    def timed(fn):
        for _ in range(warm):
            fn()
        tot = 0.0
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for _ in range(reps):
            flush.zero_()
            torch.sum(flush_rd, 0, out=flush_sum)
            # the GPU spins (~50 us) while the host issues the start event and the op, so the
            # event pair brackets the launch itself and not the Python and ctypes call overhead
            torch.cuda._sleep(100000)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            tot += e0.elapsed_time(e1)
        return tot / reps / 1e3

    results = []

    want_ops = set(o for o in args.ops.split(",") if o)

    def want(op):
        return not want_ops or op in want_ops

    def report(op, dtype, D, B, nbytes, sec):
        gbs = nbytes / sec / 1e9
        line = {"op": op, "dtype": dtype, "D": D, "B": B, "bytes": int(nbytes), "us": sec * 1e6, "GB/s": gbs,
                "frac_of_hbm_peak": gbs / peak}
        results.append(line)
        print(json.dumps(line), flush=True)

    with tempfile.TemporaryDirectory() as d:
        csm = os.path.join(d, "m.csm")
        cfg = csm_tool.base_config(**csm_tool.PRESETS["tiny"])
        csm_tool.write_csm(csm, cfg, csm_tool.random_weights(cfg, 0))
        model = cudasep.Model(csm, 0, "fp32")
        for dtype in [d for d in args.dtypes.split(",") if d]:
            dt, e = tdt[dtype], torch.tensor([], dtype=tdt[dtype]).element_size()
            for B in [int(b) for b in args.batches.split(",") if b]:
                rows = B * T * NB
                row_ops = ("copy", "rms_norm", "add", "gelu", "sigmoid_gate", "rope")
                for D in ((192, 384, 512) if any(want(o) for o in row_ops) else ()):
                    N = rows * D
                    x = torch.randn(rows, D, generator=gen, device="cuda").to(dt)
                    y = torch.empty_like(x)
                    gamma = torch.ones(D, device="cuda")
                    if want("copy"):
                        # reference line, not one of this library's ops: torch's own device copy of the
                        # same bytes under the same timing, i.e. what HBM gives a transfer of this size
                        report("copy", dtype, D, B, 2 * N * e, timed(lambda: y.copy_(x)))
                    if want("rms_norm"):
                        report("rms_norm", dtype, D, B, 2 * N * e + D * 4,
                               timed(lambda: cudasep.op_rms_norm(x, gamma, D ** 0.5, y=y)))
                    if want("add"):
                        x2 = torch.randn(rows, D, generator=gen, device="cuda").to(dt)
                        report("add", dtype, D, B, 3 * N * e, timed(lambda: cudasep.op_add(x, x2, y=y)))
                        del x2
                    if want("gelu"):
                        report("gelu", dtype, D, B, 2 * N * e, timed(lambda: cudasep.op_gelu(x, y=y)))
                    H = D // 64
                    gate = torch.rand(rows, H, generator=gen, device="cuda").to(dt)
                    if want("sigmoid_gate"):
                        report("sigmoid_gate", dtype, D, B, 2 * N * e + rows * H * e,
                               timed(lambda: cudasep.op_sigmoid_gate(x, gate, H, y=y)))
                    c, s_ = cudasep.rope_tables(T, 64)
                    ct, st = torch.from_numpy(c).cuda(), torch.from_numpy(s_).cuda()
                    xr, yr = x.view(B * NB, T, H, 64), y.view(B * NB, T, H, 64)
                    if want("rope"):
                        report("rope", dtype, D, B, 2 * N * e + 2 * c.nbytes,
                               timed(lambda: cudasep.op_rope(xr, ct, st, y=yr)))
                    del x, y, gate
                # band ops (independent of D)
                spec = torch.randn(B, 2, 1025, T, 2, generator=gen, device="cuda")
                xb = torch.empty(B, T, J2, dtype=dt, device="cuda")
                if want("band_gather"):
                    report("band_gather", dtype, 0, B, spec.numel() * 4 + xb.numel() * e,
                           timed(lambda: model.op_band_gather(spec, out_dtype=dt)))
                masks = torch.randn(1, B * T, J2, generator=gen, device="cuda").to(dt)
                if want("mask_scatter"):
                    report("mask_scatter", dtype, 0, B,
                           masks.numel() * e + spec.numel() * 4 + 1025 * 4 + B * 2 * 1025 * T * 2 * 4,
                           timed(lambda: model.op_mask_scatter(spec, masks)))
                del spec, xb, masks
        model.close()
    by_op = {}
    for r in results:
        if r["op"] != "copy":  # the reference line is not one of the ops
            by_op.setdefault(r["op"], []).append(r["frac_of_hbm_peak"])
    print(json.dumps({"metric": "tensor-op HBM GB/s vs peak", "peak_gbs": peak,
                      "peak_source": "MEASURED_PEAKS.json hbm_gbs (copy bandwidth)",
                      "median_frac_by_op": {k: sorted(v)[len(v) // 2] for k, v in by_op.items()},
                      "min_frac_by_op": {k: min(v) for k, v in by_op.items()}, "cases": len(results)}), flush=True)
    return 0


def run_single_chunk(args, wl):
    """warmup + steps forwards of one chunk batch of the workload (for ncu)."""
    import torch

    import csm_tool
    import cudasep

    cfg = csm_tool.base_config(**csm_tool.PRESETS[wl["preset"]])
    with tempfile.TemporaryDirectory() as d:
        csm = os.path.join(d, "model.csm")
        csm_tool.write_csm(csm, cfg, csm_tool.random_weights(cfg, 0))
        m = cudasep.Model(csm, 0, wl["dtype"])
        x = torch.from_numpy(np.stack([pink_noise(cfg["chunk_size"] / SR, 99 + i) for i in range(wl["chunk_batch"])]))
        x = x.cuda().contiguous()
        out = None
        for _ in range(args.warmup):
            out = m.forward(x, out=out)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            out = m.forward(x, out=out)
        e1.record()
        torch.cuda.synchronize()
        m.sync_check()
        print(json.dumps({"mode": "single_chunk", "workload": wl["desc"], "forwards": args.steps,
                          "ms_per_forward": e0.elapsed_time(e1) / max(args.steps, 1),
                          "launches_per_forward": m.last_launches()}), flush=True)
        m.close()
    return 0


def read_traffic(kind: str):
    """DRAM bytes per launch of `kind` from the committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", "ncu_traffic.txt")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        for line in f:
            parts = line.split()
            if len(parts) >= 2 and parts[0] == kind and not line.startswith("#"):
                try:
                    return float(parts[1])
                except ValueError:
                    return None
    return None


if __name__ == "__main__":
    sys.exit(main())
