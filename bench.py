#!/usr/bin/env python
"""Benchmark of the B200 synthesis engine (driver contract: one JSON line on rank 0).

Default workload: HOP synthesis of a 3840x2160 4:2:0 picture from
synthetic latents (luma 160x135x240, chroma 96x135x240, integer Laplace(1.5) with ~60% zeros)
in 512-sample tiles with a 16-sample overlap (40 tiles), random-init weights (seed 3), tiles
distributed round-robin over the ranks (tile i on rank i mod N), each rank's final layers
writing its cores as 8-bit YUV 4:2:0 samples (the fused output stage, quantize_plane_par in the
epilogue) and a final sum-reduce of the disjoint 8-bit cores to rank 0 over NCCL (the "final
gather"). One step = one picture. `--config sop1080` runs config 3 (SOP 1920x1080, one tile);
`--config conv1` / `up2` run configs 1 and 2 (a single conv layer; the upsampling stage)
through the conv-stage entry, as replicas when N > 1.

value: output Mpixel/s of the whole job, timed on the device (CUDA events bracketing each
step on the engine's stream, L2 flushed between steps, max over ranks). e2e: the same through
the public API with the inputs copied from pinned host memory and the output read back, every
step. roofline: the tcgen05 kernels (the implicit-GEMM convolution and the fused FFN, all
their launches of one step), algorithmic FLOPs (live MACs x 2) / summed CUDA-event duration,
against the measured bf16 dense peak. cpu_baseline and --impl reference: the crate's nn::fast
CPU algorithm restated in oracle/fast.c (bit-identical to the oracle's nn::reference loops) on
the box's host cores, counting output (core) pixels only: the reference arm sweeps the
picture's tile rows, one per step; cpu_baseline times one tile row on all threads and one tile
on one thread.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
       (N > 1 under torchrun, one process per GPU)
"""

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SYNTH_METRIC = "synthesis decode Mpixel/s"
STAGE_METRIC = "conv stage output Mpixel/s"
CONFIGS = {
    "hop4k": dict(kind="synth", op="hop", H=2160, W=3840, tile=512, overlap=16, seed=3,
                  lat_seed=100, metric=SYNTH_METRIC, scaling="strong",
                  desc="BASELINE config 4: HOP synthesis, 3840x2160 4:2:0, 512/16 tiles"),
    "sop1080": dict(kind="synth", op="sop", H=1080, W=1920, tile=0, overlap=0, seed=2,
                    lat_seed=100, metric=SYNTH_METRIC, scaling="strong", law="he",
                    desc="BASELINE config 3: SOP synthesis, 1920x1080 4:2:0, one tile"),
    "bop_batch64": dict(kind="batch", op="bop", H=1024, W=1024, npic=64, per_call=8, seed=4,
                        metric="batched decode + analysis Mpixel/s", scaling="strong",
                        desc="BASELINE config 5: 64 BOP 1024x1024 4:4:4 pictures, RGB analysis "
                             "+ synthesis, pictures round-robin over the GPUs, 8 per call"),
    "conv1": dict(kind="stage", shuffle=1, act="leaky", nres=0, metric=STAGE_METRIC,
                  scaling="weak",
                  desc="BASELINE config 1: conv 3x3 128->128 on 128x128, LeakyReLU(0.01)",
                  weights="N(0, 1/(9*128)) weights, N(0, 0.01^2) bias, seed 0"),
    "up2": dict(kind="stage", shuffle=2, act=None, nres=2, metric=STAGE_METRIC, scaling="weak",
                desc="BASELINE config 2: conv 3x3 192->512 + depth-to-space 2 on 68x120, two "
                     "residual blocks (conv3x3-LeakyReLU-conv3x3 + skip) at 128 channels",
                weights="He-normal weights, zero biases, seed 1"),
}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), "measured (MEASURED_PEAKS.json bf16_tflops, burst)"
    except Exception:
        return 1590.0, "fallback (1.59 PFLOP/s)"


def conv_traffic(config, algorithmic_bytes):
    """DRAM bytes (read + write) of one step's tcgen05 kernel launches (conv_tc_kernel and
    ffn_tc_kernel): the step's algorithmic bytes times the DRAM-to-algorithmic ratio measured
    by ncu on a small case of the same workload, from the committed capture summary
    profiles/tcgen05_<config>_step_dram.txt (`traffic_per_algorithmic_byte: r`), or None."""
    path = os.path.join(ROOT, "profiles", "tcgen05_%s_step_dram.txt" % config)
    try:
        with open(path) as f:
            for ln in f:
                if ln.startswith("traffic_per_algorithmic_byte:"):
                    return float(ln.split(":", 1)[1]) * algorithmic_bytes
    except OSError:
        pass
    return None


class ClockSampler:
    """SM clock and clock-event (throttle) reasons of the bench's GPU, sampled every 10 ms by
    NVML (read-only queries) from before the timed region to after it; only the samples taken
    inside the timed window (`mark_start` .. `mark_stop`) are reported, or the first one after
    it when the window is shorter than the sampling period. Falls back to `nvidia-smi -lms 200`
    when NVML is unavailable."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clocks-event reason bits
    REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
               "hw_thermal_slowdown": 0x40}

    def __init__(self, gpu):
        self.gpu = gpu
        self.proc = None
        self.nvml = None
        self.lines = []
        self.samples = []  # (time, sm_mhz, max_mhz, reason bits)
        self.t0 = self.t1 = None
        self.running = False

    def start(self):
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            try:
                bus = torch.cuda.get_device_properties(self.gpu).pci_bus_id
                h = pynvml.nvmlDeviceGetHandleByPciBusId(
                    "%08X:%02X:%02X.0" % (torch.cuda.get_device_properties(self.gpu).pci_domain_id,
                                          bus, torch.cuda.get_device_properties(self.gpu).pci_device_id))
            except Exception:
                h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            self.nvml, self.handle = pynvml, h
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            self.running = True
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
            return
        except Exception:
            self.nvml = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.FIELDS,
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _poll(self):
        nv, h = self.nvml, self.handle
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            getattr(nv, "nvmlDeviceGetCurrentClocksThrottleReasons")
        while self.running:
            try:
                self.samples.append((time.monotonic(),
                                     float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)),
                                     self.max_mhz, int(get_reasons(h))))
            except Exception:
                pass
            time.sleep(0.01)

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def mark_start(self):
        self.t0 = time.monotonic()

    def mark_stop(self):
        self.t1 = time.monotonic()

    def stop(self):
        if self.nvml:
            time.sleep(0.03)  # at least one sample after the window
            self.running = False
            self.thread.join(timeout=1)
            t0 = self.t0 if self.t0 is not None else 0.0
            t1 = self.t1 if self.t1 is not None else float("inf")
            win = [s for s in self.samples if t0 <= s[0] <= t1]
            if not win:
                win = [s for s in self.samples if s[0] > t1][:1]
            reasons = set()
            for s in win:
                for nm, bit in self.REASONS.items():
                    if s[3] & bit:
                        reasons.add(nm)
            sm = [s[1] for s in win]
            return {"sm_mhz": float(np.median(sm)) if sm else None,
                    "sm_max_mhz": self.max_mhz, "reasons": sorted(reasons),
                    "samples": len(sm), "source": "nvml, 10 ms"}
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvidia-smi, 200 ms"}


# ---------------------------------------------------------------------------------------------
# CPU side: the crate's nn::fast algorithm restated in oracle/fast.c (bit-identical to the
# oracle's nn::reference loops), timed on the box's host cores
# ---------------------------------------------------------------------------------------------

def synth_params(cfg):
    """The synthesis weights of a config: the He-normal law where BASELINE prescribes it
    (config 3), else the role-scaled random init (synthetic.make_params)."""
    import synthetic as syn
    if cfg.get("law") == "he":
        return syn.synthesis_params_he(cfg["op"], cfg["seed"])
    return syn.synthesis_params(cfg["op"], cfg["seed"])


def weights_desc(cfg):
    if cfg.get("law") == "he":
        return "random-init, seed %d, He-normal N(0, 2 / fan_in) (the prescribed law)" % cfg["seed"]
    return "random-init, seed %d (role-scaled normal)" % cfg["seed"]


def _tile_rows(cfg):
    """The workload's tiles (oracle tiling, tools/tiles.rs:39-119) grouped by tile row."""
    import oracle as zo
    H, W = cfg["H"], cfg["W"]
    lh, lw = -(-H // 16), -(-W // 16)
    tiles = zo.synthesis_tiles(H, W, lh, lw, cfg["tile"], cfg["overlap"])
    rows = {}
    for t in tiles:
        rows.setdefault(t["img_y"], []).append(t)
    return [rows[k] for k in sorted(rows)]


class CpuSynth:
    """The CPU baseline of a synthesis config: luma + chroma synthesis of whole tiles (overlap
    included, as the crate computes them), counting only the tiles' core (output) pixels."""

    def __init__(self, cfg):
        import oracle as zo
        import synthetic as syn
        self.zo, self.cfg = zo, cfg
        H, W = cfg["H"], cfg["W"]
        lh, lw = -(-H // 16), -(-W // 16)
        py, puv = synth_params(cfg)
        self.cky, self.ckuv = zo.Checkpoint(py), zo.Checkpoint(puv)
        self.ly = syn.laplace_latent(cfg["lat_seed"], "ly", (160, lh, lw), 1.5)
        self.luv = syn.laplace_latent(cfg["lat_seed"], "luv", (96, lh, lw), 1.5)
        self.rows = _tile_rows(cfg)

    def run(self, tiles, threads):
        """(core pixels, seconds) of synthesising `tiles` on `threads` host threads."""
        zo = self.zo
        zo.set_fast(True)
        zo.set_threads(threads)
        op = zo.OPS[self.cfg["op"]]
        px = 0
        t0 = time.perf_counter()
        for t in tiles:
            win = (slice(None), slice(t["lat_y"], t["lat_y"] + t["lat_h"]),
                   slice(t["lat_x"], t["lat_x"] + t["lat_w"]))
            wy = np.ascontiguousarray(self.ly[win])
            wuv = np.ascontiguousarray(self.luv[win])
            zo.synthesis_primary(self.cky, op, wy, t["img_h"], t["img_w"])
            zo.synthesis_secondary(self.ckuv, op, wy, wuv, t["img_h"], t["img_w"])
            px += t["core_h"] * t["core_w"]
        return px, time.perf_counter() - t0


class CpuStage:
    """The CPU baseline of a conv-stage config: the same layers composed from the oracle's
    primitives (conv, pixel shuffle, LeakyReLU, residual add) on the nn::fast restatement."""

    def __init__(self, cfg):
        import oracle as zo
        import synthetic as syn
        self.zo, self.cfg = zo, cfg
        self.prm, self.x = stage_inputs(cfg)

    def run(self, threads):
        zo, cfg, prm = self.zo, self.cfg, self.prm
        zo.set_fast(True)
        zo.set_threads(threads)
        t0 = time.perf_counter()
        y = zo.conv2d(self.x, prm["conv.weight"], prm["conv.bias"], pad=(1, 1))
        if cfg["act"] == "leaky":
            y = zo.leaky_relu(y)
        if cfg["shuffle"] > 1:
            y = zo.pixel_shuffle(y, cfg["shuffle"])
        for i in range(cfg["nres"]):
            p = "res.%d." % i
            t = zo.leaky_relu(zo.conv2d(y, prm[p + "conv1.weight"], prm[p + "conv1.bias"],
                                        pad=(1, 1)))
            y = zo.add(zo.conv2d(t, prm[p + "conv2.weight"], prm[p + "conv2.bias"],
                                 pad=(1, 1)), y)
        return y.shape[1] * y.shape[2], time.perf_counter() - t0


def batch_picture(cfg, i):
    """Picture i of config 5: its latents (Laplace(2.0), seed 100 + i) and its RGB picture
    (uniform 8-bit samples, seed 1100 + i)."""
    import synthetic as syn
    lh, lw = cfg["H"] // 16, cfg["W"] // 16
    ly = syn.laplace_latent(100 + i, "ly", (160, lh, lw), 2.0)
    luv = syn.laplace_latent(100 + i, "luv", (96, lh, lw), 2.0)
    rgb = np.floor(syn.uniform(1100 + i, "rgb", (cfg["H"], cfg["W"], 3), 0.0, 256.0))
    return ly, luv, rgb.astype(np.uint8)


class CpuBatch:
    """The CPU baseline of config 5: per picture, preprocess_rgb + both analysis transforms and
    the 4:4:4 synthesis of its latents, on the nn::fast restatement."""

    def __init__(self, cfg):
        import oracle as zo
        import synthetic as syn
        self.zo, self.cfg = zo, cfg
        py, puv = syn.synthesis_params(cfg["op"], cfg["seed"])
        pa, pauv = syn.analysis_params(cfg["op"], cfg["seed"])
        self.ck = [zo.Checkpoint(p) for p in (py, puv, pa, pauv)]

    def run(self, i, threads):
        zo, cfg = self.zo, self.cfg
        zo.set_fast(True)
        zo.set_threads(threads)
        op = zo.OPS[cfg["op"]]
        ly, luv, rgb = batch_picture(cfg, i)
        t0 = time.perf_counter()
        luma, chroma = zo.preprocess_rgb(rgb)
        zo.analyze_tiled(self.ck[2], op, 0, luma)
        zo.analyze_tiled(self.ck[3], op, 1, chroma)
        zo.synthesize(self.ck[0], self.ck[1], op, ly, luv, cfg["H"], cfg["W"], sv=1, sh=1)
        return cfg["H"] * cfg["W"], time.perf_counter() - t0


def stage_inputs(cfg):
    import synthetic as syn
    if cfg["name"] == "conv1":
        return syn.conv_layer_params(0), syn.uniform(0, "x", (128, 128, 128), -1.0, 1.0)
    return syn.upsample_stage_params(1), syn.normal(1, "x", (192, 68, 120))


def cpu_baseline(cfg):
    """Rank 0, N = 1: the nn::fast restatement on all host threads and on one thread, on a
    bounded sample of the workload (a few seconds each)."""
    threads = os.cpu_count() or 1
    if cfg["kind"] == "batch":
        c = CpuBatch(cfg)
        px, dt = c.run(0, threads)
        px1, dt1 = c.run(1, 1)
        return {"value": px / dt / 1e6, "unit": "Mpixel/s", "cores": threads, "kind": "port",
                "value_1core": px1 / dt1 / 1e6,
                "sample": "picture 0 (RGB analysis + synthesis) on %d threads, picture 1 on one "
                          "thread; oracle/fast.c, the crate's nn::fast convolution algorithm "
                          "restated (bit-identical to nn::reference)" % threads}
    if cfg["kind"] == "stage":
        c = CpuStage(cfg)
        c.run(threads)
        px, dt = c.run(threads)
        px1, dt1 = c.run(1)
        return {"value": px / dt / 1e6, "unit": "Mpixel/s", "cores": threads, "kind": "port",
                "value_1core": px1 / dt1 / 1e6,
                "sample": "the whole stage once (oracle/fast.c, the crate's nn::fast "
                          "convolution algorithm restated, bit-identical to nn::reference)"}
    c = CpuSynth(cfg)
    rows = c.rows
    row = rows[1] if len(rows) > 1 else rows[0]  # an interior tile row
    px, dt = c.run(row, threads)
    px1, dt1 = c.run(row[:1], 1)
    return {"value": px / dt / 1e6, "unit": "Mpixel/s", "cores": threads, "kind": "port",
            "value_1core": px1 / dt1 / 1e6,
            "sample": "tile row 1 (%d tiles, luma + chroma, output pixels of their cores) on %d "
                      "threads; its first tile on 1 thread; oracle/fast.c, the crate's nn::fast "
                      "convolution algorithm restated (bit-identical to nn::reference)"
                      % (len(row), threads)}


def config_dict(args, cfg, world):
    """The workload description both arms print (the same dict)."""
    if cfg["kind"] == "batch":
        return {"workload": args.config + ": " + cfg["desc"],
                "pictures": cfg["npic"],
                "parallelism": "pictures round-robin over %d GPU(s), no collective" % world,
                "weights": "random-init, seed %d (role-scaled normal)" % cfg["seed"],
                "l2": "flushed between steps (256 MiB write, outside the timed events)",
                "precision": "f16 operands, f32 accumulation (TMEM); the CPU arm computes f32"}
    if cfg["kind"] == "stage":
        return {"workload": args.config + ": " + cfg["desc"],
                "parallelism": "replicas: the same stage on each of %d GPU(s)" % world,
                "weights": cfg["weights"],
                "precision": "f16 operands, f32 accumulation (TMEM); the CPU arm computes f32"}
    return {"workload": args.config + ": " + cfg["desc"],
            "picture": "%dx%d 4:2:0, 8-bit YUV out" % (cfg["W"], cfg["H"]),
            "tiles": cfg.get("ntiles"),
            "parallelism": "tiles round-robin over %d GPU(s), each rank sent only the latent "
                           "rows / columns its tiles read" % world,
            "gather": cfg.get("gather", "none (one GPU)") if world > 1 else "none (one GPU)",
            "weights": weights_desc(cfg),
            "l2": "flushed between steps (256 MiB write, outside the timed events)",
            "precision": "f16 operands, f32 accumulation (TMEM); the CPU arm computes f32"}


def run_reference(args, cfg):
    """The reference's CPU path (the nn::fast restatement in oracle/, on every host thread) on
    the same workload: each step synthesises one tile row (the rows taken in turn, so the steps
    sweep the whole picture) and counts the output pixels of its tiles' cores. Imports nothing
    from the GPU package."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if cfg["kind"] == "batch":
        c = CpuBatch(cfg)
        run = lambda s: c.run(s % cfg["npic"], threads)
        sample = "one picture per step (RGB analysis + synthesis), pictures in turn"
    elif cfg["kind"] == "stage":
        c = CpuStage(cfg)
        run = lambda s: c.run(threads)
        sample = "the whole stage per step"
    else:
        c = CpuSynth(cfg)
        nrow = len(c.rows)
        run = lambda s: c.run(c.rows[s % nrow], threads)
        sample = ("one tile row per step (%d rows in turn, %d tiles in all), luma + chroma, "
                  "output pixels of the cores" % (nrow, sum(len(r) for r in c.rows)))
    for s in range(args.warmup):
        run(s)
    px = dt = 0.0
    for s in range(args.steps):
        p, d = run(args.warmup + s)
        px += p
        dt += d
    v = px / dt / 1e6
    line = {
        "impl": "reference", "metric": cfg["metric"], "value": v, "unit": "Mpixel/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
        "scaling": cfg["scaling"], "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_dict(args, cfg, world),
        "cpu_baseline": {"value": v, "unit": "Mpixel/s", "cores": threads, "kind": "port",
                         "sample": sample + "; oracle/fast.c, the crate's nn::fast convolution "
                                            "algorithm restated (bit-identical to nn::reference)"},
        "e2e": {"value": v, "unit": "Mpixel/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "the reference crate (Rust) cannot be built here (no Rust toolchain); its CPU "
                "path is timed through its algorithm restated in C (oracle/)",
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------
# GPU side
# ---------------------------------------------------------------------------------------------

def profile_step(eng, step, flush):
    """Summed CUDA-event ms, algorithmic FLOPs, algorithmic bytes and launches of the tcgen05
    kernels over one profiled step."""
    import ctypes
    import torch
    from zenjpegai_b200 import _lib
    L = _lib.lib()
    L.zjai_ctx_profile(eng.handle, 1)
    flush.zero_()
    torch.cuda.synchronize()
    step()
    ms, fl, by, nl = ctypes.c_double(), ctypes.c_double(), ctypes.c_double(), ctypes.c_int64()
    L.zjai_ctx_profile_read_bytes(eng.handle, ctypes.byref(ms), ctypes.byref(fl),
                                  ctypes.byref(by), ctypes.byref(nl))
    L.zjai_ctx_profile(eng.handle, 0)
    return ms.value, fl.value, by.value, nl.value


def layer_report(eng):
    import ctypes
    from zenjpegai_b200 import _lib
    buf = ctypes.create_string_buffer(1 << 20)
    _lib.lib().zjai_ctx_profile_report(eng.handle, buf, len(buf))
    rows = [ln.split("\t") for ln in buf.value.decode().splitlines()[1:]]
    rows.sort(key=lambda r: -float(r[2]))
    sys.stderr.write("per-layer kernel time of one step, luma and chroma serialised "
                     "(layer, launches, ms, GFLOP, TFLOP/s, GB, GB/s):\n")
    for r in rows:
        sys.stderr.write("  %-48s %4s %9s %9s %7s %8s %6s\n" % tuple(r))
    kinds = {}
    for r in rows:
        k = r[0].split("[")[-1].rstrip("]") if r[0].endswith("]") else "conv"
        kinds[k] = kinds.get(k, 0.0) + float(r[2])
    sys.stderr.write("per kernel kind (ms): %s\n" % ", ".join(
        "%s %.3f" % kv for kv in sorted(kinds.items(), key=lambda kv: -kv[1])))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="hop4k", choices=sorted(CONFIGS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", action="store_true",
                    help="print the per-layer conv time of one profiled step to stderr")
    ap.add_argument("--picture", default=None, metavar="WxH",
                    help="a synthesis config on a smaller picture of the same tiling (the small "
                         "case of the profiles' DRAM captures); the line then carries no traffic")
    ap.add_argument("--arena-gb", type=int, default=0,
                    help="device arena of the engine in GiB (default: the config's)")
    args = ap.parse_args()
    cfg = dict(CONFIGS[args.config], name=args.config)
    if args.picture:
        if cfg["kind"] != "synth":
            ap.error("--picture applies to the synthesis configs")
        pw, ph = (int(v) for v in args.picture.lower().split("x"))
        cfg.update(W=pw, H=ph, desc=cfg["desc"] + " (picture %dx%d)" % (pw, ph))
    if cfg["kind"] == "synth":
        H, W = cfg["H"], cfg["W"]
        cfg["ntiles"] = sum(len(r) for r in _tile_rows(cfg)) if cfg["tile"] else 1
    if args.impl == "reference":
        return run_reference(args, cfg)

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))

    import synthetic as syn
    import zenjpegai_b200 as zj
    from zenjpegai_b200 import sharding
    from zenjpegai_b200.decoder import Decoder

    arena = args.arena_gb << 30 if args.arena_gb else \
        {"synth": 64 << 30, "batch": 32 << 30}.get(cfg["kind"], 4 << 30)
    eng = zj.Engine(local, arena_bytes=arena)
    # one non-default stream shared by torch (copies, events, NCCL) and the engine
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    eng.set_stream(stream.cuda_stream)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    closers = []

    if cfg["kind"] == "synth":
        op = cfg["op"]
        lh, lw = -(-H // 16), -(-W // 16)
        ch, cw = -(-H // 2), -(-W // 2)
        py, puv = synth_params(cfg)
        dec = Decoder(eng, op, py, puv)
        closers.append(dec.close)
        # every step is the same call on the same buffers: replayed as a CUDA graph (captured
        # on the second call; the warm-up steps include both)
        eng.set_graphs(True)
        ly_h = torch.from_numpy(syn.laplace_latent(cfg["lat_seed"], "ly", (160, lh, lw), 1.5))
        luv_h = torch.from_numpy(syn.laplace_latent(cfg["lat_seed"], "luv", (96, lh, lw), 1.5))
        ly_h, luv_h = ly_h.pin_memory(), luv_h.pin_memory()
        ly, luv = ly_h.cuda(), luv_h.cuda()
        tiles = zj.synthesis_tiles(H, W, lh, lw, cfg["tile"], cfg["overlap"])
        mine = sharding.shard_tiles(tiles, rank, world)
        if world > 1:
            # each rank receives only the latent rows / columns its tiles read
            ly_h, luv_h, mine = sharding.compact_latent(mine, ly_h, luv_h)
            ly_h, luv_h = ly_h.pin_memory(), luv_h.pin_memory()
            ly, luv = ly_h.cuda(), luv_h.cuda()
        out8 = torch.zeros(H * W + 2 * ch * cw, dtype=torch.uint8, device="cuda")
        sizes = (H * W, ch * cw, ch * cw)
        # the 8-bit planes of the picture, written by the final layers (fused output stage)
        planes8 = (out8[:H * W].view(H, W), out8[H * W:H * W + ch * cw].view(ch, cw),
                   out8[H * W + ch * cw:].view(ch, cw))
        out8_host = torch.empty_like(out8, device="cpu").pin_memory()
        out_px = H * W
        peer = None
        if world > 1:
            # final gather: every rank's epilogue writes its cores into rank 0's planes over
            # NVLink (CUDA IPC); the NCCL sum-reduce of zero-elsewhere planes where it cannot
            peer = sharding.PeerPlanes(eng, dist, out8 if rank == 0 else None, sizes)
            if peer.ok:
                closers.append(peer.close)
            else:
                peer = None
        cfg["gather"] = ("NVLink peer writes of the 8-bit cores into rank 0's planes (CUDA IPC)"
                         if peer else "NCCL reduce of zero-elsewhere 8-bit planes")
        h2d_t = torch.tensor([float(ly_h.numel() + luv_h.numel()) * 4], dtype=torch.float64,
                             device="cuda")
        if world > 1:
            dist.all_reduce(h2d_t)
        h2d = int(h2d_t.item())
        d2h = out8.numel()

        def step(from_host=False):
            if from_host:
                ly.copy_(ly_h, non_blocking=True)
                luv.copy_(luv_h, non_blocking=True)
            if peer is not None:
                dec.synthesize_tiles(ly, luv, mine, H, W, out=peer.planes, bit_depth=8)
                peer.done()
            else:
                if world > 1:
                    # the reduce sums the ranks' disjoint cores: every rank starts from zero
                    out8.zero_()
                dec.synthesize_tiles(ly, luv, mine, H, W, out=planes8, bit_depth=8)
                sharding.gather_cores(out8, dist)
            if from_host and rank == 0:
                out8_host.copy_(out8, non_blocking=True)
    elif cfg["kind"] == "batch":
        from zenjpegai_b200.decoder import Encoder
        op = cfg["op"]
        py, puv = syn.synthesis_params(op, cfg["seed"])
        pa, pauv = syn.analysis_params(op, cfg["seed"])
        dec = Decoder(eng, op, py, puv)
        enc = Encoder(eng, op, pa, pauv)
        closers += [dec.close, enc.close]
        mine = [i for i in range(cfg["npic"]) if i % world == rank]
        pics = [batch_picture(cfg, i) for i in mine]
        ly_h = torch.from_numpy(np.stack([p[0] for p in pics])).pin_memory()
        luv_h = torch.from_numpy(np.stack([p[1] for p in pics])).pin_memory()
        rgb_h = torch.from_numpy(np.stack([p[2] for p in pics])).pin_memory()
        ly, luv, rgb = ly_h.cuda(), luv_h.cuda(), rgb_h.cuda()
        n, Hb, Wb = len(mine), cfg["H"], cfg["W"]
        planes = (torch.empty((n, Hb, Wb), dtype=torch.uint8, device="cuda"),
                  torch.empty((n, Hb, Wb), dtype=torch.uint8, device="cuda"),
                  torch.empty((n, Hb, Wb), dtype=torch.uint8, device="cuda"))
        lat_out = (torch.empty((n, 160, Hb // 16, Wb // 16), device="cuda"),
                   torch.empty((n, 96, Hb // 16, Wb // 16), device="cuda"))
        planes_h = tuple(torch.empty(p.shape, dtype=p.dtype).pin_memory() for p in planes)
        lat_h = tuple(torch.empty(l.shape).pin_memory() for l in lat_out)
        calls = [(a, min(a + cfg["per_call"], n)) for a in range(0, n, cfg["per_call"])]
        out_px = cfg["npic"] * Hb * Wb
        h2d = sum(t.numel() * t.element_size() for t in (ly_h, luv_h, rgb_h)) * world
        d2h = sum(t.numel() * t.element_size() for t in planes_h + lat_h) * world

        def step(from_host=False):
            if from_host:
                for d, hbuf in ((ly, ly_h), (luv, luv_h), (rgb, rgb_h)):
                    d.copy_(hbuf, non_blocking=True)
            for a, b in calls:
                enc.analyze_rgb(rgb[a:b], out=(lat_out[0][a:b], lat_out[1][a:b]))
                dec.synthesize_batch(ly[a:b], luv[a:b], Hb, Wb, sv=1, sh=1, bit_depth=8,
                                     out=(planes[0][a:b], planes[1][a:b], planes[2][a:b]))
            if from_host:
                for d, hbuf in zip(planes + lat_out, planes_h + lat_h):
                    hbuf.copy_(d, non_blocking=True)
    else:
        prm, x_np = stage_inputs(cfg)
        st = zj.Stage(eng, prm, shuffle=cfg["shuffle"],
                      act=zj.ACT_LEAKY if cfg["act"] == "leaky" else zj.ACT_NONE,
                      res_act=zj.ACT_LEAKY)
        closers.append(st.close)
        x_h = torch.from_numpy(x_np).pin_memory()
        x_d = x_h.cuda()
        r = cfg["shuffle"]
        oshape = (st.cout, x_np.shape[1] * r, x_np.shape[2] * r)
        y_d = torch.empty(oshape, device="cuda")
        y_h = torch.empty(oshape).pin_memory()
        out_px = oshape[1] * oshape[2] * world  # replicas: every rank's output counts
        h2d = x_h.numel() * 4
        d2h = y_h.numel() * 4

        def step(from_host=False):
            if from_host:
                x_d.copy_(x_h, non_blocking=True)
            st.forward(x_d, out=y_d)
            if from_host:
                y_h.copy_(y_d, non_blocking=True)

    def timed(n, from_host=False):
        total = 0.0
        for _ in range(n):
            flush.zero_()
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            step(from_host)
            b.record(stream)
            torch.cuda.synchronize()
            total += a.elapsed_time(b)
        t = torch.tensor([total], dtype=torch.float64, device="cuda")
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        step()
    eng.sync()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.05)
    n0 = eng.launch_count
    clocks.mark_start()
    total_ms = timed(args.steps)
    clocks.mark_stop()
    launches = eng.launch_count - n0
    clk = clocks.stop()
    eng.sync()
    e2e_ms = timed(args.steps, from_host=True)
    # live roofline of the tcgen05 kernels over one profiled step
    conv_ms, conv_fl, conv_by, conv_n = profile_step(eng, step, flush)
    if args.layers and rank == 0:
        layer_report(eng)
    stats = torch.tensor([conv_ms, conv_fl, conv_by, float(conv_n), float(launches)],
                         dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.SUM)
    conv_ms, conv_fl, conv_by, conv_n, all_launches = (float(x) for x in stats.tolist())

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(cfg)

    if rank == 0:
        peak, peak_src = peaks()
        achieved = conv_fl / (conv_ms / 1e3) / 1e12 if conv_ms > 0 else 0.0
        traffic = (conv_traffic(args.config, conv_by)
                   if world == 1 and not args.picture else None)
        line = {
            "metric": cfg["metric"],
            "value": args.steps * out_px / 1e6 / (total_ms / 1e3),
            "unit": "Mpixel/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps,
            "higher_is_better": True,
            "scaling": cfg["scaling"],
            "vs_baseline": None,
            "dtype": "f16",
            "data": "synthetic",
            "config": config_dict(args, cfg, world),
            "roofline": {
                "bound": "tensor",
                "kernel": "conv_tc_kernel + ffn_tc_kernel (tcgen05 implicit-GEMM conv and fused "
                          "FFN, all launches of a step)",
                "achieved": achieved,
                "peak": peak,
                "unit": "TFLOP/s",
                "frac": achieved / peak,
                "peak_source": peak_src,
                "launches_per_step": conv_n,
                "flops_per_step": conv_fl,
                # each launch's input, live weights, output and residual operands once: the
                # figure `traffic` is to be compared with
                "algorithmic_bytes_per_step": conv_by,
                # DRAM bytes of one step's tcgen05 launches: the algorithmic bytes times the
                # DRAM / algorithmic ratio ncu measured on a small case of this workload
                # (profiles/tcgen05_<config>_step_dram.txt), reported at N = 1 only
                "traffic": traffic,
                "traffic_unit": "bytes per step (DRAM read + write, ncu on a small case, "
                                "scaled by algorithmic bytes; a lower bound)",
            },
            "cpu_baseline": cpu,
            "e2e": {
                "value": args.steps * out_px / 1e6 / (e2e_ms / 1e3),
                "unit": "Mpixel/s",
                "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
            },
            "clocks": clk,
            "gpu_launches": int(all_launches),
        }
        print(json.dumps(line), flush=True)
    for c in closers:
        c()
    eng.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
