#!/usr/bin/env python
"""Benchmark of the B200 synthesis engine (driver contract: one JSON line on rank 0).

Default workload: HOP synthesis of a 3840x2160 4:2:0 picture from
synthetic latents (luma 160x135x240, chroma 96x135x240, integer Laplace(1.5) with ~60% zeros)
in 512-sample tiles with a 16-sample overlap (40 tiles), random-init weights (seed 3), tiles
distributed round-robin over the ranks (tile i on rank i mod N), each rank's final layers
writing its cores as 8-bit YUV 4:2:0 samples (the fused output stage, quantize_plane_par in the
epilogue) and a final sum-reduce of the disjoint 8-bit cores to rank 0 over
NCCL (the "final gather"). One step = one picture. `--config sop1080` runs config 3 (SOP
1920x1080, one tile).

value: output Mpixel/s of the whole job, timed on the device (CUDA events bracketing each
step on the engine's stream, L2 flushed between steps, max over ranks). e2e: the same through
the public API with the latents copied from pinned host memory and the 8-bit picture read
back, every step. roofline: the tcgen05 kernels (the implicit-GEMM convolution and the fused
FFN, all their launches of one step), algorithmic FLOPs (live MACs x 2) / summed CUDA-event
duration, against the measured bf16 dense peak. cpu_baseline / --impl reference: the CPU oracle (a C restatement of the crate's
f32 path) on a bounded sample of the same workload, all host threads.

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

CONFIGS = {
    "hop4k": dict(op="hop", H=2160, W=3840, tile=512, overlap=16, seed=3, lat_seed=100,
                  desc="BASELINE config 4: HOP synthesis, 3840x2160 4:2:0, 512/16 tiles"),
    "sop1080": dict(op="sop", H=1080, W=1920, tile=0, overlap=0, seed=2, lat_seed=100,
                    desc="BASELINE config 3: SOP synthesis, 1920x1080 4:2:0, one tile"),
}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), "measured (MEASURED_PEAKS.json bf16_tflops, burst)"
    except Exception:
        return 1590.0, "fallback (1.59 PFLOP/s)"


def conv_traffic(config):
    """DRAM bytes (read + write) of one step's tcgen05 kernel launches (conv_tc_kernel and
    ffn_tc_kernel), from the committed ncu capture summary
    profiles/tcgen05_<config>_step_dram.txt (`dram_bytes_per_step: N`), or None."""
    path = os.path.join(ROOT, "profiles", "tcgen05_%s_step_dram.txt" % config)
    try:
        with open(path) as f:
            for ln in f:
                if ln.startswith("dram_bytes_per_step:"):
                    return float(ln.split(":", 1)[1])
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


def cpu_sample(cfg, threads):
    """The oracle on one full-size tile (luma + chroma) of the workload: (Mpixel/s, desc)."""
    import oracle as zo
    import synthetic as syn
    zo.set_threads(threads)
    op = cfg["op"]
    py, puv = syn.synthesis_params(op, cfg["seed"])
    cky, ckuv = zo.Checkpoint(py), zo.Checkpoint(puv)
    th = cfg["tile"] or cfg["H"]
    tw = cfg["tile"] or cfg["W"]
    lh, lw = -(-th // 16), -(-tw // 16)
    ly = syn.laplace_latent(cfg["lat_seed"], "cpu/ly", (160, lh, lw), 1.5)
    luv = syn.laplace_latent(cfg["lat_seed"], "cpu/luv", (96, lh, lw), 1.5)
    t = time.perf_counter()
    zo.synthesis_primary(cky, zo.OPS[op], ly, th, tw)
    zo.synthesis_secondary(ckuv, zo.OPS[op], ly, luv, th, tw)
    dt = time.perf_counter() - t
    return th * tw / dt / 1e6, "one %dx%d tile (luma + chroma synthesis) of the workload" % (th, tw)


def run_reference(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    for _ in range(args.warmup):
        cpu_sample(cfg, threads)
    vals = [cpu_sample(cfg, threads) for _ in range(args.steps)]
    v = float(np.mean([x[0] for x in vals]))
    line = {
        "impl": "reference", "metric": "synthesis decode Mpixel/s", "value": v,
        "unit": "Mpixel/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": None, "higher_is_better": True, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.config + ": " + cfg["desc"]},
        "cpu_baseline": {"value": v, "unit": "Mpixel/s", "cores": threads, "kind": "port",
                         "sample": vals[0][1] + ", per step"},
        "e2e": {"value": v, "unit": "Mpixel/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "the reference crate (Rust) cannot be built here; its f32 CPU path is timed "
                "through the C restatement in oracle/ on all host threads",
    }
    print(json.dumps(line), flush=True)


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
    args = ap.parse_args()
    cfg = CONFIGS[args.config]
    if args.impl == "reference":
        return run_reference(args, cfg)

    import ctypes
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

    import zenjpegai_b200 as zj
    import synthetic as syn
    from zenjpegai_b200 import _lib, sharding
    from zenjpegai_b200.decoder import Decoder

    H, W, op = cfg["H"], cfg["W"], cfg["op"]
    lh, lw = -(-H // 16), -(-W // 16)
    ch, cw = -(-H // 2), -(-W // 2)
    eng = zj.Engine(local, arena_bytes=64 << 30)
    # one non-default stream shared by torch (copies, events, NCCL) and the engine
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    eng.set_stream(stream.cuda_stream)
    py, puv = syn.synthesis_params(op, cfg["seed"])
    dec = Decoder(eng, op, py, puv)
    ly_h = torch.from_numpy(syn.laplace_latent(cfg["lat_seed"], "ly", (160, lh, lw), 1.5))
    luv_h = torch.from_numpy(syn.laplace_latent(cfg["lat_seed"], "luv", (96, lh, lw), 1.5))
    ly_h, luv_h = ly_h.pin_memory(), luv_h.pin_memory()
    ly, luv = ly_h.cuda(), luv_h.cuda()
    tiles = zj.synthesis_tiles(H, W, lh, lw, cfg["tile"], cfg["overlap"])
    mine = sharding.shard_tiles(tiles, rank, world)
    out8 = torch.zeros(H * W + 2 * ch * cw, dtype=torch.uint8, device="cuda")
    # the 8-bit planes of the picture, written by the final layers (fused output stage)
    planes8 = (out8[:H * W].view(H, W), out8[H * W:H * W + ch * cw].view(ch, cw),
               out8[H * W + ch * cw:].view(ch, cw))
    out8_host = torch.empty_like(out8, device="cpu").pin_memory()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

    def step(from_host=False):
        if from_host:
            ly.copy_(ly_h, non_blocking=True)
            luv.copy_(luv_h, non_blocking=True)
        # every rank starts from a zero picture: the reduce sums the ranks' disjoint cores, so
        # a plane still holding last step's picture would add it in again
        out8.zero_()
        dec.synthesize_tiles(ly, luv, mine, H, W, out=planes8, bit_depth=8)
        sharding.gather_cores(out8, dist)
        if from_host and rank == 0:
            out8_host.copy_(out8, non_blocking=True)

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
    eng_h = eng.handle
    _lib.lib().zjai_ctx_profile(eng_h, 1)
    flush.zero_()
    torch.cuda.synchronize()
    step()
    ms, fl, nl = ctypes.c_double(), ctypes.c_double(), ctypes.c_int64()
    _lib.lib().zjai_ctx_profile_read(eng_h, ctypes.byref(ms), ctypes.byref(fl), ctypes.byref(nl))
    _lib.lib().zjai_ctx_profile(eng_h, 0)
    if args.layers and rank == 0:
        buf = ctypes.create_string_buffer(1 << 20)
        _lib.lib().zjai_ctx_profile_report(eng_h, buf, len(buf))
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
    stats = torch.tensor([ms.value, fl.value, float(nl.value), float(launches)],
                         dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.SUM)
    conv_ms, conv_fl, conv_n, all_launches = (float(x) for x in stats.tolist())

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        v, desc = cpu_sample(cfg, threads)
        cpu = {"value": v, "unit": "Mpixel/s", "cores": threads, "kind": "port",
               "sample": desc + ", oracle/ (C restatement of the crate's f32 path)"}

    if rank == 0:
        mpx = H * W / 1e6
        peak, peak_src = peaks()
        achieved = conv_fl / (conv_ms / 1e3) / 1e12 if conv_ms > 0 else 0.0
        line = {
            "metric": "synthesis decode Mpixel/s",
            "value": args.steps * mpx / (total_ms / 1e3),
            "unit": "Mpixel/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "f16",
            "data": "synthetic",
            "config": {
                "workload": args.config + ": " + cfg["desc"],
                "picture": "%dx%d 4:2:0, 8-bit YUV out" % (W, H),
                "tiles": len(tiles),
                "parallelism": "tiles round-robin over %d GPU(s), NCCL reduce of 8-bit cores"
                               % world,
                "weights": "random-init, seed %d (role-scaled normal)" % cfg["seed"],
                "l2": "flushed between steps (256 MiB write, outside the timed events)",
                "precision": "f16 operands, f32 accumulation (TMEM)",
            },
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
                # bytes per step (all tcgen05 launches of the step, like `achieved`), from the
                # committed single-pass ncu capture of this workload
                "traffic": conv_traffic(args.config),
                "traffic_unit": "bytes per step (DRAM read + write, ncu)",
            },
            "cpu_baseline": cpu,
            "e2e": {
                "value": args.steps * mpx / (e2e_ms / 1e3),
                "unit": "Mpixel/s",
                "h2d_bytes_per_step": world * (ly_h.numel() + luv_h.numel()) * 4,
                "d2h_bytes_per_step": out8.numel(),
            },
            "clocks": clk,
            "gpu_launches": int(all_launches),
        }
        print(json.dumps(line), flush=True)
    dec.close()
    eng.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
