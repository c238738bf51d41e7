"""Layer-level timing of the tcgen05 convolution kernel (`zjai_conv_bench`) and of the
other kernels of the HOP transformer blocks (`zjai_kernel_bench`: the memory-bound ones and
the fused tcgen05 FFN).

The GPU counterpart of the crate's conv microbenchmark (benches/conv_kernels.rs:165-187): the
BOP luma layer shapes at the latent size 131x88, plus the HOP shapes of a 4K picture's 28
interior 512x512 tiles run as one batch. Prints one line per layer: ms and TFLOP/s against
the measured bf16 peak (convolutions), or GB/s of algorithmic traffic against the measured
HBM copy bandwidth (the others).

Usage: python -m zenjpegai_b200.conv_bench [--only NAME] [--reps R] [--arena-gib G]
"""

import argparse
import ctypes
import json
import os

from . import Engine, _lib

H, W = 88, 131
# name, n, h, w, cin, cout, k, stride, groups, transposed, residual
LAYERS = [
    ("res_conv3x3_160_160@1/16", 1, H, W, 160, 160, 3, 1, 1, 0, 0),
    ("up1_convT4x4_160_64@1/16", 1, H, W, 160, 64, 4, 1, 1, 1, 0),
    ("resau_conv3x3_g4_64@1/8", 1, 2 * H, 2 * W, 64, 64, 3, 1, 4, 0, 0),
    ("resau_conv1x1_64_64@1/8", 1, 2 * H, 2 * W, 64, 64, 1, 1, 1, 0, 1),
    ("up2_convT4x4_64_64@1/8", 1, 2 * H, 2 * W, 64, 64, 4, 1, 1, 1, 0),
    ("conv3_3x3_64_96@1/4", 1, 4 * H, 4 * W, 64, 96, 3, 1, 1, 0, 0),
    ("conv4_1x1_96_16@1/4", 1, 4 * H, 4 * W, 96, 16, 1, 1, 1, 0, 0),
    ("hop_rb_conv3x3_128@H4x28", 28, 128, 128, 128, 128, 3, 1, 1, 0, 1),
    ("hop_resau_g4_128@H2x28", 28, 256, 256, 128, 128, 3, 1, 4, 0, 0),
    ("hop_ffn_in_1x1_128_1024@H4x28", 28, 128, 128, 128, 1024, 1, 1, 1, 0, 0),
    ("hop_ffn_out_1x1_512_128@H4x28", 28, 128, 128, 512, 128, 1, 1, 1, 0, 1),
    ("hop_prep_conv1_1x1_128_384@H4x28", 28, 128, 128, 128, 384, 1, 1, 1, 0, 0),
    ("hop_conv3_t_1x1_128_512@H4x28", 28, 128, 128, 128, 512, 1, 1, 1, 0, 0),
    ("hop_us_convT3_128@H4x28", 28, 128, 128, 128, 128, 3, 1, 1, 1, 0),
    ("hop_subscale_s2_128@H4x1", 1, 128, 128, 128, 128, 3, 2, 1, 0, 0),
    # residual 2: the network's final layer (planar f32 output, denormalised)
    ("hop_conv4_t_128_1_planar@H2x28", 28, 256, 256, 128, 1, 3, 1, 1, 1, 2),
]

KB_DW, KB_DW_GATE, KB_LN, KB_ATTN, KB_FFN = 0, 1, 2, 3, 4
# name, kind, n, h, w, c (HOP luma transformer blocks at 1/4 scale: dim 128, hidden 512)
KERNELS = [
    ("hop_ffn_dwgate_1024@H4x28", KB_DW_GATE, 28, 128, 128, 1024),
    ("hop_qkv_dw_384@H4x28", KB_DW, 28, 128, 128, 384),
    ("hop_ln_128@H4x28", KB_LN, 28, 128, 128, 128),
    ("hop_attn_128@H4x28", KB_ATTN, 28, 128, 128, 128),
    ("hop_uv_attn_64@H4x28", KB_ATTN, 28, 128, 128, 64),
    # fused FFN (project_in + depthwise + ELU gate + project_out + residual), tcgen05
    ("hop_ffn_fused_128@H4x28", KB_FFN, 28, 128, 128, 128),
    ("hop_uv_ffn_fused_64@H4x28", KB_FFN, 28, 128, 128, 64),
]


def _peaks():
    try:
        with open(os.path.join(os.path.dirname(__file__), "..", "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), float(d["hbm_gbs"]), "measured"
    except Exception:
        return 1590.0, 6650.0, "fallback"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default=None)
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--arena-gib", type=int, default=16)
    args = ap.parse_args()
    L = _lib.lib()
    eng = Engine(0, arena_bytes=args.arena_gib << 30)
    pk, hbm, src = _peaks()
    for row in LAYERS:
        name = row[0]
        if args.only and args.only not in name:
            continue
        ms, fl = ctypes.c_double(), ctypes.c_double()
        _lib.check(L.zjai_conv_bench(eng.handle, *row[1:], args.reps, ctypes.byref(ms),
                                     ctypes.byref(fl)))
        tf = fl.value / (ms.value * 1e-3) / 1e12
        print("%-32s %8.3f ms %8.1f TFLOP/s %6.1f%% of %.0f (%s)" % (
            name, ms.value, tf, 100 * tf / pk, pk, src), flush=True)
    for row in KERNELS:
        name = row[0]
        if args.only and args.only not in name:
            continue
        ms, by = ctypes.c_double(), ctypes.c_double()
        _lib.check(L.zjai_kernel_bench(eng.handle, *row[1:], args.reps, ctypes.byref(ms),
                                       ctypes.byref(by)))
        gbs = by.value / (ms.value * 1e-3) / 1e9
        if row[1] == KB_FFN:
            # algorithmic FLOPs of project_in + project_out (dim c, hidden 4c)
            n, h, w, c = row[2:]
            tf = 2.0 * n * h * w * 3 * 4 * c * c / (ms.value * 1e-3) / 1e12
            print("%-32s %8.3f ms %8.1f TFLOP/s %6.1f%% of %.0f (%s)" % (
                name, ms.value, tf, 100 * tf / pk, pk, src), flush=True)
            continue
        print("%-32s %8.3f ms %8.0f GB/s    %6.1f%% of %.0f (%s)" % (
            name, ms.value, gbs, 100 * gbs / hbm, hbm, src), flush=True)
    eng.close()


if __name__ == "__main__":
    main()
