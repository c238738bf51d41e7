"""Layer-level timing of the tcgen05 convolution kernel (`zjai_conv_bench`).

The GPU counterpart of the crate's conv microbenchmark (benches/conv_kernels.rs:165-187): the
BOP luma layer shapes at the latent size 131x88, plus the HOP shapes of a 4K picture's 28
interior 512x512 tiles run as one batch. Prints one line per layer (ms, TFLOP/s, fraction of
the measured bf16 peak). Usage: python -m zenjpegai_b200.conv_bench [--only NAME] [--reps R]
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
    ("hop_us_convT3_128@H4x28", 28, 128, 128, 128, 128, 3, 1, 1, 1, 0),
    ("hop_subscale_s2_128@H4x1", 1, 128, 128, 128, 128, 3, 2, 1, 0, 0),
]


def peak():
    try:
        with open(os.path.join(os.path.dirname(__file__), "..", "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"])
    except Exception:
        return 1590.0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default=None)
    ap.add_argument("--reps", type=int, default=20)
    args = ap.parse_args()
    L = _lib.lib()
    L.zjai_conv_bench.argtypes = [ctypes.c_void_p] + [ctypes.c_int] * 11 + [
        ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)]
    eng = Engine(0, arena_bytes=16 << 30)
    pk = peak()
    for row in LAYERS:
        name = row[0]
        if args.only and args.only not in name:
            continue
        ms, fl = ctypes.c_double(), ctypes.c_double()
        _lib.check(L.zjai_conv_bench(eng.handle, *row[1:], args.reps, ctypes.byref(ms),
                                     ctypes.byref(fl)))
        tf = fl.value / (ms.value * 1e-3) / 1e12
        print("%-32s %8.3f ms %8.1f TFLOP/s %6.1f%% of %.0f" % (name, ms.value, tf,
                                                               100 * tf / pk, pk), flush=True)
    eng.close()


if __name__ == "__main__":
    main()
