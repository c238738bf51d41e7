"""Converts the reference crate's layer golden vectors into a committed fixture.

The reference (imazen/zenjpegai) pins its layer definitions with small torch-computed tensors
in `tests/vectors/nn/*.bin` ("ZJTB" bundles: u32 count, then per tensor u16 name length, name,
u8 ndim, u32 dims, f32 data; format read by `tests/nn_vectors.rs:16-48`, written by
`scripts/ref_vectors/gen_nn_vectors.py`). This script reads those files from a reference
checkout and writes every tensor into `nn_vectors.npz` next to it, keyed `<file>/<tensor>`, so
the tests can run where the reference checkout does not exist.

Usage: python tests/golden/make_golden.py [REFERENCE_ROOT]
"""

import os
import struct
import sys

import numpy as np

FILES = [
    "conv3x3_s1_p1_bias",
    "conv3x3_s1_p1_g4_nobias",
    "conv3x3_depthwise",
    "conv1x1_nobias",
    "conv3x3_s2_p1_bias",
    "conv2x2_s1_p0",
    "conv1x3_p01_bias",
    "conv3x1_p10_bias",
    "convt4x4_s2_p1_bias",
    "convt3x3_s2_p1_op1_bias",
    "pixel_shuffle",
    "bilinear_align_corners",
    "bicubic_align_corners",
]


def read_zjtb(path):
    b = open(path, "rb").read()
    assert b[:4] == b"ZJTB", path
    pos = 4
    (count,) = struct.unpack_from("<I", b, pos)
    pos += 4
    out = {}
    for _ in range(count):
        (nlen,) = struct.unpack_from("<H", b, pos)
        pos += 2
        name = b[pos:pos + nlen].decode()
        pos += nlen
        ndim = b[pos]
        pos += 1
        shape = struct.unpack_from("<%dI" % ndim, b, pos)
        pos += 4 * ndim
        n = int(np.prod(shape)) if ndim else 1
        data = np.frombuffer(b, dtype="<f4", count=n, offset=pos).reshape(shape)
        pos += 4 * n
        out[name] = data.copy()
    assert pos == len(b), path
    return out


def main():
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("ZJAI_REFERENCE", "")
    if not root:
        sys.exit("usage: make_golden.py REFERENCE_ROOT")
    arrays = {}
    for f in FILES:
        for k, v in read_zjtb(os.path.join(root, "tests", "vectors", "nn", f + ".bin")).items():
            arrays[f + "/" + k] = v
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "nn_vectors.npz")
    np.savez_compressed(dst, **arrays)
    print("wrote", dst, len(arrays), "tensors")


if __name__ == "__main__":
    main()
