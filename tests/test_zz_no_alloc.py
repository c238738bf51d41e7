"""The allocation-free channel attention (zjai_channel_attention_static) against the regular
entry point (zjai_channel_attention) and the CPU oracle, through the C ABI, on device buffers
the test allocates before the calls.

Callers that cannot allocate device memory while they run (an external allocator or a strict
memory budget, or code that only passes pre-allocated buffers) use the static variant; its
output must match the regular path and the oracle within the layer tolerance (relative L2
1e-3) on calls in a row, since every call reuses the same static scratch. The limit case
(dim 256, 64 channels per head: the whole scratch array) is compared with the oracle only,
because the regular entry stops at dim 128.
This file is named so that pytest collects it last.
"""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL_L2 = 1e-3


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _bind(L):
    L.zjai_channel_attention_static.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                                ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                ctypes.c_void_p, ctypes.c_void_p]


def test_static_attention_matches_regular_entry():
    import torch

    import oracle as zo
    import synthetic as syn
    import zenjpegai_b200 as zj
    from zenjpegai_b200 import _lib

    L = _lib.lib()
    _bind(L)
    eng = zj.Engine(0, arena_bytes=1 << 30)
    try:
        # (dim, h, w): head widths 32 and 16 against the regular entry; the limit case dim 256
        # with 64 channels per head over 37 x 29 pixels (not a multiple of the 64-pixel chunk)
        for call, (dim, h, w) in enumerate([(128, 40, 52), (64, 64, 64), (256, 37, 29)]):
            qkv = syn.normal(20 + call, "static/qkv", (3 * dim, h, w))
            t = syn.uniform(20 + call, "static/t", (4,), 0.5, 2.0)
            oracle_out = zo.channel_attention(qkv, 4, t)
            regular = eng.channel_attention(qkv, 4, t) if dim <= 128 else None
            d_qkv = torch.from_numpy(qkv).cuda()
            d_t = torch.from_numpy(t).cuda()
            outs = []
            for _ in range(2):  # two calls in a row on the shared scratch
                d_out = torch.full((dim, h, w), float("nan"), device="cuda")
                torch.cuda.synchronize()
                zj.check(L.zjai_channel_attention_static(eng.handle, d_qkv.data_ptr(), 3 * dim,
                                                         h, w, 4, d_t.data_ptr(),
                                                         d_out.data_ptr()))
                eng.sync()
                outs.append(d_out.cpu().numpy())
            for got in outs:
                assert np.isfinite(got).all()
                assert rel_l2(got, oracle_out) < REL_L2, (dim, rel_l2(got, oracle_out))
                if regular is not None:
                    assert rel_l2(got, regular) < REL_L2, (dim, rel_l2(got, regular))
            # fixed-order reduction: the second call repeats the first to the bit
            assert np.array_equal(outs[0], outs[1])
        # sizes beyond the static scratch are rejected with a clear error
        big = torch.zeros((3 * 512, 4, 4), device="cuda")
        d_t = torch.ones(4, device="cuda")
        out = torch.zeros((512, 4, 4), device="cuda")
        st = L.zjai_channel_attention_static(eng.handle, big.data_ptr(), 3 * 512, 4, 4, 4,
                                             d_t.data_ptr(), out.data_ptr())
        assert st == _lib.LIMIT_EXCEEDED
        assert b"static scratch" in L.zjai_last_error_message()
        # host memory is refused before any kernel runs
        host_qkv = np.zeros((3 * 64, 4, 4), np.float32)
        out = torch.zeros((64, 4, 4), device="cuda")
        st = L.zjai_channel_attention_static(eng.handle, host_qkv.ctypes.data, 3 * 64, 4, 4, 4,
                                             d_t.data_ptr(), out.data_ptr())
        assert st == _lib.INVALID_ARGUMENT
        assert b"device" in L.zjai_last_error_message()
    finally:
        eng.close()
