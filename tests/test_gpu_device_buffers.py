"""Caller buffers passed as ZJAI_MEM_DEVICE are checked before any kernel touches them: a
pageable host array handed over as device memory is refused with ZJAI_INVALID_ARGUMENT (no
launch happens), and the context computes correctly afterwards."""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import oracle as zo


@pytest.fixture(scope="module")
def eng():
    import zenjpegai_b200 as zj
    e = zj.Engine(0, arena_bytes=1 << 28)
    yield e
    e.close()


def _p(a):
    return ctypes.c_void_p(a.ctypes.data)


def test_host_arrays_as_device_memory_are_refused(eng):
    from zenjpegai_b200 import _lib
    L = _lib.lib()
    x = np.linspace(-3.0, 300.0, 1000, dtype=np.float32)
    q = np.empty(1000, np.uint8)
    # input and output both host arrays, declared device memory
    st = L.zjai_quantize_plane(eng.handle, _p(x), x.size, 8, _p(q), _lib.MEM_DEVICE)
    assert st == 1  # ZJAI_INVALID_ARGUMENT
    y = np.zeros((9, 11), np.float32)
    u = np.zeros((5, 6), np.float32)
    rgb = np.empty((9, 11, 3), np.uint8)
    st = L.zjai_yuv_to_rgb(eng.handle, _p(y), _p(u), _p(u), 9, 11, 5, 6, 8, _p(rgb),
                           _lib.MEM_DEVICE)
    assert st == 1
    # the same context afterwards, with host memory declared as such
    assert L.zjai_quantize_plane(eng.handle, _p(x), x.size, 8, _p(q), _lib.MEM_HOST) == 0
    assert np.array_equal(q.astype(np.uint16), zo.quantize_plane(x))


def test_device_tensor_of_the_context_is_accepted(eng):
    import torch
    from zenjpegai_b200 import _lib
    L = _lib.lib()
    x = np.linspace(-3.0, 300.0, 1000, dtype=np.float32)
    dx = torch.from_numpy(x).cuda()
    dq = torch.empty(1000, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    st = L.zjai_quantize_plane(eng.handle, ctypes.c_void_p(dx.data_ptr()), x.size, 8,
                               ctypes.c_void_p(dq.data_ptr()), _lib.MEM_DEVICE)
    assert st == 0
    eng.sync()
    assert np.array_equal(dq.cpu().numpy().astype(np.uint16), zo.quantize_plane(x))
