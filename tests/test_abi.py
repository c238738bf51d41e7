"""The C-ABI library loads on a machine without a GPU and exports every function that
include/zjai.h declares (no compute calls here)."""

import ctypes
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "zenjpegai_b200", "libzjai.so")


@pytest.fixture(scope="module")
def built():
    if not os.path.exists(LIB):
        subprocess.run(["python", os.path.join(ROOT, "zenjpegai_b200", "build.py")], check=True)
    return LIB


def test_exports_every_declared_symbol(built):
    from zenjpegai_b200 import _lib
    names = _lib.header_functions()
    assert len(names) >= 20
    L = ctypes.CDLL(built)
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", built], capture_output=True,
                         text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert set(names) <= exported


def test_version_and_error_without_gpu(built):
    from zenjpegai_b200 import _lib
    L = _lib.lib()
    assert b"sm_100a" in L.zjai_version()
    h = ctypes.c_void_p()
    st = L.zjai_ctx_create(0, 0, ctypes.byref(h))
    if st == _lib.OK:  # a GPU is present: nothing to check here
        L.zjai_ctx_destroy(h)
        pytest.skip("GPU present")
    assert st in (_lib.INVALID_ARGUMENT, _lib.DEVICE, _lib.UNSUPPORTED)
    assert L.zjai_last_error_message()
