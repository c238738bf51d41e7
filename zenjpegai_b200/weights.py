"""Weight files: the crate's checkpoint readers (src/weights/mod.rs `Checkpoint`,
src/weights/packed.rs `PackedBundle`) over the C ABI (`zjai_ckpt_*`, `zjai_bundle_*`).

`Checkpoint` parses a PyTorch `.pth` file or a packed `ZJM1` file; `params()` gives the
f32 / f16 tensors as float32 arrays by name, the input `Network` / `LatentModel` take.
`Bundle` serves the files of a `ZJB1` / `ZJB2` bundle by their path relative to the
reference's models/ directory (e.g. "VM_common_int/Y_0.012.pth").
"""

import ctypes

import numpy as np

from . import _lib
from ._lib import check

# ZJM1 dtype codes (src/weights/packed.rs:61-75)
DTYPES = {0: np.float64, 1: np.float32, 2: np.float16, 3: np.int64, 4: np.int32, 5: np.int16,
          6: np.int8, 7: np.uint8, 8: np.bool_}


def _read(src):
    if isinstance(src, (bytes, bytearray, memoryview)):
        return bytes(src)
    with open(src, "rb") as f:
        return f.read()


class Checkpoint:
    """A parsed checkpoint: tensors (top-level and nested-dict leaves under dotted names),
    integer entries and numeric lists, like the crate's `Checkpoint`."""

    def __init__(self, src):
        data = _read(src)
        h = ctypes.c_void_p()
        check(_lib.lib().zjai_ckpt_open(data, len(data), ctypes.byref(h)))
        self.handle = h
        nt, ni, nl = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        check(_lib.lib().zjai_ckpt_count(h, ctypes.byref(nt), ctypes.byref(ni), ctypes.byref(nl)))
        self._info = []
        for i in range(nt.value):
            name, dt, nd = ctypes.c_char_p(), ctypes.c_int(), ctypes.c_int()
            dims = (ctypes.c_int64 * 8)()
            check(_lib.lib().zjai_ckpt_tensor(h, i, ctypes.byref(name), ctypes.byref(dt),
                                              ctypes.byref(nd), dims))
            self._info.append((name.value.decode(), dt.value, tuple(dims[:nd.value])))
        self._index = {n: i for i, (n, _, _) in enumerate(self._info)}
        self.ints = {}
        for i in range(ni.value):
            name, v = ctypes.c_char_p(), ctypes.c_int64()
            check(_lib.lib().zjai_ckpt_int(h, i, ctypes.byref(name), ctypes.byref(v)))
            self.ints[name.value.decode()] = v.value
        self.lists = {}
        for i in range(nl.value):
            name, vals, n = ctypes.c_char_p(), ctypes.POINTER(ctypes.c_double)(), ctypes.c_int()
            check(_lib.lib().zjai_ckpt_list(h, i, ctypes.byref(name), ctypes.byref(vals),
                                            ctypes.byref(n)))
            self.lists[name.value.decode()] = [vals[k] for k in range(n.value)]

    def names(self):
        return [n for n, _, _ in self._info]

    def __contains__(self, name):
        return name in self._index

    def info(self, name):
        """(numpy dtype, shape) of a tensor without reading it."""
        _, dt, shape = self._info[self._index[name]]
        return DTYPES[dt], shape

    def tensor(self, name):
        """The tensor as a contiguous numpy array of its own dtype."""
        i = self._index.get(name)
        if i is None:
            raise _lib.ZjaiError(_lib.MODEL, "tensor `%s` not found" % name)
        _, dt, shape = self._info[i]
        out = np.empty(shape, DTYPES[dt])
        check(_lib.lib().zjai_ckpt_read(self.handle, i, ctypes.c_void_p(out.ctypes.data),
                                        out.nbytes))
        return out

    def params(self):
        """The f32 / f16 tensors of rank <= 4 as float32 arrays (f16 upcast exactly)."""
        p, n = ctypes.POINTER(_lib.Param)(), ctypes.c_int()
        check(_lib.lib().zjai_ckpt_params(self.handle, ctypes.byref(p), ctypes.byref(n)))
        out = {}
        for k in range(n.value):
            e = p[k]
            shape = tuple(e.shape[:e.ndim])
            cnt = int(np.prod(shape)) if shape else 1
            a = np.ctypeslib.as_array(e.data, shape=(cnt,)) if cnt else np.empty(0, np.float32)
            out[e.name.decode()] = np.array(a, dtype=np.float32).reshape(shape)
        return out

    def close(self):
        if self.handle:
            _lib.lib().zjai_ckpt_close(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Bundle:
    """A `ZJB1` / `ZJB2` bundle of model files (`f16` is True for ZJB2)."""

    def __init__(self, src):
        data = _read(src)
        h = ctypes.c_void_p()
        check(_lib.lib().zjai_bundle_open(data, len(data), ctypes.byref(h)))
        self.handle = h
        n, f16 = ctypes.c_int(), ctypes.c_int()
        txt, tl = ctypes.c_void_p(), ctypes.c_size_t()
        check(_lib.lib().zjai_bundle_info(h, ctypes.byref(n), ctypes.byref(f16), ctypes.byref(txt),
                                          ctypes.byref(tl)))
        self.f16 = bool(f16.value)
        self.notice = ctypes.string_at(txt, tl.value).decode() if tl.value else ""
        self._files = {}
        for i in range(n.value):
            path, d, ln = ctypes.c_char_p(), ctypes.c_void_p(), ctypes.c_size_t()
            check(_lib.lib().zjai_bundle_file(h, i, ctypes.byref(path), ctypes.byref(d),
                                              ctypes.byref(ln)))
            self._files[path.value.decode()] = (d.value, ln.value)

    def paths(self):
        return list(self._files)

    def read(self, path):
        if path not in self._files:
            raise _lib.ZjaiError(_lib.MODEL, "bundle has no file `%s`" % path)
        d, ln = self._files[path]
        return ctypes.string_at(d, ln) if ln else b""

    def checkpoint(self, path):
        return Checkpoint(self.read(path))

    def close(self):
        if self.handle:
            _lib.lib().zjai_bundle_close(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---- model sources (src/model/mod.rs:19-240) --------------------------------------------

MODEL_BETAS = ("0.002", "0.012", "0.075", "0.5")  # beta of each model_id
COMPONENT_NAMES = ("Y", "UV")
_OP_DIRS = {0: "VM_sop", 1: "VM_bop", 2: "VM_hop"}  # SOP, BOP, HOP


def _beta(model_id):
    if not 0 <= model_id < len(MODEL_BETAS):
        raise _lib.ZjaiError(_lib.INVALID_DATA, "model_id out of range")
    return MODEL_BETAS[model_id]


def common_path(model_id, ccs):
    """The common (entropy-stage and latent networks) checkpoint of component ccs."""
    return "VM_common_int/%s_%s.pth" % (COMPONENT_NAMES[ccs], _beta(model_id))


def synthesis_path(model_id, ccs, op):
    return "%s/decoder_%s_%s.pth" % (_OP_DIRS[op], COMPONENT_NAMES[ccs], _beta(model_id))


def analysis_path(model_id, ccs, op):
    """SOP streams are encoded with the BOP analysis transform."""
    return "%s/encoder_%s_%s.pth" % (_OP_DIRS[max(op, 1)], COMPONENT_NAMES[ccs], _beta(model_id))


class ModelDir:
    """Checkpoints in a directory laid out like the reference's models/ directory."""

    def __init__(self, root):
        self.root = root

    def read(self, rel):
        import os
        path = os.path.join(self.root, rel)
        if not os.path.isfile(path):
            raise _lib.ZjaiError(_lib.MODEL, "model file `%s` not found" % rel)
        with open(path, "rb") as f:
            return f.read()


def _params(src, rel):
    ck = Checkpoint(src.read(rel))
    try:
        return ck.params()
    finally:
        ck.close()


def load_synthesis(engine, src, model_id, op, ccs):
    """SynthesisPrimary (ccs 0) / SynthesisSecondary (ccs 1) of model `model_id` at operating
    point `op`, from a ModelDir or a Bundle."""
    from . import Network, SYN_UV, SYN_Y
    return Network(engine, SYN_UV if ccs else SYN_Y, op, _params(src, synthesis_path(model_id, ccs, op)))


def load_analysis(engine, src, model_id, op, ccs):
    from . import ANA_UV, ANA_Y, Network
    return Network(engine, ANA_UV if ccs else ANA_Y, max(op, 1),
                   _params(src, analysis_path(model_id, ccs, op)))


def load_latent(engine, src, model_id, ccs):
    """The hyper-decoder and (luma) context model of the common checkpoint."""
    from . import LatentModel
    return LatentModel(engine, _params(src, common_path(model_id, ccs)))
