"""Weight-file readers (zjai_ckpt_*, zjai_bundle_*; host only, no GPU): PyTorch `.pth` files
against `torch.load` of the same file (torch writes the format, so it is the oracle here), the
packed `ZJM1` / `ZJB1` / `ZJB2` containers against a writer that follows the layout of
src/weights/packed.rs:8-43, and malformed inputs (truncations, flipped bytes) that must fail
cleanly, as the crate's fuzz regressions require (tests/fuzz_regression.rs)."""

import collections
import struct

import numpy as np
import pytest
import torch

from zenjpegai_b200 import _lib
from zenjpegai_b200 import weights as W

CODES = {np.dtype(np.float64): 0, np.dtype(np.float32): 1, np.dtype(np.float16): 2,
         np.dtype(np.int64): 3, np.dtype(np.int32): 4, np.dtype(np.int16): 5,
         np.dtype(np.int8): 6, np.dtype(np.uint8): 7, np.dtype(np.bool_): 8}


def _pad(b):
    return b + b"\0" * (-len(b) % 64)


def write_zjm(tensors, ints=()):
    """ZJM1: magic, version 1, counts, tensor table, integer table, 64-aligned payloads."""
    names = list(tensors)
    table = 16 + sum(2 + len(n.encode()) + 2 + 8 * tensors[n].ndim + 16 for n in names) + \
        sum(2 + len(n.encode()) + 8 for n, _ in ints)
    off = table + (-table % 64)
    head = b"ZJM1" + struct.pack("<III", 1, len(names), len(ints))
    payload = b""
    for n in names:
        a = np.ascontiguousarray(tensors[n])
        raw = a.tobytes()
        head += struct.pack("<H", len(n.encode())) + n.encode()
        head += struct.pack("<BB", CODES[a.dtype], a.ndim) + b"".join(struct.pack("<Q", d) for d in a.shape)
        head += struct.pack("<QQ", off, len(raw))
        payload += _pad(raw)
        off += len(_pad(raw))
    for n, v in ints:
        head += struct.pack("<H", len(n.encode())) + n.encode() + struct.pack("<q", v)
    assert len(head) == table
    return _pad(head) + payload


def write_bundle(files, notice, magic=b"ZJB1"):
    table = 16 + len(notice.encode()) + sum(2 + len(p.encode()) + 16 for p, _ in files)
    off = table + (-table % 64)
    head = magic + struct.pack("<III", 1, len(files), len(notice.encode())) + notice.encode()
    body = b""
    for p, data in files:
        head += struct.pack("<H", len(p.encode())) + p.encode() + struct.pack("<QQ", off, len(data))
        body += _pad(data)
        off += len(_pad(data))
    return _pad(head) + body


def _state(seed=0):
    g = torch.Generator().manual_seed(seed)
    sd = collections.OrderedDict()
    sd["conv.weight"] = torch.randn(8, 4, 3, 3, generator=g)
    sd["conv.bias"] = torch.randn(8, generator=g)
    sd["half"] = torch.randn(3, 5, generator=g).half()
    sd["transposed"] = torch.randn(6, 7, generator=g).t()           # strided view
    base = torch.arange(24, dtype=torch.int64)
    sd["view_a"] = base[3:11]                                        # storage offset
    sd["view_b"] = base.view(4, 6)[:, 1:5]                          # offset + strides
    sd["i32"] = torch.randint(-9, 9, (5,), dtype=torch.int32, generator=g)
    sd["i16"] = torch.randint(-9, 9, (2, 2), dtype=torch.int16, generator=g)
    sd["i8"] = torch.randint(-9, 9, (7,), dtype=torch.int8, generator=g)
    sd["u8"] = torch.randint(0, 255, (7,), dtype=torch.uint8, generator=g)
    sd["flags"] = torch.tensor([True, False, True])
    sd["f64"] = torch.randn(2, 3, dtype=torch.float64, generator=g)
    sd["scalar"] = torch.tensor(3.5)
    sd["empty"] = torch.zeros(0, 4)
    sd["param"] = torch.nn.Parameter(torch.randn(2, 2, generator=g))  # _rebuild_parameter
    return sd


def test_pth_matches_torch_load(tmp_path):
    sd = _state()
    path = tmp_path / "m.pth"
    torch.save({**sd, "epoch": 42, "step": -3,
                "clip_thres": {"E1B": {"MinList": [0.5, 1, 2.25], "w": torch.ones(2)},
                               "deep": {"a": {"b": {"too_deep": torch.ones(1)}}}}}, path)
    ck = W.Checkpoint(str(path))
    ref = torch.load(path, weights_only=False)
    for k, t in sd.items():
        got = ck.tensor(k)
        want = t.detach().numpy()
        assert got.dtype == want.dtype and got.shape == want.shape, k
        assert np.array_equal(got, want), k
    assert ck.ints == {"epoch": 42, "step": -3}
    assert ck.lists == {"clip_thres.E1B.MinList": [0.5, 1.0, 2.25]}
    assert np.array_equal(ck.tensor("clip_thres.E1B.w"), np.ones(2, np.float32))
    # nested dicts are flattened three levels deep, no further (src/weights/mod.rs:83-125)
    assert "clip_thres.deep.a.b.too_deep" not in ck
    # the f32 view: f32 and f16 tensors of rank <= 4, f16 upcast exactly
    p = ck.params()
    assert set(p) == {"conv.weight", "conv.bias", "half", "transposed", "scalar", "empty",
                      "param", "clip_thres.E1B.w"}
    assert np.array_equal(p["half"], ref["half"].float().numpy())
    assert np.array_equal(p["transposed"], ref["transposed"].numpy())
    ck.close()


def test_pth_module_state_dict(tmp_path):
    m = torch.nn.Sequential(torch.nn.Conv2d(3, 8, 3), torch.nn.ReLU(), torch.nn.Conv2d(8, 4, 1))
    path = tmp_path / "s.pth"
    torch.save(m.state_dict(), path)
    ck = W.Checkpoint(str(path))
    for k, v in m.state_dict().items():
        assert np.array_equal(ck.tensor(k), v.numpy())


def test_zjm_roundtrip_and_f16_upcast():
    rng = np.random.default_rng(1)
    t = {"w": rng.standard_normal((4, 3, 3, 3)).astype(np.float32),
         "h": rng.standard_normal((5, 6)).astype(np.float16),
         "q": rng.integers(-100, 100, (9,)).astype(np.int8),
         "b": np.array([True, False]),
         "r5": rng.standard_normal((1, 2, 1, 2, 3)).astype(np.float32)}
    ck = W.Checkpoint(write_zjm(t, [("epoch", 5), ("neg", -7)]))
    assert ck.names() == list(t)
    for k, v in t.items():
        assert np.array_equal(ck.tensor(k), v) and ck.info(k) == (v.dtype.type, v.shape)
    assert ck.ints == {"epoch": 5, "neg": -7}
    p = ck.params()
    assert set(p) == {"w", "h"}  # rank-5 tensors are not network parameters
    assert np.array_equal(p["h"], t["h"].astype(np.float32))
    # every finite and special f16 value upcasts exactly
    allh = np.arange(65536, dtype=np.uint16).view(np.float16)
    got = W.Checkpoint(write_zjm({"all": allh})).params()["all"]
    want = allh.astype(np.float32)
    assert np.array_equal(got, want, equal_nan=True)


def test_bundle():
    a = write_zjm({"x": np.ones((2, 2), np.float32)})
    b = write_zjm({"y": np.arange(3, dtype=np.int32)})
    for magic, f16 in ((b"ZJB1", False), (b"ZJB2", True)):
        bd = W.Bundle(write_bundle([("VM_common_int/Y_0.012.pth", a), ("other.pth", b)],
                                   "licence text", magic))
        assert bd.f16 is f16 and bd.notice == "licence text"
        assert bd.paths() == ["VM_common_int/Y_0.012.pth", "other.pth"]
        assert bd.read("other.pth") == b
        assert np.array_equal(bd.checkpoint("other.pth").tensor("y"), np.arange(3))
        with pytest.raises(_lib.ZjaiError):
            bd.read("missing.pth")


def test_synthesis_params_roundtrip(tmp_path):
    """A network's named parameters survive torch.save -> reader bit for bit (the input of
    zjai_net_create is then the same)."""
    import synthetic as syn
    py, _ = syn.synthesis_params("hop", 3)
    path = tmp_path / "syn.pth"
    torch.save({k: torch.from_numpy(v) for k, v in py.items()}, path)
    p = W.Checkpoint(str(path)).params()
    assert set(p) == set(py)
    for k in py:
        assert np.array_equal(p[k], py[k]), k


def _fails_cleanly(data):
    try:
        ck = W.Checkpoint(data)
    except _lib.ZjaiError as e:
        assert e.status in (_lib.MODEL, _lib.LIMIT_EXCEEDED)
        return
    # parsed: every tensor read either succeeds or fails with a status
    for n in ck.names():
        try:
            ck.tensor(n)
        except _lib.ZjaiError:
            pass
    try:
        ck.params()
    except _lib.ZjaiError:
        pass


def test_malformed_inputs_fail_cleanly(tmp_path):
    path = tmp_path / "m.pth"
    torch.save(_state(), path)
    pth = path.read_bytes()
    zjm = write_zjm({"w": np.ones((3, 3), np.float32), "i": np.arange(4, dtype=np.int64)},
                    [("epoch", 1)])
    for data in (pth, zjm):
        for cut in sorted(set(list(range(0, 200, 7)) + list(range(0, len(data), max(1, len(data) // 97))))):
            _fails_cleanly(data[:cut])
        rng = np.random.default_rng(5)
        for _ in range(150):
            b = bytearray(data)
            for i in rng.integers(0, len(b), 3):
                b[i] ^= int(rng.integers(1, 256))
            _fails_cleanly(bytes(b))
    for bad in (b"", b"ZJM1", b"PK\x05\x06" + b"\0" * 18, b"ZJB1\x01\0\0\0", b"\x80\x02."):
        with pytest.raises(_lib.ZjaiError):
            W.Checkpoint(bad)
    with pytest.raises(_lib.ZjaiError):
        W.Bundle(b"ZJB1\x01\0\0\0\x05\0\0\0\xff\xff\xff\xff")


def test_model_paths_and_sources(tmp_path):
    """Paths follow src/model/mod.rs:94-140; a ModelDir and a Bundle serve the same bytes."""
    assert W.common_path(1, 0) == "VM_common_int/Y_0.012.pth"
    assert W.synthesis_path(3, 1, 2) == "VM_hop/decoder_UV_0.5.pth"
    assert W.synthesis_path(0, 0, 0) == "VM_sop/decoder_Y_0.002.pth"
    assert W.analysis_path(2, 0, 0) == "VM_bop/encoder_Y_0.075.pth"  # SOP encodes with BOP
    with pytest.raises(_lib.ZjaiError):
        W.common_path(4, 0)
    rel = W.synthesis_path(1, 0, 1)
    (tmp_path / "VM_bop").mkdir()
    data = write_zjm({"first_stage.0.0.conv1.weight": np.ones((2, 2, 1, 1), np.float32)})
    (tmp_path / rel).write_bytes(data)
    bd = W.Bundle(write_bundle([(rel, data)], "n"))
    for src in (W.ModelDir(str(tmp_path)), bd):
        assert src.read(rel) == data
        assert np.array_equal(W._params(src, rel)["first_stage.0.0.conv1.weight"],
                              np.ones((2, 2, 1, 1), np.float32))
    with pytest.raises(_lib.ZjaiError):
        W.ModelDir(str(tmp_path)).read("VM_bop/missing.pth")


def test_extents_that_wrap_are_rejected():
    # a ZJM1 table entry whose element count times the element size wraps to 0 in 128 bits
    # (f32, shape 2^62 x 2^62 x 16, length 0) must fail cleanly, not pass the extent check
    name = b"w"
    head = b"ZJM1" + struct.pack("<III", 1, 1, 0)
    head += struct.pack("<H", len(name)) + name + struct.pack("<BB", 1, 3)
    head += b"".join(struct.pack("<Q", d) for d in (1 << 62, 1 << 62, 16))
    head += struct.pack("<QQ", 64, 0)
    data = head + b"\0" * (64 - len(head) % 64)
    with pytest.raises(_lib.ZjaiError) as e:
        W.Checkpoint(data)
    assert e.value.status == _lib.LIMIT_EXCEEDED
