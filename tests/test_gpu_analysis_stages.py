"""Per-stage parity of the analysis transforms (src/model/analysis.rs:157-311) on the GPU.

The engine's intermediate maps are captured with zjai_ctx_set_probe ("ana.act1" .. "ana.act3",
the trunk's ResAu outputs) and each stage is checked against the oracle running that stage on
the engine's OWN input for it (the picture, act1, act2, act3), so the gate measures the error
one stage adds, not the error compounded over the network. A stage is a stride-2 conv plus a
ResAu (relu6 -> grouped 3x3 -> 1x1 -> gate), at HOP with a transformer-attention module
(stage 2) or a CAB (stage 3) in front; the last stage is conv4 + conv5 (primary) or conv5.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import oracle as zo
import synthetic as syn

# One layer's f16 storage rounding is 2^-12 relative (rel L2 ~1.4e-4 for uniform rounding);
# a BOP stage stores four maps, so it adds at most a few 1e-4.
STAGE_REL = 1e-3
# HOP stage 2 runs two transformer blocks (LN, 1x1, depthwise, attention, folded projection,
# fused FFN) and stage 3 a CAB (eight 3x3 convs, a convT and the sigmoid mask) before the conv:
# about 15 stored maps.
STAGE_REL_DEEP = 2e-3


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def eng():
    import zenjpegai_b200 as zj
    e = zj.Engine(0, arena_bytes=4 << 30)
    yield e
    e.close()


@pytest.mark.parametrize("secondary", [False, True])
@pytest.mark.parametrize("op", ["bop", "hop"])
def test_analysis_per_stage(eng, op, secondary):
    import torch
    import zenjpegai_b200 as zj
    pa, puv = syn.analysis_params(op, 4)
    params = puv if secondary else pa
    h, w = (60, 100) if secondary else (120, 200)
    cin = 12 if secondary else 1
    x = np.floor(syn.uniform(9, "stage", (cin, h, w), 0.0, 256.0)).astype(np.float32)
    net = zj.Network(eng, zj.ANA_UV if secondary else zj.ANA_Y, zo.OPS[op], params)
    acts = [torch.zeros((128, -(-h // d), -(-w // d)), device="cuda") for d in (2, 4, 8)]
    for i, a in enumerate(acts):
        eng.set_probe("ana.act%d" % (i + 1), a)
    try:
        xt = torch.from_numpy(x).cuda()
        d = 8 if secondary else 16
        out = torch.zeros((96 if secondary else 160, -(-h // d), -(-w // d)), device="cuda")
        import ctypes
        from zenjpegai_b200 import _lib
        f = _lib.lib().zjai_analysis_secondary if secondary else _lib.lib().zjai_analysis_primary
        zj.check(f(net.handle, ctypes.c_void_p(xt.data_ptr()), h, w,
                   ctypes.c_void_p(out.data_ptr()), 1))
        eng.sync()
        got = [x] + [a.cpu().numpy() for a in acts] + [out.cpu().numpy()]
    finally:
        for i in range(3):
            eng.set_probe("ana.act%d" % (i + 1), None)
        net.close()
    ck = zo.Checkpoint(params)
    errs = []
    for stage in range(1, 5):
        want = zo.analysis_stage(ck, zo.OPS[op], secondary, stage, got[stage - 1], h, w)
        assert got[stage].shape == want.shape
        errs.append(rel_l2(got[stage], want))
    print("analysis %s %s per-stage rel L2: %s" % (op, "uv" if secondary else "y",
                                                    " ".join("%.2e" % e for e in errs)))
    for stage, e in enumerate(errs, 1):
        deep = op == "hop" and stage in (2, 3)
        assert e < (STAGE_REL_DEEP if deep else STAGE_REL), (stage, errs)


def test_probe_errors(eng):
    import torch
    import zenjpegai_b200 as zj
    with pytest.raises(zj.ZjaiError):
        eng.set_probe("ana.act1", np.zeros(16, np.float32))  # host memory
    pa, _ = syn.analysis_params("bop", 4)
    net = zj.Network(eng, zj.ANA_Y, zo.BOP, pa)
    small = torch.zeros(10, device="cuda")
    eng.set_probe("ana.act2", small)
    try:
        import ctypes
        from zenjpegai_b200 import _lib
        x = np.zeros((1, 64, 64), np.float32)
        out = np.empty((160, 4, 4), np.float32)
        with pytest.raises(zj.ZjaiError) as e:
            zj.check(_lib.lib().zjai_analysis_primary(net.handle, ctypes.c_void_p(x.ctypes.data),
                                                      64, 64, ctypes.c_void_p(out.ctypes.data), 0))
        assert e.value.status == zj._lib.LIMIT_EXCEEDED
    finally:
        eng.set_probe("ana.act2", None)
        net.close()
    # the context works after the refused run
    x = np.floor(syn.uniform(3, "p", (1, 32, 48), 0.0, 256.0)).astype(np.float32)
    net = zj.Network(eng, zj.ANA_Y, zo.BOP, pa)
    try:
        import ctypes
        from zenjpegai_b200 import _lib
        out = np.empty((160, 2, 3), np.float32)
        zj.check(_lib.lib().zjai_analysis_primary(net.handle, ctypes.c_void_p(x.ctypes.data),
                                                  32, 48, ctypes.c_void_p(out.ctypes.data), 0))
        assert rel_l2(out, zo.analysis_primary(zo.Checkpoint(pa), zo.BOP, x)) < 5e-3
    finally:
        net.close()
