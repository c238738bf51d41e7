"""LEF (src/filters/lef.rs) on the GPU, bit-exact against the oracle's restatement: the
reference's own unit cases (flat picture, clamped border, index checks), random pictures with
scale maps crossing every threshold of every model, odd and tiny extents, device tensors and
in-place filtering, and a 4K luma plane."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import oracle as zo


@pytest.fixture(scope="module")
def eng():
    import zenjpegai_b200 as zj
    e = zj.Engine(0, arena_bytes=1 << 30)
    yield e
    e.close()


def _case(seed, h, w, c, sh, sw):
    rng = np.random.default_rng(seed)
    y = rng.uniform(-20.0, 275.0, (h, w)).astype(np.float32)
    s = rng.integers(0, 3600, (c, sh, sw)).astype(np.int32)
    return y, s


def test_reference_unit_cases(eng):
    from zenjpegai_b200.filters import lef
    import zenjpegai_b200 as zj
    y = np.full((4, 4), 128.0, np.float32)
    y[0, 0] = 300.0
    s = np.array([[[5000]]], np.int32)
    got = lef(eng, y, s, 0, 0)
    assert got[0, 0] == 255.0 and abs(got[3, 3] - 128.0) < 1e-4
    assert np.array_equal(got, zo.lef(y, s, 0, 0))
    for bad in ((1, 0), (0, 4)):
        with pytest.raises(zj.ZjaiError):
            lef(eng, y, s, *bad)


@pytest.mark.parametrize("model", [0, 1, 2, 3])
@pytest.mark.parametrize("h,w,sh,sw", [(64, 96, 4, 6), (37, 53, 3, 4), (2, 9, 1, 1),
                                       (9, 2, 2, 1), (888, 600, 56, 38)])
def test_lef_bit_exact(eng, model, h, w, sh, sw):
    from zenjpegai_b200.filters import lef
    y, s = _case(10 * model + h, h, w, 3, sh, sw)
    assert np.array_equal(lef(eng, y, s, 1, model), zo.lef(y, s, 1, model))


def test_lef_device_and_in_place_4k(eng):
    import torch
    from zenjpegai_b200.filters import lef
    y, s = _case(99, 2160, 3840, 2, 135, 240)
    want = zo.lef(y, s, 0, 2)
    yt = torch.from_numpy(y).cuda()
    st = torch.from_numpy(s).cuda()
    got = lef(eng, yt, st, 0, 2)
    eng.sync()
    assert np.array_equal(got.cpu().numpy(), want)
    lef(eng, yt, st, 0, 2, out=yt)  # in place
    eng.sync()
    assert np.array_equal(yt.cpu().numpy(), want)


# ---- eICCI -----------------------------------------------------------------------------------

def _picture(seed, h, w):
    rng = np.random.default_rng(seed)
    base = rng.uniform(20.0, 235.0, (3, h // 8 + 2, w // 8 + 2)).astype(np.float32)
    big = np.repeat(np.repeat(base, 8, axis=1), 8, axis=2)[:, :h, :w]
    return [np.ascontiguousarray(big[i] + rng.normal(0, 6, (h, w)).astype(np.float32))
            for i in range(3)]


def _check(got, want, src):
    """The corrections (filtered minus input) within 5e-3 relative L2 of the oracle's; planes
    the filter leaves alone bit-exact."""
    for g, w_, s in zip(got, want, src):
        dw = w_.astype(np.float64) - np.clip(s, 0, 255)
        if np.abs(dw).max() < 1e-3:
            assert np.array_equal(g, w_)
        else:
            dg = g.astype(np.float64) - np.clip(s, 0, 255)
            assert np.linalg.norm(dg - dw) / np.linalg.norm(dw) < 5e-3
            assert np.abs(g - w_).max() < 0.05


@pytest.mark.parametrize("h,w,tile,overlap,sel", [
    (37, 50, 0, 0, (True, True, True, True)),
    (96, 128, 0, 0, (True, False, False, False)),
    (64, 80, 0, 0, (False, True, False, True)),
    (400, 600, 256, 32, (True, True, True, True)),
])
def test_icci_against_oracle(eng, h, w, tile, overlap, sel):
    import synthetic as syn
    from zenjpegai_b200 import filters
    use_y, use_uv, use_u, use_v = sel
    py, puv = syn.icci_params(5), syn.icci_params(6)
    ny = filters.icci_network(eng, py) if use_y else None
    nuv = filters.icci_network(eng, puv) if use_uv else None
    try:
        src = _picture(h + w, h, w)
        got = [p.copy() for p in src]
        filters.icci(eng, ny, nuv, *got, use_u=use_u, use_v=use_v, tile=tile, overlap=overlap)
        want = zo.icci_filter(zo.Checkpoint(py) if use_y else None,
                              zo.Checkpoint(puv) if use_uv else None, use_u, use_v, *src,
                              tile=tile, overlap=overlap)
        _check(got, want, src)
    finally:
        for n in (ny, nuv):
            if n:
                n.close()


def test_icci_device_tensors_and_errors(eng):
    import torch
    import synthetic as syn
    import zenjpegai_b200 as zj
    from zenjpegai_b200 import filters
    p = syn.icci_params(7)
    net = filters.icci_network(eng, p)
    try:
        src = _picture(3, 72, 88)
        host = [s.copy() for s in src]
        filters.icci(eng, net, net, *host)
        dev = [torch.from_numpy(s).cuda() for s in src]
        filters.icci(eng, net, net, *dev)
        eng.sync()
        for a, b in zip(dev, host):
            assert np.array_equal(a.cpu().numpy(), b)
        with pytest.raises(zj.ZjaiError):  # a last tile below the minimum with no room to grow
            filters.icci(eng, net, net, *[s.copy() for s in src], tile=64, overlap=8)
    finally:
        net.close()
    with pytest.raises(zj.ZjaiError):
        filters.icci_network(eng, {k: v for k, v in p.items() if not k.startswith("BNY")})
