"""EFE linear and non-linear post-filters (src/filters/efe_linear.rs, efe_nonlinear.rs) on the
GPU through the C ABI (`zjai_efe_linear`, `zjai_efe_nonlinear`), bit-exact against the
oracle's restatement: the reference's own unit cases, random coded sets over every supported
format, every split candidate and filter length, odd and tiny pictures, the on/off switch,
device tensors and in-place filtering of a 4K picture, and the crate's error statuses."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import oracle as zo
from test_efe_oracle import FORMATS, planes, ramp, random_nonlinear, random_set, wcode


@pytest.fixture(scope="module")
def eng():
    import zenjpegai_b200 as zj
    e = zj.Engine(0, arena_bytes=1 << 30)
    yield e
    e.close()


def test_reference_unit_cases(eng):
    from zenjpegai_b200.filters import efe_linear, efe_nonlinear
    # one-tap linear filter (efe_linear.rs `one_tap_filter_matches_the_formula`)
    y = ramp(5, 7, 1.5, 16.0)
    u, v = ramp(5, 7, -0.5, 130.0), ramp(5, 7, 0.25, 110.0)
    st = {"cand": [0, 0], "filter_len": [1, 1], "min_symbol": 0,
          "chroma": [[wcode(0.5)], [wcode(-0.25)]], "luma": [[wcode(0.25)], [wcode(0.0)]]}
    ou, ov = efe_linear(eng, y, u, v, (1, 1, 1, 1), (12000, 13000), st)
    f = np.float32
    assert np.array_equal(ou, ((u - f(120)) * f(1.5) + f(120)) + f(0.25) * y)
    assert np.array_equal(ov, ((v - f(130)) * f(0.75) + f(130)) + f(0))
    # tile network (efe_nonlinear.rs `tile_network_matches_the_formula`)
    codes = [wcode(0.0)] * 8
    codes[0], codes[2] = wcode(1.0), wcode(0.5)
    y = ramp(3, 5, 1.0, 35.0)
    u, v = ramp(3, 5, 2.0, 100.0), ramp(3, 5, 1.0, 50.0)
    v0 = v.copy()
    efe_nonlinear(eng, y, u, v, (1, 1, 1, 1),
                  {"tile_width": 64, "tile_height": 64, "luma_min": [1000], "luma_max": [9000],
                   "codes": [codes, None]})
    assert np.array_equal(v, v0)
    want = np.maximum((y - f(10)) + ramp(3, 5, 2.0, 100.0), 0) + f(0.5) * np.maximum(y - f(30), 0)
    assert np.array_equal(u, want)
    # switch (efe_nonlinear.rs `switch_takes_filtered_average_or_alternative`)
    fu, fv = ramp(4, 6, 1.0, 10.0), ramp(4, 6, 1.0, 50.0)
    au, av = ramp(4, 6, -1.0, 200.0), ramp(4, 6, -1.0, 150.0)
    mask = np.array([0, 1, 2, 2, 1, 0], np.uint8).reshape(2, 3)
    want_u, want_v = zo.efe_nonlinear(ramp(4, 6, 1.0, 35.0), fu, fv, (1, 1, 1, 1),
                                      {"mask_bs": 2, "masks": [mask, None]}, alt=(au, av))
    efe_nonlinear(eng, ramp(4, 6, 1.0, 35.0), fu, fv, (1, 1, 1, 1),
                  {"mask_bs": 2, "masks": [mask, None]}, alt=(au, av))
    assert np.array_equal(fu, want_u) and np.array_equal(fv, want_v)


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("size", [(37, 53), (64, 96), (9, 5), (130, 67), (2, 2), (1, 3)])
def test_linear_bit_exact(eng, fmt, size):
    from zenjpegai_b200.filters import efe_linear
    rng = np.random.default_rng(hash((fmt, size, 1)) % 2**32)
    y, u, v = planes(rng, *size, fmt)
    for _ in range(3):
        st = random_set(rng, fmt)
        mean = (int(rng.integers(5000, 20000)), int(rng.integers(5000, 20000)))
        want = zo.efe_linear(y, u, v, fmt, mean, st)
        got = efe_linear(eng, y, u, v, fmt, mean, st)
        assert np.array_equal(got[0], want[0]) and np.array_equal(got[1], want[1]), st["cand"]


@pytest.mark.parametrize("fmt", [(1, 1, 1, 1), (1, 1, 2, 2), (2, 2, 2, 2)])
def test_linear_every_candidate_and_length(eng, fmt):
    from zenjpegai_b200.filters import efe_linear
    rng = np.random.default_rng(7)
    y, u, v = planes(rng, 150, 171, fmt)
    for cand in range(8):
        for fl in range(1, 5):
            st = random_set(rng, fmt, fl=fl, cand=cand)
            want = zo.efe_linear(y, u, v, fmt, (12345, 6789), st)
            got = efe_linear(eng, y, u, v, fmt, (12345, 6789), st)
            assert np.array_equal(got[0], want[0]) and np.array_equal(got[1], want[1]), (cand, fl)


def test_linear_device_in_place_4k(eng):
    import torch
    from zenjpegai_b200.filters import efe_linear
    fmt = (2, 2, 2, 2)
    rng = np.random.default_rng(11)
    y, u, v = planes(rng, 2160, 3840, fmt)
    st = random_set(rng, fmt, fl=4, cand=6)
    want = zo.efe_linear(y, u, v, fmt, (11000, 13000), st)
    ty, tu, tv = (torch.from_numpy(a).cuda() for a in (y, u, v))
    efe_linear(eng, ty, tu, tv, fmt, (11000, 13000), st, out=(tu, tv))
    torch.cuda.synchronize()
    assert np.array_equal(tu.cpu().numpy(), want[0])
    assert np.array_equal(tv.cpu().numpy(), want[1])


def test_linear_errors_match_the_oracle(eng):
    import zenjpegai_b200 as zj
    from zenjpegai_b200.filters import efe_linear
    rng = np.random.default_rng(5)
    y, u, v = planes(rng, 20, 24, (2, 2, 2, 2))
    st = random_set(rng, (2, 2, 2, 2), fl=2, cand=1)
    off = {"cand": [None, None], "filter_len": [0, 0], "chroma": [None, None],
           "luma": [None, None]}
    cases = [((2, 2, 2, 2), dict(st, filter_len=[5, 2]), u, v),
             ((2, 2, 2, 2), dict(st, cand=[8, 1]), u, v),
             ((2, 2, 2, 2), st, u[:-1].copy(), v[:-1].copy()),
             ((2, 1, 2, 1), st, u, v),
             ((1, 1, 1, 1), off, y, y)]
    for fmt, s, pu, pv in cases:
        with pytest.raises(zo.EfeError) as e:
            zo.efe_linear(y, pu, pv, fmt, (100, 100), s)
        with pytest.raises(zj.ZjaiError) as g:
            efe_linear(eng, y, pu, pv, fmt, (100, 100), s)
        assert g.value.status == e.value.status, (fmt, s["cand"])


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("size", [(41, 58), (7, 3), (200, 333)])
def test_nonlinear_bit_exact(eng, fmt, size):
    from zenjpegai_b200.filters import efe_nonlinear
    rng = np.random.default_rng(hash((fmt, size, 2)) % 2**32)
    y, u, v = planes(rng, *size, fmt)
    for masks in (False, True):
        prm = random_nonlinear(rng, *u.shape, masks)
        alt = (rng.uniform(0, 255, u.shape).astype(np.float32),
               rng.uniform(0, 255, u.shape).astype(np.float32))
        want = zo.efe_nonlinear(y, u, v, fmt, prm, alt=alt)
        gu, gv = u.copy(), v.copy()
        efe_nonlinear(eng, y, gu, gv, fmt, prm, alt=alt)
        assert np.array_equal(gu, want[0]) and np.array_equal(gv, want[1])


def test_nonlinear_device_4k(eng):
    import torch
    from zenjpegai_b200.filters import efe_nonlinear
    fmt = (2, 2, 2, 2)
    rng = np.random.default_rng(13)
    y, u, v = planes(rng, 2160, 3840, fmt)
    prm = random_nonlinear(rng, *u.shape, True)
    alt = (rng.uniform(0, 255, u.shape).astype(np.float32),
           rng.uniform(0, 255, u.shape).astype(np.float32))
    want = zo.efe_nonlinear(y, u, v, fmt, prm, alt=alt)
    ty, tu, tv, ta, tb = (torch.from_numpy(a).cuda() for a in (y, u, v) + alt)
    efe_nonlinear(eng, ty, tu, tv, fmt, prm, alt=(ta, tb))
    torch.cuda.synchronize()
    assert np.array_equal(tu.cpu().numpy(), want[0])
    assert np.array_equal(tv.cpu().numpy(), want[1])


def test_nonlinear_errors_match_the_oracle(eng):
    import zenjpegai_b200 as zj
    from zenjpegai_b200.filters import efe_nonlinear
    rng = np.random.default_rng(17)
    fmt = (1, 1, 1, 1)
    y, u, v = planes(rng, 30, 40, fmt)
    good = random_nonlinear(rng, *u.shape, True)
    alt = (u.copy(), v.copy())
    cases = [(dict(good, tile_width=0), alt),
             (dict(good, luma_min=good["luma_min"][:1], luma_max=good["luma_max"][:1]), alt),
             (dict(good, mask_bs=good["mask_bs"] + 7), alt),
             (good, None)]
    for prm, a in cases:
        with pytest.raises(zo.EfeError) as e:
            zo.efe_nonlinear(y, u, v, fmt, prm, alt=a)
        with pytest.raises(zj.ZjaiError) as g:
            efe_nonlinear(eng, y, u.copy(), v.copy(), fmt, prm, alt=a)
        assert g.value.status == e.value.status
    with pytest.raises(zj.ZjaiError) as g:
        efe_nonlinear(eng, y, u, v, (2, 1, 2, 1), good, alt=alt)
    assert g.value.status == zj._lib.UNSUPPORTED
