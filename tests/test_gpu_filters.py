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
