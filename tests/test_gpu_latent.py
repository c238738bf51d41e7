"""GPU parity of the latent-domain float networks (hyper-decoder z_hat -> psi, context model
psi, residual -> y_hat; src/model/{hyper_decoder,mcm}.rs, src/decoder/reconstruct.rs:107-230)
through the C ABI, against the CPU oracle.

Tolerances (f16 activations, f32 accumulation, like the synthesis layers): psi within
PSI_REL relative L2; the context model's prediction (y_hat minus the residual, i.e. the four
stages' means, whose error compounds through the stage-to-stage context) within MEAN_REL; the
residual itself passes through in f32, so y_hat minus the residual is what is gated.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import oracle as zo
import synthetic as syn

PSI_REL = 2e-3
MEAN_REL = 5e-3


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def eng():
    import zenjpegai_b200 as zj
    e = zj.Engine(0, arena_bytes=4 << 30)
    yield e
    e.close()


def _model(eng, chs, context, seed=21):
    import zenjpegai_b200 as zj
    p = syn.latent_params(seed, chs, context)
    return zj.LatentModel(eng, p), zo.Checkpoint(p)


def _inputs(chs, h, w, seed=30):
    hz, wz = -(-h // 4), -(-w // 4)
    z = np.round(syn.laplace_latent(seed, "z", (chs, hz, wz), 2.0)).astype(np.float32)
    res = syn.laplace_latent(seed, "res", (chs, h, w), 1.0)
    return z, res


@pytest.mark.parametrize("chs,h,w", [(160, 16, 24), (160, 17, 23), (96, 9, 14), (160, 1, 1)])
def test_hyper_decode(eng, chs, h, w):
    m, ck = _model(eng, chs, False)
    try:
        z, _ = _inputs(chs, h, w)
        hh, hw = -(-h // 2), -(-w // 2)
        got = m.hyper_decode(z, hh, hw)
        want = zo.hyper_decode(ck, z, hh, hw)
        assert got.shape == want.shape
        assert rel_l2(got, want) < PSI_REL
    finally:
        m.close()


@pytest.mark.parametrize("h,w", [(16, 24), (17, 23), (1, 1), (2, 3)])
def test_context_decompress(eng, h, w):
    m, ck = _model(eng, 160, True)
    try:
        _, res = _inputs(160, h, w)
        psi = syn.normal(40, "psi", (640, -(-h // 2), -(-w // 2)))
        got = m.decompress(res, psi)
        want = zo.context_decompress(ck, res, psi)
        assert rel_l2(got - res, want - res) < MEAN_REL
    finally:
        m.close()


def test_no_context_bit_exact(eng):
    """Chroma (no context model): upshuffle_psi + residual is one f32 add, bit-exact."""
    m, ck = _model(eng, 96, False)
    try:
        _, res = _inputs(96, 11, 14)
        psi = syn.normal(41, "psi", (384, 6, 7))
        got = m.decompress(res, psi)
        assert np.array_equal(got, zo.context_decompress(ck, res, psi))
    finally:
        m.close()


@pytest.mark.parametrize("chs,context", [(160, True), (96, False)])
def test_reconstruct_latent_4k(eng, chs, context):
    """One 4K picture's latent (3840 x 2160: luma latent 135 x 240, z 34 x 60; chroma 4:2:0
    latent 68 x 120, z 17 x 30): psi and y_hat against the oracle, and the fused call equal to
    the two separate calls."""
    m, ck = _model(eng, chs, context)
    try:
        h, w = (135, 240) if chs == 160 else (68, 120)
        z, res = _inputs(chs, h, w)
        hh, hw = -(-h // 2), -(-w // 2)
        y, psi = m.reconstruct(z, res, with_psi=True)
        zo.set_fast(True)
        zo.set_threads(16)
        try:
            wpsi = zo.hyper_decode(ck, z, hh, hw)
            wy = zo.context_decompress(ck, res, wpsi)
        finally:
            zo.set_fast(False)
        assert rel_l2(psi, wpsi) < PSI_REL
        assert rel_l2(y - res, wy - res) < MEAN_REL
        psi2 = m.hyper_decode(z, hh, hw)
        assert np.array_equal(psi2, psi)
        assert np.array_equal(m.decompress(res, psi2), y)
    finally:
        m.close()


def test_device_tensors(eng):
    import torch
    m, ck = _model(eng, 160, True)
    try:
        z, res = _inputs(160, 20, 28)
        y_host, psi_host = m.reconstruct(z, res, with_psi=True)
        zt = torch.from_numpy(z).cuda()
        rt = torch.from_numpy(res).cuda()
        y_dev, psi_dev = m.reconstruct(zt, rt, with_psi=True)
        torch.cuda.synchronize()
        assert np.array_equal(y_dev.cpu().numpy(), y_host)
        assert np.array_equal(psi_dev.cpu().numpy(), psi_host)
    finally:
        m.close()


def test_errors(eng):
    import zenjpegai_b200 as zj
    m, _ = _model(eng, 160, True)
    try:
        z = np.zeros((160, 2, 2), np.float32)
        with pytest.raises(zj.ZjaiError):
            m.hyper_decode(z, 5, 4)  # larger than the 4 x 4 upsampled map
        with pytest.raises(zj.ZjaiError):
            m.decompress(np.zeros((160, 4, 4), np.float32), np.zeros((640, 3, 2), np.float32))
    finally:
        m.close()
    with pytest.raises(zj.ZjaiError):
        zj.LatentModel(eng, syn.latent_params(1, 48, context=True))  # context needs 32 | C
