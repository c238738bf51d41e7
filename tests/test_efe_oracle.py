"""The EFE post-filters' oracle (oracle/oracle.c `zo_efe_linear`, `zo_efe_nonlinear`), pinned
on the CPU.

Known answers: the reference's own unit tests for these filters
(src/filters/efe_linear.rs `split_edges_round_half_to_even_like_python`,
`one_tap_filter_matches_the_formula`, `formats_without_an_oracle_are_rejected`;
src/filters/efe_nonlinear.rs `tile_network_matches_the_formula`,
`switch_takes_filtered_average_or_alternative`), restated here with the same inputs and
expected values. The multi-tap paths (filters up to 4 x 4, DCT-IF taps, several regions, odd
sizes, every supported format) are checked against a float64 numpy restatement of the
reference's PyTorch formulation (pixel unshuffle, replicate padding, convolution per region,
pixel shuffle).
"""

import numpy as np
import pytest

import oracle as zo

# `EFElinear.cands` (src/filters/efe_linear.rs:34-73) and `DCT_IF_4TAP` (:77-110): format
# constants
SPLITS = [
    [[0, 1, 0, 1]],
    [[0, .5, 0, 1], [.5, 1, 0, 1]],
    [[0, 1, 0, .5], [0, 1, .5, 1]],
    [[0, 1, 0, .33], [0, 1, .33, .66], [0, 1, .66, 1]],
    [[0, .33, 0, 1], [.33, .66, 0, 1], [.66, 1, 0, 1]],
    [[0, .5, 0, .5], [0, .5, .5, 1], [.5, 1, 0, .5], [.5, 1, .5, 1]],
    [[0, .33, 0, .5], [0, .33, .5, 1], [.33, .66, 0, .5], [.33, .66, .5, 1], [.66, 1, 0, .5],
     [.66, 1, .5, 1]],
    [[0, .5, 0, .33], [.5, 1, 0, .33], [0, .5, .33, .66], [.5, 1, .33, .66], [0, .5, .66, 1],
     [.5, 1, .66, 1]],
]
DCT_IF = np.zeros((4, 4, 4))
DCT_IF[1, 1] = [-0.0625, -0.4375, 0.5625, -0.0625]
DCT_IF[2, :, 1] = [-0.0625, -0.4375, 0.5625, -0.0625]
DCT_IF[3] = np.outer([-0.0625, 0.5625, 0.5625, -0.0625], [-0.0625, 0.5625, 0.5625, -0.0625])
DCT_IF[3, 1, 1] -= 1.0  # the diagonal kernel carries -1 at its centre tap

# (s_ver, s_hor, c_ver, c_hor) the reference decodes (efe_linear.rs:364-379)
FORMATS = [(1, 1, 1, 1), (1, 1, 1, 2), (1, 1, 2, 2), (1, 2, 1, 2), (2, 2, 2, 2)]


def ramp(h, w, scale, base):
    return (base + scale * np.arange(h * w, dtype=np.float32)).reshape(h, w).astype(np.float32)


def wcode(w):
    """Weight code of w (the reference tests' `code`, round half away from zero)."""
    return int(np.floor(abs(w) * 2048 + 0.5) * np.sign(w)) + 32767


def test_dct_if_table_matches_the_listed_taps():
    # the diagonal kernel as efe_linear.rs:90-109 lists it
    d = DCT_IF[3].ravel()
    assert d[0] == 0.00390625 and d[1] == -0.03515625 and d[5] == -0.68359375
    assert d[6] == 0.31640625 and d[10] == 0.31640625 and d[15] == 0.00390625


def test_split_edges_known_answers():
    for s, want in [(444, [160, 224, 320, 480]), (280, [96, 160, 192, 320]),
                    (101, [32, 64, 96, 128]), (50, [32, 32, 64, 96]), (20, [32, 32, 32, 64]),
                    (129, [64, 64, 96, 160])]:
        assert [zo.efe_split_edge(f, s) for f in (0.33, 0.5, 0.66, 1.0)] == want, s
        # Python's own round (half to even) gives the same
        assert [int(round(f * (s + 31) / 32)) * 32 for f in (0.33, 0.5, 0.66, 1.0)] == want


def test_one_tap_filter_matches_the_formula():
    h, w = 5, 7
    y = ramp(h, w, 1.5, 16.0)
    u, v = ramp(h, w, -0.5, 130.0), ramp(h, w, 0.25, 110.0)
    st = {"cand": [0, 0], "filter_len": [1, 1], "min_symbol": 0,
          "chroma": [[wcode(0.5)], [wcode(-0.25)]], "luma": [[wcode(0.25)], [wcode(0.0)]]}
    ou, ov = zo.efe_linear(y, u, v, (1, 1, 1, 1), (12000, 13000), st)
    f = np.float32
    want_u = ((u - f(120)) * f(1.5) + f(120)) + f(0.25) * y
    want_v = ((v - f(130)) * f(0.75) + f(130)) + f(0)
    assert np.array_equal(ou, want_u)
    assert np.array_equal(ov, want_v)


def test_formats_without_an_oracle_are_rejected():
    st = {"cand": [None, None], "filter_len": [0, 0], "chroma": [None, None],
          "luma": [None, None]}
    y = u = v = ramp(4, 4, 1.0, 0.0)
    for fmt in [(1, 1, 1, 1), (2, 1, 2, 1), (1, 2, 2, 2)]:
        with pytest.raises(zo.EfeError) as e:
            zo.efe_linear(y, u, v, fmt, (0, 0), st)
        assert e.value.status == 2


def test_unfiltered_planes_below_the_source_resolution_get_the_dct_if_taps():
    # 4:4:4 source coded 4:2:0: an unfiltered plane still goes through the DCT-IF kernels
    y = ramp(6, 8, 1.0, 20.0)
    u, v = ramp(6, 8, 0.5, 90.0), ramp(6, 8, -0.25, 140.0)
    st = {"cand": [None, None], "filter_len": [0, 0], "chroma": [None, None],
          "luma": [None, None]}
    ou, ov = zo.efe_linear(y, u, v, (1, 1, 2, 2), (10000, 12000), st)
    ru, rv = linear_f64(y, u, v, (1, 1, 2, 2), (10000, 12000), st)
    assert np.abs(ou - ru).max() < 1e-3 and np.abs(ov - rv).max() < 1e-3
    assert not np.array_equal(ou, u)


def test_tile_network_matches_the_formula():
    codes = [wcode(0.0)] * 8
    codes[0], codes[2] = wcode(1.0), wcode(0.5)
    prm = {"tile_width": 64, "tile_height": 64, "luma_min": [1000], "luma_max": [9000],
           "codes": [codes, None]}
    y = ramp(3, 5, 1.0, 35.0)
    u, v = ramp(3, 5, 2.0, 100.0), ramp(3, 5, 1.0, 50.0)
    ou, ov = zo.efe_nonlinear(y, u, v, (1, 1, 1, 1), prm)
    assert np.array_equal(ov, v)
    f = np.float32
    want = np.maximum((y - f(10)) + u, 0) + f(0.5) * np.maximum(y - f(30), 0)
    assert np.array_equal(ou, want)


def test_switch_takes_filtered_average_or_alternative():
    fu, fv = ramp(4, 6, 1.0, 10.0), ramp(4, 6, 1.0, 50.0)
    au, av = ramp(4, 6, -1.0, 200.0), ramp(4, 6, -1.0, 150.0)
    y = ramp(4, 6, 1.0, 35.0)
    mask = np.array([0, 1, 2, 2, 1, 0], np.uint8).reshape(2, 3)
    prm = {"mask_bs": 2, "masks": [mask, None]}
    ou, ov = zo.efe_nonlinear(y, fu, fv, (1, 1, 1, 1), prm, alt=(au, av))
    assert np.array_equal(ov, fv)
    for r in range(4):
        for x in range(6):
            m = mask[r // 2, x // 2]
            want = fu[r, x] if m == 0 else (au[r, x] + fu[r, x]) / np.float32(2) if m == 1 \
                else au[r, x]
            assert ou[r, x] == want, (r, x)
    # masks need the EFE linear filter's second picture
    with pytest.raises(zo.EfeError) as e:
        zo.efe_nonlinear(y, fu, fv, (1, 1, 1, 1), prm)
    assert e.value.status == 6
    # a mask that does not cover the picture
    with pytest.raises(zo.EfeError) as e:
        zo.efe_nonlinear(y, fu, fv, (1, 1, 1, 1), {"mask_bs": 4, "masks": [mask, None]},
                         alt=(au, av))
    assert e.value.status == 6
    # the reference looks at the U mask alone: a V mask by itself does nothing
    ou, ov = zo.efe_nonlinear(y, fu, fv, (1, 1, 1, 1),
                              {"mask_bs": 2, "masks": [None, np.full((2, 3), 2, np.uint8)]})
    assert np.array_equal(ov, fv) and np.array_equal(ou, fu)


# ---- float64 restatement of the reference's PyTorch formulation -------------------------------

def deinteger(code):
    return (code - 32767) / 2048.0


def kernels(st, p, coded_444, s0, s1):
    """[(rows, cols, k, before, chroma[4] (k x k), luma (k x k))] of plane p."""
    weighted = st["cand"][p] is not None and st["cand"][p] >= 0
    cand = st["cand"][p] if weighted else 0
    fl = st["filter_len"][p] if weighted else 0
    out = []
    cw = np.asarray(st["chroma"][p], np.int64).ravel() if weighted else None
    lw = np.asarray(st["luma"][p], np.int64).ravel() if weighted else None
    ms = st.get("min_symbol", 0)
    for num, sp in enumerate(SPLITS[cand]):
        edge = lambda f, s: int(round(f * (s + 31) / 32)) * 32  # noqa: E731
        rows = (edge(sp[0], s0), min(edge(sp[1], s0), s0))
        cols = (edge(sp[2], s1), min(edge(sp[3], s1), s1))
        if rows[0] >= rows[1] or cols[0] >= cols[1]:
            continue
        if coded_444:
            k, before, off, centre = fl, (fl - 1) // 2, 0, (fl - 1) // 2
        else:
            k, before, off, centre = 4, 1, 1 - (max(fl, 1) - 1) // 2, 1
        luma = np.zeros((k, k))
        chroma = np.zeros((4, k, k))
        if weighted:
            nph = 1 if coded_444 else 4
            c = deinteger(cw[num * nph * fl * fl:(num + 1) * nph * fl * fl] + ms).reshape(nph, fl, fl)
            luma[off:off + fl, off:off + fl] = deinteger(
                lw[num * fl * fl:(num + 1) * fl * fl] + ms).reshape(fl, fl)
            for i in range(4):
                chroma[i, off:off + fl, off:off + fl] = c[0 if coded_444 else i]
        for i in range(4):
            if not coded_444:
                chroma[i] += DCT_IF[i]
            chroma[i, centre, centre] += 1.0
        out.append((rows, cols, k, before, chroma, luma))
    return out


def phase_padded(x, fv, fh, py, px, s0, s1):
    """`pixelUnshuffleGeneral` phase (py, px) of x, completed to s0 x s1 by clamping into the
    plane, then replicate-padded by 1 before and 2 after."""
    h, w = x.shape
    rows = np.minimum(np.arange(s0) * fv + py, h - 1)
    cols = np.arange(s1) * fh + px
    cols = np.where(cols < w, cols, w - 1)
    return np.pad(x[rows][:, cols].astype(np.float64), ((1, 2), (1, 2)), mode="edge")


def linear_f64(y, u, v, fmt, mean, st):
    s_ver, s_hor, c_ver, c_hor = fmt
    fv, fh = 3 - s_ver, 3 - s_hor
    h, w = y.shape
    s0, s1 = (h + 1) // 2, (w + 1) // 2
    coded_444 = (c_ver, c_hor) == (s_ver, s_hor)
    outs = []
    for p, src in enumerate((u, v)):
        m = float(np.float32(mean[p] / 100.0))
        out = np.zeros(src.shape)
        for rows, cols, k, before, chroma, luma in kernels(st, p, coded_444, s0, s1):
            for py in range(fv):
                for px in range(fh):
                    g = py * 2 + px
                    cp = phase_padded(src, fv, fh, py, px, s0, s1) - m
                    lp = phase_padded(y, 2, 2, py, px, s0, s1)
                    acc = np.zeros((rows[1] - rows[0], cols[1] - cols[0]))
                    for ky in range(k):
                        for kx in range(k):
                            r0, c0 = rows[0] + 1 + ky - before, cols[0] + 1 + kx - before
                            win = (slice(r0, r0 + acc.shape[0]), slice(c0, c0 + acc.shape[1]))
                            acc += chroma[g, ky, kx] * cp[win] + luma[ky, kx] * lp[win]
                    acc += m
                    # pixelShuffleGeneral, cropped to the plane
                    dst = out[py::fv, px::fh]
                    hh = min(rows[1], dst.shape[0]) - rows[0]
                    ww = min(cols[1], dst.shape[1]) - cols[0]
                    if hh > 0 and ww > 0:
                        dst[rows[0]:rows[0] + hh, cols[0]:cols[0] + ww] = acc[:hh, :ww]
        outs.append(out)
    return outs


def random_set(rng, fmt, fl=None, cand=None):
    coded_444 = (fmt[2], fmt[3]) == (fmt[0], fmt[1])
    st = {"cand": [], "filter_len": [], "min_symbol": int(rng.integers(0, 3000)),
          "chroma": [], "luma": []}
    for p in range(2):
        c = int(rng.integers(0, 8)) if cand is None else cand
        f = int(rng.integers(1, 5)) if fl is None else fl
        n = len(SPLITS[c])
        nph = 1 if coded_444 else 4
        # weights within about +-0.4 of zero: codes near 32767 - min_symbol
        base = 32767 - st["min_symbol"]
        st["cand"].append(c)
        st["filter_len"].append(f)
        st["chroma"].append(rng.integers(base - 800, base + 800, n * nph * f * f))
        st["luma"].append(rng.integers(base - 800, base + 800, n * f * f))
    return st


def planes(rng, h, w, fmt):
    ch, cw = -(-h // fmt[0]), -(-w // fmt[1])  # chroma planes of a source subsampled s_ver x s_hor
    y = rng.uniform(0, 255, (h, w)).astype(np.float32)
    u = rng.uniform(0, 255, (ch, cw)).astype(np.float32)
    v = rng.uniform(0, 255, (ch, cw)).astype(np.float32)
    return y, u, v


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("size", [(37, 53), (64, 96), (9, 5), (130, 67)])
def test_linear_oracle_against_float64(fmt, size):
    rng = np.random.default_rng(hash((fmt, size)) % 2**32)
    y, u, v = planes(rng, *size, fmt)
    for trial in range(3):
        st = random_set(rng, fmt)
        mean = (int(rng.integers(5000, 20000)), int(rng.integers(5000, 20000)))
        ou, ov = zo.efe_linear(y, u, v, fmt, mean, st)
        ru, rv = linear_f64(y, u, v, fmt, mean, st)
        assert np.abs(ou - ru).max() < 2e-3, (trial, st["cand"], st["filter_len"])
        assert np.abs(ov - rv).max() < 2e-3, (trial, st["cand"], st["filter_len"])


def test_linear_rejects_bad_sets_and_sizes():
    rng = np.random.default_rng(3)
    y, u, v = planes(rng, 20, 24, (2, 2, 2, 2))
    st = random_set(rng, (2, 2, 2, 2), fl=2, cand=1)
    bad = dict(st, filter_len=[5, 2])
    with pytest.raises(zo.EfeError) as e:
        zo.efe_linear(y, u, v, (2, 2, 2, 2), (100, 100), bad)
    assert e.value.status == 6
    bad = dict(st, cand=[8, 1])
    with pytest.raises(zo.EfeError) as e:
        zo.efe_linear(y, u, v, (2, 2, 2, 2), (100, 100), bad)
    assert e.value.status == 6
    with pytest.raises(zo.EfeError) as e:
        zo.efe_linear(y, u[:-1], v[:-1], (2, 2, 2, 2), (100, 100), st)
    assert e.value.status == 1


def nonlinear_f64(y, u, v, fmt, prm, alt=None):
    sv, sh = fmt[0], fmt[1]
    yd = y[::sv, ::sh].astype(np.float64)
    hh, ww = yd.shape
    out = [u.astype(np.float64), v.astype(np.float64)]
    th, tw = prm.get("tile_height", 0), prm.get("tile_width", 0)
    for p in range(2):
        codes = prm.get("codes", [None, None])[p]
        if codes is None:
            continue
        codes = np.asarray(codes, np.int64).reshape(-1, 8)
        nj = -(-ww // tw)
        for r in range(hh):
            for x in range(ww):
                idx = (r // th) * nj + x // tw
                wt = deinteger(codes[idx] + prm.get("min_symbol", 0))
                mn = prm["luma_min"][idx] / 100.0
                gap = (prm["luma_max"][idx] / 100.0 - mn) / 8
                l = yd[r, x]
                acc = max(wt[0] * (l - mn) + out[p][r, x], 0.0)
                for k in range(1, 8):
                    acc += wt[k] * max(l - (mn + k * gap), 0.0)
                out[p][r, x] = acc
    masks = prm.get("masks", [None, None])
    if masks[0] is not None:
        bs = prm["mask_bs"]
        for p in range(2):
            if masks[p] is None:
                continue
            m = np.repeat(np.repeat(np.asarray(masks[p]), bs, 0), bs, 1)[:hh, :ww]
            a = alt[p].astype(np.float64)
            out[p] = np.where(m == 0, out[p], np.where(m == 2, a, (a + out[p]) / 2))
    return out


def random_nonlinear(rng, hh, ww, with_masks):
    th, tw = int(rng.integers(4, 40)), int(rng.integers(4, 40))
    n = -(-hh // th) * -(-ww // tw)
    lmin = rng.integers(0, 12000, n)
    lmax = lmin + rng.integers(100, 13000, n)
    ms = int(rng.integers(0, 2000))
    base = 32767 - ms
    prm = {"min_symbol": ms, "tile_width": tw, "tile_height": th, "luma_min": lmin,
           "luma_max": lmax,
           "codes": [rng.integers(base - 600, base + 600, 8 * n),
                     None if rng.random() < 0.3 else rng.integers(base - 600, base + 600, 8 * n)]}
    if with_masks:
        bs = int(rng.integers(2, 17))
        my, mx = -(-hh // bs), -(-ww // bs)
        prm["mask_bs"] = bs
        prm["masks"] = [rng.integers(0, 3, (my, mx)), rng.integers(0, 3, (my, mx))]
    return prm


@pytest.mark.parametrize("fmt", FORMATS)
def test_nonlinear_oracle_against_float64(fmt):
    rng = np.random.default_rng(hash(fmt) % 2**32)
    y, u, v = planes(rng, 41, 58, fmt)
    for masks in (False, True):
        prm = random_nonlinear(rng, *u.shape, masks)
        alt = (rng.uniform(0, 255, u.shape).astype(np.float32),
               rng.uniform(0, 255, u.shape).astype(np.float32))
        ou, ov = zo.efe_nonlinear(y, u, v, fmt, prm, alt=alt)
        ru, rv = nonlinear_f64(y, u, v, fmt, prm, alt)
        assert np.abs(ou - ru).max() < 2e-3
        assert np.abs(ov - rv).max() < 2e-3
