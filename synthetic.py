"""Deterministic synthetic inputs and random-init weights for the benchmark configurations.

There are no trained checkpoints and no test pictures in this environment, so every tensor is
generated: SplitMix64 seeded per tensor as `seed ^ fnv1a64(name)`; uniforms are the top 24
bits / 2^24; normals are Box-Muller; Laplace variates use the inverse CDF. The oracle and the
GPU path read the same arrays, so both sides see bit-identical inputs.

The parameter names and shapes follow the reference's loaders (src/model/load.rs) and
topologies (src/model/synthesis.rs, attention.rs, analysis.rs).
"""

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def fnv1a64(s):
    h = 0xCBF29CE484222325
    for b in s.encode():
        h ^= b
        h = (h * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def splitmix64(seed, n):
    """n consecutive SplitMix64 outputs from state `seed` (uint64 array)."""
    with np.errstate(over="ignore"):
        i = np.arange(1, n + 1, dtype=np.uint64)
        z = np.uint64(seed) + i * _GOLDEN
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def _stream(seed, name, n):
    return splitmix64(np.uint64(seed) ^ np.uint64(fnv1a64(name)), n)


def uniform(seed, name, shape, lo=0.0, hi=1.0):
    n = int(np.prod(shape))
    u = ((_stream(seed, name, n) >> np.uint64(40)).astype(np.float64) + 0.5) / float(1 << 24)
    return (lo + (hi - lo) * u).astype(np.float32).reshape(shape)


def normal(seed, name, shape, std=1.0, mean=0.0):
    n = int(np.prod(shape))
    r = _stream(seed, name, 2 * n) >> np.uint64(40)
    u1 = (r[0::2].astype(np.float64) + 0.5) / float(1 << 24)
    u2 = (r[1::2].astype(np.float64) + 0.5) / float(1 << 24)
    z = np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)
    return (mean + std * z).astype(np.float32).reshape(shape)


def laplace_latent(seed, name, shape, scale, zero_p=0.442):
    """Integer latent: Laplace(scale) rounded, then zeroed with probability zero_p (so that
    about 60% of the values are zero at scale 1.5)."""
    n = int(np.prod(shape))
    r = _stream(seed, name, 2 * n) >> np.uint64(40)
    u = (r[0::2].astype(np.float64) + 0.5) / float(1 << 24) - 0.5
    x = -scale * np.sign(u) * np.log(1.0 - 2.0 * np.abs(u))
    x = np.rint(x)
    keep = (r[1::2].astype(np.float64) + 0.5) / float(1 << 24) >= zero_p
    return np.where(keep, x, 0.0).astype(np.float32).reshape(shape)


# ---------------------------------------------------------------------------------------------
# parameter specs: list of (name, shape, kind, effective fan_in = fan_in / gain^2)
#
# Plain He-normal everywhere (std sqrt(2 / fan_in)) makes the ResAU gates x * (1 + m)
# compound: HOP activations then pass 1e5 (beyond the f16 range) and 99.9% of the output
# samples clamp to 0 or 255, which leaves nothing for the 8-bit comparison to check. The
# weights are therefore normal with std gain * sqrt(1 / fan_in), the gain set by the layer's
# role: He (sqrt 2) before a ReLU/ReLU6, 1 for linear layers, a small gain on the ResAU mask
# conv (the gate stays near 1 + small) and on the residual branch, and an output gain that
# keeps the decoded samples mostly inside [0, 255].
# ---------------------------------------------------------------------------------------------
HE = 2.0 ** 0.5
MASK_GAIN = 0.1
RES_GAIN = 0.5
OUT_GAIN = 0.25

def _conv(specs, prefix, cin, cout, kh, kw, groups=1, bias=True, gain=1.0):
    specs.append((prefix + ".weight", (cout, cin // groups, kh, kw), "w",
                   cin // groups * kh * kw / gain ** 2))
    if bias:
        specs.append((prefix + ".bias", (cout,), "b", 0))


def _convt(specs, prefix, cin, cout, k, gain=1.0):
    # stride-2 transposed conv: about k*k/4 taps reach each output
    specs.append((prefix + ".weight", (cin, cout, k, k), "wt", max(1, cin * k * k // 4) / gain ** 2))
    specs.append((prefix + ".bias", (cout,), "b", 0))


def _resau(specs, prefix, c, per_group):
    _conv(specs, prefix + ".conv", c, c, 3, 3, groups=c // per_group, bias=False, gain=HE)
    _conv(specs, prefix + ".conv2", c, c, 1, 1, bias=False, gain=MASK_GAIN)


def _rb(specs, prefix, c):
    _conv(specs, prefix + ".conv1", c, c, 3, 3, gain=HE)
    _conv(specs, prefix + ".conv2", c, c, 3, 3, gain=RES_GAIN)


def _cab(specs, prefix, c):
    _rb(specs, prefix + ".residual_trunk.0", c)
    _rb(specs, prefix + ".residual_trunk.1", c)
    _conv(specs, prefix + ".subscale", c, c, 3, 3)
    _rb(specs, prefix + ".residual_mask2.0", c)
    _rb(specs, prefix + ".residual_mask3.0", c)
    _convt(specs, prefix + ".upscale", c, c, 3)


def _tb(specs, prefix, dim):
    hidden = 4 * dim
    specs.append((prefix + ".prep_data.norm1.weight", (dim,), "lnw", 0))
    specs.append((prefix + ".prep_data.norm1.bias", (dim,), "lnb", 0))
    _conv(specs, prefix + ".prep_data.conv1", dim, 3 * dim, 1, 1, bias=False)
    _conv(specs, prefix + ".prep_data.conv2", 3 * dim, 3 * dim, 3, 3, groups=3 * dim, bias=False)
    specs.append((prefix + ".attn.temperature", (4, 1, 1), "temp", 0))
    _conv(specs, prefix + ".attn.project_out", dim, dim, 1, 1, bias=False)
    specs.append((prefix + ".ffn.norm1.weight", (dim,), "lnw", 0))
    specs.append((prefix + ".ffn.norm1.bias", (dim,), "lnb", 0))
    _conv(specs, prefix + ".ffn.project_in", dim, 2 * hidden, 1, 1, bias=False)
    _conv(specs, prefix + ".ffn.dwconv", 2 * hidden, 2 * hidden, 3, 3, groups=2 * hidden,
          bias=False)
    _conv(specs, prefix + ".ffn.project_out", hidden, dim, 1, 1, bias=False)


def _tam(specs, prefix, dim, downsample):
    if downsample:
        _conv(specs, prefix + ".ds_conv", dim, dim, 3, 3)
        _convt(specs, prefix + ".us_conv", dim, dim, 3)
    _tb(specs, prefix + ".TABs.0", dim)
    _tb(specs, prefix + ".TABs.1", dim)


def _upsample(specs, op, prefix, cin, cout):
    if op == "bop":
        _convt(specs, prefix, cin, cout, 4)
    else:
        _conv(specs, prefix + ".conv", cin, 4 * cout, 2, 2, bias=False)


def synthesis_primary_spec(op):
    """`SynthesisPrimary::load` (synthesis.rs:241-246 -> LightPrimary::load :521-548,
    HopPrimary::load :340-354)."""
    s = []
    if op == "hop":
        c = 128
        _rb(s, "first_stage.0.0", 160)
        _convt(s, "first_stage.1", 160, c, 3)
        _resau(s, "first_stage.2", c, c // 4)
        _convt(s, "conv2_t", c, c, 3)
        _cab(s, "CAB", c)
        _resau(s, "iact2", c, c // 4)
        _conv(s, "conv3_t", c, 4 * c, 1, 1)
        _tam(s, "TAM", c, True)
        _resau(s, "iact3", c, c // 4)
        _convt(s, "conv4_t", c, 1, 3, gain=OUT_GAIN)
        return s
    c1, c2, c3 = (64, 32, 32) if op == "sop" else (64, 64, 96)
    _conv(s, "first_stage.0.0.conv1", 160, 160, 3, 3)
    _upsample(s, op, "first_stage.1", 160, c1)
    _resau(s, "first_stage.2", c1, 16)
    _upsample(s, op, "conv2_t", c1, c2)
    _resau(s, "iact2", c2, 16)
    _conv(s, "conv3", c2, c3, 3, 3)
    _resau(s, "iact3", c3, 16)
    _conv(s, "conv4", c3, 16, 1, 1, bias=False, gain=OUT_GAIN)
    return s


def synthesis_secondary_spec(op):
    """`SynthesisSecondary::load` (synthesis.rs:971-990)."""
    s = []
    _conv(s, "first_stage.conv1", 256, 48, 3, 3)
    if op == "hop":
        c = 64
        _convt(s, "conv2_t", 144, c, 3)
        _cab(s, "CAB", c)
        _resau(s, "iact2", c, c // 4)
        _conv(s, "conv3_t", c, 4 * c, 1, 1)
        _tam(s, "TAM", c, False)
        _resau(s, "iact3", c, c // 4)
        _convt(s, "conv4_t", c, 8, 3, gain=OUT_GAIN)
        return s
    c2, c3 = (32, 32) if op == "sop" else (64, 128)
    _upsample(s, op, "conv2_t", 144, c2)
    _resau(s, "iact2", c2, 16)
    _conv(s, "conv3", c2, c3, 3, 3)
    _resau(s, "iact3", c3, 16)
    _conv(s, "conv4", c3, 128, 1, 1, bias=False, gain=OUT_GAIN)
    return s


def analysis_spec(op, secondary):
    """`AnalysisPrimary::load` / `AnalysisSecondary::load` (analysis.rs:229-289)."""
    s = []
    c = 128
    pg = 32 if op == "hop" else 16
    _conv(s, "conv1", 12 if secondary else 1, c, 3, 3)
    _resau(s, "act1", c, pg)
    if op == "hop":
        _tam(s, "TAM", c, not secondary)
    _conv(s, "conv2", c, c, 3, 3)
    _resau(s, "act2", c, pg)
    if op == "hop":
        _cab(s, "cab", c)
    _conv(s, "conv3", c, c, 3, 3)
    _resau(s, "act3", c, pg)
    if secondary:
        _conv(s, "conv5", c, 96, 1, 1, bias=False)
    else:
        _conv(s, "conv4", c, 160, 3, 3)
        _conv(s, "conv5", 160, 160, 1, 1, bias=False)
    return s


def latent_spec(chs, context):
    """`HyperDecoder::load` (hyper_decoder.rs:24-42) and, with `context`, `ContextModel::load`
    (mcm.rs:119-156) for `chs` latent channels."""
    s = []
    _conv(s, "hyper_decoder.conv1", chs, chs, 1, 1, bias=False)
    _convt(s, "hyper_decoder.conv2", chs, chs, 4, gain=HE)
    _conv(s, "hyper_decoder.conv3", chs, chs, 3, 3, gain=HE)
    _conv(s, "hyper_decoder.conv4", chs, 4 * chs, 3, 3)
    if context:
        for st in range(4):
            p = "context.MCM.%d" % st
            if st:
                _conv(s, p + ".conv.0", st * chs, chs, 1, 1, bias=False)
                _conv(s, p + ".conv.1", chs, chs, 3, 3, groups=chs // 32)
            f = p + ".fusion_pred_net"
            _conv(s, f + ".conv1", 2 * chs if st else chs, chs, 1, 1, bias=False, gain=HE)
            _conv(s, f + ".conv2", chs, chs, 1, 1, bias=False, gain=HE)
            _conv(s, f + ".conv3", chs, chs, 1, 1, bias=False)
    return s


def make_params(spec, seed, tag=""):
    """Normal weights (std sqrt(1 / effective fan_in), see the gains above), N(0, 0.01^2)
    biases, LN weight 1 + N(0, 0.1^2) and bias N(0, 0.05^2), temperature U(0.5, 2)."""
    out = {}
    for name, shape, kind, fan_in in spec:
        key = tag + name
        if kind in ("w", "wt"):
            out[name] = normal(seed, key, shape, std=float(np.sqrt(1.0 / fan_in)))
        elif kind == "b":
            out[name] = normal(seed, key, shape, std=0.01)
        elif kind == "lnw":
            out[name] = normal(seed, key, shape, std=0.1, mean=1.0)
        elif kind == "lnb":
            out[name] = normal(seed, key, shape, std=0.05)
        elif kind == "temp":
            out[name] = uniform(seed, key, shape, 0.5, 2.0)
        else:
            raise ValueError(kind)
    return out


def he_normal(spec, seed, tag=""):
    """The law BASELINE prescribes: every conv / transposed-conv weight N(0, 2 / fan_in) with
    PyTorch's fan_in (dim 1 x kernel taps: in / groups x kh x kw for a conv [out][in / g][kh][kw],
    out x k x k for a transposed conv [in][out][k][k]); biases, layer-norm parameters and
    temperatures as in make_params."""
    out = make_params(spec, seed, tag)
    for name, shape, kind, _ in spec:
        if kind in ("w", "wt"):
            fan = int(np.prod(shape[1:]))
            out[name] = normal(seed, tag + name, shape, std=float(np.sqrt(2.0 / fan)))
    return out


def synthesis_params_he(op, seed):
    """(luma params, chroma params) with the prescribed He-normal weight law."""
    return (he_normal(synthesis_primary_spec(op), seed, "Y/"),
            he_normal(synthesis_secondary_spec(op), seed, "UV/"))


def synthesis_params(op, seed):
    """(luma params, chroma params) for operating point `op` ('sop' | 'bop' | 'hop')."""
    return (make_params(synthesis_primary_spec(op), seed, "Y/"),
            make_params(synthesis_secondary_spec(op), seed, "UV/"))


def analysis_params(op, seed):
    return (make_params(analysis_spec(op, False), seed, "AY/"),
            make_params(analysis_spec(op, True), seed, "AUV/"))


def icci_params(seed):
    """One eICCI network (`IcciNet::load`, src/model/icci.rs:181-212): both trunks (48
    features; luma 2 residual blocks, chroma 4), batch norms with running statistics, the
    learned residual scales and the three last convs."""
    out = {}
    nf, bands = 48, 16

    def conv(name, cout, cin, kh, kw, gain=1.0):
        fan = cin * kh * kw
        out[name + ".weight"] = normal(seed, "IC/" + name, (cout, cin, kh, kw),
                                       std=float(np.sqrt(gain / fan)))
        out[name + ".bias"] = normal(seed, "IC/" + name + ".b", (cout,), std=0.01)

    def bn(name):
        out[name + ".weight"] = normal(seed, "IC/" + name + ".g", (nf,), std=0.1, mean=1.0)
        out[name + ".bias"] = normal(seed, "IC/" + name + ".be", (nf,), std=0.05)
        out[name + ".running_mean"] = normal(seed, "IC/" + name + ".m", (nf,), std=0.05)
        out[name + ".running_var"] = uniform(seed, "IC/" + name + ".v", (nf,), 0.5, 1.5)

    def scalar(name, lo, hi):
        out[name] = uniform(seed, "IC/" + name, (1,), lo, hi)

    for first, bnn, hidden, blocks in (("conv_first_Y", "BNY", "hidden_layer_Y", 2),
                                       ("conv_firstUV", "BNUV", "hidden_layer_UV", 4)):
        conv(first, nf, 3 * bands, 3, 3, 2.0)
        bn(bnn)
        for i in range(blocks):
            p = "%s.%d" % (hidden, i)
            conv(p + ".conv1", nf, nf, 1, 3, 2.0)
            conv(p + ".conv2", nf, nf, 3, 1, 1.0)
            bn(p + ".BN1")
            bn(p + ".BN2")
            scalar(p + ".scale", 0.1, 0.5)
    for last, sc in (("conv_last_Y", "scaleY"), ("conv_last_u", "scaleU"), ("conv_last_v", "scaleV")):
        conv(last, bands, nf, 3, 3, 1.0)
        scalar(sc, 0.01, 0.05)
    return out


def latent_params(seed, chs=160, context=True):
    """A component's latent networks (hyper-decoder, optional context model)."""
    return make_params(latent_spec(chs, context), seed, "L%d/" % chs)


def conv_layer_params(seed=0):
    """conv 3x3 128 -> 128, weights N(0, 1/(9*128)), bias N(0, 0.01^2)
    (read as standard deviation 0.01), as a conv stage's `conv.*` parameters."""
    return {"conv.weight": normal(seed, "w", (128, 128, 3, 3),
                                  std=float(np.sqrt(1.0 / (9 * 128)))),
            "conv.bias": normal(seed, "b", (128,), std=0.01)}


def upsample_stage_params(seed=1, cin=192, cout=128, nres=2):
    """conv 3x3 cin -> 4 cout (then depth-to-space 2) and `nres` residual
    blocks of two 3x3 convs at cout channels; He-normal weights (variance 2 / fan_in), zero
    biases (the configuration names no bias law)."""
    he = lambda name, shape: normal(seed, name, shape,
                                    std=float(np.sqrt(2.0 / (shape[1] * shape[2] * shape[3]))))
    out = {"conv.weight": he("up/w", (4 * cout, cin, 3, 3)),
           "conv.bias": np.zeros(4 * cout, np.float32)}
    for i in range(nres):
        for j in (1, 2):
            p = "res.%d.conv%d" % (i, j)
            out[p + ".weight"] = he(p + "/w", (cout, cout, 3, 3))
            out[p + ".bias"] = np.zeros(cout, np.float32)
    return out
