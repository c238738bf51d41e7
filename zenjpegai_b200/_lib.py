"""ctypes binding of `libzjai.so` (the C ABI of include/zjai.h).

This is the Python host side above the C ABI. It fails loudly: if the CUDA library is not
built or cannot be loaded, importing the binding raises; there is no CPU fallback.
"""

import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libzjai.so")
HEADER = os.path.join(HERE, "..", "include", "zjai.h")

OK, INVALID_ARGUMENT, UNSUPPORTED, LIMIT_EXCEEDED, CANCELLED, MODEL, INVALID_DATA, DEVICE, \
    DEVICE_TIMEOUT = range(9)
STATUS_NAMES = ["OK", "INVALID_ARGUMENT", "UNSUPPORTED", "LIMIT_EXCEEDED", "CANCELLED", "MODEL",
                "INVALID_DATA", "DEVICE", "DEVICE_TIMEOUT"]
MEM_HOST, MEM_DEVICE = 0, 1
SOP, BOP, HOP = 0, 1, 2
SYN_Y, SYN_UV, ANA_Y, ANA_UV = 0, 1, 2, 3
LATENT = 5
ICCI = 6
ACT_NONE, ACT_RELU, ACT_LEAKY, ACT_SIGMOID, ACT_RELU6 = range(5)


class ZjaiError(RuntimeError):
    """A failing zjai call: `.status` is the zjai_status code, mirroring the crate's Error."""

    def __init__(self, status, msg):
        name = STATUS_NAMES[status] if 0 <= status < len(STATUS_NAMES) else str(status)
        super().__init__("%s: %s" % (name, msg))
        self.status = status


_f = ctypes.POINTER(ctypes.c_float)
_i = ctypes.c_int
_vp = ctypes.c_void_p


class Param(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("ndim", _i), ("shape", ctypes.c_int64 * 4),
                ("data", _f)]


class Tile(ctypes.Structure):
    _fields_ = [(k, _i) for k in (
        "img_x", "img_y", "img_w", "img_h", "lat_x", "lat_y", "lat_w", "lat_h",
        "core_x", "core_y", "core_w", "core_h", "off_x", "off_y")]


_u32p = ctypes.POINTER(ctypes.c_uint32)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_u8p = ctypes.POINTER(ctypes.c_uint8)


class EfeLinearSet(ctypes.Structure):
    _fields_ = [("cand", _i * 2), ("filter_len", _i * 2), ("min_symbol", _i),
                ("chroma_codes", _u32p * 2), ("luma_codes", _u32p * 2)]


class EfeNonlinearParams(ctypes.Structure):
    _fields_ = [("min_symbol", _i), ("tile_width", _i), ("tile_height", _i), ("ntiles", _i),
                ("luma_min", _u16p), ("luma_max", _u16p), ("codes", _u32p * 2),
                ("ncodes", _i * 2), ("mask_bs", _i), ("mask_h", _i), ("mask_w", _i),
                ("mask", _u8p * 2)]


class CabTape(ctypes.Structure):
    _fields_ = [("trunk_pre", _vp), ("sig", _vp), ("rb_c1", _vp * 2), ("mask_c1", _vp * 2)]


class CabWeights(ctypes.Structure):
    _fields_ = [("trunk", (_vp * 2) * 2), ("subscale", _vp), ("mask2", _vp * 2),
                ("mask3", _vp * 2), ("upscale", _vp)]


class TbTape(ctypes.Structure):
    _fields_ = [(k, _vp) for k in ("x_in", "qkv", "attn", "x_mid", "gate")]


class TbWeights(ctypes.Structure):
    _fields_ = [(k, _vp) for k in ("prep_norm", "prep_conv1", "prep_conv2", "temperature",
                                   "attn_out", "ffn_norm", "ffn_in", "ffn_dw", "ffn_out")]


_lib = None


def header_functions():
    """Names of every function declared in include/zjai.h."""
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(zjai_[a-z0-9_]+)\s*\(", src)))


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError("zenjpegai_b200: %s is not built (run zenjpegai_b200/build.py)"
                          % LIB_PATH)
    L = ctypes.CDLL(LIB_PATH)
    L.zjai_version.restype = ctypes.c_char_p
    L.zjai_last_error_message.restype = ctypes.c_char_p
    L.zjai_ctx_create.argtypes = [_i, ctypes.c_size_t, ctypes.POINTER(_vp)]
    L.zjai_ctx_destroy.argtypes = [_vp]
    L.zjai_ctx_set_stream.argtypes = [_vp, _vp]
    L.zjai_ctx_sync.argtypes = [_vp]
    L.zjai_ctx_set_output_clamp.argtypes = [_vp, _i]
    L.zjai_ctx_set_wait_limit.argtypes = [_vp, ctypes.c_int64]
    L.zjai_ctx_launch_count.argtypes = [_vp]
    L.zjai_ctx_launch_count.restype = ctypes.c_int64
    L.zjai_ctx_profile.argtypes = [_vp, _i]
    L.zjai_ctx_set_graphs.argtypes = [_vp, _i]
    L.zjai_ctx_set_probe.argtypes = [_vp, ctypes.c_char_p, _vp, ctypes.c_int64]
    L.zjai_ctx_profile_read_bytes.argtypes = [_vp, ctypes.POINTER(ctypes.c_double),
                                              ctypes.POINTER(ctypes.c_double),
                                              ctypes.POINTER(ctypes.c_double),
                                              ctypes.POINTER(ctypes.c_int64)]
    L.zjai_ctx_profile_read.argtypes = [_vp, ctypes.POINTER(ctypes.c_double),
                                        ctypes.POINTER(ctypes.c_double),
                                        ctypes.POINTER(ctypes.c_int64)]
    L.zjai_net_create.argtypes = [_vp, _i, _i, ctypes.POINTER(Param), _i, ctypes.POINTER(_vp)]
    L.zjai_net_destroy.argtypes = [_vp]
    L.zjai_synth_out_size.argtypes = [_i, _i, _i, _i, ctypes.POINTER(_i), ctypes.POINTER(_i)]
    L.zjai_synthesis_primary.argtypes = [_vp, _vp, _i, _i, _i, _i, _vp, _i]
    L.zjai_synthesis_secondary.argtypes = [_vp, _vp, _i, _i, _vp, _i, _i, _i, _i, _vp, _i]
    L.zjai_analysis_primary.argtypes = [_vp, _vp, _i, _i, _vp, _i]
    L.zjai_analysis_secondary.argtypes = [_vp, _vp, _i, _i, _vp, _i]
    L.zjai_synthesize_rgb.argtypes = [_vp, _vp, _vp, _vp, _vp] + [_i] * 7 + [_vp, _i, _vp]
    L.zjai_synthesize_batch.argtypes = [_vp, _vp, _vp, _i, _vp, _vp] + [_i] * 11 + [_vp, _vp,
                                                                                  _vp, _i, _vp]
    L.zjai_preprocess_rgb.argtypes = [_vp, _vp, _i, _i, _vp, _vp, _i]
    L.zjai_analyze_rgb.argtypes = [_vp, _vp, _vp, _i, _vp, _i, _i, _vp, _vp, _i]
    L.zjai_ipc_export.argtypes = [_vp, _vp, _vp, ctypes.POINTER(ctypes.c_uint64)]
    L.zjai_ipc_import.argtypes = [_vp, _vp, ctypes.c_uint64, ctypes.POINTER(_vp)]
    L.zjai_ipc_close.argtypes = [_vp, _vp]
    L.zjai_stage_create.argtypes = [_vp, _i, _i, _i, ctypes.POINTER(Param), _i,
                                     ctypes.POINTER(_vp)]
    L.zjai_stage_forward.argtypes = [_vp, _vp, _i, _i, _i, _vp, _i]
    L.zjai_ckpt_open.argtypes = [_vp, ctypes.c_size_t, ctypes.POINTER(_vp)]
    L.zjai_ckpt_close.argtypes = [_vp]
    L.zjai_ckpt_count.argtypes = [_vp, ctypes.POINTER(_i), ctypes.POINTER(_i), ctypes.POINTER(_i)]
    L.zjai_ckpt_tensor.argtypes = [_vp, _i, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(_i),
                                   ctypes.POINTER(_i), ctypes.POINTER(ctypes.c_int64)]
    L.zjai_ckpt_find.argtypes = [_vp, ctypes.c_char_p, ctypes.POINTER(_i)]
    L.zjai_ckpt_read.argtypes = [_vp, _i, _vp, ctypes.c_size_t]
    L.zjai_ckpt_int.argtypes = [_vp, _i, ctypes.POINTER(ctypes.c_char_p),
                                ctypes.POINTER(ctypes.c_int64)]
    L.zjai_ckpt_list.argtypes = [_vp, _i, ctypes.POINTER(ctypes.c_char_p),
                                 ctypes.POINTER(ctypes.POINTER(ctypes.c_double)), ctypes.POINTER(_i)]
    L.zjai_ckpt_params.argtypes = [_vp, ctypes.POINTER(ctypes.POINTER(Param)), ctypes.POINTER(_i)]
    L.zjai_bundle_open.argtypes = [_vp, ctypes.c_size_t, ctypes.POINTER(_vp)]
    L.zjai_bundle_close.argtypes = [_vp]
    L.zjai_bundle_info.argtypes = [_vp, ctypes.POINTER(_i), ctypes.POINTER(_i),
                                   ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_size_t)]
    L.zjai_bundle_file.argtypes = [_vp, _i, ctypes.POINTER(ctypes.c_char_p),
                                   ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_size_t)]
    L.zjai_icci_filter.argtypes = [_vp, _vp, _vp, _i, _i, _vp, _vp, _vp, _i, _i, _i, _i, _i]
    L.zjai_lef.argtypes = [_vp, _vp, _i, _i, _vp, _i, _i, _i, _i, _i, _i, _vp, _i]
    L.zjai_efe_linear.argtypes = [_vp, _vp, _i, _i, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i,
                                  ctypes.POINTER(EfeLinearSet), _vp, _vp, _i]
    L.zjai_efe_nonlinear.argtypes = [_vp, _vp, _i, _i, _vp, _vp, _i, _i, _i, _i, _i, _i,
                                     ctypes.POINTER(EfeNonlinearParams), _vp, _vp, _i]
    L.zjai_hyper_decode.argtypes = [_vp, _vp, _i, _i, _i, _i, _vp, _i]
    L.zjai_context_decompress.argtypes = [_vp, _vp, _i, _i, _vp, _vp, _i]
    L.zjai_reconstruct_latent.argtypes = [_vp, _vp, _i, _i, _vp, _i, _i, _vp, _vp, _i]
    L.zjai_synthesis_tiles.argtypes = [_i] * 6 + [ctypes.POINTER(Tile), _i, ctypes.POINTER(_i)]
    L.zjai_synthesize.argtypes = [_vp, _vp, _vp, _vp, _vp] + [_i] * 10 + [_vp, _vp, _vp, _i, _vp]
    L.zjai_synthesize_q.argtypes = [_vp, _vp, _vp, _vp, _vp] + [_i] * 11 + [_vp, _vp, _vp, _i,
                                                                            _vp]
    L.zjai_synthesize_tiles.argtypes = [_vp, _vp, _vp, _vp, _vp, _i, _i, ctypes.POINTER(Tile),
                                        _i, _i, _i, _i, _i, _vp, _vp, _vp, _i, _vp]
    L.zjai_synthesize_tiles_q.argtypes = [_vp, _vp, _vp, _vp, _vp, _i, _i, ctypes.POINTER(Tile),
                                          _i, _i, _i, _i, _i, _i, _vp, _vp, _vp, _i, _vp]
    L.zjai_quantize_plane.argtypes = [_vp, _vp, ctypes.c_int64, _i, _vp, _i]
    L.zjai_yuv_to_rgb.argtypes = [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _i]
    L.zjai_conv2d.argtypes = [_vp, _vp, _i, _i, _i, _vp, _vp, _i, _i, _i, _i, _i, _i, _i,
                              ctypes.POINTER(_i), _i, _vp, _i]
    L.zjai_conv_transpose2d.argtypes = [_vp, _vp, _i, _i, _i, _vp, _vp, _i, _i, _i, _i, _vp, _i]
    L.zjai_conv2d_backward.argtypes = [_vp, _vp, _i, _i, _i, _vp, _i, _i, _i, _i, _i, _i, _i,
                                       _vp, _i, _i, _vp, _i]
    L.zjai_conv_transpose2d_backward.argtypes = [_vp, _vp, _i, _i, _i, _vp, _i, _i, _i, _i, _i,
                                                 _vp, _i]
    L.zjai_residual_block_backward.argtypes = [_vp, _vp, _vp, _i, _i, _i, _vp, _vp, _vp, _i]
    L.zjai_cab_backward.argtypes = [_vp, _vp, _i, _i, _i, ctypes.POINTER(CabTape),
                                    ctypes.POINTER(CabWeights), _vp, _i]
    L.zjai_elu_gate_backward.argtypes = [_vp, _vp, _vp, _vp, ctypes.c_int64, _vp, _vp, _i]
    L.zjai_layer_norm_backward.argtypes = [_vp, _vp, _vp, _i, _i, _i, _vp, _vp, _i]
    L.zjai_channel_attention_backward.argtypes = [_vp, _vp, _i, _i, _i, _i, _vp, _vp, _vp, _vp,
                                                  _i]
    L.zjai_transformer_block_backward.argtypes = [_vp, _vp, _i, _i, _i, _i, _i,
                                                  ctypes.POINTER(TbTape),
                                                  ctypes.POINTER(TbWeights), _vp, _i]
    L.zjai_layer_norm.argtypes = [_vp, _vp, _i, _i, _i, _vp, _vp, _vp, _i]
    L.zjai_channel_attention.argtypes = [_vp, _vp, _i, _i, _i, _i, _vp, _vp, _i]
    L.zjai_depthwise3x3.argtypes = [_vp, _vp, _i, _i, _i, _vp, _vp, _i]
    L.zjai_depthwise3x3_elu_gate.argtypes = [_vp, _vp, _i, _i, _i, _vp, _vp, _i]
    L.zjai_transformer_ffn.argtypes = [_vp, _vp, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _i]
    _dp = ctypes.POINTER(ctypes.c_double)
    L.zjai_conv_bench.argtypes = [_vp] + [_i] * 11 + [_dp, _dp]
    L.zjai_kernel_bench.argtypes = [_vp] + [_i] * 6 + [_dp, _dp]
    _lib = L
    return L


def check(status):
    if status != OK:
        msg = lib().zjai_last_error_message().decode(errors="replace")
        raise ZjaiError(status, msg)
