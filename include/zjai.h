/*
 * zjai — B200 (sm_100a) engine for the JPEG AI synthesis / analysis networks.
 *
 * Plain C ABI (no C++ or torch types): opaque handles, plain pointers and sizes, an int
 * status. It replaces the float-network path of the imazen/zenjpegai crate behind the
 * crate's own interfaces; each entry names the reference interface it stands in for
 * (paths are files of that crate). A Rust `extern "C"` binding of this header is mechanical:
 * one `extern "C"` declaration per function, `#[repr(C)]` mirrors of the two structs.
 *
 * Conventions
 *  - Tensors crossing the ABI are planar f32 `[c][h][w]`, like the crate's `Tensor<f32>`
 *    (src/tensor.rs:10-120). `mem` says whether the pointers are host (ZJAI_MEM_HOST) or
 *    device (ZJAI_MEM_DEVICE) memory of the context's GPU. Host calls are synchronous: they
 *    return after the output has been written. Device calls are ordered on the context's
 *    stream and return after the work has been enqueued (zjai_ctx_sync waits). Buffers passed
 *    as ZJAI_MEM_DEVICE are checked first (device memory of the context's GPU, managed
 *    memory or mapped pinned host memory); anything else returns ZJAI_INVALID_ARGUMENT before
 *    any kernel runs.
 *  - The caller owns inputs and outputs; the library owns weights and scratch.
 *  - One call in flight per context at a time; separate contexts are independent and may be
 *    used from separate host threads.
 *  - Every function returns a zjai_status; zjai_last_error_message() describes the last
 *    failure on the calling thread.
 */
#ifndef ZJAI_H
#define ZJAI_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* Status codes: the variants of the crate's `Error` (src/error.rs:10-31) this path can
 * produce, plus the device-side failures. */
typedef enum {
  ZJAI_OK = 0,
  ZJAI_INVALID_ARGUMENT = 1, /* Error::InvalidArgument */
  ZJAI_UNSUPPORTED = 2,      /* Error::Unsupported */
  ZJAI_LIMIT_EXCEEDED = 3,   /* Error::LimitExceeded (arena / size limits, or an activation
                              * beyond the f16 range, reported at the next synchronising call) */
  ZJAI_CANCELLED = 4,        /* Error::Cancelled (the caller's stop flag was set) */
  ZJAI_MODEL = 5,            /* Error::Model (missing / mis-shaped parameter) */
  ZJAI_INVALID_DATA = 6,     /* Error::InvalidData (malformed tile geometry) */
  ZJAI_DEVICE = 7,           /* a CUDA call failed */
  ZJAI_DEVICE_TIMEOUT = 8    /* a kernel's bounded wait gave up (status word set) */
} zjai_status;

enum { ZJAI_MEM_HOST = 0, ZJAI_MEM_DEVICE = 1 };

/* Operating points (src/header.rs `OperatingPoint`). */
enum { ZJAI_SOP = 0, ZJAI_BOP = 1, ZJAI_HOP = 2 };

/* Network kinds: synthesis primary / secondary (src/model/synthesis.rs), analysis primary /
 * secondary (src/model/analysis.rs), and the latent-domain float networks of one component's
 * common modules (src/model/common.rs:34-131): the hyper-decoder (hyper_decoder.rs) and, when
 * the checkpoint holds it, the context model (mcm.rs); one network of the eICCI post-filter bank
 * (src/model/icci.rs `IcciNet`). */
enum { ZJAI_SYN_Y = 0, ZJAI_SYN_UV = 1, ZJAI_ANA_Y = 2, ZJAI_ANA_UV = 3, ZJAI_LATENT = 5,
       ZJAI_ICCI = 6 };

/* Epilogue activations of the layer entry points. ZJAI_ACT_LEAKY is LeakyReLU(0.01), which
 * the reference does not have (only relu / relu6, src/nn/fast/layers.rs:174-186); it exists
 * for the benchmark configurations that prescribe it. */
enum { ZJAI_ACT_NONE = 0, ZJAI_ACT_RELU = 1, ZJAI_ACT_LEAKY = 2, ZJAI_ACT_SIGMOID = 3,
       ZJAI_ACT_RELU6 = 4 };

typedef struct zjai_ctx zjai_ctx;
typedef struct zjai_net zjai_net;

/* ---------------------------------------------------------------------------------------- */
/* Library / context                                                                          */
/* ---------------------------------------------------------------------------------------- */

const char *zjai_version(void);

/* Message of the last failing call on this thread ("" if none). */
const char *zjai_last_error_message(void);

/* Context on CUDA device `device`: a stream, a device arena of `arena_bytes` (0 = default
 * 4 GiB) for activations and staging, and the kernels' status word. Stands in for the
 * crate's `Engine` (src/nn/fast/mod.rs:127-169): the GPU is one more engine kind. */
int zjai_ctx_create(int device, size_t arena_bytes, zjai_ctx **out);
int zjai_ctx_destroy(zjai_ctx *ctx);

/* Use the caller's CUDA stream (a cudaStream_t) instead of the context's own; NULL restores
 * the context's stream. */
int zjai_ctx_set_stream(zjai_ctx *ctx, void *cuda_stream);

/* Wait for all work enqueued on the context's stream, then report a kernel status word
 * (ZJAI_DEVICE_TIMEOUT) if a bounded wait gave up. */
int zjai_ctx_sync(zjai_ctx *ctx);

/* Limit of the convolution kernel's pipeline waits (a stage, a halo or an accumulator that
 * does not arrive), in SM clock cycles; 0 restores the default of 4e9 cycles (about 2 s at
 * the boost clock). A wait that runs out makes the kernel record its status word, drain the
 * copies and MMAs it has in flight and end; the next synchronising call on the context then
 * returns ZJAI_DEVICE_TIMEOUT, clears the status word, and the context stays usable. No
 * counterpart in the reference (its CPU path has no device waits): a watchdog bound for
 * callers that prefer to fail fast, and the way the timeout path is exercised in tests. */
int zjai_ctx_set_wait_limit(zjai_ctx *ctx, int64_t cycles);

/* CUDA graphs for repeated device calls of the tiled synthesis (zjai_synthesize_tiles,
 * zjai_synthesize_tiles_q; ZJAI_MEM_DEVICE, no cancel flag): with graphs enabled, the first call
 * with a given set of arguments (networks, pointers, sizes, tile list) runs as usual, the second
 * is captured into a graph and every later one replays it with one launch. The arguments'
 * pointers must then stay valid and keep their meaning (same buffers); destroying a network of
 * the context drops the graphs. Off by default; disabling drops the graphs. */
int zjai_ctx_set_graphs(zjai_ctx *ctx, int enable);

/* Capture a named intermediate map of the networks this context runs (a debugging and
 * per-stage parity facility; the reference has no counterpart, its Python oracle dumps the
 * same names): every later network run that reaches the point `name` writes the map there
 * as planar f32 [n][c][h][w] into `dst` (device memory of the context's GPU, `capacity`
 * floats; a larger map fails the call with ZJAI_LIMIT_EXCEEDED). Points: "ana.act1",
 * "ana.act2", "ana.act3" (the analysis trunk's ResAu outputs, analysis.rs:157-206). A tiled
 * call writes each tile in turn (the last one stays). dst = NULL removes the capture. */
int zjai_ctx_set_probe(zjai_ctx *ctx, const char *name, float *dst, int64_t capacity);

/* Diagnostics: with clamp = 0 the f32 planes of zjai_synthesis_primary / _secondary /
 * zjai_synthesize* are the denormalised x * 128 + 127.5 without the [0, 255] clamp of
 * `denormalize` (synthesis.rs:188-192), so tests can compare the networks' values where the
 * clamp would saturate them (quantized outputs clamp regardless). Default 1. */
int zjai_ctx_set_output_clamp(zjai_ctx *ctx, int clamp);

/* Number of kernels this context has launched since creation (for launch accounting). */
int64_t zjai_ctx_launch_count(const zjai_ctx *ctx);

/* Kernel timing, the GPU counterpart of the crate's `DecodeStats` probe
 * (src/decoder/stats.rs:1-40): while enabled, every convolution launch is bracketed by two
 * CUDA events on its stream. zjai_ctx_profile_read waits for the context's streams and
 * returns the summed device time (ms), the algorithmic FLOPs (live MACs x 2) and the number
 * of convolution launches recorded since the previous read. */
int zjai_ctx_profile(zjai_ctx *ctx, int enable);
/* Per-layer totals of the recorded launches (tab-separated text: layer, launches, ms, GFLOP,
 * TFLOP/s; layers of networks are tagged "<kind><batch>:<parameter prefix>") accumulated by
 * zjai_ctx_profile_read since the previous report; written NUL-terminated into buf. */
int zjai_ctx_profile_report(zjai_ctx *ctx, char *buf, size_t len);
int zjai_ctx_profile_read(zjai_ctx *ctx, double *conv_ms, double *conv_flops,
                          int64_t *conv_launches);
/* zjai_ctx_profile_read that also returns the convolution launches' algorithmic bytes (each
 * launch's input, live weights, output, residual operands and relu6 copy counted once). */
int zjai_ctx_profile_read_bytes(zjai_ctx *ctx, double *conv_ms, double *conv_flops,
                                double *conv_bytes, int64_t *conv_launches);

/* ---------------------------------------------------------------------------------------- */
/* Networks (model load + GPU-resident packed weights)                                        */
/* ---------------------------------------------------------------------------------------- */

/* One named f32 parameter in PyTorch layout, as the crate's checkpoint readers hand them to
 * the loaders (src/model/load.rs:11-85; src/weights/mod.rs:135). */
typedef struct {
  const char *name;  /* e.g. "first_stage.0.0.conv1.weight" */
  int ndim;
  int64_t shape[4];
  const float *data; /* host memory */
} zjai_param;

/* Build network `kind` for operating point `op` from named parameters: validates every
 * name and shape like the crate's loaders (ZJAI_MODEL on mismatch), packs the weights into
 * GPU-resident f16 K-major tiles. Replaces `SynthesisPrimary::load` (synthesis.rs:241-246),
 * `SynthesisSecondary::load` (:971-990), `AnalysisPrimary::load` (analysis.rs:229-239),
 * `AnalysisSecondary::load` (:280-289). */
int zjai_net_create(zjai_ctx *ctx, int kind, int op, const zjai_param *params, int nparams,
                    zjai_net **out);
int zjai_net_destroy(zjai_net *net);

/* Output extent of a synthesis network for a tile of h x w picture samples (the maps are
 * cropped for the tile inside the network; the caller crops the result to h x w). */
int zjai_synth_out_size(int kind, int op, int h, int w, int *out_h, int *out_w);

/* `SynthesisPrimary::forward` (synthesis.rs:253-274): y_hat [160][lh][lw] -> out
 * [1][oh][ow] in [0, 255], (oh, ow) from zjai_synth_out_size. */
int zjai_synthesis_primary(zjai_net *net, const float *y_hat, int lh, int lw, int h, int w,
                           float *out, int mem);

/* `SynthesisSecondary::forward` (synthesis.rs:992-1038): luma latent [160][llh][llw] and
 * chroma latent [96][lh][lw] -> out [2][oh][ow] in [0, 255]. */
int zjai_synthesis_secondary(zjai_net *net, const float *y_hat_luma, int llh, int llw,
                             const float *y_hat_chroma, int lh, int lw, int h, int w,
                             float *out, int mem);

/* `AnalysisPrimary::forward` (analysis.rs:242-269): x [1][h][w] in [0, 255] ->
 * [160][ceil(h/16)][ceil(w/16)]. */
int zjai_analysis_primary(zjai_net *net, const float *x, int h, int w, float *out, int mem);

/* `AnalysisSecondary::forward` (analysis.rs:292-311): x [12][h][w] ->
 * [96][ceil(h/8)][ceil(w/8)]. */
int zjai_analysis_secondary(zjai_net *net, const float *x, int h, int w, float *out, int mem);

/* A convolution stage composed from the crate's layer primitives, for the single-layer and
 * upsampling-stage configurations of the benchmark (the crate has no such network): a conv
 * `conv.weight` [cout * shuffle^2][cin][k][k] (odd k, stride 1, zero pad k / 2, `conv.bias`
 * optional) followed by `act` and, when shuffle > 1, the depth-to-space `pixel_shuffle`
 * (src/nn/fast/layers.rs:233-261); then residual blocks `res.<i>.conv{1,2}.{weight,bias}`
 * ([cout][cout][3][3], i = 0, 1, .. while present), each `ResidualBlock::forward`
 * (src/model/attention.rs:36-43: conv1 -> `res_act` -> conv2, plus the block's input) with
 * `res_act` in place of its ReLU (ZJAI_ACT_LEAKY for LeakyReLU(0.01)). Weights are packed
 * once, GPU resident, like zjai_net_create (destroy with zjai_net_destroy). */
int zjai_stage_create(zjai_ctx *ctx, int shuffle, int act, int res_act, const zjai_param *params,
                      int nparams, zjai_net **out);
/* Runs a stage: x [cin][h][w] -> out [cout][h * shuffle][w * shuffle], planar f32. */
int zjai_stage_forward(zjai_net *net, const float *x, int c, int h, int w, float *out, int mem);

/* `colour::preprocess_rgb` (src/encoder/colour.rs:535-541, with source_planes :390-436 and
 * preprocess :462-495 for 4:4:4 coding): an 8-bit interleaved RGB picture [h][w][3] ->
 * luma [h][w] and chroma [12][ceil(h/2)][ceil(w/2)] (planar f32 in [0, 255]: BT.709 Y, U, V,
 * the chroma tensor the four pixel-unshuffle phases of the edge-replicated Y, then U, then V),
 * bit-exact with the crate's f32 arithmetic. */
int zjai_preprocess_rgb(zjai_ctx *ctx, const uint8_t *rgb, int h, int w, float *luma,
                        float *chroma, int mem);

/* The encoder's analysis of n same-size 8-bit RGB pictures [n][h][w][3] in one call:
 * preprocess_rgb, then `AnalysisPrimary::forward` / `AnalysisSecondary::forward`
 * (analysis.rs:242-311) on all n pictures as one batch, tiled like the crate's encoder above
 * 1,048,576 luma / 262,144 chroma samples per plane (encoder/tiles.rs:51-156, each tile's
 * latent core kept; encoder/mod.rs:1128-1170). lat_y [n][160][ceil(h/16)][ceil(w/16)],
 * lat_uv [n][96][ceil(ceil(h/2)/8)][ceil(ceil(w/2)/8)]. */
int zjai_analyze_rgb(zjai_ctx *ctx, zjai_net *net_y, zjai_net *net_uv, int n,
                     const uint8_t *rgb, int h, int w, float *lat_y, float *lat_uv, int mem);

/* Latent-domain float networks of one component, from a ZJAI_LATENT network (zjai_net_create
 * with the common checkpoint's "hyper_decoder.*" and optional "context.MCM.*" parameters; the
 * operating point is not used). C is the checkpoint's channel count (160 luma, 96 chroma). */

/* `HyperDecoder::forward_f32` (src/model/hyper_decoder.rs:94-113; `forward` :47-90 on i8 values
 * gives the same output): z_hat [C][hz][wz] -> psi [4C][out_h][out_w], the 2x upsampled map
 * cropped to (out_h, out_w) (at most 2 hz x 2 wz). */
int zjai_hyper_decode(zjai_net *net, const float *z_hat, int hz, int wz, int out_h, int out_w,
                      float *psi, int mem);

/* The latent y_hat [C][h][w] from the dequantised residual [C][h][w] and psi
 * [4C][ceil(h/2)][ceil(w/2)] (src/decoder/reconstruct.rs:200-212): `ContextModel::decompress`
 * (src/model/mcm.rs:161-257, four stages over the 2x2 grid) when the network holds a context
 * model, else `upshuffle_psi` (mcm.rs:742-760) plus the residual. */
int zjai_context_decompress(zjai_net *net, const float *residual, int h, int w, const float *psi,
                            float *y_hat, int mem);

/* One region of `reconstruct_latent` (src/decoder/reconstruct.rs:107-230, a picture without
 * independent regions): psi = hyper-decoder(z_hat) at ceil(h/2) x ceil(w/2), then y_hat as
 * zjai_context_decompress, psi kept on the device between the two. psi (output) may be null. */
int zjai_reconstruct_latent(zjai_net *net, const float *z_hat, int hz, int wz,
                            const float *residual, int h, int w, float *psi, float *y_hat,
                            int mem);

/* ---------------------------------------------------------------------------------------- */
/* Weight files (host only): the crate's checkpoint readers                                  */
/* ---------------------------------------------------------------------------------------- */

/* A parsed checkpoint: `Checkpoint::parse` (src/weights/mod.rs:131-183) of a PyTorch `.pth`
 * file (an uncompressed ZIP with a pickled state dict; a data-only pickle interpreter, no code
 * runs) or a packed `ZJM1` file (src/weights/packed.rs:8-21). The bytes are copied. Tensors:
 * those at the top level of the state dict, then the tensors of nested dicts under dotted
 * names (three levels at most, like the crate); integer entries; numeric lists of nested
 * dicts. Dtype codes are ZJM1's: 0 f64, 1 f32, 2 f16, 3 i64, 4 i32, 5 i16, 6 i8, 7 u8,
 * 8 bool. Malformed files fail with ZJAI_MODEL. */
typedef struct zjai_ckpt zjai_ckpt;
int zjai_ckpt_open(const void *data, size_t len, zjai_ckpt **out);
int zjai_ckpt_close(zjai_ckpt *ck);
int zjai_ckpt_count(const zjai_ckpt *ck, int *ntensors, int *nints, int *nlists);
/* Tensor i: name (valid until close), dtype code, rank, dims (up to 8). */
int zjai_ckpt_tensor(const zjai_ckpt *ck, int i, const char **name, int *dtype, int *ndim,
                     int64_t *shape);
int zjai_ckpt_find(const zjai_ckpt *ck, const char *name, int *index);
/* Tensor i as contiguous row-major little-endian bytes (a strided view is gathered). */
int zjai_ckpt_read(const zjai_ckpt *ck, int i, void *dst, size_t capacity);
int zjai_ckpt_int(const zjai_ckpt *ck, int i, const char **name, int64_t *value);
int zjai_ckpt_list(const zjai_ckpt *ck, int i, const char **name, const double **values, int *n);
/* The f32 and f16 tensors of rank <= 4 as f32 parameters (f16 upcast exactly, like
 * `Checkpoint::f32`), ready for zjai_net_create / zjai_stage_create; the array and its data
 * stay valid until close. */
int zjai_ckpt_params(zjai_ckpt *ck, const zjai_param **params, int *n);

/* A `ZJB1` bundle (or `ZJB2`, its f16-weight variant; f16 = 1): files addressed by their path
 * relative to the reference's models/ directory, plus the notice that travels with the weights
 * (src/weights/packed.rs:23-43, `PackedBundle`). File data points into the bundle's copy. */
typedef struct zjai_bundle zjai_bundle;
int zjai_bundle_open(const void *data, size_t len, zjai_bundle **out);
int zjai_bundle_close(zjai_bundle *b);
int zjai_bundle_info(const zjai_bundle *b, int *nfiles, int *f16, const char **notice,
                     size_t *notice_len);
int zjai_bundle_file(const zjai_bundle *b, int i, const char **path, const void **data,
                     size_t *len);

/* LEF, the luma edge filter (src/filters/lef.rs:100-171, the last post-filter of
 * filters::apply): luma [h][w] in [0, 255] -> out [h][w], sharpened where channel `channel` of
 * the luma sigma-index map scale_log [c][sh][sw] (int32, nearest-upsampled to the picture)
 * crosses the thresholds of model `model_id`; bit-exact with the crate's f32 arithmetic.
 * out may equal luma. */
int zjai_lef(zjai_ctx *ctx, const float *luma, int h, int w, const int32_t *scale_log, int c,
             int sh, int sw, int channel, int model_id, int bit_depth, float *out, int mem);

/* The eICCI post-filter (src/filters/icci.rs:175-325) of a 4:4:4 picture, in place on its planes
 * y, u, v [h][w] in [0, 255]: normalised, then per filter tile (tile_size / overlap as signalled;
 * tile_size 0: one tile; tiles in raster order, each reading the cores its predecessors wrote,
 * like the crate) two Haar levels per plane, the luma network `net_y` and / or the chroma network
 * `net_uv` (ZJAI_ICCI networks of the bank the header selects; NULL: that part not filtered;
 * use_u / use_v: the chroma planes corrected), inverse transform, core written back; finally
 * clamped and scaled back. 4:2:0 / 4:2:2 sources are up-sampled to 4:4:4 by the caller (the
 * crate's `to_444_`); eICCI is not signalled for 4:2:0. */
int zjai_icci_filter(zjai_ctx *ctx, zjai_net *net_y, zjai_net *net_uv, int use_u, int use_v,
                     float *y, float *u, float *v, int h, int w, int tile_size, int overlap,
                     int mem);

/* One coded EFE linear filter set (src/header.rs:623-639 `EfeLinearSet`): per chroma plane p
 * (0 = U, 1 = V) the split candidate cand[p] (0..7, -1: plane not filtered), the filter side
 * filter_len[p] (1..4) and the weight codes of the split's regions in order (1, 2, 2, 3, 3, 4, 6
 * and 6 regions for candidates 0..7): chroma_codes[p] holds regions x P x fL x fL codes (P = 1
 * for a picture coded at the source's chroma resolution, else the 4 sub-sampling phases),
 * luma_codes[p] regions x fL x fL. min_symbol is added to every code. Host memory. */
typedef struct {
  int cand[2];
  int filter_len[2];
  int min_symbol;
  const uint32_t *chroma_codes[2];
  const uint32_t *luma_codes[2];
} zjai_efe_linear_set;

/* EFE linear (src/filters/efe_linear.rs:403-460, `filter_plane` :308-359): the luma-aided
 * linear filter of the chroma planes with one coded set, bit-exact with the crate's f32
 * arithmetic. y [h][w], u / v [ch][cw] in [0, 255] of a source subsampled s_ver x s_hor
 * (1 or 2) and coded c_ver x c_hor; mean_u / mean_v the B1 codes (1/100 units). Writes the
 * filtered planes to out_u / out_v (which may equal u / v). The crate runs it once per coded
 * set: the first set (`upsample_set`) gives the alternative picture of the EFE non-linear
 * filter's on/off switch, the second the filtered picture. Formats the reference does not
 * decode return ZJAI_UNSUPPORTED, like a plane left unfiltered in a picture coded at the
 * source's chroma resolution; mis-sized planes ZJAI_INVALID_ARGUMENT; sets out of range
 * ZJAI_INVALID_DATA. */
int zjai_efe_linear(zjai_ctx *ctx, const float *y, int h, int w, const float *u, const float *v,
                    int ch, int cw, int s_ver, int s_hor, int c_ver, int c_hor, int mean_u,
                    int mean_v, const zjai_efe_linear_set *set, float *out_u, float *out_v,
                    int mem);

/* EFE non-linear parameters (src/header.rs:655-682): the per-tile luma network
 * (tile_width x tile_height chroma samples, ntiles entries of luma_min / luma_max in 1/100
 * units, 8 weight codes per tile in codes[p], ncodes[p] of them; codes[p] NULL: plane p not
 * filtered) and the on/off switch (mask[p]: mask_h x mask_w values in 0..2 for blocks of
 * mask_bs samples, NULL: no mask). Host memory. */
typedef struct {
  int min_symbol;
  int tile_width, tile_height, ntiles;
  const uint16_t *luma_min, *luma_max;
  const uint32_t *codes[2];
  int ncodes[2];
  int mask_bs, mask_h, mask_w;
  const uint8_t *mask[2];
} zjai_efe_nonlinear_params;

/* EFE non-linear (src/filters/efe_nonlinear.rs:190-237), in place on u / v [ch][cw] (ch =
 * ceil(h / s_ver), cw = ceil(w / s_hor)): the tile network on the planes whose codes are given,
 * then, when the U mask is given (the reference looks at it alone), the on/off switch of each
 * masked plane towards alt_u / alt_v (the EFE linear filter's alternative picture, required
 * then). Bit-exact with the crate's f32 arithmetic; status codes as zjai_efe_linear. */
int zjai_efe_nonlinear(zjai_ctx *ctx, const float *y, int h, int w, float *u, float *v, int ch,
                       int cw, int s_ver, int s_hor, int c_ver, int c_hor,
                       const zjai_efe_nonlinear_params *prm, const float *alt_u,
                       const float *alt_v, int mem);

/* One synthesis tile (src/tools/tiles.rs:26-32 `SynthesisTile`). */
typedef struct {
  int img_x, img_y, img_w, img_h;
  int lat_x, lat_y, lat_w, lat_h;
  int core_x, core_y, core_w, core_h;
  int off_x, off_y;
} zjai_tile;

/* `synthesis_tiles` (src/tools/tiles.rs:39-119) without independent regions. tile_size <= 0
 * means one tile. Returns ZJAI_INVALID_DATA for malformed geometry; *count receives the
 * number of tiles (at most max_tiles are written). */
int zjai_synthesis_tiles(int height, int width, int latent_h, int latent_w, int tile_size,
                         int overlap, zjai_tile *tiles, int max_tiles, int *count);

/* `synthesize_with` (src/decoder/reconstruct.rs:274-331, 379-464): whole-picture synthesis,
 * tile by tile, written straight into the output planes: rec_y [out_h][out_w] cropped to
 * the displayed size, rec_u / rec_v [ceil(out_h/sv)][ceil(out_w/sh)] subsampled. Luma and
 * chroma run on two streams. `cancel` (may be NULL) is polled between tiles; when it reads
 * non-zero the call returns ZJAI_CANCELLED (enough::Stop, reconstruct.rs:391,432). */
int zjai_synthesize(zjai_ctx *ctx, zjai_net *net_y, zjai_net *net_uv, const float *y_hat_y,
                    const float *y_hat_uv, int lh, int lw, int height, int width, int out_h,
                    int out_w, int tile_size, int overlap, int sv, int sh, float *rec_y,
                    float *rec_u, float *rec_v, int mem, const volatile int *cancel);

/* The per-tile half of zjai_synthesize (the `par_map` over tiles of reconstruct.rs:390 and
 * :432): synthesizes only the listed tiles and writes only their cores. Tiles of one shape
 * run as one batch. This is the unit a multi-GPU scheduler shards (e.g. tile i on GPU
 * i mod N); planes not covered by the listed cores are left untouched (device) or zero
 * (host). */
int zjai_synthesize_tiles(zjai_ctx *ctx, zjai_net *net_y, zjai_net *net_uv,
                          const float *y_hat_y, const float *y_hat_uv, int lh, int lw,
                          const zjai_tile *tiles, int ntiles, int out_h, int out_w, int sv,
                          int sh, float *rec_y, float *rec_u, float *rec_v, int mem,
                          const volatile int *cancel);

/* Fused output stage (the `emit_output` step the reference's GPU backend fuses,
 * gpu/src/kernels.rs:715,910): zjai_synthesize_tiles / zjai_synthesize with the planes
 * quantized by the final layers' epilogue, exactly as `quantize_plane_par` (output.rs:330-342)
 * quantizes the f32 planes: uint8 samples for bit_depth 8, else uint16 (bit_depth 9..16). No
 * f32 planes are written. */
int zjai_synthesize_tiles_q(zjai_ctx *ctx, zjai_net *net_y, zjai_net *net_uv,
                            const float *y_hat_y, const float *y_hat_uv, int lh, int lw,
                            const zjai_tile *tiles, int ntiles, int out_h, int out_w, int sv,
                            int sh, int bit_depth, void *rec_y, void *rec_u, void *rec_v,
                            int mem, const volatile int *cancel);
int zjai_synthesize_q(zjai_ctx *ctx, zjai_net *net_y, zjai_net *net_uv, const float *y_hat_y,
                      const float *y_hat_uv, int lh, int lw, int height, int width, int out_h,
                      int out_w, int tile_size, int overlap, int sv, int sh, int bit_depth,
                      void *rec_y, void *rec_u, void *rec_v, int mem,
                      const volatile int *cancel);

/* Multi-GPU final gather without a collective (the crate has none: its tiles are gathered in
 * one address space, reconstruct.rs:379-464). The process owning the picture exports the
 * allocation holding its device planes (`ptr` may point inside it): a 64-byte CUDA IPC handle
 * and the offset of `ptr` in the allocation. Another process on the same box maps it with
 * zjai_ipc_import and passes the mapped pointer as the output planes of zjai_synthesize_tiles_q
 * (mem = ZJAI_MEM_DEVICE): the final layers then store that rank's cores straight into the
 * owner's planes over NVLink. The caller orders the owner's reads after the writers' work
 * (e.g. a stream-ordered all-reduce after the synthesis); zjai_ipc_close unmaps. */
int zjai_ipc_export(zjai_ctx *ctx, const void *ptr, void *handle, uint64_t *offset);
int zjai_ipc_import(zjai_ctx *ctx, const void *handle, uint64_t offset, void **ptr);
int zjai_ipc_close(zjai_ctx *ctx, void *ptr);

/* Synthesis straight to RGB, the decoder's `decode` output for a 4:2:0 stream
 * (reconstruct.rs:274-331, then output.rs:124-262 `to_source_format_par` bicubic 4:2:0 ->
 * 4:4:4, `to_rgb_planes_owned_par` BT.709, `quantize_par` :407-438): the f32 planes stay in
 * device memory and the output stage reads them there, as the crate's GPU backend does in
 * `emit_output` (gpu/src/kernels.rs:910); rgb [height][width][3], uint8 for bit_depth 8, uint16
 * for 10. Bit-exact with zjai_synthesize (sv = sh = 2) followed by zjai_yuv_to_rgb. */
int zjai_synthesize_rgb(zjai_ctx *ctx, zjai_net *net_y, zjai_net *net_uv, const float *y_hat_y,
                        const float *y_hat_uv, int lh, int lw, int height, int width,
                        int tile_size, int overlap, int bit_depth, void *rgb, int mem,
                        const volatile int *cancel);

/* A batch of n independent pictures of one size synthesised in one call (the crate decodes
 * them one `synthesize_with` call at a time, reconstruct.rs:274-331; here every tile of every
 * picture runs in the same shape batches): latents y_hat_y [n][160][lh][lw], y_hat_uv
 * [n][96][lh][lw]; planes rec_y [n][out_h][out_w], rec_u / rec_v [n][ceil(out_h/sv)]
 * [ceil(out_w/sh)], f32 for bit_depth 0, else the quantized samples of zjai_synthesize_q. */
int zjai_synthesize_batch(zjai_ctx *ctx, zjai_net *net_y, zjai_net *net_uv, int n,
                          const float *y_hat_y, const float *y_hat_uv, int lh, int lw, int height,
                          int width, int out_h, int out_w, int tile_size, int overlap, int sv,
                          int sh, int bit_depth, void *rec_y, void *rec_u, void *rec_v, int mem,
                          const volatile int *cancel);

/* ---------------------------------------------------------------------------------------- */
/* Output stage (src/decoder/output.rs)                                                       */
/* ---------------------------------------------------------------------------------------- */

/* `quantize_plane_par` (output.rs:330-342): clip to [0,255], scale to 2^depth-1, round half
 * to even; 8-bit output as uint8 when bit_depth == 8 (out_u8), else uint16 (out_u16). */
int zjai_quantize_plane(zjai_ctx *ctx, const float *x, int64_t n, int bit_depth, void *out,
                        int mem);

/* `to_source_format_par` bicubic 4:2:0 -> 4:4:4 (output.rs:103-151, align_corners) then
 * `to_rgb_planes_owned_par` BT.709 (:218-262) and `quantize_par` (:407-438): planes
 * y [h][w], u / v [ch][cw] -> interleaved RGB [h][w][3] (uint8 for 8-bit, else uint16). */
int zjai_yuv_to_rgb(zjai_ctx *ctx, const float *y, const float *u, const float *v, int h,
                    int w, int ch, int cw, int bit_depth, void *rgb, int mem);

/* ---------------------------------------------------------------------------------------- */
/* nn layer interface (src/nn/fast/layers.rs, src/nn/fast/math.rs)                           */
/* ---------------------------------------------------------------------------------------- */

/* `ConvLayer::{new,with_extra_pad,forward}` (layers.rs:30-123) on planar f32 tensors:
 * weight [oc][c/groups][kh][kw], bias [oc] or NULL, extra = [top, left, bottom, right] zero
 * border or NULL; `act` is applied after the bias. */
int zjai_conv2d(zjai_ctx *ctx, const float *x, int c, int h, int w, const float *weight,
                const float *bias, int oc, int kh, int kw, int stride, int pad_h, int pad_w,
                int groups, const int *extra, int act, float *out, int mem);

/* `ConvTransposeLayer::forward` (layers.rs:135-171): weight [c][oc][k][k], stride 2. */
int zjai_conv_transpose2d(zjai_ctx *ctx, const float *x, int c, int h, int w,
                          const float *weight, const float *bias, int oc, int k, int pad,
                          int out_pad, float *out, int mem);

/* The RDLR VJPs of those two layers: input gradients, which the encoder's latent refinement
 * chains through the synthesis network. `ConvLayer::backward` (layers.rs:72-90, over
 * `conv2d_backward`, reference.rs:241-292): dout [oc][oh][ow], the output extent of the layer
 * above on an input [c][h][w] with the zero border `extra` (or NULL) -> din [c][h][w]; strides 1
 * and 2 (stride 2: dense square kernels without extra border). `ConvTransposeLayer::backward`
 * (layers.rs:156-160, `conv_transpose2d_backward`, reference.rs:294-336) of a stride-2
 * transposed conv with weight [c][oc][k][k] on an input [c][h][w]. Both run as convolutions
 * on the tensor cores (f16 operands, d_out scaled by a power of two first, f32 accumulation):
 * within about 1e-3 relative L2 of the crate's f32 loops, not bit-exact. */
int zjai_conv2d_backward(zjai_ctx *ctx, const float *dout, int oc, int oh, int ow,
                         const float *weight, int c, int kh, int kw, int stride, int pad_h,
                         int pad_w, int groups, const int *extra, int h, int w, float *din,
                         int mem);
int zjai_conv_transpose2d_backward(zjai_ctx *ctx, const float *dout, int oc, int oh, int ow,
                                   const float *weight, int c, int k, int pad, int h, int w,
                                   float *din, int mem);
/* `ResidualBlock::backward` (src/model/attention.rs:58-75), the first network-level VJP of the
 * RDLR HOP chain: d_out [c][h][w] of `conv3x3 -> ReLU -> conv3x3 + x` and its tape conv1_out
 * [c][h][w] (conv1's output before the ReLU) -> din = d_out + conv1^T(relu'(conv1_out) .
 * conv2^T d_out); w1 / w2 the convs' weights [c][c][3][3]. Tolerance as zjai_conv2d_backward. */
int zjai_residual_block_backward(zjai_ctx *ctx, const float *dout, const float *conv1_out,
                                 int c, int h, int w, const float *w1, const float *w2,
                                 float *din, int mem);

/* `Cab::backward` (src/model/attention.rs:182-223) of the CAB block x + trunk(x) .
 * sigmoid(mask(x)) on c channels at h x w (even): the tape of `Cab::forward_tape` — trunk_pre
 * (the trunk's output before the product), sig (the sigmoid of the mask), rb_c1 (the trunk
 * residual blocks' conv1 outputs) [c][h][w], and mask_c1 (the mask residual blocks' conv1
 * outputs) [c][h/2][w/2] — and the layers' weights ([c][c][3][3] each: the residual blocks'
 * conv1 and conv2, the stride-2 subscale conv, the upscale transposed conv [c][c][3][3]). All
 * arrays in the memory `mem` names. Tolerance as zjai_conv2d_backward. */
typedef struct {
  const float *trunk_pre, *sig;
  const float *rb_c1[2];
  const float *mask_c1[2];
} zjai_cab_tape;
typedef struct {
  const float *trunk[2][2];  /* residual_trunk.{0,1}.{conv1,conv2} */
  const float *subscale;
  const float *mask2[2];     /* residual_mask2.0.{conv1,conv2} */
  const float *mask3[2];     /* residual_mask3.0.{conv1,conv2} */
  const float *upscale;
} zjai_cab_weights;
int zjai_cab_backward(zjai_ctx *ctx, const float *dout, int c, int h, int w,
                      const zjai_cab_tape *tape, const zjai_cab_weights *wts, float *din,
                      int mem);

/* The transformer block's per-pixel VJPs. `elu_gate_backward` (src/nn/fast/math.rs:838-858)
 * of y = elu(a) . b over n elements: d_a = elu'(a) . b . d, d_b = elu(a) . d (the GPU's expf in
 * place of the crate's exp: within a few ulp). `layer_norm_channels_backward` (math.rs:860-913):
 * d, x [c][h][w] (x the forward's input), weight [c] -> dx, the statistics recomputed with f64
 * sums as the crate does. */
int zjai_elu_gate_backward(zjai_ctx *ctx, const float *d, const float *a, const float *b,
                           int64_t n, float *d_a, float *d_b, int mem);
int zjai_layer_norm_backward(zjai_ctx *ctx, const float *d, const float *x, int c, int h, int w,
                             const float *weight, float *dx, int mem);
/* `channel_attention_backward` (src/nn/fast/math.rs:668-836): qkv [3 dim][h][w] (the forward's
 * input), temperature [heads], attn [dim][dim / heads] (the forward's softmax weights, its
 * tape), d_out [dim][h][w] -> dqkv [3 dim][h][w]: the softmax VJP of d_out . v^T, dq, dk through
 * the L2-norm backward, dv = attn^T . d_out; f64 sums, within about 1e-5 relative L2 of the
 * crate's dot8 sums. */
int zjai_channel_attention_backward(zjai_ctx *ctx, const float *qkv, int c3, int h, int w,
                                    int heads, const float *temperature, const float *attn,
                                    const float *dout, float *dqkv, int mem);

/* `TransformerBlock::backward` (src/model/attention.rs:435-480) from the tape of
 * `forward_tape`: x_in, x_mid [dim][h][w] (the block's input and its input after the attention
 * half), qkv [3 dim][h][w], attn [dim][dim / heads], gate [2 hidden][h][w] (the depthwise conv's
 * output, the ELU gate's two halves); weights: the two layer norms' weights [dim], prep_conv1
 * [3 dim][dim], prep_conv2 [3 dim][1][3][3], temperature [heads], attn_out [dim][dim], ffn_in
 * [2 hidden][dim], ffn_dw [2 hidden][1][3][3], ffn_out [dim][hidden]; 3 dim and 2 hidden
 * multiples of 8. d_out [dim][h][w] -> din. Tolerance as zjai_conv2d_backward. */
typedef struct {
  const float *x_in, *qkv, *attn, *x_mid, *gate;
} zjai_tb_tape;
typedef struct {
  const float *prep_norm, *prep_conv1, *prep_conv2, *temperature, *attn_out;
  const float *ffn_norm, *ffn_in, *ffn_dw, *ffn_out;
} zjai_tb_weights;
int zjai_transformer_block_backward(zjai_ctx *ctx, const float *dout, int dim, int hidden,
                                    int heads, int h, int w, const zjai_tb_tape *tape,
                                    const zjai_tb_weights *wts, float *din, int mem);

/* `math::layer_norm_channels` (math.rs:423-448), out of place. */
int zjai_layer_norm(zjai_ctx *ctx, const float *x, int c, int h, int w, const float *weight,
                    const float *bias, float *out, int mem);

/* `math::channel_attention` (math.rs:512-603): qkv [3*dim][h][w] -> [dim][h][w]. */
int zjai_channel_attention(zjai_ctx *ctx, const float *qkv, int c3, int h, int w, int heads,
                           const float *temperature, float *out, int mem);

/* Depthwise 3x3, stride 1, pad 1, no bias (`PackedDepthwise`, depthwise.rs:118-209). */
int zjai_depthwise3x3(zjai_ctx *ctx, const float *x, int c, int h, int w, const float *weight,
                      float *out, int mem);

/* The FFN's depthwise 3x3 followed by its ELU gate (TransformerBlock::forward,
 * attention.rs:347-355: `ffn_dw.forward` then `math::elu_gate(x1, x2)`, math.rs:376), fused:
 * x [c][h][w] (c a multiple of 16) -> out [c/2][h][w], out[k] = elu(dw[k]) * dw[k + c/2]. */
int zjai_depthwise3x3_elu_gate(zjai_ctx *ctx, const float *x, int c, int h, int w,
                               const float *weight, float *out, int mem);

/* The feed-forward half of `TransformerBlock::forward` (attention.rs:346-371) on one picture:
 * out = x + W_out . gate(dw3x3(W_in . layer_norm(x))), gate(t) = elu(t[:hidden]) * t[hidden:]
 * (math.rs:376). x / out [c][h][w], norm weight / bias [c], w_in [2 hidden][c], w_dw
 * [2 hidden][9], w_out [c][hidden]; c 64 or 128, hidden a multiple of 64. Runs the layer norm
 * and the fused tcgen05 FFN kernel (the 2 hidden-channel intermediates stay on chip). */
int zjai_transformer_ffn(zjai_ctx *ctx, const float *x, int c, int h, int w, int hidden,
                         const float *norm_weight, const float *norm_bias, const float *w_in,
                         const float *w_dw, const float *w_out, float *out, int mem);

/* Layer-level timing harness, the GPU counterpart of the crate's conv microbenchmark
 * (benches/conv_kernels.rs:165-187: `PackedConv::new` + `forward` on layer shapes): packs a
 * random conv (or, with `transposed`, a stride-2 transposed conv: k 3 -> p1 op1, k 4 -> p1) of
 * the given geometry, runs it `reps` times on n pseudo-random NHWC f16 maps of h x w in the
 * context arena (`residual` 0: ReLU epilogue; 1: ReLU plus a residual add; 2: the planar f32
 * output of a network's final layer, denormalised) and returns the mean device time per
 * launch in *ms and the algorithmic FLOPs per launch in *flops (may be NULL). */
int zjai_conv_bench(zjai_ctx *ctx, int n, int h, int w, int cin, int cout, int k, int stride,
                    int groups, int transposed, int residual, int reps, double *ms,
                    double *flops);

/* Kernels of the HOP transformer blocks timed alone (the same harness for the steps of
 * attention.rs:328-372): `kind` is ZJAI_KB_DW (depthwise 3x3 over c channels),
 * ZJAI_KB_DW_GATE (depthwise 3x3 over c channels fused with the FFN's ELU gate, c/2 out),
 * ZJAI_KB_LN (layer norm over c channels), ZJAI_KB_ATTN (channel attention on a 3c-channel
 * qkv map, 4 heads) or ZJAI_KB_FFN (the fused FFN kernel, x += W_out . gate(dw3x3(W_in . ln))
 * with dim c (64 or 128) and hidden 4c, random weights). Runs `reps` times on n pseudo-random
 * NHWC f16 maps of h x w in the context arena; returns the mean device time per run in *ms
 * and the algorithmic bytes per run (each input element read once, each output element
 * written once) in *bytes. */
enum { ZJAI_KB_DW = 0, ZJAI_KB_DW_GATE = 1, ZJAI_KB_LN = 2, ZJAI_KB_ATTN = 3, ZJAI_KB_FFN = 4 };
int zjai_kernel_bench(zjai_ctx *ctx, int kind, int n, int h, int w, int c, int reps, double *ms,
                      double *bytes);

/* Channel attention that allocates nothing. It has no counterpart in the reference: it is
 * zjai_channel_attention for callers that must not allocate device memory during a call
 * (code running under an external allocator or a strict memory budget, callers that only
 * hand in pre-allocated buffers). qkv [3*dim][h][w], temperature [heads] and out [dim][h][w]
 * are caller-owned DEVICE buffers of the context's GPU (planar f32); host memory (pageable or
 * pinned) is rejected with ZJAI_INVALID_ARGUMENT before anything runs. The call's scratch is
 * one fixed-size device array in the library (130 KiB, held by every GPU that loads the
 * library), so dim <= 256 and dim / heads <= 64, and larger sizes return ZJAI_LIMIT_EXCEEDED.
 * The first call on a device looks the array's address up (cudaGetSymbolAddress); make that
 * first call before any stream capture. All calls share the array: calls that overlap on the
 * GPU (other streams or contexts) race. The Gram reduction runs in a fixed order (no atomics),
 * so repeated calls give identical results. The work is enqueued on the context's stream and
 * the call returns without waiting. */
int zjai_channel_attention_static(zjai_ctx *ctx, const float *qkv, int c3, int h, int w,
                                  int heads, const float *temperature, float *out);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif
#endif /* ZJAI_H */
