/*
 * CPU oracle for the JPEG AI synthesis / analysis path (TEST INFRASTRUCTURE ONLY).
 *
 * A plain-C restatement of the reference crate's f32 CPU path (imazen/zenjpegai, Rust):
 * the numeric contract of `src/nn/mod.rs:1-45` (bias-initialised FMA accumulation in
 * (ic, ky, kx) order over a zero-padded input), the plain loops of `src/nn/reference.rs`,
 * the pointwise / reduction maths of `src/nn/fast/math.rs` (Cephes exp, f64 sums, `dot8`),
 * the topologies of `src/model/{synthesis,attention,analysis}.rs`, the tiling of
 * `src/tools/tiles.rs`, the tile assembly of `src/decoder/reconstruct.rs` and the output
 * stage of `src/decoder/output.rs`.
 *
 * Only the test suite, `__graft_entry__.smoke()` and the `cpu_baseline` leg of `bench.py`
 * may load this library, and only as the checker / the timed CPU baseline. The product
 * (`zenjpegai_b200`) never links or calls it.
 *
 * Parity pin: the layer functions are checked against the reference's own golden vectors
 * (the `.bin` files of `tests/vectors/nn/`, torch-computed, converted into `tests/golden/`), with the
 * reference's tolerance (max |d| / max(|y|, 1) < 2e-6) and bit-exactness for the pure
 * permutations and resamplers. Whole-network parity to upstream PyTorch is not pinnable here
 * (no checkpoints, no reference dumps); the topology follows the cited Rust source.
 */
#ifndef ZJAI_ORACLE_H
#define ZJAI_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- threading of the oracle's loops (OpenMP); 1 = serial ---------------------------- */
void zo_set_threads(int n);
int zo_get_threads(void);
/* 1: zo_conv2d / zo_conv_transpose2d run the restatement of the crate's nn::fast algorithm
 * (fast.c: blocked layout, register tiles, per-row threads), which gives the same bits; the
 * timed CPU baseline. 0 (default): the nn::reference loops. */
void zo_set_fast(int on);
/* 0: `denormalize` without its [0, 255] clamp (diagnostics); 1 (default): as the crate. */
void zo_set_output_clamp(int on);
int zo_get_fast(void);
/* nn::fast restatements (fast.c); return 1 when the geometry is not handled there */
int zf_conv2d(const float *x, int c, int h, int w, const float *weight, const float *bias,
              int oc, int kh, int kw, int stride, int pad_h, int pad_w, int groups,
              const int extra[4], float *out);
int zf_conv_transpose2d(const float *x, int c, int h, int w, const float *weight,
                        const float *bias, int oc, int k, int stride, int pad, int out_pad,
                        float *out);

/* ---- layer functions (planar [c][h][w] f32 tensors, caller-owned buffers) -------------- */

/* Output size of a convolution over an input of h x w with extra padding [t, l, b, r]. */
void zo_conv2d_out_size(int h, int w, int kh, int kw, int stride, int pad_h, int pad_w,
                        const int extra[4], int *oh, int *ow);

/* `nn::reference::conv2d` (reference.rs:92-133) with `ConvLayer::with_extra_pad`'s zero
 * border (layers.rs:100-115). weight [oc][c/groups][kh][kw], bias may be NULL. */
int zo_conv2d(const float *x, int c, int h, int w, const float *weight, const float *bias,
              int oc, int kh, int kw, int stride, int pad_h, int pad_w, int groups,
              const int extra[4], float *out);

/* `nn::reference::conv_transpose2d` (reference.rs:155-236). weight [c][oc][k][k]. */
void zo_conv_transpose2d_out_size(int h, int w, int k, int stride, int pad, int out_pad,
                                  int *oh, int *ow);
int zo_conv_transpose2d(const float *x, int c, int h, int w, const float *weight,
                        const float *bias, int oc, int k, int stride, int pad, int out_pad,
                        float *out);

/* `pixel_shuffle` (reference.rs:353-375): [c*r*r, h, w] -> [c, h*r, w*r]. */
int zo_pixel_shuffle(const float *x, int c, int h, int w, int r, float *out);

/* Elementwise ops (layers.rs:174-229, math.rs:371-397). In place on n values. */
void zo_relu(float *x, int64_t n);
void zo_relu6(float *x, int64_t n);
void zo_add(float *dst, const float *src, int64_t n);
void zo_gate(float *x, const float *mask, int64_t n);
void zo_mul(float *a, const float *b, int64_t n);
void zo_sigmoid(float *x, int64_t n);
void zo_elu_gate(float *a, const float *b, int64_t n);
float zo_exp(float x);
void zo_denormalize(float *x, int64_t n);

/* `math::layer_norm_channels` (math.rs:423-448), in place on [c][h][w]. */
int zo_layer_norm_channels(float *x, int c, int h, int w, const float *weight,
                           const float *bias);

/* `math::channel_attention` (math.rs:512-603): qkv [3*dim][h][w] -> out [dim][h][w]. */
int zo_channel_attention(const float *qkv, int c3, int h, int w, int heads,
                         const float *temperature, float *out);

/* `dot8` (math.rs:452-465). */
double zo_dot8(const float *a, const float *b, int64_t n);

/* ---- named parameters (a checkpoint stand-in) ------------------------------------------ */
typedef struct {
    const char *name;
    int ndim;
    int shape[4];
    const float *data;
} zo_param;

typedef struct {
    const zo_param *params;
    int n;
} zo_ckpt;

enum { ZO_SOP = 0, ZO_BOP = 1, ZO_HOP = 2 };

/* Per-layer dump hook: called with each named intermediate map (planar). NULL = off. */
typedef void (*zo_dump_fn)(const char *name, const float *data, int c, int h, int w);
void zo_set_dump(zo_dump_fn fn);

/* Output size of a synthesis network for a tile of h x w picture samples. */
void zo_synth_out_size(int op, int secondary, int h, int w, int *oh, int *ow);

/* `SynthesisPrimary::forward` (synthesis.rs:262-274 -> LightPrimary / HopPrimary):
 * y_hat [160][lh][lw] -> out [1][oh][ow] in [0, 255] (oh, ow from zo_synth_out_size). */
int zo_synthesis_primary(const zo_ckpt *ck, int op, const float *y_hat, int lh, int lw,
                         int h, int w, float *out);

/* `SynthesisSecondary::forward_with` (synthesis.rs:1004-1038): luma latent [160][llh][llw]
 * and chroma latent [96][lh][lw] -> out [2][oh][ow] in [0, 255]. */
int zo_synthesis_secondary(const zo_ckpt *ck, int op, const float *y_hat_luma, int llh,
                           int llw, const float *y_hat_chroma, int lh, int lw, int h, int w,
                           float *out);

/* `AnalysisPrimary::forward` (analysis.rs:242-269): [1][h][w] in [0,255] ->
 * [160][ceil(h/16)][ceil(w/16)]. */
int zo_analysis_primary(const zo_ckpt *ck, int op, const float *x, int h, int w, float *out);
/* One analysis stage (1..4) of an h x w picture from its input: picture -> act1 -> act2 ->
 * act3 -> latent (Trunk::forward, analysis.rs:157-206, and the heads :242-311); the stage's
 * input is [1 or 12][h][w] for stage 1, else [128][ceil(h / d)][ceil(w / d)], d = 2, 4, 8. */
int zo_analysis_stage(const zo_ckpt *ck, int op, int secondary, int stage, const float *x, int c,
                      int h, int w, float *out);

/* `AnalysisSecondary::forward` (analysis.rs:292-311): [12][h][w] -> [96][ceil(h/8)][ceil(w/8)]. */
int zo_analysis_secondary(const zo_ckpt *ck, int op, const float *x, int h, int w, float *out);

/* ---- tiling (tiles.rs:39-119, without independent regions) ------------------------------ */
typedef struct {
    int img_x, img_y, img_w, img_h;
    int lat_x, lat_y, lat_w, lat_h;
    int core_x, core_y, core_w, core_h;
    int off_x, off_y;
} zo_tile;

/* tile_size <= 0: one tile covering the picture. Returns the tile count, or -1 on malformed
 * geometry. Writes at most max_tiles entries. */
int zo_synthesis_tiles(int height, int width, int latent_h, int latent_w, int tile_size,
                       int overlap, zo_tile *tiles, int max_tiles);

/* `synthesize_with` (reconstruct.rs:274-331, 379-464): whole-picture synthesis into
 * rec_y [out_h][out_w], rec_u / rec_v [ceil(out_h/sv)][ceil(out_w/sh)]. */
int zo_synthesize(const zo_ckpt *ck_y, const zo_ckpt *ck_uv, int op, const float *y_hat_y,
                  const float *y_hat_uv, int lh, int lw, int height, int width, int out_h,
                  int out_w, int tile_size, int overlap, int sv, int sh, float *rec_y,
                  float *rec_u, float *rec_v);

/* ---- output stage (output.rs) ---------------------------------------------------------- */
void zo_quantize_plane(const float *x, int64_t n, int bit_depth, uint16_t *out);
int zo_resize_bicubic(const float *src, int c, int h, int w, int out_h, int out_w,
                      float *out);
/* BT.709 YCbCr -> RGB in place (y->r, u->g, v->b), output.rs:218-262 */
void zo_to_rgb_planes(float *y, float *u, float *v, int64_t n);
/* interleaved RGB quantisation, output.rs:407-438 */
void zo_quantize_rgb(const float *r, const float *g, const float *b, int64_t n, int bit_depth,
                     uint16_t *out);

/* ---- encoder pre-processing (colour.rs) and analysis helpers ---------------------------- */
void zo_normalize(const float *x, int64_t n, float *out);
int zo_pad_amount(int len, int divider);

/* `preprocess_rgb` (colour.rs:535-541 -> source_planes colour.rs:390-436 and preprocess
 * colour.rs:462-495, 4:4:4 coded) of an 8-bit interleaved RGB picture [h][w][3]: luma [h][w]
 * in [0, 255], chroma [12][ph / 2][pw / 2] (ph, pw = h, w rounded up to even): the four
 * pixel-unshuffle phases of the replicate-padded luma, then of U, then of V. */
void zo_preprocess_rgb(const uint8_t *rgb, int h, int w, float *luma, float *chroma);

/* One analysis tile (encoder/tiles.rs:33-49 `AnalysisTile`, without the hyper-latent grid):
 * the plane area the analysis runs on, the latent area it produces, the kept core of that
 * latent (whole-latent coordinates) and the core's offset inside the tile's own latent. */
typedef struct {
    int img_x, img_y, img_w, img_h;
    int lat_x, lat_y, lat_w, lat_h;
    int core_x, core_y, core_w, core_h;
    int off_x, off_y;
} zo_atile;

/* `analysis_tiles` (encoder/tiles.rs:51-156, no independent regions) of component ccs (0 luma,
 * 1 chroma) for a plane of h x w samples with latent lh x lw. Returns the tile count (-1:
 * malformed geometry); writes at most max_tiles. */
int zo_analysis_tiles(int ccs, int h, int w, int lh, int lw, zo_atile *tiles, int max_tiles);

/* HyperDecoder::forward_f32 (hyper_decoder.rs:94-113): z [c][hz][wz] -> psi
 * [4c][out_h][out_w]. -1 when (out_h, out_w) exceeds the upsampled map. */
int zo_hyper_decode(const zo_ckpt *ck, const float *z, int c, int hz, int wz, int out_h,
                    int out_w, float *psi);
/* reconstruct.rs:200-212: ContextModel::decompress (mcm.rs:161-257) when the checkpoint holds
 * a context model, else upshuffle_psi (mcm.rs:742-760) + residual. residual, y [c][h][w],
 * psi [4c][ceil(h/2)][ceil(w/2)]. */
int zo_context_decompress(const zo_ckpt *ck, int c, const float *residual, int h, int w,
                          const float *psi, float *y);
/* The encoder's tiled analysis transform of component ccs: plane x [1 or 12][h][w] -> latent
 * [160 or 96][ceil(h / d)][ceil(w / d)] (d = 16 or 8), each tile analysed on its own and its
 * latent core kept (encoder/mod.rs:1128-1170). */
int zo_analyze_tiled(const zo_ckpt *ck, int op, int ccs, const float *x, int h, int w,
                     float *out);

/* LEF (src/filters/lef.rs:100-171): luma [h][w] -> out, steered by channel `channel` of the
 * luma sigma-index map scale_log [c][sh][sw]; -1 on the inputs the crate rejects. */
int zo_lef(const float *luma, int h, int w, const int32_t *scale_log, int c, int sh, int sw,
           int channel, int model_id, int bit_depth, float *out);
/* torch nearest-neighbour source index (lef.rs:67-74) */
int zo_nearest_index(int i, int src, int dst);

/* eICCI (src/filters/icci.rs:175-325, network src/model/icci.rs) of a 4:4:4 picture in place:
 * planes y, u, v [h][w] in [0, 255]; ck_y / ck_uv the networks for luma / chroma (NULL: plane
 * not filtered), use_u / use_v the chroma planes filtered; tile_size 0: one tile. */
int zo_icci_filter(const zo_ckpt *ck_y, const zo_ckpt *ck_uv, int use_u, int use_v, float *y,
                   float *u, float *v, int h, int w, int tile_size, int overlap);
void zo_dwt2_block(const float p[16], float out[16]);
void zo_idwt2_block(const float s[16], float out[16]);

/* EFE linear (src/filters/efe_linear.rs:120-460). One coded filter set (header.rs:623-639):
 * per chroma plane p the split candidate cand[p] (0..7, -1: not filtered), the filter side
 * filter_len[p], and the weight codes of the split's regions in order, chroma_codes[p]
 * regions x P x fL x fL (P = 1 for pictures coded at the source's chroma resolution, else 4)
 * and luma_codes[p] regions x fL x fL; min_symbol is added to every code. */
typedef struct {
    int cand[2], filter_len[2], min_symbol;
    const uint32_t *chroma_codes[2], *luma_codes[2];
} zo_efe_linear_set;
/* `split_edge` (efe_linear.rs:128-131) */
int zo_efe_split_edge(double fraction, int s);
/* `apply` (efe_linear.rs:403-460) with one set: y [h][w], u / v [ch][cw] in [0, 255] of a
 * source subsampled s_ver x s_hor and coded c_ver x c_hor; mean_* the B1 codes (1/100 units).
 * Writes the filtered chroma planes. Returns the crate's error as a zjai_status number
 * (0 ok, 1 invalid argument, 2 unsupported, 6 invalid data). */
int zo_efe_linear(const float *y, int h, int w, const float *u, const float *v, int ch, int cw,
                  int s_ver, int s_hor, int c_ver, int c_hor, int mean_u, int mean_v,
                  const zo_efe_linear_set *set, float *out_u, float *out_v);

/* EFE non-linear (src/filters/efe_nonlinear.rs:177-237) in place on u / v [ch][cw]: the
 * per-tile luma network where codes[p] is given (8 codes per tile, ncodes[p] of them), then the
 * on/off switch towards alt_u / alt_v where mask[0] is given (mask_h x mask_w values per plane,
 * blocks of mask_bs samples); source / coded formats as zo_efe_linear. Return codes as
 * zo_efe_linear. */
typedef struct {
    int min_symbol;
    int tile_width, tile_height, ntiles;
    const uint16_t *luma_min, *luma_max;
    const uint32_t *codes[2];
    int ncodes[2];
    int mask_bs, mask_h, mask_w;
    const uint8_t *mask[2];
} zo_efe_nonlinear_params;
int zo_efe_nonlinear(const float *y, int h, int w, float *u, float *v, int ch, int cw,
                     int s_ver, int s_hor, int c_ver, int c_hor,
                     const zo_efe_nonlinear_params *prm, const float *alt_u, const float *alt_v);

/* RDLR layer VJPs, the input gradients of the conv layers. `conv2d_backward`
 * (reference.rs:241-292) through `ConvLayer::backward` (layers.rs:72-90): d_out [oc][oh][ow]
 * of a conv with weight [oc][c/groups][kh][kw] and zero border extra ([top, left, bottom,
 * right] or NULL) on an input [c][h][w] -> din [c][h][w]. */
int zo_conv2d_backward(const float *dout, int oc, int oh, int ow, const float *weight, int c,
                       int kh, int kw, int stride, int pad_h, int pad_w, int groups,
                       const int extra[4], int h, int w, float *din);
/* `conv_transpose2d_backward` (reference.rs:294-336): d_out [oc][oh][ow] of a transposed conv
 * with weight [c][oc][k][k] on an input [c][h][w] -> din [c][h][w]. */
int zo_conv_transpose2d_backward(const float *dout, int oc, int oh, int ow, const float *weight,
                                 int c, int k, int stride, int pad, int h, int w, float *din);
/* `ResidualBlock::backward` (attention.rs:58-75): d_out and the tape conv1_out [c][h][w], conv
 * weights [c][c][3][3] -> din [c][h][w]. */
int zo_residual_block_backward(const float *dout, const float *conv1_out, int c, int h, int w,
                               const float *w1, const float *w2, float *din);
/* `Cab::backward` (attention.rs:182-223): tape t = {trunk_pre, sig, trunk RB0 conv1 output,
 * trunk RB1 conv1 output} [c][h][w], mask_c1 = the mask RBs' conv1 outputs [c][h/2][w/2];
 * weights wt = trunk0 conv1, conv2, trunk1 conv1, conv2, subscale, mask2 conv1, conv2, mask3
 * conv1, conv2, upscale (each [c][c][3][3]). */
int zo_cab_backward(const float *dout, int c, int h, int w, const float *const t[4],
                    const float *const mask_c1[2], const float *const wt[10], float *din);
/* `elu_gate_backward` (math.rs:838-858) and `layer_norm_channels_backward` (math.rs:860-913). */
void zo_elu_gate_backward(const float *d, const float *a, const float *b, int64_t n, float *d_a,
                          float *d_b);
int zo_layer_norm_backward(const float *d, const float *x, int c, int h, int w,
                           const float *weight, float *dx);
/* The softmax weights attn [dim][c] of `channel_attention` (the backward's tape) and
 * `channel_attention_backward` (math.rs:668-836): d_out [dim][h][w] -> dqkv [3 dim][h][w]. */
int zo_channel_attention_weights(const float *qkv, int c3, int h, int w, int heads,
                                 const float *temperature, float *attn);
int zo_channel_attention_backward(const float *qkv, int c3, int h, int w, int heads,
                                  const float *temperature, const float *attn,
                                  const float *dout, float *dqkv);
/* `TransformerBlock::backward` (attention.rs:435-480): tape = {x_in, qkv, attn, x_mid, gate},
 * wt = {prep_norm.weight, prep_conv1, prep_conv2, temperature, attn_out, ffn_norm.weight,
 * ffn_in, ffn_dw, ffn_out}; d_out [dim][h][w] -> din [dim][h][w]. */
int zo_transformer_block_backward(const float *dout, int dim, int hidden, int heads, int h, int w,
                                  const float *const tape[5], const float *const wt[9],
                                  float *din);
/* `Tam::backward` (attention.rs:578-600): the two blocks' VJPs, between the VJPs of the
 * stride-2 ds_conv and the transposed us_conv when resample is set; h x w the TAM's input. */
int zo_tam_backward(const float *dout, int dim, int hidden, int heads, int h, int w, int resample,
                    const float *const tape0[5], const float *const tape1[5],
                    const float *const wt0[9], const float *const wt1[9], const float *ds_w,
                    const float *us_w, float *din);

#ifdef __cplusplus
}
#endif
#endif
