// Network objects and the per-call runner that executes a topology on a batch of tiles.
#pragma once
#include <array>
#include <map>
#include <string>
#include <vector>

#include "engine.h"

namespace zjai {

// A loaded network: packed conv layers and small f32 parameter vectors, GPU resident.
struct Net {
  Ctx* ctx = nullptr;
  int kind = 0, op = 0;
  // unique per loaded network for the life of the process (graph cache keys: a network created
  // at the address of a destroyed one is a different network)
  uint64_t uid = 0;
  std::map<std::string, ConvLayer> convs;
  std::map<std::string, float*> vecs;  // LN weight/bias, temperature, depthwise weights [c][9]
  // f16 scale of the per-picture weights W_o . blockdiag(A) of each transformer block's folded
  // attention projection (keyed by the block prefix)
  std::map<std::string, float> fold_scale;
  // fused FFN weights of each transformer block whose shape the fused kernel takes (keyed by
  // the block prefix)
  std::map<std::string, FfnLayer> ffns;
  // conv stage (zjai_stage_create): activation of the first conv, its pixel shuffle, the
  // activation inside the residual blocks, their number, input and output channels
  int st_act = 0, st_shuffle = 1, st_res_act = 0, st_nres = 0, st_cin = 0, st_cout = 0;
  // latent networks (ZJAI_LATENT): latent channel count, and whether the checkpoint holds the
  // context model
  int lat_c = 0;
  bool lat_ctx = false;
  ~Net();
};

// eICCI network shape (src/model/icci.rs:33-40)
constexpr int kIcciFeatures = 48, kIcciBands = 16, kIcciLumaBlocks = 2, kIcciChromaBlocks = 4;

// Net::kind of a conv stage (not one of the crate's network kinds)
constexpr int kStageKind = 4;

// Where a synthesis network's final planar output goes.
struct FinalOut {
  float* plane0 = nullptr;
  float* plane1 = nullptr;       // second plane (chroma V); null: plane0 + plane_stride
  long long plane_stride = 0, row = 0, img = 0;
  // per-tile {py0, px0, cy0, cy1, cx0, cx1, plane base} (device) or null
  const int* win = nullptr;
  int sv = 1, sh = 1;
  int full_h = -1, full_w = -1;  // clip of the network output extent (-1: natural)
  // fused output stage: planes of quantized samples (1 = uint8, 2 = uint16, to qmax)
  int qbytes = 0;
  float qmax = 255.f;
};

// Executes one network on a batch of `n` same-shape inputs on one stream, allocating its
// activations from one arena. Temporaries of each block are released when the block has been
// enqueued (the stream orders their reuse).
struct Runner {
  Ctx* ctx = nullptr;
  Net* net = nullptr;
  Arena* arena = nullptr;
  cudaStream_t stream = nullptr;
  int n = 1;
  const volatile int* cancel = nullptr;
  bool count_flops = false;
  double flops = 0.0;

  int alloc(int h, int w, int c, TView* v);
  const ConvLayer* layer(const std::string& name);
  int conv(const std::string& name, const TView& in, ConvOut o);
  // conv with an explicit packed layer (a variant of the loaded layer `name`)
  int conv_layer(const std::string& name, const ConvLayer& L, const TView& in, ConvOut o);
  std::string kind_tag() const;
  // A memory-bound kernel (`launches` launches issued by `f` on this runner's stream), profiled
  // under "<kind tag><name>[<kind>]" with its algorithmic bytes.
  template <class F>
  void mem_kernel(const std::string& name, const char* kind, double bytes, int launches, F&& f) {
    cudaStream_t saved = ctx->stream;
    ctx->stream = stream;
    if (ctx->profiling) ctx->tag = kind_tag() + name + "[" + kind + "]";
    timed_launch(ctx, false, 0.0, bytes, f);
    ctx->stream = saved;
    ctx->launches += launches;
  }
  int out_extent(const std::string& name, int h, int w, int* oh, int* ow);
  int stop_check();
  // copy `t` as planar f32 [n][c][h][w] into the capture registered under `name`, if any
  int probe(const char* name, const TView& t);

  int resau(const std::string& p, const TView& x, const TView& a, int ch, int cw, TView* y);
  int rb(const std::string& p, const TView& x, const TView& y, const TView* relu6_out = nullptr,
         int act = ACT_RELU);
  int cab(const std::string& p, const TView& x, const TView& out, const TView* a_out);
  int tb(const std::string& p, const TView& x);
  int tam(const std::string& p, const TView& x, bool ds, int ch, int cw, TView* y, TView* a_out);
  int upsample(const std::string& p, const TView& x, int ch, int cw, TView* y, TView* a_out);
  int final_planar(const std::string& name, const TView& x, const FinalOut& fo);

  int primary(const TView& y, int h, int w, const FinalOut& fo);
  int secondary(const TView& cat, const TView& x144, int h, int w, const FinalOut& fo);
  int analysis(const TView& x, int h, int w, float* out);
  // conv stage: x (NHWC, st_cin channels) -> planar f32 out [st_cout][h * r][w * r]
  int stage(const TView& x, float* out);
  // eICCI trunk + last convs on the 48 sub-bands: planar f32 corrections [16][h][w] of the
  // luma (c0) or of u (c0) and v (c1) when `chroma`; a null pointer skips that output
  int icci(const TView& x, bool chroma, float* c0, float* c1);
  // hyper-decoder: z (NHWC, lat_c channels) -> psi planar f32 [4 lat_c][out_h][out_w]
  int hyper(const TView& z, int out_h, int out_w, float* psi);
  // latent from psi planar f32 [4C][ceil(h/2)][ceil(w/2)] and the residual planar f32
  // [C][h][w] -> y planar f32 [C][h][w] (context model, or upshuffle_psi + residual)
  int latent(const float* psi, const float* res, int h, int w, float* y);
};

struct ArenaMark {
  Arena* a;
  size_t m;
  explicit ArenaMark(Arena* ar) : a(ar), m(ar->mark()) {}
  ~ArenaMark() { a->release(m); }
};

int load_network(Ctx* ctx, int kind, int op, const zjai_param* params, int nparams, Net** out);
int load_stage(Ctx* ctx, int shuffle, int act, int res_act, const zjai_param* params,
               int nparams, Net** out);
int synthesis_tiles(int height, int width, int latent_h, int latent_w, int tile_size,
                    int overlap, std::vector<zjai_tile>* out);
void synth_out_size(int kind, int op, int h, int w, int* oh, int* ow);

void launch_replicate_pad(const TView& src, const TView& dst, cudaStream_t s);
void launch_normalize_pad(const float* src, int c, int h, int w, const TView& dst, cudaStream_t s);
// normalize_pad of the h x w window at (y0, x0) of planar pictures [n][c][SH][SW]
void launch_normalize_pad_window(const float* src, int c, int SH, int SW, int y0, int x0, int h,
                                 int w, const TView& dst, cudaStream_t s);
// The luma analysis input as the nine taps of its first layer per output pixel: dst
// [n][cdiv(h, 2)][cdiv(w, 2)][9 (16 in memory)] from the h x w window at (y0, x0) of one-channel
// planar pictures [n][SH][SW] (normalize_pad's values; see the kernel)
void launch_normalize_im2col(const float* src, int SH, int SW, int y0, int x0, int h, int w,
                             const TView& dst, cudaStream_t s);
// colour.rs preprocess_rgb of n pictures [n][h][w][3] -> luma [n][h][w], chroma
// [n][12][ph / 2][pw / 2] (planar f32, [0, 255])
void launch_preprocess_rgb(const uint8_t* rgb, int n, int h, int w, float* luma, float* chroma,
                           cudaStream_t s);
// output.cu: bicubic 4:2:0 -> 4:4:4, BT.709 and quantisation of device planes into interleaved
// RGB (uint8 for 8 bits, else uint16), on stream s
int output_yuv_to_rgb(Ctx* ctx, const float* y, const float* u, const float* v, int h, int w,
                      int ch, int cw, int bit_depth, void* rgb, cudaStream_t s);
// context-model layout kernels (kernels_misc.cu): psi quarters into the joined buffer J
// (channel k of quarter s at k + (s + 1) C), one stage's residual add / y_hat scatter / context
// write, and upshuffle_psi + residual
void launch_psi_to_joined(const float* psi, int C, int hh, int hw, const TView& J, cudaStream_t s);
void launch_mcm_stage(const float* mean, const float* res, int C, int h, int w, int py, int px,
                      float* y, const TView* ctx, cudaStream_t s);
void launch_upshuffle_add(const float* psi, const float* res, int C, int h, int w, float* y,
                          cudaStream_t s);
void launch_copy_core(const float* tile, int n, int C, int th, int tw, int oy, int ox, int core_h,
                      int core_w, float* full, int LH, int LW, int cy, int cx, cudaStream_t s);

// `analysis_tiles` (encoder/tiles.rs:51-156, no independent regions) of component ccs for a
// plane of h x w samples with latent lh x lw: {img x, y, w, h, latent x, y, w, h, core x, y, w,
// h, core offset x, y} per tile.
int analysis_tiles(int ccs, int h, int w, int lh, int lw, std::vector<std::array<int, 14>>* out);

}  // namespace zjai
