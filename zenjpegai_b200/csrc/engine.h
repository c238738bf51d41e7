// Host-side engine internals: context, device arena, NHWC tensor views, packed layers.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <array>
#include <atomic>
#include <cstdint>
#include <map>
#include <string>
#include <utility>
#include <vector>

#include "../../include/zjai.h"
#include "conv_tc.cuh"

namespace zjai {

// ---- errors -------------------------------------------------------------------------------
struct Error {
  int code;
  std::string msg;
};
void set_last_error(int code, const std::string& msg);
#define ZJAI_TRY(expr)                         \
  do {                                         \
    int _st = (expr);                          \
    if (_st != ZJAI_OK) return _st;            \
  } while (0)
int fail(int code, const std::string& msg);  // records and returns code
int cuda_check(cudaError_t e, const char* what);

// ---- device arena (bump allocator, 256-byte aligned) ---------------------------------------
struct Arena {
  char* base = nullptr;
  size_t cap = 0, top = 0, peak = 0;
  void* alloc(size_t bytes);  // nullptr when exhausted
  size_t mark() const { return top; }
  void release(size_t m) { top = m; }
};

// NHWC f16 view: element (n, y, x, c) at p[n*img + y*row + x*pix + c]. A crop is a view with
// smaller h / w over the same memory; a channel slice is a view with an offset pointer.
struct TView {
  __half* p = nullptr;
  int n = 1, h = 0, w = 0, c = 0;
  long long pix = 0, row = 0, img = 0;
  // rows / cols actually backed by zeroed memory beyond (h, w) (stride-2 inputs need even)
  int alloc_h = 0, alloc_w = 0;
  TView crop(int hh, int ww) const {
    TView v = *this;
    v.h = hh;
    v.w = ww;
    return v;
  }
  TView channels(int c0, int cc) const {
    TView v = *this;
    v.p = p + c0;
    v.c = cc;
    return v;
  }
};

// A captured call (zjai_ctx_set_graphs): the instantiated graph, the pinned host copies its
// uploads read at every replay, and the kernel launches it holds.
struct GraphEntry {
  cudaGraphExec_t exec = nullptr;
  std::vector<void*> pins;
  long long launches = 0;
  int calls = 0;  // eager calls seen with this key (negative: capture failed, stay eager)
};

struct Ctx {
  int device = 0;
  int sms = 148;
  cudaStream_t own = nullptr, stream = nullptr, stream2 = nullptr;
  cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
  Arena arena;   // work of `stream`
  Arena arena2;  // work of `stream2` (chroma synthesis runs beside luma)
  Arena* cur_arena = nullptr;  // arena of the network runner currently launching (or null)
  // kernel status words: [0] the code of a bounded wait that gave up, [1] set when a residual /
  // gate epilogue produced an activation beyond the f16 range
  int* d_err = nullptr;
  // final synthesis layers clamp the denormalised planes to [0, 255] (false: the raw
  // x * 128 + 127.5, zjai_ctx_set_output_clamp)
  bool clamp_output = true;
  // CUDA graphs of repeated tiled-synthesis calls (zjai_ctx_set_graphs): per call signature the
  // entry; while a call is being captured, the pinned host copies of its uploads are collected
  // in capture_pins
  bool graphs = false;
  std::map<std::string, GraphEntry> graph_cache;
  std::vector<void*>* capture_pins = nullptr;
  void clear_graphs();
  // captures of named intermediate maps (zjai_ctx_set_probe): name -> (device buffer of planar
  // f32 [n][c][h][w], its capacity in floats)
  std::map<std::string, std::pair<float*, long long>> probes;
  // limit of the convolution kernel's pipeline waits in SM cycles (0: the kernel's default of
  // about 2 s), zjai_ctx_set_wait_limit
  long long wait_cycles = 0;
  std::atomic<long long> launches{0};
  // Tiled synthesis runs the shape groups' chains concurrently once their arena needs are
  // known: per group key (operating point, tile h, w, latent h, w, batch) the bytes its luma
  // and its chroma chains took from the arenas, recorded by a sequential call; and a pool of
  // streams (luma, chroma per group) and events for the fork and join.
  std::map<std::array<int, 6>, std::pair<size_t, size_t>> group_need;
  std::vector<cudaStream_t> group_streams;
  std::vector<cudaEvent_t> group_events;
  // driver entry point
  void* encode_fn = nullptr;
  int driver_version = 0;
  // kernel timing (the crate's DecodeStats probe, per launch): when `profiling`, every conv
  // launch (and every memory-bound kernel of the networks) is bracketed by two events and its
  // algorithmic FLOPs (conv) or bytes (the others) are recorded
  bool profiling = false;
  std::vector<cudaEvent_t> ev_pool;
  struct ConvRecord {
    cudaEvent_t start, stop;
    double flops, bytes;
    std::string tag;
    bool conv;
  };
  std::vector<ConvRecord> conv_records;
  std::string tag;  // name of the layer being launched (for the profile report)
  // per-tag totals accumulated by zjai_ctx_profile_read: launches, ms, flops, bytes
  struct TagTotal {
    long long launches = 0;
    double ms = 0.0, flops = 0.0, bytes = 0.0;
  };
  std::vector<std::pair<std::string, TagTotal>> tag_totals;
  cudaEvent_t take_event();
};

// Launch `f` on ctx->stream; when profiling, bracket it with events and record its work
// (algorithmic FLOPs for a conv, algorithmic bytes for a memory-bound kernel) under ctx->tag.
template <class F>
void timed_launch(Ctx* ctx, bool conv, double flops, double bytes, F&& f) {
  if (!ctx->profiling) {
    f();
    return;
  }
  Ctx::ConvRecord r{ctx->take_event(), ctx->take_event(), flops, bytes, ctx->tag, conv};
  cudaEventRecord(r.start, ctx->stream);
  f();
  cudaEventRecord(r.stop, ctx->stream);
  ctx->conv_records.push_back(r);
}

// Host -> device copy on stream s; during a graph capture the source is first copied into
// pinned memory kept with the graph (replays read it), otherwise copied as given.
int h2d_async(Ctx* ctx, void* dst, const void* src, size_t bytes, cudaStream_t s);

// Allocate an NHWC f16 tensor in the arena; channels padded to `cpad` (multiple of 8), and
// rows / cols rounded up to even so any stride-2 consumer can read it. Zero-filled when
// `zero` (async on ctx stream).
int alloc_tensor(Ctx* ctx, int n, int h, int w, int c, TView* out, bool zero = false,
                 Arena* arena = nullptr, cudaStream_t stream = nullptr);

// ---- TMA descriptors ------------------------------------------------------------------------
int make_act_map(Ctx* ctx, CUtensorMap* m, const TView& v, int kc, int bw, int bh);
int make_act_map_s2(Ctx* ctx, CUtensorMap* m, const TView& v, int img, int kc, int bw, int bh);
// box [bc channels, bx, by] over an NHWC f16 view, no swizzle (shared-memory image
// [by][bx][bc])
int make_tile_map(Ctx* ctx, CUtensorMap* m, const TView& v, int bc, int bx, int by);
// output map of the TMA-store epilogue: box [16 channels, bx, by] over an NHWC f16 view
int make_store_map(Ctx* ctx, CUtensorMap* m, const TView& v, int bx, int by);

// ---- packed convolution ---------------------------------------------------------------------
// A convolution (or a stride-2 transposed convolution rewritten as a phase convolution)
// packed for conv_tc_kernel: weights [tap][npad][cin_pad] f16 scaled by 2^s, bias [npad] f32
// in the same (phase-major) column order.
struct ConvLayer {
  int cin = 0, kc = 64, cchunks = 1, cin_pad = 64;
  int kh = 1, kw = 1, pad_t = 0, pad_l = 0, pad_b = 0, pad_r = 0, stride = 1;
  int ncols = 0, bn = 16, n_tiles = 1, npad = 16;
  int R = 1, cph = 1;
  int transposed = 0, t_k = 0, t_pad = 0, t_outpad = 0;  // convT output-size rule
  float scale = 1.f;
  __half* w = nullptr;
  long long w_img = 0;  // per-picture weight sets (stride in halves), 0: one set
  // live K steps per N tile (ConvArgs::klist / koff), null when every block is live
  uint32_t* klist = nullptr;
  int* koff = nullptr;
  // grouped packing (ConvArgs::grp_n / grp_pc): output columns per group and groups per
  // 64-channel chunk, 0 for a dense layer
  int grp_n = 0, grp_pc = 0;
  // live taps per N tile of a halo-mode transposed conv (ConvArgs::tmask), tmask_on = 0: all
  int tmask_on = 0;
  uint32_t tmask[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  float* bias = nullptr;
  long long flops_per_px = 0;  // algorithmic MACs*2 per conv-output pixel (live taps only)
  // conv output extent (GEMM M space) and shuffled output extent for an input of h x w
  void out_size(int h, int w, int* oh, int* ow, int* out_h, int* out_w) const;
};

// Pack a PyTorch conv (weight [cout][cin/groups][kh][kw]) with zero border `extra` and an
// optional pixel shuffle `ps` folded into the column order.
int pack_conv(Ctx* ctx, ConvLayer* L, const float* w, const float* b, int cin, int cout, int kh,
              int kw, int stride, int pad_h, int pad_w, int groups, const int* extra, int ps);
// Pack a PyTorch stride-2 transposed conv (weight [cin][cout][k][k]) as a phase conv; `post_ps`
// folds a following pixel shuffle (HOP chroma output) into the columns.
int pack_convT(Ctx* ctx, ConvLayer* L, const float* w, const float* b, int cin, int cout, int k,
               int pad, int out_pad, int post_ps);
void free_conv(ConvLayer* L);
// Power-of-two scale that brings max |w| into [2^13, 2^14) (the packed f16 weight scale).
float pow2_weight_scale(const float* w, size_t n);

// Epilogue / output description for one conv launch.
struct ConvOut {
  int act1 = ACT_NONE, op = OP_NONE, act2 = ACT_NONE;
  TView out;                 // NHWC output (logical extent = crop)
  const TView* r1 = nullptr;  // residual operands in output space
  const TView* r2 = nullptr;
  const TView* out2 = nullptr;  // relu6 copy
  // planar f32 output
  bool planar = false, denorm = false;
  bool clamp = true;  // denormalised planar output clamped to [0, 255]
  float* pout = nullptr;
  float* pout2 = nullptr;
  const int* img_win = nullptr;  // per-image output windows (device), see ConvArgs
  long long p_plane = 0, p_row = 0, p_img = 0;
  int py0 = 0, px0 = 0, cy0 = 0, cy1 = 1 << 30, cx0 = 0, cx1 = 1 << 30, sv = 1, sh = 1;
  int out_h = -1, out_w = -1;  // planar: network output extent clip (-1 = from layer)
  // planar: quantized samples (1 = uint8, 2 = uint16, to qmax) instead of f32 (ConvArgs)
  int qbytes = 0;
  float qmax = 255.f;
};

int run_conv(Ctx* ctx, const ConvLayer& L, const TView& in, const ConvOut& o);

// Fused feed-forward half of a transformer block (ffn_tc.cu): W_in [2 hidden][dim] and
// W_out [dim][hidden] packed into the kernel's 128-row / dim-row blocks, the depthwise weights
// [2 hidden][9] regrouped per chunk, tap and channel pair.
struct FfnLayer {
  int dim = 0, hidden = 0;
  __half* win = nullptr;
  __half* wout = nullptr;
  float* wdw = nullptr;
  float scale_in = 1.f, scale_out = 1.f;
};
// The fused kernel's shapes: dim 64 or 128, hidden a multiple of 64.
bool ffn_fusable(int dim, int hidden);
int pack_ffn(Ctx* ctx, FfnLayer* L, const float* w_in, const float* w_dw, const float* w_out,
             int dim, int hidden);
void free_ffn(FfnLayer* L);
// x += W_out . gate(dw3x3(W_in . ln)) in place on x (NHWC f16, dim channels), on ctx->stream.
int run_ffn(Ctx* ctx, const FfnLayer& L, const TView& ln, const TView& x);

// ---- elementwise / layout kernels (kernels_misc.cu) ---------------------------------------
// planar f32 [n][c][h][w] window (y0, x0, h, w of a [c][H][W] source) -> NHWC f16 view
void launch_planar_to_nhwc(const float* src, int c, int H, int W, int y0, int x0,
                           const TView& dst, cudaStream_t s);
void launch_nhwc_to_planar(const TView& src, float* dst, cudaStream_t s);
void launch_relu6(const TView& src, const TView& dst, cudaStream_t s);

}  // namespace zjai
