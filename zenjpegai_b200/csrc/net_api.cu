// C ABI of the networks, the tiling scheduler and the attention-block layer entries.
#include <algorithm>
#include <map>
#include <tuple>
#include <vector>

#include "api_common.h"
#include "kernels_attn.h"
#include "net.h"

struct zjai_net : zjai::Net {};

using namespace zjai;

namespace {

int cdiv(int a, int b) { return (a + b - 1) / b; }

int net_enter(zjai_net* net) {
  if (!net || !net->ctx) return fail(ZJAI_INVALID_ARGUMENT, "null network");
  return ctx_enter(static_cast<zjai_ctx*>(net->ctx));
}

// Device int array (arena) holding `v`.
int upload_ints(Ctx* ctx, Arena* arena, const std::vector<int>& v, cudaStream_t s, int** out) {
  int* d = static_cast<int*>(arena->alloc(v.size() * sizeof(int) + 16));
  if (!d) return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (descriptors)");
  ZJAI_TRY(h2d_async(ctx, d, v.data(), v.size() * sizeof(int), s));
  *out = d;
  return ZJAI_OK;
}

Runner make_runner(Ctx* ctx, Net* net, Arena* arena, cudaStream_t s, int n,
                   const volatile int* cancel) {
  Runner r;
  r.ctx = ctx;
  r.net = net;
  r.arena = arena;
  r.stream = s;
  r.n = n;
  r.cancel = cancel;
  return r;
}

// Sync after a failure so the context and its arena stay usable (the group streams too: a
// failure or cancellation can leave chains of a concurrent tiled synthesis enqueued).
int settle(Ctx* ctx, int st) {
  cudaStreamSynchronize(ctx->stream);
  cudaStreamSynchronize(ctx->stream2);
  for (cudaStream_t gs : ctx->group_streams) cudaStreamSynchronize(gs);
  return st;
}

}  // namespace

namespace zjai {

// The pictures of a batched synthesis: per tile its picture (latents [picture][C][lh][lw]),
// and the samples of one picture's luma / chroma output plane (the planes are
// [picture][h][w]). Empty: every tile belongs to the one picture.
struct TilePictures {
  std::vector<int> pic;
  long long plane_y = 0, plane_uv = 0;
};

// One shape group of a tiled synthesis: the latent windows of its tiles gathered into one
// batch, the luma network on stream `sy` with arena `ay`, the chroma network on `sc` with `ac`
// (after the gather). Output planes are device pointers.
struct GroupJob {
  int img_h, img_w, lat_h, lat_w;
  std::vector<int> idx;
};

static int run_group(Ctx* ctx, Net* ny, Net* nuv, const float* lat_y, const float* lat_uv, int lh,
                     int lw, const std::vector<zjai_tile>& tiles, const TilePictures& pics,
                     const GroupJob& g, int out_h, int out_w, int sv, int sh, float* rec_y,
                     float* rec_u, float* rec_v, const volatile int* cancel, double* flops,
                     int qbytes, float qmax, cudaStream_t sy, cudaStream_t sc, Arena* ay,
                     Arena* ac, cudaEvent_t ev) {
  const int n = (int)g.idx.size();
  const int cw_ = cdiv(out_w, sh);
  std::vector<int> origin, win_y, win_uv;
  for (int i : g.idx) {
    const zjai_tile& t = tiles[i];
    const int p = pics.pic.empty() ? 0 : pics.pic[i];
    origin.insert(origin.end(), {t.lat_x, t.lat_y, p});
    const std::initializer_list<int> w = {t.img_y, t.img_x, t.core_y,
                                          std::min(t.core_y + t.core_h, out_h), t.core_x,
                                          std::min(t.core_x + t.core_w, out_w)};
    win_y.insert(win_y.end(), w);
    win_y.push_back((int)(p * pics.plane_y));
    win_uv.insert(win_uv.end(), w);
    win_uv.push_back((int)(p * pics.plane_uv));
  }
  // each stream reads descriptor copies from its own arena
  int *d_origin, *d_origin2, *d_win_y, *d_win_uv;
  ZJAI_TRY(upload_ints(ctx, ay, origin, sy, &d_origin));
  ZJAI_TRY(upload_ints(ctx, ay, win_y, sy, &d_win_y));
  ZJAI_TRY(upload_ints(ctx, ac, origin, sc, &d_origin2));
  ZJAI_TRY(upload_ints(ctx, ac, win_uv, sc, &d_win_uv));
  // latent windows: [n][lat_h][lat_w][256] = luma 160 | chroma 96 (luma stream)
  TView cat;
  ZJAI_TRY(alloc_tensor(ctx, n, g.lat_h, g.lat_w, 256, &cat, false, ay, sy));
  launch_gather_latent(lat_y, 160, lh, lw, d_origin, cat.channels(0, 160), sy);
  launch_gather_latent(lat_uv, 96, lh, lw, d_origin, cat.channels(160, 96), sy);
  ctx->launches += 2;
  ZJAI_TRY(cuda_check(cudaEventRecord(ev, sy), "event"));
  // luma
  {
    Runner r = make_runner(ctx, ny, ay, sy, n, cancel);
    r.count_flops = flops != nullptr;
    FinalOut fo;
    fo.plane0 = rec_y;
    fo.row = out_w;
    fo.win = d_win_y;
    fo.qbytes = qbytes;
    fo.qmax = qmax;
    ZJAI_TRY(r.primary(cat.channels(0, 160), g.img_h, g.img_w, fo));
    if (flops) *flops += r.flops;
  }
  // chroma (reads `cat`, gathered on the luma stream)
  ZJAI_TRY(cuda_check(cudaStreamWaitEvent(sc, ev, 0), "event wait"));
  {
    Runner r = make_runner(ctx, nuv, ac, sc, n, cancel);
    r.count_flops = flops != nullptr;
    TView x144;
    ZJAI_TRY(alloc_tensor(ctx, n, g.lat_h, g.lat_w, 144, &x144, false, ac, sc));
    launch_gather_latent(lat_uv, 96, lh, lw, d_origin2, x144.channels(48, 96), sc);
    ctx->launches++;
    FinalOut fo;
    fo.plane0 = rec_u;
    fo.plane1 = rec_v;
    fo.row = cw_;
    fo.win = d_win_uv;
    fo.sv = sv;
    fo.sh = sh;
    fo.qbytes = qbytes;
    fo.qmax = qmax;
    ZJAI_TRY(r.secondary(cat, x144, g.img_h, g.img_w, fo));
    if (flops) *flops += r.flops;
  }
  return ZJAI_OK;
}

// The pool of group streams / events, created on first use.
static int group_pool(Ctx* ctx, size_t streams, size_t events) {
  // Streams 0 and 1 carry the luma and chroma chains of the largest shape group (groups run
  // largest first), the step's critical path: at the greatest priority their blocks are
  // scheduled ahead of the other chains', which fill the SMs they leave (4K HOP step 8.30 ->
  // 8.12 ms; raising every luma chain instead was not steadily better). Graph replays keep the
  // priorities (node priorities).
  while (ctx->group_streams.size() < streams) {
    int least = 0, greatest = 0;
    ZJAI_TRY(cuda_check(cudaDeviceGetStreamPriorityRange(&least, &greatest), "priority range"));
    cudaStream_t s;
    const int prio = ctx->group_streams.size() < 2 ? greatest : least;
    ZJAI_TRY(cuda_check(cudaStreamCreateWithPriority(&s, cudaStreamNonBlocking, prio), "stream"));
    ctx->group_streams.push_back(s);
  }
  while (ctx->group_events.size() < events) {
    cudaEvent_t e;
    ZJAI_TRY(cuda_check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "event"));
    ctx->group_events.push_back(e);
  }
  return ZJAI_OK;
}

// Synthesis of the listed tiles: same-shape tiles run as one batch, luma and chroma of a batch
// on two streams (reconstruct.rs:314-323 runs the two components side by side). The shape
// groups' chains (e.g. interior, bottom-row, right-column and corner tiles) run one after
// another on the context's two streams the first time a group shape is seen, which records how
// much of each arena every chain takes; once every group's needs are known and fit, each group
// runs on its own pair of streams in its own slice of the arenas, so the small groups' chains
// overlap the large one's. Output planes are device pointers.
int synthesize_tiles_dev(Ctx* ctx, Net* ny, Net* nuv, const float* lat_y, const float* lat_uv,
                         int lh, int lw, const std::vector<zjai_tile>& tiles, int out_h, int out_w,
                         int sv, int sh, float* rec_y, float* rec_u, float* rec_v,
                         const volatile int* cancel, double* flops, int bit_depth,
                         const TilePictures& pics) {
  // bit_depth > 0: the final layers write quantized samples (uint8 for 8 bits, else uint16)
  // into rec_* instead of f32 planes
  const int qbytes = bit_depth <= 0 ? 0 : bit_depth == 8 ? 1 : 2;
  const float qmax = bit_depth <= 0 ? 255.f : (float)((1u << bit_depth) - 1);
  if (!ny || !nuv || ny->kind != ZJAI_SYN_Y || nuv->kind != ZJAI_SYN_UV || ny->op != nuv->op)
    return fail(ZJAI_INVALID_ARGUMENT, "synthesize: needs a SYN_Y and a SYN_UV network of one op");
  if (sv <= 0 || sh <= 0) return fail(ZJAI_INVALID_DATA, "chroma subsampling factor");
  // group same-shape tiles (largest group first: it sets the critical path)
  std::map<std::tuple<int, int, int, int>, std::vector<int>> by_shape;
  for (size_t i = 0; i < tiles.size(); ++i) {
    const zjai_tile& t = tiles[i];
    if (t.lat_x < 0 || t.lat_y < 0 || t.lat_x + t.lat_w > lw || t.lat_y + t.lat_h > lh)
      return fail(ZJAI_INVALID_DATA, "synthesis tile outside the latent");
    by_shape[std::make_tuple(t.img_h, t.img_w, t.lat_h, t.lat_w)].push_back((int)i);
  }
  std::vector<GroupJob> groups;
  for (auto& kv : by_shape)
    groups.push_back({std::get<0>(kv.first), std::get<1>(kv.first), std::get<2>(kv.first),
                      std::get<3>(kv.first), kv.second});
  std::stable_sort(groups.begin(), groups.end(), [](const GroupJob& a, const GroupJob& b) {
    return a.idx.size() * a.img_h * a.img_w > b.idx.size() * b.img_h * b.img_w;
  });
  auto key = [&](const GroupJob& g) {
    return std::array<int, 6>{ny->op, g.img_h, g.img_w, g.lat_h, g.lat_w, (int)g.idx.size()};
  };
  // concurrent chains when every group's arena needs are known and fit
  bool concurrent = !ctx->profiling && groups.size() > 1 && groups.size() <= 4;
  size_t sum_y = 0, sum_c = 0;
  for (const GroupJob& g : groups) {
    auto it = ctx->group_need.find(key(g));
    if (it == ctx->group_need.end()) {
      concurrent = false;
      break;
    }
    // slack for the 256-byte alignment of each slice
    sum_y += it->second.first + 1024;
    sum_c += it->second.second + 1024;
  }
  if (concurrent && (sum_y > ctx->arena.cap - ctx->arena.top || sum_c > ctx->arena2.cap - ctx->arena2.top))
    concurrent = false;
  if (!concurrent) {
    // while profiling, chroma runs after luma on one stream so per-layer events see no overlap
    cudaStream_t s1 = ctx->stream, s2 = ctx->profiling ? ctx->stream : ctx->stream2;
    ZJAI_TRY(cuda_check(cudaEventRecord(ctx->ev_fork, s1), "event"));
    ZJAI_TRY(cuda_check(cudaStreamWaitEvent(s2, ctx->ev_fork, 0), "event wait"));
    for (const GroupJob& g : groups) {
      if (cancel && *cancel) return fail(ZJAI_CANCELLED, "stopped: cancelled by the caller");
      const size_t m1 = ctx->arena.top, m2 = ctx->arena2.top;
      ctx->arena.peak = m1;
      ctx->arena2.peak = m2;
      ZJAI_TRY(run_group(ctx, ny, nuv, lat_y, lat_uv, lh, lw, tiles, pics, g, out_h, out_w, sv, sh,
                         rec_y, rec_u, rec_v, cancel, flops, qbytes, qmax, s1, s2, &ctx->arena,
                         &ctx->arena2, ctx->ev_fork));
      ctx->group_need[key(g)] = {ctx->arena.peak - m1, ctx->arena2.peak - m2};
    }
    ZJAI_TRY(cuda_check(cudaEventRecord(ctx->ev_join, s2), "event"));
    return cuda_check(cudaStreamWaitEvent(s1, ctx->ev_join, 0), "event wait");
  }
  const size_t ng = groups.size();
  // events: fork, then per group one for its gather and one each for its two chains' ends
  ZJAI_TRY(group_pool(ctx, 2 * ng, 1 + 3 * ng));
  cudaEvent_t fork = ctx->group_events[0];
  ZJAI_TRY(cuda_check(cudaEventRecord(fork, ctx->stream), "event"));
  std::vector<Arena> ay(ng), ac(ng);
  for (size_t i = 0; i < ng; ++i) {
    const auto& need = ctx->group_need[key(groups[i])];
    auto carve = [](Arena& main, size_t bytes, Arena* sub) {
      const size_t start = (main.top + 255) & ~size_t(255);
      sub->base = main.base + start;
      sub->cap = bytes + 768;
      sub->top = sub->peak = 0;
      main.top = start + sub->cap;
      main.peak = std::max(main.peak, main.top);
    };
    carve(ctx->arena, need.first, &ay[i]);
    carve(ctx->arena2, need.second, &ac[i]);
  }
  for (size_t i = 0; i < ng; ++i) {
    if (cancel && *cancel) return fail(ZJAI_CANCELLED, "stopped: cancelled by the caller");
    cudaStream_t sy = ctx->group_streams[2 * i], sc = ctx->group_streams[2 * i + 1];
    ZJAI_TRY(cuda_check(cudaStreamWaitEvent(sy, fork, 0), "event wait"));
    ZJAI_TRY(cuda_check(cudaStreamWaitEvent(sc, fork, 0), "event wait"));
    ZJAI_TRY(run_group(ctx, ny, nuv, lat_y, lat_uv, lh, lw, tiles, pics, groups[i], out_h, out_w, sv,
                       sh, rec_y, rec_u, rec_v, cancel, flops, qbytes, qmax, sy, sc, &ay[i],
                       &ac[i], ctx->group_events[1 + 3 * i]));
  }
  // join every chain back into the context's stream
  for (size_t i = 0; i < ng; ++i) {
    for (int k = 0; k < 2; ++k) {
      cudaEvent_t e = ctx->group_events[2 + 3 * i + k];
      ZJAI_TRY(cuda_check(cudaEventRecord(e, ctx->group_streams[2 * i + k]), "event"));
      ZJAI_TRY(cuda_check(cudaStreamWaitEvent(ctx->stream, e, 0), "event wait"));
    }
  }
  return ZJAI_OK;
}

}  // namespace zjai

extern "C" {

int zjai_net_create(zjai_ctx* ctx, int kind, int op, const zjai_param* params, int nparams,
                    zjai_net** out) {
  if (!out) return fail(ZJAI_INVALID_ARGUMENT, "null output handle");
  *out = nullptr;
  ZJAI_TRY(ctx_enter(ctx));
  if ((kind < ZJAI_SYN_Y || kind > ZJAI_ANA_UV) && kind != ZJAI_LATENT && kind != ZJAI_ICCI)
    return fail(ZJAI_INVALID_ARGUMENT, "unknown network kind");
  Net* n = nullptr;
  ZJAI_TRY(load_network(ctx, kind, op, params, nparams, &n));
  // the C handle is the same object
  *out = reinterpret_cast<zjai_net*>(n);
  return ZJAI_OK;
}

int zjai_net_destroy(zjai_net* net) {
  if (!net) return ZJAI_OK;
  cudaSetDevice(net->ctx->device);
  cudaDeviceSynchronize();
  net->ctx->clear_graphs();  // graphs may hold this network's weights
  delete reinterpret_cast<Net*>(net);
  return ZJAI_OK;
}

int zjai_synth_out_size(int kind, int op, int h, int w, int* out_h, int* out_w) {
  if (!out_h || !out_w || h <= 0 || w <= 0) return fail(ZJAI_INVALID_ARGUMENT, "synth_out_size");
  if (kind != ZJAI_SYN_Y && kind != ZJAI_SYN_UV) return fail(ZJAI_INVALID_ARGUMENT, "not a synthesis network");
  synth_out_size(kind, op, h, w, out_h, out_w);
  return ZJAI_OK;
}

int zjai_synthesis_primary(zjai_net* net, const float* y_hat, int lh, int lw, int h, int w,
                           float* out, int mem) {
  ZJAI_TRY(net_enter(net));
  Net* n = reinterpret_cast<Net*>(net);
  Ctx* ctx = n->ctx;
  if (n->kind != ZJAI_SYN_Y) return fail(ZJAI_INVALID_ARGUMENT, "not a primary synthesis network");
  if (!y_hat || !out || lh <= 0 || lw <= 0 || h <= 0 || w <= 0)
    return fail(ZJAI_INVALID_ARGUMENT, "synthesis_primary: bad arguments");
  ArenaScope scope(ctx);
  int oh, ow;
  synth_out_size(ZJAI_SYN_Y, n->op, h, w, &oh, &ow);
  const float* dy;
  ZJAI_TRY(stage_in(ctx, y_hat, (size_t)160 * lh * lw, mem, &dy));
  int* d_origin;
  ZJAI_TRY(upload_ints(ctx, &ctx->arena, {0, 0, 0}, ctx->stream, &d_origin));
  TView y;
  ZJAI_TRY(alloc_tensor(ctx, 1, lh, lw, 160, &y));
  launch_gather_latent(dy, 160, lh, lw, d_origin, y, ctx->stream);
  float* dout;
  ZJAI_TRY(stage_out_alloc(ctx, out, (size_t)oh * ow, mem, &dout));
  Runner r = make_runner(ctx, n, &ctx->arena, ctx->stream, 1, nullptr);
  FinalOut fo;
  fo.plane0 = dout;
  fo.row = ow;
  fo.img = (long long)oh * ow;
  int st = r.primary(y, h, w, fo);
  if (st != ZJAI_OK) return settle(ctx, st);
  ZJAI_TRY(stage_out_finish(ctx, out, dout, (size_t)oh * ow, mem));
  return finish_call(ctx, mem);
}

int zjai_synthesis_secondary(zjai_net* net, const float* y_hat_luma, int llh, int llw,
                             const float* y_hat_chroma, int lh, int lw, int h, int w, float* out,
                             int mem) {
  ZJAI_TRY(net_enter(net));
  Net* n = reinterpret_cast<Net*>(net);
  Ctx* ctx = n->ctx;
  if (n->kind != ZJAI_SYN_UV) return fail(ZJAI_INVALID_ARGUMENT, "not a secondary synthesis network");
  if (!y_hat_luma || !y_hat_chroma || !out || lh <= 0 || lw <= 0 || h <= 0 || w <= 0)
    return fail(ZJAI_INVALID_ARGUMENT, "synthesis_secondary: bad arguments");
  if (lh > llh || lw > llw)
    return fail(ZJAI_INVALID_ARGUMENT, "chroma latent larger than the luma latent");
  ArenaScope scope(ctx);
  int oh, ow;
  synth_out_size(ZJAI_SYN_UV, n->op, h, w, &oh, &ow);
  const float *dl, *dc;
  ZJAI_TRY(stage_in(ctx, y_hat_luma, (size_t)160 * llh * llw, mem, &dl));
  ZJAI_TRY(stage_in(ctx, y_hat_chroma, (size_t)96 * lh * lw, mem, &dc));
  int* d_origin;
  ZJAI_TRY(upload_ints(ctx, &ctx->arena, {0, 0, 0}, ctx->stream, &d_origin));
  TView cat, x144;
  ZJAI_TRY(alloc_tensor(ctx, 1, lh, lw, 256, &cat));
  ZJAI_TRY(alloc_tensor(ctx, 1, lh, lw, 144, &x144));
  launch_gather_latent(dl, 160, llh, llw, d_origin, cat.channels(0, 160), ctx->stream);
  launch_gather_latent(dc, 96, lh, lw, d_origin, cat.channels(160, 96), ctx->stream);
  launch_gather_latent(dc, 96, lh, lw, d_origin, x144.channels(48, 96), ctx->stream);
  float* dout;
  ZJAI_TRY(stage_out_alloc(ctx, out, (size_t)2 * oh * ow, mem, &dout));
  Runner r = make_runner(ctx, n, &ctx->arena, ctx->stream, 1, nullptr);
  FinalOut fo;
  fo.plane0 = dout;
  fo.plane_stride = (long long)oh * ow;
  fo.row = ow;
  fo.img = 2LL * oh * ow;
  int st = r.secondary(cat, x144, h, w, fo);
  if (st != ZJAI_OK) return settle(ctx, st);
  ZJAI_TRY(stage_out_finish(ctx, out, dout, (size_t)2 * oh * ow, mem));
  return finish_call(ctx, mem);
}

static int analysis_entry(zjai_net* net, int kind, int cin, int cout, int down, const float* x,
                          int h, int w, float* out, int mem) {
  ZJAI_TRY(net_enter(net));
  Net* n = reinterpret_cast<Net*>(net);
  Ctx* ctx = n->ctx;
  if (n->kind != kind) return fail(ZJAI_INVALID_ARGUMENT, "wrong analysis network kind");
  if (!x || !out || h <= 0 || w <= 0) return fail(ZJAI_INVALID_ARGUMENT, "analysis: bad arguments");
  ArenaScope scope(ctx);
  const float* dx;
  ZJAI_TRY(stage_in(ctx, x, (size_t)cin * h * w, mem, &dx));
  TView t;
  if (cin == 1 && n->convs.count("conv1#im2col")) {
    // luma: the first layer's taps per output pixel, for its 1x1 form
    ZJAI_TRY(alloc_tensor(ctx, 1, cdiv(h, 2), cdiv(w, 2), 9, &t));
    launch_normalize_im2col(dx, h, w, 0, 0, h, w, t, ctx->stream);
  } else {
    ZJAI_TRY(alloc_tensor(ctx, 1, 2 * cdiv(h, 2), 2 * cdiv(w, 2), cin, &t, true));
    launch_normalize_pad(dx, cin, h, w, t, ctx->stream);
  }
  const size_t nout = (size_t)cout * cdiv(h, down) * cdiv(w, down);
  float* dout;
  ZJAI_TRY(stage_out_alloc(ctx, out, nout, mem, &dout));
  Runner r = make_runner(ctx, n, &ctx->arena, ctx->stream, 1, nullptr);
  int st = r.analysis(t, h, w, dout);
  if (st != ZJAI_OK) return settle(ctx, st);
  ZJAI_TRY(stage_out_finish(ctx, out, dout, nout, mem));
  return finish_call(ctx, mem);
}

int zjai_analysis_primary(zjai_net* net, const float* x, int h, int w, float* out, int mem) {
  return analysis_entry(net, ZJAI_ANA_Y, 1, 160, 16, x, h, w, out, mem);
}

int zjai_analysis_secondary(zjai_net* net, const float* x, int h, int w, float* out, int mem) {
  return analysis_entry(net, ZJAI_ANA_UV, 12, 96, 8, x, h, w, out, mem);
}

int zjai_preprocess_rgb(zjai_ctx* ctx, const uint8_t* rgb, int h, int w, float* luma,
                        float* chroma, int mem) {
  ZJAI_TRY(ctx_enter(ctx));
  if (!rgb || !luma || !chroma || h <= 0 || w <= 0)
    return fail(ZJAI_INVALID_ARGUMENT, "preprocess_rgb: bad arguments");
  if (mem != ZJAI_MEM_HOST && mem != ZJAI_MEM_DEVICE)
    return fail(ZJAI_INVALID_ARGUMENT, "mem must be HOST or DEVICE");
  ArenaScope scope(ctx);
  const size_t nrgb = (size_t)h * w * 3, nl = (size_t)h * w;
  const size_t nc = (size_t)12 * ((h + 1) / 2) * ((w + 1) / 2);
  const uint8_t* drgb = rgb;
  if (mem == ZJAI_MEM_DEVICE) ZJAI_TRY(check_device_buffer(ctx, rgb, "RGB input"));
  if (mem == ZJAI_MEM_HOST) {
    uint8_t* d = static_cast<uint8_t*>(ctx->arena.alloc(nrgb));
    if (!d) return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (RGB staging)");
    ZJAI_TRY(cuda_check(cudaMemcpyAsync(d, rgb, nrgb, cudaMemcpyHostToDevice, ctx->stream), "H2D"));
    drgb = d;
  }
  float *dl, *dc;
  ZJAI_TRY(stage_out_alloc(ctx, luma, nl, mem, &dl));
  ZJAI_TRY(stage_out_alloc(ctx, chroma, nc, mem, &dc));
  launch_preprocess_rgb(drgb, 1, h, w, dl, dc, ctx->stream);
  ctx->launches++;
  ZJAI_TRY(stage_out_finish(ctx, luma, dl, nl, mem));
  ZJAI_TRY(stage_out_finish(ctx, chroma, dc, nc, mem));
  return finish_call(ctx, mem);
}

// Analysis of one component of n same-size pictures: plane [n][c][H][W] (planar f32 in
// [0, 255]) -> latent [n][cout][LH][LW], tile by tile above the tiling threshold, each tile of
// all n pictures one batch.
static int analyze_component(Ctx* ctx, Net* net, int ccs, int n, const float* plane, int c, int H,
                             int W, float* out) {
  const int d = ccs ? 8 : 16, cout = ccs ? 96 : 160;
  const int LH = cdiv(H, d), LW = cdiv(W, d);
  std::vector<std::array<int, 14>> tiles;
  ZJAI_TRY(analysis_tiles(ccs, H, W, LH, LW, &tiles));
  const bool whole = tiles.size() == 1;
  for (const auto& t : tiles) {
    ArenaMark mark(&ctx->arena);
    const int tx = t[0], ty = t[1], tw = t[2], th = t[3], tlw = t[6], tlh = t[7];
    TView x;
    if (c == 1 && net->convs.count("conv1#im2col")) {
      // luma: the first layer's taps per output pixel, for its 1x1 form
      ZJAI_TRY(alloc_tensor(ctx, n, cdiv(th, 2), cdiv(tw, 2), 9, &x));
      launch_normalize_im2col(plane, H, W, ty, tx, th, tw, x, ctx->stream);
    } else {
      ZJAI_TRY(alloc_tensor(ctx, n, 2 * cdiv(th, 2), 2 * cdiv(tw, 2), c, &x, true));
      launch_normalize_pad_window(plane, c, H, W, ty, tx, th, tw, x, ctx->stream);
    }
    ctx->launches++;
    float* tout = out;
    if (!whole) {
      tout = static_cast<float*>(ctx->arena.alloc((size_t)n * cout * tlh * tlw * sizeof(float)));
      if (!tout) return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (analysis tile)");
    }
    Runner r = make_runner(ctx, net, &ctx->arena, ctx->stream, n, nullptr);
    ZJAI_TRY(r.analysis(x, th, tw, tout));
    if (!whole) {
      launch_copy_core(tout, n, cout, tlh, tlw, t[13], t[12], t[11], t[10], out, LH, LW, t[9],
                       t[8], ctx->stream);
      ctx->launches++;
    }
  }
  return ZJAI_OK;
}

int zjai_analyze_rgb(zjai_ctx* ctx, zjai_net* net_y, zjai_net* net_uv, int n, const uint8_t* rgb,
                     int h, int w, float* lat_y, float* lat_uv, int mem) {
  ZJAI_TRY(ctx_enter(ctx));
  Net* ny = reinterpret_cast<Net*>(net_y);
  Net* nuv = reinterpret_cast<Net*>(net_uv);
  if (!ny || !nuv || ny->kind != ZJAI_ANA_Y || nuv->kind != ZJAI_ANA_UV || ny->op != nuv->op)
    return fail(ZJAI_INVALID_ARGUMENT, "analyze_rgb: needs an ANA_Y and an ANA_UV network of one op");
  if (!rgb || !lat_y || !lat_uv || n <= 0 || h <= 0 || w <= 0)
    return fail(ZJAI_INVALID_ARGUMENT, "analyze_rgb: bad arguments");
  if (mem != ZJAI_MEM_HOST && mem != ZJAI_MEM_DEVICE)
    return fail(ZJAI_INVALID_ARGUMENT, "mem must be HOST or DEVICE");
  ArenaScope scope(ctx);
  const int ch = (h + 1) / 2, cw = (w + 1) / 2;
  const size_t nrgb = (size_t)n * h * w * 3;
  const uint8_t* drgb = rgb;
  if (mem == ZJAI_MEM_DEVICE) ZJAI_TRY(check_device_buffer(ctx, rgb, "RGB input"));
  if (mem == ZJAI_MEM_HOST) {
    uint8_t* d = static_cast<uint8_t*>(ctx->arena.alloc(nrgb));
    if (!d) return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (RGB staging)");
    ZJAI_TRY(cuda_check(cudaMemcpyAsync(d, rgb, nrgb, cudaMemcpyHostToDevice, ctx->stream), "H2D"));
    drgb = d;
  }
  float* dl = static_cast<float*>(ctx->arena.alloc((size_t)n * h * w * sizeof(float)));
  float* dc = static_cast<float*>(ctx->arena.alloc((size_t)n * 12 * ch * cw * sizeof(float)));
  if (!dl || !dc) return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (analysis inputs)");
  launch_preprocess_rgb(drgb, n, h, w, dl, dc, ctx->stream);
  ctx->launches++;
  const size_t ny_out = (size_t)n * 160 * cdiv(h, 16) * cdiv(w, 16);
  const size_t nuv_out = (size_t)n * 96 * cdiv(ch, 8) * cdiv(cw, 8);
  float *oy, *ouv;
  ZJAI_TRY(stage_out_alloc(ctx, lat_y, ny_out, mem, &oy));
  ZJAI_TRY(stage_out_alloc(ctx, lat_uv, nuv_out, mem, &ouv));
  int st = analyze_component(ctx, ny, 0, n, dl, 1, h, w, oy);
  if (st == ZJAI_OK) st = analyze_component(ctx, nuv, 1, n, dc, 12, ch, cw, ouv);
  if (st != ZJAI_OK) return settle(ctx, st);
  ZJAI_TRY(stage_out_finish(ctx, lat_y, oy, ny_out, mem));
  ZJAI_TRY(stage_out_finish(ctx, lat_uv, ouv, nuv_out, mem));
  return finish_call(ctx, mem);
}

int zjai_stage_create(zjai_ctx* ctx, int shuffle, int act, int res_act, const zjai_param* params,
                      int nparams, zjai_net** out) {
  if (!out) return fail(ZJAI_INVALID_ARGUMENT, "null output handle");
  *out = nullptr;
  ZJAI_TRY(ctx_enter(ctx));
  Net* n = nullptr;
  ZJAI_TRY(load_stage(ctx, shuffle, act, res_act, params, nparams, &n));
  *out = reinterpret_cast<zjai_net*>(n);
  return ZJAI_OK;
}

int zjai_stage_forward(zjai_net* net, const float* x, int c, int h, int w, float* out, int mem) {
  ZJAI_TRY(net_enter(net));
  Net* n = reinterpret_cast<Net*>(net);
  Ctx* ctx = n->ctx;
  if (n->kind != kStageKind) return fail(ZJAI_INVALID_ARGUMENT, "not a conv stage");
  if (!x || !out || h <= 0 || w <= 0 || c != n->st_cin)
    return fail(ZJAI_INVALID_ARGUMENT, "stage: input must be [" + std::to_string(n->st_cin) +
                                           "][h][w] and an output given");
  ArenaScope scope(ctx);
  const float* dx;
  ZJAI_TRY(stage_in(ctx, x, (size_t)c * h * w, mem, &dx));
  TView t;
  ZJAI_TRY(planar_to_tensor(ctx, dx, c, h, w, &t));
  const size_t nout = (size_t)n->st_cout * h * n->st_shuffle * w * n->st_shuffle;
  float* dout;
  ZJAI_TRY(stage_out_alloc(ctx, out, nout, mem, &dout));
  Runner r = make_runner(ctx, n, &ctx->arena, ctx->stream, 1, nullptr);
  int st = r.stage(t, dout);
  if (st != ZJAI_OK) return settle(ctx, st);
  ZJAI_TRY(stage_out_finish(ctx, out, dout, nout, mem));
  return finish_call(ctx, mem);
}

// ---- latent-domain networks -----------------------------------------------------------------

static int latent_net(zjai_net* net, Net** out) {
  ZJAI_TRY(net_enter(net));
  Net* n = reinterpret_cast<Net*>(net);
  if (n->kind != ZJAI_LATENT) return fail(ZJAI_INVALID_ARGUMENT, "not a latent network");
  *out = n;
  return ZJAI_OK;
}

int zjai_hyper_decode(zjai_net* net, const float* z_hat, int hz, int wz, int out_h, int out_w,
                      float* psi, int mem) {
  Net* n;
  ZJAI_TRY(latent_net(net, &n));
  Ctx* ctx = n->ctx;
  if (!z_hat || !psi || hz <= 0 || wz <= 0 || out_h <= 0 || out_w <= 0)
    return fail(ZJAI_INVALID_ARGUMENT, "hyper_decode: bad arguments");
  const int c = n->lat_c;
  ArenaScope scope(ctx);
  const float* dz;
  ZJAI_TRY(stage_in(ctx, z_hat, (size_t)c * hz * wz, mem, &dz));
  TView t;
  ZJAI_TRY(planar_to_tensor(ctx, dz, c, hz, wz, &t));
  const size_t npsi = (size_t)4 * c * out_h * out_w;
  float* dpsi;
  ZJAI_TRY(stage_out_alloc(ctx, psi, npsi, mem, &dpsi));
  Runner r = make_runner(ctx, n, &ctx->arena, ctx->stream, 1, nullptr);
  const int st = r.hyper(t, out_h, out_w, dpsi);
  if (st != ZJAI_OK) return settle(ctx, st);
  ZJAI_TRY(stage_out_finish(ctx, psi, dpsi, npsi, mem));
  return finish_call(ctx, mem);
}

int zjai_context_decompress(zjai_net* net, const float* residual, int h, int w, const float* psi,
                            float* y_hat, int mem) {
  Net* n;
  ZJAI_TRY(latent_net(net, &n));
  Ctx* ctx = n->ctx;
  if (!residual || !psi || !y_hat || h <= 0 || w <= 0)
    return fail(ZJAI_INVALID_ARGUMENT, "context_decompress: bad arguments");
  const int c = n->lat_c;
  ArenaScope scope(ctx);
  const size_t ny = (size_t)c * h * w, npsi = (size_t)4 * c * cdiv(h, 2) * cdiv(w, 2);
  const float *dres, *dpsi;
  ZJAI_TRY(stage_in(ctx, residual, ny, mem, &dres));
  ZJAI_TRY(stage_in(ctx, psi, npsi, mem, &dpsi));
  float* dy;
  ZJAI_TRY(stage_out_alloc(ctx, y_hat, ny, mem, &dy));
  Runner r = make_runner(ctx, n, &ctx->arena, ctx->stream, 1, nullptr);
  const int st = r.latent(dpsi, dres, h, w, dy);
  if (st != ZJAI_OK) return settle(ctx, st);
  ZJAI_TRY(stage_out_finish(ctx, y_hat, dy, ny, mem));
  return finish_call(ctx, mem);
}

int zjai_reconstruct_latent(zjai_net* net, const float* z_hat, int hz, int wz,
                            const float* residual, int h, int w, float* psi, float* y_hat,
                            int mem) {
  Net* n;
  ZJAI_TRY(latent_net(net, &n));
  Ctx* ctx = n->ctx;
  if (!z_hat || !residual || !y_hat || hz <= 0 || wz <= 0 || h <= 0 || w <= 0)
    return fail(ZJAI_INVALID_ARGUMENT, "reconstruct_latent: bad arguments");
  const int c = n->lat_c, hh = cdiv(h, 2), hw = cdiv(w, 2);
  ArenaScope scope(ctx);
  const size_t ny = (size_t)c * h * w, npsi = (size_t)4 * c * hh * hw;
  const float *dz, *dres;
  ZJAI_TRY(stage_in(ctx, z_hat, (size_t)c * hz * wz, mem, &dz));
  ZJAI_TRY(stage_in(ctx, residual, ny, mem, &dres));
  TView t;
  ZJAI_TRY(planar_to_tensor(ctx, dz, c, hz, wz, &t));
  float* dpsi = nullptr;
  if (psi) {
    ZJAI_TRY(stage_out_alloc(ctx, psi, npsi, mem, &dpsi));
  } else {
    dpsi = static_cast<float*>(ctx->arena.alloc(npsi * sizeof(float)));
    if (!dpsi) return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (psi)");
  }
  float* dy;
  ZJAI_TRY(stage_out_alloc(ctx, y_hat, ny, mem, &dy));
  Runner r = make_runner(ctx, n, &ctx->arena, ctx->stream, 1, nullptr);
  int st = r.hyper(t, hh, hw, dpsi);
  if (st == ZJAI_OK) st = r.latent(dpsi, dres, h, w, dy);
  if (st != ZJAI_OK) return settle(ctx, st);
  if (psi) ZJAI_TRY(stage_out_finish(ctx, psi, dpsi, npsi, mem));
  ZJAI_TRY(stage_out_finish(ctx, y_hat, dy, ny, mem));
  return finish_call(ctx, mem);
}

int zjai_synthesis_tiles(int height, int width, int latent_h, int latent_w, int tile_size,
                         int overlap, zjai_tile* tiles, int max_tiles, int* count) {
  std::vector<zjai_tile> v;
  ZJAI_TRY(synthesis_tiles(height, width, latent_h, latent_w, tile_size, overlap, &v));
  if (count) *count = (int)v.size();
  for (int i = 0; i < (int)v.size() && i < max_tiles && tiles; ++i) tiles[i] = v[i];
  return ZJAI_OK;
}

}  // extern "C"

// zjai_synthesize_tiles with f32 planes (bit_depth 0) or quantized sample planes (8: uint8,
// else uint16), written by the final layers' epilogue; `npic` pictures of one size (latents
// [npic][C][lh][lw], planes [npic][h][w]) each cut into the same `tiles`.
static int synthesize_tiles_entry(zjai_ctx* ctx, zjai_net* net_y, zjai_net* net_uv,
                                  const float* y_hat_y, const float* y_hat_uv, int lh, int lw,
                                  const zjai_tile* tiles, int ntiles, int out_h, int out_w,
                                  int sv, int sh, int bit_depth, void* rec_y, void* rec_u,
                                  void* rec_v, int mem, const volatile int* cancel,
                                  int npic = 1) {
  ZJAI_TRY(ctx_enter(ctx));
  if (!y_hat_y || !y_hat_uv || !rec_y || !rec_u || !rec_v || (ntiles > 0 && !tiles) ||
      lh <= 0 || lw <= 0 || out_h <= 0 || out_w <= 0 || npic <= 0)
    return fail(ZJAI_INVALID_ARGUMENT, "synthesize: bad arguments");
  if (sv <= 0 || sh <= 0) return fail(ZJAI_INVALID_DATA, "chroma subsampling factor");
  if (bit_depth < 0 || bit_depth > 16 || (bit_depth > 0 && bit_depth < 8))
    return fail(ZJAI_INVALID_ARGUMENT, "synthesize: bit depth must be 8..16 (or 0 for f32)");
  const size_t es = bit_depth == 0 ? sizeof(float) : bit_depth == 8 ? 1 : 2;  // sample bytes
  const int ch = cdiv(out_h, sv), cw = cdiv(out_w, sh);
  const size_t ny = (size_t)out_h * out_w, nc = (size_t)ch * cw;
  if ((double)ny * npic > 2147483647.0)
    return fail(ZJAI_LIMIT_EXCEEDED, "synthesize: more than 2^31 output samples per call");
  // CUDA graph of a repeated device call (zjai_ctx_set_graphs): the first call with these
  // arguments runs eagerly, the second is captured and every later one replays the graph
  GraphEntry* ge = nullptr;
  if (ctx->graphs && mem == ZJAI_MEM_DEVICE && !cancel && !ctx->profiling && ctx->probes.empty()) {
    std::string key;
    auto put = [&](const void* p, size_t n) { key.append(static_cast<const char*>(p), n); };
    const uint64_t ids[2] = {net_y ? net_y->uid : 0, net_uv ? net_uv->uid : 0};
    const void* ptrs[5] = {y_hat_y, y_hat_uv, rec_y, rec_u, rec_v};
    const long long vals[10] = {lh, lw, ntiles, out_h, out_w, sv, sh, bit_depth, npic,
                                ctx->wait_cycles};
    put(ids, sizeof ids);
    put(ptrs, sizeof ptrs);
    put(vals, sizeof vals);
    const bool clamp = ctx->clamp_output;
    put(&clamp, sizeof clamp);
    put(tiles, sizeof(zjai_tile) * (size_t)ntiles);
    ge = &ctx->graph_cache[key];
    if (ge->exec) {
      ZJAI_TRY(cuda_check(cudaGraphLaunch(ge->exec, ctx->stream), "graph launch"));
      ctx->launches += ge->launches;
      return finish_call(ctx, mem);
    }
    if (ge->calls++ < 1) ge = nullptr;  // first call: eager
  }
  if (ge) {
    // capture this call; a call that fails to capture runs eagerly (and is never captured again)
    std::vector<void*> pins;
    const long long l0 = ctx->launches;
    ZJAI_TRY(cuda_check(cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeRelaxed),
                        "begin capture"));
    ctx->capture_pins = &pins;
    ctx->graphs = false;
    const int st = synthesize_tiles_entry(ctx, net_y, net_uv, y_hat_y, y_hat_uv, lh, lw, tiles,
                                          ntiles, out_h, out_w, sv, sh, bit_depth, rec_y, rec_u,
                                          rec_v, mem, cancel, npic);
    ctx->graphs = true;
    ctx->capture_pins = nullptr;
    cudaGraph_t g = nullptr;
    const cudaError_t ce = cudaStreamEndCapture(ctx->stream, &g);
    cudaGraphExec_t exec = nullptr;
    if (st == ZJAI_OK && ce == cudaSuccess && g &&
        cudaGraphInstantiate(&exec, g, cudaGraphInstantiateFlagUseNodePriority) == cudaSuccess) {
      cudaGraphDestroy(g);
      ge->exec = exec;
      ge->pins.swap(pins);
      ge->launches = ctx->launches - l0;
      ctx->launches = l0 + ge->launches;
      ZJAI_TRY(cuda_check(cudaGraphLaunch(exec, ctx->stream), "graph launch"));
      return finish_call(ctx, mem);
    }
    if (g) cudaGraphDestroy(g);
    for (void* p : pins) cudaFreeHost(p);
    cudaGetLastError();
    ge->calls = -(1 << 30);
    ctx->launches = l0;
    ctx->graphs = false;
    const int st2 = synthesize_tiles_entry(ctx, net_y, net_uv, y_hat_y, y_hat_uv, lh, lw, tiles,
                                           ntiles, out_h, out_w, sv, sh, bit_depth, rec_y, rec_u,
                                           rec_v, mem, cancel, npic);
    ctx->graphs = true;
    return st2;
  }
  ArenaScope scope(ctx);
  const size_t m2 = ctx->arena2.mark();
  struct Rel {
    Arena* a;
    size_t m;
    ~Rel() { a->release(m); }
  } rel{&ctx->arena2, m2};
  const float *dy, *duv;
  ZJAI_TRY(stage_in(ctx, y_hat_y, (size_t)npic * 160 * lh * lw, mem, &dy));
  ZJAI_TRY(stage_in(ctx, y_hat_uv, (size_t)npic * 96 * lh * lw, mem, &duv));
  char *oy = static_cast<char*>(rec_y), *ou = static_cast<char*>(rec_u),
       *ov = static_cast<char*>(rec_v);
  const size_t all = (size_t)npic * (ny + 2 * nc) * es;
  if (mem == ZJAI_MEM_DEVICE)
    for (const void* pl : {rec_y, rec_u, rec_v}) ZJAI_TRY(check_device_buffer(ctx, pl, "output plane"));
  if (mem == ZJAI_MEM_HOST) {
    oy = static_cast<char*>(ctx->arena.alloc(all));
    if (!oy) return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (output planes)");
    ou = oy + npic * ny * es;
    ov = ou + npic * nc * es;
    ZJAI_TRY(cuda_check(cudaMemsetAsync(oy, 0, all, ctx->stream), "memset"));
  }
  std::vector<zjai_tile> tv;
  TilePictures pics;
  for (int p = 0; p < npic; ++p)
    for (int i = 0; i < ntiles; ++i) {
      tv.push_back(tiles[i]);
      if (npic > 1) pics.pic.push_back(p);
    }
  pics.plane_y = (long long)ny;
  pics.plane_uv = (long long)nc;
  int st = synthesize_tiles_dev(ctx, reinterpret_cast<Net*>(net_y), reinterpret_cast<Net*>(net_uv),
                                dy, duv, lh, lw, tv, out_h, out_w, sv, sh,
                                reinterpret_cast<float*>(oy), reinterpret_cast<float*>(ou),
                                reinterpret_cast<float*>(ov), cancel, nullptr, bit_depth, pics);
  if (st != ZJAI_OK) return settle(ctx, st);
  if (mem == ZJAI_MEM_HOST) {
    ZJAI_TRY(cuda_check(cudaMemcpyAsync(rec_y, oy, npic * ny * es, cudaMemcpyDeviceToHost, ctx->stream), "D2H"));
    ZJAI_TRY(cuda_check(cudaMemcpyAsync(rec_u, ou, npic * nc * es, cudaMemcpyDeviceToHost, ctx->stream), "D2H"));
    ZJAI_TRY(cuda_check(cudaMemcpyAsync(rec_v, ov, npic * nc * es, cudaMemcpyDeviceToHost, ctx->stream), "D2H"));
  }
  return finish_call(ctx, mem);
}

extern "C" {

int zjai_synthesize_tiles(zjai_ctx* ctx, zjai_net* net_y, zjai_net* net_uv, const float* y_hat_y,
                          const float* y_hat_uv, int lh, int lw, const zjai_tile* tiles,
                          int ntiles, int out_h, int out_w, int sv, int sh, float* rec_y,
                          float* rec_u, float* rec_v, int mem, const volatile int* cancel) {
  return synthesize_tiles_entry(ctx, net_y, net_uv, y_hat_y, y_hat_uv, lh, lw, tiles, ntiles,
                                out_h, out_w, sv, sh, 0, rec_y, rec_u, rec_v, mem, cancel);
}

int zjai_synthesize_tiles_q(zjai_ctx* ctx, zjai_net* net_y, zjai_net* net_uv,
                            const float* y_hat_y, const float* y_hat_uv, int lh, int lw,
                            const zjai_tile* tiles, int ntiles, int out_h, int out_w, int sv,
                            int sh, int bit_depth, void* rec_y, void* rec_u, void* rec_v,
                            int mem, const volatile int* cancel) {
  if (bit_depth < 8) return fail(ZJAI_INVALID_ARGUMENT, "synthesize: bit depth must be 8..16");
  return synthesize_tiles_entry(ctx, net_y, net_uv, y_hat_y, y_hat_uv, lh, lw, tiles, ntiles,
                                out_h, out_w, sv, sh, bit_depth, rec_y, rec_u, rec_v, mem,
                                cancel);
}

int zjai_synthesize(zjai_ctx* ctx, zjai_net* net_y, zjai_net* net_uv, const float* y_hat_y,
                    const float* y_hat_uv, int lh, int lw, int height, int width, int out_h,
                    int out_w, int tile_size, int overlap, int sv, int sh, float* rec_y,
                    float* rec_u, float* rec_v, int mem, const volatile int* cancel) {
  std::vector<zjai_tile> v;
  ZJAI_TRY(synthesis_tiles(height, width, lh, lw, tile_size, overlap, &v));
  return zjai_synthesize_tiles(ctx, net_y, net_uv, y_hat_y, y_hat_uv, lh, lw, v.data(),
                               (int)v.size(), out_h, out_w, sv, sh, rec_y, rec_u, rec_v, mem,
                               cancel);
}

// Whole-picture synthesis straight to RGB: the f32 planes stay in the arena and the output
// stage (bicubic 4:2:0 -> 4:4:4, BT.709, rounding) reads them there, so only the RGB samples
// reach the caller (the reference GPU backend's emit_output, gpu/src/kernels.rs:910).
int zjai_synthesize_rgb(zjai_ctx* ctx, zjai_net* net_y, zjai_net* net_uv, const float* y_hat_y,
                        const float* y_hat_uv, int lh, int lw, int height, int width,
                        int tile_size, int overlap, int bit_depth, void* rgb, int mem,
                        const volatile int* cancel) {
  ZJAI_TRY(ctx_enter(ctx));
  if (!y_hat_y || !y_hat_uv || !rgb || lh <= 0 || lw <= 0 || height <= 0 || width <= 0)
    return fail(ZJAI_INVALID_ARGUMENT, "synthesize_rgb: bad arguments");
  if (bit_depth != 8 && bit_depth != 10)
    return fail(ZJAI_INVALID_ARGUMENT, "synthesize_rgb: bit depth must be 8 or 10");
  if (mem != ZJAI_MEM_HOST && mem != ZJAI_MEM_DEVICE)
    return fail(ZJAI_INVALID_ARGUMENT, "mem must be HOST or DEVICE");
  std::vector<zjai_tile> tiles;
  ZJAI_TRY(synthesis_tiles(height, width, lh, lw, tile_size, overlap, &tiles));
  ArenaScope scope(ctx);
  const size_t m2 = ctx->arena2.mark();
  struct Rel {
    Arena* a;
    size_t m;
    ~Rel() { a->release(m); }
  } rel{&ctx->arena2, m2};
  const float *dy, *duv;
  ZJAI_TRY(stage_in(ctx, y_hat_y, (size_t)160 * lh * lw, mem, &dy));
  ZJAI_TRY(stage_in(ctx, y_hat_uv, (size_t)96 * lh * lw, mem, &duv));
  const int ch = cdiv(height, 2), cw = cdiv(width, 2);
  const size_t ny = (size_t)height * width, nc = (size_t)ch * cw;
  float* planes = static_cast<float*>(ctx->arena.alloc((ny + 2 * nc) * sizeof(float)));
  const size_t ob = ny * 3 * (bit_depth == 8 ? 1 : 2);
  if (mem == ZJAI_MEM_DEVICE) ZJAI_TRY(check_device_buffer(ctx, rgb, "RGB output"));
  void* dout = mem == ZJAI_MEM_HOST ? ctx->arena.alloc(ob + 16) : rgb;
  if (!planes || !dout) return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (RGB planes)");
  int st = synthesize_tiles_dev(ctx, reinterpret_cast<Net*>(net_y), reinterpret_cast<Net*>(net_uv),
                                dy, duv, lh, lw, tiles, height, width, 2, 2, planes, planes + ny,
                                planes + ny + nc, cancel, nullptr, 0, TilePictures());
  if (st == ZJAI_OK)
    st = output_yuv_to_rgb(ctx, planes, planes + ny, planes + ny + nc, height, width, ch, cw,
                           bit_depth, dout, ctx->stream);
  if (st != ZJAI_OK) return settle(ctx, st);
  if (mem == ZJAI_MEM_HOST)
    ZJAI_TRY(cuda_check(cudaMemcpyAsync(rgb, dout, ob, cudaMemcpyDeviceToHost, ctx->stream), "D2H"));
  return finish_call(ctx, mem);
}

int zjai_synthesize_batch(zjai_ctx* ctx, zjai_net* net_y, zjai_net* net_uv, int n,
                          const float* y_hat_y, const float* y_hat_uv, int lh, int lw, int height,
                          int width, int out_h, int out_w, int tile_size, int overlap, int sv,
                          int sh, int bit_depth, void* rec_y, void* rec_u, void* rec_v, int mem,
                          const volatile int* cancel) {
  std::vector<zjai_tile> v;
  ZJAI_TRY(synthesis_tiles(height, width, lh, lw, tile_size, overlap, &v));
  return synthesize_tiles_entry(ctx, net_y, net_uv, y_hat_y, y_hat_uv, lh, lw, v.data(),
                                (int)v.size(), out_h, out_w, sv, sh, bit_depth, rec_y, rec_u,
                                rec_v, mem, cancel, n);
}

int zjai_synthesize_q(zjai_ctx* ctx, zjai_net* net_y, zjai_net* net_uv, const float* y_hat_y,
                      const float* y_hat_uv, int lh, int lw, int height, int width, int out_h,
                      int out_w, int tile_size, int overlap, int sv, int sh, int bit_depth,
                      void* rec_y, void* rec_u, void* rec_v, int mem,
                      const volatile int* cancel) {
  std::vector<zjai_tile> v;
  ZJAI_TRY(synthesis_tiles(height, width, lh, lw, tile_size, overlap, &v));
  return zjai_synthesize_tiles_q(ctx, net_y, net_uv, y_hat_y, y_hat_uv, lh, lw, v.data(),
                                 (int)v.size(), out_h, out_w, sv, sh, bit_depth, rec_y, rec_u,
                                 rec_v, mem, cancel);
}

// ---- attention-block layer entries ---------------------------------------------------------

int zjai_layer_norm(zjai_ctx* ctx, const float* x, int c, int h, int w, const float* weight,
                    const float* bias, float* out, int mem) {
  ZJAI_TRY(ctx_enter(ctx));
  if (!x || !weight || !bias || !out || c <= 0 || c > 512 || c % 8 || h <= 0 || w <= 0)
    return fail(ZJAI_INVALID_ARGUMENT, "layer norm: parameter length");
  ArenaScope scope(ctx);
  const float *dx, *dw, *db;
  ZJAI_TRY(stage_in(ctx, x, (size_t)c * h * w, mem, &dx));
  ZJAI_TRY(stage_in(ctx, weight, (size_t)c, mem, &dw));
  ZJAI_TRY(stage_in(ctx, bias, (size_t)c, mem, &db));
  TView t, o;
  ZJAI_TRY(planar_to_tensor(ctx, dx, c, h, w, &t));
  ZJAI_TRY(alloc_tensor(ctx, 1, h, w, c, &o));
  launch_layer_norm(t, o, dw, db, ctx->stream);
  float* dout;
  ZJAI_TRY(stage_out_alloc(ctx, out, (size_t)c * h * w, mem, &dout));
  launch_nhwc_to_planar(o, dout, ctx->stream);
  ZJAI_TRY(stage_out_finish(ctx, out, dout, (size_t)c * h * w, mem));
  return finish_call(ctx, mem);
}

int zjai_channel_attention(zjai_ctx* ctx, const float* qkv, int c3, int h, int w, int heads,
                           const float* temperature, float* out, int mem) {
  ZJAI_TRY(ctx_enter(ctx));
  if (!qkv || !temperature || !out || heads <= 0 || c3 % (3 * heads) || h <= 0 || w <= 0)
    return fail(ZJAI_INVALID_ARGUMENT, "attention: channel / head counts");
  const int dim = c3 / 3, c = dim / heads;
  if (dim % 8 || c % 8 || c > 64 || 2 * dim > 256)
    return fail(ZJAI_UNSUPPORTED, "attention: head sizes must be multiples of 8, at most 64");
  ArenaScope scope(ctx);
  const float *dq, *dt;
  ZJAI_TRY(stage_in(ctx, qkv, (size_t)c3 * h * w, mem, &dq));
  ZJAI_TRY(stage_in(ctx, temperature, (size_t)heads, mem, &dt));
  TView t, o;
  ZJAI_TRY(planar_to_tensor(ctx, dq, c3, h, w, &t));
  ZJAI_TRY(alloc_tensor(ctx, 1, h, w, dim, &o));
  float* scratch =
      static_cast<float*>(ctx->arena.alloc(attention_scratch_floats(1, dim, heads, h * w, ctx->sms) * sizeof(float)));
  if (!scratch) return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (attention)");
  launch_attention(t, o, heads, dt, scratch, ctx->sms, ctx->stream);
  float* dout;
  ZJAI_TRY(stage_out_alloc(ctx, out, (size_t)dim * h * w, mem, &dout));
  launch_nhwc_to_planar(o, dout, ctx->stream);
  ZJAI_TRY(stage_out_finish(ctx, out, dout, (size_t)dim * h * w, mem));
  return finish_call(ctx, mem);
}

static int depthwise_call(zjai_ctx* ctx, const float* x, int c, int h, int w,
                          const float* weight, float* out, int mem, bool gate) {
  ZJAI_TRY(ctx_enter(ctx));
  if (!x || !weight || !out || c <= 0 || c % (gate ? 16 : 8) || h <= 0 || w <= 0)
    return fail(ZJAI_INVALID_ARGUMENT,
                gate ? "depthwise elu gate: bad arguments (channels must be a multiple of 16)"
                     : "depthwise: bad arguments (channels must be a multiple of 8)");
  ArenaScope scope(ctx);
  const float *dx, *dw;
  ZJAI_TRY(stage_in(ctx, x, (size_t)c * h * w, mem, &dx));
  ZJAI_TRY(stage_in(ctx, weight, (size_t)c * 9, mem, &dw));
  const int co = gate ? c / 2 : c;
  TView t, o;
  ZJAI_TRY(planar_to_tensor(ctx, dx, c, h, w, &t));
  ZJAI_TRY(alloc_tensor(ctx, 1, h, w, co, &o));
  ZJAI_TRY(launch_dw3x3(ctx, t, o, dw, gate, ctx->stream));
  float* dout;
  ZJAI_TRY(stage_out_alloc(ctx, out, (size_t)co * h * w, mem, &dout));
  launch_nhwc_to_planar(o, dout, ctx->stream);
  ZJAI_TRY(stage_out_finish(ctx, out, dout, (size_t)co * h * w, mem));
  return finish_call(ctx, mem);
}

int zjai_depthwise3x3(zjai_ctx* ctx, const float* x, int c, int h, int w, const float* weight,
                      float* out, int mem) {
  return depthwise_call(ctx, x, c, h, w, weight, out, mem, false);
}

int zjai_depthwise3x3_elu_gate(zjai_ctx* ctx, const float* x, int c, int h, int w,
                               const float* weight, float* out, int mem) {
  return depthwise_call(ctx, x, c, h, w, weight, out, mem, true);
}

// The feed-forward half of TransformerBlock::forward (attention.rs:346-371) on one picture:
// out = x + W_out . gate(dw3x3(W_in . layer_norm(x))), the LN kernel then the fused FFN kernel.
int zjai_transformer_ffn(zjai_ctx* ctx, const float* x, int c, int h, int w, int hidden,
                         const float* norm_weight, const float* norm_bias, const float* w_in,
                         const float* w_dw, const float* w_out, float* out, int mem) {
  ZJAI_TRY(ctx_enter(ctx));
  if (!x || !norm_weight || !norm_bias || !w_in || !w_dw || !w_out || !out || h <= 0 || w <= 0)
    return fail(ZJAI_INVALID_ARGUMENT, "transformer ffn: bad arguments");
  if (!ffn_fusable(c, hidden))
    return fail(ZJAI_UNSUPPORTED, "transformer ffn: channels must be 64 or 128 and the hidden "
                                  "width a multiple of 64");
  ArenaScope scope(ctx);
  std::vector<float> bi, bd, bo;
  const float *hi, *hd, *ho;
  ZJAI_TRY(fetch_host(w_in, (size_t)2 * hidden * c, mem, &bi, &hi));
  ZJAI_TRY(fetch_host(w_dw, (size_t)2 * hidden * 9, mem, &bd, &hd));
  ZJAI_TRY(fetch_host(w_out, (size_t)c * hidden, mem, &bo, &ho));
  FfnLayer F;
  struct Guard {
    FfnLayer* f;
    ~Guard() {
      cudaDeviceSynchronize();
      free_ffn(f);
    }
  } guard{&F};
  ZJAI_TRY(pack_ffn(ctx, &F, hi, hd, ho, c, hidden));
  const float *dx, *dnw, *dnb;
  ZJAI_TRY(stage_in(ctx, x, (size_t)c * h * w, mem, &dx));
  ZJAI_TRY(stage_in(ctx, norm_weight, (size_t)c, mem, &dnw));
  ZJAI_TRY(stage_in(ctx, norm_bias, (size_t)c, mem, &dnb));
  TView t, ln;
  ZJAI_TRY(planar_to_tensor(ctx, dx, c, h, w, &t));
  ZJAI_TRY(alloc_tensor(ctx, 1, h, w, c, &ln));
  launch_layer_norm(t, ln, dnw, dnb, ctx->stream);
  ZJAI_TRY(run_ffn(ctx, F, ln, t));
  float* dout;
  ZJAI_TRY(stage_out_alloc(ctx, out, (size_t)c * h * w, mem, &dout));
  launch_nhwc_to_planar(t, dout, ctx->stream);
  ZJAI_TRY(stage_out_finish(ctx, out, dout, (size_t)c * h * w, mem));
  return finish_call(ctx, mem);
}

}  // extern "C"
