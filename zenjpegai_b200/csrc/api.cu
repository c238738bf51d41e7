// The C ABI (include/zjai.h): contexts and the nn layer entry points. Network, synthesis and
// output-stage entries live in net.cu / output.cu.
#include <algorithm>
#include <cstring>
#include <vector>

#include "api_common.h"

using namespace zjai;

namespace zjai {

int ctx_enter(zjai_ctx* ctx) {
  if (!ctx) return fail(ZJAI_INVALID_ARGUMENT, "null context");
  return cuda_check(cudaSetDevice(ctx->device), "cudaSetDevice");
}

int ctx_check_status(Ctx* ctx) {
  int err[2] = {0, 0};
  ZJAI_TRY(cuda_check(cudaMemcpyAsync(err, ctx->d_err, sizeof err, cudaMemcpyDeviceToHost,
                                      ctx->stream),
                      "status word read"));
  ZJAI_TRY(cuda_check(cudaStreamSynchronize(ctx->stream), "stream sync"));
  if (err[0] != 0 || err[1] != 0) {
    cudaMemsetAsync(ctx->d_err, 0, sizeof err, ctx->stream);
    cudaStreamSynchronize(ctx->stream);
    if (err[0] != 0)
      return fail(ZJAI_DEVICE_TIMEOUT,
                  "a kernel's bounded wait gave up (device status " + std::to_string(err[0]) + ")");
    return fail(ZJAI_LIMIT_EXCEEDED,
                "an activation left the f16 range (|x| > 65504) in a residual or gate epilogue: "
                "the weights / inputs exceed what the f16 activation storage holds");
  }
  return ZJAI_OK;
}

// End of an entry point: host-memory calls are synchronous (wait, then report the kernels'
// status word); device-memory calls return once their work is enqueued on the stream.
int finish_call(Ctx* ctx, int mem) {
  if (mem == ZJAI_MEM_DEVICE) return cuda_check(cudaGetLastError(), "launch");
  return ctx_check_status(ctx);
}

// Device copy of a caller tensor (host or device) as f32; returns a device pointer.
int check_device_buffer(Ctx* ctx, const void* p, const char* what) {
  if (!p) return fail(ZJAI_INVALID_ARGUMENT, std::string(what) + ": null buffer");
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return fail(ZJAI_INVALID_ARGUMENT, std::string(what) + ": not a CUDA-visible buffer");
  }
  const bool ok = (at.type == cudaMemoryTypeDevice && at.device == ctx->device) ||
                  at.type == cudaMemoryTypeManaged ||
                  (at.type == cudaMemoryTypeHost && at.devicePointer != nullptr);
  if (!ok)
    return fail(ZJAI_INVALID_ARGUMENT,
                std::string(what) + ": ZJAI_MEM_DEVICE needs memory the context's GPU can address");
  return ZJAI_OK;
}

int stage_in(Ctx* ctx, const float* p, size_t n, int mem, const float** out) {
  if (mem == ZJAI_MEM_DEVICE) {
    if (n) ZJAI_TRY(check_device_buffer(ctx, p, "input"));
    *out = p;
    return ZJAI_OK;
  }
  if (mem != ZJAI_MEM_HOST) return fail(ZJAI_INVALID_ARGUMENT, "mem must be HOST or DEVICE");
  float* d = static_cast<float*>(ctx->arena.alloc(n * sizeof(float)));
  if (!d) return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (input staging)");
  ZJAI_TRY(cuda_check(
      cudaMemcpyAsync(d, p, n * sizeof(float), cudaMemcpyHostToDevice, ctx->stream), "H2D"));
  *out = d;
  return ZJAI_OK;
}

int stage_out_alloc(Ctx* ctx, float* p, size_t n, int mem, float** dev) {
  if (mem == ZJAI_MEM_DEVICE) {
    if (n) ZJAI_TRY(check_device_buffer(ctx, p, "output"));
    *dev = p;
    return ZJAI_OK;
  }
  if (mem != ZJAI_MEM_HOST) return fail(ZJAI_INVALID_ARGUMENT, "mem must be HOST or DEVICE");
  *dev = static_cast<float*>(ctx->arena.alloc(n * sizeof(float)));
  if (!*dev) return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (output staging)");
  return ZJAI_OK;
}

int stage_out_finish(Ctx* ctx, float* host, const float* dev, size_t n, int mem) {
  if (mem == ZJAI_MEM_DEVICE) return ZJAI_OK;
  return cuda_check(
      cudaMemcpyAsync(host, dev, n * sizeof(float), cudaMemcpyDeviceToHost, ctx->stream), "D2H");
}

// Host copy of a caller array that the host must read (weights, biases, LN parameters):
// device arrays are copied down, host arrays are used in place.
int fetch_host(const float* p, size_t n, int mem, std::vector<float>* buf, const float** out) {
  if (!p) {
    *out = nullptr;
    return ZJAI_OK;
  }
  if (mem == ZJAI_MEM_HOST) {
    *out = p;
    return ZJAI_OK;
  }
  buf->resize(n);
  ZJAI_TRY(cuda_check(cudaMemcpy(buf->data(), p, n * sizeof(float), cudaMemcpyDeviceToHost),
                      "parameter D2H"));
  *out = buf->data();
  return ZJAI_OK;
}

// Planar f32 [c][h][w] (device) -> fresh zeroed NHWC f16 tensor.
int planar_to_tensor(Ctx* ctx, const float* d, int c, int h, int w, TView* out) {
  ZJAI_TRY(alloc_tensor(ctx, 1, h, w, c, out, true));
  launch_planar_to_nhwc(d, c, h, w, 0, 0, *out, ctx->stream);
  ctx->launches++;
  return cuda_check(cudaGetLastError(), "planar_to_nhwc");
}

}  // namespace zjai

extern "C" {

const char* zjai_version(void) { return "zjai 0.1.0 (sm_100a tcgen05)"; }

const char* zjai_last_error_message(void) { return zjai::last_error_cstr(); }

int zjai_ctx_create(int device, size_t arena_bytes, zjai_ctx** out) {
  if (!out) return fail(ZJAI_INVALID_ARGUMENT, "null output handle");
  *out = nullptr;
  int ndev = 0;
  ZJAI_TRY(cuda_check(cudaGetDeviceCount(&ndev), "cudaGetDeviceCount"));
  if (device < 0 || device >= ndev) return fail(ZJAI_INVALID_ARGUMENT, "no such CUDA device");
  ZJAI_TRY(cuda_check(cudaSetDevice(device), "cudaSetDevice"));
  cudaDeviceProp prop;
  ZJAI_TRY(cuda_check(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties"));
  if (prop.major != 10)
    return fail(ZJAI_UNSUPPORTED, std::string("zjai needs an sm_100 GPU, found ") + prop.name);
  zjai_ctx* c = new zjai_ctx();
  c->device = device;
  c->sms = prop.multiProcessorCount;
  if (arena_bytes == 0) arena_bytes = size_t(8) << 30;
  if (arena_bytes < (size_t(64) << 20)) arena_bytes = size_t(64) << 20;
  int st = ZJAI_OK;
  if ((st = cuda_check(cudaStreamCreateWithFlags(&c->own, cudaStreamNonBlocking), "stream")) ||
      (st = cuda_check(cudaStreamCreateWithFlags(&c->stream2, cudaStreamNonBlocking), "stream")) ||
      (st = cuda_check(cudaEventCreateWithFlags(&c->ev_fork, cudaEventDisableTiming), "event")) ||
      (st = cuda_check(cudaEventCreateWithFlags(&c->ev_join, cudaEventDisableTiming), "event")) ||
      (st = cuda_check(cudaMalloc(&c->arena.base, arena_bytes), "arena cudaMalloc")) ||
      (st = cuda_check(cudaMalloc(&c->d_err, 2 * sizeof(int)), "status cudaMalloc")) ||
      (st = cuda_check(cudaMemset(c->d_err, 0, 2 * sizeof(int)), "status memset")) ||
      (st = cuda_check(cudaDriverGetVersion(&c->driver_version), "driver version"))) {
    zjai_ctx_destroy(c);
    return st;
  }
  // luma / single-stream work gets 5/8 of the arena, the chroma stream the rest
  const size_t first = (arena_bytes / 8 * 5) & ~size_t(255);
  c->arena.cap = first;
  c->arena2.base = c->arena.base + first;
  c->arena2.cap = arena_bytes - first;
  c->stream = c->own;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &c->encode_fn, cudaEnableDefault, &q) !=
          cudaSuccess ||
      q != cudaDriverEntryPointSuccess || !c->encode_fn) {
    zjai_ctx_destroy(c);
    return fail(ZJAI_DEVICE, "cuTensorMapEncodeTiled entry point not available");
  }
  *out = c;
  return ZJAI_OK;
}

int zjai_ctx_destroy(zjai_ctx* ctx) {
  if (!ctx) return ZJAI_OK;
  cudaSetDevice(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  ctx->clear_graphs();
  if (ctx->arena.base) cudaFree(ctx->arena.base);
  if (ctx->d_err) cudaFree(ctx->d_err);
  if (ctx->ev_fork) cudaEventDestroy(ctx->ev_fork);
  if (ctx->ev_join) cudaEventDestroy(ctx->ev_join);
  for (cudaStream_t gs : ctx->group_streams) {
    cudaStreamSynchronize(gs);
    cudaStreamDestroy(gs);
  }
  for (cudaEvent_t ge : ctx->group_events) cudaEventDestroy(ge);
  if (ctx->stream2) cudaStreamDestroy(ctx->stream2);
  if (ctx->own) cudaStreamDestroy(ctx->own);
  delete ctx;
  return ZJAI_OK;
}

int zjai_ctx_set_stream(zjai_ctx* ctx, void* s) {
  ZJAI_TRY(ctx_enter(ctx));
  ctx->stream = s ? static_cast<cudaStream_t>(s) : ctx->own;
  return ZJAI_OK;
}

int zjai_ctx_sync(zjai_ctx* ctx) {
  ZJAI_TRY(ctx_enter(ctx));
  return ctx_check_status(ctx);
}

int zjai_ctx_set_output_clamp(zjai_ctx* ctx, int clamp) {
  if (!ctx) return fail(ZJAI_INVALID_ARGUMENT, "null context");
  ctx->clamp_output = clamp != 0;
  return ZJAI_OK;
}

int zjai_ctx_set_probe(zjai_ctx* ctx, const char* name, float* dst, int64_t capacity) {
  ZJAI_TRY(ctx_enter(ctx));
  if (!name) return fail(ZJAI_INVALID_ARGUMENT, "probe: null name");
  if (!dst) {
    ctx->probes.erase(name);
    return ZJAI_OK;
  }
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, dst) != cudaSuccess || at.type != cudaMemoryTypeDevice ||
      at.device != ctx->device) {
    cudaGetLastError();
    return fail(ZJAI_INVALID_ARGUMENT, "probe: the buffer must be device memory of the context's GPU");
  }
  if (capacity <= 0) return fail(ZJAI_INVALID_ARGUMENT, "probe: capacity must be positive");
  ctx->probes[name] = {dst, (long long)capacity};
  return ZJAI_OK;
}

int zjai_ctx_set_graphs(zjai_ctx* ctx, int enable) {
  ZJAI_TRY(ctx_enter(ctx));
  ZJAI_TRY(cuda_check(cudaStreamSynchronize(ctx->stream), "stream sync"));
  ctx->graphs = enable != 0;
  if (!ctx->graphs) ctx->clear_graphs();
  return ZJAI_OK;
}

int zjai_ctx_set_wait_limit(zjai_ctx* ctx, int64_t cycles) {
  if (!ctx) return fail(ZJAI_INVALID_ARGUMENT, "null context");
  if (cycles < 0) return fail(ZJAI_INVALID_ARGUMENT, "wait limit must be >= 0 (0: default)");
  ctx->wait_cycles = cycles;
  return ZJAI_OK;
}

int64_t zjai_ctx_launch_count(const zjai_ctx* ctx) { return ctx ? (int64_t)ctx->launches : 0; }

int zjai_ctx_profile(zjai_ctx* ctx, int enable) {
  ZJAI_TRY(ctx_enter(ctx));
  ctx->profiling = enable != 0;
  return ZJAI_OK;
}

int zjai_ctx_profile_read(zjai_ctx* ctx, double* conv_ms, double* conv_flops,
                          int64_t* conv_launches) {
  return zjai_ctx_profile_read_bytes(ctx, conv_ms, conv_flops, nullptr, conv_launches);
}

int zjai_ctx_profile_read_bytes(zjai_ctx* ctx, double* conv_ms, double* conv_flops,
                                double* conv_bytes, int64_t* conv_launches) {
  ZJAI_TRY(ctx_enter(ctx));
  ZJAI_TRY(cuda_check(cudaStreamSynchronize(ctx->stream), "stream sync"));
  ZJAI_TRY(cuda_check(cudaStreamSynchronize(ctx->stream2), "stream sync"));
  double ms = 0.0, fl = 0.0, by = 0.0;
  int64_t nconv = 0;
  for (auto& r : ctx->conv_records) {
    float t = 0.f;
    ZJAI_TRY(cuda_check(cudaEventElapsedTime(&t, r.start, r.stop), "event time"));
    if (r.conv) {
      ms += t;
      fl += r.flops;
      by += r.bytes;
      ++nconv;
    }
    auto it = std::find_if(ctx->tag_totals.begin(), ctx->tag_totals.end(),
                           [&](const std::pair<std::string, Ctx::TagTotal>& p) { return p.first == r.tag; });
    if (it == ctx->tag_totals.end()) {
      ctx->tag_totals.push_back({r.tag, Ctx::TagTotal()});
      it = ctx->tag_totals.end() - 1;
    }
    it->second.launches++;
    it->second.ms += t;
    it->second.flops += r.flops;
    it->second.bytes += r.bytes;
    ctx->ev_pool.push_back(r.start);
    ctx->ev_pool.push_back(r.stop);
  }
  if (conv_launches) *conv_launches = nconv;
  ctx->conv_records.clear();
  if (conv_ms) *conv_ms = ms;
  if (conv_flops) *conv_flops = fl;
  if (conv_bytes) *conv_bytes = by;
  return ZJAI_OK;
}

int zjai_ctx_profile_report(zjai_ctx* ctx, char* buf, size_t len) {
  ZJAI_TRY(ctx_enter(ctx));
  std::string s = "layer\tlaunches\tms\tGFLOP\tTFLOP/s\tGB\tGB/s\n";
  for (auto& p : ctx->tag_totals) {
    char line[512];
    const double ms = p.second.ms;
    snprintf(line, sizeof line, "%s\t%lld\t%.4f\t%.3f\t%.1f\t%.4f\t%.0f\n", p.first.c_str(),
             p.second.launches, ms, p.second.flops / 1e9,
             ms > 0 ? p.second.flops / (ms * 1e9) : 0.0, p.second.bytes / 1e9,
             ms > 0 ? p.second.bytes / (ms * 1e6) : 0.0);
    s += line;
  }
  ctx->tag_totals.clear();
  if (buf && len) {
    const size_t n = std::min(len - 1, s.size());
    memcpy(buf, s.data(), n);
    buf[n] = 0;
  }
  return ZJAI_OK;
}

int zjai_conv2d(zjai_ctx* ctx, const float* x, int c, int h, int w, const float* weight,
                const float* bias, int oc, int kh, int kw, int stride, int pad_h, int pad_w,
                int groups, const int* extra, int act, float* out, int mem) {
  ZJAI_TRY(ctx_enter(ctx));
  if (!x || !weight || !out || c <= 0 || h <= 0 || w <= 0 || oc <= 0)
    return fail(ZJAI_INVALID_ARGUMENT, "conv2d: bad arguments");
  if (act < ZJAI_ACT_NONE || act > ZJAI_ACT_RELU6)
    return fail(ZJAI_INVALID_ARGUMENT, "conv2d: unknown activation");
  if (groups == c && groups > 1 && oc == c && kh == 3 && kw == 3 && stride == 1 && pad_h == 1 &&
      pad_w == 1 && !bias && act == ZJAI_ACT_NONE && !(extra && (extra[0] | extra[1] | extra[2] | extra[3])))
    return zjai_depthwise3x3(ctx, x, c, h, w, weight, out, mem);
  ArenaScope scope(ctx);
  std::vector<float> wbuf, bbuf;
  const float *hw, *hb;
  if (groups <= 0 || c % groups) return fail(ZJAI_INVALID_ARGUMENT, "conv2d: groups");
  ZJAI_TRY(fetch_host(weight, (size_t)oc * (c / groups) * kh * kw, mem, &wbuf, &hw));
  ZJAI_TRY(fetch_host(bias, (size_t)oc, mem, &bbuf, &hb));
  ConvLayer L;
  ZJAI_TRY(pack_conv(ctx, &L, hw, hb, c, oc, kh, kw, stride, pad_h, pad_w, groups, extra, 1));
  LayerGuard guard(&L);
  int oh, ow, out_h, out_w;
  L.out_size(h, w, &oh, &ow, &out_h, &out_w);
  if (oh <= 0 || ow <= 0) return fail(ZJAI_INVALID_ARGUMENT, "conv2d: input smaller than the kernel");
  const float* dx;
  ZJAI_TRY(stage_in(ctx, x, (size_t)c * h * w, mem, &dx));
  TView tin;
  ZJAI_TRY(planar_to_tensor(ctx, dx, c, h, w, &tin));
  float* dout;
  const size_t nout = (size_t)oc * out_h * out_w;
  ZJAI_TRY(stage_out_alloc(ctx, out, nout, mem, &dout));
  ConvOut o;
  o.act1 = act;
  o.planar = true;
  o.pout = dout;
  o.p_plane = (long long)out_h * out_w;
  o.p_row = out_w;
  ZJAI_TRY(run_conv(ctx, L, tin, o));
  ZJAI_TRY(stage_out_finish(ctx, out, dout, nout, mem));
  return ctx_check_status(ctx);
}

int zjai_conv_transpose2d(zjai_ctx* ctx, const float* x, int c, int h, int w,
                          const float* weight, const float* bias, int oc, int k, int pad,
                          int out_pad, float* out, int mem) {
  ZJAI_TRY(ctx_enter(ctx));
  if (!x || !weight || !out || c <= 0 || h <= 0 || w <= 0 || oc <= 0)
    return fail(ZJAI_INVALID_ARGUMENT, "conv_transpose2d: bad arguments");
  ArenaScope scope(ctx);
  std::vector<float> wbuf, bbuf;
  const float *hw, *hb;
  ZJAI_TRY(fetch_host(weight, (size_t)c * oc * k * k, mem, &wbuf, &hw));
  ZJAI_TRY(fetch_host(bias, (size_t)oc, mem, &bbuf, &hb));
  ConvLayer L;
  ZJAI_TRY(pack_convT(ctx, &L, hw, hb, c, oc, k, pad, out_pad, 1));
  LayerGuard guard(&L);
  int oh, ow, out_h, out_w;
  L.out_size(h, w, &oh, &ow, &out_h, &out_w);
  const float* dx;
  ZJAI_TRY(stage_in(ctx, x, (size_t)c * h * w, mem, &dx));
  TView tin;
  ZJAI_TRY(planar_to_tensor(ctx, dx, c, h, w, &tin));
  float* dout;
  const size_t nout = (size_t)oc * out_h * out_w;
  ZJAI_TRY(stage_out_alloc(ctx, out, nout, mem, &dout));
  ConvOut o;
  o.planar = true;
  o.pout = dout;
  o.p_plane = (long long)out_h * out_w;
  o.p_row = out_w;
  ZJAI_TRY(run_conv(ctx, L, tin, o));
  ZJAI_TRY(stage_out_finish(ctx, out, dout, nout, mem));
  return ctx_check_status(ctx);
}

}  // extern "C"
