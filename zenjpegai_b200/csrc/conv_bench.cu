// Layer-level timing harnesses: the GPU counterpart of the crate's benches/conv_kernels.rs
// (PackedConv::new + forward on network layer shapes), timing conv_tc_kernel alone, and the
// same for the memory-bound kernels of the transformer blocks.
#include <random>
#include <vector>

#include "api_common.h"
#include "kernels_attn.h"

namespace zjai {
namespace {

// Deterministic pseudo-random f16 fill (values in [-1, 1)), so timing is not taken on zeros.
__global__ void fill_kernel(__half* p, long long n, uint32_t seed) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    uint32_t x = (uint32_t)i * 2654435761u ^ seed;
    x ^= x >> 15;
    x *= 2246822519u;
    x ^= x >> 13;
    p[i] = __float2half_rn((float)(x & 0xFFFF) / 32768.f - 1.f);
  }
}

}  // namespace
}  // namespace zjai

using namespace zjai;

extern "C" int zjai_conv_bench(zjai_ctx* ctx, int n, int h, int w, int cin, int cout, int k,
                               int stride, int groups, int transposed, int residual, int reps,
                               double* ms, double* flops) {
  ZJAI_TRY(ctx_enter(ctx));
  if (n <= 0 || h <= 0 || w <= 0 || cin <= 0 || cout <= 0 || k <= 0 || reps <= 0 || !ms)
    return fail(ZJAI_INVALID_ARGUMENT, "conv_bench: bad arguments");
  ArenaScope scope(ctx);
  std::mt19937 rng(1234);
  std::normal_distribution<float> nd(0.f, 1.f);
  ConvLayer L;
  if (!transposed) {
    std::vector<float> wt((size_t)cout * (cin / groups) * k * k), b(cout);
    for (auto& v : wt) v = nd(rng) / sqrtf((float)(cin / groups * k * k));
    for (auto& v : b) v = 0.01f * nd(rng);
    ZJAI_TRY(pack_conv(ctx, &L, wt.data(), b.data(), cin, cout, k, k, stride, k / 2, k / 2,
                       groups, nullptr, 1));
  } else {
    std::vector<float> wt((size_t)cin * cout * k * k), b(cout);
    for (auto& v : wt) v = nd(rng) / sqrtf((float)(cin * k * k / 4));
    for (auto& v : b) v = 0.01f * nd(rng);
    ZJAI_TRY(pack_convT(ctx, &L, wt.data(), b.data(), cin, cout, k, 1, k == 3 ? 1 : 0, 1));
  }
  LayerGuard guard(&L);
  int oh, ow, out_h, out_w;
  L.out_size(h, w, &oh, &ow, &out_h, &out_w);
  TView x, y;
  ZJAI_TRY(alloc_tensor(ctx, n, h, w, cin, &x));
  fill_kernel<<<1024, 256, 0, ctx->stream>>>(x.p, (long long)n * x.img, 17u);
  ConvOut o;
  if (residual == 2) {
    // a synthesis network's final layer: planar f32 planes [n][cph][out_h][out_w], denormalised
    const long long plane = (long long)out_h * out_w;
    float* pl = static_cast<float*>(ctx->arena.alloc(sizeof(float) * plane * L.cph * n));
    if (!pl) return fail(ZJAI_LIMIT_EXCEEDED, "conv_bench: arena exhausted");
    o.planar = true;
    o.denorm = true;
    o.pout = pl;
    o.p_plane = plane;
    o.p_row = out_w;
    o.p_img = plane * L.cph;
  } else {
    ZJAI_TRY(alloc_tensor(ctx, n, out_h, out_w, L.cph, &y));
    fill_kernel<<<1024, 256, 0, ctx->stream>>>(y.p, (long long)n * y.img, 29u);
    o.out = y;
    o.act1 = ACT_RELU;
    if (residual) {
      o.op = OP_ADD;
      o.r1 = &y;
    }
  }
  ZJAI_TRY(run_conv(ctx, L, x, o));  // warm-up
  cudaEvent_t e0, e1;
  ZJAI_TRY(cuda_check(cudaEventCreate(&e0), "event"));
  ZJAI_TRY(cuda_check(cudaEventCreate(&e1), "event"));
  cudaEventRecord(e0, ctx->stream);
  for (int i = 0; i < reps; ++i) ZJAI_TRY(run_conv(ctx, L, x, o));
  cudaEventRecord(e1, ctx->stream);
  ZJAI_TRY(cuda_check(cudaEventSynchronize(e1), "event sync"));
  float t = 0.f;
  cudaEventElapsedTime(&t, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  *ms = (double)t / reps;
  if (flops) *flops = (double)L.flops_per_px * oh * ow * n;
  return ctx_check_status(ctx);
}

extern "C" int zjai_kernel_bench(zjai_ctx* ctx, int kind, int n, int h, int w, int c, int reps,
                                 double* ms, double* bytes) {
  ZJAI_TRY(ctx_enter(ctx));
  if (kind < ZJAI_KB_DW || kind > ZJAI_KB_FFN || n <= 0 || h <= 0 || w <= 0 || c <= 0 ||
      c % 8 || reps <= 0 || !ms)
    return fail(ZJAI_INVALID_ARGUMENT, "kernel_bench: bad arguments");
  if ((kind == ZJAI_KB_DW_GATE && c % 16) || (kind == ZJAI_KB_LN && c > 512) ||
      (kind == ZJAI_KB_ATTN && c % 4) || (kind == ZJAI_KB_FFN && !ffn_fusable(c, 4 * c)))
    return fail(ZJAI_UNSUPPORTED, "kernel_bench: channel count not supported by this kernel");
  ArenaScope scope(ctx);
  const int cin = kind == ZJAI_KB_ATTN ? 3 * c : c;
  const int cout = kind == ZJAI_KB_DW_GATE ? c / 2 : c;
  TView x, y;
  ZJAI_TRY(alloc_tensor(ctx, n, h, w, cin, &x));
  ZJAI_TRY(alloc_tensor(ctx, n, h, w, cout, &y));
  fill_kernel<<<1024, 256, 0, ctx->stream>>>(x.p, (long long)n * x.img, 17u);
  // per-channel parameters: depthwise weights [c][9], or gamma / beta, or the temperatures
  std::vector<float> hp((size_t)c * 9 + 2 * c + 4);
  std::mt19937 rng(99);
  std::uniform_real_distribution<float> ud(-0.3f, 0.3f);
  for (auto& v : hp) v = ud(rng);
  for (int i = 0; i < 4; ++i) hp[(size_t)c * 9 + 2 * c + i] = 1.f + 0.25f * i;
  float* dp = static_cast<float*>(ctx->arena.alloc(hp.size() * sizeof(float)));
  float* scratch = static_cast<float*>(
      ctx->arena.alloc(attention_scratch_floats(n, c, 4, h * w, ctx->sms) * sizeof(float)));
  if (!dp || !scratch) return fail(ZJAI_LIMIT_EXCEEDED, "kernel_bench: arena exhausted");
  ZJAI_TRY(cuda_check(cudaMemcpyAsync(dp, hp.data(), hp.size() * sizeof(float),
                                      cudaMemcpyHostToDevice, ctx->stream),
                      "kernel_bench params"));
  const float* wt = dp;
  const float* gamma = dp + (size_t)c * 9;
  const float* temp = gamma + 2 * c;
  // fused FFN: random W_in [8c][c], depthwise [8c][9], W_out [c][4c] (x = ln, y = residual)
  FfnLayer F;
  struct Guard {
    FfnLayer* f;
    ~Guard() {
      cudaDeviceSynchronize();
      free_ffn(f);
    }
  } guard{&F};
  if (kind == ZJAI_KB_FFN) {
    const int hidden = 4 * c;
    std::vector<float> wi((size_t)2 * hidden * c), wd((size_t)2 * hidden * 9),
        wo((size_t)c * hidden);
    std::uniform_real_distribution<float> wdist(-0.1f, 0.1f);
    for (auto& v : wi) v = wdist(rng);
    for (auto& v : wd) v = ud(rng);
    for (auto& v : wo) v = wdist(rng);
    ZJAI_TRY(pack_ffn(ctx, &F, wi.data(), wd.data(), wo.data(), c, hidden));
    fill_kernel<<<1024, 256, 0, ctx->stream>>>(y.p, (long long)n * y.img, 23u);
  }
  int st = ZJAI_OK;
  auto run = [&] {
    switch (kind) {
      case ZJAI_KB_FFN: st = run_ffn(ctx, F, x, y); break;
      case ZJAI_KB_DW: launch_dw3x3(ctx, x, y, wt, false, ctx->stream); break;
      case ZJAI_KB_DW_GATE: launch_dw3x3(ctx, x, y, wt, true, ctx->stream); break;
      case ZJAI_KB_LN: launch_layer_norm(x, y, gamma, gamma + c, ctx->stream); break;
      default: launch_attention(x, y, 4, temp, scratch, ctx->sms, ctx->stream); break;
    }
  };
  run();  // warm-up
  ZJAI_TRY(st);
  cudaEvent_t e0, e1;
  ZJAI_TRY(cuda_check(cudaEventCreate(&e0), "event"));
  ZJAI_TRY(cuda_check(cudaEventCreate(&e1), "event"));
  cudaEventRecord(e0, ctx->stream);
  for (int i = 0; i < reps; ++i) run();
  cudaEventRecord(e1, ctx->stream);
  ZJAI_TRY(cuda_check(cudaEventSynchronize(e1), "event sync"));
  float t = 0.f;
  cudaEventElapsedTime(&t, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  ZJAI_TRY(cuda_check(cudaGetLastError(), "kernel_bench launch"));
  *ms = (double)t / reps;
  // attention reads q, k (Gram) and v (apply) and writes the output
  const double px = (double)n * h * w;
  // the fused FFN reads ln and the residual and writes x
  if (bytes)
    *bytes = 2.0 * px * (kind == ZJAI_KB_ATTN ? 4.0 * c
                         : kind == ZJAI_KB_FFN ? 3.0 * c
                                               : (double)(cin + cout));
  return ctx_check_status(ctx);
}
