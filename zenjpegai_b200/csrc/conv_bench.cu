// Layer-level timing harness: the GPU counterpart of the crate's benches/conv_kernels.rs
// (PackedConv::new + forward on network layer shapes), timing conv_tc_kernel alone.
#include <random>
#include <vector>

#include "api_common.h"

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
  ZJAI_TRY(alloc_tensor(ctx, n, out_h, out_w, L.cph, &y));
  fill_kernel<<<1024, 256, 0, ctx->stream>>>(x.p, (long long)n * x.img, 17u);
  fill_kernel<<<1024, 256, 0, ctx->stream>>>(y.p, (long long)n * y.img, 29u);
  ConvOut o;
  o.out = y;
  o.act1 = ACT_RELU;
  if (residual) {
    o.op = OP_ADD;
    o.r1 = &y;
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
