// Enhancement post-filters on the reconstructed planes (src/filters/): LEF, the luma edge
// filter (src/filters/lef.rs), bit-exact with the crate's f32 arithmetic.
#include <cstdint>

#include "api_common.h"

namespace zjai {
namespace {

// LEF.recSharpThrList / recSharpMagList (lef.rs:29-44): sigma-index thresholds and gains per
// model_id; constants of the reference, not signalled
__constant__ int kLefThr[4][3] = {{600, 1200, 2000}, {800, 1400, 2400}, {1000, 1600, 2800},
                                  {1200, 2000, 3200}};
__constant__ float kLefMag[4][3] = {{1.10f, 1.13f, 1.16f}, {1.07f, 1.09f, 1.11f},
                                    {1.03f, 1.04f, 1.05f}, {1.01f, 1.02f, 1.03f}};

// torch nearest interpolation source index, min(floor(i * (src / dst)), src - 1) in f32
__device__ __forceinline__ int nearest(int i, int src, int dst) {
  const float scale = __fdiv_rn((float)src, (float)dst);
  const int v = (int)floorf(__fmul_rn((float)i, scale));
  return v < src - 1 ? v : src - 1;
}

__device__ __forceinline__ float clamp01(float v) { return v < 0.f ? 0.f : v > 1.f ? 1.f : v; }

// One output sample per thread: x = Y / 255; the border ring and pictures under 3 columns keep
// clamp(x) * 255; inside, the 3x3 [5 5 5; 5 24 5; 5 5 5] / 64 blur accumulated by fused
// multiply-adds in (ky, kx) order, then clamp(blur + (x - blur) * gain) * 255, every other
// operation rounded on its own (lef.rs:78-97, 139-168).
__global__ void lef_kernel(const float* __restrict__ luma, int h, int w,
                           const int32_t* __restrict__ region, int sh, int sw, int model,
                           float* __restrict__ out) {
  const int X = blockIdx.x * blockDim.x + threadIdx.x;
  if (X >= w) return;
  const float range = 255.f, outer = 5.f / 64.f, centre = 24.f / 64.f;
  const int rx = nearest(X, sw, w);
  for (int Y = blockIdx.y; Y < h; Y += gridDim.y) {
    const float* row = luma + (long long)Y * w;
    const float cur = __fdiv_rn(__ldg(row + X), range);
    if (Y == 0 || Y + 1 == h || w < 3 || X == 0 || X + 1 == w) {
      out[(long long)Y * w + X] = __fmul_rn(clamp01(cur), range);
      continue;
    }
    const int s = __ldg(region + (long long)nearest(Y, sh, h) * sw + rx);
    const int* t = kLefThr[model];
    const float g = s >= t[2] ? kLefMag[model][2]
                  : s >= t[1] ? kLefMag[model][1]
                  : s >= t[0] ? kLefMag[model][0] : 1.f;
    float acc = 0.f;
#pragma unroll
    for (int dy = -1; dy <= 1; ++dy) {
      const float* r = row + (long long)dy * w;
#pragma unroll
      for (int dx = -1; dx <= 1; ++dx) {
        const float v = __fdiv_rn(__ldg(r + X + dx), range);
        acc = __fmaf_rn(v, dy == 0 && dx == 0 ? centre : outer, acc);
      }
    }
    const float blur = clamp01(acc);
    const float diff = __fmul_rn(__fsub_rn(cur, blur), g);
    out[(long long)Y * w + X] = __fmul_rn(clamp01(__fadd_rn(blur, diff)), range);
  }
}

}  // namespace
}  // namespace zjai

using namespace zjai;

int zjai_lef(zjai_ctx* ctx, const float* luma, int h, int w, const int32_t* scale_log, int c,
             int sh, int sw, int channel, int model_id, int bit_depth, float* out, int mem) {
  ZJAI_TRY(ctx_enter(ctx));
  if (!luma || !scale_log || !out) return fail(ZJAI_INVALID_ARGUMENT, "LEF: null pointer");
  if (mem != ZJAI_MEM_HOST && mem != ZJAI_MEM_DEVICE)
    return fail(ZJAI_INVALID_ARGUMENT, "mem must be HOST or DEVICE");
  // the crate's checks (lef.rs:108-126)
  if (model_id < 0 || model_id > 3) return fail(ZJAI_INVALID_DATA, "LEF: model_id out of range");
  if (channel < 0 || channel >= c) return fail(ZJAI_INVALID_DATA, "LEF: channel index out of range");
  if (h <= 0 || w <= 0 || sh <= 0 || sw <= 0)
    return fail(ZJAI_INVALID_ARGUMENT, "LEF: empty picture or scale map");
  if (bit_depth < 1 || bit_depth > 16) return fail(ZJAI_INVALID_ARGUMENT, "LEF: bit depth");
  ArenaScope scope(ctx);
  const size_t n = (size_t)h * w, nr = (size_t)sh * sw;
  const float* din;
  ZJAI_TRY(stage_in(ctx, luma, n, mem, &din));
  const int32_t* dreg = scale_log + (size_t)channel * nr;
  if (mem == ZJAI_MEM_HOST) {
    int32_t* d = static_cast<int32_t*>(ctx->arena.alloc(nr * sizeof(int32_t)));
    if (!d) return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (LEF scale map)");
    ZJAI_TRY(cuda_check(cudaMemcpyAsync(d, dreg, nr * sizeof(int32_t), cudaMemcpyHostToDevice,
                                        ctx->stream),
                        "H2D"));
    dreg = d;
  } else if (din == out) {
    // in place on the device: the stencil reads the input's neighbours, so filter a copy
    float* copy = static_cast<float*>(ctx->arena.alloc(n * sizeof(float)));
    if (!copy) return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (LEF input copy)");
    ZJAI_TRY(cuda_check(cudaMemcpyAsync(copy, din, n * sizeof(float), cudaMemcpyDeviceToDevice,
                                        ctx->stream),
                        "LEF copy"));
    din = copy;
  }
  float* dout;
  ZJAI_TRY(stage_out_alloc(ctx, out, n, mem, &dout));
  dim3 grid((w + 255) / 256, h < 65535 ? h : 65535);
  ctx->launches++;
  if (ctx->profiling) ctx->tag = "LEF";
  timed_launch(ctx, false, 0.0, 8.0 * n + 4.0 * nr, [&] {
    lef_kernel<<<grid, 256, 0, ctx->stream>>>(din, h, w, dreg, sh, sw, model_id, dout);
  });
  ZJAI_TRY(cuda_check(cudaGetLastError(), "LEF launch"));
  ZJAI_TRY(stage_out_finish(ctx, out, dout, n, mem));
  return finish_call(ctx, mem);
}
