// Enhancement post-filters on the reconstructed planes (src/filters/): LEF, the luma edge
// filter (src/filters/lef.rs), bit-exact with the crate's f32 arithmetic, and eICCI
// (src/filters/icci.rs; its network in net.cu, `Runner::icci`).
#include <cstdint>
#include <vector>

#include "api_common.h"
#include "net.h"

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

// a failed call leaves nothing of itself queued on the context's stream
int settle_stream(Ctx* ctx, int st) {
  cudaStreamSynchronize(ctx->stream);
  return st;
}

// ---- eICCI transforms (src/model/icci.rs:245-470) -------------------------------------------

__device__ __forceinline__ void haar4(float x1, float x2, float x3, float x4, float* o) {
  o[0] = __fadd_rn(__fadd_rn(__fadd_rn(x1, x2), x3), x4);
  o[1] = __fadd_rn(__fadd_rn(__fsub_rn(-x1, x2), x3), x4);
  o[2] = __fadd_rn(__fsub_rn(__fadd_rn(-x1, x2), x3), x4);
  o[3] = __fadd_rn(__fsub_rn(__fsub_rn(x1, x2), x3), x4);
}
__device__ __forceinline__ void ihaar4(float x1, float x2, float x3, float x4, float* o) {
  o[0] = __fadd_rn(__fsub_rn(__fsub_rn(x1, x2), x3), x4);
  o[1] = __fsub_rn(__fadd_rn(__fsub_rn(x1, x2), x3), x4);
  o[2] = __fsub_rn(__fsub_rn(__fadd_rn(x1, x2), x3), x4);
  o[3] = __fadd_rn(__fadd_rn(__fadd_rn(x1, x2), x3), x4);
}

// tile_input (icci.rs:405-438): per 4 x 4 block of the tile (x0, y0, tw x th) of each normalised
// plane, replicate-padded right / bottom, the two-level Haar bands (dwt2_block, icci.rs:326-360)
// as f32 planar [48][bh][bw] (the exact input the corrections are added to) and as the NHWC
// f16 network input [bh][bw][48]. One thread per (plane, block).
__global__ void icci_dwt_kernel(const float* __restrict__ y, const float* __restrict__ u,
                                const float* __restrict__ v, int w, int x0, int y0, int tw,
                                int th, int bh, int bw, float* __restrict__ bands,
                                __half* __restrict__ x16, long long pix, long long row) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long nb = (long long)bh * bw;
  if (idx >= 3 * nb) return;
  const int p = (int)(idx / nb), b = (int)(idx - (long long)p * nb);
  const int by = b / bw, bx = b - by * bw;
  const float* src = p == 0 ? y : p == 1 ? u : v;
  float q[4][4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int sy = y0 + min(4 * by + r, th - 1);
#pragma unroll
    for (int c = 0; c < 4; ++c)
      q[r][c] = __ldg(src + (long long)sy * w + x0 + min(4 * bx + c, tw - 1));
  }
  float l1[2][2][4];
#pragma unroll
  for (int iy = 0; iy < 2; ++iy)
#pragma unroll
    for (int ix = 0; ix < 2; ++ix) {
      const int r = 2 * iy, c = 2 * ix;
      haar4(q[r][c] * 0.5f, q[r + 1][c] * 0.5f, q[r][c + 1] * 0.5f, q[r + 1][c + 1] * 0.5f,
            l1[iy][ix]);
    }
  float o[16];
#pragma unroll
  for (int k = 0; k < 4; ++k)
    haar4(l1[0][0][k] * 0.5f, l1[1][0][k] * 0.5f, l1[0][1][k] * 0.5f, l1[1][1][k] * 0.5f,
          o + 4 * k);
  __half2 h[8];
#pragma unroll
  for (int k = 0; k < 16; ++k) bands[(long long)(p * 16 + k) * nb + b] = o[k];
#pragma unroll
  for (int k = 0; k < 8; ++k) h[k] = __floats2half2_rn(o[2 * k], o[2 * k + 1]);
  uint4* d = reinterpret_cast<uint4*>(x16 + (long long)by * row + (long long)bx * pix + p * 16);
  d[0] = *reinterpret_cast<const uint4*>(&h[0]);
  d[1] = *reinterpret_cast<const uint4*>(&h[4]);
}

// tile_output + write_core (icci.rs:441-470, filters/icci.rs:160-173): per block, the inverse
// transform (idwt2_block, icci.rs:363-402) of correction + input bands of plane p, its samples
// inside the tile's core written back to the plane. One thread per block.
__global__ void icci_out_kernel(const float* __restrict__ corr, const float* __restrict__ bands,
                                int p, int bh, int bw, float* __restrict__ plane, int w, int x0,
                                int y0, int cx0, int cy0, int cx1, int cy1) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  const int nb = bh * bw;
  if (b >= nb) return;
  const int by = b / bw, bx = b - by * bw;
  float s[16];
#pragma unroll
  for (int k = 0; k < 16; ++k)
    s[k] = __fadd_rn(__ldg(corr + (long long)k * nb + b), __ldg(bands + (long long)(p * 16 + k) * nb + b));
  float q[4][2][2];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float r[4];
    ihaar4(s[4 * i] * 0.5f, s[4 * i + 1] * 0.5f, s[4 * i + 2] * 0.5f, s[4 * i + 3] * 0.5f, r);
    q[i][0][0] = r[0];
    q[i][0][1] = r[2];
    q[i][1][0] = r[1];
    q[i][1][1] = r[3];
  }
#pragma unroll
  for (int dy = 0; dy < 2; ++dy)
#pragma unroll
    for (int dx = 0; dx < 2; ++dx) {
      float r[4];
      ihaar4(q[0][dy][dx] * 0.5f, q[1][dy][dx] * 0.5f, q[2][dy][dx] * 0.5f, q[3][dy][dx] * 0.5f, r);
      const int fy[4] = {4 * by + 2 * dy, 4 * by + 2 * dy + 1, 4 * by + 2 * dy, 4 * by + 2 * dy + 1};
      const int fx[4] = {4 * bx + 2 * dx, 4 * bx + 2 * dx, 4 * bx + 2 * dx + 1, 4 * bx + 2 * dx + 1};
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (fy[k] >= cy0 && fy[k] < cy1 && fx[k] >= cx0 && fx[k] < cx1)
          plane[(long long)(y0 + fy[k]) * w + x0 + fx[k]] = r[k];
    }
}

// s / 255 (normalise) or clamp(s, 0, 1) * 255 (finish) of the three planes
__global__ void icci_scale_kernel(float* __restrict__ y, float* __restrict__ u,
                                  float* __restrict__ v, long long n, int finish) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 3 * n) return;
  float* p = i < n ? y : i < 2 * n ? u : v;
  const long long j = i % n;
  const float s = p[j];
  p[j] = finish ? __fmul_rn(clamp01(s), 255.f) : __fdiv_rn(s, 255.f);
}

// One axis of the filter tiling (filters/icci.rs:68-96): (start, length) per tile; false when
// the tiling leaves a tile below the minimum size or not larger than its overlap.
bool icci_axis(int len, int tile, int overlap, std::vector<std::pair<int, int>>* out) {
  constexpr int kMinTile = 176;  // EfficientICCIFilter.tile_min_size_for_MSSSIM
  tile = tile < len ? tile : len;
  if (tile <= overlap || len <= overlap) return false;
  out->clear();
  for (int p = 0; p < len - overlap; p += tile - overlap)
    out->push_back({p, tile < len - p ? tile : len - p});
  const size_t n = out->size();
  if ((*out)[n - 1].second < kMinTile) {
    if (n < 2 || (*out)[n - 2].second <= kMinTile + overlap) return false;
    (*out)[n - 2].second -= kMinTile;
    (*out)[n - 1].first -= kMinTile;
    (*out)[n - 1].second += kMinTile;
  }
  return true;
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
  if (mem == ZJAI_MEM_DEVICE) {
    ZJAI_TRY(check_device_buffer(ctx, scale_log, "LEF scale map"));
    ZJAI_TRY(check_device_buffer(ctx, out, "LEF output"));
  }
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

struct zjai_net : zjai::Net {};

int zjai_icci_filter(zjai_ctx* ctx, zjai_net* net_y, zjai_net* net_uv, int use_u, int use_v,
                     float* y, float* u, float* v, int h, int w, int tile_size, int overlap,
                     int mem) {
  ZJAI_TRY(ctx_enter(ctx));
  if (!y || !u || !v || h <= 0 || w <= 0) return fail(ZJAI_INVALID_ARGUMENT, "eICCI: empty picture");
  if (mem != ZJAI_MEM_HOST && mem != ZJAI_MEM_DEVICE)
    return fail(ZJAI_INVALID_ARGUMENT, "mem must be HOST or DEVICE");
  for (zjai_net* n : {net_y, net_uv})
    if (n && (n->kind != ZJAI_ICCI || n->ctx != ctx))
      return fail(ZJAI_INVALID_ARGUMENT, "eICCI: not an eICCI network of this context");
  std::vector<std::pair<int, int>> rows{{0, h}}, cols{{0, w}};
  if (tile_size > 0) {
    if (overlap < 0 || !icci_axis(h, tile_size, overlap, &rows) || !icci_axis(w, tile_size, overlap, &cols))
      return fail(ZJAI_INVALID_DATA, "eICCI: tiling leaves a tile below the minimum size or "
                                     "not larger than its overlap");
  } else {
    overlap = 0;
  }
  const int half = overlap / 2;
  if (mem == ZJAI_MEM_DEVICE)
    for (float* pl : {y, u, v}) ZJAI_TRY(check_device_buffer(ctx, pl, "eICCI plane"));
  ArenaScope scope(ctx);
  const long long n = (long long)h * w;
  float* d[3] = {y, u, v};
  if (mem == ZJAI_MEM_HOST) {
    for (int p = 0; p < 3; ++p) {
      float* t = static_cast<float*>(ctx->arena.alloc(n * sizeof(float)));
      if (!t) return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (eICCI planes)");
      ZJAI_TRY(cuda_check(cudaMemcpyAsync(t, (p == 0 ? y : p == 1 ? u : v), n * sizeof(float),
                                          cudaMemcpyHostToDevice, ctx->stream), "H2D"));
      d[p] = t;
    }
  }
  const int sblocks = (int)((3 * n + 255) / 256);
  icci_scale_kernel<<<sblocks, 256, 0, ctx->stream>>>(d[0], d[1], d[2], n, 0);
  ctx->launches++;
  const bool want_uv = net_uv && (use_u || use_v);
  for (auto& r : rows)
    for (auto& c : cols) {
      const int x0 = c.first, y0 = r.first, tw = c.second, th = r.second;
      const int left = x0 == 0 ? 0 : half, top = y0 == 0 ? 0 : half;
      const int right = x0 + tw >= w ? 0 : half, bottom = y0 + th >= h ? 0 : half;
      if (tw <= left + right || th <= top + bottom)
        return settle_stream(ctx, fail(ZJAI_INVALID_DATA, "eICCI: tile is all overlap"));
      if (!net_y && !want_uv) continue;
      ArenaMark mark(&ctx->arena);
      const int bh = (th + 3) / 4, bw = (tw + 3) / 4;
      const long long nb = (long long)bh * bw;
      float* bands = static_cast<float*>(ctx->arena.alloc(48 * nb * sizeof(float)));
      float* corr = static_cast<float*>(ctx->arena.alloc(3 * 16 * nb * sizeof(float)));
      TView x16;
      if (!bands || !corr) return settle_stream(ctx, fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (eICCI)"));
      int st = alloc_tensor(ctx, 1, bh, bw, 3 * kIcciBands, &x16);
      if (st != ZJAI_OK) return settle_stream(ctx, st);
      icci_dwt_kernel<<<(int)((3 * nb + 127) / 128), 128, 0, ctx->stream>>>(
          d[0], d[1], d[2], w, x0, y0, tw, th, bh, bw, bands, x16.p, x16.pix, x16.row);
      ctx->launches++;
      float* cy = net_y ? corr : nullptr;
      float* cu = want_uv && use_u ? corr + 16 * nb : nullptr;
      float* cv = want_uv && use_v ? corr + 32 * nb : nullptr;
      if (net_y) {
        Runner rn;
        rn.ctx = ctx;
        rn.net = net_y;
        rn.arena = &ctx->arena;
        rn.stream = ctx->stream;
        st = rn.icci(x16, false, cy, nullptr);
        if (st != ZJAI_OK) return settle_stream(ctx, st);
      }
      if (want_uv) {
        Runner rn;
        rn.ctx = ctx;
        rn.net = net_uv;
        rn.arena = &ctx->arena;
        rn.stream = ctx->stream;
        st = rn.icci(x16, true, cu, cv);
        if (st != ZJAI_OK) return settle_stream(ctx, st);
      }
      const float* cs[3] = {cy, cu, cv};
      for (int p = 0; p < 3; ++p) {
        if (!cs[p]) continue;
        icci_out_kernel<<<(int)((nb + 127) / 128), 128, 0, ctx->stream>>>(
            cs[p], bands, p, bh, bw, d[p], w, x0, y0, left, top, tw - right, th - bottom);
        ctx->launches++;
      }
    }
  icci_scale_kernel<<<sblocks, 256, 0, ctx->stream>>>(d[0], d[1], d[2], n, 1);
  ctx->launches++;
  ZJAI_TRY(cuda_check(cudaGetLastError(), "eICCI launch"));
  if (mem == ZJAI_MEM_HOST)
    for (int p = 0; p < 3; ++p)
      ZJAI_TRY(cuda_check(cudaMemcpyAsync((p == 0 ? y : p == 1 ? u : v), d[p], n * sizeof(float),
                                          cudaMemcpyDeviceToHost, ctx->stream), "D2H"));
  return finish_call(ctx, mem);
}
