// Layout and elementwise kernels: planar f32 <-> NHWC f16 conversion, relu6.
#include "engine.h"
#include "net.h"

namespace zjai {

namespace {

__global__ void planar_to_nhwc_kernel(const float* __restrict__ src, int c, int H, int W, int y0,
                                      int x0, __half* __restrict__ dst, int n_img, int h, int w,
                                      long long pix, long long row, long long img,
                                      long long src_img) {
  long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long total = (long long)n_img * h * w;
  if (idx >= total) return;
  int x = (int)(idx % w);
  long long r = idx / w;
  int y = (int)(r % h);
  int n = (int)(r / h);
  const float* s = src + n * src_img + (long long)(y0 + y) * W + (x0 + x);
  __half* d = dst + n * img + (long long)y * row + (long long)x * pix;
  const long long plane = (long long)H * W;
  int ch = 0;
  for (; ch + 2 <= c; ch += 2) {
    float a = __ldg(s + ch * plane), b = __ldg(s + (ch + 1) * plane);
    *reinterpret_cast<__half2*>(d + ch) = __floats2half2_rn(a, b);
  }
  if (ch < c) d[ch] = __float2half_rn(__ldg(s + ch * plane));
}

__global__ void nhwc_to_planar_kernel(const __half* __restrict__ src, int n_img, int c, int h,
                                      int w, long long pix, long long row, long long img,
                                      float* __restrict__ dst) {
  long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long total = (long long)n_img * h * w;
  if (idx >= total) return;
  int x = (int)(idx % w);
  long long r = idx / w;
  int y = (int)(r % h);
  int n = (int)(r / h);
  const __half* s = src + n * img + (long long)y * row + (long long)x * pix;
  float* d = dst + (long long)n * c * h * w + (long long)y * w + x;
  for (int ch = 0; ch < c; ++ch) d[(long long)ch * h * w] = __half2float(s[ch]);
}

__global__ void relu6_kernel(const __half* __restrict__ src, __half* __restrict__ dst, int n_img,
                             int h, int w, int c8, long long spix, long long srow, long long simg,
                             long long dpix, long long drow, long long dimg) {
  long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long total = (long long)n_img * h * w * c8;
  if (idx >= total) return;
  int cg = (int)(idx % c8);
  long long r = idx / c8;
  int x = (int)(r % w);
  r /= w;
  int y = (int)(r % h);
  int n = (int)(r / h);
  uint4 u = *reinterpret_cast<const uint4*>(src + n * simg + y * srow + x * spix + cg * 8);
  __half2* hv = reinterpret_cast<__half2*>(&u);
  const __half2 z = __float2half2_rn(0.f), six = __float2half2_rn(6.f);
#pragma unroll
  for (int i = 0; i < 4; ++i) hv[i] = __hmin2(__hmax2(hv[i], z), six);
  *reinterpret_cast<uint4*>(dst + n * dimg + y * drow + x * dpix + cg * 8) = u;
}

inline int blocks_for(long long n, int t) { return (int)((n + t - 1) / t); }

// Edge-replicate the region of `dst` (extent H x W) outside src's extent h x w; src and dst
// share memory (`F.pad(x, (0, right, 0, bottom), mode="replicate")`, analysis.rs:48-71).
__global__ void replicate_pad_kernel(__half* __restrict__ p, int n_img, int h, int w, int H, int W,
                                     int c8, long long pix, long long row, long long img) {
  long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long total = (long long)n_img * H * W * c8;
  if (idx >= total) return;
  const int cg = (int)(idx % c8);
  long long r = idx / c8;
  const int x = (int)(r % W);
  r /= W;
  const int y = (int)(r % H), n = (int)(r / H);
  if (y < h && x < w) return;
  const int sy = y < h ? y : h - 1, sx = x < w ? x : w - 1;
  __half* b = p + n * img;
  *reinterpret_cast<uint4*>(b + y * row + x * pix + cg * 8) =
      *reinterpret_cast<const uint4*>(b + sy * row + sx * pix + cg * 8);
}

// (x - 127.5) / 128 of planar f32 pictures [n][c][h][w] into NHWC f16 with edge replication
// up to dst's extent (analysis.rs:36-39 normalize, then the first padding layer).
__global__ void normalize_pad_kernel(const float* __restrict__ src, int c, int h, int w,
                                     __half* __restrict__ dst, int n_img, int H, int W,
                                     long long pix, long long row, long long img) {
  long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long total = (long long)n_img * H * W;
  if (idx >= total) return;
  const int x = (int)(idx % W);
  long long r = idx / W;
  const int y = (int)(r % H), n = (int)(r / H);
  const int sy = y < h ? y : h - 1, sx = x < w ? x : w - 1;
  const float* s = src + (long long)n * c * h * w + (long long)sy * w + sx;
  __half* d = dst + n * img + y * row + x * pix;
  for (int ch = 0; ch < c; ++ch)
    d[ch] = __float2half_rn((__ldg(s + (long long)ch * h * w) - 127.5f) / 128.0f);
}

}  // namespace

void launch_replicate_pad(const TView& src, const TView& dst, cudaStream_t s) {
  if (dst.h == src.h && dst.w == src.w) return;
  const int c8 = (src.c + 7) / 8;
  long long total = (long long)dst.n * dst.h * dst.w * c8;
  replicate_pad_kernel<<<blocks_for(total, 256), 256, 0, s>>>(dst.p, dst.n, src.h, src.w, dst.h,
                                                               dst.w, c8, dst.pix, dst.row, dst.img);
}

void launch_normalize_pad(const float* src, int c, int h, int w, const TView& dst, cudaStream_t s) {
  long long total = (long long)dst.n * dst.h * dst.w;
  normalize_pad_kernel<<<blocks_for(total, 256), 256, 0, s>>>(src, c, h, w, dst.p, dst.n, dst.h,
                                                               dst.w, dst.pix, dst.row, dst.img);
}

void launch_planar_to_nhwc(const float* src, int c, int H, int W, int y0, int x0,
                           const TView& dst, cudaStream_t s) {
  long long total = (long long)dst.n * dst.h * dst.w;
  if (total == 0) return;
  planar_to_nhwc_kernel<<<blocks_for(total, 256), 256, 0, s>>>(
      src, c, H, W, y0, x0, dst.p, dst.n, dst.h, dst.w, dst.pix, dst.row, dst.img,
      (long long)c * H * W);
}

void launch_nhwc_to_planar(const TView& src, float* dst, cudaStream_t s) {
  long long total = (long long)src.n * src.h * src.w;
  if (total == 0) return;
  nhwc_to_planar_kernel<<<blocks_for(total, 256), 256, 0, s>>>(src.p, src.n, src.c, src.h, src.w,
                                                                src.pix, src.row, src.img, dst);
}

void launch_relu6(const TView& src, const TView& dst, cudaStream_t s) {
  int c8 = (src.c + 7) / 8;
  long long total = (long long)src.n * src.h * src.w * c8;
  if (total == 0) return;
  relu6_kernel<<<blocks_for(total, 256), 256, 0, s>>>(src.p, dst.p, src.n, src.h, src.w, c8,
                                                      src.pix, src.row, src.img, dst.pix, dst.row,
                                                      dst.img);
}

}  // namespace zjai
