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

// (x - 127.5) / 128 of planar f32 pictures [n][c][SH][SW] into NHWC f16 with edge replication
// up to dst's extent (analysis.rs:36-39 normalize, then the first padding layer); the picture
// read is the h x w window at (y0, x0) of each plane (an analysis tile, or the whole plane).
__global__ void normalize_pad_kernel(const float* __restrict__ src, int c, int SH, int SW, int y0,
                                     int x0, int h, int w, __half* __restrict__ dst, int n_img,
                                     int H, int W, long long pix, long long row, long long img) {
  long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long total = (long long)n_img * H * W;
  if (idx >= total) return;
  const int x = (int)(idx % W);
  long long r = idx / W;
  const int y = (int)(r % H), n = (int)(r / H);
  const int sy = y0 + (y < h ? y : h - 1), sx = x0 + (x < w ? x : w - 1);
  const long long plane = (long long)SH * SW;
  const float* s = src + (long long)n * c * plane + (long long)sy * SW + sx;
  __half* d = dst + n * img + y * row + x * pix;
  for (int ch = 0; ch < c; ++ch)
    d[ch] = __float2half_rn((__ldg(s + (long long)ch * plane) - 127.5f) / 128.0f);
}

// `preprocess_rgb` (colour.rs:535-541 -> source_planes colour.rs:390-436, preprocess
// colour.rs:462-495 for 4:4:4 coding) of 8-bit RGB pictures [n][h][w][3]: one thread per
// (picture, chroma sample): the 2 x 2 luma samples it covers (rows / columns past the picture
// replicate its last one, `replicate_pad`) are converted to BT.709 Y, U, V in [0, 255] with every
// operation rounded on its own (the reference's f32 order, no contraction), written as the
// luma plane [n][h][w] and the 12 unshuffled chroma channels [n][12][ph / 2][pw / 2].
__global__ void preprocess_rgb_kernel(const uint8_t* __restrict__ rgb, int n_img, int h, int w,
                                      float* __restrict__ luma, float* __restrict__ chroma) {
  const int ch = (h + 1) / 2, cw = (w + 1) / 2;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)n_img * ch * cw) return;
  const int cx = (int)(idx % cw);
  const long long r = idx / cw;
  const int cy = (int)(r % ch), n = (int)(r / ch);
  const float KR = 0.2126f, KG = 0.7152f, KB = 0.0722f, KBY = 1.8556f, KRY = 1.5748f;
  const long long cplane = (long long)ch * cw;
  float* cb = chroma + (long long)n * 12 * cplane + (long long)cy * cw + cx;
  const uint8_t* pic = rgb + (long long)n * h * w * 3;
  float* lp = luma + (long long)n * h * w;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int py = 2 * cy + (k >> 1), px = 2 * cx + (k & 1);
    const int sy = py < h ? py : h - 1, sx = px < w ? px : w - 1;
    const uint8_t* q = pic + ((long long)sy * w + sx) * 3;
    const float rr = __fdiv_rn((float)q[0], 255.f), gg = __fdiv_rn((float)q[1], 255.f),
                bb = __fdiv_rn((float)q[2], 255.f);
    const float y = __fadd_rn(__fadd_rn(__fmul_rn(KR, rr), __fmul_rn(KG, gg)), __fmul_rn(KB, bb));
    const float y255 = __fmul_rn(y, 255.f);
    const float u255 = __fmul_rn(__fadd_rn(__fdiv_rn(__fsub_rn(bb, y), KBY), 0.5f), 255.f);
    const float v255 = __fmul_rn(__fadd_rn(__fdiv_rn(__fsub_rn(rr, y), KRY), 0.5f), 255.f);
    cb[k * cplane] = y255;
    cb[(4 + k) * cplane] = u255;
    cb[(8 + k) * cplane] = v255;
    if (py < h && px < w) lp[(long long)py * w + px] = y255;
  }
}

// The kept core of each picture's tile latent: tile [n][C][th][tw] rows oy .. oy + core_h,
// columns ox .. ox + core_w -> full [n][C][LH][LW] at (cy, cx).
__global__ void copy_core_kernel(const float* __restrict__ tile, int n_img, int C, int th, int tw,
                                 int oy, int ox, int core_h, int core_w,
                                 float* __restrict__ full, int LH, int LW, int cy, int cx) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long total = (long long)n_img * C * core_h * core_w;
  if (idx >= total) return;
  const int x = (int)(idx % core_w);
  long long r = idx / core_w;
  const int y = (int)(r % core_h);
  r /= core_h;  // picture * C + channel
  full[(r * LH + cy + y) * LW + cx + x] = tile[(r * th + oy + y) * tw + ox + x];
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
  launch_normalize_pad_window(src, c, h, w, 0, 0, h, w, dst, s);
}

void launch_normalize_pad_window(const float* src, int c, int SH, int SW, int y0, int x0, int h,
                                 int w, const TView& dst, cudaStream_t s) {
  long long total = (long long)dst.n * dst.h * dst.w;
  normalize_pad_kernel<<<blocks_for(total, 256), 256, 0, s>>>(src, c, SH, SW, y0, x0, h, w,
                                                               dst.p, dst.n, dst.h, dst.w,
                                                               dst.pix, dst.row, dst.img);
}

void launch_preprocess_rgb(const uint8_t* rgb, int n, int h, int w, float* luma, float* chroma,
                           cudaStream_t s) {
  const long long total = (long long)n * ((h + 1) / 2) * ((w + 1) / 2);
  if (total == 0) return;
  preprocess_rgb_kernel<<<blocks_for(total, 256), 256, 0, s>>>(rgb, n, h, w, luma, chroma);
}

void launch_copy_core(const float* tile, int n, int C, int th, int tw, int oy, int ox, int core_h,
                      int core_w, float* full, int LH, int LW, int cy, int cx, cudaStream_t s) {
  const long long total = (long long)n * C * core_h * core_w;
  if (total == 0) return;
  copy_core_kernel<<<blocks_for(total, 256), 256, 0, s>>>(tile, n, C, th, tw, oy, ox, core_h,
                                                           core_w, full, LH, LW, cy, cx);
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
