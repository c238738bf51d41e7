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

// The luma analysis's first layer (3x3, stride 2, pad 1, one input channel) as a 1x1 conv:
// per output pixel (oy, ox) of the h1 x w1 output, its nine input taps (ky, kx) as channels
// 3 ky + kx (channels 9..15 zero). A tap reads input (2 oy - 1 + ky, 2 ox - 1 + kx) of the
// normalize_pad picture (the h x w window at (y0, x0) of the planar source, normalised to
// (s - 127.5) / 128 in f16, its rows / columns past the window replicating the last one), and 0
// above or left of it (the conv's zero padding; the padded picture has 2 h1 x 2 w1 samples,
// so no tap falls below or right of it). The f16 values equal normalize_pad's.
__global__ void normalize_im2col_kernel(const float* __restrict__ src, int SH, int SW, int y0,
                                        int x0, int h, int w, __half* __restrict__ dst, int n_img,
                                        int h1, int w1, long long pix, long long row,
                                        long long img) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)n_img * h1 * w1) return;
  const int ox = (int)(idx % w1);
  const long long r = idx / w1;
  const int oy = (int)(r % h1), n = (int)(r / h1);
  const float* s = src + (long long)n * SH * SW;
  __half v[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) v[k] = __float2half_rn(0.f);
#pragma unroll
  for (int ky = 0; ky < 3; ++ky) {
    const int y = 2 * oy - 1 + ky;
    if (y < 0) continue;
    const int sy = y0 + (y < h ? y : h - 1);
#pragma unroll
    for (int kx = 0; kx < 3; ++kx) {
      const int x = 2 * ox - 1 + kx;
      if (x < 0) continue;
      const int sx = x0 + (x < w ? x : w - 1);
      v[3 * ky + kx] = __float2half_rn((__ldg(s + (long long)sy * SW + sx) - 127.5f) / 128.0f);
    }
  }
  uint4* d = reinterpret_cast<uint4*>(dst + n * img + oy * row + ox * pix);
  d[0] = *reinterpret_cast<const uint4*>(&v[0]);
  d[1] = *reinterpret_cast<const uint4*>(&v[8]);
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

// Context model (mcm.rs:161-257) layout kernels. The half-resolution maps of one picture are
// hh x hw pixels; tiles of 32 pixels x 32 channels go through shared memory so that the planar
// f32 side is read / written along rows and the NHWC f16 side along channels.
constexpr int kLatTile = 32;

// psi planar f32 [4C][hh][hw] -> the joined buffer J (NHWC f16, 8C channels a pixel): channel k
// of quarter s = k / C lands at channel k + (s + 1) C, i.e. beside the slot [2sC, 2sC + C) the
// stage's context branch writes, so that J channels [2sC, 2sC + 2C) are cat(t_s, psi_s).
// Grid (ceil(hh*hw / 32), 4C / 32); C a multiple of 32.
__global__ void psi_to_joined_kernel(const float* __restrict__ psi, int C, int npix,
                                     __half* __restrict__ J, int hw, long long pix, long long row) {
  __shared__ float t[kLatTile][kLatTile + 1];
  const int p0 = blockIdx.x * kLatTile, k0 = blockIdx.y * kLatTile;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 256 threads: 8 rows of 32
  for (int r = ty; r < kLatTile; r += 8) {
    const int p = p0 + tx;
    t[r][tx] = p < npix ? __ldg(psi + (long long)(k0 + r) * npix + p) : 0.f;
  }
  __syncthreads();
  const int kd = k0 + (k0 / C + 1) * C;  // the 32-channel block never straddles a quarter
  for (int i = threadIdx.x; i < kLatTile * 16; i += 256) {
    const int pp = i >> 4, pair = i & 15, p = p0 + pp;
    if (p >= npix) continue;
    const int y = p / hw, x = p - y * hw;
    *reinterpret_cast<__half2*>(J + y * row + x * pix + kd + 2 * pair) =
        __floats2half2_rn(t[2 * pair][pp], t[2 * pair + 1][pp]);
  }
}

// One context-model stage's output (mcm.rs:208-247): stage = mean + residual at latent
// position (2y + py, 2x + px) (a position past an odd edge keeps the mean: the reference's
// zero padding), y_hat at that position = stage, and, when ctx is given, the stage as NHWC
// f16 into the context buffer (channels [0, C) of the view). mean planar f32 [C][hh][hw],
// residual / y_hat planar f32 [C][h][w]. Grid (ceil(hh*hw / 32), C / 32).
__global__ void mcm_stage_kernel(const float* __restrict__ mean, const float* __restrict__ res,
                                 int h, int w, int hh, int hw, int py, int px,
                                 float* __restrict__ y, __half* __restrict__ ctx, long long pix,
                                 long long row) {
  __shared__ float t[kLatTile][kLatTile + 1];
  const int npix = hh * hw;
  const int p0 = blockIdx.x * kLatTile, k0 = blockIdx.y * kLatTile;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const long long plane = (long long)h * w;
  for (int r = ty; r < kLatTile; r += 8) {
    const int p = p0 + tx;
    if (p >= npix) continue;
    const int yy = p / hw, xx = p - yy * hw;
    const int sy = 2 * yy + py, sx = 2 * xx + px;
    float v = __ldg(mean + (long long)(k0 + r) * npix + p);
    if (sy < h && sx < w) {
      const long long i = (long long)(k0 + r) * plane + (long long)sy * w + sx;
      v = v + __ldg(res + i);
      y[i] = v;
    }
    t[r][tx] = v;
  }
  if (!ctx) return;
  __syncthreads();
  for (int i = threadIdx.x; i < kLatTile * 16; i += 256) {
    const int pp = i >> 4, pair = i & 15, p = p0 + pp;
    if (p >= npix) continue;
    const int yy = p / hw, xx = p - yy * hw;
    *reinterpret_cast<__half2*>(ctx + yy * row + xx * pix + k0 + 2 * pair) =
        __floats2half2_rn(t[2 * pair][pp], t[2 * pair + 1][pp]);
  }
}

// Without a context model (reconstruct.rs:200-212): y = upshuffle_psi(psi) + residual, where
// sample (Y, X) of channel c takes psi channel STAGE_LUT[(Y % 2) * 2 + X % 2] * C + c at
// (Y / 2, X / 2) (mcm.rs:733-760). One thread per latent sample.
__global__ void upshuffle_add_kernel(const float* __restrict__ psi, const float* __restrict__ res,
                                     int C, int h, int w, float* __restrict__ y) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long plane = (long long)h * w;
  if (idx >= C * plane) return;
  const int c = (int)(idx / plane);
  const int r = (int)(idx - (long long)c * plane);
  const int Y = r / w, X = r - Y * w;
  const int hh = (h + 1) / 2, hw = (w + 1) / 2;
  const int q = (Y & 1) * 2 + (X & 1);
  const int s = q == 0 ? 0 : q == 1 ? 2 : q == 2 ? 3 : 1;  // STAGE_LUT
  const float m = __ldg(psi + ((long long)(s * C + c) * hh + (Y >> 1)) * hw + (X >> 1));
  y[idx] = m + __ldg(res + idx);
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

void launch_normalize_im2col(const float* src, int SH, int SW, int y0, int x0, int h, int w,
                             const TView& dst, cudaStream_t s) {
  const long long total = (long long)dst.n * dst.h * dst.w;
  if (total == 0) return;
  normalize_im2col_kernel<<<blocks_for(total, 256), 256, 0, s>>>(
      src, SH, SW, y0, x0, h, w, dst.p, dst.n, dst.h, dst.w, dst.pix, dst.row, dst.img);
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

void launch_psi_to_joined(const float* psi, int C, int hh, int hw, const TView& J, cudaStream_t s) {
  const int npix = hh * hw;
  dim3 grid((npix + kLatTile - 1) / kLatTile, 4 * C / kLatTile);
  psi_to_joined_kernel<<<grid, 256, 0, s>>>(psi, C, npix, J.p, hw, J.pix, J.row);
}

void launch_mcm_stage(const float* mean, const float* res, int C, int h, int w, int py, int px,
                      float* y, const TView* ctx, cudaStream_t s) {
  const int hh = (h + 1) / 2, hw = (w + 1) / 2;
  dim3 grid((hh * hw + kLatTile - 1) / kLatTile, C / kLatTile);
  mcm_stage_kernel<<<grid, 256, 0, s>>>(mean, res, h, w, hh, hw, py, px, y,
                                        ctx ? ctx->p : nullptr, ctx ? ctx->pix : 0,
                                        ctx ? ctx->row : 0);
}

void launch_upshuffle_add(const float* psi, const float* res, int C, int h, int w, float* y,
                          cudaStream_t s) {
  const long long total = (long long)C * h * w;
  if (total == 0) return;
  upshuffle_add_kernel<<<blocks_for(total, 256), 256, 0, s>>>(psi, res, C, h, w, y);
}

}  // namespace zjai
