// RDLR layer VJPs: the input gradients of the conv layers (src/nn/reference.rs:238-336 through
// src/nn/fast/layers.rs:72-90, 156-160), which the encoder's latent refinement chains through
// the synthesis network. Each is itself a convolution, run on the tcgen05 conv kernel:
//
// * conv2d, stride 1: the full convolution of d_out with the kernel flipped by 180 degrees and
//   its channel axes swapped (padding kh - 1 - pad), per group; the extra zero border of the
//   forward is dropped by the planar epilogue's crop window. Depthwise 3x3 layers run on the
//   depthwise kernel with the flipped taps.
// * conv2d, stride 2: the stride-2 transposed conv with the same weights (a conv weight
//   [oc][c][k][k] is a transposed-conv weight with c outputs), cut to the input extent.
// * conv_transpose2d: the stride-2 conv with the same weights (a transposed-conv weight
//   [c][oc][k][k] is a conv weight with c outputs).
// * ResidualBlock (attention.rs:58-75): conv2's VJP, masked by relu' of the block's tape
//   (conv1's output), conv1's VJP, plus the skip's d_out.
//
// The tensor cores take f16 operands: d_out is scaled by a power of two that brings its largest
// magnitude into [2^13, 2^14) before the f16 conversion (RDLR gradients are small: unscaled
// they would fall into the f16 subnormals) and the epilogue multiplies it back out exactly
// (the depthwise kernel, whose outputs are f16 too, gets [2^7, 2^8)).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "api_common.h"
#include "kernels_attn.h"

namespace zjai {
namespace {

// largest |x| as the bits of a non-negative float (which order like the unsigned integers)
__global__ void amax_kernel(const float* __restrict__ x, size_t n, unsigned* __restrict__ out) {
  float m = 0.f;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    m = fmaxf(m, fabsf(x[i]));
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(m));
}

__global__ void scale_kernel(const float* __restrict__ x, size_t n, float s,
                             float* __restrict__ y) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    y[i] = x[i] * s;
}

// relu' of the tape: g = 0 where the pre-activation p <= 0 (attention.rs:64-69)
__global__ void relu_mask_kernel(float* __restrict__ g, const float* __restrict__ p, size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    if (p[i] <= 0.f) g[i] = 0.f;
}

__global__ void add_kernel(float* __restrict__ a, const float* __restrict__ b, size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    a[i] += b[i];
}

// grid of the grid-stride elementwise kernels
int launch_elementwise_blocks(Ctx* ctx, size_t n) {
  return (int)std::max<size_t>(1, std::min<size_t>((n + 255) / 256, (size_t)ctx->sms * 8));
}

// Power of two that brings amax into [2^(top - 1), 2^top) (1 for zero or non-finite amax).
float grad_scale(float amax, int top) {
  if (!(amax > 0.f) || !std::isfinite(amax)) return 1.f;
  int e;
  std::frexp(amax, &e);  // amax in [2^(e - 1), 2^e)
  return std::ldexp(1.f, std::max(-100, std::min(100, top - e)));
}

// d_out (device, planar [c][h][w]) scaled by the power of two of grad_scale(max |d_out|, top)
// and converted to NHWC f16 in t; *s receives the scale.
int stage_grad(Ctx* ctx, const float* d, int c, int h, int w, int top, TView* t, float* s) {
  const size_t n = (size_t)c * h * w;
  unsigned* dmax = static_cast<unsigned*>(ctx->arena.alloc(sizeof(unsigned)));
  float* scaled = static_cast<float*>(ctx->arena.alloc(n * sizeof(float)));
  if (!dmax || !scaled) return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (VJP d_out)");
  ZJAI_TRY(cuda_check(cudaMemsetAsync(dmax, 0, sizeof(unsigned), ctx->stream), "memset"));
  const int blocks = launch_elementwise_blocks(ctx, n);
  amax_kernel<<<blocks, 256, 0, ctx->stream>>>(d, n, dmax);
  ctx->launches++;
  unsigned bits = 0;
  ZJAI_TRY(cuda_check(cudaMemcpyAsync(&bits, dmax, sizeof(unsigned), cudaMemcpyDeviceToHost,
                                      ctx->stream),
                      "VJP d_out range"));
  ZJAI_TRY(cuda_check(cudaStreamSynchronize(ctx->stream), "VJP d_out range"));
  float amax;
  std::memcpy(&amax, &bits, sizeof amax);
  *s = grad_scale(amax, top);
  scale_kernel<<<blocks, 256, 0, ctx->stream>>>(d, n, *s, scaled);
  ctx->launches++;
  ZJAI_TRY(cuda_check(cudaGetLastError(), "VJP d_out scale"));
  return planar_to_tensor(ctx, scaled, c, h, w, t);
}

// run a packed layer on the staged gradient into planar din [c][h][w]: output pixel (0, 0) is
// input pixel (-y0, -x0), pixels outside [0, h) x [0, w) dropped
int run_into(Ctx* ctx, ConvLayer& L, float s, const TView& t, float* din, int h, int w, int y0,
             int x0) {
  L.scale /= s;
  ConvOut o;
  o.planar = true;
  o.pout = din;
  o.p_plane = (long long)h * w;
  o.p_row = w;
  o.py0 = -y0;
  o.px0 = -x0;
  o.cy0 = 0;
  o.cy1 = h;
  o.cx0 = 0;
  o.cx1 = w;
  return run_conv(ctx, L, t, o);
}

// the input gradient of a stride-1 conv (weight [oc][c/groups][kh][kw], host) from the device
// planar gradient dd [oc][oh][ow] into the device planar din [c][h][w] of an input with zero
// border (pt, pl) in front: the flipped, channel-swapped kernel with padding k - 1 - pad
int conv_vjp_s1(Ctx* ctx, const float* dd, int oc, int oh, int ow, const float* hw, int c, int kh,
                int kw, int pad_h, int pad_w, int groups, int h, int w, int pt, int pl,
                float* din) {
  const int icg = c / groups, ocg = oc / groups;
  // W'[g icg + ci][co][ky][kx] = w[g ocg + co][ci][kh - 1 - ky][kw - 1 - kx]
  std::vector<float> wt((size_t)c * ocg * kh * kw);
  for (int g = 0; g < groups; ++g)
    for (int co = 0; co < ocg; ++co)
      for (int ci = 0; ci < icg; ++ci)
        for (int ky = 0; ky < kh; ++ky)
          for (int kx = 0; kx < kw; ++kx)
            wt[((((size_t)g * icg + ci) * ocg + co) * kh + ky) * kw + kx] =
                hw[((((size_t)g * ocg + co) * icg + ci) * kh + kh - 1 - ky) * kw + kw - 1 - kx];
  ConvLayer L;
  ZJAI_TRY(pack_conv(ctx, &L, wt.data(), nullptr, oc, c, kh, kw, 1, kh - 1 - pad_h,
                     kw - 1 - pad_w, groups, nullptr, 1));
  LayerGuard guard(&L);
  TView t;
  float s;
  ZJAI_TRY(stage_grad(ctx, dd, oc, oh, ow, 14, &t, &s));
  return run_into(ctx, L, s, t, din, h, w, pt, pl);
}

}  // namespace
}  // namespace zjai

using namespace zjai;

extern "C" {

int zjai_conv2d_backward(zjai_ctx* ctx, const float* dout, int oc, int oh, int ow,
                         const float* weight, int c, int kh, int kw, int stride, int pad_h,
                         int pad_w, int groups, const int* extra, int h, int w, float* din,
                         int mem) {
  ZJAI_TRY(ctx_enter(ctx));
  if (!dout || !weight || !din || c <= 0 || oc <= 0 || h <= 0 || w <= 0 || kh <= 0 || kw <= 0)
    return fail(ZJAI_INVALID_ARGUMENT, "conv2d_backward: bad arguments");
  if (mem != ZJAI_MEM_HOST && mem != ZJAI_MEM_DEVICE)
    return fail(ZJAI_INVALID_ARGUMENT, "mem must be HOST or DEVICE");
  if (groups <= 0 || c % groups || oc % groups)
    return fail(ZJAI_INVALID_ARGUMENT, "conv2d_backward: groups");
  if (stride != 1 && stride != 2) return fail(ZJAI_UNSUPPORTED, "conv2d_backward: stride 1 or 2");
  const int pt = extra ? extra[0] : 0, pl = extra ? extra[1] : 0;
  const int pb = extra ? extra[2] : 0, pr = extra ? extra[3] : 0;
  if (pt < 0 || pl < 0 || pb < 0 || pr < 0)
    return fail(ZJAI_INVALID_ARGUMENT, "conv2d_backward: negative border");
  const int H = h + pt + pb, W = w + pl + pr;
  if (oh != (H + 2 * pad_h - kh) / stride + 1 || ow != (W + 2 * pad_w - kw) / stride + 1 ||
      H + 2 * pad_h < kh || W + 2 * pad_w < kw)
    return fail(ZJAI_INVALID_ARGUMENT, "conv2d_backward: d_out extent is not the layer's output");
  const bool depthwise = groups == c && oc == c && kh == 3 && kw == 3 && stride == 1 &&
                         pad_h == 1 && pad_w == 1 && !(pt | pl | pb | pr) && c % 8 == 0;
  if (stride == 1 && !depthwise && (pad_h > kh - 1 || pad_w > kw - 1))
    return fail(ZJAI_UNSUPPORTED, "conv2d_backward: padding wider than the kernel");
  if (stride == 2 && (groups != 1 || kh != kw || pad_h != pad_w || pt | pl | pb | pr))
    return fail(ZJAI_UNSUPPORTED,
                "conv2d_backward: stride 2 needs a dense square kernel and no extra border");
  if (stride == 2 && pad_h >= kh)
    return fail(ZJAI_UNSUPPORTED, "conv2d_backward: padding wider than the kernel");
  ArenaScope scope(ctx);
  const int icg = c / groups;
  std::vector<float> wbuf;
  const float* hw;
  ZJAI_TRY(fetch_host(weight, (size_t)oc * icg * kh * kw, mem, &wbuf, &hw));
  const float* dd;
  ZJAI_TRY(stage_in(ctx, dout, (size_t)oc * oh * ow, mem, &dd));
  float* ddin;
  const size_t nin = (size_t)c * h * w;
  ZJAI_TRY(stage_out_alloc(ctx, din, nin, mem, &ddin));
  if (depthwise) {
    // flipped taps [c][9]; the depthwise kernel stores f16, so the scale leaves room for the
    // sum of nine products
    std::vector<float> flip((size_t)c * 9);
    for (int ch = 0; ch < c; ++ch)
      for (int t = 0; t < 9; ++t) flip[(size_t)ch * 9 + t] = hw[(size_t)ch * 9 + 8 - t];
    float* dwt = static_cast<float*>(ctx->arena.alloc(flip.size() * sizeof(float)));
    if (!dwt) return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (VJP weights)");
    ZJAI_TRY(cuda_check(cudaMemcpyAsync(dwt, flip.data(), flip.size() * sizeof(float),
                                        cudaMemcpyHostToDevice, ctx->stream),
                        "VJP weights H2D"));
    TView t, o;
    float s;
    ZJAI_TRY(stage_grad(ctx, dd, oc, oh, ow, 8, &t, &s));
    ZJAI_TRY(alloc_tensor(ctx, 1, h, w, c, &o));
    ZJAI_TRY(launch_dw3x3(ctx, t, o, dwt, false, ctx->stream));
    float* tmp = static_cast<float*>(ctx->arena.alloc(nin * sizeof(float)));
    if (!tmp) return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (VJP output)");
    launch_nhwc_to_planar(o, tmp, ctx->stream);
    scale_kernel<<<launch_elementwise_blocks(ctx, nin), 256, 0, ctx->stream>>>(tmp, nin, 1.f / s,
                                                                             ddin);
    ctx->launches += 3;
    // `flip` is a host vector: its copy must have been read before it goes
    ZJAI_TRY(cuda_check(cudaStreamSynchronize(ctx->stream), "VJP depthwise"));
  } else if (stride == 1) {
    ZJAI_TRY(conv_vjp_s1(ctx, dd, oc, oh, ow, hw, c, kh, kw, pad_h, pad_w, groups, h, w, pt, pl,
                         ddin));
  } else {
    // out_pad 1: the transposed conv covers the input extent (one row / column beyond it where
    // the forward's output size rounded down, dropped by the crop)
    ConvLayer L;
    ZJAI_TRY(pack_convT(ctx, &L, hw, nullptr, oc, c, kh, pad_h, 1, 1));
    LayerGuard guard(&L);
    TView t;
    float s;
    ZJAI_TRY(stage_grad(ctx, dd, oc, oh, ow, 14, &t, &s));
    ZJAI_TRY(run_into(ctx, L, s, t, ddin, h, w, 0, 0));
  }
  ZJAI_TRY(stage_out_finish(ctx, din, ddin, nin, mem));
  return ctx_check_status(ctx);
}

int zjai_conv_transpose2d_backward(zjai_ctx* ctx, const float* dout, int oc, int oh, int ow,
                                   const float* weight, int c, int k, int pad, int h, int w,
                                   float* din, int mem) {
  ZJAI_TRY(ctx_enter(ctx));
  if (!dout || !weight || !din || c <= 0 || oc <= 0 || h <= 0 || w <= 0 || k <= 0 || pad < 0)
    return fail(ZJAI_INVALID_ARGUMENT, "conv_transpose2d_backward: bad arguments");
  if (mem != ZJAI_MEM_HOST && mem != ZJAI_MEM_DEVICE)
    return fail(ZJAI_INVALID_ARGUMENT, "mem must be HOST or DEVICE");
  // the stride-2 conv of d_out gives floor((oh + 2 pad - k) / 2) + 1 rows: the input's
  if (oh + 2 * pad < k || ow + 2 * pad < k || (oh + 2 * pad - k) / 2 + 1 != h ||
      (ow + 2 * pad - k) / 2 + 1 != w)
    return fail(ZJAI_INVALID_ARGUMENT,
                "conv_transpose2d_backward: d_out extent is not the layer's output");
  ArenaScope scope(ctx);
  std::vector<float> wbuf;
  const float* hw;
  ZJAI_TRY(fetch_host(weight, (size_t)c * oc * k * k, mem, &wbuf, &hw));
  const float* dd;
  ZJAI_TRY(stage_in(ctx, dout, (size_t)oc * oh * ow, mem, &dd));
  float* ddin;
  const size_t nin = (size_t)c * h * w;
  ZJAI_TRY(stage_out_alloc(ctx, din, nin, mem, &ddin));
  ConvLayer L;
  // weight [c][oc][k][k] read as a conv weight with c outputs and oc inputs
  ZJAI_TRY(pack_conv(ctx, &L, hw, nullptr, oc, c, k, k, 2, pad, pad, 1, nullptr, 1));
  LayerGuard guard(&L);
  TView t;
  float s;
  ZJAI_TRY(stage_grad(ctx, dd, oc, oh, ow, 14, &t, &s));
  ZJAI_TRY(run_into(ctx, L, s, t, ddin, h, w, 0, 0));
  ZJAI_TRY(stage_out_finish(ctx, din, ddin, nin, mem));
  return ctx_check_status(ctx);
}

int zjai_residual_block_backward(zjai_ctx* ctx, const float* dout, const float* conv1_out,
                                 int c, int h, int w, const float* w1, const float* w2,
                                 float* din, int mem) {
  ZJAI_TRY(ctx_enter(ctx));
  if (!dout || !conv1_out || !w1 || !w2 || !din || c <= 0 || h <= 0 || w <= 0)
    return fail(ZJAI_INVALID_ARGUMENT, "residual_block_backward: bad arguments");
  if (mem != ZJAI_MEM_HOST && mem != ZJAI_MEM_DEVICE)
    return fail(ZJAI_INVALID_ARGUMENT, "mem must be HOST or DEVICE");
  ArenaScope scope(ctx);
  const size_t n = (size_t)c * h * w, nw = (size_t)c * c * 9;
  std::vector<float> b1, b2;
  const float *h1, *h2;
  ZJAI_TRY(fetch_host(w1, nw, mem, &b1, &h1));
  ZJAI_TRY(fetch_host(w2, nw, mem, &b2, &h2));
  const float *dd, *dp;
  ZJAI_TRY(stage_in(ctx, dout, n, mem, &dd));
  ZJAI_TRY(stage_in(ctx, conv1_out, n, mem, &dp));
  float* ddin;
  ZJAI_TRY(stage_out_alloc(ctx, din, n, mem, &ddin));
  float* d = static_cast<float*>(ctx->arena.alloc(n * sizeof(float)));
  if (!d) return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (residual block VJP)");
  const int blocks = launch_elementwise_blocks(ctx, n);
  // conv2^T d_out, masked by relu'(conv1_out); conv1^T of that, plus the skip's d_out
  ZJAI_TRY(conv_vjp_s1(ctx, dd, c, h, w, h2, c, 3, 3, 1, 1, 1, h, w, 0, 0, d));
  relu_mask_kernel<<<blocks, 256, 0, ctx->stream>>>(d, dp, n);
  ZJAI_TRY(conv_vjp_s1(ctx, d, c, h, w, h1, c, 3, 3, 1, 1, 1, h, w, 0, 0, ddin));
  add_kernel<<<blocks, 256, 0, ctx->stream>>>(ddin, dd, n);
  ctx->launches += 2;
  ZJAI_TRY(cuda_check(cudaGetLastError(), "residual block VJP"));
  ZJAI_TRY(stage_out_finish(ctx, din, ddin, n, mem));
  return ctx_check_status(ctx);
}

}  // extern "C"
