// RDLR VJPs: the input gradients of the synthesis network's layers and blocks
// (src/nn/reference.rs:238-336 through src/nn/fast/layers.rs:72-90, 156-160; math.rs:838-913;
// attention.rs:58-75, 182-223), which the encoder's latent refinement chains through the
// network. The conv VJPs are themselves convolutions, run on the tcgen05 conv kernel:
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
// * the transformer block's other pieces: the ELU gate (math.rs:838-858), the channel layer
//   norm (math.rs:860-913) and the channel attention (math.rs:668-836), as elementwise,
//   per-position and row-reduction kernels; and the block itself (attention.rs:435-480): the
//   feed-forward branch added to d_out, the attention branch of that added to it.
// * CAB (attention.rs:182-223): d_out split into the trunk's (times sigma) and the mask's
//   (times trunk and sigma'), the trunk's two residual blocks, the mask chain back to full
//   resolution (upscale, two residual blocks, subscale), and the skip.
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

// the input gradient of a stride-2 3x3-style conv (weight [oc][c][k][k], host, padding pad)
// from dd [oc][oh][ow] into din [c][h][w]: the stride-2 transposed conv over the same weights
// with output padding 1, cut to the input extent
int conv_vjp_s2(Ctx* ctx, const float* dd, int oc, int oh, int ow, const float* hw, int c, int k,
                int pad, int h, int w, float* din) {
  ConvLayer L;
  ZJAI_TRY(pack_convT(ctx, &L, hw, nullptr, oc, c, k, pad, 1, 1));
  LayerGuard guard(&L);
  TView t;
  float s;
  ZJAI_TRY(stage_grad(ctx, dd, oc, oh, ow, 14, &t, &s));
  return run_into(ctx, L, s, t, din, h, w, 0, 0);
}

// the input gradient of a stride-2 transposed conv (weight [c][oc][k][k], host) from dd
// [oc][oh][ow] into din [c][h][w]: the stride-2 conv over the same weights
int convT_vjp(Ctx* ctx, const float* dd, int oc, int oh, int ow, const float* hw, int c, int k,
              int pad, int h, int w, float* din) {
  ConvLayer L;
  ZJAI_TRY(pack_conv(ctx, &L, hw, nullptr, oc, c, k, k, 2, pad, pad, 1, nullptr, 1));
  LayerGuard guard(&L);
  TView t;
  float s;
  ZJAI_TRY(stage_grad(ctx, dd, oc, oh, ow, 14, &t, &s));
  return run_into(ctx, L, s, t, din, h, w, 0, 0);
}

// ResidualBlock::backward (attention.rs:58-75) on device planar arrays: din = dd +
// conv1^T(relu'(tape) . conv2^T dd); host weights [c][c][3][3]
int rb_vjp(Ctx* ctx, const float* dd, const float* tape, const float* h1, const float* h2, int c,
           int h, int w, float* din) {
  const size_t n = (size_t)c * h * w;
  const size_t mark = ctx->arena.mark();
  float* d = static_cast<float*>(ctx->arena.alloc(n * sizeof(float)));
  if (!d) return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (residual block VJP)");
  const int blocks = launch_elementwise_blocks(ctx, n);
  ZJAI_TRY(conv_vjp_s1(ctx, dd, c, h, w, h2, c, 3, 3, 1, 1, 1, h, w, 0, 0, d));
  relu_mask_kernel<<<blocks, 256, 0, ctx->stream>>>(d, tape, n);
  ZJAI_TRY(conv_vjp_s1(ctx, d, c, h, w, h1, c, 3, 3, 1, 1, 1, h, w, 0, 0, din));
  add_kernel<<<blocks, 256, 0, ctx->stream>>>(din, dd, n);
  ctx->launches += 2;
  ZJAI_TRY(cuda_check(cudaGetLastError(), "residual block VJP"));
  // every use of d is queued on the stream, which orders its next user after them
  ctx->arena.release(mark);
  return ZJAI_OK;
}

// Cab::backward's split of d_out (attention.rs:185-203, 209-211): d_trunk = o . sig and
// d_sig = (o . trunk) . (sig . (1 - sig)), each product rounded on its own
__global__ void cab_split_kernel(const float* __restrict__ o, const float* __restrict__ sig,
                                 const float* __restrict__ trunk, size_t n,
                                 float* __restrict__ d_trunk, float* __restrict__ d_sig) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const float s = sig[i];
    d_trunk[i] = __fmul_rn(o[i], s);
    d_sig[i] = __fmul_rn(__fmul_rn(o[i], trunk[i]), __fmul_rn(s, __fsub_rn(1.f, s)));
  }
}

// elu_gate_backward (math.rs:838-858), one element per thread: d_a = (elu'(a) . b) . d,
// d_b = elu(a) . d
__global__ void elu_gate_bwd_kernel(const float* __restrict__ d, const float* __restrict__ a,
                                    const float* __restrict__ b, size_t n,
                                    float* __restrict__ d_a, float* __restrict__ d_b) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const float av = a[i];
    const float e = av > 0.f ? 0.f : expf(av);
    const float elu = av > 0.f ? av : __fsub_rn(e, 1.f);
    const float delu = av > 0.f ? 1.f : e;
    d_a[i] = __fmul_rn(__fmul_rn(delu, b[i]), d[i]);
    d_b[i] = __fmul_rn(elu, d[i]);
  }
}

// layer_norm_channels_backward (math.rs:860-913), one position per thread over planar
// [c][n]: the forward's mean and variance in f64 (channel order), its f32 deviation and
// normalised x, then d_x[c] = (dy[c] - s1 / c - xn[c] . s2 / c) / sigma with dy = d . w and the
// f64 sums s1, s2; adjacent threads read adjacent positions of each channel plane
__global__ void ln_bwd_kernel(const float* __restrict__ d, const float* __restrict__ x, int c,
                              long long n, const float* __restrict__ wt,
                              float* __restrict__ dx) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    double mean = 0.0, var = 0.0;
    for (int ch = 0; ch < c; ++ch) mean += (double)__ldg(x + ch * n + i);
    mean /= c;
    for (int ch = 0; ch < c; ++ch) {
      const double dv = (double)__ldg(x + ch * n + i) - mean;
      var += dv * dv;
    }
    const float sig = __fsqrt_rn(__fadd_rn((float)(var / c), 1e-5f));
    const float m = (float)mean;
    double s1 = 0.0, s2 = 0.0;
    for (int ch = 0; ch < c; ++ch) {
      const float xn = __fdiv_rn(__fsub_rn(__ldg(x + ch * n + i), m), sig);
      const float dy = __fmul_rn(__ldg(d + ch * n + i), __ldg(wt + ch));
      s1 += (double)dy;
      s2 += (double)dy * (double)xn;
    }
    const float m1 = __fdiv_rn((float)s1, (float)c), m2 = __fdiv_rn((float)s2, (float)c);
    for (int ch = 0; ch < c; ++ch) {
      const float xn = __fdiv_rn(__fsub_rn(__ldg(x + ch * n + i), m), sig);
      const float dy = __fmul_rn(__ldg(d + ch * n + i), __ldg(wt + ch));
      dx[ch * n + i] = __fdiv_rn(__fsub_rn(__fsub_rn(dy, m1), __fmul_rn(xn, m2)), sig);
    }
  }
}

// ---- channel_attention_backward (math.rs:668-836) ----------------------------------------
// One block per pair: the dot product over the pixels of rows a[ra] and b[rb] (f64 partial
// sums, a shared-memory tree): out[o] = sum_l a[ra][l] b[rb][l], rows n floats apart.
__global__ void __launch_bounds__(256) row_dot_kernel(const float* __restrict__ a,
                                                      const float* __restrict__ b,
                                                      const int* __restrict__ pairs, long long n,
                                                      double* __restrict__ out) {
  __shared__ double part[256];
  const int ra = pairs[2 * blockIdx.x], rb = pairs[2 * blockIdx.x + 1];
  const float* x = a + (long long)ra * n;
  const float* y = b + (long long)rb * n;
  double s = 0.0;
  for (long long l = threadIdx.x; l < n; l += blockDim.x) s += (double)x[l] * (double)y[l];
  part[threadIdx.x] = s;
  __syncthreads();
  for (int o = 128; o > 0; o >>= 1) {
    if ((int)threadIdx.x < o) part[threadIdx.x] += part[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) out[blockIdx.x] = part[0];
}

// q and k rows divided by their clamped L2 norms (norm2: the rows' squared norms)
__global__ void normalise_rows_kernel(const float* __restrict__ qkv, const double* __restrict__ norm2,
                                      int rows, long long n, float* __restrict__ qk,
                                      float* __restrict__ norms) {
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < rows * n;
       e += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(e / n);
    const float nv = fmaxf((float)sqrt(norm2[r]), 1e-12f);
    qk[e] = __fdiv_rn(qkv[e], nv);
    if (e % n == 0) norms[r] = nv;
  }
}

// the row softmax VJP in place on da [dim][c] (= d_out . v^T): da = a . (da - sum_j a_j da_j),
// the row sum in f64
__global__ void softmax_vjp_kernel(const double* __restrict__ dots, const float* __restrict__ attn,
                                   int dim, int c, float* __restrict__ da) {
  const int ri = blockIdx.x * blockDim.x + threadIdx.x;
  if (ri >= dim) return;
  double sdot = 0.0;
  for (int j = 0; j < c; ++j) {
    const float v = (float)dots[(long long)ri * c + j];
    da[(long long)ri * c + j] = v;
    sdot += (double)attn[(long long)ri * c + j] * (double)v;
  }
  for (int j = 0; j < c; ++j) {
    const long long e = (long long)ri * c + j;
    da[e] = __fmul_rn(attn[e], __fsub_rn(da[e], (float)sdot));
  }
}

// acc rows of dq (T . da . k), dk (T . da^T . q) and dv (attn^T . d_out, final), one pixel of one
// row per thread, the c terms in order
__global__ void attn_grad_acc_kernel(const float* __restrict__ qk, const float* __restrict__ dout,
                                     const float* __restrict__ da, const float* __restrict__ attn,
                                     const float* __restrict__ temp, int dim, int c, long long n,
                                     float* __restrict__ out) {
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < 3LL * dim * n;
       e += (long long)gridDim.x * blockDim.x) {
    const int ri = (int)(e / n);
    const long long l = e - (long long)ri * n;
    double acc = 0.0;
    if (ri < dim) {
      const int head = ri / c;
      const float* k = qk + (long long)dim * n;
      for (int i = 0; i < c; ++i)
        acc += (double)__fmul_rn(temp[head], da[(long long)ri * c + i]) *
               (double)k[(long long)(head * c + i) * n + l];
    } else if (ri < 2 * dim) {
      const int head = (ri - dim) / c, j = (ri - dim) % c;
      for (int i = 0; i < c; ++i)
        acc += (double)__fmul_rn(temp[head], da[(long long)(head * c + i) * c + j]) *
               (double)qk[(long long)(head * c + i) * n + l];
    } else {
      const int head = (ri - 2 * dim) / c, j = (ri - 2 * dim) % c;
      for (int i = 0; i < c; ++i)
        acc += (double)attn[(long long)(head * c + i) * c + j] *
               (double)dout[(long long)(head * c + i) * n + l];
    }
    out[e] = (float)acc;
  }
}

// the L2-norm backward of the q / k rows: out = (acc - <x, acc> x) / |x|
__global__ void l2_backward_kernel(const float* __restrict__ qk, const double* __restrict__ proj,
                                   const float* __restrict__ norms, int rows, long long n,
                                   float* __restrict__ out) {
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < rows * n;
       e += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(e / n);
    out[e] = (float)(((double)out[e] - proj[r] * (double)qk[e]) / (double)norms[r]);
  }
}

// the input gradient of a depthwise 3x3 conv (padding 1, weight [c][1][3][3], host) from the
// device planar dd [c][h][w] into din: the depthwise kernel with the flipped taps; its f16
// outputs get the scale [2^7, 2^8), undone by scale_kernel (c a multiple of 8)
int dw_vjp(Ctx* ctx, const float* dd, int c, int h, int w, const float* hw, float* din) {
  const size_t nin = (size_t)c * h * w;
  const size_t mark = ctx->arena.mark();
  std::vector<float> flip((size_t)c * 9);
  for (int ch = 0; ch < c; ++ch)
    for (int t = 0; t < 9; ++t) flip[(size_t)ch * 9 + t] = hw[(size_t)ch * 9 + 8 - t];
  float* dwt = static_cast<float*>(ctx->arena.alloc(flip.size() * sizeof(float)));
  float* tmp = static_cast<float*>(ctx->arena.alloc(nin * sizeof(float)));
  if (!dwt || !tmp) return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (depthwise VJP)");
  ZJAI_TRY(cuda_check(cudaMemcpyAsync(dwt, flip.data(), flip.size() * sizeof(float),
                                      cudaMemcpyHostToDevice, ctx->stream),
                      "VJP weights H2D"));
  TView t, o;
  float s;
  ZJAI_TRY(stage_grad(ctx, dd, c, h, w, 8, &t, &s));
  ZJAI_TRY(alloc_tensor(ctx, 1, h, w, c, &o));
  ZJAI_TRY(launch_dw3x3(ctx, t, o, dwt, false, ctx->stream));
  launch_nhwc_to_planar(o, tmp, ctx->stream);
  scale_kernel<<<launch_elementwise_blocks(ctx, nin), 256, 0, ctx->stream>>>(tmp, nin, 1.f / s,
                                                                           din);
  ctx->launches += 3;
  // `flip` is a host vector: its copy must have been read before it goes
  ZJAI_TRY(cuda_check(cudaStreamSynchronize(ctx->stream), "VJP depthwise"));
  ctx->arena.release(mark);
  return ZJAI_OK;
}

// channel_attention_backward (math.rs:668-836) on device arrays: qkv [3 dim][n], temp [heads],
// attn [dim][c], dout [dim][n] -> out [3 dim][n]
int attn_vjp(Ctx* ctx, const float* dq, int c3, long long n, int heads, const float* dt,
             const float* da_in, const float* dd, float* out) {
  const int dim = c3 / 3, c = dim / heads;
  const size_t mark = ctx->arena.mark();
  // the row pairs of the three dot-product passes: q, k norms (2 dim), d_out . v (dim c), and
  // the projections <x, acc> of the dq / dk rows (2 dim)
  const int np_norm = 2 * dim, np_dot = dim * c;
  std::vector<int> pairs(2 * (size_t)(np_norm + np_dot + np_norm));
  for (int r = 0; r < np_norm; ++r) pairs[2 * r] = pairs[2 * r + 1] = r;
  for (int ri = 0; ri < dim; ++ri)
    for (int j = 0; j < c; ++j) {
      const size_t p = (size_t)np_norm + (size_t)ri * c + j;
      pairs[2 * p] = ri;
      pairs[2 * p + 1] = (ri / c) * c + j;
    }
  for (int r = 0; r < np_norm; ++r) {
    const size_t p = (size_t)np_norm + np_dot + r;
    pairs[2 * p] = pairs[2 * p + 1] = r;
  }
  int* dpairs = static_cast<int*>(ctx->arena.alloc(pairs.size() * sizeof(int)));
  double* dots =
      static_cast<double*>(ctx->arena.alloc((size_t)(2 * np_norm + np_dot) * sizeof(double)));
  float* qk = static_cast<float*>(ctx->arena.alloc((size_t)2 * dim * n * sizeof(float)));
  float* norms = static_cast<float*>(ctx->arena.alloc((size_t)2 * dim * sizeof(float)));
  float* dam = static_cast<float*>(ctx->arena.alloc((size_t)dim * c * sizeof(float)));
  if (!dpairs || !dots || !qk || !norms || !dam)
    return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (attention VJP)");
  ZJAI_TRY(cuda_check(cudaMemcpyAsync(dpairs, pairs.data(), pairs.size() * sizeof(int),
                                      cudaMemcpyHostToDevice, ctx->stream),
                      "attention VJP pairs"));
  const int eb = (int)std::min<long long>((3LL * dim * n + 255) / 256, (long long)ctx->sms * 8);
  row_dot_kernel<<<np_norm, 256, 0, ctx->stream>>>(dq, dq, dpairs, n, dots);
  normalise_rows_kernel<<<eb, 256, 0, ctx->stream>>>(dq, dots, 2 * dim, n, qk, norms);
  row_dot_kernel<<<np_dot, 256, 0, ctx->stream>>>(dd, dq + 2LL * dim * n, dpairs + 2 * np_norm, n,
                                                  dots + np_norm);
  softmax_vjp_kernel<<<(dim + 127) / 128, 128, 0, ctx->stream>>>(dots + np_norm, da_in, dim, c,
                                                                 dam);
  attn_grad_acc_kernel<<<eb, 256, 0, ctx->stream>>>(qk, dd, dam, da_in, dt, dim, c, n, out);
  // <x, acc> of each dq / dk row: x = the normalised q / k row, acc = that row of out
  row_dot_kernel<<<np_norm, 256, 0, ctx->stream>>>(qk, out, dpairs + 2 * (np_norm + np_dot), n,
                                                   dots + np_norm + np_dot);
  l2_backward_kernel<<<eb, 256, 0, ctx->stream>>>(qk, dots + np_norm + np_dot, norms, 2 * dim, n,
                                                  out);
  ctx->launches += 7;
  ZJAI_TRY(cuda_check(cudaGetLastError(), "attention VJP"));
  // `pairs` is a host vector: its copy must have been read before it goes
  ZJAI_TRY(cuda_check(cudaStreamSynchronize(ctx->stream), "attention VJP"));
  ctx->arena.release(mark);
  return ZJAI_OK;
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
    ZJAI_TRY(dw_vjp(ctx, dd, c, h, w, hw, ddin));
  } else if (stride == 1) {
    ZJAI_TRY(conv_vjp_s1(ctx, dd, oc, oh, ow, hw, c, kh, kw, pad_h, pad_w, groups, h, w, pt, pl,
                         ddin));
  } else {
    ZJAI_TRY(conv_vjp_s2(ctx, dd, oc, oh, ow, hw, c, kh, pad_h, h, w, ddin));
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
  // weight [c][oc][k][k] read as a conv weight with c outputs and oc inputs
  ZJAI_TRY(convT_vjp(ctx, dd, oc, oh, ow, hw, c, k, pad, h, w, ddin));
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
  ZJAI_TRY(rb_vjp(ctx, dd, dp, h1, h2, c, h, w, ddin));
  ZJAI_TRY(stage_out_finish(ctx, din, ddin, n, mem));
  return ctx_check_status(ctx);
}

int zjai_cab_backward(zjai_ctx* ctx, const float* dout, int c, int h, int w,
                      const zjai_cab_tape* tape, const zjai_cab_weights* wts, float* din,
                      int mem) {
  ZJAI_TRY(ctx_enter(ctx));
  if (!dout || !tape || !wts || !din || c <= 0 || h <= 0 || w <= 0)
    return fail(ZJAI_INVALID_ARGUMENT, "cab_backward: bad arguments");
  if (mem != ZJAI_MEM_HOST && mem != ZJAI_MEM_DEVICE)
    return fail(ZJAI_INVALID_ARGUMENT, "mem must be HOST or DEVICE");
  // the mask branch runs at the subscale conv's output extent, which the upscale doubles back
  const int mh = (h - 1) / 2 + 1, mw = (w - 1) / 2 + 1;
  if (2 * mh != h || 2 * mw != w)
    return fail(ZJAI_INVALID_ARGUMENT, "CAB: odd feature map size");
  const float* tp[6] = {tape->trunk_pre, tape->sig, tape->rb_c1[0], tape->rb_c1[1],
                        tape->mask_c1[0], tape->mask_c1[1]};
  const float* wp[10] = {wts->trunk[0][0], wts->trunk[0][1], wts->trunk[1][0], wts->trunk[1][1],
                         wts->subscale,    wts->mask2[0],    wts->mask2[1],    wts->mask3[0],
                         wts->mask3[1],    wts->upscale};
  for (const float* p : tp)
    if (!p) return fail(ZJAI_INVALID_ARGUMENT, "cab_backward: missing tape array");
  for (const float* p : wp)
    if (!p) return fail(ZJAI_INVALID_ARGUMENT, "cab_backward: missing weight");
  ArenaScope scope(ctx);
  const size_t n = (size_t)c * h * w, nm = (size_t)c * mh * mw, nw = (size_t)c * c * 9;
  std::vector<float> wb[10];
  const float* hw[10];
  for (int i = 0; i < 10; ++i) ZJAI_TRY(fetch_host(wp[i], nw, mem, &wb[i], &hw[i]));
  const float *dd, *dt[6];
  ZJAI_TRY(stage_in(ctx, dout, n, mem, &dd));
  for (int i = 0; i < 6; ++i) ZJAI_TRY(stage_in(ctx, tp[i], i < 4 ? n : nm, mem, &dt[i]));
  float* ddin;
  ZJAI_TRY(stage_out_alloc(ctx, din, n, mem, &ddin));
  float* d_trunk = static_cast<float*>(ctx->arena.alloc(n * sizeof(float)));
  float* d_sig = static_cast<float*>(ctx->arena.alloc(n * sizeof(float)));
  float* t1 = static_cast<float*>(ctx->arena.alloc(n * sizeof(float)));
  float* m1 = static_cast<float*>(ctx->arena.alloc(nm * sizeof(float)));
  float* m2 = static_cast<float*>(ctx->arena.alloc(nm * sizeof(float)));
  if (!d_trunk || !d_sig || !t1 || !m1 || !m2)
    return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (CAB VJP)");
  const int blocks = launch_elementwise_blocks(ctx, n);
  cab_split_kernel<<<blocks, 256, 0, ctx->stream>>>(dd, dt[1], dt[0], n, d_trunk, d_sig);
  ctx->launches++;
  // trunk branch: residual blocks 1 then 0
  ZJAI_TRY(rb_vjp(ctx, d_trunk, dt[3], hw[2], hw[3], c, h, w, t1));
  ZJAI_TRY(rb_vjp(ctx, t1, dt[2], hw[0], hw[1], c, h, w, ddin));
  // mask branch: upscale (transposed conv 3x3, padding 1), mask3, mask2, subscale (3x3 stride 2)
  ZJAI_TRY(convT_vjp(ctx, d_sig, c, h, w, hw[9], c, 3, 1, mh, mw, m1));
  ZJAI_TRY(rb_vjp(ctx, m1, dt[5], hw[7], hw[8], c, mh, mw, m2));
  ZJAI_TRY(rb_vjp(ctx, m2, dt[4], hw[5], hw[6], c, mh, mw, m1));
  ZJAI_TRY(conv_vjp_s2(ctx, m1, c, mh, mw, hw[4], c, 3, 1, h, w, t1));
  // d_x = trunk branch + mask branch + d_out (the skip), in that order
  add_kernel<<<blocks, 256, 0, ctx->stream>>>(ddin, t1, n);
  add_kernel<<<blocks, 256, 0, ctx->stream>>>(ddin, dd, n);
  ctx->launches += 2;
  ZJAI_TRY(cuda_check(cudaGetLastError(), "CAB VJP"));
  ZJAI_TRY(stage_out_finish(ctx, din, ddin, n, mem));
  return ctx_check_status(ctx);
}

int zjai_elu_gate_backward(zjai_ctx* ctx, const float* d, const float* a, const float* b,
                           int64_t n, float* d_a, float* d_b, int mem) {
  ZJAI_TRY(ctx_enter(ctx));
  if (!d || !a || !b || !d_a || !d_b || n <= 0)
    return fail(ZJAI_INVALID_ARGUMENT, "elu_gate_backward: bad arguments");
  if (mem != ZJAI_MEM_HOST && mem != ZJAI_MEM_DEVICE)
    return fail(ZJAI_INVALID_ARGUMENT, "mem must be HOST or DEVICE");
  ArenaScope scope(ctx);
  const float *dd, *da, *db;
  ZJAI_TRY(stage_in(ctx, d, (size_t)n, mem, &dd));
  ZJAI_TRY(stage_in(ctx, a, (size_t)n, mem, &da));
  ZJAI_TRY(stage_in(ctx, b, (size_t)n, mem, &db));
  float *oa, *ob;
  ZJAI_TRY(stage_out_alloc(ctx, d_a, (size_t)n, mem, &oa));
  ZJAI_TRY(stage_out_alloc(ctx, d_b, (size_t)n, mem, &ob));
  elu_gate_bwd_kernel<<<launch_elementwise_blocks(ctx, (size_t)n), 256, 0, ctx->stream>>>(
      dd, da, db, (size_t)n, oa, ob);
  ctx->launches++;
  ZJAI_TRY(cuda_check(cudaGetLastError(), "elu gate VJP"));
  ZJAI_TRY(stage_out_finish(ctx, d_a, oa, (size_t)n, mem));
  ZJAI_TRY(stage_out_finish(ctx, d_b, ob, (size_t)n, mem));
  return finish_call(ctx, mem);
}

int zjai_layer_norm_backward(zjai_ctx* ctx, const float* d, const float* x, int c, int h, int w,
                             const float* weight, float* dx, int mem) {
  ZJAI_TRY(ctx_enter(ctx));
  if (!d || !x || !weight || !dx || c <= 0 || h <= 0 || w <= 0)
    return fail(ZJAI_INVALID_ARGUMENT, "layer norm backward: shape");
  if (mem != ZJAI_MEM_HOST && mem != ZJAI_MEM_DEVICE)
    return fail(ZJAI_INVALID_ARGUMENT, "mem must be HOST or DEVICE");
  ArenaScope scope(ctx);
  const long long n = (long long)h * w;
  const size_t nt = (size_t)c * n;
  const float *dd, *dxin, *dw;
  ZJAI_TRY(stage_in(ctx, d, nt, mem, &dd));
  ZJAI_TRY(stage_in(ctx, x, nt, mem, &dxin));
  ZJAI_TRY(stage_in(ctx, weight, (size_t)c, mem, &dw));
  float* out;
  ZJAI_TRY(stage_out_alloc(ctx, dx, nt, mem, &out));
  ln_bwd_kernel<<<launch_elementwise_blocks(ctx, (size_t)n), 256, 0, ctx->stream>>>(
      dd, dxin, c, n, dw, out);
  ctx->launches++;
  ZJAI_TRY(cuda_check(cudaGetLastError(), "layer norm VJP"));
  ZJAI_TRY(stage_out_finish(ctx, dx, out, nt, mem));
  return finish_call(ctx, mem);
}

int zjai_channel_attention_backward(zjai_ctx* ctx, const float* qkv, int c3, int h, int w,
                                    int heads, const float* temperature, const float* attn,
                                    const float* dout, float* dqkv, int mem) {
  ZJAI_TRY(ctx_enter(ctx));
  if (!qkv || !temperature || !attn || !dout || !dqkv || h <= 0 || w <= 0 || heads <= 0 ||
      c3 <= 0 || c3 % (3 * heads))
    return fail(ZJAI_INVALID_ARGUMENT, "attention: channel / head counts");
  if (mem != ZJAI_MEM_HOST && mem != ZJAI_MEM_DEVICE)
    return fail(ZJAI_INVALID_ARGUMENT, "mem must be HOST or DEVICE");
  ArenaScope scope(ctx);
  const int dim = c3 / 3, c = dim / heads;
  const long long n = (long long)h * w;
  const float *dq, *dt, *da_in, *dd;
  ZJAI_TRY(stage_in(ctx, qkv, (size_t)c3 * n, mem, &dq));
  ZJAI_TRY(stage_in(ctx, temperature, (size_t)heads, mem, &dt));
  ZJAI_TRY(stage_in(ctx, attn, (size_t)dim * c, mem, &da_in));
  ZJAI_TRY(stage_in(ctx, dout, (size_t)dim * n, mem, &dd));
  float* out;
  ZJAI_TRY(stage_out_alloc(ctx, dqkv, (size_t)c3 * n, mem, &out));
  ZJAI_TRY(attn_vjp(ctx, dq, c3, n, heads, dt, da_in, dd, out));
  ZJAI_TRY(stage_out_finish(ctx, dqkv, out, (size_t)c3 * n, mem));
  return finish_call(ctx, mem);
}

int zjai_transformer_block_backward(zjai_ctx* ctx, const float* dout, int dim, int hidden,
                                    int heads, int h, int w, const zjai_tb_tape* tape,
                                    const zjai_tb_weights* wts, float* din, int mem) {
  ZJAI_TRY(ctx_enter(ctx));
  if (!dout || !tape || !wts || !din || dim <= 0 || hidden <= 0 || heads <= 0 || h <= 0 ||
      w <= 0 || dim % heads || (3 * dim) % 8 || (2 * hidden) % 8)
    return fail(ZJAI_INVALID_ARGUMENT, "transformer_block_backward: shapes");
  if (mem != ZJAI_MEM_HOST && mem != ZJAI_MEM_DEVICE)
    return fail(ZJAI_INVALID_ARGUMENT, "mem must be HOST or DEVICE");
  const float* tp[5] = {tape->x_in, tape->qkv, tape->attn, tape->x_mid, tape->gate};
  const float* wp[9] = {wts->prep_norm,  wts->prep_conv1, wts->prep_conv2,
                        wts->temperature, wts->attn_out,  wts->ffn_norm,
                        wts->ffn_in,     wts->ffn_dw,     wts->ffn_out};
  for (const float* p : tp)
    if (!p) return fail(ZJAI_INVALID_ARGUMENT, "transformer_block_backward: missing tape array");
  for (const float* p : wp)
    if (!p) return fail(ZJAI_INVALID_ARGUMENT, "transformer_block_backward: missing weight");
  ArenaScope scope(ctx);
  const long long n = (long long)h * w;
  const int c = dim / heads;
  const size_t tn[5] = {(size_t)dim * n, (size_t)3 * dim * n, (size_t)dim * c, (size_t)dim * n,
                        (size_t)2 * hidden * n};
  // conv weights on the host (packing), the rest staged on the device
  std::vector<float> wb[9];
  const float* hw[9] = {};
  const size_t wn[9] = {(size_t)dim, (size_t)3 * dim * dim, (size_t)3 * dim * 9, (size_t)heads,
                        (size_t)dim * dim, (size_t)dim, (size_t)2 * hidden * dim,
                        (size_t)2 * hidden * 9, (size_t)dim * hidden};
  for (int i : {1, 2, 4, 6, 7, 8}) ZJAI_TRY(fetch_host(wp[i], wn[i], mem, &wb[i], &hw[i]));
  const float *dd, *dt[5], *dprep_norm, *dtemp, *dffn_norm;
  ZJAI_TRY(stage_in(ctx, dout, (size_t)dim * n, mem, &dd));
  for (int i = 0; i < 5; ++i) ZJAI_TRY(stage_in(ctx, tp[i], tn[i], mem, &dt[i]));
  ZJAI_TRY(stage_in(ctx, wp[0], wn[0], mem, &dprep_norm));
  ZJAI_TRY(stage_in(ctx, wp[3], wn[3], mem, &dtemp));
  ZJAI_TRY(stage_in(ctx, wp[5], wn[5], mem, &dffn_norm));
  float* ddin;
  ZJAI_TRY(stage_out_alloc(ctx, din, (size_t)dim * n, mem, &ddin));
  float* df = static_cast<float*>(ctx->arena.alloc((size_t)hidden * n * sizeof(float)));
  float* g1 = static_cast<float*>(ctx->arena.alloc((size_t)2 * hidden * n * sizeof(float)));
  float* g2 = static_cast<float*>(ctx->arena.alloc((size_t)2 * hidden * n * sizeof(float)));
  float* dm = static_cast<float*>(ctx->arena.alloc((size_t)dim * n * sizeof(float)));
  float* dln = static_cast<float*>(ctx->arena.alloc((size_t)dim * n * sizeof(float)));
  float* q1 = static_cast<float*>(ctx->arena.alloc((size_t)3 * dim * n * sizeof(float)));
  float* q2 = static_cast<float*>(ctx->arena.alloc((size_t)3 * dim * n * sizeof(float)));
  if (!df || !g1 || !g2 || !dm || !dln || !q1 || !q2)
    return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (transformer block VJP)");
  const size_t nd = (size_t)dim * n, nh = (size_t)hidden * n;
  // feed-forward branch: project_out, the ELU gate, the depthwise conv, project_in, its norm
  ZJAI_TRY(conv_vjp_s1(ctx, dd, dim, h, w, hw[8], hidden, 1, 1, 0, 0, 1, h, w, 0, 0, df));
  elu_gate_bwd_kernel<<<launch_elementwise_blocks(ctx, nh), 256, 0, ctx->stream>>>(
      df, dt[4], dt[4] + nh, nh, g1, g1 + nh);
  ctx->launches++;
  ZJAI_TRY(dw_vjp(ctx, g1, 2 * hidden, h, w, hw[7], g2));
  ZJAI_TRY(conv_vjp_s1(ctx, g2, 2 * hidden, h, w, hw[6], dim, 1, 1, 0, 0, 1, h, w, 0, 0, dm));
  ln_bwd_kernel<<<launch_elementwise_blocks(ctx, (size_t)n), 256, 0, ctx->stream>>>(
      dm, dt[3], dim, n, dffn_norm, dln);
  // d_xmid = d_out + that branch
  ZJAI_TRY(cuda_check(cudaMemcpyAsync(ddin, dd, nd * sizeof(float), cudaMemcpyDeviceToDevice,
                                      ctx->stream),
                      "d_xmid"));
  add_kernel<<<launch_elementwise_blocks(ctx, nd), 256, 0, ctx->stream>>>(ddin, dln, nd);
  ctx->launches += 2;
  // attention branch on d_xmid: project_out, the attention, the depthwise conv, project_in,
  // its norm; added to d_xmid
  ZJAI_TRY(conv_vjp_s1(ctx, ddin, dim, h, w, hw[4], dim, 1, 1, 0, 0, 1, h, w, 0, 0, dm));
  ZJAI_TRY(attn_vjp(ctx, dt[1], 3 * dim, n, heads, dtemp, dt[2], dm, q1));
  ZJAI_TRY(dw_vjp(ctx, q1, 3 * dim, h, w, hw[2], q2));
  ZJAI_TRY(conv_vjp_s1(ctx, q2, 3 * dim, h, w, hw[1], dim, 1, 1, 0, 0, 1, h, w, 0, 0, dm));
  ln_bwd_kernel<<<launch_elementwise_blocks(ctx, (size_t)n), 256, 0, ctx->stream>>>(
      dm, dt[0], dim, n, dprep_norm, dln);
  add_kernel<<<launch_elementwise_blocks(ctx, nd), 256, 0, ctx->stream>>>(ddin, dln, nd);
  ctx->launches += 2;
  ZJAI_TRY(cuda_check(cudaGetLastError(), "transformer block VJP"));
  ZJAI_TRY(stage_out_finish(ctx, din, ddin, (size_t)dim * n, mem));
  return ctx_check_status(ctx);
}

}  // extern "C"
