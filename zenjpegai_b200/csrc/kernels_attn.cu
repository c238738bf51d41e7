// Memory-bound kernels of the HOP attention blocks on NHWC f16 maps:
//  - layer norm over channels (math.rs:423-448), one warp per pixel, warp-shuffle sums;
//  - depthwise 3x3 (depthwise.rs), optionally fused with the FFN's ELU gate (math.rs:376);
//  - transposed ("channel") attention (math.rs:512-603) in three steps: a split-pixel Gram
//    Q.K^T plus squared norms, a tiny per-row softmax, and the A.V apply.
// Plus the latent gather that turns planar f32 latent windows into NHWC f16 tile batches.
#include "engine.h"
#include "kernels_attn.h"

namespace zjai {

namespace {

inline int blocks_for(long long n, int t) { return (int)((n + t - 1) / t); }

__device__ __forceinline__ void ld8(const __half* p, float (&v)[8]) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

__device__ __forceinline__ void st8(__half* p, const float (&v)[8]) {
  uint4 u;
  __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}

// ---- layer norm ---------------------------------------------------------------------------
// One warp per pixel; lane l holds channels l*8 .. l*8+7 of each 256-channel slab.
__global__ void layer_norm_kernel(const __half* __restrict__ x, __half* __restrict__ y, int n_img,
                                  int h, int w, int c, long long xpix, long long xrow,
                                  long long ximg, long long ypix, long long yrow, long long yimg,
                                  const float* __restrict__ gamma,
                                  const float* __restrict__ beta) {
  const int warps = blockDim.x >> 5;
  long long pixel = (long long)blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (pixel >= (long long)n_img * h * w) return;
  const int px = (int)(pixel % w);
  const long long r = pixel / w;
  const int py = (int)(r % h), n = (int)(r / h);
  const __half* xp = x + n * ximg + py * xrow + px * xpix;
  __half* yp = y + n * yimg + py * yrow + px * ypix;
  float v[2][8];
  float sum = 0.f;
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    const int c0 = s * 256 + lane * 8;
    if (c0 < c) {
      ld8(xp + c0, v[s]);
#pragma unroll
      for (int i = 0; i < 8; ++i) sum += v[s][i];
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float mean = sum / (float)c;
  float sq = 0.f;
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    const int c0 = s * 256 + lane * 8;
    if (c0 < c) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float d = v[s][i] - mean;
        sq += d * d;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  const float denom = sqrtf(sq / (float)c + 1e-5f);
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    const int c0 = s * 256 + lane * 8;
    if (c0 < c) {
      float o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        o[i] = (v[s][i] - mean) / denom * __ldg(gamma + c0 + i) + __ldg(beta + c0 + i);
      st8(yp + c0, o);
    }
  }
}

// ---- depthwise 3x3 ------------------------------------------------------------------------
// Thread per (group of 8 channels, segment of kDwSeg pixels of one row); consecutive threads
// take consecutive channel groups, so every 16-byte load of a warp is part of one contiguous
// run. The 3x3 weights of the thread's 8 channels sit in registers. Weights [c][9] f32.
// gate: out has c/2 channels, out[k] = elu(dw[k]) * dw[k + c/2] (the FFN gate, math.rs:376).
constexpr int kDwSeg = 4;

__device__ __forceinline__ void dw_source(const __half* __restrict__ xb, int py, int px0, int h,
                                          int w, long long xrow, long long xpix, int c0,
                                          const float* __restrict__ wt, float (&acc)[kDwSeg][8]) {
  float wr[9][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int t = 0; t < 9; ++t) wr[t][i] = __ldg(wt + (c0 + i) * 9 + t);
#pragma unroll
  for (int p = 0; p < kDwSeg; ++p)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[p][i] = 0.f;
#pragma unroll
  for (int ky = 0; ky < 3; ++ky) {
    const int yy = py + ky - 1;
    if (yy < 0 || yy >= h) continue;
    float v[kDwSeg + 2][8];
#pragma unroll
    for (int q = 0; q < kDwSeg + 2; ++q) {
      const int xx = px0 + q - 1;
      if (xx >= 0 && xx < w) {
        ld8(xb + yy * xrow + xx * xpix + c0, v[q]);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[q][i] = 0.f;
      }
    }
#pragma unroll
    for (int p = 0; p < kDwSeg; ++p)
#pragma unroll
      for (int kx = 0; kx < 3; ++kx)
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[p][i] = fmaf(wr[ky * 3 + kx][i], v[p + kx][i], acc[p][i]);
  }
}

__global__ void __launch_bounds__(256) dw3x3_kernel(const __half* __restrict__ x,
                                                    __half* __restrict__ y, int n_img, int h,
                                                    int w, int c, long long xpix, long long xrow,
                                                    long long ximg, long long ypix,
                                                    long long yrow, long long yimg,
                                                    const float* __restrict__ wt, int gate) {
  const int cg_out = (gate ? c / 2 : c) / 8;
  const int segs = (w + kDwSeg - 1) / kDwSeg;
  long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long total = (long long)n_img * h * segs * cg_out;
  if (idx >= total) return;
  const int cg = (int)(idx % cg_out);
  long long r = idx / cg_out;
  const int sg = (int)(r % segs);
  r /= segs;
  const int py = (int)(r % h), n = (int)(r / h);
  const int px0 = sg * kDwSeg;
  const __half* xb = x + n * ximg;
  float a[kDwSeg][8];
  dw_source(xb, py, px0, h, w, xrow, xpix, cg * 8, wt, a);
  if (gate) {
    float b[kDwSeg][8];
    dw_source(xb, py, px0, h, w, xrow, xpix, cg * 8 + c / 2, wt, b);
#pragma unroll
    for (int p = 0; p < kDwSeg; ++p)
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float e = a[p][i] > 0.f ? a[p][i] : expf(a[p][i]) - 1.f;
        a[p][i] = e * b[p][i];
      }
  }
#pragma unroll
  for (int p = 0; p < kDwSeg; ++p)
    if (px0 + p < w) st8(y + n * yimg + py * yrow + (px0 + p) * ypix + cg * 8, a[p]);
}

// ---- channel attention -------------------------------------------------------------------
// gram[n][h][i][j] += sum_p q[p][h*c+i] * k[p][h*c+j]; sq[n][0|1][ch] += q^2 / k^2.
// Block: 256 threads, a chunk of 32 pixels of q and k staged in shared memory as f32.
constexpr int kGramPix = 32;

__global__ void attn_gram_kernel(const __half* __restrict__ qkv, int n_img, int npix, int w,
                                 int dim, int heads, long long pix, long long row, long long img,
                                 float* __restrict__ gram, float* __restrict__ sq,
                                 int chunks_per_block) {
  extern __shared__ float sm[];  // [kGramPix][2*dim]
  const int n = blockIdx.y;
  const int c = dim / heads;
  const int per_head = c * c;
  const int entries = heads * per_head;
  const int per_thread = (entries + blockDim.x - 1) / blockDim.x;  // <= 16
  float acc[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i] = 0.f;
  float sqacc = 0.f;
  const __half* base = qkv + n * img;
  for (int ch = 0; ch < chunks_per_block; ++ch) {
    const int p0 = (blockIdx.x * chunks_per_block + ch) * kGramPix;
    if (p0 >= npix) break;
    __syncthreads();
    // stage q and k (2*dim channels) of up to kGramPix pixels
    const int groups = 2 * dim / 8;
    for (int t = threadIdx.x; t < kGramPix * groups; t += blockDim.x) {
      const int pp = t / groups, g = t % groups;
      float v[8];
      const int p = p0 + pp;
      if (p < npix) {
        ld8(base + (p / w) * row + (p % w) * pix + g * 8, v);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) sm[pp * 2 * dim + g * 8 + i] = v[i];
    }
    __syncthreads();
    for (int e = 0; e < per_thread; ++e) {
      const int id = threadIdx.x + e * blockDim.x;
      if (id >= entries) break;
      const int hd = id / per_head, ij = id % per_head;
      const int qi = hd * c + ij / c, kj = dim + hd * c + ij % c;
      float s = 0.f;
#pragma unroll 8
      for (int pp = 0; pp < kGramPix; ++pp) s = fmaf(sm[pp * 2 * dim + qi], sm[pp * 2 * dim + kj], s);
      acc[e] += s;
    }
    if (threadIdx.x < 2 * dim) {
      float s = 0.f;
      for (int pp = 0; pp < kGramPix; ++pp) {
        const float v = sm[pp * 2 * dim + threadIdx.x];
        s = fmaf(v, v, s);
      }
      sqacc += s;
    }
  }
  for (int e = 0; e < per_thread; ++e) {
    const int id = threadIdx.x + e * blockDim.x;
    if (id < entries) atomicAdd(gram + (long long)n * entries + id, acc[e]);
  }
  if (threadIdx.x < 2 * dim) atomicAdd(sq + (long long)n * 2 * dim + threadIdx.x, sqacc);
}

// attn[n][h][i][j] = softmax_j( G_ij / (max(|q_i|, eps) max(|k_j|, eps)) * T[h] )
__global__ void attn_softmax_kernel(const float* __restrict__ gram, const float* __restrict__ sq,
                                    const float* __restrict__ temp, float* __restrict__ attn,
                                    int n_img, int dim, int heads) {
  const int c = dim / heads;
  long long row = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= (long long)n_img * dim) return;
  const int n = (int)(row / dim), ri = (int)(row % dim);
  const int hd = ri / c;
  const float* g = gram + (long long)n * dim * c + (long long)ri * c;
  const float* s = sq + (long long)n * 2 * dim;
  const float nq = fmaxf(sqrtf(s[ri]), 1e-12f);
  float vals[64];
  float mx = -INFINITY;
  for (int j = 0; j < c; ++j) {
    const float nk = fmaxf(sqrtf(s[dim + hd * c + j]), 1e-12f);
    const float v = g[j] / (nq * nk) * temp[hd];
    vals[j] = v;
    mx = fmaxf(mx, v);
  }
  float sum = 0.f;
  for (int j = 0; j < c; ++j) {
    vals[j] = expf(vals[j] - mx);
    sum += vals[j];
  }
  float* a = attn + (long long)n * dim * c + (long long)ri * c;
  for (int j = 0; j < c; ++j) a[j] = vals[j] / sum;
}

// out[p][h*c+i] = sum_j attn[h][i][j] * v[p][h*c+j]. Block = one group of 8 output channels
// (blockIdx.y) and 256 pixels (one per thread): every shared-memory read of the attention
// rows is a broadcast.
__global__ void __launch_bounds__(256) attn_apply_kernel(
    const __half* __restrict__ qkv, const float* __restrict__ attn, __half* __restrict__ out,
    int n_img, int h, int w, int dim, int heads, long long pix, long long row, long long img,
    long long opix, long long orow, long long oimg) {
  __shared__ float sa[8 * 64];  // the 8 attention rows of this channel group (c <= 64)
  const int c = dim / heads;
  const int n = blockIdx.z, g = blockIdx.y;
  const int i0 = g * 8, hd = i0 / c;
  for (int t = threadIdx.x; t < 8 * c; t += blockDim.x)
    sa[t] = attn[(long long)n * dim * c + (long long)i0 * c + t];
  __syncthreads();
  const long long p = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= (long long)h * w) return;
  const int py = (int)(p / w), px = (int)(p % w);
  const __half* vp = qkv + n * img + py * row + px * pix + 2 * dim + hd * c;
  float o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int j0 = 0; j0 < c; j0 += 8) {
    float v[8];
    ld8(vp + j0, v);
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = fmaf(sa[i * c + j0 + jj], v[jj], o[i]);
    }
  }
  st8(out + n * oimg + py * orow + px * opix + i0, o);
}

// planar f32 latent [C][LH][LW] -> NHWC f16 [n][h][w] at channel offset; per-image window
// origins (x, y) in `origin` (device int pairs).
__global__ void gather_latent_kernel(const float* __restrict__ src, int C, int LH, int LW,
                                     const int* __restrict__ origin, __half* __restrict__ dst,
                                     int n_img, int h, int w, long long pix, long long row,
                                     long long img) {
  long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long total = (long long)n_img * h * w;
  if (idx >= total) return;
  const int x = (int)(idx % w);
  long long r = idx / w;
  const int y = (int)(r % h), n = (int)(r / h);
  const int sx = origin[2 * n] + x, sy = origin[2 * n + 1] + y;
  const long long plane = (long long)LH * LW;
  const float* s = src + (long long)sy * LW + sx;
  __half* d = dst + n * img + (long long)y * row + (long long)x * pix;
  for (int ch = 0; ch + 1 < C; ch += 2)
    *reinterpret_cast<__half2*>(d + ch) = __floats2half2_rn(__ldg(s + ch * plane), __ldg(s + (ch + 1) * plane));
  if (C & 1) d[C - 1] = __float2half_rn(__ldg(s + (C - 1) * plane));
}

}  // namespace

void launch_layer_norm(const TView& x, const TView& y, const float* gamma, const float* beta,
                       cudaStream_t s) {
  long long pixels = (long long)x.n * x.h * x.w;
  layer_norm_kernel<<<blocks_for(pixels, 8), 256, 0, s>>>(x.p, y.p, x.n, x.h, x.w, x.c, x.pix,
                                                          x.row, x.img, y.pix, y.row, y.img,
                                                          gamma, beta);
}

void launch_dw3x3(const TView& x, const TView& y, const float* wt, bool gate, cudaStream_t s) {
  const int cg_out = (gate ? x.c / 2 : x.c) / 8;
  const int segs = (x.w + kDwSeg - 1) / kDwSeg;
  long long total = (long long)x.n * x.h * segs * cg_out;
  dw3x3_kernel<<<blocks_for(total, 256), 256, 0, s>>>(x.p, y.p, x.n, x.h, x.w, x.c, x.pix, x.row,
                                                       x.img, y.pix, y.row, y.img, wt, gate ? 1 : 0);
}

void launch_attention(const TView& qkv, const TView& out, int heads, const float* temp,
                      float* scratch, cudaStream_t s) {
  const int dim = qkv.c / 3;
  const int c = dim / heads;
  const int n = qkv.n;
  float* gram = scratch;                              // n * dim * c
  float* sq = gram + (size_t)n * dim * c;             // n * 2 * dim
  float* attn = sq + (size_t)n * 2 * dim;             // n * dim * c
  cudaMemsetAsync(gram, 0, sizeof(float) * ((size_t)n * dim * c + (size_t)n * 2 * dim), s);
  const int npix = qkv.h * qkv.w;
  const int chunks = (npix + kGramPix - 1) / kGramPix;
  const int cpb = std::max(1, chunks / 64);
  dim3 g1((chunks + cpb - 1) / cpb, n);
  attn_gram_kernel<<<g1, 256, kGramPix * 2 * dim * sizeof(float), s>>>(
      qkv.p, n, npix, qkv.w, dim, heads, qkv.pix, qkv.row, qkv.img, gram, sq, cpb);
  attn_softmax_kernel<<<blocks_for((long long)n * dim, 128), 128, 0, s>>>(gram, sq, temp, attn, n,
                                                                         dim, heads);
  dim3 g3(blocks_for((long long)npix, 256), dim / 8, n);
  attn_apply_kernel<<<g3, 256, 0, s>>>(qkv.p, attn, out.p, n, qkv.h, qkv.w, dim, heads, qkv.pix,
                                       qkv.row, qkv.img, out.pix, out.row, out.img);
}

size_t attention_scratch_floats(int n_img, int dim, int heads) {
  const int c = dim / heads;
  return (size_t)n_img * (2 * (size_t)dim * c + 2 * (size_t)dim);
}

void launch_gather_latent(const float* src, int C, int LH, int LW, const int* origin,
                          const TView& dst, cudaStream_t s) {
  long long total = (long long)dst.n * dst.h * dst.w;
  gather_latent_kernel<<<blocks_for(total, 256), 256, 0, s>>>(src, C, LH, LW, origin, dst.p, dst.n,
                                                               dst.h, dst.w, dst.pix, dst.row,
                                                               dst.img);
}

}  // namespace zjai
