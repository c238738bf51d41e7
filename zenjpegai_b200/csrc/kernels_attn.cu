// Memory-bound kernels of the HOP attention blocks on NHWC f16 maps:
//  - layer norm over channels (math.rs:423-448), one warp per pixel, warp-shuffle sums;
//  - depthwise 3x3 (depthwise.rs), optionally fused with the FFN's ELU gate (math.rs:376);
//  - transposed ("channel") attention (math.rs:512-603) in three steps: a split-pixel Gram
//    Q.K^T plus squared norms, a tiny per-row softmax, and the A.V apply.
// Plus the latent gather that turns planar f32 latent windows into NHWC f16 tile batches.
#include "engine.h"
#include "gate.cuh"
#include "kernels_attn.h"
#include "ptx.cuh"

#include <algorithm>
#include <type_traits>

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

// Layer norm for c <= 256: a pixel is a segment of LPP lanes (LPP = c/8 rounded up to a power
// of two), lane l of a segment holding channels 8l .. 8l+7; sums are segment-local shuffles.
// A thread handles kLnPix pixels (their loads issued together), its gamma / beta stay in
// registers. Two-pass mean and variance in f32 like layer_norm_kernel; the normalisation
// multiplies by one reciprocal of the deviation per pixel.
constexpr int kLnPix = 8;

// Element offset of pixel p (raster order over n, h, w) in a view; `dense`: the view's pixels
// are contiguous (row == w * pix, img == h * row), so no division is needed.
__device__ __forceinline__ long long pix_off(int p, int h, int w, long long pix, long long row,
                                             long long img, bool dense) {
  if (dense) return (long long)p * pix;
  const int r = p / w;
  return (long long)(r / h) * img + (long long)(r % h) * row + (long long)(p - r * w) * pix;
}

template <int LPP>
__global__ void __launch_bounds__(256) layer_norm_seg_kernel(
    const __half* __restrict__ x, __half* __restrict__ y, int npix, int h, int w, int c,
    long long xpix, long long xrow, long long ximg, bool xdense, long long ypix,
    long long yrow, long long yimg, bool ydense, const float* __restrict__ gamma,
    const float* __restrict__ beta) {
  constexpr int SEGS = 256 / LPP;  // pixels per block and pass
  const int sub = threadIdx.x % LPP;
  const int c0 = sub * 8;
  const bool act = c0 < c;
  float gm[8], bt[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    gm[i] = act ? __ldg(gamma + c0 + i) : 0.f;
    bt[i] = act ? __ldg(beta + c0 + i) : 0.f;
  }
  // the pixels' raw f16 (16 bytes each) in flight together, unpacked one pixel at a time
  uint4 raw[kLnPix];
  int pxl[kLnPix];
#pragma unroll
  for (int k = 0; k < kLnPix; ++k) {
    pxl[k] = (blockIdx.x * kLnPix + k) * SEGS + threadIdx.x / LPP;
    const int p = pxl[k];
    raw[k] = (act && p < npix)
                 ? *reinterpret_cast<const uint4*>(x + pix_off(p, h, w, xpix, xrow, ximg, xdense) + c0)
                 : make_uint4(0u, 0u, 0u, 0u);
  }
#pragma unroll
  for (int k = 0; k < kLnPix; ++k) {
    float v[8];
    {
      const __half2* hh = reinterpret_cast<const __half2*>(&raw[k]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(hh[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
      }
    }
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) sum += v[i];
#pragma unroll
    for (int o = LPP / 2; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float mean = sum / (float)c;
    float sq = 0.f;
    if (act) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float d = v[i] - mean;
        sq += d * d;
      }
    }
#pragma unroll
    for (int o = LPP / 2; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    const float inv = 1.f / sqrtf(sq / (float)c + 1e-5f);  // one division per pixel
    const int p = pxl[k];
    if (act && p < npix) {
      float o8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) o8[i] = (v[i] - mean) * inv * gm[i] + bt[i];
      st8(y + pix_off(p, h, w, ypix, yrow, yimg, ydense) + c0, o8);
    }
  }
}

// ---- depthwise 3x3 ------------------------------------------------------------------------
// Block = a tile of kDwTH rows x TW columns x 64 output channels. Its input (with the
// one-pixel halo) is staged in shared memory by 16-byte cp.async copies, zero-filled outside
// the picture (the convolution's zero padding), as [row][col][8-channel group] chunks.
// Thread = (8-channel group of one source, column): it walks the tile's input rows top to
// bottom, adding each row into the three output rows that it feeds (accumulators in
// registers, the thread's 3x3 weights too) and writing an output row as soon as its last
// input row is in. Per output the taps accumulate in (ky, kx) row-major order, two channels
// per packed f32x2 FMA. Weights [c][9].
// gate: out has c/2 channels, out[k] = elu(dw[k]) * dw[k + c/2] (the FFN gate, math.rs:376);
// the thread of group g of the first half and the thread of group g of the second half sit 8
// lanes apart and swap half their sums by shuffles: the first writes output channels 0..3 of
// the group, the second channels 4..7.
constexpr int kDwTH = 8;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem),
               "r"(src_bytes)
               : "memory");
}

template <bool GATE>
struct DwShape {
  static constexpr int G = GATE ? 16 : 8;  // source channel groups per block
  static constexpr int TW = 256 / G;       // tile columns (one thread per group and column)
  static constexpr int SW = TW + 2, SH = kDwTH + 2;
  static constexpr int smem = SH * SW * G * 16;
};

// Spatial tile s of picture n at (ty, tx): s = (n * tiles_y + ty) * tiles_x + tx.
struct DwTiles {
  int tiles_x, tiles_y, count;
};

// Issue the cp.async copies of spatial tile `s` (channel block cb) into `buf`.
template <bool GATE>
__device__ __forceinline__ void dw_stage(uint4* buf, const __half* __restrict__ x, int s,
                                         const DwTiles& T, int cb, int h, int w, int c,
                                         long long xpix, long long xrow, long long ximg) {
  using S = DwShape<GATE>;
  constexpr int P = 256 / S::G;  // positions advanced per pass (< SW)
  const int cg_out = (GATE ? c / 2 : c) / 8;
  const int tx = s % T.tiles_x, ty = (s / T.tiles_x) % T.tiles_y, n = s / (T.tiles_x * T.tiles_y);
  const int x0 = tx * S::TW, y0 = ty * kDwTH;
  // thread = (channel group g, first position q0); position q = r * SW + cx
  const int g = threadIdx.x % S::G;
  const int grp = cb * 8 + (g & 7);
  const bool gok = grp < cg_out;
  const __half* xb = x + n * ximg + (GATE && g >= 8 ? c / 2 : 0) + grp * 8;
  int cx = threadIdx.x / S::G, r = 0;
  for (int q = cx; q < S::SH * S::SW; q += P) {
    const int yy = y0 - 1 + r, xx = x0 - 1 + cx;
    const bool ok = gok && yy >= 0 && yy < h && xx >= 0 && xx < w;
    cp_async16(buf + q * S::G + g, ok ? xb + yy * xrow + xx * xpix : x, ok ? 16 : 0);
    cx += P;
    if (cx >= S::SW) {
      cx -= S::SW;
      ++r;
    }
  }
}

__device__ __forceinline__ float elu1(float a) { return a > 0.f ? a : __expf(a) - 1.f; }

// Persistent: block b keeps channel block cb = b % cblocks (its weights stay in registers) and
// walks the spatial tiles s = b / cblocks, + gridDim.x / cblocks, ...; the copies of the next
// tile run while the current one is computed (two shared-memory buffers).
template <bool GATE>
__global__ void __launch_bounds__(256, 2)
    dw3x3_kernel(const __half* __restrict__ x, __half* __restrict__ y, int h, int w, int c,
                 long long xpix, long long xrow, long long ximg, long long ypix, long long yrow,
                 long long yimg, const float* __restrict__ wt, DwTiles T, int cblocks) {
  using S = DwShape<GATE>;
  extern __shared__ __align__(16) uint4 dw_tile[];
  const int cg_out = (GATE ? c / 2 : c) / 8;
  const int cb = blockIdx.x % cblocks;
  const int sstep = gridDim.x / cblocks;
  const int g = threadIdx.x % S::G, xl = threadIdx.x / S::G;
  const int grp = cb * 8 + (g & 7);
  const bool gvalid = grp < cg_out;
  const int ch = (GATE && g >= 8 ? c / 2 : 0) + grp * 8;

  int s = blockIdx.x / cblocks;
  if (s < T.count) dw_stage<GATE>(dw_tile, x, s, T, cb, h, w, c, xpix, xrow, ximg);
  asm volatile("cp.async.commit_group;\n" ::: "memory");
  float2 wr[9][4];  // channel pairs (2k, 2k + 1)
#pragma unroll
  for (int k = 0; k < 4; ++k)
#pragma unroll
    for (int t = 0; t < 9; ++t)
      wr[t][k] = gvalid ? make_float2(__ldg(wt + (ch + 2 * k) * 9 + t),
                                      __ldg(wt + (ch + 2 * k + 1) * 9 + t))
                        : make_float2(0.f, 0.f);

  for (int it = 0; s < T.count; s += sstep, ++it) {
    uint4* cur = dw_tile + (it & 1) * (S::smem / 16);
    if (s + sstep < T.count)
      dw_stage<GATE>(dw_tile + ((it + 1) & 1) * (S::smem / 16), x, s + sstep, T, cb, h, w, c,
                     xpix, xrow, ximg);
    asm volatile("cp.async.commit_group;\n" ::: "memory");
    asm volatile("cp.async.wait_group 1;\n" ::: "memory");
    __syncthreads();

    const int tx = s % T.tiles_x, ty = (s / T.tiles_x) % T.tiles_y;
    const int n = s / (T.tiles_x * T.tiles_y);
    const int x0 = tx * S::TW, y0 = ty * kDwTH;
    const bool xvalid = gvalid && x0 + xl < w;
    // gate: the first-half thread writes output channels 0..3 of the group, the second-half
    // thread channels 4..7
    const bool hi = GATE && g >= 8;
    __half* yb = y + n * yimg + (x0 + xl) * ypix + grp * 8 + (hi ? 4 : 0);
    float2 acc[3][4];
#pragma unroll
    for (int k = 0; k < 3; ++k)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[k][i] = make_float2(0.f, 0.f);
#pragma unroll
    for (int r = 0; r < S::SH; ++r) {
#pragma unroll
      for (int kx = 0; kx < 3; ++kx) {
        const uint4 u = cur[(r * S::SW + xl + kx) * S::G + g];
        const __half2* hv = reinterpret_cast<const __half2*>(&u);
        float2 v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = __half22float2(hv[i]);
#pragma unroll
        for (int ky = 0; ky < 3; ++ky) {
          const int o = r - ky;
          if (o >= 0 && o < kDwTH) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
              acc[o % 3][i] = ffma2(wr[ky * 3 + kx][i], v[i], acc[o % 3][i]);
          }
        }
      }
      if (r >= 2) {
        const int o = r - 2;
        float2(&a)[4] = acc[o % 3];
        const bool store = xvalid && y0 + o < h;
        if (GATE) {
          // swap halves with the partner 8 lanes away: the first-half thread sends pairs 2, 3
          // and receives the second half's pairs 0, 1 (and the other way round)
          float2 snd[2] = {hi ? a[0] : a[2], hi ? a[1] : a[3]}, rcv[2];
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            rcv[i].x = __shfl_xor_sync(0xffffffffu, snd[i].x, 8);
            rcv[i].y = __shfl_xor_sync(0xffffffffu, snd[i].y, 8);
          }
          if (store) {
            float o4[4];
#pragma unroll
            for (int i = 0; i < 2; ++i) {
              const float2 e = hi ? rcv[i] : a[i];      // first-half (ELU) operand
              const float2 m = hi ? a[2 + i] : rcv[i];  // second-half (multiplier) operand
              o4[2 * i] = elu1(e.x) * m.x;
              o4[2 * i + 1] = elu1(e.y) * m.y;
            }
            uint2 pk;
            *reinterpret_cast<__half2*>(&pk.x) = __floats2half2_rn(o4[0], o4[1]);
            *reinterpret_cast<__half2*>(&pk.y) = __floats2half2_rn(o4[2], o4[3]);
            *reinterpret_cast<uint2*>(yb + (y0 + o) * yrow) = pk;
          }
        } else if (store) {
          uint4 pk;
          __half2* ph = reinterpret_cast<__half2*>(&pk);
#pragma unroll
          for (int i = 0; i < 4; ++i) ph[i] = __floats2half2_rn(a[i].x, a[i].y);
          *reinterpret_cast<uint4*>(yb + (y0 + o) * yrow) = pk;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) a[i] = make_float2(0.f, 0.f);
      }
    }
    __syncthreads();  // all reads of `cur` done before the next iteration refills it
  }
  asm volatile("cp.async.wait_all;\n" ::: "memory");
}

// ---- depthwise 3x3, row-streaming ----------------------------------------------------------
// Work unit = (picture, strip of TW columns, band of U.band rows, block of 64 output
// channels). A producer warp streams the unit's input rows with their one-pixel halo (band
// rows + 2 rows of TW + 2 columns) through a ring of kDsStages shared-memory stages, one TMA
// box [64 channels, TW + 2, 1 row] per 64-channel slab (gate: two slabs, the block's channels
// of the first and of the second half); rows and columns outside the picture arrive as zeros,
// the convolution's padding. 256 compute threads = (column pair, slab, 8-channel group): per
// input row a thread reads its four staged columns (8 channels each) once, adds them into the
// three output rows they feed for both of its output columns (rolling accumulators), and
// stores an output row as soon as its last input row is in. Per output the taps accumulate in
// (ky, kx) row-major order, two channels per packed f32x2 FMA (as in dw3x3_kernel).
constexpr int kDsThreads = 512;  // compute threads; one more warp produces
constexpr int kDsStages = 16;
constexpr int kDsBand = 64;  // tallest band

template <bool GATE>
struct DsShape {
  static constexpr int NS = GATE ? 2 : 1;               // 64-channel slabs per staged row
  // threads per column pair: a thread holds 2 channel pairs (gate: one ELU pair and its
  // multiplier pair; plain: 4 consecutive channels)
  static constexpr int LPC = GATE ? 32 : 16;
  static constexpr int TW = 2 * kDsThreads / LPC;       // strip width: gate 32, plain 64
  static constexpr int SW = TW + 2;                     // staged columns
  static constexpr uint32_t slab = SW * 128u;           // bytes of one slab row
  static constexpr uint32_t stage = NS * slab;
  static constexpr uint32_t smem = kDsStages * stage + 2u * kDsStages * 8u + 16u;
};

// unit u: cb = u % cblocks, band, strip, picture in that order of significance
struct DsUnits {
  int strips, bands, cblocks, count;
  int band;  // rows per band (8 .. kDsBand)
};

template <bool GATE>
__global__ void __launch_bounds__(kDsThreads + 32, 1)
    dw3x3_stream_kernel(const __grid_constant__ CUtensorMap tm, __half* __restrict__ y, int h,
                        int w, int c, long long ypix, long long yrow, long long yimg,
                        const float* __restrict__ wt, DsUnits U, int* err) {
  using S = DsShape<GATE>;
  extern __shared__ __align__(128) uint8_t ds_smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(ds_smem + kDsStages * S::stage);
  uint64_t* empty = full + kDsStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kDsStages);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cout = GATE ? c / 2 : c;  // output channels (first-half offset of the gate)
  if (threadIdx.x == 0) {
    for (int i = 0; i < kDsStages; ++i) {
      mbar_init(smem_u32(&full[i]), 1);
      mbar_init(smem_u32(&empty[i]), kDsThreads / 32);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kDsThreads / 32) {
    // ---- producer: one lane issues the row copies of every unit of this CTA
    if (lane != 0) return;
    tma_prefetch_desc(&tm);
    int stage = 0;
    uint32_t phase = 0;
    long long issued = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < U.count; u += gridDim.x) {
      const int cb = u % U.cblocks;
      int rest = u / U.cblocks;
      const int band = rest % U.bands;
      rest /= U.bands;
      const int strip = rest % U.strips, n = rest / U.strips;
      const int x0 = strip * S::TW, y0 = band * U.band;
      const int rows = min(U.band, h - y0);
      for (int r = 0; r < rows + 2; ++r) {
        if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1u, abort_flag, err, DEV_TIMEOUT_EMPTY)) {
          ok = false;
          break;
        }
        const uint32_t fb = smem_u32(&full[stage]);
        const uint32_t dst = smem_u32(ds_smem + stage * S::stage);
        mbar_arrive_expect_tx(fb, S::stage);
        tma_load_4d(dst, &tm, fb, cb * 64, x0 - 1, y0 - 1 + r, n);
        if (GATE) tma_load_4d(dst + S::slab, &tm, fb, cout + cb * 64, x0 - 1, y0 - 1 + r, n);
        ++issued;
        if (++stage == kDsStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    // every copy issued has landed before the CTA's shared memory goes away (consumers that
    // gave up do not wait for the last ones)
    const int last = issued < kDsStages ? (int)issued : kDsStages;
    for (int k = 0; k < last; ++k) {
      int st = stage - 1 - k;
      uint32_t ph = phase;
      if (st < 0) {
        st += kDsStages;
        ph ^= 1u;
      }
      mbar_wait_drain(smem_u32(&full[st]), ph, err);
    }
    return;
  }

  // ---- compute threads: (column pair, two channel pairs). Plain: channels 4l .. 4l+3 of the
  // block for lane l of the column pair; gate: ELU-operand pair (2l, 2l+1) of the block's first
  // half as pair 0 and the matching multiplier pair of the second half as pair 1, so the gate
  // needs no exchange between threads.
  const int t = threadIdx.x;
  const int lane_ch = t % S::LPC;
  const int cp = t / S::LPC;  // column pair
  // staged row: column 2 cp (staged column 0 is picture column x0 - 1)
  const uint32_t my_off = (2 * cp) * 128u + lane_ch * (GATE ? 4u : 8u);
  int stage = 0;
  uint32_t phase = 0;
  int wcb = -1;
  float2 wr[9][2];  // the thread's two channel pairs, per tap
  for (int u = blockIdx.x; u < U.count; u += gridDim.x) {
    const int cb = u % U.cblocks;
    int rest = u / U.cblocks;
    const int band = rest % U.bands;
    rest /= U.bands;
    const int strip = rest % U.strips, n = rest / U.strips;
    const int x0 = strip * S::TW, y0 = band * U.band;
    const int rows = min(U.band, h - y0);
    const int ch0 = cb * 64 + lane_ch * (GATE ? 2 : 4);  // first output channel
    const bool cvalid = ch0 < cout;
    if (cb != wcb) {
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int ch = GATE ? ch0 + k * cout : ch0 + 2 * k;
#pragma unroll
        for (int tp = 0; tp < 9; ++tp)
          wr[tp][k] = cvalid ? make_float2(__ldg(wt + ch * 9 + tp), __ldg(wt + (ch + 1) * 9 + tp))
                             : make_float2(0.f, 0.f);
      }
      wcb = cb;
    }
    const int xo = x0 + 2 * cp;  // the thread's first output column
    const bool st0 = cvalid && xo < w, st1 = cvalid && xo + 1 < w;
    __half* yb = y + n * yimg + (long long)xo * ypix + ch0;
    // acc[o % 3][column][pair]: output row o is started (first tap a product) by input row o
    // and complete after input row o + 2; rows outside the band fill slots nobody stores
    float2 acc[3][2][2];

    // staged column j of the current stage as the thread's 2 channel pairs
    auto load_col = [&](const uint8_t* src, int j, float2 (&v)[2]) {
      if (GATE) {
        const uint32_t e = *reinterpret_cast<const uint32_t*>(src + j * 128);
        const uint32_t m = *reinterpret_cast<const uint32_t*>(src + S::slab + j * 128);
        v[0] = __half22float2(*reinterpret_cast<const __half2*>(&e));
        v[1] = __half22float2(*reinterpret_cast<const __half2*>(&m));
      } else {
        const uint2 q = *reinterpret_cast<const uint2*>(src + j * 128);
        v[0] = __half22float2(*reinterpret_cast<const __half2*>(&q.x));
        v[1] = __half22float2(*reinterpret_cast<const __half2*>(&q.y));
      }
    };
    // input row r (picture row y0 - 1 + r) with J = r % 3 known at compile time, so the
    // accumulator slot of output row r - ky ((J - ky) mod 3) is static
    auto row = [&](auto JJ, int r) -> bool {
      constexpr int J = decltype(JJ)::value;
      if (!mbar_wait(smem_u32(&full[stage]), phase, abort_flag, err, DEV_TIMEOUT_FULL))
        return false;
      const uint8_t* src = ds_smem + stage * S::stage + my_off;
      float2 v[4][2];
#pragma unroll
      for (int j = 0; j < 4; ++j) load_col(src, j, v[j]);
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&empty[stage]));
      if (++stage == kDsStages) {
        stage = 0;
        phase ^= 1u;
      }
      // per output the taps go in (ky, kx) order: this row is tap row ky of output r - ky
#pragma unroll
      for (int kx = 0; kx < 3; ++kx)
#pragma unroll
        for (int ky = 0; ky < 3; ++ky)
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            float2(&a)[2][2] = acc[(J - ky + 3) % 3];
            const float2 wv = wr[ky * 3 + kx][i];
            if (ky == 0 && kx == 0) {
              a[0][i] = __fmul2_rn(wv, v[0][i]);
              a[1][i] = __fmul2_rn(wv, v[1][i]);
            } else {
              a[0][i] = ffma2(wv, v[kx][i], a[0][i]);
              a[1][i] = ffma2(wv, v[kx + 1][i], a[1][i]);
            }
          }
      const int o = r - 2;  // complete with this row
      if (o >= 0 && o < rows) {
        const float2(&ao)[2][2] = acc[(J + 1) % 3];
        __half* yr = yb + (long long)(y0 + o) * yrow;
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const float2(&a)[2] = ao[q];
          if (!(q == 0 ? st0 : st1)) continue;
          if (GATE) {
            *reinterpret_cast<__half2*>(yr + q * ypix) = __float22half2_rn(elu_gate2(a[0], a[1]));
          } else {
            uint2 pk;
            *reinterpret_cast<__half2*>(&pk.x) = __floats2half2_rn(a[0].x, a[0].y);
            *reinterpret_cast<__half2*>(&pk.y) = __floats2half2_rn(a[1].x, a[1].y);
            *reinterpret_cast<uint2*>(yr + q * ypix) = pk;
          }
        }
      }
      return true;
    };
    bool ok = true;
    for (int r = 0; ok && r < rows + 2; r += 3) {
      ok = row(std::integral_constant<int, 0>{}, r);
      if (ok && r + 1 < rows + 2) ok = row(std::integral_constant<int, 1>{}, r + 1);
      if (ok && r + 2 < rows + 2) ok = row(std::integral_constant<int, 2>{}, r + 2);
    }
    if (!ok) return;
  }
}

// ---- channel attention -------------------------------------------------------------------
// gram[n][h][i][j] += sum_p q[p][h*c+i] * k[p][h*c+j]; sq[n][0|1][ch] += q^2 / k^2.
// Block: 256 threads, a chunk of 32 pixels of q and k staged in shared memory as f32.
constexpr int kGramPix = 32;

__global__ void attn_gram_kernel(const __half* __restrict__ qkv, int n_img, int npix, int w,
                                 int dim, int heads, long long pix, long long row, long long img,
                                 float* __restrict__ part, int nparts, int chunks_per_block) {
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
  // this block's partial slot: Gram [dim][c] then the squared norms [2 dim]
  float* slot = part + ((long long)n * nparts + blockIdx.x) * (entries + 2 * dim);
  for (int e = 0; e < per_thread; ++e) {
    const int id = threadIdx.x + e * blockDim.x;
    if (id < entries) slot[id] = acc[e];
  }
  if (threadIdx.x < 2 * dim) slot[entries + threadIdx.x] = sqacc;
}

// Gram on the tensor cores (mma.sync m16n8k16, f16 in, f32 accumulate) for head widths
// HC = 16 or 32 and heads dividing 8. Block = 8 warps over a contiguous pixel range of one
// picture (blockIdx.y); pixels arrive in chunks of kGramChunk as f16 rows [q | k] (row pitch
// padded by 16 bytes so the 8 rows of an ldmatrix hit 8 distinct bank groups), by 16-byte
// cp.async copies, double-buffered. Warp w takes head w % heads and a 1/(8/heads) slice of
// each chunk's pixels. With S the staged rows [pixel][channel]: G_h = Q_h^T K_h is an MMA whose
// A operand (channels x pixels) and B operand (pixels x channels) both come from S through
// ldmatrix.trans. The squared norms sum_p q_i^2 and sum_p k_j^2 are the diagonals of Q_h^T Q_h
// and K_h^T K_h, taken from the diagonal 8x8 blocks only. Partial sums go to gram / sq by
// atomics at the end.
constexpr int kGramChunk = 64;

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int HC>
__global__ void __launch_bounds__(256, 2) attn_gram_mma_kernel(
    const __half* __restrict__ qkv, int npix, int w, int dim, int heads, long long pix,
    long long row, long long img, bool dense, float* __restrict__ part, int nparts,
    int px_per_block) {
  constexpr int MT = HC / 16, NT = HC / 8;
  extern __shared__ __align__(16) __half gsm[];  // [2][kGramChunk][rs]
  const int rs = 2 * dim + 8;                    // padded row pitch (halves)
  const int n = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hd = warp % heads, slice = warp / heads, nslices = 8 / heads;
  const int kpw = kGramChunk / nslices / 16;  // 16-pixel k-steps per warp and chunk
  const int groups = 2 * dim / 8;
  const __half* base = qkv + n * img;
  const int p_begin = blockIdx.x * px_per_block;
  const int p_end = min(npix, p_begin + px_per_block);
  const int nchunks = (p_end - p_begin + kGramChunk - 1) / kGramChunk;

  // thread = (8-channel group g0, pixel pp0 + k * pstep of each chunk); groups divides 256
  const int g0 = threadIdx.x % groups, pstep = 256 / groups;
  auto stage = [&](int chunk, int buf) {
    __half* dst = gsm + buf * kGramChunk * rs + g0 * 8;
    const int p0 = p_begin + chunk * kGramChunk;
    for (int pp = threadIdx.x / groups; pp < kGramChunk; pp += pstep) {
      const int p = p0 + pp;
      const bool ok = p < p_end;
      // contiguous views need no division
      const long long off =
          dense ? (long long)p * pix : (long long)(p / w) * row + (long long)(p % w) * pix;
      cp_async16(dst + pp * rs, ok ? base + off + g0 * 8 : qkv, ok ? 16 : 0);
    }
  };

  float G[MT][NT][4], Dq[MT][2][4], Dk[MT][2][4];
#pragma unroll
  for (int a = 0; a < MT; ++a) {
#pragma unroll
    for (int b = 0; b < NT; ++b)
#pragma unroll
      for (int e = 0; e < 4; ++e) G[a][b][e] = 0.f;
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
      for (int e = 0; e < 4; ++e) Dq[a][b][e] = Dk[a][b][e] = 0.f;
  }
  // ldmatrix row address of this lane: matrix mi = lane / 8, row r = lane % 8
  const int mi = lane >> 3, r8 = lane & 7;
  const int qcol = hd * HC, kcol = dim + hd * HC;

  if (nchunks > 0) stage(0, 0);
  asm volatile("cp.async.commit_group;\n" ::: "memory");
  for (int ch = 0; ch < nchunks; ++ch) {
    if (ch + 1 < nchunks) stage(ch + 1, (ch + 1) & 1);
    asm volatile("cp.async.commit_group;\n" ::: "memory");
    asm volatile("cp.async.wait_group 1;\n" ::: "memory");
    __syncthreads();
    const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(gsm + (ch & 1) * kGramChunk * rs);
    for (int ks = 0; ks < kpw; ++ks) {
      const int p0 = (slice * kpw + ks) * 16;
      // A operands (channels x pixels): matrices (m 0-7, k 0-7), (m 8-15, k 0-7),
      // (m 0-7, k 8-15), (m 8-15, k 8-15)
      uint32_t aq[MT][4], ak[MT][4];
      const int arow = p0 + ((mi & 2) ? 8 : 0) + r8;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int acol = mt * 16 + ((mi & 1) ? 8 : 0);
        ldsm_x4_t(sbase + (uint32_t)(arow * rs + qcol + acol) * 2u, aq[mt]);
        ldsm_x4_t(sbase + (uint32_t)(arow * rs + kcol + acol) * 2u, ak[mt]);
      }
      // B operands (pixels x channels), two n-tiles per ldmatrix: (k 0-7, j), (k 8-15, j),
      // (k 0-7, j+1), (k 8-15, j+1)
      uint32_t bk[NT][2], bq[NT][2];
      const int brow = p0 + ((mi & 1) ? 8 : 0) + r8;
#pragma unroll
      for (int j = 0; j < NT; j += 2) {
        const int bcol = (j + (mi >> 1)) * 8;
        uint32_t t[4];
        ldsm_x4_t(sbase + (uint32_t)(brow * rs + kcol + bcol) * 2u, t);
        bk[j][0] = t[0];
        bk[j][1] = t[1];
        bk[j + 1][0] = t[2];
        bk[j + 1][1] = t[3];
        ldsm_x4_t(sbase + (uint32_t)(brow * rs + qcol + bcol) * 2u, t);
        bq[j][0] = t[0];
        bq[j][1] = t[1];
        bq[j + 1][0] = t[2];
        bq[j + 1][1] = t[3];
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma16816(G[mt][nt], aq[mt], bk[nt][0], bk[nt][1]);
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          mma16816(Dq[mt][e], aq[mt], bq[2 * mt + e][0], bq[2 * mt + e][1]);
          mma16816(Dk[mt][e], ak[mt], bk[2 * mt + e][0], bk[2 * mt + e][1]);
        }
      }
    }
    __syncthreads();  // all reads of this buffer done before it is refilled
  }
  asm volatile("cp.async.wait_all;\n" ::: "memory");

  // The partial slot of (block, pixel slice): Gram [dim][HC] then the squared norms [2 dim];
  // this warp writes its head's rows and norms, each entry once (no atomics: the softmax sums
  // the slots in a fixed order, so the result does not depend on scheduling).
  // accumulator element e of a tile: row gid (+8 for e >= 2), column 2 * tig + (e & 1)
  const int gid = lane >> 2, tig = lane & 3;
  float* gn = part + ((long long)n * nparts + blockIdx.x * nslices + slice) * (dim * HC + 2 * dim);
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = mt * 16 + gid + (e >= 2 ? 8 : 0), j = nt * 8 + 2 * tig + (e & 1);
        gn[(hd * HC + i) * HC + j] = G[mt][nt][e];
      }
  // diagonals: n-tile 2mt holds rows mt*16 + 0..7 (elements 0, 1), n-tile 2mt+1 rows
  // mt*16 + 8..15 (elements 2, 3); element (gid, 2 tig + b) is diagonal when gid == 2 tig + b
  float* sn = gn + dim * HC;
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int e = 0; e < 2; ++e)
#pragma unroll
      for (int b = 0; b < 2; ++b)
        if (gid == 2 * tig + b) {
          const int i = mt * 16 + e * 8 + gid;
          sn[hd * HC + i] = Dq[mt][e][2 * e + b];
          sn[dim + hd * HC + i] = Dk[mt][e][2 * e + b];
        }
}

// attn[n][h][i][j] = softmax_j( G_ij / (max(|q_i|, eps) max(|k_j|, eps)) * T[h] )
// red[n][e] = sum over the nparts partial slots of part[n][k][e] (one thread per element,
// coalesced): the Gram [dim][c] and squared norms [2 dim] of each picture. Eight accumulators
// (slot k goes to accumulator k % 8) keep eight loads in flight per thread; they are combined
// in a fixed tree, so the result is the same on every run.
__global__ void attn_reduce_kernel(const float* __restrict__ part, int nparts, long long stride,
                                   int n_img, float* __restrict__ red) {
  const long long id = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (id >= (long long)n_img * stride) return;
  const long long n = id / stride, e = id - n * stride;
  const float* p = part + n * nparts * stride + e;
  float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  int k = 0;
  for (; k + 8 <= nparts; k += 8) {
#pragma unroll
    for (int j = 0; j < 8; ++j) a[j] += __ldg(p + (long long)(k + j) * stride);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j)
    if (k + j < nparts) a[j] += __ldg(p + (long long)(k + j) * stride);
  red[id] = ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
}

// One attention row (picture n, row ri = h*c + i) from the reduced Gram and norms.
__global__ void attn_softmax_kernel(const float* __restrict__ red, const float* __restrict__ temp,
                                    float* __restrict__ attn, int n_img, int dim, int heads) {
  const int c = dim / heads;
  long long row = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= (long long)n_img * dim) return;
  const int n = (int)(row / dim), ri = (int)(row % dim);
  const int hd = ri / c;
  const long long stride = (long long)dim * c + 2 * dim;
  const float* g = red + n * stride + (long long)ri * c;
  const float* sq = red + n * stride + (long long)dim * c;
  const float nq = fmaxf(sqrtf(sq[ri]), 1e-12f);
  float vals[64];
  float mx = -INFINITY;
  for (int j = 0; j < c; ++j) {
    const float nk = fmaxf(sqrtf(sq[dim + hd * c + j]), 1e-12f);
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

// out[p][h*C+i] = sum_j attn[h][i][j] * v[p][h*C+j] for head width C (16 or 32): thread =
// (pixel, head), warp = 32 pixels of one head, so every shared-memory read of the attention
// matrix is a broadcast; v is read once. Block = 256 threads = 8 warps over heads x pixels.
template <int C>
__global__ void __launch_bounds__(256) attn_apply_head_kernel(
    const __half* __restrict__ qkv, const float* __restrict__ attn, __half* __restrict__ out,
    int h, int w, int dim, int heads, long long pix, long long row, long long img, long long opix,
    long long orow, long long oimg) {
  extern __shared__ __align__(16) float sa[];  // [heads][C][C] of picture n
  const int n = blockIdx.y;
  for (int t = threadIdx.x; t < dim * C; t += blockDim.x) sa[t] = attn[(long long)n * dim * C + t];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hd = warp % heads;
  const int pw = 8 / heads;  // pixel warps per block
  const long long p = ((long long)blockIdx.x * pw + warp / heads) * 32 + lane;
  if (warp >= pw * heads || p >= (long long)h * w) return;
  const int py = (int)(p / w), px = (int)(p % w);
  const __half* vp = qkv + n * img + py * row + px * pix + 2 * dim + hd * C;
  float v[C];
#pragma unroll
  for (int j0 = 0; j0 < C; j0 += 8) {
    float t8[8];
    ld8(vp + j0, t8);
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) v[j0 + jj] = t8[jj];
  }
  const float* A = sa + hd * C * C;
  __half* op = out + n * oimg + py * orow + px * opix + hd * C;
#pragma unroll
  for (int i0 = 0; i0 < C; i0 += 8) {
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < C; j += 4) {
        const float4 a4 = *reinterpret_cast<const float4*>(A + (i0 + i) * C + j);
        s = fmaf(a4.x, v[j], s);
        s = fmaf(a4.y, v[j + 1], s);
        s = fmaf(a4.z, v[j + 2], s);
        s = fmaf(a4.w, v[j + 3], s);
      }
      o[i] = s;
    }
    st8(op + i0, o);
  }
}

// The attention apply folded into the following 1x1 projection (attention.rs:328-372 applies
// project_out to A.V): W'_n[k][h*c + j] = sum_i W_o[k][h*c + i] * A_n[h][i][j], one weight set
// per picture, scaled by `s` and written as f16 straight into conv_tc_kernel's blocked weight
// image (K-step blocks [bn][kc], 16-byte chunk j of row r at j ^ f(r)). Rows / columns beyond
// dim (padding of the packed layer) are zero. W_o is PyTorch [dim][dim] f32.
__global__ void attn_fold_kernel(const float* __restrict__ wo, const float* __restrict__ attn,
                                 int dim, int c, float s, __half* __restrict__ wout, int npad,
                                 int cin_pad, int kc, int bn) {
  const int n = blockIdx.y;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= npad * cin_pad) return;
  const int r = idx / cin_pad, j = idx % cin_pad;
  float acc = 0.f;
  if (r < dim && j < dim) {
    const int hd = j / c, jj = j % c;
    const float* A = attn + (long long)n * dim * c + (long long)hd * c * c;
    const float* W = wo + (long long)r * dim + hd * c;
    for (int i = 0; i < c; ++i) acc = fmaf(__ldg(W + i), __ldg(A + i * c + jj), acc);
  }
  const int cc = j / kc, col = j % kc, nt = r / bn, rr = r % bn;
  const int f = kc == 64 ? (rr & 7) : kc == 32 ? ((rr >> 1) & 3) : ((rr >> 2) & 1);
  __half* blk = wout + (long long)n * npad * cin_pad + ((long long)cc * (npad / bn) + nt) * bn * kc;
  blk[rr * kc + (((col >> 3) ^ f) << 3) + (col & 7)] = __float2half_rn(acc * s);
}

// attn_reduce_kernel + attn_softmax_kernel + attn_fold_kernel in one launch for the common
// shapes (c = 16 or 32, packed layer without padding rows or columns, power-of-two kc / bn):
// block (head hd, picture n) of kFoldThreads threads
//  1. sums the head's Gram block and norms over the partial slots (every thread eight slots
//     in flight, the same fixed combination as attn_reduce_kernel),
//  2. takes the c x c softmax with a warp per row (32 / c rows per warp, shuffle reductions of
//     the row max and sum in a fixed tree),
//  3. writes the head's columns of W_o . blockdiag(A) in the packed layout from the head's W_o
//     columns staged in shared memory (dim <= 256).
constexpr int kFoldThreads = 512;
template <int C>
__global__ void __launch_bounds__(kFoldThreads) attn_fold_fused_kernel(
    const float* __restrict__ part, int nparts, long long stride, const float* __restrict__ temp,
    const float* __restrict__ wo, int dim, float s, __half* __restrict__ wout, int npad,
    int cin_pad, int lkc, int lbn) {
  __shared__ float sa[C * C];    // the head's Gram block, then its attention matrix
  __shared__ float sn[2 * C];    // q norms of its rows, k norms of its columns
  __shared__ float sw[256 * C];  // W_o[r][hd * C + i] at sw[r * C + i]
  const int hd = blockIdx.x, n = blockIdx.y;
  const float* p = part + (long long)n * nparts * stride;
  for (int e = threadIdx.x; e < C * C + 2 * C; e += blockDim.x) {
    const long long off = e < C * C     ? (long long)(hd * C + e / C) * C + e % C
                          : e < C * C + C ? (long long)dim * C + hd * C + (e - C * C)
                                          : (long long)dim * C + dim + hd * C + (e - C * C - C);
    const float* q = p + off;
    float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    int k = 0;
    for (; k + 8 <= nparts; k += 8) {
#pragma unroll
      for (int j = 0; j < 8; ++j) a[j] += __ldg(q + (long long)(k + j) * stride);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (k + j < nparts) a[j] += __ldg(q + (long long)(k + j) * stride);
    const float v = ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
    if (e < C * C)
      sa[e] = v;
    else
      sn[e - C * C] = v;
  }
  for (int e = threadIdx.x; e < dim * C; e += blockDim.x)
    sw[e] = __ldg(wo + (long long)(e / C) * dim + hd * C + e % C);
  __syncthreads();
  {
    // softmax: lane l of a warp is column l % C of row (warp * 32 + l) / C (+ 32 / C rows per
    // pass over the warps)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int RPW = 32 / C;  // rows per warp per pass
    const int j = lane % C;
    const float tmp = temp[hd];
    const float nk = fmaxf(sqrtf(sn[C + j]), 1e-12f);
    for (int i = warp * RPW + lane / C; i < C; i += (kFoldThreads / 32) * RPW) {
      const float nq = fmaxf(sqrtf(sn[i]), 1e-12f);
      const float v = sa[i * C + j] / (nq * nk) * tmp;
      float mx = v;
#pragma unroll
      for (int o = C / 2; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float ex = expf(v - mx);
      float sum = ex;
#pragma unroll
      for (int o = C / 2; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      sa[i * C + j] = ex / sum;
    }
  }
  __syncthreads();
  const int kc = 1 << lkc, bnm = (1 << lbn) - 1;
  for (int idx = threadIdx.x; idx < dim * C; idx += blockDim.x) {
    const int r = idx / C, jj = idx % C, j = hd * C + jj;
    float acc = 0.f;
#pragma unroll 8
    for (int i = 0; i < C; ++i) acc = fmaf(sw[r * C + i], sa[i * C + jj], acc);
    const int cc = j >> lkc, col = j & (kc - 1), nt = r >> lbn, rr = r & bnm;
    const int f = kc == 64 ? (rr & 7) : kc == 32 ? ((rr >> 1) & 3) : ((rr >> 2) & 1);
    __half* blk = wout + (long long)n * npad * cin_pad +
                  ((((long long)cc * (npad >> lbn) + nt) << lbn) << lkc);
    blk[(rr << lkc) + (((col >> 3) ^ f) << 3) + (col & 7)] = __float2half_rn(acc * s);
  }
}

// planar f32 latents [pictures][C][LH][LW] -> NHWC f16 [n][h][w] at channel offset; per-image
// window origin (x, y) and picture index in `origin` (device int triplets).
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
  const int sx = origin[3 * n] + x, sy = origin[3 * n + 1] + y;
  const long long plane = (long long)LH * LW;
  src += (long long)origin[3 * n + 2] * C * plane;  // the tile's picture
  const float* s = src + (long long)sy * LW + sx;
  __half* d = dst + n * img + (long long)y * row + (long long)x * pix;
  for (int ch = 0; ch + 1 < C; ch += 2)
    *reinterpret_cast<__half2*>(d + ch) = __floats2half2_rn(__ldg(s + ch * plane), __ldg(s + (ch + 1) * plane));
  if (C & 1) d[C - 1] = __float2half_rn(__ldg(s + (C - 1) * plane));
}

// The same gather with one thread per (pixel, group of 8 channels), x fastest: the 8 plane
// reads of a warp are coalesced along x and each thread writes one 16-byte store (C % 8 == 0
// and 16-byte aligned channel groups).
__global__ void gather_latent8_kernel(const float* __restrict__ src, int C, int LH, int LW,
                                      const int* __restrict__ origin, __half* __restrict__ dst,
                                      int n_img, int h, int w, long long pix, long long row,
                                      long long img) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int groups = C >> 3;
  const long long total = (long long)n_img * h * w * groups;
  if (idx >= total) return;
  const int x = (int)(idx % w);
  long long r = idx / w;
  const int g = (int)(r % groups);
  r /= groups;
  const int y = (int)(r % h), n = (int)(r / h);
  const int sx = origin[3 * n] + x, sy = origin[3 * n + 1] + y;
  const long long plane = (long long)LH * LW;
  src += (long long)origin[3 * n + 2] * C * plane;  // the tile's picture
  const float* sp = src + (long long)(8 * g) * plane + (long long)sy * LW + sx;
  uint4 u;
  __half2* hv = reinterpret_cast<__half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i)
    hv[i] = __floats2half2_rn(__ldg(sp + (2 * i) * plane), __ldg(sp + (2 * i + 1) * plane));
  *reinterpret_cast<uint4*>(dst + n * img + (long long)y * row + (long long)x * pix + 8 * g) = u;
}

}  // namespace

void launch_layer_norm(const TView& x, const TView& y, const float* gamma, const float* beta,
                       cudaStream_t s) {
  long long pixels = (long long)x.n * x.h * x.w;
  if (x.c <= 256 && pixels < (1ll << 30)) {
    const int lpp = x.c <= 64 ? 8 : x.c <= 128 ? 16 : 32;
    const int grid = blocks_for(pixels, kLnPix * (256 / lpp));
    const bool xd = x.row == x.w * x.pix && x.img == x.h * x.row;
    const bool yd = y.row == y.w * y.pix && y.img == y.h * y.row;
#define ZJAI_LN_SEG(L)                                                                       \
  layer_norm_seg_kernel<L><<<grid, 256, 0, s>>>(x.p, y.p, (int)pixels, x.h, x.w, x.c, x.pix,  \
                                                x.row, x.img, xd, y.pix, y.row, y.img, yd,    \
                                                gamma, beta)
    if (lpp == 8)
      ZJAI_LN_SEG(8);
    else if (lpp == 16)
      ZJAI_LN_SEG(16);
    else
      ZJAI_LN_SEG(32);
#undef ZJAI_LN_SEG
    return;
  }
  layer_norm_kernel<<<blocks_for(pixels, 8), 256, 0, s>>>(x.p, y.p, x.n, x.h, x.w, x.c, x.pix,
                                                          x.row, x.img, y.pix, y.row, y.img,
                                                          gamma, beta);
}

template <bool GATE>
static void launch_dw3x3_t(const TView& x, const TView& y, const float* wt, int sms,
                           cudaStream_t s) {
  using S = DwShape<GATE>;
  static bool attr_set = false;  // two tile buffers exceed the default 48 KB window
  if (!attr_set) {
    cudaFuncSetAttribute(dw3x3_kernel<GATE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         2 * S::smem);
    attr_set = true;
  }
  const int cg_out = (GATE ? x.c / 2 : x.c) / 8;
  const int cblocks = (cg_out + 7) / 8;
  DwTiles T;
  T.tiles_x = (x.w + S::TW - 1) / S::TW;
  T.tiles_y = (x.h + kDwTH - 1) / kDwTH;
  T.count = x.n * T.tiles_x * T.tiles_y;
  const int per = std::max(1, std::min(T.count, 2 * sms / cblocks));  // two CTAs per SM
  dw3x3_kernel<GATE><<<cblocks * per, 256, 2 * S::smem, s>>>(
      x.p, y.p, x.h, x.w, x.c, x.pix, x.row, x.img, y.pix, y.row, y.img, wt, T, cblocks);
}

template <bool GATE>
static int launch_dw3x3_stream(Ctx* ctx, const TView& x, const TView& y, const float* wt,
                               cudaStream_t s) {
  using S = DsShape<GATE>;
  CUtensorMap tm;
  ZJAI_TRY(make_tile_map(ctx, &tm, x, 64, S::SW, 1));
  static bool attr_set = false;  // the stage ring exceeds the default 48 KB window
  if (!attr_set) {
    cudaFuncSetAttribute(dw3x3_stream_kernel<GATE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         S::smem);
    attr_set = true;
  }
  DsUnits U;
  U.strips = (x.w + S::TW - 1) / S::TW;
  U.cblocks = ((GATE ? x.c / 2 : x.c) + 63) / 64;
  // Band height: a multiprocessor's time is about its rounds of units times the rows a unit
  // stages (band + 2 halo rows); take the band that minimises that product (the tallest on a
  // tie), so that the last round of units does not leave most multiprocessors idle.
  U.band = kDsBand;
  long long best = -1;
  for (int b = kDsBand; b >= 8; --b) {
    const long long units = (long long)x.n * U.strips * ((x.h + b - 1) / b) * U.cblocks;
    const long long cost = (units + ctx->sms - 1) / ctx->sms * (b + 2);
    if (best < 0 || cost < best) {
      best = cost;
      U.band = b;
    }
  }
  U.bands = (x.h + U.band - 1) / U.band;
  U.count = x.n * U.strips * U.bands * U.cblocks;
  const int grid = std::min(U.count, ctx->sms);
  dw3x3_stream_kernel<GATE><<<grid, kDsThreads + 32, S::smem, s>>>(
      tm, y.p, x.h, x.w, x.c, y.pix, y.row, y.img, wt, U, ctx->d_err);
  return cuda_check(cudaGetLastError(), "dw3x3_stream_kernel launch");
}

int launch_dw3x3(Ctx* ctx, const TView& x, const TView& y, const float* wt, bool gate,
                 cudaStream_t s) {
  if (x.n * x.h * x.w == 0 || x.c == 0) return ZJAI_OK;
  // the streaming kernel's TMA boxes start at channel multiples of 8 (16 bytes): the gate's
  // second half must start on one
  const bool tma_ok = (reinterpret_cast<uintptr_t>(x.p) & 15) == 0 && x.pix % 8 == 0 &&
                      x.row % 8 == 0 && x.img % 8 == 0 && (!gate || (x.c / 2) % 8 == 0);
  if (tma_ok)
    return gate ? launch_dw3x3_stream<true>(ctx, x, y, wt, s)
                : launch_dw3x3_stream<false>(ctx, x, y, wt, s);
  if (gate)
    launch_dw3x3_t<true>(x, y, wt, ctx->sms, s);
  else
    launch_dw3x3_t<false>(x, y, wt, ctx->sms, s);
  return cuda_check(cudaGetLastError(), "dw3x3_kernel launch");
}

// Launch geometry of the Gram step: `blocks` per picture, `per_block` pixels (mma path) or
// pixel chunks (generic path) per block, and the partial slots per picture (one per block and
// pixel slice) that the softmax sums.
struct GramPlan {
  bool mma;
  int blocks, per_block, nparts;
};
static GramPlan gram_plan(int n, int dim, int heads, int npix, int sms) {
  const int c = dim / heads;
  GramPlan g;
  g.mma = (c == 16 || c == 32) && (heads == 2 || heads == 4 || heads == 8);
  if (g.mma) {
    // two blocks per SM (registers allow two) over the whole batch, one wave, whole chunks
    // per block; 8 / heads warps share a head's pixels (the slices)
    const int chunks = (npix + kGramChunk - 1) / kGramChunk;
    // (at most 16 blocks per picture: small batches keep few partial slots to sum)
    const int splits = std::max(1, std::min(std::min(chunks, 16), (2 * sms) / std::max(1, n)));
    g.per_block = ((chunks + splits - 1) / splits) * kGramChunk;
    g.blocks = (npix + g.per_block - 1) / g.per_block;
    g.nparts = g.blocks * (8 / heads);
  } else {
    const int chunks = (npix + kGramPix - 1) / kGramPix;
    g.per_block = std::max(1, chunks / 64);
    g.blocks = (chunks + g.per_block - 1) / g.per_block;
    g.nparts = g.blocks;
  }
  return g;
}

// Gram, norms and softmax: the attention matrices attn[n][h][i][j] (in the scratch).
// The Gram partial slots (at scratch), then (unless gram_only) their ordered sum and the
// softmax; returns the attention matrices [n][dim][c].
static float* attention_weights(const TView& qkv, int heads, const float* temp, float* scratch,
                                int sms, cudaStream_t s, bool gram_only = false) {
  const int dim = qkv.c / 3;
  const int c = dim / heads;
  const int n = qkv.n;
  const int npix = qkv.h * qkv.w;
  const GramPlan gp = gram_plan(n, dim, heads, npix, sms);
  const long long stride = (long long)dim * c + 2 * dim;  // Gram [dim][c], norms [2 dim]
  float* part = scratch;                                  // n * nparts partial slots
  float* red = part + (size_t)n * gp.nparts * stride;     // n reduced slots
  float* attn = red + (size_t)n * stride;                 // n * dim * c
  if (gp.mma) {
    const int smem = 2 * kGramChunk * (2 * dim + 8) * (int)sizeof(__half);
    static bool attr_set = false;
    if (!attr_set) {  // covers dim <= 8 * 32
      const int most = 2 * kGramChunk * (2 * 256 + 8) * (int)sizeof(__half);
      cudaFuncSetAttribute(attn_gram_mma_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           most);
      cudaFuncSetAttribute(attn_gram_mma_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           most);
      attr_set = true;
    }
    dim3 g1(gp.blocks, n);
    const bool dense = qkv.row == qkv.w * qkv.pix;  // rows contiguous within a picture
    if (c == 32)
      attn_gram_mma_kernel<32><<<g1, 256, smem, s>>>(qkv.p, npix, qkv.w, dim, heads, qkv.pix,
                                                     qkv.row, qkv.img, dense, part, gp.nparts,
                                                     gp.per_block);
    else
      attn_gram_mma_kernel<16><<<g1, 256, smem, s>>>(qkv.p, npix, qkv.w, dim, heads, qkv.pix,
                                                     qkv.row, qkv.img, dense, part, gp.nparts,
                                                     gp.per_block);
  } else {
    dim3 g1(gp.blocks, n);
    attn_gram_kernel<<<g1, 256, kGramPix * 2 * dim * sizeof(float), s>>>(
        qkv.p, n, npix, qkv.w, dim, heads, qkv.pix, qkv.row, qkv.img, part, gp.nparts,
        gp.per_block);
  }
  if (gram_only) return attn;
  attn_reduce_kernel<<<blocks_for((long long)n * stride, 256), 256, 0, s>>>(part, gp.nparts,
                                                                           stride, n, red);
  attn_softmax_kernel<<<blocks_for((long long)n * dim, 128), 128, 0, s>>>(red, temp, attn, n, dim,
                                                                         heads);
  return attn;
}

static bool pow2(int v) { return v > 0 && (v & (v - 1)) == 0; }

static bool fold_fused(int dim, int heads, const ConvLayer& L) {
  const int c = dim / heads;
  return (c == 16 || c == 32) && dim <= 256 && L.npad == dim && L.cin_pad == dim &&
         pow2(L.kc) && pow2(L.bn);
}

int attention_fold_launches(int dim, int heads, const ConvLayer& L) {
  return fold_fused(dim, heads, L) ? 2 : 4;
}

void launch_attention_fold(const TView& qkv, int heads, const float* temp, const float* wo,
                           float wscale, const ConvLayer& L, __half* wout, float* scratch,
                           int sms, cudaStream_t s) {
  const int dim = qkv.c / 3;
  const int c = dim / heads;
  const int n = qkv.n;
  if (fold_fused(dim, heads, L)) {
    // Gram partial slots, then their ordered sum + softmax + fold per (head, picture)
    const GramPlan gp = gram_plan(n, dim, heads, qkv.h * qkv.w, sms);
    const long long stride = (long long)dim * c + 2 * dim;
    attention_weights(qkv, heads, temp, scratch, sms, s, /*gram_only=*/true);
    const int lkc = __builtin_ctz((unsigned)L.kc), lbn = __builtin_ctz((unsigned)L.bn);
    dim3 g(heads, n);
    if (c == 32)
      attn_fold_fused_kernel<32><<<g, kFoldThreads, 0, s>>>(scratch, gp.nparts, stride, temp, wo,
                                                            dim, wscale, wout, L.npad, L.cin_pad,
                                                            lkc, lbn);
    else
      attn_fold_fused_kernel<16><<<g, kFoldThreads, 0, s>>>(scratch, gp.nparts, stride, temp, wo,
                                                            dim, wscale, wout, L.npad, L.cin_pad,
                                                            lkc, lbn);
    return;
  }
  const float* attn = attention_weights(qkv, heads, temp, scratch, sms, s);
  dim3 g(blocks_for((long long)L.npad * L.cin_pad, 256), n);
  attn_fold_kernel<<<g, 256, 0, s>>>(wo, attn, dim, dim / heads, wscale, wout, L.npad,
                                     L.cin_pad, L.kc, L.bn);
}

void launch_attention(const TView& qkv, const TView& out, int heads, const float* temp,
                      float* scratch, int sms, cudaStream_t s) {
  const int dim = qkv.c / 3;
  const int c = dim / heads;
  const int n = qkv.n;
  const int npix = qkv.h * qkv.w;
  const float* attn = attention_weights(qkv, heads, temp, scratch, sms, s);
  if ((c == 16 || c == 32) && 8 % heads == 0) {
    const int px_per_block = 32 * (8 / heads);
    dim3 g3(blocks_for((long long)npix, px_per_block), n);
    const size_t smem = sizeof(float) * dim * c;
    if (c == 32)
      attn_apply_head_kernel<32><<<g3, 256, smem, s>>>(qkv.p, attn, out.p, qkv.h, qkv.w, dim,
                                                       heads, qkv.pix, qkv.row, qkv.img, out.pix,
                                                       out.row, out.img);
    else
      attn_apply_head_kernel<16><<<g3, 256, smem, s>>>(qkv.p, attn, out.p, qkv.h, qkv.w, dim,
                                                       heads, qkv.pix, qkv.row, qkv.img, out.pix,
                                                       out.row, out.img);
  } else {
    dim3 g3(blocks_for((long long)npix, 256), dim / 8, n);
    attn_apply_kernel<<<g3, 256, 0, s>>>(qkv.p, attn, out.p, n, qkv.h, qkv.w, dim, heads,
                                         qkv.pix, qkv.row, qkv.img, out.pix, out.row, out.img);
  }
}

size_t attention_scratch_floats(int n_img, int dim, int heads, int npix, int sms) {
  const int c = dim / heads;
  const GramPlan gp = gram_plan(n_img, dim, heads, npix, sms);
  return (size_t)n_img * ((size_t)(gp.nparts + 1) * ((size_t)dim * c + 2 * (size_t)dim) +
                          (size_t)dim * c);
}

void launch_gather_latent(const float* src, int C, int LH, int LW, const int* origin,
                          const TView& dst, cudaStream_t s) {
  long long total = (long long)dst.n * dst.h * dst.w;
  if (C % 8 == 0 && dst.pix % 8 == 0 && dst.row % 8 == 0 && dst.img % 8 == 0 &&
      (reinterpret_cast<uintptr_t>(dst.p) & 15) == 0) {
    gather_latent8_kernel<<<blocks_for(total * (C / 8), 256), 256, 0, s>>>(
        src, C, LH, LW, origin, dst.p, dst.n, dst.h, dst.w, dst.pix, dst.row, dst.img);
    return;
  }
  gather_latent_kernel<<<blocks_for(total, 256), 256, 0, s>>>(src, C, LH, LW, origin, dst.p, dst.n,
                                                               dst.h, dst.w, dst.pix, dst.row,
                                                               dst.img);
}

}  // namespace zjai
