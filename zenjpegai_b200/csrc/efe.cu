// EFE post-filters on the reconstructed chroma planes (src/filters/efe_linear.rs,
// src/filters/efe_nonlinear.rs): the luma-aided linear filter and the luma-driven non-linear
// correction with its on/off switch, bit-exact with the crate's f32 arithmetic.
//
// The host resolves the coded parameters (regions and kernels of the linear filter, per-tile
// network weights of the non-linear one) exactly as the crate does; each kernel then computes
// output samples. The crate materialises replicate-padded phase planes (`phase_plane`); here
// the kernels read the samples a padded-plane position stands for straight from the
// full-resolution planes (`phase_col`), so nothing but the outputs is written.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <vector>

#include "api_common.h"

namespace zjai {
namespace {

constexpr int kEfeMaxRegions = 6;  // largest split (header.rs:619)
constexpr int kEfeBins = 8;        // `hist_split_num` (efe_nonlinear.rs:27)

// `EFElinear.cands` (efe_linear.rs:34-73): the regions of each candidate split as fractions
// [row_start, row_end, col_start, col_end] of the phase plane; region counts header.rs:619.
// Constants of the format.
constexpr int kNSplits[8] = {1, 2, 2, 3, 3, 4, 6, 6};
constexpr double kSplits[8][6][4] = {
    {{0, 1, 0, 1}},
    {{0, .5, 0, 1}, {.5, 1, 0, 1}},
    {{0, 1, 0, .5}, {0, 1, .5, 1}},
    {{0, 1, 0, .33}, {0, 1, .33, .66}, {0, 1, .66, 1}},
    {{0, .33, 0, 1}, {.33, .66, 0, 1}, {.66, 1, 0, 1}},
    {{0, .5, 0, .5}, {0, .5, .5, 1}, {.5, 1, 0, .5}, {.5, 1, .5, 1}},
    {{0, .33, 0, .5}, {0, .33, .5, 1}, {.33, .66, 0, .5}, {.33, .66, .5, 1}, {.66, 1, 0, .5},
     {.66, 1, .5, 1}},
    {{0, .5, 0, .33}, {.5, 1, 0, .33}, {0, .5, .33, .66}, {.5, 1, .33, .66}, {0, .5, .66, 1},
     {.5, 1, .66, 1}},
};
// `EFElinear.DCT_IF_4TAP` (efe_linear.rs:77-110): 4x4 half-sample interpolation taps of the
// sub-sampling phases (none, horizontal, vertical, diagonal). Constants of the format.
constexpr float kDctIf[4][16] = {
    {0},
    {0, 0, 0, 0, -0.0625f, -0.4375f, 0.5625f, -0.0625f, 0, 0, 0, 0, 0, 0, 0, 0},
    {0, -0.0625f, 0, 0, 0, -0.4375f, 0, 0, 0, 0.5625f, 0, 0, 0, -0.0625f, 0, 0},
    {0.00390625f, -0.03515625f, -0.03515625f, 0.00390625f,
     -0.03515625f, -0.68359375f, 0.31640625f, -0.03515625f,
     -0.03515625f, 0.31640625f, 0.31640625f, -0.03515625f,
     0.00390625f, -0.03515625f, -0.03515625f, 0.00390625f},
};

// `deinteger` (efe_linear.rs:113-115)
float deinteger(long long code) { return (float)(code - 32767) / 2048.0f; }

// `split_edge` (efe_linear.rs:128-131): round(f * (s + 31) / 32) * 32, ties to even
int split_edge(double f, int s) { return (int)std::nearbyint(f * (double)(s + 31) / 32.0) * 32; }

struct EfeRegion {
  int r0, r1, c0, c1, k, before;
  float chroma[4][16];  // per sub-sampling phase group, k x k taps (identity / DCT-IF in)
  float luma[16];
};

struct EfeLinearTables {
  EfeRegion reg[2][kEfeMaxRegions];
  int nreg[2];
  float mean[2];
};

// `regions` (efe_linear.rs:134-219) of plane p. Returns a zjai status.
int build_regions(const zjai_efe_linear_set& set, int p, bool coded_444, int s0, int s1,
                  EfeLinearTables* t) {
  const bool weighted = set.cand[p] >= 0;
  const int cand = weighted ? set.cand[p] : 0, fl = weighted ? set.filter_len[p] : 0;
  if (set.cand[p] < -1 || cand >= 8 || fl < 0 || fl > 4 || (weighted && fl == 0))
    return fail(ZJAI_INVALID_DATA, "EFE linear: filter set out of range");
  if (weighted && (!set.chroma_codes[p] || !set.luma_codes[p]))
    return fail(ZJAI_INVALID_DATA, "EFE linear: filter count");
  int n = 0;
  for (int num = 0; num < kNSplits[cand]; ++num) {
    const double* sp = kSplits[cand][num];
    const int r0 = split_edge(sp[0], s0), c0 = split_edge(sp[2], s1);
    const int r1 = std::min(split_edge(sp[1], s0), s0), c1 = std::min(split_edge(sp[3], s1), s1);
    if (r0 >= r1 || c0 >= c1) continue;  // small pictures leave some regions empty
    EfeRegion& r = t->reg[p][n++];
    r = EfeRegion{};
    r.r0 = r0, r.r1 = r1, r.c0 = c0, r.c1 = c1;
    // fL x fL kernels at the source's chroma resolution; else a 4x4 kernel with the fL x fL
    // filter placed at `off` and the DCT-IF taps added
    int off;
    if (coded_444) {
      r.k = fl;
      r.before = fl > 0 ? (fl - 1) / 2 : 0;
      off = 0;
    } else {
      r.k = 4;
      r.before = 1;
      off = 1 - (std::max(fl, 1) - 1) / 2;
    }
    const int k = r.k, centre = coded_444 ? (fl - 1) / 2 : 1;
    if (weighted) {
      const int phases = coded_444 ? 1 : 4;
      const uint32_t* cw = set.chroma_codes[p] + (size_t)num * phases * fl * fl;
      const uint32_t* lw = set.luma_codes[p] + (size_t)num * fl * fl;
      for (int ky = 0; ky < fl; ++ky)
        for (int kx = 0; kx < fl; ++kx) {
          const int dst = (off + ky) * k + off + kx;
          r.luma[dst] = deinteger((long long)lw[ky * fl + kx] + set.min_symbol);
          for (int i = 0; i < 4; ++i) {
            const int ph = coded_444 ? 0 : i;
            r.chroma[i][dst] = deinteger((long long)cw[(ph * fl + ky) * fl + kx] + set.min_symbol);
          }
        }
    }
    for (int i = 0; i < 4; ++i) {
      if (!coded_444)
        for (int q = 0; q < k * k; ++q) r.chroma[i][q] += kDctIf[i][q];
      r.chroma[i][centre * k + centre] += 1.0f;
    }
  }
  t->nreg[p] = n;
  return ZJAI_OK;
}

// `supported_format` (efe_linear.rs:364-379): the source / coded chroma formats the
// reference produces and decodes
bool supported_format(int s_ver, int s_hor, int c_ver, int c_hor) {
  if (s_ver == 1 && s_hor == 1)
    return (c_ver == 1 && c_hor == 1) || (c_ver == 1 && c_hor == 2) || (c_ver == 2 && c_hor == 2);
  if (s_ver == 1 && s_hor == 2) return c_ver == 1 && c_hor == 2;
  if (s_ver == 2 && s_hor == 2) return c_ver == 2 && c_hor == 2;
  return false;
}

// Column of src (a plane w samples wide) that position sx (>= 0) of phase px sampled every fh
// samples stands for in `phase_plane` (efe_linear.rs:238-275): the direct samples, then, past
// them, the plane's last column where the phase plane is wider than the phase has samples (odd
// widths), else the phase's last sample (the right border).
__device__ __forceinline__ int phase_col(int sx, int px, int fh, int w, int direct, int s1) {
  if (sx < direct) return px + sx * fh;
  return direct < s1 ? w - 1 : px + (direct - 1) * fh;
}

// `filter_plane` (efe_linear.rs:308-359). A block takes a 32 x 32 tile of one phase plane
// (blockIdx.z = plane * groups + sub-sampling phase group): split edges are multiples of 32, so
// the tile lies in one region (or in none: its samples stay 0). The block stages the padded
// windows of the chroma phase (mean subtracted) and of the luma phase that its taps reach in
// shared memory, each sample read once from the full-resolution plane with the padded phase
// plane's clamping done as index arithmetic; a thread then sums its four outputs' chroma and
// luma taps in (ky, kx) order, zero taps skipped, each a separate multiply and add, and stores
// (acc + mean) + luma.
constexpr int kEfeTile = 32, kEfeWin = kEfeTile + 3;
__global__ void __launch_bounds__(256) efe_linear_kernel(
    const float* __restrict__ y, int h, int w, const float* __restrict__ u,
    const float* __restrict__ v, int ch, int cw, int fv, int fh, int s0, int s1,
    const EfeLinearTables* __restrict__ tab, float* __restrict__ out_u,
    float* __restrict__ out_v) {
  __shared__ float cwin[kEfeWin][kEfeWin], lwin[kEfeWin][kEfeWin];
  __shared__ float wc[16], wl[16];  // taps at [ky * 4 + kx], zero outside the k x k kernel
  const int ngroups = fv * fh;
  const int p = blockIdx.z / ngroups, gi = blockIdx.z - p * ngroups;
  const int py = gi / fh, px = gi - py * fh, group = py * 2 + px;
  const int xx0 = blockIdx.x * kEfeTile, yy0 = blockIdx.y * kEfeTile;
  const int tid = threadIdx.y * 32 + threadIdx.x;
  const float* src = p ? v : u;
  float* out = p ? out_v : out_u;
  const EfeRegion* reg = nullptr;
  for (int i = 0; i < tab->nreg[p]; ++i) {
    const EfeRegion* r = &tab->reg[p][i];
    if (r->r0 <= yy0 && yy0 < r->r1 && r->c0 <= xx0 && xx0 < r->c1) reg = r;
  }
  const int k = reg ? reg->k : 0, before = reg ? reg->before : 0;
  const float mean = tab->mean[p];
  if (reg) {
    if (tid < 16) {
      const int ky = tid >> 2, kx = tid & 3;
      const bool in = ky < k && kx < k;
      wc[tid] = in ? reg->chroma[group][ky * k + kx] : 0.f;
      wl[tid] = in ? reg->luma[ky * k + kx] : 0.f;
    }
    // samples of the phase available without clamping (`direct` of phase_plane)
    const int dc = cw > px ? min((cw - px + fh - 1) / fh, s1) : 0;
    const int dl = w > px ? min((w - px + 1) / 2, s1) : 0;
    const int wn = kEfeTile + k - 1;
    // the window's columns (phase column xx0 + j - before clamped at 0, the right side by
    // phase_col) are the same for every row: a thread keeps its one or two
    const int j0 = threadIdx.x, j1 = threadIdx.x + 32;
    const int cx0 = phase_col(max(xx0 - before + j0, 0), px, fh, cw, dc, s1);
    const int lx0 = phase_col(max(xx0 - before + j0, 0), px, 2, w, dl, s1);
    const int cx1 = phase_col(max(xx0 - before + j1, 0), px, fh, cw, dc, s1);
    const int lx1 = phase_col(max(xx0 - before + j1, 0), px, 2, w, dl, s1);
    for (int i = threadIdx.y; i < wn; i += 8) {
      // padded row yy0 + i + 1 - before: phase row yy0 + i - before clamped to the plane
      const int sy = min(max(yy0 - before + i, 0), s0 - 1);
      const float* crow = src + (long long)min(sy * fv + py, ch - 1) * cw;
      const float* lrow = y + (long long)min(sy * 2 + py, h - 1) * w;
      cwin[i][j0] = __fsub_rn(__ldg(crow + cx0), mean);
      lwin[i][j0] = __ldg(lrow + lx0);
      if (j1 < wn) {
        cwin[i][j1] = __fsub_rn(__ldg(crow + cx1), mean);
        lwin[i][j1] = __ldg(lrow + lx1);
      }
    }
  }
  __syncthreads();
  // a thread's four outputs are the vertically adjacent rows r0 .. r0 + 3 of its column: each
  // window sample it loads serves every output whose taps reach it, in the outputs' (ky, kx)
  // order (window row rr = q + ky, so rr ascending is ky ascending for output q)
  const int tx = threadIdx.x, ox = (xx0 + tx) * fh + px, r0 = threadIdx.y * 4;
  float acc[4] = {0.f, 0.f, 0.f, 0.f}, lum[4] = {0.f, 0.f, 0.f, 0.f};
  if (reg) {
    float wcr[16], wlr[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      wcr[i] = wc[i];
      wlr[i] = wl[i];
    }
#pragma unroll
    for (int rr = 0; rr < 7; ++rr) {
      if (rr >= k + 3) break;
#pragma unroll
      for (int kx = 0; kx < 4; ++kx) {
        if (kx >= k) break;
        const float cv = cwin[r0 + rr][tx + kx], lv = lwin[r0 + rr][tx + kx];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int ky = rr - q;
          if (ky < 0 || ky > 3 || ky >= k) continue;
          const float a = wcr[ky * 4 + kx], b = wlr[ky * 4 + kx];
          if (a != 0.f) acc[q] = __fadd_rn(acc[q], __fmul_rn(a, cv));
          if (b != 0.f) lum[q] = __fadd_rn(lum[q], __fmul_rn(b, lv));
        }
      }
    }
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int oy = (yy0 + r0 + q) * fv + py;
    if (oy >= ch || ox >= cw) continue;
    out[(long long)oy * cw + ox] = reg ? __fadd_rn(__fadd_rn(acc[q], mean), lum[q]) : 0.f;
  }
}

// Per-tile parameters of the non-linear filter (efe_nonlinear.rs:37-48): w0, b0, the seven
// ceilings and the seven weights of conv2.
struct EfeTile {
  float w0, b0, ceil[kEfeBins - 1], w[kEfeBins - 1];
};

// One chroma sample per thread, both planes (blockIdx.z): the tile network where the plane's
// filter is on (efe_nonlinear.rs:128-138: relu(w0 l + x + b0) + sum w_k relu(l + ceil_k), each
// operation rounded on its own), then the on/off switch (efe_nonlinear.rs:145-187: mask 0 keeps
// it, 2 takes the alternative sample, else their mean). Tile (i, j) covers rows [i th,
// min((i + 1) th, hh)) and columns likewise: `tile_edge` (round(a / n * n) in doubles) is the
// identity on these integers.
__global__ void efe_nonlinear_kernel(const float* __restrict__ y, int w, int sv, int sh,
                                     float* __restrict__ u, float* __restrict__ v, int hh, int ww,
                                     const EfeTile* __restrict__ tiles_u,
                                     const EfeTile* __restrict__ tiles_v, int th, int tw, int nj,
                                     const uint8_t* __restrict__ mask_u,
                                     const uint8_t* __restrict__ mask_v, int bs, int mx,
                                     const float* __restrict__ alt_u,
                                     const float* __restrict__ alt_v) {
  const int x = blockIdx.x * blockDim.x + threadIdx.x, p = blockIdx.z;
  if (x >= ww) return;
  float* plane = p ? v : u;
  const EfeTile* tiles = p ? tiles_v : tiles_u;
  const uint8_t* mask = p ? mask_v : mask_u;
  for (int r = blockIdx.y; r < hh; r += gridDim.y) {
    const long long i = (long long)r * ww + x;
    float val = plane[i];
    if (tiles) {
      const EfeTile& t = tiles[(r / th) * nj + x / tw];
      const float l = __ldg(y + (long long)r * sv * w + (long long)x * sh);
      float acc = fmaxf(__fadd_rn(__fadd_rn(__fmul_rn(t.w0, l), val), t.b0), 0.f);
#pragma unroll
      for (int k = 0; k < kEfeBins - 1; ++k)
        acc = __fadd_rn(acc, __fmul_rn(t.w[k], fmaxf(__fadd_rn(l, t.ceil[k]), 0.f)));
      val = acc;
    }
    if (mask) {
      const uint8_t m = __ldg(mask + (long long)(r / bs) * mx + x / bs);
      if (m != 0) {
        const float a = __ldg((p ? alt_v : alt_u) + i);
        val = m == 2 ? a : __fdiv_rn(__fadd_rn(a, val), 2.0f);
      }
    }
    plane[i] = val;
  }
}

// copy a host parameter array of n elements into the call's arena
template <class T>
int stage_bytes(Ctx* ctx, const T* p, size_t n, const T** out, const char* what) {
  T* d = static_cast<T*>(ctx->arena.alloc(n * sizeof(T)));
  if (!d) return fail(ZJAI_LIMIT_EXCEEDED, std::string("device arena exhausted (") + what + ")");
  ZJAI_TRY(cuda_check(cudaMemcpyAsync(d, p, n * sizeof(T), cudaMemcpyHostToDevice, ctx->stream),
                      "EFE parameters H2D"));
  *out = d;
  return ZJAI_OK;
}

}  // namespace
}  // namespace zjai

using namespace zjai;

int zjai_efe_linear(zjai_ctx* ctx, const float* y, int h, int w, const float* u, const float* v,
                    int ch, int cw, int s_ver, int s_hor, int c_ver, int c_hor, int mean_u,
                    int mean_v, const zjai_efe_linear_set* set, float* out_u, float* out_v,
                    int mem) {
  ZJAI_TRY(ctx_enter(ctx));
  if (!y || !u || !v || !set || !out_u || !out_v)
    return fail(ZJAI_INVALID_ARGUMENT, "EFE linear: null pointer");
  if (mem != ZJAI_MEM_HOST && mem != ZJAI_MEM_DEVICE)
    return fail(ZJAI_INVALID_ARGUMENT, "mem must be HOST or DEVICE");
  // the crate's checks, in its order (efe_linear.rs:403-423, 134-160, 318-326)
  if (!supported_format(s_ver, s_hor, c_ver, c_hor))
    return fail(ZJAI_UNSUPPORTED, "EFE filters: chroma format the reference software does not support");
  if (h <= 0 || w <= 0) return fail(ZJAI_INVALID_ARGUMENT, "EFE linear: empty picture");
  const int fv = 3 - s_ver, fh = 3 - s_hor, s0 = (h + 1) / 2, s1 = (w + 1) / 2;
  if (ch <= 0 || cw <= 0 || (ch + fv - 1) / fv != s0 || (cw + fh - 1) / fh != s1)
    return fail(ZJAI_INVALID_ARGUMENT, "EFE linear: chroma plane size does not match the source format");
  const bool coded_444 = c_ver == s_ver && c_hor == s_hor;
  EfeLinearTables tab{};
  // float(code) / 100 in doubles, narrowed to f32 (efe_linear.rs:425-429)
  tab.mean[0] = (float)((double)mean_u / 100.0);
  tab.mean[1] = (float)((double)mean_v / 100.0);
  for (int p = 0; p < 2; ++p) {
    if (set->cand[p] < 0 && coded_444)
      return fail(ZJAI_UNSUPPORTED,
                  "EFE linear: unfiltered plane in a picture coded at the source's chroma resolution");
    ZJAI_TRY(build_regions(*set, p, coded_444, s0, s1, &tab));
  }
  ArenaScope scope(ctx);
  const size_t n = (size_t)h * w, nc = (size_t)ch * cw;
  const float *dy, *du, *dv;
  ZJAI_TRY(stage_in(ctx, y, n, mem, &dy));
  ZJAI_TRY(stage_in(ctx, u, nc, mem, &du));
  ZJAI_TRY(stage_in(ctx, v, nc, mem, &dv));
  if (mem == ZJAI_MEM_DEVICE) {
    // outputs over the inputs: the taps read neighbours, so filter copies
    for (const float** in : {&du, &dv}) {
      if (*in != out_u && *in != out_v) continue;
      float* copy = static_cast<float*>(ctx->arena.alloc(nc * sizeof(float)));
      if (!copy) return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (EFE input copy)");
      ZJAI_TRY(cuda_check(cudaMemcpyAsync(copy, *in, nc * sizeof(float), cudaMemcpyDeviceToDevice,
                                          ctx->stream),
                          "EFE copy"));
      *in = copy;
    }
  }
  const EfeLinearTables* dtab;
  ZJAI_TRY(stage_bytes(ctx, &tab, 1, &dtab, "EFE linear tables"));
  // the tables live in a host local: the copy must have read them before this call returns
  ZJAI_TRY(cuda_check(cudaStreamSynchronize(ctx->stream), "EFE tables H2D"));
  float *dou, *dov;
  ZJAI_TRY(stage_out_alloc(ctx, out_u, nc, mem, &dou));
  ZJAI_TRY(stage_out_alloc(ctx, out_v, nc, mem, &dov));
  dim3 grid((s1 + kEfeTile - 1) / kEfeTile, (s0 + kEfeTile - 1) / kEfeTile, 2 * fv * fh);
  ctx->launches++;
  if (ctx->profiling) ctx->tag = "EFE linear";
  timed_launch(ctx, false, 0.0, 4.0 * n + 16.0 * nc, [&] {
    efe_linear_kernel<<<grid, dim3(32, 8), 0, ctx->stream>>>(dy, h, w, du, dv, ch, cw, fv, fh,
                                                             s0, s1, dtab, dou, dov);
  });
  ZJAI_TRY(cuda_check(cudaGetLastError(), "EFE linear launch"));
  ZJAI_TRY(stage_out_finish(ctx, out_u, dou, nc, mem));
  ZJAI_TRY(stage_out_finish(ctx, out_v, dov, nc, mem));
  return finish_call(ctx, mem);
}

int zjai_efe_nonlinear(zjai_ctx* ctx, const float* y, int h, int w, float* u, float* v, int ch,
                       int cw, int s_ver, int s_hor, int c_ver, int c_hor,
                       const zjai_efe_nonlinear_params* prm, const float* alt_u,
                       const float* alt_v, int mem) {
  ZJAI_TRY(ctx_enter(ctx));
  if (!y || !u || !v || !prm) return fail(ZJAI_INVALID_ARGUMENT, "EFE non-linear: null pointer");
  if (mem != ZJAI_MEM_HOST && mem != ZJAI_MEM_DEVICE)
    return fail(ZJAI_INVALID_ARGUMENT, "mem must be HOST or DEVICE");
  if (!supported_format(s_ver, s_hor, c_ver, c_hor))
    return fail(ZJAI_UNSUPPORTED, "EFE filters: chroma format the reference software does not support");
  if (h < 0 || w < 0) return fail(ZJAI_INVALID_ARGUMENT, "EFE non-linear: picture size");
  // `downsample`: luma at the chroma positions (efe_nonlinear.rs:115-121)
  const int hh = (h + s_ver - 1) / s_ver, ww = (w + s_hor - 1) / s_hor;
  if (ch != hh || cw != ww)
    return fail(ZJAI_INVALID_ARGUMENT,
                "EFE non-linear: chroma plane size does not match the source format");
  // per-tile networks (`tiles`, efe_nonlinear.rs:55-98)
  std::vector<EfeTile> tiles[2];
  const int th = prm->tile_height, tw = prm->tile_width;
  const int nj = tw > 0 ? (ww + tw - 1) / tw : 0;
  for (int p = 0; p < 2; ++p) {
    if (!prm->codes[p] || hh == 0 || ww == 0) continue;
    if (th <= 0 || tw <= 0) return fail(ZJAI_INVALID_DATA, "EFE non-linear: zero tile size");
    const int ni = (hh + th - 1) / th, count = ni * nj;
    if (prm->ntiles < count || prm->ncodes[p] < count * kEfeBins || !prm->luma_min ||
        !prm->luma_max)
      return fail(ZJAI_INVALID_DATA, "EFE non-linear: fewer tile parameters than tiles");
    tiles[p].resize(count);
    for (int idx = 0; idx < count; ++idx) {
      const uint32_t* cd = prm->codes[p] + (size_t)idx * kEfeBins;
      float wf[kEfeBins];
      for (int k = 0; k < kEfeBins; ++k) wf[k] = deinteger((long long)cd[k] + prm->min_symbol);
      // Python doubles, narrowed to f32 where they meet a tensor
      const double minimum = (double)prm->luma_min[idx] / 100.0;
      const double gap = ((double)prm->luma_max[idx] / 100.0 - minimum) / kEfeBins;
      auto ceil_k = [&](int k) { return -(1.0f * (float)minimum + (float)k * (float)gap); };
      EfeTile& t = tiles[p][idx];
      t.w0 = wf[0];
      t.b0 = wf[0] * ceil_k(0);
      for (int k = 0; k < kEfeBins - 1; ++k) {
        t.ceil[k] = ceil_k(k + 1);
        t.w[k] = wf[k + 1];
      }
    }
  }
  // the on/off switch: `has_first_mask` (efe_nonlinear.rs:31-33) — the U mask decides
  const bool sw = prm->mask[0] && (prm->mask_h > 0 || prm->mask_w > 0);
  const int bs = prm->mask_bs;
  if (sw) {
    if (!alt_u || !alt_v)
      return fail(ZJAI_INVALID_DATA,
                  "EFE non-linear: on/off masks without the EFE linear filter's alternative picture");
    if (bs <= 0 || prm->mask_h != (hh + bs - 1) / bs || prm->mask_w != (ww + bs - 1) / bs)
      return fail(ZJAI_INVALID_DATA, "EFE non-linear: mask size does not cover the picture");
  }
  if (hh == 0 || ww == 0 || (tiles[0].empty() && tiles[1].empty() && !sw))
    return finish_call(ctx, mem);
  ArenaScope scope(ctx);
  const size_t n = (size_t)h * w, nc = (size_t)hh * ww;
  const float *dy, *du, *dv, *dau = nullptr, *dav = nullptr;
  ZJAI_TRY(stage_in(ctx, y, n, mem, &dy));
  ZJAI_TRY(stage_in(ctx, u, nc, mem, &du));
  ZJAI_TRY(stage_in(ctx, v, nc, mem, &dv));
  const EfeTile* dt[2] = {nullptr, nullptr};
  const uint8_t* dm[2] = {nullptr, nullptr};
  for (int p = 0; p < 2; ++p)
    if (!tiles[p].empty()) ZJAI_TRY(stage_bytes(ctx, tiles[p].data(), tiles[p].size(), &dt[p], "EFE tiles"));
  if (sw) {
    ZJAI_TRY(stage_in(ctx, alt_u, nc, mem, &dau));
    ZJAI_TRY(stage_in(ctx, alt_v, nc, mem, &dav));
    const size_t nm = (size_t)prm->mask_h * prm->mask_w;
    for (int p = 0; p < 2; ++p)
      if (prm->mask[p]) ZJAI_TRY(stage_bytes(ctx, prm->mask[p], nm, &dm[p], "EFE masks"));
  }
  // the tile tables live in host vectors: the copies must have read them before they go
  ZJAI_TRY(cuda_check(cudaStreamSynchronize(ctx->stream), "EFE parameters H2D"));
  ctx->launches++;
  if (ctx->profiling) ctx->tag = "EFE non-linear";
  dim3 grid((ww + 127) / 128, std::min(hh, 65535), 2);
  float* pu = const_cast<float*>(du);
  float* pv = const_cast<float*>(dv);
  timed_launch(ctx, false, 0.0, 4.0 * nc * (sw ? 7.0 : 5.0), [&] {
    efe_nonlinear_kernel<<<grid, 128, 0, ctx->stream>>>(dy, w, s_ver, s_hor, pu, pv, hh, ww,
                                                        dt[0], dt[1], th, tw, nj, dm[0], dm[1],
                                                        bs, prm->mask_w, dau, dav);
  });
  ZJAI_TRY(cuda_check(cudaGetLastError(), "EFE non-linear launch"));
  ZJAI_TRY(stage_out_finish(ctx, u, pu, nc, mem));
  ZJAI_TRY(stage_out_finish(ctx, v, pv, nc, mem));
  return finish_call(ctx, mem);
}
