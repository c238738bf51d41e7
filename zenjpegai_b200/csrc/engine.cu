// Host engine: errors, context, arena, TMA descriptors, weight packing, conv launch.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "engine.h"

namespace zjai {

// ---- errors -------------------------------------------------------------------------------
static thread_local std::string g_last_error;

void set_last_error(int code, const std::string& msg) {
  (void)code;
  g_last_error = msg;
}

const char* last_error_cstr() { return g_last_error.c_str(); }

int fail(int code, const std::string& msg) {
  set_last_error(code, msg);
  return code;
}

int cuda_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return ZJAI_OK;
  return fail(ZJAI_DEVICE, std::string(what) + ": " + cudaGetErrorString(e));
}

cudaEvent_t Ctx::take_event() {
  if (!ev_pool.empty()) {
    cudaEvent_t e = ev_pool.back();
    ev_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

void Ctx::clear_graphs() {
  for (auto& kv : graph_cache) {
    if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    for (void* p : kv.second.pins) cudaFreeHost(p);
  }
  graph_cache.clear();
}

int h2d_async(Ctx* ctx, void* dst, const void* src, size_t bytes, cudaStream_t s) {
  if (ctx->capture_pins) {
    void* pin = nullptr;
    ZJAI_TRY(cuda_check(cudaHostAlloc(&pin, bytes, cudaHostAllocDefault), "cudaHostAlloc"));
    std::memcpy(pin, src, bytes);
    ctx->capture_pins->push_back(pin);
    src = pin;
  }
  return cuda_check(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, s), "H2D");
}

// ---- arena --------------------------------------------------------------------------------
void* Arena::alloc(size_t bytes) {
  size_t start = (top + 255) & ~size_t(255);
  if (start + bytes > cap) return nullptr;
  top = start + bytes;
  peak = std::max(peak, top);
  return base + start;
}

int alloc_tensor(Ctx* ctx, int n, int h, int w, int c, TView* out, bool zero, Arena* arena,
                 cudaStream_t stream) {
  if (!arena) arena = &ctx->arena;
  if (!stream) stream = ctx->stream;
  int cp = (c + 7) & ~7;
  int ah = (h + 1) & ~1, aw = (w + 1) & ~1;
  size_t bytes = (size_t)n * ah * aw * cp * sizeof(__half);
  void* p = arena->alloc(bytes);
  if (!p)
    return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (" + std::to_string(bytes) +
                                         " more bytes, capacity " +
                                         std::to_string(arena->cap) + ")");
  TView v;
  v.p = static_cast<__half*>(p);
  v.n = n;
  v.h = h;
  v.w = w;
  v.c = c;
  v.pix = cp;
  v.row = (long long)aw * cp;
  v.img = (long long)ah * aw * cp;
  v.alloc_h = ah;
  v.alloc_w = aw;
  if (zero) ZJAI_TRY(cuda_check(cudaMemsetAsync(p, 0, bytes, stream), "memset"));
  *out = v;
  return ZJAI_OK;
}

// ---- TMA descriptors ------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static CUtensorMapSwizzle swizzle_for(int kc) {
  return kc == 64 ? CU_TENSOR_MAP_SWIZZLE_128B
                  : kc == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B;
}

static int encode(Ctx* ctx, CUtensorMap* m, int rank, void* addr, const cuuint64_t* dims,
                  const cuuint64_t* strides, const cuuint32_t* box, CUtensorMapSwizzle sw,
                  size_t span_bytes) {
  cuuint32_t es[5] = {1, 1, 1, 1, 1};
  if ((reinterpret_cast<uintptr_t>(addr) & 15) != 0)
    return fail(ZJAI_INVALID_ARGUMENT, "TMA base address not 16-byte aligned");
  for (int i = 0; i < rank - 1; ++i)
    if (strides[i] % 16 != 0)
      return fail(ZJAI_INVALID_ARGUMENT, "TMA stride not a multiple of 16 bytes");
  auto fn = reinterpret_cast<EncodeTiledFn>(ctx->encode_fn);
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, rank, addr, dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[256];
    snprintf(buf, sizeof buf, "cuTensorMapEncodeTiled failed (%d), rank %d", (int)r, rank);
    return fail(ZJAI_DEVICE, buf);
  }
  // Same workaround CUTLASS applies to tiled descriptors of tensors under 128 KiB on drivers
  // up to 13.1 (cute/atom/copy_traits_sm90_tma.hpp).
  if (ctx->driver_version <= 13010 && span_bytes < 131072)
    reinterpret_cast<uint64_t*>(m)[1] &= ~(1ull << 21);
  return ZJAI_OK;
}

int make_act_map(Ctx* ctx, CUtensorMap* m, const TView& v, int kc, int bw, int bh) {
  cuuint64_t dims[4] = {(cuuint64_t)v.c, (cuuint64_t)v.w, (cuuint64_t)v.h, (cuuint64_t)v.n};
  cuuint64_t strides[3] = {(cuuint64_t)v.pix * 2, (cuuint64_t)v.row * 2, (cuuint64_t)v.img * 2};
  cuuint32_t box[4] = {(cuuint32_t)kc, (cuuint32_t)bw, (cuuint32_t)bh, 1};
  size_t span = (size_t)v.img * v.n * 2;
  return encode(ctx, m, 4, v.p, dims, strides, box, swizzle_for(kc), span);
}

int make_act_map_s2(Ctx* ctx, CUtensorMap* m, const TView& v, int img, int kc, int bw, int bh) {
  int h2 = (v.h + 1) / 2, w2 = (v.w + 1) / 2;
  if (2 * h2 > v.alloc_h || 2 * w2 > v.alloc_w)
    return fail(ZJAI_INVALID_ARGUMENT, "stride-2 input without an even backing extent");
  cuuint64_t dims[5] = {(cuuint64_t)v.c, 2, (cuuint64_t)w2, 2, (cuuint64_t)h2};
  cuuint64_t strides[4] = {(cuuint64_t)v.pix * 2, (cuuint64_t)v.pix * 4, (cuuint64_t)v.row * 2,
                           (cuuint64_t)v.row * 4};
  cuuint32_t box[5] = {(cuuint32_t)kc, 1, (cuuint32_t)bw, 1, (cuuint32_t)bh};
  return encode(ctx, m, 5, v.p + (long long)img * v.img, dims, strides, box, swizzle_for(kc),
                (size_t)v.img * 2);
}

int make_tile_map(Ctx* ctx, CUtensorMap* m, const TView& v, int bc, int bx, int by) {
  cuuint64_t dims[4] = {(cuuint64_t)v.c, (cuuint64_t)v.w, (cuuint64_t)v.h, (cuuint64_t)v.n};
  cuuint64_t strides[3] = {(cuuint64_t)v.pix * 2, (cuuint64_t)v.row * 2, (cuuint64_t)v.img * 2};
  cuuint32_t box[4] = {(cuuint32_t)bc, (cuuint32_t)bx, (cuuint32_t)by, 1};
  return encode(ctx, m, 4, v.p, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE,
                (size_t)v.img * v.n * 2);
}

int make_store_map(Ctx* ctx, CUtensorMap* m, const TView& v, int bx, int by) {
  return make_tile_map(ctx, m, v, 16, bx, by);
}

// Picture `img` of an NHWC view as {C, R (dx), W / R, R (dy), H / R}: element (c, dx, X, dy, Y)
// is pixel (R Y + dy, R X + dx), so a box [16, 1, bx, 1, by] is one phase of bx x by pixels.
static int make_phase_store_map(Ctx* ctx, CUtensorMap* m, const TView& v, int img, int R, int bx,
                                int by) {
  cuuint64_t dims[5] = {(cuuint64_t)v.c, (cuuint64_t)R, (cuuint64_t)(v.w / R), (cuuint64_t)R,
                        (cuuint64_t)(v.h / R)};
  cuuint64_t strides[4] = {(cuuint64_t)v.pix * 2, (cuuint64_t)v.pix * 2 * R,
                           (cuuint64_t)v.row * 2, (cuuint64_t)v.row * 2 * R};
  cuuint32_t box[5] = {16, 1, (cuuint32_t)bx, 1, (cuuint32_t)by};
  return encode(ctx, m, 5, v.p + (long long)img * v.img, dims, strides, box,
                CU_TENSOR_MAP_SWIZZLE_NONE, (size_t)v.img * 2);
}

// ---- packing --------------------------------------------------------------------------------
static void choose_k(int cin, int* kc, int* cchunks) {
  *kc = cin > 32 ? 64 : cin > 16 ? 32 : 16;
  *cchunks = (cin + *kc - 1) / *kc;
}

static void choose_n(int ncols, int* bn, int* n_tiles) {
  int nt = (ncols + 255) / 256;
  int per = (ncols + nt - 1) / nt;
  *bn = (per + 15) & ~15;
  *n_tiles = nt;
}

// Power-of-two scale that brings the largest |w| into [2^13, 2^14): f16 keeps its full
// 11-bit significand for every weight that matters, far from overflow.
float pow2_weight_scale(const float* w, size_t n) {
  float mx = 0.f;
  for (size_t i = 0; i < n; ++i) mx = std::max(mx, std::fabs(w[i]));
  if (mx == 0.f || !std::isfinite(mx)) return 1.f;
  int e;
  std::frexp(mx, &e);  // mx = f * 2^e, f in [0.5, 1)
  int s = 14 - e;
  s = std::max(-24, std::min(s, 40));
  return std::ldexp(1.f, s);
}

// `wf` is [tap][npad][cin_pad]. The device copy is one contiguous block per K step and N tile
// — [bn rows][kc columns] f16, block (tap * cchunks + cc) * n_tiles + nt — already in the
// swizzled shared-memory image the MMA reads (16-byte chunk j of row r stored at j ^ f(r), the
// same XOR the TMA applies for 128/64/32-byte swizzles), so the kernel fetches each block with
// one bulk copy. A grouped layer (grp_pc > 0, one N tile) keeps only the output rows of the
// chunk's groups: rows cc * grp_pc * grp_n .. + grp_pc * grp_n. With `sparse_k` the K steps
// whose block is all zero are listed per N tile (ConvArgs::klist) so the kernel skips them.
static int upload_layer(Ctx* ctx, ConvLayer* L, const std::vector<float>& wf,
                        const std::vector<float>& bf, bool sparse_k) {
  float s = pow2_weight_scale(wf.data(), wf.size());
  L->scale = 1.f / s;
  const int taps = L->kh * L->kw, kc = L->kc, bn = L->bn;
  const int brows = L->grp_pc ? L->grp_pc * L->grp_n : bn;
  const int chunks16 = kc / 8;  // 16-byte chunks per row
  std::vector<__half> wh((size_t)taps * L->cchunks * L->n_tiles * brows * kc);
  size_t blk = 0;
  for (int tap = 0; tap < taps; ++tap)
    for (int cc = 0; cc < L->cchunks; ++cc)
      for (int nt = 0; nt < L->n_tiles; ++nt, ++blk) {
        __half* dst = wh.data() + blk * (size_t)brows * kc;
        const int row0 = L->grp_pc ? cc * brows : nt * bn;
        for (int r = 0; r < brows; ++r) {
          const int f = kc == 64 ? (r & 7) : kc == 32 ? ((r >> 1) & 3) : ((r >> 2) & 1);
          const float* src = wf.data() + ((size_t)tap * L->npad + row0 + r) * L->cin_pad + cc * kc;
          for (int j = 0; j < chunks16; ++j)
            for (int e = 0; e < 8; ++e)
              dst[(size_t)r * kc + ((j ^ f) * 8) + e] = __float2half_rn(src[j * 8 + e] * s);
        }
      }
  ZJAI_TRY(cuda_check(cudaMalloc(&L->w, wh.size() * sizeof(__half)), "cudaMalloc weights"));
  ZJAI_TRY(cuda_check(cudaMemcpy(L->w, wh.data(), wh.size() * sizeof(__half),
                                 cudaMemcpyHostToDevice),
                      "upload weights"));
  ZJAI_TRY(cuda_check(cudaMalloc(&L->bias, bf.size() * sizeof(float)), "cudaMalloc bias"));
  ZJAI_TRY(cuda_check(
      cudaMemcpy(L->bias, bf.data(), bf.size() * sizeof(float), cudaMemcpyHostToDevice),
      "upload bias"));
  // Live K steps per N tile: a block [bn rows][kc columns] of tap `tap`, chunk cc that is all
  // zero contributes nothing. A tile keeps at least its first K step (it initialises the
  // accumulator). When every block is live the kernel runs the dense loop (no lists).
  if (!sparse_k || L->grp_pc) return ZJAI_OK;
  const int ksteps = taps * L->cchunks;
  std::vector<int> koff(1, 0);
  std::vector<uint32_t> klist;
  for (int nt = 0; nt < L->n_tiles; ++nt) {
    const size_t before = klist.size();
    for (int kidx = 0; kidx < ksteps; ++kidx) {
      const int tap = kidx / L->cchunks, cc = kidx % L->cchunks;
      bool live = false;
      for (int r = 0; r < bn && !live; ++r) {
        const float* src =
            wf.data() + ((size_t)tap * L->npad + nt * bn + r) * L->cin_pad + cc * kc;
        for (int j = 0; j < kc && !live; ++j) live = src[j] != 0.f;
      }
      if (live)
        klist.push_back((uint32_t)kidx | (uint32_t)(tap % L->kw) << 16 |
                        (uint32_t)(tap / L->kw) << 21 | (uint32_t)cc << 26);
    }
    if (klist.size() == before) klist.push_back(0u);  // (tap 0, chunk 0)
    koff.push_back((int)klist.size());
  }
  if (klist.size() < (size_t)ksteps * L->n_tiles) {
    ZJAI_TRY(cuda_check(cudaMalloc(&L->klist, klist.size() * sizeof(uint32_t)), "cudaMalloc"));
    ZJAI_TRY(cuda_check(cudaMemcpy(L->klist, klist.data(), klist.size() * sizeof(uint32_t),
                                   cudaMemcpyHostToDevice),
                        "upload K list"));
    ZJAI_TRY(cuda_check(cudaMalloc(&L->koff, koff.size() * sizeof(int)), "cudaMalloc"));
    ZJAI_TRY(cuda_check(
        cudaMemcpy(L->koff, koff.data(), koff.size() * sizeof(int), cudaMemcpyHostToDevice),
        "upload K offsets"));
  }
  (void)ctx;
  return ZJAI_OK;
}

int pack_conv(Ctx* ctx, ConvLayer* L, const float* w, const float* b, int cin, int cout, int kh,
              int kw, int stride, int pad_h, int pad_w, int groups, const int* extra, int ps) {
  if (groups <= 0 || cin % groups || cout % groups || kh <= 0 || kw <= 0)
    return fail(ZJAI_MODEL, "conv2d: inconsistent channel/group/kernel configuration");
  if (stride != 1 && stride != 2) return fail(ZJAI_UNSUPPORTED, "conv2d: stride must be 1 or 2");
  if (ps < 1 || cout % (ps * ps)) return fail(ZJAI_INVALID_ARGUMENT, "pixel shuffle factor");
  const int et = extra ? extra[0] : 0, el = extra ? extra[1] : 0, eb = extra ? extra[2] : 0,
            er = extra ? extra[3] : 0;
  if (stride == 2 && (et || el || eb || er))
    return fail(ZJAI_UNSUPPORTED, "conv2d: extra padding with stride 2");
  *L = ConvLayer();
  L->cin = cin;
  // A stride-1 multi-tap grouped conv whose groups tile 64-channel chunks (16 or 32 input
  // channels a group) runs in halo mode without the zeros of the other groups: each K step
  // multiplies only a group's own channels into its own ocg output columns (ConvArgs::grp_pc).
  // Other grouped convs are dense-ified (zero weights between the groups).
  const int icg0 = cin / groups, ocg0 = cout / groups;
  const bool per_group = groups > 1 && ps == 1 && stride == 1 && kh * kw > 1 &&
                         (icg0 == 16 || icg0 == 32) && cin % 64 == 0 && ocg0 % 16 == 0 &&
                         cout <= 256 && !extra;
  choose_k(cin, &L->kc, &L->cchunks);
  L->cin_pad = L->kc * L->cchunks;
  L->kh = kh;
  L->kw = kw;
  L->stride = stride;
  L->pad_t = pad_h + et;
  L->pad_l = pad_w + el;
  L->pad_b = pad_h + eb;
  L->pad_r = pad_w + er;
  L->R = ps;
  L->cph = cout / (ps * ps);
  L->ncols = cout;
  choose_n(cout, &L->bn, &L->n_tiles);
  if (per_group) {
    // one pseudo-group per 64-channel chunk: the chunk's groups side by side (their weights
    // block-diagonal), 64 / icg0 * ocg0 output columns, one UMMA chain per subtile and chunk
    L->grp_n = ocg0 * (64 / icg0);
    L->grp_pc = 1;
  }
  L->npad = L->bn * L->n_tiles;
  const int taps = kh * kw, icg = cin / groups, ocg = cout / groups, r2 = ps * ps;
  std::vector<float> wf((size_t)taps * L->npad * L->cin_pad, 0.f), bf(L->npad, 0.f);
  for (int n = 0; n < cout; ++n) {
    const int phase = n / L->cph, co = n % L->cph;
    const int oc = co * r2 + phase;  // PyTorch pixel-shuffle channel order
    const int g = oc / ocg;
    if (b) bf[n] = b[oc];
    for (int i = 0; i < icg; ++i)
      for (int ky = 0; ky < kh; ++ky)
        for (int kx = 0; kx < kw; ++kx)
          wf[((size_t)(ky * kw + kx) * L->npad + n) * L->cin_pad + g * icg + i] =
              w[(((size_t)oc * icg + i) * kh + ky) * kw + kx];
  }
  L->flops_per_px = 2LL * cout * icg * kh * kw;
  return upload_layer(ctx, L, wf, bf, false);
}

int pack_convT(Ctx* ctx, ConvLayer* L, const float* w, const float* b, int cin, int cout, int k,
               int pad, int out_pad, int post_ps) {
  if (k <= 0 || pad >= k || out_pad >= 2 || post_ps < 1 || cout % (post_ps * post_ps))
    return fail(ZJAI_MODEL, "conv_transpose2d: unsupported geometry");
  *L = ConvLayer();
  // Output row 2i + p reads input row i + d with kernel row ky = p + pad - 2d.
  int dmin = 1 << 20, dmax = -(1 << 20);
  for (int p = 0; p < 2; ++p)
    for (int d = -k; d <= k; ++d) {
      int ky = p + pad - 2 * d;
      if (ky >= 0 && ky < k) {
        dmin = std::min(dmin, d);
        dmax = std::max(dmax, d);
      }
    }
  const int win = dmax - dmin + 1;
  L->cin = cin;
  choose_k(cin, &L->kc, &L->cchunks);
  L->cin_pad = L->kc * L->cchunks;
  L->kh = L->kw = win;
  L->stride = 1;
  L->pad_t = L->pad_l = -dmin;
  L->pad_b = L->pad_r = dmax;
  L->transposed = 1;
  L->t_k = k;
  L->t_pad = pad;
  L->t_outpad = out_pad;
  const int r2 = post_ps;
  L->R = 2 * r2;
  L->cph = cout / (r2 * r2);
  L->ncols = 4 * cout;
  // Each phase reads only some taps of the window (1, 2, 2 and 4 of the 2 x 2 window for
  // k = 3): an N tile whose phases leave taps unused skips them (ConvArgs::tmask). Narrower
  // tiles of single phases were measured slower in the network (the halo is re-read per N tile
  // and the MMA is not what bounds these layers), so the tiles stay as wide as choose_n makes
  // them.
  choose_n(L->ncols, &L->bn, &L->n_tiles);
  L->npad = L->bn * L->n_tiles;
  const int taps = win * win;
  std::vector<float> wf((size_t)taps * L->npad * L->cin_pad, 0.f), bf(L->npad, 0.f);
  long long live = 0;
  for (int n = 0; n < L->ncols; ++n) {
    const int q = n / L->cph, cc = n % L->cph;
    const int Y = q / L->R, X = q % L->R;
    const int py = Y / r2, dy2 = Y % r2, px = X / r2, dx2 = X % r2;
    const int co = cc * r2 * r2 + dy2 * r2 + dx2;
    if (b) bf[n] = b[co];
    for (int ty = 0; ty < win; ++ty) {
      const int ky = py + pad - 2 * (ty + dmin);
      if (ky < 0 || ky >= k) continue;
      for (int tx = 0; tx < win; ++tx) {
        const int kx = px + pad - 2 * (tx + dmin);
        if (kx < 0 || kx >= k) continue;
        ++live;
        for (int ci = 0; ci < cin; ++ci)
          wf[((size_t)(ty * win + tx) * L->npad + n) * L->cin_pad + ci] =
              w[(((size_t)ci * cout + co) * k + ky) * k + kx];
      }
    }
  }
  // live (tap, column) pairs summed over all columns = MACs per input pixel / cin
  L->flops_per_px = 2LL * live * cin;
  if (taps <= 32 && L->n_tiles > 1 && L->n_tiles <= kMaxTapMasks) {
    bool any_dead = false;
    for (int nt = 0; nt < L->n_tiles; ++nt) {
      uint32_t m = 0;
      for (int tap = 0; tap < taps; ++tap) {
        bool on = false;
        for (int n = nt * L->bn; n < (nt + 1) * L->bn && !on; ++n) {
          const float* row = wf.data() + ((size_t)tap * L->npad + n) * L->cin_pad;
          for (int ci = 0; ci < cin && !on; ++ci) on = row[ci] != 0.f;
        }
        if (on) m |= 1u << tap;
      }
      if (!m) m = 1u;  // a tile's first UMMA initialises its accumulator
      any_dead |= m != (taps == 32 ? 0xFFFFFFFFu : (1u << taps) - 1u);
      L->tmask[nt] = m;
    }
    L->tmask_on = any_dead ? 1 : 0;
  }
  return upload_layer(ctx, L, wf, bf, false);
}

void free_conv(ConvLayer* L) {
  if (L->w) cudaFree(L->w);
  if (L->bias) cudaFree(L->bias);
  if (L->klist) cudaFree(L->klist);
  if (L->koff) cudaFree(L->koff);
  L->w = nullptr;
  L->bias = nullptr;
  L->klist = nullptr;
  L->koff = nullptr;
}

void ConvLayer::out_size(int h, int w, int* oh, int* ow, int* out_h, int* out_w) const {
  if (!transposed) {
    *oh = (h + pad_t + pad_b - kh) / stride + 1;
    *ow = (w + pad_l + pad_r - kw) / stride + 1;
    *out_h = *oh * R;
    *out_w = *ow * R;
  } else {
    const int th = (h - 1) * 2 + t_k + t_outpad - 2 * t_pad;
    const int tw = (w - 1) * 2 + t_k + t_outpad - 2 * t_pad;
    *oh = (th + 1) / 2;
    *ow = (tw + 1) / 2;
    *out_h = th * (R / 2);
    *out_w = tw * (R / 2);
  }
}

// ---- launch ---------------------------------------------------------------------------------
static void pick_tile(int oh, int ow, int* bw, int* bh) {
  long long best = -1;
  int bbw = 16;
  const int cands[5] = {16, 32, 8, 64, 128};
  for (int c : cands) {
    int h = 128 / c;
    long long area = (long long)((ow + c - 1) / c) * c * ((oh + h - 1) / h) * h;
    if (best < 0 || area < best) {
      best = area;
      bbw = c;
    }
  }
  *bw = bbw;
  *bh = 128 / bbw;
}

int run_conv(Ctx* ctx, const ConvLayer& L, const TView& in, const ConvOut& o) {
  if (in.c != L.cin)
    return fail(ZJAI_INVALID_ARGUMENT, "conv: input channel count mismatch (" +
                                           std::to_string(in.c) + " vs " +
                                           std::to_string(L.cin) + ")");
  if (in.h <= 0 || in.w <= 0) return fail(ZJAI_INVALID_ARGUMENT, "conv: empty input");
  int oh, ow, out_h, out_w;
  L.out_size(in.h, in.w, &oh, &ow, &out_h, &out_w);
  if (oh <= 0 || ow <= 0) return fail(ZJAI_INVALID_ARGUMENT, "conv: input smaller than kernel");
  // Requested output extent (a crop of the natural one).
  int want_h = o.planar ? (o.out_h >= 0 ? o.out_h : out_h) : o.out.h;
  int want_w = o.planar ? (o.out_w >= 0 ? o.out_w : out_w) : o.out.w;
  if (want_h > out_h || want_w > out_w)
    return fail(ZJAI_INVALID_ARGUMENT, "conv: output view larger than the layer's output");
  oh = std::min(oh, (want_h + L.R - 1) / L.R);
  ow = std::min(ow, (want_w + L.R - 1) / L.R);
  if (!o.planar && (L.cph % 8 != 0))
    return fail(ZJAI_UNSUPPORTED, "conv: NHWC output needs a multiple of 8 channels");
  // the NHWC epilogues carry the sigmoid only in the CAB op (its one use on the networks)
  if (!o.planar && ((o.act1 == ACT_SIGMOID && o.op != OP_CAB) || o.act2 == ACT_SIGMOID))
    return fail(ZJAI_UNSUPPORTED, "conv: NHWC output takes the sigmoid only with the CAB op");

  ConvArgs a;
  memset(&a, 0, sizeof a);
  // Halo mode: a stride-1 conv with several taps and 64-channel chunks reads each chunk's
  // input once per tile (tile 8 x 16 plus its halo) instead of once per tap.
  // (A grouped layer is packed for halo mode and always qualifies.)
  a.halo = L.stride == 1 && L.kh * L.kw > 1 && L.kc == 64 && !L.klist && L.kw <= 9 &&
           L.kh <= 9;
  if (a.halo) {
    a.bw = 8;
    a.bh = 16;
  } else {
    pick_tile(oh, ow, &a.bw, &a.bh);
  }
  // Two M subtiles per tile (two accumulators of bn columns each, double-buffered: 4 bn TMEM
  // columns) when the N tile allows it and the picture is taller than one subtile.
  a.msub = (L.bn <= 128 && oh > a.bh) ? 2 : 1;
  if (a.halo) {
    a.hw = a.bw + L.kw - 1;
    a.hh = a.bh * a.msub + L.kh - 1;
    a.halo_bytes = ((uint32_t)a.hw * a.hh * L.kc * 2u + 1023u) & ~1023u;
  }
  a.tiles_x = (ow + a.bw - 1) / a.bw;
  a.tiles_y = (oh + a.bh * a.msub - 1) / (a.bh * a.msub);
  a.n_tiles = L.n_tiles;
  a.kw = L.kw;
  a.taps = L.kh * L.kw;
  a.pad_t = L.pad_t;
  a.pad_l = L.pad_l;
  a.s2 = L.stride == 2;
  a.cchunks = L.cchunks;
  a.kc = L.kc;
  a.bn = L.bn;
  const int brows = L.grp_pc ? L.grp_pc * L.grp_n : L.bn;
  const uint32_t stage =
      a.halo ? conv_bstage_bytes(L.kc, brows) : conv_stage_bytes(L.kc, brows, a.msub);
  a.grp_n = L.grp_n;
  a.grp_pc = L.grp_pc;
  // NHWC outputs leave through the TMA-store epilogue (staging slots in smem): unshuffled ones,
  // and shuffled ones whose phases are whole 16-channel chunks over an extent divisible by R
  // (so the phase maps clip exactly at the view's edge)
  const bool shuffle_store = !o.planar && L.R > 1 && L.cph % 16 == 0 &&
                             want_w % L.R == 0 && want_h % L.R == 0;
  const bool staged = !o.planar && (L.R == 1 || shuffle_store);
  // Halo ring depth: a layer with little MMA work per halo (narrow N) is bound by the halo
  // loads' latency, so it keeps up to kMaxHaloSlots halos in flight while at least 8 weight
  // stages still fit; the others keep 2 and spend the memory on weight stages.
  constexpr uint32_t kSmemMax = 232448u;
  // Residual prefetch: a TMA-store epilogue with a residual op loads each work item's residual
  // box(es) into shared memory one item ahead. Only 1x1 convs, whose few K steps leave the
  // epilogue on the critical path; a multi-tap conv keeps that memory for weight stages.
  a.nres = staged && o.op != OP_NONE && L.kh * L.kw == 1 ? (o.op == OP_CAB ? 2 : 1) : 0;
  if (a.nres && conv_fixed_smem(L.npad, staged, a.nres) + (a.halo ? 2 * a.halo_bytes : 0u) +
                        2 * stage > kSmemMax)
    a.nres = 0;
  a.hslots = 2;
  if (a.halo)
    for (int hs = kMaxHaloSlots; hs > 2; --hs)
      if (conv_fixed_smem(L.npad, staged, a.nres) + hs * a.halo_bytes + 8 * stage <= kSmemMax) {
        a.hslots = hs;
        break;
      }
  const uint32_t fixed =
      conv_fixed_smem(L.npad, staged, a.nres) + (a.halo ? a.hslots * a.halo_bytes : 0u);
  if (fixed + 2 * stage > kSmemMax)
    return fail(ZJAI_UNSUPPORTED, "conv: too many output columns for one launch");
  a.stages = (int)std::min<uint32_t>(kMaxStages, (kSmemMax - fixed) / stage);
  int tc = 32;
  while (tc < 2 * a.msub * L.bn) tc *= 2;
  a.tmem_cols = tc;
  a.oh = oh;
  a.ow = ow;
  a.bias = L.bias;
  a.scale = L.scale;
  a.act1 = o.act1;
  a.op = o.op;
  a.act2 = o.act2;
  a.R = L.R;
  a.lR = __builtin_ctz((unsigned)L.R);
  a.lbw = __builtin_ctz((unsigned)a.bw);
  if ((L.R & (L.R - 1)) != 0) return fail(ZJAI_UNSUPPORTED, "conv: shuffle factor must be a power of two");
  a.cph = L.cph;
  a.err = ctx->d_err;
  a.wait_cycles = ctx->wait_cycles;
  if (!o.planar) {
    a.out = o.out.p;
    a.out_pix = o.out.pix;
    a.out_row = o.out.row;
    a.out_img = o.out.img;
    a.out_h = want_h;
    a.out_w = want_w;
    if (o.op != OP_NONE) {
      if (!o.r1) return fail(ZJAI_INVALID_ARGUMENT, "conv: residual operand missing");
      a.r1 = o.r1->p;
      a.r1_pix = o.r1->pix;
      a.r1_row = o.r1->row;
      a.r1_img = o.r1->img;
    }
    if (o.op == OP_CAB) {
      if (!o.r2) return fail(ZJAI_INVALID_ARGUMENT, "conv: CAB operand missing");
      a.r2 = o.r2->p;
      a.r2_pix = o.r2->pix;
      a.r2_row = o.r2->row;
      a.r2_img = o.r2->img;
    }
    if (o.out2) {
      a.out2 = o.out2->p;
      a.o2_pix = o.out2->pix;
      a.o2_row = o.out2->row;
      a.o2_img = o.out2->img;
    }
  } else {
    a.planar = 1;
    a.denorm = o.denorm ? (o.clamp ? 1 : 2) : 0;
    a.pout = o.pout;
    a.pout2 = o.pout2;
    a.img_win = o.img_win;
    a.p_plane = o.p_plane;
    a.p_row = o.p_row;
    a.p_img = o.p_img;
    a.out_h = want_h;
    a.out_w = want_w;
    a.py0 = o.py0;
    a.px0 = o.px0;
    a.cy0 = o.cy0;
    a.cy1 = o.cy1;
    a.cx0 = o.cx0;
    a.cx1 = o.cx1;
    a.sv = o.sv;
    a.sh = o.sh;
    a.qbytes = o.qbytes;
    a.qmax = o.qmax;
    const bool pow2 = (o.sv & (o.sv - 1)) == 0 && (o.sh & (o.sh - 1)) == 0;
    a.lsv = pow2 ? __builtin_ctz((unsigned)o.sv) : -1;
    a.lsh = pow2 ? __builtin_ctz((unsigned)o.sh) : -1;
  }

  CUtensorMap tmO;  // output map of the TMA-store epilogue (unused in the other modes)
  memset(&tmO, 0, sizeof tmO);
  const int sbx = std::min(a.bw, 32);
  if (staged && !shuffle_store) ZJAI_TRY(make_store_map(ctx, &tmO, o.out, sbx, 32 / sbx));
  if (shuffle_store) {
    // per-picture phase maps in device memory (from the caller's arena, ordered on its stream)
    std::vector<CUtensorMap> pm(o.out.n);
    for (int i = 0; i < o.out.n; ++i)
      ZJAI_TRY(make_phase_store_map(ctx, &pm[i], o.out, i, L.R, sbx, 32 / sbx));
    Arena* ar = ctx->cur_arena ? ctx->cur_arena : &ctx->arena;
    void* dm = ar->alloc(sizeof(CUtensorMap) * pm.size());
    if (!dm) return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (tensor maps)");
    ZJAI_TRY(h2d_async(ctx, dm, pm.data(), sizeof(CUtensorMap) * pm.size(), ctx->stream));
    a.tmO_img = static_cast<const CUtensorMap*>(dm);
  }
  if (a.nres) {
    // residual maps with the output map's box: r1 then r2, one each or one per picture each
    const TView* rv[2] = {o.r1, o.r2};
    std::vector<CUtensorMap> rm;
    for (int k = 0; k < a.nres; ++k) {
      if (!shuffle_store) {
        CUtensorMap m;
        ZJAI_TRY(make_store_map(ctx, &m, *rv[k], sbx, 32 / sbx));
        rm.push_back(m);
      } else {
        for (int i = 0; i < o.out.n; ++i) {
          CUtensorMap m;
          ZJAI_TRY(make_phase_store_map(ctx, &m, *rv[k], i, L.R, sbx, 32 / sbx));
          rm.push_back(m);
        }
      }
    }
    Arena* ar = ctx->cur_arena ? ctx->cur_arena : &ctx->arena;
    void* dm = ar->alloc(sizeof(CUtensorMap) * rm.size());
    if (!dm) return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (tensor maps)");
    ZJAI_TRY(h2d_async(ctx, dm, rm.data(), sizeof(CUtensorMap) * rm.size(), ctx->stream));
    a.tmR = static_cast<const CUtensorMap*>(dm);
  }
  a.wblk = L.w;
  a.wblk_img = L.w_img;
  a.klist = L.klist;
  a.koff = L.koff;
  a.tmask_on = L.tmask_on;
  for (int i = 0; i < kMaxTapMasks; ++i) a.tmask[i] = L.tmask[i];
  cudaError_t lerr = cudaSuccess;
  char detail[256] = "";
  // Algorithmic bytes of the launch (the profile's memory figure for it): the input once, the
  // live weights once (f16: 2 bytes a MAC of one pixel = flops_per_px), the output once, and
  // the residual operands and the relu6 copy once each.
  const double out_elems = (double)in.n * want_h * want_w * L.cph;
  const double out_elt = o.planar ? (o.qbytes ? (double)o.qbytes : 4.0) : 2.0;
  const int extra_ops = o.planar ? 0 : (o.op == OP_CAB ? 2 : o.op != OP_NONE ? 1 : 0) +
                                          (o.out2 ? 1 : 0);
  const double bytes = 2.0 * in.n * in.h * in.w * L.cin + (double)L.flops_per_px +
                       out_elems * out_elt + 2.0 * out_elems * extra_ops;
  // an error left by an earlier asynchronous launch must not be reported as this one's
  ZJAI_TRY(cuda_check(cudaGetLastError(), "before conv launch"));
  if (!a.s2) {
    CUtensorMap tmA;
    if (a.halo)
      ZJAI_TRY(make_act_map(ctx, &tmA, in, L.kc, a.hw, a.hh));
    else
      ZJAI_TRY(make_act_map(ctx, &tmA, in, L.kc, a.bw, a.bh * a.msub));
    a.n_img = in.n;
    a.num_tiles = a.tiles_x * a.tiles_y * a.n_img * a.n_tiles;
    const double fl = (double)L.flops_per_px * oh * ow * in.n;
    ctx->launches++;
    timed_launch(ctx, true, fl, bytes, [&] {
      lerr = launch_conv(tmA, tmO, a, std::min(a.num_tiles, ctx->sms), ctx->stream, detail,
                         (int)sizeof detail);
    });
  } else {
    // The parity-split 5-D view has no batch axis: one tensor map per picture, kept in a
    // device array (from the caller's arena, ordered on its stream) that the producer indexes
    // by the tile's picture. One launch covers the whole batch.
    std::vector<CUtensorMap> maps(in.n);
    for (int i = 0; i < in.n; ++i)
      ZJAI_TRY(make_act_map_s2(ctx, &maps[i], in, i, L.kc, a.bw, a.bh * a.msub));
    Arena* ar = ctx->cur_arena ? ctx->cur_arena : &ctx->arena;
    void* dmaps = ar->alloc(sizeof(CUtensorMap) * maps.size());
    if (!dmaps) return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (tensor maps)");
    ZJAI_TRY(h2d_async(ctx, dmaps, maps.data(), sizeof(CUtensorMap) * maps.size(), ctx->stream));
    a.tmA_img = static_cast<const CUtensorMap*>(dmaps);
    a.n_img = in.n;
    a.num_tiles = a.tiles_x * a.tiles_y * a.n_img * a.n_tiles;
    const double fl = (double)L.flops_per_px * oh * ow * in.n;
    ctx->launches++;
    timed_launch(ctx, true, fl, bytes, [&] {
      lerr = launch_conv(maps[0], tmO, a, std::min(a.num_tiles, ctx->sms), ctx->stream, detail,
                         (int)sizeof detail);
    });
  }
  if (lerr != cudaSuccess) return fail(ZJAI_DEVICE, std::string("conv launch: ") + detail);
  return ZJAI_OK;
}

}  // namespace zjai
