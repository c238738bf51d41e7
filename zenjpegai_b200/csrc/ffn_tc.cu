// Fused FFN kernel (the scheme is in ffn_tc.cuh).
#include "ffn_tc.cuh"
#include "gate.cuh"
#include "ptx.cuh"

namespace zjai {

namespace {

constexpr uint32_t kXChunkBytes = 256u * 128u;  // one 64-channel slab of the halo, 256 rows
constexpr uint32_t kWinBytes = 64u * 128u;      // one W_in block [64][64] (a slice, K 64)
constexpr int kWinSlots = 4;
constexpr int kWoSlots = 2;                      // W_out blocks [dim][32]
constexpr uint32_t kGBytes = 256u * 64u;        // gated block of a slice: 2 x 128 rows x 32 ch
// f16 halo image of a slice: 64 channels (128 B) per pixel at a 136-byte pitch, so the
// drain's lanes (consecutive pixels, one 8-byte channel-pair slot) and the depthwise lanes
// (16 slots of one pixel per half-warp) both hit distinct banks
constexpr uint32_t kHPitch = 136u;
constexpr uint32_t kHBytes = (((uint32_t)kFfnHalo * kHPitch) + 127u) & ~127u;
constexpr uint32_t kWdBytes = 9u * 16u * 16u;   // depthwise weights of a slice, f32
constexpr int kWdSlots = 4;
constexpr uint32_t kBarBytes = 512u;  // mbarriers, TMEM address, abort word
constexpr uint32_t kGroupThreads = 32u * kFfnGroupWarps;

enum FfnBar : int {
  B_XF, B_XE,                                  // halo slabs full / free
  B_WIF, B_WIE = B_WIF + kWinSlots,            // W_in ring
  B_WOF = B_WIE + kWinSlots, B_WOE = B_WOF + kWoSlots,  // W_out ring
  B_WDF = B_WOE + kWoSlots, B_WDE = B_WDF + kWdSlots,  // depthwise weights ring
  // per warp group g (slices of parity g), two of each:
  B_INF = B_WDE + kWdSlots,  // project_in accumulator of the group's slice complete
  B_INE = B_INF + 2,         // ... drained (group threads)
  B_HF = B_INE + 2,          // halo image written (group threads)
  B_HE = B_HF + 2,           // ... read by every group thread
  B_GF = B_HE + 2,           // gated block written (group threads)
  B_GE = B_GF + 2,           // ... consumed by project_out
  B_OF = B_GE + 2,           // project_out accumulators of a tile complete
  B_OE,                      // ... drained (group 1's threads)
  B_DRAIN,                   // the two issuers' end-of-kernel drains
  B_COUNT = B_DRAIN + 2
};
static_assert(B_COUNT * 8 + 8 <= (int)kBarBytes, "FFN barrier area");

__device__ __forceinline__ float2 h2f(uint32_t u) {
  return __half22float2(*reinterpret_cast<const __half2*>(&u));
}
__device__ __forceinline__ uint32_t f2h(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

}  // namespace

size_t ffn_smem_bytes(int dim) {
  const size_t x = (size_t)(dim / 64) * kXChunkBytes;
  const size_t wo = (size_t)kWoSlots * dim * 64u;
  return 1024 + x + kWinSlots * kWinBytes + wo + 2u * kGBytes + 2u * kHBytes +
         kWdSlots * kWdBytes + kBarBytes;
}

__global__ void __launch_bounds__(kFfnThreads, 1)
    ffn_tc_kernel(const __grid_constant__ CUtensorMap tmX, const FfnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int kxn = a.dim >> 6;                   // 64-channel slabs of ln (K blocks of project_in)
  const uint32_t wob = (uint32_t)a.dim * 64u;  // one W_out block [dim][32]
  uint8_t* sX = smem;
  uint8_t* sWin = sX + kxn * kXChunkBytes;
  uint8_t* sWout = sWin + kWinSlots * kWinBytes;
  uint8_t* sG = sWout + kWoSlots * wob;  // 2 (per group)
  uint8_t* sH = sG + 2 * kGBytes;        // 2 (per group)
  uint8_t* sWd = sH + 2 * kHBytes;       // kWdSlots
  uint64_t* bars = reinterpret_cast<uint64_t*>(sWd + kWdSlots * kWdBytes);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + B_COUNT);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(bar(B_XF), 1);
    mbar_init(bar(B_XE), 1);
    for (int i = 0; i < kWinSlots; ++i) {
      mbar_init(bar(B_WIF + i), 1);
      mbar_init(bar(B_WIE + i), 1);
    }
    for (int i = 0; i < kWoSlots; ++i) {
      mbar_init(bar(B_WOF + i), 1);
      mbar_init(bar(B_WOE + i), 1);
    }
    for (int i = 0; i < kWdSlots; ++i) {
      mbar_init(bar(B_WDF + i), 1);
      mbar_init(bar(B_WDE + i), kGroupThreads);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(bar(B_INF + g), 1);
      mbar_init(bar(B_INE + g), kGroupThreads);
      mbar_init(bar(B_HF + g), kGroupThreads);
      mbar_init(bar(B_HE + g), kGroupThreads);
      mbar_init(bar(B_GF + g), kGroupThreads);
      mbar_init(bar(B_GE + g), 1);
      mbar_init(bar(B_DRAIN + g), 1);
    }
    mbar_init(bar(B_OF), 1);
    mbar_init(bar(B_OE), kGroupThreads);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&tmX);
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512u);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int S = a.nslice;  // slices per tile (even)

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    // Per tile the halo slabs, then per slice its W_in blocks and depthwise weights (the
    // project_out warp loads its own W_out blocks); the rings are deep enough that a wait here
    // does not hold back the next slice's project_in.
    if (lane == 0) {
      long long xi = 0, wi = 0, wd = 0;  // loads issued per ring
      const uint32_t xbox = (uint32_t)kFfnHalo * 128u;
      bool ok = true;
      for (int t = blockIdx.x; t < a.num_tiles && ok && !*abort_flag; t += gridDim.x) {
        const int tx = t % a.tiles_x, rest = t / a.tiles_x;
        const int ty = rest % a.tiles_y, n = rest / a.tiles_y;
        if (!mbar_wait_idle(bar(B_XE), (uint32_t)(xi & 1) ^ 1u, abort_flag, a.err,
                            DEV_TIMEOUT_EMPTY, 64))
          break;
        mbar_arrive_expect_tx(bar(B_XF), xbox * kxn);
        for (int kx = 0; kx < kxn; ++kx)
          tma_load_4d(smem_u32(sX) + kx * kXChunkBytes, &tmX, bar(B_XF), 64 * kx,
                      tx * kFfnTW - 1, ty * kFfnTH - 1, n);
        ++xi;
        {  // the tile's residual rows into L2 for its output stage, a whole tile later
          const int y0 = ty * kFfnTH, x0 = tx * kFfnTW;
          const int cols = min(kFfnTW, a.w - x0);
          const uint32_t rb = (uint32_t)(cols * a.x_pix * 2);
          for (int r = 0; r < kFfnTH && y0 + r < a.h; ++r)
            bulk_prefetch_l2(a.x + n * a.x_img + (long long)(y0 + r) * a.x_row +
                                 (long long)x0 * a.x_pix,
                             rb);
        }
        for (int c = 0; c < S && ok; ++c) {
          for (int kx = 0; kx < kxn && ok; ++kx) {
            const int s = (int)(wi % kWinSlots);
            ok = mbar_wait_idle(bar(B_WIE + s), (uint32_t)((wi / kWinSlots) & 1) ^ 1u,
                                abort_flag, a.err, DEV_TIMEOUT_EMPTY, 64);
            if (!ok) break;
            mbar_arrive_expect_tx(bar(B_WIF + s), kWinBytes);
            bulk_load(smem_u32(sWin) + s * kWinBytes, a.win + (size_t)(c * kxn + kx) * 4096,
                      kWinBytes, bar(B_WIF + s));
            ++wi;
          }
          if (!ok) break;
          {
            const int s = (int)(wd % kWdSlots);
            ok = mbar_wait_idle(bar(B_WDE + s), (uint32_t)((wd / kWdSlots) & 1) ^ 1u,
                                abort_flag, a.err, DEV_TIMEOUT_EMPTY, 64);
            if (!ok) break;
            mbar_arrive_expect_tx(bar(B_WDF + s), kWdBytes);
            bulk_load(smem_u32(sWd) + s * kWdBytes, a.wdw + (size_t)c * (kWdBytes / 4),
                      kWdBytes, bar(B_WDF + s));
            ++wd;
          }
        }
      }
      // every copy issued lands before the CTA's shared memory goes away
      if (xi > 0) mbar_wait_drain(bar(B_XF), (uint32_t)((xi - 1) & 1), a.err);
      auto drain_ring = [&](int base, int slots, long long issued) {
        for (int s = 0; s < slots; ++s)
          if (issued > s) {
            const long long last = ((issued - 1 - s) / slots) * slots + s;
            mbar_wait_drain(bar(base + s), (uint32_t)((last / slots) & 1), a.err);
          }
      };
      drain_ring(B_WIF, kWinSlots, wi);
      drain_ring(B_WDF, kWdSlots, wd);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- project_in issuer
    // Slice c (global index gc) goes into TMEM columns [128 g, 128 g + 128) of its group
    // g = c & 1 (two subtiles of N = 64: 32 ELU operands, 32 multipliers), once that group has
    // drained its previous slice.
    if (lane == 0) {
      const uint32_t id_in = idesc_f16(64u);
      const uint64_t dX = smem_desc(smem_u32(sX), 128u);
      const uint64_t dWi = smem_desc(smem_u32(sWin), 128u);
      long long wi = 0;
      bool ok = true;
      int it = 0;
      for (int t = blockIdx.x; t < a.num_tiles && ok && !*abort_flag; t += gridDim.x, ++it) {
        if (!mbar_wait(bar(B_XF), (uint32_t)(it & 1), abort_flag, a.err, DEV_TIMEOUT_FULL)) break;
        tc_fence_after();
        for (int c = 0; c < S && ok; ++c) {
          const long long gc = (long long)it * S + c;
          const int g = c & 1;
          if (!mbar_wait_sleep(bar(B_INE + g), (uint32_t)((gc >> 1) & 1) ^ 1u, abort_flag, a.err,
                               DEV_TIMEOUT_ACC_EMPTY)) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int kx = 0; kx < kxn; ++kx) {
            const int s = (int)(wi % kWinSlots);
            if (!mbar_wait(bar(B_WIF + s), (uint32_t)((wi / kWinSlots) & 1), abort_flag, a.err,
                           DEV_TIMEOUT_FULL)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t db = dWi + (uint64_t)((s * kWinBytes) >> 4);
            const uint64_t da = dX + (uint64_t)((kx * kXChunkBytes) >> 4);
            // the two subtiles' chains interleaved: consecutive UMMAs into one accumulator
            // serialise, independent ones overlap
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
#pragma unroll
              for (int sub = 0; sub < 2; ++sub)
                umma_f16(tmem + g * 128 + sub * 64, da + (uint64_t)sub * (16384u >> 4) + 2 * kk,
                         db + 2 * kk, id_in, (kx | kk) ? 1u : 0u);
            umma_commit(bar(B_WIE + s));
            ++wi;
          }
          if (!ok) break;
          umma_commit(bar(B_INF + g));
        }
        if (ok) umma_commit(bar(B_XE));  // the halo slabs are free
      }
      umma_commit(bar(B_DRAIN));
      mbar_wait_drain(bar(B_DRAIN), 0, a.err);
    }
  } else if (warp == kFfnOutWarp) {
    // ---------------------------------------------------------------- project_out issuer
    // Slice c's gated block (K = 32) times W_out[:, 32 c .. 32 c + 31] accumulates into TMEM
    // columns [256, 256 + 2 dim), in slice order. This thread also streams the W_out blocks
    // through a two-slot ring: after issuing slice gc it loads slice gc + 1's block into the
    // slot slice gc - 1 used (a slice's depthwise takes far longer than the copy).
    if (lane == 0) {
      const uint32_t id_out = idesc_f16((uint32_t)a.dim);
      const uint64_t dWo = smem_desc(smem_u32(sWout), 64u);
      const uint64_t dG = smem_desc(smem_u32(sG), 64u);
      long long wo = 0, wl = 0;  // slices issued, W_out blocks loaded
      auto load_wo = [&](int c) {
        const int s = (int)(wl & 1);
        mbar_arrive_expect_tx(bar(B_WOF + s), wob);
        bulk_load(smem_u32(sWout) + s * wob, a.wout + (size_t)c * a.dim * 32, wob,
                  bar(B_WOF + s));
        ++wl;
      };
      if (blockIdx.x < a.num_tiles) load_wo(0);
      bool ok = true;
      int it = 0;
      for (int t = blockIdx.x; t < a.num_tiles && ok && !*abort_flag; t += gridDim.x, ++it) {
        for (int c = 0; c < S; ++c) {
          const long long gc = (long long)it * S + c;
          const int g = c & 1, s = (int)(wo & 1);
          if (!mbar_wait_sleep(bar(B_GF + g), (uint32_t)((gc >> 1) & 1), abort_flag, a.err,
                               DEV_TIMEOUT_FULL) ||
              !mbar_wait(bar(B_WOF + s), (uint32_t)((wo >> 1) & 1), abort_flag, a.err,
                         DEV_TIMEOUT_FULL) ||
              (c == 0 && !mbar_wait_sleep(bar(B_OE), (uint32_t)(it & 1) ^ 1u, abort_flag, a.err,
                                          DEV_TIMEOUT_ACC_EMPTY))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t db = dWo + (uint64_t)((s * wob) >> 4);
          const uint64_t da = dG + (uint64_t)((g * kGBytes) >> 4);
#pragma unroll
          for (int kk = 0; kk < 2; ++kk)
#pragma unroll
            for (int sub = 0; sub < 2; ++sub)
              umma_f16(tmem + 256 + sub * a.dim, da + (uint64_t)sub * (8192u >> 4) + 2 * kk,
                       db + 2 * kk, id_out, (c > 0 || kk) ? 1u : 0u);
          umma_commit(bar(B_WOE + s));
          umma_commit(bar(B_GE + g));
          ++wo;
          // the next slice's W_out block (the next tile's first after the last), into the slot
          // of slice gc - 1 once its UMMAs are complete
          if (c + 1 < S || t + (int)gridDim.x < a.num_tiles) {
            if (wo >= 2 &&
                !mbar_wait(bar(B_WOE + (int)(wl & 1)), (uint32_t)(((wl - 2) >> 1) & 1), abort_flag,
                           a.err, DEV_TIMEOUT_EMPTY)) {
              ok = false;
              break;
            }
            load_wo(c + 1 < S ? c + 1 : 0);
          }
        }
        if (ok) umma_commit(bar(B_OF));
      }
      // the W_out copies in flight land before shared memory goes away
      for (int s = 0; s < 2; ++s)
        if (wl > s) {
          const long long last = ((wl - 1 - s) / 2) * 2 + s;
          mbar_wait_drain(bar(B_WOF + s), (uint32_t)((last >> 1) & 1), a.err);
        }
      umma_commit(bar(B_DRAIN + 1));
      mbar_wait_drain(bar(B_DRAIN + 1), 0, a.err);
    }
  } else {
    // ---------------------------------------------------------------- compute warps
    // Two groups of 8 warps; group g takes the slices c = g, g + 2, ..: drains its project_in
    // accumulator into its f16 halo image, then runs the depthwise 3x3 + ELU gate into its
    // gated block while the other group drains or computes the neighbouring slice.
    const int cw = warp - 2;  // 0 .. 15
    const int g = cw >> 3, w8 = cw & 7;
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const uint32_t trow = tmem + ((uint32_t)(32 * q) << 16);
    // drain role: subtile dsub, TMEM row 32 q + lane = halo pixel p
    const int dsub = w8 >> 2;
    const int p = dsub * 128 + 32 * q + lane;
    // depthwise role: output columns 2 cp, 2 cp + 1, rows 6 rh .. 6 rh + 5, channel pair j of
    // the slice (ELU operands 2j, 2j + 1 and their multipliers)
    const int j = lane & 15, cp = 2 * (w8 & 3) + (lane >> 4), rh = w8 >> 2;
    uint8_t* const hbuf = sH + g * kHBytes;
    uint8_t* const gbuf = sG + g * kGBytes;
    bool ok = true;
    int it = 0;
    for (int t = blockIdx.x; t < a.num_tiles && ok; t += gridDim.x, ++it) {
      const int tx = t % a.tiles_x, rest = t / a.tiles_x;
      const int ty = rest % a.tiles_y, n = rest / a.tiles_y;
      for (int c = g; c < S; c += 2) {
        const long long gc = (long long)it * S + c;
        const uint32_t ph = (uint32_t)((gc >> 1) & 1);  // phase of this group's barriers
        // ---- drain project_in: halo pixel p at p * kHPitch, channel pair k in the 8-byte
        // slot k: {elu operands 2k, 2k + 1, multipliers 2k, 2k + 1}
        if (!mbar_wait_sleep(bar(B_INF + g), ph, abort_flag, a.err, DEV_TIMEOUT_ACC_FULL)) {
          ok = false;
          break;
        }
        tc_fence_after();
        {
          // f16 of acc * scale + 0 (the unfused layer's epilogue with its zero bias)
          uint32_t hv[16][2];
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            float ve[16], vm[16];
            tmem_ld16x2(trow + g * 128 + dsub * 64 + 16 * hh,
                        trow + g * 128 + dsub * 64 + 32 + 16 * hh, ve, vm);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              hv[8 * hh + i][0] =
                  f2h(ve[2 * i] * a.scale_in + 0.f, ve[2 * i + 1] * a.scale_in + 0.f);
              hv[8 * hh + i][1] =
                  f2h(vm[2 * i] * a.scale_in + 0.f, vm[2 * i + 1] * a.scale_in + 0.f);
            }
          }
          tc_fence_before();
          mbar_arrive(bar(B_INE + g));
          // the accumulator is in registers; the halo image is free once every thread of the
          // group has finished the group's previous slice
          if (!mbar_wait_sleep(bar(B_HE + g), ph ^ 1u, abort_flag, a.err, DEV_TIMEOUT_ACC_FULL)) {
            ok = false;
            break;
          }
          if (p < kFfnHalo) {
            uint2* hp = reinterpret_cast<uint2*>(hbuf + p * kHPitch);
#pragma unroll
            for (int k = 0; k < 16; ++k) hp[k] = make_uint2(hv[k][0], hv[k][1]);
          }
        }
        mbar_arrive(bar(B_HF + g));
        const int ws = (int)(gc % kWdSlots);
        if (!mbar_wait_sleep(bar(B_HF + g), ph, abort_flag, a.err, DEV_TIMEOUT_ACC_FULL) ||
            !mbar_wait_sleep(bar(B_WDF + ws), (uint32_t)((gc / kWdSlots) & 1), abort_flag, a.err,
                             DEV_TIMEOUT_FULL) ||
            !mbar_wait_sleep(bar(B_GE + g), ph ^ 1u, abort_flag, a.err, DEV_TIMEOUT_ACC_FULL)) {
          ok = false;
          break;
        }
        // depthwise weights of the thread's channels per tap ([tap][pair] in the slice's slot)
        float4 wr[9];
        {
          const float4* wsrc = reinterpret_cast<const float4*>(sWd + ws * kWdBytes) + j;
#pragma unroll
          for (int tp = 0; tp < 9; ++tp) wr[tp] = wsrc[tp * 16];
        }
        // ---- depthwise 3x3 + gate over halo rows 6 rh .. 6 rh + 7 (rolling 3-row
        // accumulators; per output the taps in (ky, kx) order, the first one a product)
        {
          // gated block row op = (6 rh + o) * 16 + 2 cp + col: 64 bytes per row (64-byte
          // swizzle), the channel pair's 4 bytes in 16-byte chunk (j / 4) ^ ((op / 2) & 3), and
          // (op / 2) & 3 = cp & 3
          uint8_t* gcol[2];
#pragma unroll
          for (int col = 0; col < 2; ++col)
            gcol[col] = gbuf + (6 * rh * kFfnTW + 2 * cp + col) * 64 +
                        (((j >> 2) ^ (cp & 3)) << 4) + ((j & 3) << 2);
          const uint8_t* hrow = hbuf + (6 * rh * kFfnHW + 2 * cp) * kHPitch + 8 * j;
          float2 acc[3][2][2];
          auto row = [&](auto JJ, int i) {
            constexpr int J = decltype(JJ)::value;
            // halo column jx is tap kx = jx of output column 0 and kx = jx - 1 of column 1:
            // per accumulator the taps of a row still come in kx order
#pragma unroll
            for (int jx = 0; jx < 4; ++jx) {
              const uint2 u = *reinterpret_cast<const uint2*>(hrow + (i * kFfnHW + jx) * kHPitch);
              const float2 v[2] = {h2f(u.x), h2f(u.y)};
#pragma unroll
              for (int ky = 0; ky < 3; ++ky)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                  // input row i is tap ky of output row i - ky: rows outside the band's six
                  // take nothing (a compile-time condition once the rows are unrolled)
                  if (i - ky < 0 || i - ky > 5) continue;
                  float2(&s)[2][2] = acc[(J - ky + 3) % 3];
                  if (jx < 3) {
                    const float4 w4 = wr[ky * 3 + jx];
                    const float2 wv = e ? make_float2(w4.z, w4.w) : make_float2(w4.x, w4.y);
                    s[0][e] = (ky == 0 && jx == 0) ? __fmul2_rn(wv, v[e]) : ffma2(wv, v[e], s[0][e]);
                  }
                  if (jx > 0) {
                    const float4 w4 = wr[ky * 3 + jx - 1];
                    const float2 wv = e ? make_float2(w4.z, w4.w) : make_float2(w4.x, w4.y);
                    s[1][e] = (ky == 0 && jx == 1) ? __fmul2_rn(wv, v[e]) : ffma2(wv, v[e], s[1][e]);
                  }
                }
            }
            const int o = i - 2;  // output row complete with this input row
            if (o >= 0) {
              const float2(&so)[2][2] = acc[(J + 1) % 3];
#pragma unroll
              for (int col = 0; col < 2; ++col) {
                const float2 y = elu_gate2(so[col][0], so[col][1]);
                *reinterpret_cast<uint32_t*>(gcol[col] + o * (kFfnTW * 64)) = f2h(y.x, y.y);
              }
            }
          };
#pragma unroll
          for (int i = 0; i < 8; i += 3) {
            row(std::integral_constant<int, 0>{}, i);
            row(std::integral_constant<int, 1>{}, i + 1);
            if (i + 2 < 8) row(std::integral_constant<int, 2>{}, i + 2);
          }
        }
        fence_proxy_async_smem();  // the gated block is read by the tensor cores
        mbar_arrive(bar(B_GF + g));
        mbar_arrive(bar(B_HE + g));
        mbar_arrive(bar(B_WDE + ws));
      }
      if (!ok) break;
      // ---- output: x += W_out . gate(..) for the tile's 192 pixels, by group 1 (which has
      // the tile's last slice) while group 0 goes on with the next tile's first slice. Warp
      // (q, part) of the group takes channels [part * dim / 2, + dim / 2) of its TMEM lane
      // quarter's pixels in both subtiles (subtile 1 holds 64 pixels: quarters 0 and 1). The
      // residual loads (L2 hits: the producer prefetched the tile's rows) of the first subtile
      // are issued before waiting for the last slice's project_out.
      if (g == 1) {
        const int part = w8 >> 2;
        const int half = a.dim >> 1;  // 64 or 32 channels per thread and pixel
        bool first = true;
        for (int osub = 0; osub < 2; ++osub) {
          if (osub == 1 && q >= 2) break;  // warp-uniform
          const int o = osub * 128 + 32 * q + lane;
          const int Y = ty * kFfnTH + (o >> 4), X = tx * kFfnTW + (o & 15);
          const bool valid = Y < a.h && X < a.w;
          __half* xp = a.x + n * a.x_img + (long long)Y * a.x_row + (long long)X * a.x_pix +
                       part * half;
          uint4 res[8];
#pragma unroll
          for (int k = 0; k < 8; ++k)
            res[k] = (valid && 8 * k < half) ? *reinterpret_cast<const uint4*>(xp + 8 * k)
                                             : make_uint4(0u, 0u, 0u, 0u);
          if (first) {
            if (!mbar_wait_sleep(bar(B_OF), (uint32_t)(it & 1), abort_flag, a.err,
                                 DEV_TIMEOUT_ACC_FULL)) {
              ok = false;
              break;
            }
            tc_fence_after();
            first = false;
          }
#pragma unroll
          for (int cb = 0; cb < 64; cb += 32) {
            if (cb >= half) break;
            float v[32];
            tmem_ld32(trow + 256 + osub * a.dim + part * half + cb, v);
            if (valid) {
#pragma unroll
              for (int g8 = 0; g8 < 4; ++g8) {
                uint4* pp = reinterpret_cast<uint4*>(xp + cb + 8 * g8);
                const uint4 r = res[cb / 8 + g8];
                const uint32_t rr[4] = {r.x, r.y, r.z, r.w};
                uint32_t w4[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const float2 rf = h2f(rr[e]);
                  const float y0 = __fmul_rn(v[8 * g8 + 2 * e], a.scale_out) + rf.x;
                  const float y1 = __fmul_rn(v[8 * g8 + 2 * e + 1], a.scale_out) + rf.y;
                  w4[e] = f2h(y0, y1);
                }
                *pp = make_uint4(w4[0], w4[1], w4[2], w4[3]);
              }
            }
          }
        }
        if (!ok) break;
        tc_fence_before();
        mbar_arrive(bar(B_OE));
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512u);
  }
}

cudaError_t launch_ffn(const CUtensorMap& tmX, const FfnArgs& a, int grid, cudaStream_t stream) {
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(ffn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
    attr_set = true;
  }
  ffn_tc_kernel<<<grid, kFfnThreads, ffn_smem_bytes(a.dim), stream>>>(tmX, a);
  return cudaGetLastError();
}

}  // namespace zjai

// ---- host side ---------------------------------------------------------------------------
#include <algorithm>
#include <vector>

#include "engine.h"

namespace zjai {

bool ffn_fusable(int dim, int hidden) {
  return (dim == 64 || dim == 128) && hidden > 0 && hidden % 64 == 0;
}

// One swizzled row of `len` (64 or 32) halves: 16-byte chunk j of row r at j ^ (r & 7) (128-byte
// rows) or j ^ ((r / 2) & 3) (64-byte rows), the shared-memory image the UMMA descriptors read.
static void put_row(__half* dst, int r, int len, const float* src, float s) {
  const int f = len == 64 ? (r & 7) : ((r >> 1) & 3);
  for (int k = 0; k < len; ++k)
    dst[(size_t)r * len + (((k >> 3) ^ f) << 3) + (k & 7)] = __float2half_rn(src[k] * s);
}

int pack_ffn(Ctx* ctx, FfnLayer* L, const float* w_in, const float* w_dw, const float* w_out,
             int dim, int hidden) {
  (void)ctx;
  if (!ffn_fusable(dim, hidden)) return fail(ZJAI_UNSUPPORTED, "fused FFN: unsupported shape");
  *L = FfnLayer();
  L->dim = dim;
  L->hidden = hidden;
  // the same power-of-two scales as the unfused layers' packing (max |w| in [2^13, 2^14))
  const float si = pow2_weight_scale(w_in, (size_t)2 * hidden * dim);
  const float so = pow2_weight_scale(w_out, (size_t)dim * hidden);
  L->scale_in = 1.f / si;
  L->scale_out = 1.f / so;
  const int ns = hidden / 32, kxn = dim / 64;
  std::vector<__half> wi((size_t)ns * kxn * 64 * 64), wo((size_t)ns * dim * 32);
  for (int c = 0; c < ns; ++c)
    for (int kx = 0; kx < kxn; ++kx) {
      __half* blk = wi.data() + (size_t)(c * kxn + kx) * 64 * 64;
      for (int r = 0; r < 64; ++r) {
        const int oc = r < 32 ? 32 * c + r : hidden + 32 * c + (r - 32);
        put_row(blk, r, 64, w_in + (size_t)oc * dim + 64 * kx, si);
      }
    }
  for (int c = 0; c < ns; ++c)
    for (int r = 0; r < dim; ++r)
      put_row(wo.data() + (size_t)c * dim * 32, r, 32, w_out + (size_t)r * hidden + 32 * c, so);
  // depthwise weights [slice][tap][pair j] {w[32c + 2j], w[32c + 2j + 1], w[hidden + 32c + 2j],
  // w[hidden + 32c + 2j + 1]} at the tap
  std::vector<float> wd((size_t)ns * 9 * 16 * 4);
  for (int c = 0; c < ns; ++c)
    for (int tp = 0; tp < 9; ++tp)
      for (int j = 0; j < 16; ++j) {
        const int e0 = 32 * c + 2 * j, m0 = hidden + e0;
        float* d = wd.data() + ((size_t)(c * 9 + tp) * 16 + j) * 4;
        d[0] = w_dw[(size_t)e0 * 9 + tp];
        d[1] = w_dw[(size_t)(e0 + 1) * 9 + tp];
        d[2] = w_dw[(size_t)m0 * 9 + tp];
        d[3] = w_dw[(size_t)(m0 + 1) * 9 + tp];
      }
  ZJAI_TRY(cuda_check(cudaMalloc(&L->wdw, wd.size() * sizeof(float)), "cudaMalloc FFN weights"));
  ZJAI_TRY(cuda_check(
      cudaMemcpy(L->wdw, wd.data(), wd.size() * sizeof(float), cudaMemcpyHostToDevice),
      "upload FFN weights"));
  ZJAI_TRY(cuda_check(cudaMalloc(&L->win, wi.size() * sizeof(__half)), "cudaMalloc FFN weights"));
  ZJAI_TRY(cuda_check(cudaMalloc(&L->wout, wo.size() * sizeof(__half)), "cudaMalloc FFN weights"));
  ZJAI_TRY(cuda_check(
      cudaMemcpy(L->win, wi.data(), wi.size() * sizeof(__half), cudaMemcpyHostToDevice),
      "upload FFN weights"));
  return cuda_check(
      cudaMemcpy(L->wout, wo.data(), wo.size() * sizeof(__half), cudaMemcpyHostToDevice),
      "upload FFN weights");
}

void free_ffn(FfnLayer* L) {
  if (L->win) cudaFree(L->win);
  if (L->wout) cudaFree(L->wout);
  if (L->wdw) cudaFree(L->wdw);
  L->win = L->wout = nullptr;
  L->wdw = nullptr;
}

int run_ffn(Ctx* ctx, const FfnLayer& L, const TView& ln, const TView& x) {
  if (!L.win || ln.c != L.dim || x.c != L.dim || ln.h != x.h || ln.w != x.w || ln.n != x.n)
    return fail(ZJAI_INVALID_ARGUMENT, "fused FFN: operand shapes");
  if ((x.pix % 8) || (x.row % 8) || (x.img % 8) ||
      (reinterpret_cast<uintptr_t>(x.p) & 15))
    return fail(ZJAI_INVALID_ARGUMENT, "fused FFN: residual not 16-byte aligned");
  if (x.h <= 0 || x.w <= 0 || x.n <= 0) return ZJAI_OK;
  CUtensorMap tm;
  ZJAI_TRY(make_act_map(ctx, &tm, ln, 64, kFfnHW, kFfnHH));
  FfnArgs a;
  a.n_img = x.n;
  a.h = x.h;
  a.w = x.w;
  a.dim = L.dim;
  a.nslice = L.hidden / 32;
  a.tiles_x = (x.w + kFfnTW - 1) / kFfnTW;
  a.tiles_y = (x.h + kFfnTH - 1) / kFfnTH;
  a.num_tiles = a.tiles_x * a.tiles_y * x.n;
  a.win = L.win;
  a.wout = L.wout;
  a.wdw = L.wdw;
  a.scale_in = L.scale_in;
  a.scale_out = L.scale_out;
  a.x = x.p;
  a.x_pix = x.pix;
  a.x_row = x.row;
  a.x_img = x.img;
  a.err = ctx->d_err;
  ZJAI_TRY(cuda_check(cudaGetLastError(), "before FFN launch"));
  const double px = (double)x.n * x.h * x.w;
  const double fl = 2.0 * px * (2.0 * L.hidden * L.dim + (double)L.hidden * L.dim);
  // algorithmic bytes: ln read, x read and written, the three weight sets once
  const double bytes = 2.0 * px * 3.0 * L.dim +
                       2.0 * (3.0 * L.hidden * L.dim) + 4.0 * 2.0 * L.hidden * 9.0;
  cudaError_t e = cudaSuccess;
  ctx->launches++;
  timed_launch(ctx, true, fl, bytes, [&] {
    e = launch_ffn(tm, a, std::min(a.num_tiles, ctx->sms), ctx->stream);
  });
  return cuda_check(e, "FFN launch");
}

}  // namespace zjai
