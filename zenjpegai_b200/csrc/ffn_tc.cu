// Fused FFN kernel (the scheme is in ffn_tc.cuh).
#include "ffn_tc.cuh"
#include "gate.cuh"
#include "ptx.cuh"

namespace zjai {

namespace {

constexpr uint32_t kXChunkBytes = 256u * 128u;  // one 64-channel slab of the halo, 256 rows
constexpr uint32_t kWinBytes = 128u * 128u;     // one W_in block [128][64]
constexpr uint32_t kGBytes = 256u * 128u;       // gated block, 2 subtiles x 128 rows x 64 ch
constexpr uint32_t kWdBytes = 9u * 32u * 16u;    // depthwise weights of a chunk, f32
// f16 halo image: 128 channels (256 B) per pixel at a 264-byte pitch, so the drain's lanes
// (consecutive pixels, one 8-byte channel-pair slot) and the depthwise lanes (one pixel, 32
// consecutive slots) both hit distinct banks
constexpr uint32_t kHPitch = 264u;
constexpr uint32_t kHBytes = (((uint32_t)kFfnHalo * kHPitch) + 127u) & ~127u;

constexpr uint32_t kBarBytes = 256u;  // mbarriers, TMEM address, abort word

enum FfnBar : int {
  B_XF, B_XE,             // halo slabs full / free
  B_WIF, B_WIE = B_WIF + 2,  // W_in ring (2 slots)
  B_WOF = B_WIE + 2, B_WOE,  // W_out block (1 slot: reloaded while the next chunk's
                             // depthwise runs)
  B_WDF, B_WDE = B_WDF + 2,  // depthwise weights (2 slots)
  B_INF = B_WDE + 2,      // project_in accumulators of a chunk complete
  B_INE,                  // ... drained (compute threads)
  B_HF,                   // f16 halo image written (compute threads)
  B_HE,                   // ... read by every compute thread
  B_GF,                   // gated block written (compute threads)
  B_GE,                   // ... consumed by project_out
  B_OF,                   // project_out accumulators of a tile complete
  B_OE,                   // ... drained (compute threads)
  B_DRAIN,
  B_COUNT
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
  const size_t wo = (size_t)dim * 128u;
  return 1024 + x + 2u * kWinBytes + wo + kGBytes + kHBytes + 2u * kWdBytes + kBarBytes;
}

__global__ void __launch_bounds__(kFfnThreads, 1)
    ffn_tc_kernel(const __grid_constant__ CUtensorMap tmX, const FfnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int kxn = a.dim >> 6;  // 64-channel slabs of ln (K blocks of project_in)
  const uint32_t wob = (uint32_t)a.dim * 128u;  // one W_out block [dim][64]
  uint8_t* sX = smem;
  uint8_t* sWin = sX + kxn * kXChunkBytes;
  uint8_t* sWout = sWin + 2 * kWinBytes;
  uint8_t* sG = sWout + wob;
  uint8_t* sH = sG + kGBytes;
  uint8_t* sWd = sH + kHBytes;  // 2 slots of kWdBytes
  uint64_t* bars = reinterpret_cast<uint64_t*>(sWd + 2 * kWdBytes);  // kBarBytes
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + B_COUNT);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr uint32_t kCT = 32u * kFfnComputeWarps;  // compute threads (per-thread arrivals)
  if (threadIdx.x == 0) {
    mbar_init(bar(B_XF), 1);
    mbar_init(bar(B_XE), 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(B_WIF + i), 1);
      mbar_init(bar(B_WIE + i), 1);
      mbar_init(bar(B_WDF + i), 1);
      mbar_init(bar(B_WDE + i), kCT);
    }
    mbar_init(bar(B_WOF), 1);
    mbar_init(bar(B_WOE), 1);
    mbar_init(bar(B_INF), 1);
    mbar_init(bar(B_INE), kCT);
    mbar_init(bar(B_HF), kCT);
    mbar_init(bar(B_HE), kCT);
    mbar_init(bar(B_GF), kCT);
    mbar_init(bar(B_GE), 1);
    mbar_init(bar(B_OF), 1);
    mbar_init(bar(B_OE), kCT);
    mbar_init(bar(B_DRAIN), 1);
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
  const int nchunk = a.nchunk;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      long long xi = 0, wi = 0, wo = 0, wd = 0;  // loads issued per barrier set
      const uint32_t xbox = (uint32_t)kFfnHalo * 128u;
      for (int t = blockIdx.x; t < a.num_tiles && !*abort_flag; t += gridDim.x) {
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
        bool ok = true;
        for (int c = 0; c < nchunk && ok; ++c) {
          for (int kx = 0; kx < kxn; ++kx) {
            const int s = (int)(wi & 1);
            if (!mbar_wait_idle(bar(B_WIE + s), (uint32_t)((wi >> 1) & 1) ^ 1u, abort_flag, a.err,
                                DEV_TIMEOUT_EMPTY, 64)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(bar(B_WIF + s), kWinBytes);
            bulk_load(smem_u32(sWin) + s * kWinBytes, a.win + (size_t)(c * kxn + kx) * 8192,
                      kWinBytes, bar(B_WIF + s));
            ++wi;
          }
          if (!ok) break;
          const int s = (int)(wd & 1);
          if (!mbar_wait_idle(bar(B_WDE + s), (uint32_t)((wd >> 1) & 1) ^ 1u, abort_flag, a.err,
                              DEV_TIMEOUT_EMPTY, 64)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(bar(B_WDF + s), kWdBytes);
          bulk_load(smem_u32(sWd) + s * kWdBytes, a.wdw + (size_t)c * (kWdBytes / 4), kWdBytes,
                    bar(B_WDF + s));
          ++wd;
          if (!mbar_wait_idle(bar(B_WOE), (uint32_t)(wo & 1) ^ 1u, abort_flag, a.err,
                              DEV_TIMEOUT_EMPTY, 64)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(bar(B_WOF), wob);
          bulk_load(smem_u32(sWout), a.wout + (size_t)c * a.dim * 64, wob, bar(B_WOF));
          ++wo;
        }
        if (!ok) break;
      }
      // every copy issued lands before the CTA's shared memory goes away
      if (xi > 0) mbar_wait_drain(bar(B_XF), (uint32_t)((xi - 1) & 1), a.err);
      for (int s = 0; s < 2; ++s) {
        if (wi > s) {
          const long long last = ((wi - 1 - s) / 2) * 2 + s;
          mbar_wait_drain(bar(B_WIF + s), (uint32_t)((last >> 1) & 1), a.err);
        }
        if (wd > s) {
          const long long last = ((wd - 1 - s) / 2) * 2 + s;
          mbar_wait_drain(bar(B_WDF + s), (uint32_t)((last >> 1) & 1), a.err);
        }
      }
      if (wo > 0) mbar_wait_drain(bar(B_WOF), (uint32_t)((wo - 1) & 1), a.err);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    // Per tile: in(0), then for c = 1 .. nchunk: in(c) (c < nchunk) and out(c - 1). in(c) is
    // 2 subtiles x dim / 16 UMMAs (M 128, N 128) into TMEM columns [0, 256); out(c) 2 x 4
    // UMMAs (N = dim) into columns [256, 256 + 2 dim).
    if (lane == 0) {
      const uint32_t id_in = idesc_f16(128u), id_out = idesc_f16((uint32_t)a.dim);
      const uint64_t dX = smem_desc(smem_u32(sX), 128u);
      const uint64_t dWi = smem_desc(smem_u32(sWin), 128u);
      const uint64_t dWo = smem_desc(smem_u32(sWout), 128u);
      const uint64_t dG = smem_desc(smem_u32(sG), 128u);
      long long wi = 0, wo = 0;
      bool ok = true;
      int it = 0;
      for (int t = blockIdx.x; t < a.num_tiles && ok && !*abort_flag; t += gridDim.x, ++it) {
        if (!mbar_wait(bar(B_XF), (uint32_t)(it & 1), abort_flag, a.err, DEV_TIMEOUT_FULL)) break;
        tc_fence_after();
        for (int c = 0; c <= nchunk && ok; ++c) {
          const long long g = (long long)it * nchunk + c;  // global chunk index
          if (c < nchunk) {
            if (!mbar_wait_sleep(bar(B_INE), (uint32_t)(g & 1) ^ 1u, abort_flag, a.err,
                                 DEV_TIMEOUT_ACC_EMPTY)) {
              ok = false;
              break;
            }
            tc_fence_after();
            for (int kx = 0; kx < kxn; ++kx) {
              const int s = (int)(wi & 1);
              if (!mbar_wait(bar(B_WIF + s), (uint32_t)((wi >> 1) & 1), abort_flag, a.err,
                             DEV_TIMEOUT_FULL)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint64_t db = dWi + (uint64_t)((s * kWinBytes) >> 4);
#pragma unroll
              for (int sub = 0; sub < 2; ++sub) {
                const uint64_t da = dX + (uint64_t)((kx * kXChunkBytes + sub * 16384u) >> 4);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                  umma_f16(tmem + sub * 128, da + 2 * kk, db + 2 * kk, id_in,
                           (kx | kk) ? 1u : 0u);
              }
              umma_commit(bar(B_WIE + s));
              ++wi;
            }
            if (!ok) break;
            umma_commit(bar(B_INF));
            if (c == nchunk - 1) umma_commit(bar(B_XE));  // the halo slabs are free
          }
          if (c > 0) {
            if (!mbar_wait_sleep(bar(B_GF), (uint32_t)((g - 1) & 1), abort_flag, a.err,
                                 DEV_TIMEOUT_FULL) ||
                !mbar_wait(bar(B_WOF), (uint32_t)(wo & 1), abort_flag, a.err,
                           DEV_TIMEOUT_FULL) ||
                (c == 1 && !mbar_wait_sleep(bar(B_OE), (uint32_t)(it & 1) ^ 1u, abort_flag, a.err,
                                            DEV_TIMEOUT_ACC_EMPTY))) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t db = dWo;
#pragma unroll
            for (int sub = 0; sub < 2; ++sub) {
              const uint64_t da = dG + (uint64_t)((sub * 16384u) >> 4);
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                umma_f16(tmem + 256 + sub * a.dim, da + 2 * kk, db + 2 * kk, id_out,
                         (c > 1 || kk) ? 1u : 0u);
            }
            umma_commit(bar(B_WOE));
            umma_commit(bar(B_GE));
            ++wo;
            if (c == nchunk) umma_commit(bar(B_OF));
          }
        }
      }
      umma_commit(bar(B_DRAIN));
      mbar_wait_drain(bar(B_DRAIN), 0, a.err);
    }
  } else {
    // ---------------------------------------------------------------- compute warps
    const int cw = warp - 2;
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    // drain role: subtile `dsub`, channel pairs [16 dh, 16 dh + 16) of the chunk
    const int dsub = (cw >> 2) >> 1, dh = (cw >> 2) & 1;
    const int p = dsub * 128 + 32 * q + lane;  // halo pixel of this thread's TMEM row
    const uint32_t trow = tmem + ((uint32_t)(32 * q) << 16);
    // depthwise role: output columns 2 cp, 2 cp + 1, rows 6 rh .. 6 rh + 5, channel pair j
    const int cp = cw & 7, rh = cw >> 3, j = lane;
    bool ok = true;
    int it = 0;
    for (int t = blockIdx.x; t < a.num_tiles && ok; t += gridDim.x, ++it) {
      const int tx = t % a.tiles_x, rest = t / a.tiles_x;
      const int ty = rest % a.tiles_y, n = rest / a.tiles_y;
      for (int c = 0; c < nchunk; ++c) {
        const long long g = (long long)it * nchunk + c;
        // ---- drain project_in: f16 halo image, pixel p at p * kHPitch, channel pair k in
        // the 8-byte slot k: {elu operands 2k, 2k + 1, multipliers 2k, 2k + 1}
        if (!mbar_wait_sleep(bar(B_INF), (uint32_t)(g & 1), abort_flag, a.err,
                             DEV_TIMEOUT_ACC_FULL)) {
          ok = false;
          break;
        }
        tc_fence_after();
        {
          // f16 of acc * scale + 0 (the unfused layer's epilogue with its zero bias), 16
          // channel pairs in two halves of 8
          uint32_t hv[2][8][2];
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            float ve[16], vm[16];
            tmem_ld16x2(trow + dsub * 128 + 32 * dh + 16 * hh,
                        trow + dsub * 128 + 64 + 32 * dh + 16 * hh, ve, vm);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              hv[hh][i][0] = f2h(ve[2 * i] * a.scale_in + 0.f, ve[2 * i + 1] * a.scale_in + 0.f);
              hv[hh][i][1] = f2h(vm[2 * i] * a.scale_in + 0.f, vm[2 * i + 1] * a.scale_in + 0.f);
            }
          }
          tc_fence_before();
          mbar_arrive(bar(B_INE));
          // the accumulators are in registers; the halo image is free once every thread has
          // finished the previous chunk's depthwise
          if (!mbar_wait_sleep(bar(B_HE), (uint32_t)(g & 1) ^ 1u, abort_flag, a.err,
                               DEV_TIMEOUT_ACC_FULL)) {
            ok = false;
            break;
          }
          if (p < kFfnHalo) {
            uint2* hp = reinterpret_cast<uint2*>(sH + p * kHPitch) + 16 * dh;
#pragma unroll
            for (int hh = 0; hh < 2; ++hh)
#pragma unroll
              for (int i = 0; i < 8; ++i) hp[8 * hh + i] = make_uint2(hv[hh][i][0], hv[hh][i][1]);
          }
        }
        mbar_arrive(bar(B_HF));
        if (!mbar_wait_sleep(bar(B_HF), (uint32_t)(g & 1), abort_flag, a.err, DEV_TIMEOUT_ACC_FULL) ||
            !mbar_wait_sleep(bar(B_WDF + (int)(g & 1)), (uint32_t)((g >> 1) & 1), abort_flag, a.err,
                             DEV_TIMEOUT_FULL) ||
            !mbar_wait_sleep(bar(B_GE), (uint32_t)(g & 1) ^ 1u, abort_flag, a.err,
                       DEV_TIMEOUT_ACC_FULL)) {
          ok = false;
          break;
        }
        // depthwise weights of the thread's channels {elu 2j, 2j + 1, multipliers 2j, 2j + 1}
        // per tap ([tap][pair] in the chunk's slot)
        float4 wr[9];
        {
          const float4* ws = reinterpret_cast<const float4*>(sWd + (g & 1) * kWdBytes) + j;
#pragma unroll
          for (int tp = 0; tp < 9; ++tp) wr[tp] = ws[tp * 32];
        }
        // ---- depthwise 3x3 + gate over halo rows 6 rh .. 6 rh + 7 (rolling 3-row
        // accumulators; per output the taps in (ky, kx) order, the first one a product)
        {
          // gated block row op = (6 rh + o) * 16 + 2 cp + col: 128 bytes per row, the channel
          // pair's 4 bytes in 16-byte chunk (j / 4) ^ (op & 7), and op & 7 = (2 cp + col) & 7
          uint8_t* gcol[2];
#pragma unroll
          for (int col = 0; col < 2; ++col)
            gcol[col] = sG + (6 * rh * kFfnTW + 2 * cp + col) * 128 +
                        (((j >> 2) ^ ((2 * cp + col) & 7)) << 4) + ((j & 3) << 2);
          float2 acc[3][2][2];
          auto row = [&](auto JJ, int i) {
            constexpr int J = decltype(JJ)::value;
            const int p0 = (6 * rh + i) * kFfnHW + 2 * cp;
            // halo column jx is tap kx = jx of output column 0 and kx = jx - 1 of column 1:
            // per accumulator the taps of a row still come in kx order
#pragma unroll
            for (int jx = 0; jx < 4; ++jx) {
              const int pp = p0 + jx;
              const uint2 u = *reinterpret_cast<const uint2*>(sH + pp * kHPitch + 8 * j);
              const float2 v[2] = {h2f(u.x), h2f(u.y)};
#pragma unroll
              for (int ky = 0; ky < 3; ++ky)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
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
                *reinterpret_cast<uint32_t*>(gcol[col] + o * (kFfnTW * 128)) = f2h(y.x, y.y);
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
        mbar_arrive(bar(B_GF));
        mbar_arrive(bar(B_HE));
        mbar_arrive(bar(B_WDE + (int)(g & 1)));
      }
      if (!ok) break;
      // ---- output: x += W_out . gate(..) for the tile's 192 pixels
      if (!mbar_wait_sleep(bar(B_OF), (uint32_t)(it & 1), abort_flag, a.err, DEV_TIMEOUT_ACC_FULL)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (!(dsub == 1 && q >= 2)) {  // subtile 1 holds 64 pixels
        const int o = dsub * 128 + 32 * q + lane;
        const int Y = ty * kFfnTH + (o >> 4), X = tx * kFfnTW + (o & 15);
        const bool valid = Y < a.h && X < a.w;
        const int half = a.dim >> 1;
        __half* xp = a.x + n * a.x_img + (long long)Y * a.x_row + (long long)X * a.x_pix +
                     dh * half;
        for (int cb = 0; cb < half; cb += 32) {
          float v[32];
          tmem_ld32(trow + 256 + dsub * a.dim + dh * half + cb, v);
          if (valid) {
#pragma unroll
            for (int g8 = 0; g8 < 4; ++g8) {
              uint4* pp = reinterpret_cast<uint4*>(xp + cb + 8 * g8);
              const uint4 r = *pp;
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
      tc_fence_before();
      mbar_arrive(bar(B_OE));
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

// One 128-byte-swizzled row of 64 halves: 16-byte chunk j of row r at j ^ (r & 7).
static void put_row(__half* dst, int r, const float* src, int stride, float s) {
  for (int k = 0; k < 64; ++k)
    dst[(size_t)r * 64 + (((k >> 3) ^ (r & 7)) << 3) + (k & 7)] =
        __float2half_rn(src[(size_t)k * stride] * s);
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
  const int nchunk = hidden / 64, kxn = dim / 64;
  std::vector<__half> wi((size_t)nchunk * kxn * 128 * 64), wo((size_t)nchunk * dim * 64);
  for (int c = 0; c < nchunk; ++c)
    for (int kx = 0; kx < kxn; ++kx) {
      __half* blk = wi.data() + (size_t)(c * kxn + kx) * 128 * 64;
      for (int r = 0; r < 128; ++r) {
        const int oc = r < 64 ? 64 * c + r : hidden + 64 * c + (r - 64);
        put_row(blk, r, w_in + (size_t)oc * dim + 64 * kx, 1, si);
      }
    }
  for (int c = 0; c < nchunk; ++c)
    for (int r = 0; r < dim; ++r)
      put_row(wo.data() + (size_t)c * dim * 64, r, w_out + (size_t)r * hidden + 64 * c, 1, so);
  // depthwise weights [chunk][tap][pair j] {w[64c + 2j], w[64c + 2j + 1], w[hidden + 64c + 2j],
  // w[hidden + 64c + 2j + 1]} at the tap
  std::vector<float> wd((size_t)nchunk * 9 * 32 * 4);
  for (int c = 0; c < nchunk; ++c)
    for (int tp = 0; tp < 9; ++tp)
      for (int j = 0; j < 32; ++j) {
        const int e0 = 64 * c + 2 * j, m0 = hidden + e0;
        float* d = wd.data() + ((size_t)(c * 9 + tp) * 32 + j) * 4;
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
  a.nchunk = L.hidden / 64;
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
  cudaError_t e = cudaSuccess;
  ctx->launches++;
  timed_launch(ctx, true, fl, 0.0, [&] {
    e = launch_ffn(tm, a, std::min(a.num_tiles, ctx->sms), ctx->stream);
  });
  return cuda_check(e, "FFN launch");
}

}  // namespace zjai
