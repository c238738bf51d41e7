// tcgen05 implicit-GEMM convolution kernel (see conv_tc.cuh for the scheme).
#include "conv_tc.cuh"
#include "ptx.cuh"

namespace zjai {

namespace {

template <int ACT>
__device__ __forceinline__ float act(float v) {
  if constexpr (ACT == ACT_RELU) return v > 0.f ? v : 0.f;
  if constexpr (ACT == ACT_LEAKY) return v > 0.f ? v : v * 0.01f;
  if constexpr (ACT == ACT_SIGMOID) return 1.f / (1.f + expf(-v));
  if constexpr (ACT == ACT_RELU6) return fminf(fmaxf(v, 0.f), 6.f);
  return v;
}

__device__ __forceinline__ float act_rt(float v, int a) {
  switch (a) {
    case ACT_RELU: return act<ACT_RELU>(v);
    case ACT_LEAKY: return act<ACT_LEAKY>(v);
    case ACT_SIGMOID: return act<ACT_SIGMOID>(v);
    case ACT_RELU6: return act<ACT_RELU6>(v);
    default: return v;
  }
}

struct TileCoord {
  int img, oy0, ox0, n0;
};

__device__ __forceinline__ TileCoord decode_tile(const ConvArgs& a, int t) {
  TileCoord c;
  int nt = t % a.n_tiles;
  int mt = t / a.n_tiles;
  int tx = mt % a.tiles_x;
  int rest = mt / a.tiles_x;
  int ty = rest % a.tiles_y;
  c.img = rest / a.tiles_y;
  c.oy0 = ty * a.bh;
  c.ox0 = tx * a.bw;
  c.n0 = nt * a.bn;
  return c;
}

__device__ __forceinline__ void unpack_h8(const uint4& u, float (&v)[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

__device__ __forceinline__ uint4 pack_h8(const float (&v)[8]) {
  uint4 u;
  __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
  return u;
}

// Activation of an 8-vector (one uniform branch per group, not per element).
__device__ __forceinline__ void act8(float (&x)[8], int a) {
  switch (a) {
    case ACT_RELU:
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = act<ACT_RELU>(x[e]);
      break;
    case ACT_LEAKY:
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = act<ACT_LEAKY>(x[e]);
      break;
    case ACT_SIGMOID:
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = act<ACT_SIGMOID>(x[e]);
      break;
    case ACT_RELU6:
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = act<ACT_RELU6>(x[e]);
      break;
    default:
      break;
  }
}

constexpr int kChunk = 16;  // accumulator columns per TMEM load and epilogue step

// One chunk of accumulator columns [col0, col0 + 16) of this thread's pixel, NHWC f16 out.
// Column n lands in output pixel (R*oy + dy, R*ox + dx), channel co, with (phase, co) read from
// the shared table (phase = dy*R + dx). Each 8-column group is one 16-byte store. Residual
// operands are loaded for both groups before any store (in-place ops read exactly the elements
// this thread then writes).
template <int OP>
__device__ __forceinline__ void epi_nhwc(const ConvArgs& a, const float (&v)[kChunk], int col0,
                                         int img, int oy, int ox, bool valid, const uint32_t* tab,
                                         const float* btab) {
  constexpr int G = kChunk / 8;
  int Yg[G], Xg[G], cg[G];
  bool ok[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const uint32_t e = tab[col0 + 8 * g];
    const int p = (int)(e >> 16);
    cg[g] = (int)(e & 0xFFFFu);
    Yg[g] = oy * a.R + (p >> a.lR);
    Xg[g] = ox * a.R + (p & (a.R - 1));
    ok[g] = valid && p < a.R * a.R && Yg[g] < a.out_h && Xg[g] < a.out_w;
  }
  uint4 r1[G], r2[G];
  if constexpr (OP != OP_NONE) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      if (ok[g]) {
        r1[g] = __ldg(reinterpret_cast<const uint4*>(a.r1 + img * a.r1_img + Yg[g] * a.r1_row +
                                                     Xg[g] * a.r1_pix + cg[g]));
        if constexpr (OP == OP_CAB)
          r2[g] = __ldg(reinterpret_cast<const uint4*>(a.r2 + img * a.r2_img + Yg[g] * a.r2_row +
                                                       Xg[g] * a.r2_pix + cg[g]));
      }
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (!ok[g]) continue;
    float x[8];
    const float4 b0 = *reinterpret_cast<const float4*>(btab + col0 + 8 * g);
    const float4 b1 = *reinterpret_cast<const float4*>(btab + col0 + 8 * g + 4);
    x[0] = v[8 * g + 0] * a.scale + b0.x;
    x[1] = v[8 * g + 1] * a.scale + b0.y;
    x[2] = v[8 * g + 2] * a.scale + b0.z;
    x[3] = v[8 * g + 3] * a.scale + b0.w;
    x[4] = v[8 * g + 4] * a.scale + b1.x;
    x[5] = v[8 * g + 5] * a.scale + b1.y;
    x[6] = v[8 * g + 6] * a.scale + b1.z;
    x[7] = v[8 * g + 7] * a.scale + b1.w;
    act8(x, a.act1);
    if constexpr (OP != OP_NONE) {
      float q1[8];
      unpack_h8(r1[g], q1);
      if constexpr (OP == OP_ADD) {
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = x[e] + q1[e];
      } else if constexpr (OP == OP_GATE) {
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = q1[e] * (1.f + x[e]);
      } else {
        float q2[8];
        unpack_h8(r2[g], q2);
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = q2[e] + q1[e] * x[e];
      }
    }
    act8(x, a.act2);
    *reinterpret_cast<uint4*>(a.out + img * a.out_img + Yg[g] * a.out_row + Xg[g] * a.out_pix +
                              cg[g]) = pack_h8(x);
    if (a.out2) {
#pragma unroll
      for (int k = 0; k < 8; ++k) x[k] = fminf(fmaxf(x[k], 0.f), 6.f);
      *reinterpret_cast<uint4*>(a.out2 + img * a.o2_img + Yg[g] * a.o2_row + Xg[g] * a.o2_pix +
                                cg[g]) = pack_h8(x);
    }
  }
}

// NHWC f16 output without a pixel shuffle (R == 1): column n is channel n of this thread's
// pixel. The chunk's 16 f16 results go to this lane's 32 bytes of the warp's staging slot
// (`dst`), from which one TMA store writes the warp's 32 pixels; the store clips pixels and
// channels outside the output view, so lanes outside it (or columns at or past cph, packing
// padding) may stage anything but must not read residuals. The element offsets of the pixel in
// r1 / r2 / out2 (p1, p2, p2o) are computed once per tile; residuals are read before the
// results are staged (in-place ops read exactly what this warp's store then overwrites).
template <int OP>
__device__ __forceinline__ void epi_r1(const ConvArgs& a, const float (&v)[kChunk], int col0,
                                       long long p1, long long p2, long long p2o, bool valid,
                                       const float* btab, uint4* dst) {
  constexpr int G = kChunk / 8;
  uint4 r1[G], r2[G];
  if constexpr (OP != OP_NONE) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int c = col0 + 8 * g;
      r1[g] = r2[g] = make_uint4(0u, 0u, 0u, 0u);
      if (valid && c < a.cph) {
        r1[g] = __ldg(reinterpret_cast<const uint4*>(a.r1 + p1 + c));
        if constexpr (OP == OP_CAB) r2[g] = __ldg(reinterpret_cast<const uint4*>(a.r2 + p2 + c));
      }
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const int c = col0 + 8 * g;
    float x[8];
    const float4 b0 = *reinterpret_cast<const float4*>(btab + c);
    const float4 b1 = *reinterpret_cast<const float4*>(btab + c + 4);
    x[0] = v[8 * g + 0] * a.scale + b0.x;
    x[1] = v[8 * g + 1] * a.scale + b0.y;
    x[2] = v[8 * g + 2] * a.scale + b0.z;
    x[3] = v[8 * g + 3] * a.scale + b0.w;
    x[4] = v[8 * g + 4] * a.scale + b1.x;
    x[5] = v[8 * g + 5] * a.scale + b1.y;
    x[6] = v[8 * g + 6] * a.scale + b1.z;
    x[7] = v[8 * g + 7] * a.scale + b1.w;
    act8(x, a.act1);
    if constexpr (OP != OP_NONE) {
      float q1[8];
      unpack_h8(r1[g], q1);
      if constexpr (OP == OP_ADD) {
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = x[e] + q1[e];
      } else if constexpr (OP == OP_GATE) {
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = q1[e] * (1.f + x[e]);
      } else {
        float q2[8];
        unpack_h8(r2[g], q2);
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = q2[e] + q1[e] * x[e];
      }
    }
    act8(x, a.act2);
    dst[g] = pack_h8(x);
    if (a.out2 && valid && c < a.cph) {
#pragma unroll
      for (int k = 0; k < 8; ++k) x[k] = fminf(fmaxf(x[k], 0.f), 6.f);
      *reinterpret_cast<uint4*>(a.out2 + p2o + c) = pack_h8(x);
    }
  }
}

// Planar f32 output (final layers and the layer entry points): one scalar per column.
__device__ __forceinline__ void epi_planar(const ConvArgs& a, const float (&v)[kChunk], int col0,
                                           int img, int oy, int ox, bool valid,
                                           const uint32_t* tab, const float* btab) {
  if (!valid) return;
  int py0 = a.py0, px0 = a.px0, cy0 = a.cy0, cy1 = a.cy1, cx0 = a.cx0, cx1 = a.cx1;
  if (a.img_win) {
    const int* wv = a.img_win + 6 * img;
    py0 = wv[0];
    px0 = wv[1];
    cy0 = wv[2];
    cy1 = wv[3];
    cx0 = wv[4];
    cx1 = wv[5];
  }
#pragma unroll
  for (int j = 0; j < kChunk; ++j) {
    const uint32_t e = tab[col0 + j];
    const int p = (int)(e >> 16), ch = (int)(e & 0xFFFFu);
    if (p >= a.R * a.R) continue;
    const int Y = oy * a.R + (p >> a.lR), X = ox * a.R + (p & (a.R - 1));
    if (Y >= a.out_h || X >= a.out_w) continue;
    const int PY = py0 + Y, PX = px0 + X;
    if (PY < cy0 || PY >= cy1 || PX < cx0 || PX >= cx1) continue;
    if (PY % a.sv || PX % a.sh) continue;
    float x = act_rt(v[j] * a.scale + btab[col0 + j], a.act1);
    if (a.denorm) x = fminf(fmaxf(x * 128.f + 127.5f, 0.f), 255.f);
    float* dst = (ch == 1 && a.pout2) ? a.pout2 : a.pout + ch * a.p_plane;
    dst[(a.img_win ? 0 : img * a.p_img) + (PY / a.sv) * a.p_row + PX / a.sh] = x;
  }
}

}  // namespace

// Epilogue output modes: NHWC without a pixel shuffle, NHWC through the shuffle table, planar.
constexpr int kModeR1 = 0, kModeShuffle = 1, kModePlanar = 2;

// One CTA of kConvThreads (18 warps) per SM: 18 x 32 x 112 registers fill the register file.
template <int MODE, int OP>
__global__ void __maxnreg__(112)
    conv_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmO,
                   const ConvArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = a.stages;
  const uint32_t a_bytes = 128u * a.kc * 2u;
  const uint32_t b_bytes = (uint32_t)a.bn * a.kc * 2u;
  const uint32_t stage_bytes = conv_stage_bytes(a.kc, a.bn);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * stage_bytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* accf = bars + 2 * S;
  uint64_t* acce = bars + 2 * S + 2;
  uint64_t* drain = bars + 2 * S + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint32_t* tab = reinterpret_cast<uint32_t*>(smem + S * stage_bytes + kBarrierBytes);
  const int npad = a.n_tiles * a.bn;
  float* btab = reinterpret_cast<float*>(tab + npad);
  // TMA-store staging: two kEpiSlotBytes slots per epilogue warp (128-byte aligned)
  uint8_t* staging = reinterpret_cast<uint8_t*>(btab + npad);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(smem_u32(&full[i]), 1);
      mbar_init(smem_u32(&empty[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&accf[i]), 1);
      mbar_init(smem_u32(&acce[i]), kEpiThreads);
    }
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  // column -> (phase, channel) table of the packed column order, and the bias per column
  for (int n = threadIdx.x; n < npad; n += blockDim.x) {
    tab[n] = ((uint32_t)(n / a.cph) << 16) | (uint32_t)(n % a.cph);
    btab[n] = a.bias ? a.bias[n] : 0.f;
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), (uint32_t)a.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int ksteps = a.taps * a.cchunks;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      for (int t = blockIdx.x; t < a.num_tiles && !*abort_flag; t += gridDim.x) {
        const TileCoord tc = decode_tile(a, t);
        int tap = 0, cc = 0;
        for (int ks = 0; ks < ksteps; ++ks) {
          if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1u, abort_flag, a.err,
                         DEV_TIMEOUT_EMPTY))
            goto producer_done;
          const int ky = tap / a.kw, kx = tap - ky * a.kw;
          const uint32_t sA = smem_u32(smem + stage * stage_bytes);
          const uint32_t sB = sA + a_bytes;
          const uint32_t fb = smem_u32(&full[stage]);
          mbar_arrive_expect_tx(fb, a_bytes + b_bytes);
          if (!a.s2) {
            tma_load_4d(sA, &tmA, fb, cc * a.kc, tc.ox0 + kx - a.pad_l, tc.oy0 + ky - a.pad_t,
                        tc.img);
          } else {
            const int dx = kx - a.pad_l, dy = ky - a.pad_t;
            tma_load_5d(sA, a.tmA_img + tc.img, fb, cc * a.kc, dx & 1, tc.ox0 + (dx >> 1), dy & 1,
                        tc.oy0 + (dy >> 1));
          }
          bulk_load(sB,
                    a.wblk + (size_t)tc.img * a.wblk_img +
                        ((size_t)(tap * a.cchunks + cc) * a.n_tiles + tc.n0 / a.bn) *
                                 ((size_t)a.bn * a.kc),
                    b_bytes, fb);
          ++issued;
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
          if (++cc == a.cchunks) {
            cc = 0;
            ++tap;
          }
        }
      }
    producer_done:
      // Drain: every stage's most recent load must have landed before the CTA may exit.
      for (int s = 0; s < S; ++s) {
        if (issued > s) {
          long long last = ((issued - 1 - s) / S) * S + s;  // last load index into stage s
          mbar_wait_drain(smem_u32(&full[s]), (uint32_t)((last / S) & 1), a.err);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16((uint32_t)a.bn);
      const uint32_t row_bytes = (uint32_t)a.kc * 2u;
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int t = blockIdx.x; t < a.num_tiles && !*abort_flag; t += gridDim.x) {
        if (!mbar_wait(smem_u32(&acce[acc]), acc_phase ^ 1u, abort_flag, a.err,
                       DEV_TIMEOUT_ACC_EMPTY))
          break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * a.bn);
        bool ok = true;
        for (int ks = 0; ks < ksteps; ++ks) {
          if (!mbar_wait(smem_u32(&full[stage]), phase, abort_flag, a.err, DEV_TIMEOUT_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sA = smem_u32(smem + stage * stage_bytes);
          const uint32_t sB = sA + a_bytes;
          for (int k = 0; k < a.kc / 16; ++k) {
            const uint64_t ad = smem_desc(sA + k * 32u, row_bytes);
            const uint64_t bd = smem_desc(sB + k * 32u, row_bytes);
            umma_f16(d_tmem, ad, bd, idesc, (ks | k) != 0 ? 1u : 0u);
          }
          umma_commit(smem_u32(&empty[stage]));
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(smem_u32(&accf[acc]));
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // Drain: all issued MMAs must complete before TMEM is released.
      umma_commit(smem_u32(drain));
      mbar_wait_drain(smem_u32(drain), 0, a.err);
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    // kEpiWarpgroups warpgroups; warp w reads TMEM lanes 32*(w%4).. (its accumulator rows =
    // pixels), warpgroup g takes the column chunks c with c % kEpiWarpgroups == g.
    const int q = warp & 3;
    const int wg = (warp - 2) >> 2;
    const int m = q * 32 + lane;  // accumulator row == pixel index in the tile
    const int nchunks = a.bn / kChunk;
    // TMA-store mode: this warp's two staging slots, and the origin of its 32-pixel box
    // [16, bx, 32 / bx] relative to the tile (pixels m0 .. m0 + 31 of the tile, raster order)
    uint8_t* wslots = staging + (warp - 2) * 2 * kEpiSlotBytes;
    int slot = 0;
    const int m0 = q * 32;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < a.num_tiles; t += gridDim.x) {
      if (!mbar_wait(smem_u32(&accf[acc]), acc_phase, abort_flag, a.err, DEV_TIMEOUT_ACC_FULL))
        break;
      tc_fence_after();
      const TileCoord tc = decode_tile(a, t);
      const int oy = tc.oy0 + (m >> a.lbw), ox = tc.ox0 + (m & (a.bw - 1));
      const bool valid = oy < a.oh && ox < a.ow;
      long long p1 = 0, p2 = 0, p2o = 0;
      if constexpr (MODE == kModeR1) {
        if constexpr (OP != OP_NONE) p1 = tc.img * a.r1_img + oy * a.r1_row + ox * a.r1_pix;
        if constexpr (OP == OP_CAB) p2 = tc.img * a.r2_img + oy * a.r2_row + ox * a.r2_pix;
        p2o = tc.img * a.o2_img + oy * a.o2_row + ox * a.o2_pix;
      }
      if (wg >= nchunks) {
        tc_fence_before();
        mbar_arrive(smem_u32(&acce[acc]));
      }
      for (int c = wg; c < nchunks; c += kEpiWarpgroups) {
        float v[kChunk];
        tmem_ld16(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * a.bn + c * kChunk), v);
        if (c + kEpiWarpgroups >= nchunks) {  // this thread's last read of the accumulator
          tc_fence_before();
          mbar_arrive(smem_u32(&acce[acc]));
        }
        const int col0 = tc.n0 + c * kChunk;
        if constexpr (MODE == kModeR1) {
          // the slot about to be filled was last stored two chunks ago: wait for that read
          if (lane == 0) bulk_wait_read<1>();
          __syncwarp();
          uint8_t* sl = wslots + slot * kEpiSlotBytes;
          epi_r1<OP>(a, v, col0, p1, p2, p2o, valid, btab, reinterpret_cast<uint4*>(sl + lane * 32));
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_4d(&tmO, smem_u32(sl), col0, tc.ox0 + (m0 & (a.bw - 1)),
                         tc.oy0 + (m0 >> a.lbw), tc.img);
            bulk_commit();
          }
          slot ^= 1;
        } else if constexpr (MODE == kModePlanar) {
          epi_planar(a, v, col0, tc.img, oy, ox, valid, tab, btab);
        } else {
          epi_nhwc<OP>(a, v, col0, tc.img, oy, ox, valid, tab, btab);
        }
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    // every TMA store of this warp complete before the CTA (and its shared memory) ends
    if constexpr (MODE == kModeR1) {
      if (lane == 0) bulk_wait_all();
    }
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, (uint32_t)a.tmem_cols);
  }
}

void launch_conv(const CUtensorMap& tmA, const CUtensorMap& tmO, const ConvArgs& a, int grid,
                 cudaStream_t stream) {
  const uint32_t smem =
      conv_smem_bytes(a.kc, a.bn, a.stages, a.n_tiles * a.bn, !a.planar && a.R == 1);
  // one instantiation per (output mode, epilogue op), each with its own register allocation
  using K = void (*)(CUtensorMap, CUtensorMap, ConvArgs);
  static const K kernels[3][4] = {
      {conv_tc_kernel<kModeR1, OP_NONE>, conv_tc_kernel<kModeR1, OP_ADD>,
       conv_tc_kernel<kModeR1, OP_GATE>, conv_tc_kernel<kModeR1, OP_CAB>},
      {conv_tc_kernel<kModeShuffle, OP_NONE>, conv_tc_kernel<kModeShuffle, OP_ADD>,
       conv_tc_kernel<kModeShuffle, OP_GATE>, conv_tc_kernel<kModeShuffle, OP_CAB>},
      {conv_tc_kernel<kModePlanar, OP_NONE>, conv_tc_kernel<kModePlanar, OP_NONE>,
       conv_tc_kernel<kModePlanar, OP_NONE>, conv_tc_kernel<kModePlanar, OP_NONE>}};
  static bool attr_set = false;
  if (!attr_set) {
    for (auto& row : kernels)
      for (K k : row)
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
    attr_set = true;
  }
  const int mode = a.planar ? kModePlanar : a.R == 1 ? kModeR1 : kModeShuffle;
  kernels[mode][a.op & 3]<<<grid, kConvThreads, smem, stream>>>(tmA, tmO, a);
}

}  // namespace zjai
