// tcgen05 implicit-GEMM convolution kernel (see conv_tc.cuh for the scheme).
#include <cstdio>
#include <cstring>

#include "conv_tc.cuh"
#include "sample.cuh"
#include "ptx.cuh"

namespace zjai {

namespace {

template <int ACT>
__device__ __forceinline__ float act(float v) {
  if constexpr (ACT == ACT_RELU) return v > 0.f ? v : 0.f;
  if constexpr (ACT == ACT_LEAKY) return v > 0.f ? v : v * 0.01f;
  // sigma(v) = 1 / (1 + e^-v) (math.rs:370-373) with the fast exponential and division: a
  // few ulp of f32, far below the f16 the result is stored in (a denominator beyond 2^126,
  // v < -87, gives 0)
  if constexpr (ACT == ACT_SIGMOID) return __fdividef(1.f, 1.f + __expf(-v));
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
  c.oy0 = ty * a.bh * a.msub;
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

// The activations of the NHWC epilogues. The sigmoid (with its exponential and division) is
// compiled in only where SIG is set (the CAB epilogue, the one NHWC layer that uses it): its
// code in the other instantiations' chunk loop made every chunk slower, sigmoid or not.
template <bool SIG>
__device__ __forceinline__ void act8_fast(float (&x)[8], int a) {
  if (a == ACT_NONE) return;
  if (a == ACT_RELU) {
#pragma unroll
    for (int e = 0; e < 8; ++e) x[e] = x[e] > 0.f ? x[e] : 0.f;
    return;
  }
  if constexpr (SIG) {
    if (a == ACT_SIGMOID) {
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = act<ACT_SIGMOID>(x[e]);
      return;
    }
  }
  if (a == ACT_RELU6) {
#pragma unroll
    for (int e = 0; e < 8; ++e) x[e] = act<ACT_RELU6>(x[e]);
  } else if (a == ACT_LEAKY) {
#pragma unroll
    for (int e = 0; e < 8; ++e) x[e] = act<ACT_LEAKY>(x[e]);
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
                                         const float* btab, float& rmax) {
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
    act8_fast<OP == OP_CAB>(x, a.act1);
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
    act8_fast<false>(x, a.act2);
    if constexpr (OP != OP_NONE) {
#pragma unroll
      for (int e = 0; e < 8; ++e) rmax = fmaxf(rmax, fabsf(x[e]));
    }
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

// NHWC f16 output through the TMA store (R == 1, or a shuffled output whose 16-column chunk
// lies in one phase): packed columns col0 .. col0 + 15 are channels ch0 .. ch0 + 15 of this
// thread's output pixel. The chunk's 16 f16 results go to this lane's 32 bytes of the warp's
// staging slot (`dst`), from which one TMA store writes the warp's 32 pixels; the store clips
// pixels and channels outside the output view, so lanes outside it (or channels at or past cph,
// packing padding) may stage anything but must not read residuals. p1 / p2 / p2o are the
// element offsets of the output pixel in r1 / r2 / out2; residuals are read before the results
// are staged (in-place ops read exactly what this warp's store then overwrites).
// rs1 / rs2: the thread's residual channels ch0 .. ch0 + 15 already in shared memory (the
// prefetched boxes), or null to load them from global memory here.
template <int OP>
__device__ __forceinline__ void epi_staged(const ConvArgs& a, const float (&v)[kChunk],
                                           int col0, int ch0, long long p1, long long p2,
                                           long long p2o, bool valid, const float* btab,
                                           uint4* dst, const uint4* rs1, const uint4* rs2,
                                           float& rmax) {
  constexpr int G = kChunk / 8;
  uint4 r1[G], r2[G];
  if constexpr (OP != OP_NONE) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int c = ch0 + 8 * g;
      r1[g] = r2[g] = make_uint4(0u, 0u, 0u, 0u);
      if (rs1) {
        r1[g] = rs1[g];
        if constexpr (OP == OP_CAB) r2[g] = rs2[g];
      } else if (valid && c < a.cph) {
        r1[g] = __ldg(reinterpret_cast<const uint4*>(a.r1 + p1 + c));
        if constexpr (OP == OP_CAB) r2[g] = __ldg(reinterpret_cast<const uint4*>(a.r2 + p2 + c));
      }
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const int c = ch0 + 8 * g;
    // packed f32 pairs (FFMA2 / FADD2 / FMUL2): per lane the same IEEE operations as the
    // scalar expressions in the comments, in half the instructions
    float x[8];
    const float4 b0 = *reinterpret_cast<const float4*>(btab + col0 + 8 * g);
    const float4 b1 = *reinterpret_cast<const float4*>(btab + col0 + 8 * g + 4);
    {
      // x = v * scale + b (one fused multiply-add)
      const float2 s2 = make_float2(a.scale, a.scale);
      const float2 bb[4] = {make_float2(b0.x, b0.y), make_float2(b0.z, b0.w),
                            make_float2(b1.x, b1.y), make_float2(b1.z, b1.w)};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 r = __ffma2_rn(make_float2(v[8 * g + 2 * i], v[8 * g + 2 * i + 1]), s2, bb[i]);
        x[2 * i] = r.x;
        x[2 * i + 1] = r.y;
      }
    }
    act8_fast<OP == OP_CAB>(x, a.act1);
    if constexpr (OP != OP_NONE) {
      const __half2* h1 = reinterpret_cast<const __half2*>(&r1[g]);
      const __half2* h2 = reinterpret_cast<const __half2*>(&r2[g]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 q1 = __half22float2(h1[i]), xi = make_float2(x[2 * i], x[2 * i + 1]);
        float2 r;
        if constexpr (OP == OP_ADD) {
          r = __fadd2_rn(xi, q1);  // x + q1
        } else if constexpr (OP == OP_GATE) {
          r = __fmul2_rn(q1, __fadd2_rn(make_float2(1.f, 1.f), xi));  // q1 * (1 + x)
        } else {
          r = __ffma2_rn(q1, xi, __half22float2(h2[i]));  // q2 + q1 * x, fused
        }
        x[2 * i] = r.x;
        x[2 * i + 1] = r.y;
      }
    }
    act8_fast<false>(x, a.act2);
    // residual / gate outputs grow along the network: track the largest stored magnitude of
    // the pixels this thread owns (lanes outside the view stage values nobody stores)
    if constexpr (OP != OP_NONE) {
      if (valid && c < a.cph) {
#pragma unroll
        for (int e = 0; e < 8; ++e) rmax = fmaxf(rmax, fabsf(x[e]));
      }
    }
    const uint4 packed = pack_h8(x);
    dst[g] = packed;
    if (a.out2 && valid && c < a.cph) {
      // relu6 of the stored f16 values (clamping commutes with the monotonic rounding)
      uint4 q = packed;
      __half2* h = reinterpret_cast<__half2*>(&q);
      const __half2 z = __float2half2_rn(0.f), six = __float2half2_rn(6.f);
#pragma unroll
      for (int i = 0; i < 4; ++i) h[i] = __hmin2(__hmax2(h[i], z), six);
      *reinterpret_cast<uint4*>(a.out2 + p2o + c) = q;
    }
  }
}

// Planar f32 output (final layers and the layer entry points): one scalar per column.
__device__ __forceinline__ void epi_planar(const ConvArgs& a, const float (&v)[kChunk], int col0,
                                           int img, int oy, int ox, bool valid,
                                           const uint32_t* tab, const float* btab) {
  if (!valid) return;
  int py0 = a.py0, px0 = a.px0, cy0 = a.cy0, cy1 = a.cy1, cx0 = a.cx0, cx1 = a.cx1;
  long long base = a.img_win ? 0 : img * a.p_img;
  if (a.img_win) {
    const int* wv = a.img_win + 7 * img;
    base = wv[6];
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
    // chroma subsampling: keep the samples on the sv x sh grid (power-of-two factors by
    // shifts and masks)
    int SY, SX;
    if (a.lsv >= 0) {
      if ((PY & ((1 << a.lsv) - 1)) | (PX & ((1 << a.lsh) - 1))) continue;
      SY = PY >> a.lsv;
      SX = PX >> a.lsh;
    } else {
      if (PY % a.sv || PX % a.sh) continue;
      SY = PY / a.sv;
      SX = PX / a.sh;
    }
    float x = act_rt(v[j] * a.scale + btab[col0 + j], a.act1);
    if (a.denorm) {
      x = x * 128.f + 127.5f;
      if (a.denorm == 1) x = fminf(fmaxf(x, 0.f), 255.f);  // 2: unclamped (diagnostics)
    }
    const long long ei = base + (long long)SY * a.p_row + SX;
    const bool second = ch == 1 && a.pout2;  // plane 1 has its own pointer
    if (a.qbytes) {
      // fused output stage: the sample quantize_plane_par would make of x
      const unsigned qv = quantize_sample(x, a.qmax);
      char* base = reinterpret_cast<char*>(second ? a.pout2 : a.pout) +
                   (second ? 0 : (long long)ch * a.p_plane * a.qbytes);
      if (a.qbytes == 1)
        reinterpret_cast<uint8_t*>(base)[ei] = (uint8_t)qv;
      else
        reinterpret_cast<uint16_t*>(base)[ei] = (uint16_t)qv;
    } else {
      (second ? a.pout2 : a.pout + ch * a.p_plane)[ei] = x;
    }
  }
}

}  // namespace

// Epilogue output modes: NHWC without a pixel shuffle, NHWC through the shuffle table, planar.
// kModeShuffleStore: shuffled NHWC through TMA stores of one phase per 16-column chunk.
// kModeR1Pre: kModeR1 with the residual prefetch (1x1 convs with a residual op).
constexpr int kModeR1 = 0, kModeShuffle = 1, kModePlanar = 2, kModeShuffleStore = 3,
              kModeR1Pre = 4;

// One CTA of kConvThreads (19 warps) per SM. The launch bound makes ptxas fit the register
// allocation to 19 warps (at most 96 registers a thread: allocations are rounded per warp and
// warps per four).
template <int MODE, int OP>
__global__ void __launch_bounds__(kConvThreads, 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmO,
                   const ConvArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = a.stages;
  const uint32_t sub_bytes = 128u * a.kc * 2u;      // A tile of one subtile
  const uint32_t a_bytes = sub_bytes * a.msub;      // A tiles of a stage
  const int brows = a.grp_pc ? a.grp_pc * a.grp_n : a.bn;  // rows of one weight block
  const uint32_t b_bytes = (uint32_t)brows * a.kc * 2u;
  // stage = A tiles + B block; in halo mode a stage holds only the B block and the A halos
  // have their own a.hslots-slot ring after the stages
  const uint32_t stage_bytes =
      a.halo ? conv_bstage_bytes(a.kc, brows) : conv_stage_bytes(a.kc, brows, a.msub);
  const uint32_t ring_bytes =
      conv_ring_bytes(a.kc, brows, a.msub, S, a.halo ? a.halo_bytes : 0u, a.hslots);
  uint8_t* halo_ring = smem + S * stage_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + ring_bytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* accf = bars + 2 * S;
  uint64_t* acce = bars + 2 * S + 2;
  uint64_t* drain = bars + 2 * S + 4;
  uint64_t* fullA = bars + 2 * S + 5;            // halo ring
  uint64_t* emptyA = bars + 2 * S + 5 + kMaxHaloSlots;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 5 + 2 * kMaxHaloSlots);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint64_t* rbar = bars + 2 * S + 5 + 2 * kMaxHaloSlots + 1;  // 2 per epilogue warp
  uint32_t* tab = reinterpret_cast<uint32_t*>(smem + ring_bytes + kBarrierBytes);
  const int npad = a.n_tiles * a.bn;
  float* btab = reinterpret_cast<float*>(tab + npad);
  // TMA-store staging: two kEpiSlotBytes slots per epilogue warp (128-byte aligned), then
  // the same again per prefetched residual operand
  uint8_t* staging = reinterpret_cast<uint8_t*>(btab + npad);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // limit of the pipeline waits (the drain waits keep kWaitCycles)
  const long long wl = a.wait_cycles > 0 ? a.wait_cycles : kWaitCycles;

  if (threadIdx.x == 0) {
    // the MMA issuers' commits arrive on the empty, accumulator-full and drain barriers
    for (int i = 0; i < S; ++i) {
      mbar_init(smem_u32(&full[i]), 1);
      mbar_init(smem_u32(&empty[i]), (uint32_t)a.msub);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&accf[i]), (uint32_t)a.msub);
      mbar_init(smem_u32(&acce[i]), kEpiThreads);
    }
    mbar_init(smem_u32(drain), (uint32_t)a.msub);
    for (int i = 0; i < a.hslots; ++i) {
      mbar_init(smem_u32(&fullA[i]), 1);
      mbar_init(smem_u32(&emptyA[i]), (uint32_t)a.msub);
    }
    if (a.nres)
      for (int i = 0; i < 2 * (kEpiThreads / 32); ++i) mbar_init(smem_u32(&rbar[i]), 1);
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
    // One thread; everything per K step is adds and compares (a single thread's dependent
    // instruction chain is what bounds the K-step rate, so no divisions here).
    if (lane == 0 && a.halo) {
      // halo mode: per tile and channel chunk cc, one halo box into the halo ring, then the
      // taps' B blocks (block tap * cchunks + cc) into the stage ring
      int stage = 0, hs = 0;
      uint32_t phase = 0, hphase = 0;
      long long issued = 0, hissued = 0;
      const uint32_t s_base = smem_u32(smem), fb_base = smem_u32(full), eb_base = smem_u32(empty);
      const uint32_t h_base = smem_u32(halo_ring);
      const uint32_t hfb = smem_u32(fullA), heb = smem_u32(emptyA);
      const uint32_t hbox = (uint32_t)a.hw * a.hh * a.kc * 2u;  // bytes the halo box delivers
      const size_t kstride = (size_t)a.n_tiles * brows * a.kc;
      for (int t = blockIdx.x; t < a.num_tiles && !*abort_flag; t += gridDim.x) {
        const TileCoord tc = decode_tile(a, t);
        const int nt = tc.n0 / a.bn;
        const __half* wbase = a.wblk + (size_t)tc.img * a.wblk_img + (size_t)nt * brows * a.kc;
        const uint32_t live = a.tmask_on ? a.tmask[nt] : 0xFFFFFFFFu;
        for (int cc = 0; cc < a.cchunks; ++cc) {
          if (!mbar_wait_idle(heb + 8u * hs, hphase ^ 1u, abort_flag, a.err, DEV_TIMEOUT_EMPTY, 64, wl))
            goto halo_done;
          mbar_arrive_expect_tx(hfb + 8u * hs, hbox);
          tma_load_4d(h_base + hs * a.halo_bytes, &tmA, hfb + 8u * hs, cc * a.kc,
                      tc.ox0 - a.pad_l, tc.oy0 - a.pad_t, tc.img);
          ++hissued;
          if (++hs == a.hslots) {
            hs = 0;
            hphase ^= 1u;
          }
          for (int tap = 0; tap < a.taps; ++tap) {
            if (!((live >> tap) & 1u)) continue;
            if (!mbar_wait_idle(eb_base + 8u * stage, phase ^ 1u, abort_flag, a.err,
                                DEV_TIMEOUT_EMPTY, 64, wl))
              goto halo_done;
            const uint32_t fb = fb_base + 8u * stage;
            mbar_arrive_expect_tx(fb, b_bytes);
            bulk_load(s_base + stage * stage_bytes,
                      wbase + (size_t)(tap * a.cchunks + cc) * kstride, b_bytes, fb);
            ++issued;
            if (++stage == S) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
      }
    halo_done:
      for (int s = 0; s < S; ++s) {
        if (issued > s) {
          long long last = ((issued - 1 - s) / S) * S + s;
          mbar_wait_drain(smem_u32(&full[s]), (uint32_t)((last / S) & 1), a.err);
        }
      }
      for (int s = 0; s < a.hslots; ++s) {
        if (hissued > s) {
          long long last = ((hissued - 1 - s) / a.hslots) * a.hslots + s;
          mbar_wait_drain(smem_u32(&fullA[s]), (uint32_t)((last / a.hslots) & 1), a.err);
        }
      }
    } else if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      const uint32_t s_base = smem_u32(smem), fb_base = smem_u32(full), eb_base = smem_u32(empty);
      const uint32_t tx_bytes = a_bytes + b_bytes;
      const size_t kstride = (size_t)a.n_tiles * brows * a.kc;  // halves per K step of weights
      for (int t = blockIdx.x; t < a.num_tiles && !*abort_flag; t += gridDim.x) {
        const TileCoord tc = decode_tile(a, t);
        const int nt = tc.n0 / a.bn;
        const int k0 = a.koff ? a.koff[nt] : 0, k1 = a.koff ? a.koff[nt + 1] : ksteps;
        const __half* wbase = a.wblk + (size_t)tc.img * a.wblk_img + (size_t)nt * brows * a.kc;
        const CUtensorMap* tm5 = a.s2 ? a.tmA_img + tc.img : nullptr;
        int ky = 0, kx = 0, cc = 0, kidx = 0;  // dense order: tap-major, chunk-minor
        for (int i = k0; i < k1; ++i) {
          if (a.klist) {  // kidx | kx << 16 | ky << 21 | cc << 26
            const uint32_t e = __ldg(a.klist + i);
            kidx = (int)(e & 0xFFFFu);
            kx = (int)((e >> 16) & 31u);
            ky = (int)((e >> 21) & 31u);
            cc = (int)(e >> 26);
          }
          if (!mbar_wait_idle(eb_base + 8u * stage, phase ^ 1u, abort_flag, a.err,
                              DEV_TIMEOUT_EMPTY, 64, wl))
            goto producer_done;
          const uint32_t sA = s_base + stage * stage_bytes;
          const uint32_t fb = fb_base + 8u * stage;
          mbar_arrive_expect_tx(fb, tx_bytes);
          if (!a.s2) {
            tma_load_4d(sA, &tmA, fb, cc * a.kc, tc.ox0 + kx - a.pad_l, tc.oy0 + ky - a.pad_t,
                        tc.img);
          } else {
            const int dx = kx - a.pad_l, dy = ky - a.pad_t;
            tma_load_5d(sA, tm5, fb, cc * a.kc, dx & 1, tc.ox0 + (dx >> 1), dy & 1,
                        tc.oy0 + (dy >> 1));
          }
          bulk_load(sA + a_bytes, wbase + (size_t)kidx * kstride, b_bytes, fb);
          ++issued;
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
          if (!a.klist) {
            ++kidx;
            if (++cc == a.cchunks) {
              cc = 0;
              if (++kx == a.kw) {
                kx = 0;
                ++ky;
              }
            }
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
  } else if (warp == 1 || warp == kMma2Warp) {
    // ------------------------------------------------------------------ MMA issuers
    // One thread per M subtile: lane 0 of warp 1 issues subtile 0, lane 0 of the last warp
    // subtile 1 (msub == 2), so the two serial issue chains (barrier tests, descriptor
    // arithmetic, commits) overlap. Both follow the same stage / halo / accumulator sequence,
    // test the same full barriers and commit to the same empty / accumulator barriers
    // (arrival count msub). Descriptors of stage 0 are built once; a stage, tap or K slice
    // moves only the start address field (16-byte units).
    const int j = warp == 1 ? 0 : 1;  // subtile
    const uint32_t idesc = idesc_f16((uint32_t)(a.grp_pc ? a.grp_n : brows));
    const uint32_t d_off = (uint32_t)(j * a.bn);  // the subtile's accumulator columns
    if (lane == 0 && j < a.msub && a.halo) {
      // halo mode: per tile and chunk, wait for the halo, then per tap wait for its B block and
      // issue 4 UMMAs whose A operand starts at halo pixel (ky, kx)
      const uint64_t dB0 = smem_desc(smem_u32(smem), 128u);
      const uint64_t dstage = stage_bytes >> 4;
      const uint32_t fb_base = smem_u32(full), eb_base = smem_u32(empty);
      const uint32_t hfb = smem_u32(fullA), heb = smem_u32(emptyA);
      // A descriptor of halo slot 0's window at tap (0, 0): rows 128 bytes apart, 8-row groups
      // (one tile row) hw * 128 bytes apart; a tap or a slot moves only the start address
      // field (no carry out of its 14 bits below 256 KB), so the per-tap descriptors are
      // additions: +8 per kx, +8 (hw - kw) more at the end of a tap row. Subtile 1 starts bh
      // tile rows down.
      const uint64_t dH0 = ((uint64_t)((smem_u32(halo_ring) >> 4) & 0x3FFFu) | (1ull << 16) |
                            ((uint64_t)((a.hw * 128) >> 4) << 32) | (1ull << 46) | (2ull << 61)) +
                           (uint64_t)j * (uint64_t)((a.bh * a.hw * 128) >> 4);
      const uint64_t dslot = a.halo_bytes >> 4, row_skip = (uint64_t)(a.hw - a.kw) * 8u;
      int stage = 0, hs = 0;
      uint32_t phase = 0, hphase = 0;
      uint64_t db = dB0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int t = blockIdx.x; t < a.num_tiles && !*abort_flag; t += gridDim.x) {
        if (!mbar_wait_idle(smem_u32(&acce[acc]), acc_phase ^ 1u, abort_flag, a.err,
                            DEV_TIMEOUT_ACC_EMPTY, 64, wl))
          break;
        tc_fence_after();
        const uint32_t d0 = tmem_base + (uint32_t)(acc * a.msub * a.bn) + d_off;
        const int nt = t % a.n_tiles;
        const uint32_t live = a.tmask_on ? a.tmask[nt] : 0xFFFFFFFFu;
        bool ok = true;
        for (int cc = 0; cc < a.cchunks && ok; ++cc) {
          if (!mbar_wait(hfb + 8u * hs, hphase, abort_flag, a.err, DEV_TIMEOUT_FULL, wl)) {
            ok = false;
            break;
          }
          // grouped: this chunk's (pseudo-)group owns accumulator columns cc * grp_n ..
          // (grp_n wide) and its first live tap starts them; dense: the tile's first UMMA
          // starts all
          const uint32_t d = d0 + (a.grp_pc ? (uint32_t)(cc * a.grp_n) : 0u);
          bool fresh = a.grp_pc || cc == 0;
          uint64_t da = dH0 + (uint64_t)hs * dslot;
          int kx = 0;
          for (int tap = 0; tap < a.taps; ++tap) {
            if ((live >> tap) & 1u) {
              if (!mbar_wait(fb_base + 8u * stage, phase, abort_flag, a.err, DEV_TIMEOUT_FULL,
                             wl)) {
                ok = false;
                break;
              }
              tc_fence_after();
              umma_f16(d, da, db, idesc, fresh ? 0u : 1u);
              umma_f16(d, da + 2, db + 2, idesc, 1u);
              umma_f16(d, da + 4, db + 4, idesc, 1u);
              umma_f16(d, da + 6, db + 6, idesc, 1u);
              umma_commit(eb_base + 8u * stage);
              fresh = false;
              db += dstage;
              if (++stage == S) {
                stage = 0;
                phase ^= 1u;
                db = dB0;
              }
            }
            da += 8;
            if (++kx == a.kw) {
              kx = 0;
              da += row_skip;
            }
          }
          umma_commit(heb + 8u * hs);  // the halo is free once this chunk's UMMAs complete
          if (++hs == a.hslots) {
            hs = 0;
            hphase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(smem_u32(&accf[acc]));
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      umma_commit(smem_u32(drain));
      mbar_wait_drain(smem_u32(drain), 0, a.err);
    } else if (lane == 0 && j < a.msub) {
      // subtile 1's A tile follows subtile 0's; B follows the A tiles of the stage
      const uint64_t dA0 = smem_desc(smem_u32(smem), (uint32_t)a.kc * 2u) +
                           (uint64_t)j * (sub_bytes >> 4);
      const uint64_t dBoff = (a_bytes >> 4) - (uint64_t)j * (sub_bytes >> 4);
      const uint64_t dstage = stage_bytes >> 4;
      const uint32_t fb_base = smem_u32(full), eb_base = smem_u32(empty);
      const int kk = a.kc >> 4;  // UMMAs per K step: 4, 2 or 1
      int stage = 0;
      uint32_t phase = 0;
      uint64_t da = dA0;  // stage's A descriptor (B at dBoff from it)
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int t = blockIdx.x; t < a.num_tiles && !*abort_flag; t += gridDim.x) {
        if (!mbar_wait_idle(smem_u32(&acce[acc]), acc_phase ^ 1u, abort_flag, a.err,
                            DEV_TIMEOUT_ACC_EMPTY, 64, wl))
          break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * a.msub * a.bn) + d_off;
        const int nt = t % a.n_tiles;
        const int k0 = a.koff ? a.koff[nt] : 0, k1 = a.koff ? a.koff[nt + 1] : ksteps;
        bool ok = true;
        uint32_t accum = 0u;  // the tile's first UMMA overwrites the accumulator
        for (int i = k0; i < k1; ++i) {
          if (!mbar_wait(fb_base + 8u * stage, phase, abort_flag, a.err, DEV_TIMEOUT_FULL, wl)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t db = da + dBoff;
          umma_f16(d, da, db, idesc, accum);
          if (kk >= 2) umma_f16(d, da + 2, db + 2, idesc, 1u);
          if (kk == 4) {
            umma_f16(d, da + 4, db + 4, idesc, 1u);
            umma_f16(d, da + 6, db + 6, idesc, 1u);
          }
          accum = 1u;
          umma_commit(eb_base + 8u * stage);
          da += dstage;
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
            da = dA0;
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
    // Residual prefetch (kModeR1Pre): while it finishes one work item (subtile, chunk) the
    // warp has the residual box(es) of its next one loaded into its two residual slots (r1, and
    // r2 kEpiStagingBytes further), one mbarrier per slot.
    constexpr bool pre = MODE == kModeR1Pre && OP != OP_NONE;
    uint8_t* rslots = staging + kEpiStagingBytes + (warp - 2) * 2 * kEpiSlotBytes;
    const uint32_t rb0 = smem_u32(&rbar[(warp - 2) * 2]);
    uint32_t rissue = 0, ruse = 0;  // residual boxes issued / consumed by this warp
    // issue the residual box(es) of item (subtile sub, chunk c) of the tile at tcn
    auto res_issue = [&](const TileCoord& tcn, int sub, int c) {
      const int col0 = tcn.n0 + c * kChunk;
      const int y = tcn.oy0 + sub * a.bh + (m0 >> a.lbw), x = tcn.ox0 + (m0 & (a.bw - 1));
      const uint32_t sl = rissue & 1u;
      __syncwarp();  // every lane's reads of this slot (two items ago) are done
      if (lane == 0) {
        fence_proxy_async_smem();
        const uint32_t bar = rb0 + 8u * sl;
        const uint32_t dst = smem_u32(rslots + sl * kEpiSlotBytes);
        mbar_arrive_expect_tx(bar, (uint32_t)a.nres * kEpiSlotBytes);
        tma_load_4d(dst, &a.tmR[0], bar, col0, x, y, tcn.img);
        if constexpr (OP == OP_CAB)
          tma_load_4d(dst + kEpiStagingBytes, &a.tmR[1], bar, col0, x, y, tcn.img);
      }
      ++rissue;
    };
    // this warpgroup's items of a tile: wide accumulators (nchunks >= kEpiWarpgroups) take
    // chunks wg, wg + kEpiWarpgroups, .. of every subtile; narrow ones deal the items
    // it = sub * nchunks + c round-robin to the warpgroups
    const bool wide = nchunks >= kEpiWarpgroups;
    const int items = a.msub * nchunks;
    // first item of a tile (false: this warpgroup has none)
    auto first_item = [&](int& sub, int& c) {
      if (wide) {
        sub = 0;
        c = wg;
        return true;
      }
      sub = wg / nchunks;
      c = wg - sub * nchunks;
      return wg < items;
    };
    // item after (sub, c) in the same tile (false: none)
    auto next_item = [&](int& sub, int& c) {
      if (wide) {
        if (c + kEpiWarpgroups < nchunks) {
          c += kEpiWarpgroups;
          return true;
        }
        c = wg;
        return ++sub < a.msub;
      }
      const int it = sub * nchunks + c + kEpiWarpgroups;
      sub = it / nchunks;
      c = it - sub * nchunks;
      return it < items;
    };
    float rmax = 0.f;  // largest |stored value| of a residual / gate epilogue (range check)
    if (pre && (int)blockIdx.x < a.num_tiles) {
      int s0, c0;
      if (first_item(s0, c0)) res_issue(decode_tile(a, blockIdx.x), s0, c0);
    }
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < a.num_tiles; t += gridDim.x) {
      if (!mbar_wait_idle(smem_u32(&accf[acc]), acc_phase, abort_flag, a.err, DEV_TIMEOUT_ACC_FULL,
                          128, wl))
        break;
      tc_fence_after();
      const TileCoord tc = decode_tile(a, t);
      const int tnext = t + (int)gridDim.x;
      // this thread's pixel in subtile `sub` and its residual / copy offsets
      struct Geo {
        int sy0, oy, ox;
        bool valid;
        long long p1, p2, p2o;
      };
      auto geo = [&](int sub) {
        Geo g;
        g.sy0 = tc.oy0 + sub * a.bh;  // first row of the subtile
        g.oy = g.sy0 + (m >> a.lbw);
        g.ox = tc.ox0 + (m & (a.bw - 1));
        g.valid = g.oy < a.oh && g.ox < a.ow;
        g.p1 = g.p2 = g.p2o = 0;
        if constexpr (MODE == kModeR1 || MODE == kModeR1Pre) {
          if constexpr (OP != OP_NONE)
            g.p1 = tc.img * a.r1_img + g.oy * a.r1_row + g.ox * a.r1_pix;
          if constexpr (OP == OP_CAB)
            g.p2 = tc.img * a.r2_img + g.oy * a.r2_row + g.ox * a.r2_pix;
          g.p2o = tc.img * a.o2_img + g.oy * a.o2_row + g.ox * a.o2_pix;
        }
        return g;
      };
      // column chunk c of subtile `sub`; `last`: this thread's last TMEM read of the tile
      auto chunk = [&](const Geo& g, int sub, int c, bool last) {
        const int sy0 = g.sy0, oy = g.oy, ox = g.ox;
        const bool valid = g.valid;
        const long long p1 = g.p1, p2 = g.p2, p2o = g.p2o;
        const uint32_t tcol = (uint32_t)((acc * a.msub + sub) * a.bn);
        const int col0 = tc.n0 + c * kChunk;
        // residuals: start the next item's boxes, then take this item's
        const uint4 *rs1 = nullptr, *rs2 = nullptr;
        if constexpr (pre) {
          int ns = sub, nc = c;
          if (next_item(ns, nc)) {
            res_issue(tc, ns, nc);
          } else if (tnext < a.num_tiles && first_item(ns, nc)) {
            res_issue(decode_tile(a, tnext), ns, nc);
          }
          const uint32_t sl = ruse & 1u;
          mbar_wait(rb0 + 8u * sl, (ruse >> 1) & 1u, abort_flag, a.err, DEV_TIMEOUT_FULL, wl);
          rs1 = reinterpret_cast<const uint4*>(rslots + sl * kEpiSlotBytes + lane * 32);
          rs2 = rs1 + kEpiStagingBytes / 16;
          ++ruse;
        }
        {
          float v[kChunk];
          tmem_ld16(tmem_base + ((uint32_t)(q * 32) << 16) + tcol + (uint32_t)(c * kChunk), v);
          if (last) {
            tc_fence_before();
            mbar_arrive(smem_u32(&acce[acc]));
          }
          if constexpr (MODE == kModeR1 || MODE == kModeR1Pre) {
            // the slot about to be filled was last stored two chunks ago: wait for that read
            if (lane == 0) bulk_wait_read<1>();
            __syncwarp();
            uint8_t* sl = wslots + slot * kEpiSlotBytes;
            epi_staged<OP>(a, v, col0, col0, p1, p2, p2o, valid, btab,
                           reinterpret_cast<uint4*>(sl + lane * 32), rs1, rs2, rmax);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_4d(&tmO, smem_u32(sl), col0, tc.ox0 + (m0 & (a.bw - 1)),
                           sy0 + (m0 >> a.lbw), tc.img);
              bulk_commit();
            }
            slot ^= 1;
          } else if constexpr (MODE == kModeShuffleStore) {
            // the chunk is channels ch0 .. ch0 + 15 of phase p = (dy, dx): output pixel
            // (R oy + dy, R ox + dx); columns of phases >= R^2 are packing padding
            const uint32_t e = tab[col0];
            const int p = (int)(e >> 16), ch0 = (int)(e & 0xFFFFu);
            if (p < a.R * a.R) {
              const int dy = p >> a.lR, dx = p & (a.R - 1);
              const long long Y = (long long)oy * a.R + dy, X = (long long)ox * a.R + dx;
              const long long q1 = tc.img * a.r1_img + Y * a.r1_row + X * a.r1_pix;
              const long long q2 = tc.img * a.r2_img + Y * a.r2_row + X * a.r2_pix;
              const long long q2o = tc.img * a.o2_img + Y * a.o2_row + X * a.o2_pix;
              if (lane == 0) bulk_wait_read<1>();
              __syncwarp();
              uint8_t* sl = wslots + slot * kEpiSlotBytes;
              epi_staged<OP>(a, v, col0, ch0, q1, q2, q2o, valid, btab,
                             reinterpret_cast<uint4*>(sl + lane * 32), rs1, rs2, rmax);
              fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) {
                tma_store_5d(a.tmO_img + tc.img, smem_u32(sl), ch0, dx,
                             tc.ox0 + (m0 & (a.bw - 1)), dy, sy0 + (m0 >> a.lbw));
                bulk_commit();
              }
              slot ^= 1;
            }
          } else if constexpr (MODE == kModePlanar) {
            epi_planar(a, v, col0, tc.img, oy, ox, valid, tab, btab);
          } else {
            epi_nhwc<OP>(a, v, col0, tc.img, oy, ox, valid, tab, btab, rmax);
          }
        }
      };
      if (wide) {
        // warpgroup wg takes the chunks wg, wg + kEpiWarpgroups, .. of every subtile
        for (int sub = 0; sub < a.msub; ++sub) {
          const Geo g = geo(sub);
          for (int c = wg; c < nchunks; c += kEpiWarpgroups)
            chunk(g, sub, c, sub == a.msub - 1 && c + kEpiWarpgroups >= nchunks);
        }
      } else {
        // narrow accumulators: the items (subtile, chunk) = (it / nchunks, it % nchunks) are
        // dealt round-robin to the warpgroups, so the subtiles of a tile drain in parallel
        if (wg >= items) {
          tc_fence_before();
          mbar_arrive(smem_u32(&acce[acc]));
        }
        for (int it = wg; it < items; it += kEpiWarpgroups) {
          const int sub = it / nchunks;
          chunk(geo(sub), sub, it - sub * nchunks, it + kEpiWarpgroups >= items);
        }
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    // an activation beyond the f16 range (it would be stored as inf): flag it for the host
    if constexpr (OP != OP_NONE) {
      if (!(rmax <= 65504.f)) atomicOr(a.err + 1, 1);
    }
    // residual boxes still in flight (a wait gave up) land before shared memory goes away
    for (; ruse < rissue; ++ruse) mbar_wait_drain(rb0 + 8u * (ruse & 1u), (ruse >> 1) & 1u, a.err);
    // every TMA store of this warp complete before the CTA (and its shared memory) ends
    if constexpr (MODE == kModeR1 || MODE == kModeR1Pre || MODE == kModeShuffleStore) {
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

cudaError_t launch_conv(const CUtensorMap& tmA, const CUtensorMap& tmO, const ConvArgs& a,
                        int grid, cudaStream_t stream, char* detail, int detail_len) {
  const uint32_t smem =
      conv_smem_bytes(a.kc, a.grp_pc ? a.grp_pc * a.grp_n : a.bn, a.msub, a.stages,
                      a.n_tiles * a.bn,
                      conv_staged_output(a), a.halo ? a.halo_bytes : 0u, a.hslots, a.nres);
  // one instantiation per (output mode, epilogue op), each with its own register allocation
  using K = void (*)(CUtensorMap, CUtensorMap, ConvArgs);
  static const K kernels[5][4] = {
      {conv_tc_kernel<kModeR1, OP_NONE>, conv_tc_kernel<kModeR1, OP_ADD>,
       conv_tc_kernel<kModeR1, OP_GATE>, conv_tc_kernel<kModeR1, OP_CAB>},
      {conv_tc_kernel<kModeShuffle, OP_NONE>, conv_tc_kernel<kModeShuffle, OP_ADD>,
       conv_tc_kernel<kModeShuffle, OP_GATE>, conv_tc_kernel<kModeShuffle, OP_CAB>},
      {conv_tc_kernel<kModePlanar, OP_NONE>, conv_tc_kernel<kModePlanar, OP_NONE>,
       conv_tc_kernel<kModePlanar, OP_NONE>, conv_tc_kernel<kModePlanar, OP_NONE>},
      {conv_tc_kernel<kModeShuffleStore, OP_NONE>, conv_tc_kernel<kModeShuffleStore, OP_ADD>,
       conv_tc_kernel<kModeShuffleStore, OP_GATE>, conv_tc_kernel<kModeShuffleStore, OP_CAB>},
      {conv_tc_kernel<kModeR1, OP_NONE>, conv_tc_kernel<kModeR1Pre, OP_ADD>,
       conv_tc_kernel<kModeR1Pre, OP_GATE>, conv_tc_kernel<kModeR1Pre, OP_CAB>}};
  static bool attr_set = false;
  if (!attr_set) {
    for (auto& row : kernels)
      for (K k : row)
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
    attr_set = true;
  }
  const int mode = a.planar ? kModePlanar
                   : a.R == 1 ? (a.nres ? kModeR1Pre : kModeR1)
                   : a.tmO_img ? kModeShuffleStore
                               : kModeShuffle;
  kernels[mode][a.op & 3]<<<grid, kConvThreads, smem, stream>>>(tmA, tmO, a);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess && detail) {
    cudaFuncAttributes fa;
    memset(&fa, 0, sizeof fa);
    cudaFuncGetAttributes(&fa, kernels[mode][a.op & 3]);
    snprintf(detail, detail_len,
             "mode %d op %d smem %u stages %d grid %d (kernel: %d registers, %d threads max, "
             "%d dynamic smem max, %zu static smem): %s",
             mode, a.op, smem, a.stages, grid, fa.numRegs, fa.maxThreadsPerBlock,
             fa.maxDynamicSharedSizeBytes, fa.sharedSizeBytes, cudaGetErrorString(e));
  }
  return e;
}

}  // namespace zjai
