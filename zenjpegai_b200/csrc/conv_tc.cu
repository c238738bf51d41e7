// tcgen05 implicit-GEMM convolution kernel (see conv_tc.cuh for the scheme).
#include "conv_tc.cuh"
#include "ptx.cuh"

namespace zjai {

namespace {

__device__ __forceinline__ float apply_act(float v, int act) {
  switch (act) {
    case ACT_RELU: return v > 0.f ? v : 0.f;
    case ACT_LEAKY: return v > 0.f ? v : v * 0.01f;
    case ACT_SIGMOID: return 1.f / (1.f + expf(-v));
    case ACT_RELU6: return fminf(fmaxf(v, 0.f), 6.f);
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

__device__ __forceinline__ void load_h8(const __half* p, float (&v)[8]) {
  uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

__device__ __forceinline__ void store_h8(__half* p, const float (&v)[8]) {
  uint4 u;
  __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}

}  // namespace

__global__ void __launch_bounds__(kConvThreads, 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const ConvArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = a.stages;
  const uint32_t a_bytes = 128u * a.kc * 2u;
  const uint32_t b_bytes = (uint32_t)a.bn * a.kc * 2u;
  const uint32_t stage_bytes = conv_stage_bytes(a.kc, a.bn);
  float* staging = reinterpret_cast<float*>(smem + S * stage_bytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * stage_bytes + kStagingBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* accf = bars + 2 * S;
  uint64_t* acce = bars + 2 * S + 2;
  uint64_t* drain = bars + 2 * S + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(smem_u32(&full[i]), 1);
      mbar_init(smem_u32(&empty[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&accf[i]), 1);
      mbar_init(smem_u32(&acce[i]), 128);
    }
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
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
        for (int ks = 0; ks < ksteps; ++ks) {
          if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1u, abort_flag, a.err,
                         DEV_TIMEOUT_EMPTY))
            goto producer_done;
          const int tap = ks / a.cchunks;
          const int cc = ks - tap * a.cchunks;
          const int ky = tap / a.kw, kx = tap - (tap / a.kw) * a.kw;
          const uint32_t sA = smem_u32(smem + stage * stage_bytes);
          const uint32_t sB = sA + a_bytes;
          const uint32_t fb = smem_u32(&full[stage]);
          mbar_arrive_expect_tx(fb, a_bytes + b_bytes);
          if (!a.s2) {
            tma_load_4d(sA, &tmA, fb, cc * a.kc, tc.ox0 + kx - a.pad_l, tc.oy0 + ky - a.pad_t,
                        tc.img);
          } else {
            const int dx = kx - a.pad_l, dy = ky - a.pad_t;
            tma_load_5d(sA, &tmA, fb, cc * a.kc, dx & 1, tc.ox0 + (dx >> 1), dy & 1,
                        tc.oy0 + (dy >> 1));
          }
          tma_load_2d(sB, &tmB, fb, cc * a.kc, tap * (a.n_tiles * a.bn) + tc.n0);
          ++issued;
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
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
    // ------------------------------------------------------------------ epilogue (4 warps)
    const int q = warp & 3;                 // TMEM lane quarter of this warp
    const int m = q * 32 + lane;            // accumulator row == pixel index in the tile
    const int et = threadIdx.x - 64;        // 0..127
    const int cw = (a.bn % 32) == 0 ? 32 : 16;  // columns per chunk
    const int nchunk4 = cw / 4;             // float4 chunks per staging row
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < a.num_tiles; t += gridDim.x) {
      if (!mbar_wait(smem_u32(&accf[acc]), acc_phase, abort_flag, a.err, DEV_TIMEOUT_ACC_FULL))
        break;
      tc_fence_after();
      const TileCoord tc = decode_tile(a, t);
      const int nchunks = a.bn / cw;
      for (int c = 0; c < nchunks; ++c) {
        const int col0 = tc.n0 + c * cw;
        float v[32];
        const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * a.bn + c * cw);
        if (cw == 32)
          tmem_ld32(taddr, v);
        else
          tmem_ld16(taddr, v);
        if (c == nchunks - 1) {
          tc_fence_before();
          mbar_arrive(smem_u32(&acce[acc]));
        }
        // phase 1: scale, bias, activation -> staging row m (float4 chunks XOR-swizzled)
        float4* srow = reinterpret_cast<float4*>(staging + m * 32);
#pragma unroll
        for (int j4 = 0; j4 < 8; ++j4) {
          if (j4 < nchunk4) {
            float r[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int j = j4 * 4 + e;
              float b = a.bias ? __ldg(a.bias + col0 + j) : 0.f;
              r[e] = apply_act(v[j] * a.scale + b, a.act1);
            }
            srow[j4 ^ (m & (nchunk4 - 1))] = make_float4(r[0], r[1], r[2], r[3]);
          }
        }
        named_bar_sync(1, 128);
        // phase 2: output-space pass
        if (!a.planar) {
          const int groups = cw / 8;
          for (int it = et; it < 128 * groups; it += 128) {
            const int pm = it / groups, g = it - (it / groups) * groups;
            const int oy = tc.oy0 + pm / a.bw, ox = tc.ox0 + pm % a.bw;
            if (oy >= a.oh || ox >= a.ow) continue;
            const int n = col0 + 8 * g;
            const int p = n / a.cph, co = n - (n / a.cph) * a.cph;
            if (p >= a.R * a.R) continue;
            const int Y = oy * a.R + p / a.R, X = ox * a.R + p % a.R;
            if (Y >= a.out_h || X >= a.out_w) continue;
            const float4* rrow = reinterpret_cast<const float4*>(staging + pm * 32);
            const float4 lo = rrow[(2 * g) ^ (pm & (nchunk4 - 1))];
            const float4 hi = rrow[(2 * g + 1) ^ (pm & (nchunk4 - 1))];
            float x[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
            if (a.op != OP_NONE) {
              float r1[8];
              load_h8(a.r1 + tc.img * a.r1_img + Y * a.r1_row + X * a.r1_pix + co, r1);
              if (a.op == OP_ADD) {
#pragma unroll
                for (int e = 0; e < 8; ++e) x[e] = x[e] + r1[e];
              } else if (a.op == OP_GATE) {
#pragma unroll
                for (int e = 0; e < 8; ++e) x[e] = r1[e] * (1.f + x[e]);
              } else {
                float r2[8];
                load_h8(a.r2 + tc.img * a.r2_img + Y * a.r2_row + X * a.r2_pix + co, r2);
#pragma unroll
                for (int e = 0; e < 8; ++e) x[e] = r2[e] + r1[e] * x[e];
              }
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) x[e] = apply_act(x[e], a.act2);
            store_h8(a.out + tc.img * a.out_img + Y * a.out_row + X * a.out_pix + co, x);
            if (a.out2) {
#pragma unroll
              for (int e = 0; e < 8; ++e) x[e] = fminf(fmaxf(x[e], 0.f), 6.f);
              store_h8(a.out2 + tc.img * a.o2_img + Y * a.o2_row + X * a.o2_pix + co, x);
            }
          }
        } else {
          int py0 = a.py0, px0 = a.px0, cy0 = a.cy0, cy1 = a.cy1, cx0 = a.cx0, cx1 = a.cx1;
          if (a.img_win) {
            const int* wv = a.img_win + 6 * tc.img;
            py0 = wv[0];
            px0 = wv[1];
            cy0 = wv[2];
            cy1 = wv[3];
            cx0 = wv[4];
            cx1 = wv[5];
          }
          for (int it = et; it < 128 * cw; it += 128) {
            const int pm = it / cw, j = it - (it / cw) * cw;
            const int oy = tc.oy0 + pm / a.bw, ox = tc.ox0 + pm % a.bw;
            if (oy >= a.oh || ox >= a.ow) continue;
            const int n = col0 + j;
            const int p = n / a.cph, ch = n - (n / a.cph) * a.cph;
            if (p >= a.R * a.R) continue;
            const int Y = oy * a.R + p / a.R, X = ox * a.R + p % a.R;
            if (Y >= a.out_h || X >= a.out_w) continue;
            const int PY = py0 + Y, PX = px0 + X;
            if (PY < cy0 || PY >= cy1 || PX < cx0 || PX >= cx1) continue;
            if (PY % a.sv || PX % a.sh) continue;
            const float4* rrow = reinterpret_cast<const float4*>(staging + pm * 32);
            const float4 f4 = rrow[(j >> 2) ^ (pm & (nchunk4 - 1))];
            float x = (j & 3) == 0 ? f4.x : (j & 3) == 1 ? f4.y : (j & 3) == 2 ? f4.z : f4.w;
            if (a.denorm) x = fminf(fmaxf(x * 128.f + 127.5f, 0.f), 255.f);
            float* dst = (ch == 1 && a.pout2) ? a.pout2 : a.pout + ch * a.p_plane;
            dst[(a.img_win ? 0 : tc.img * a.p_img) + (PY / a.sv) * a.p_row + PX / a.sh] = x;
          }
        }
        named_bar_sync(1, 128);
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, (uint32_t)a.tmem_cols);
  }
}

void launch_conv(const CUtensorMap& tmA, const CUtensorMap& tmB, const ConvArgs& a, int grid,
                 cudaStream_t stream) {
  const uint32_t smem = conv_smem_bytes(a.kc, a.bn, a.stages);
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(conv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
    attr_set = true;
  }
  conv_tc_kernel<<<grid, kConvThreads, smem, stream>>>(tmA, tmB, a);
}

}  // namespace zjai
