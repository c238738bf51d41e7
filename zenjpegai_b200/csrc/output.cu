// Output stage (src/decoder/output.rs): quantisation of planes and 4:2:0 -> RGB conversion.
// Every step is the same f32 operation the reference performs, in its order: the `__f*_rn`
// intrinsics keep the compiler from contracting a multiply and an add that the reference
// rounds separately, and `__fmaf_rn` is used exactly where the reference fuses.
#include "api_common.h"
#include "sample.cuh"

namespace zjai {

namespace {

inline int blocks_for(long long n, int t) { return (int)((n + t - 1) / t); }


// quantize_plane_par (output.rs:330-342)
__global__ void quantize_plane_kernel(const float* __restrict__ x, long long n, float mx,
                                      int bytes, void* out) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const unsigned q = quantize_sample(x[i], mx);
  if (bytes == 1)
    static_cast<uint8_t*>(out)[i] = (uint8_t)q;
  else
    static_cast<uint16_t*>(out)[i] = (uint16_t)q;
}

constexpr float kA = -0.75f;
// PyTorch's CPU build contracts these polynomials into FMAs (output.rs:62-80).
__device__ __forceinline__ float cubic1(float x) {
  const float p = __fmaf_rn(kA + 2.0f, x, -(kA + 3.0f));
  return __fmaf_rn(__fmul_rn(p, x), x, 1.0f);
}
__device__ __forceinline__ float cubic2(float x) {
  float p = __fmaf_rn(kA, x, -5.0f * kA);
  p = __fmaf_rn(p, x, 8.0f * kA);
  return __fmaf_rn(p, x, -4.0f * kA);
}
// fma(x3, c3, fma(x2, c2, fma(x0, c0, x1 * c1))) (output.rs:85-91)
__device__ __forceinline__ float dot4(const float (&x)[4], const float (&c)[4]) {
  float acc = __fmul_rn(x[1], c[1]);
  acc = __fmaf_rn(x[0], c[0], acc);
  acc = __fmaf_rn(x[2], c[2], acc);
  return __fmaf_rn(x[3], c[3], acc);
}
// cubic_taps (output.rs:94-113), align_corners = True
__device__ __forceinline__ void cubic_taps(int dst, int in_len, int out_len, int (&idx)[4],
                                           float (&wt)[4]) {
  const float scale = out_len > 1 ? __fdiv_rn((float)(in_len - 1), (float)(out_len - 1)) : 0.f;
  const float real = __fmul_rn(scale, (float)dst);
  const float base = floorf(real);
  const float t = __fsub_rn(real, base);
  const int b = (int)base;
#pragma unroll
  for (int k = 0; k < 4; ++k) idx[k] = min(max(b - 1 + k, 0), in_len - 1);
  const float u = __fsub_rn(1.0f, t);
  wt[0] = cubic2(__fadd_rn(t, 1.0f));
  wt[1] = cubic1(t);
  wt[2] = cubic1(u);
  wt[3] = cubic2(__fadd_rn(u, 1.0f));
}

__device__ __forceinline__ float bicubic_at(const float* __restrict__ src, int h, int w, int oy,
                                            int ox, int out_h, int out_w) {
  int iy[4], ix[4];
  float wy[4], wx[4];
  cubic_taps(oy, h, out_h, iy, wy);
  cubic_taps(ox, w, out_w, ix, wx);
  float rows[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float* r = src + (long long)iy[k] * w;
    const float v[4] = {__ldg(r + ix[0]), __ldg(r + ix[1]), __ldg(r + ix[2]), __ldg(r + ix[3])};
    rows[k] = dot4(v, wx);
  }
  return dot4(rows, wy);
}

// to_source_format_par bicubic (output.rs:161-204) + to_rgb_planes_owned_par BT.709
// (:218-262) + quantize_par (:407-438), one thread per output pixel.
__global__ void yuv_to_rgb_kernel(const float* __restrict__ py, const float* __restrict__ pu,
                                  const float* __restrict__ pv, int h, int w, int ch, int cw,
                                  float kry, float kby, float gu, float gv, float mx, int bytes,
                                  void* out) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)h * w) return;
  const int oy = (int)(i / w), ox = (int)(i % w);
  float U, V;
  if (ch == h && cw == w) {
    U = pu[i];
    V = pv[i];
  } else {
    U = bicubic_at(pu, ch, cw, oy, ox, h, w);
    V = bicubic_at(pv, ch, cw, oy, ox, h, w);
  }
  const float y = convert_range(py[i], 255.f, 1.f);
  const float u = __fsub_rn(convert_range(U, 255.f, 1.f), 0.5f);
  const float v = __fsub_rn(convert_range(V, 255.f, 1.f), 0.5f);
  const float rv = __fadd_rn(y, __fmul_rn(kry, v));
  const float gvv = __fsub_rn(__fsub_rn(y, __fmul_rn(gu, u)), __fmul_rn(gv, v));
  const float bv = __fadd_rn(y, __fmul_rn(kby, u));
  const float r = clampf(convert_range(rv, 1.f, 255.f), 0.f, 255.f);
  const float g = clampf(convert_range(gvv, 1.f, 255.f), 0.f, 255.f);
  const float b = clampf(convert_range(bv, 1.f, 255.f), 0.f, 255.f);
  const unsigned qr = q_sample(convert_range(r, 255.f, mx), mx);
  const unsigned qg = q_sample(convert_range(g, 255.f, mx), mx);
  const unsigned qb = q_sample(convert_range(b, 255.f, mx), mx);
  if (bytes == 1) {
    uint8_t* o = static_cast<uint8_t*>(out) + 3 * i;
    o[0] = (uint8_t)qr;
    o[1] = (uint8_t)qg;
    o[2] = (uint8_t)qb;
  } else {
    uint16_t* o = static_cast<uint16_t*>(out) + 3 * i;
    o[0] = (uint16_t)qr;
    o[1] = (uint16_t)qg;
    o[2] = (uint16_t)qb;
  }
}

}  // namespace

int output_quantize(Ctx* ctx, const float* x, long long n, int bit_depth, void* out,
                    cudaStream_t s) {
  if (bit_depth != 8 && bit_depth != 10)
    return fail(ZJAI_INVALID_ARGUMENT, "output bit depth must be 8 or 10");
  const float mx = (float)((1u << bit_depth) - 1);
  if (n > 0)
    quantize_plane_kernel<<<blocks_for(n, 256), 256, 0, s>>>(x, n, mx, bit_depth == 8 ? 1 : 2, out);
  ctx->launches++;
  return cuda_check(cudaGetLastError(), "quantize");
}

int output_yuv_to_rgb(Ctx* ctx, const float* y, const float* u, const float* v, int h, int w,
                      int ch, int cw, int bit_depth, void* rgb, cudaStream_t s) {
  if (bit_depth != 8 && bit_depth != 10)
    return fail(ZJAI_INVALID_ARGUMENT, "output bit depth must be 8 or 10");
  if (h <= 0 || w <= 0 || ch <= 0 || cw <= 0) return fail(ZJAI_INVALID_ARGUMENT, "resize: empty input");
  const double KR = 0.2126, KG = 0.7152, KB = 0.0722, KBY = 1.8556, KRY = 1.5748;
  const float mx = (float)((1u << bit_depth) - 1);
  yuv_to_rgb_kernel<<<blocks_for((long long)h * w, 256), 256, 0, s>>>(
      y, u, v, h, w, ch, cw, (float)KRY, (float)KBY, (float)(KB * KBY / KG), (float)(KR * KRY / KG),
      mx, bit_depth == 8 ? 1 : 2, rgb);
  ctx->launches++;
  return cuda_check(cudaGetLastError(), "yuv_to_rgb");
}

}  // namespace zjai

using namespace zjai;

extern "C" {

int zjai_quantize_plane(zjai_ctx* ctx, const float* x, int64_t n, int bit_depth, void* out,
                        int mem) {
  ZJAI_TRY(ctx_enter(ctx));
  if (!x || !out || n < 0) return fail(ZJAI_INVALID_ARGUMENT, "quantize: bad arguments");
  ArenaScope scope(ctx);
  const float* dx;
  ZJAI_TRY(stage_in(ctx, x, (size_t)n, mem, &dx));
  const size_t ob = (size_t)n * (bit_depth == 8 ? 1 : 2);
  void* dout = out;
  if (mem == ZJAI_MEM_DEVICE && n) ZJAI_TRY(check_device_buffer(ctx, out, "quantize output"));
  if (mem == ZJAI_MEM_HOST) {
    dout = ctx->arena.alloc(ob + 16);
    if (!dout) return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (quantize)");
  }
  ZJAI_TRY(output_quantize(ctx, dx, n, bit_depth, dout, ctx->stream));
  if (mem == ZJAI_MEM_HOST)
    ZJAI_TRY(cuda_check(cudaMemcpyAsync(out, dout, ob, cudaMemcpyDeviceToHost, ctx->stream), "D2H"));
  return finish_call(ctx, mem);
}

int zjai_yuv_to_rgb(zjai_ctx* ctx, const float* y, const float* u, const float* v, int h, int w,
                    int ch, int cw, int bit_depth, void* rgb, int mem) {
  ZJAI_TRY(ctx_enter(ctx));
  if (!y || !u || !v || !rgb) return fail(ZJAI_INVALID_ARGUMENT, "yuv_to_rgb: bad arguments");
  ArenaScope scope(ctx);
  const float *dy, *du, *dv;
  ZJAI_TRY(stage_in(ctx, y, (size_t)h * w, mem, &dy));
  ZJAI_TRY(stage_in(ctx, u, (size_t)ch * cw, mem, &du));
  ZJAI_TRY(stage_in(ctx, v, (size_t)ch * cw, mem, &dv));
  const size_t ob = (size_t)h * w * 3 * (bit_depth == 8 ? 1 : 2);
  void* dout = rgb;
  if (mem == ZJAI_MEM_DEVICE) ZJAI_TRY(check_device_buffer(ctx, rgb, "RGB output"));
  if (mem == ZJAI_MEM_HOST) {
    dout = ctx->arena.alloc(ob + 16);
    if (!dout) return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (rgb)");
  }
  ZJAI_TRY(output_yuv_to_rgb(ctx, dy, du, dv, h, w, ch, cw, bit_depth, dout, ctx->stream));
  if (mem == ZJAI_MEM_HOST)
    ZJAI_TRY(cuda_check(cudaMemcpyAsync(rgb, dout, ob, cudaMemcpyDeviceToHost, ctx->stream), "D2H"));
  return finish_call(ctx, mem);
}

}  // extern "C"
