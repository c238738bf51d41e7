// Packed f32 arithmetic of the depthwise 3x3 and the FFN ELU gate, shared by the streaming
// depthwise kernel and the fused FFN kernel so both produce the same bits.
#pragma once
#include <cuda_fp16.h>

namespace zjai {

// Packed f32 pair FMA (sm_100 FFMA2): per lane exactly fmaf(a, b, c).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  return __ffma2_rn(a, b, c);
}

// 2^x by the SFU (flush-to-zero: 2^x below 2^-126 is 0)
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// The FFN gate elu(e) * m (math.rs:376) for a channel pair: elu(e) = e for e > 0, else
// e^e - 1 = 2^(e log2 e) - 1; the product with m is one packed multiply either way.
__device__ __forceinline__ float2 elu_gate2(float2 e, float2 m) {
  const float2 t = __fmul2_rn(e, make_float2(1.44269504088896341f, 1.44269504088896341f));
  const float2 em1 = __fadd2_rn(make_float2(ex2_ftz(t.x), ex2_ftz(t.y)), make_float2(-1.f, -1.f));
  return __fmul2_rn(make_float2(e.x > 0.f ? e.x : em1.x, e.y > 0.f ? e.y : em1.y), m);
}

}  // namespace zjai
