// Sample quantisation shared by the output stage and the final layers' fused epilogue
// (src/decoder/output.rs:330-342 `quantize_plane_par`). Every step is the f32 operation the
// reference performs, in its order (`__f*_rn` keeps the compiler from contracting them).
#pragma once
#include <cuda_runtime.h>

namespace zjai {

__device__ __forceinline__ float clampf(float v, float lo, float hi) {
  return v < lo ? lo : (v > hi ? hi : v);
}

// RangesOps.convert_range for ranges starting at zero: ((x - 0) / in_max) * out_max + 0
__device__ __forceinline__ float convert_range(float x, float in_max, float out_max) {
  return __fadd_rn(__fmul_rn(__fdiv_rn(__fsub_rn(x, 0.f), in_max), out_max), 0.f);
}

// f32 -> integer sample, round half to even, clamped to [0, mx]; NaN -> 0 (Rust's `as`).
__device__ __forceinline__ unsigned q_sample(float v, float mx) {
  v = clampf(rintf(v), 0.f, mx);
  return v == v ? (unsigned)v : 0u;
}

// quantize_plane_par of one sample in [0, 255] to 2^depth - 1 = mx
__device__ __forceinline__ unsigned quantize_sample(float x, float mx) {
  return q_sample(convert_range(clampf(x, 0.f, 255.f), 255.f, mx), mx);
}

}  // namespace zjai
