// Fused feed-forward half of a HOP transformer block on sm_100a (TransformerBlock::forward,
// attention.rs:346-371):
//
//   x += W_out . gate(dw3x3(W_in . ln)),   gate(t) = elu(t[:hidden]) * t[hidden:]
//
// with ln the block's layer-normed input (NHWC f16), W_in [2 hidden][dim], dw3x3 the
// depthwise 3x3 (pad 1, no bias) over the 2 hidden channels and W_out [dim][hidden]. One
// kernel per map: the 2 hidden-channel intermediates never leave the multiprocessor.
//
// Scheme (one CTA per SM, persistent over output tiles of kFfnTH x kFfnTW pixels):
//  - the tile's 3x3 halo of ln, (kFfnTH + 2) x (kFfnTW + 2) = 252 pixels, arrives by TMA
//    (128-byte swizzle, zeros outside the picture = the depthwise conv's zero padding) and is
//    the M extent (two 128-row subtiles) of project_in;
//  - per chunk of 64 gated channels (k .. k + 63 and their multipliers hidden + k ..), one
//    N = 128 UMMA chain per subtile into TMEM (K = dim);
//  - 16 compute warps drain it to an f16 halo image in shared memory (the unfused path's f16
//    intermediate), then run the depthwise 3x3 + ELU gate on CUDA cores, writing the chunk's
//    gated 192 x 64 block in the UMMA operand layout;
//  - project_out accumulates that block times W_out[:, k .. k + 63] into a second TMEM
//    accumulator (N = dim) while the next chunk's project_in runs;
//  - after the last chunk the compute warps add the residual and store x in place.
// Weights stream from L2 by bulk copies into two-slot rings. Every wait is bounded.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cstddef>
#include <cstdint>

namespace zjai {

constexpr int kFfnTW = 16, kFfnTH = 12;  // output tile
constexpr int kFfnHW = kFfnTW + 2, kFfnHH = kFfnTH + 2;
constexpr int kFfnHalo = kFfnHW * kFfnHH;  // 252 halo pixels (<= 256 rows of two subtiles)
constexpr int kFfnComputeWarps = 16;
constexpr int kFfnThreads = 32 * (2 + kFfnComputeWarps);

struct FfnArgs {
  int n_img, h, w;
  int dim;     // 64 or 128 (K of project_in, N of project_out)
  int nchunk;  // hidden / 64
  int tiles_x, tiles_y, num_tiles;
  // W_in blocks [nchunk][dim / 64][128 rows][64 halves]: rows 0..63 are output channels
  // 64 c + r (the ELU operands), rows 64..127 channels hidden + 64 c + r - 64 (their
  // multipliers); W_out blocks [nchunk][dim rows][64 halves] (columns 64 c ..); both f16 of
  // the weights times a power-of-two scale, 128-byte swizzled rows (16-byte chunk j of row r
  // at j ^ (r & 7))
  const __half* win;
  const __half* wout;
  // depthwise weights [nchunk][9 taps][32 pairs] x {elu 2j, 2j + 1, multipliers 2j, 2j + 1}
  // f32 (gated channels 64 c + 2j ..)
  const float* wdw;
  float scale_in, scale_out;  // weight unscales
  __half* x;         // residual in / output, NHWC, dim channels
  long long x_pix, x_row, x_img;
  int* err;
};

// Dynamic shared memory of the kernel for `dim` (1 KB alignment slack included).
size_t ffn_smem_bytes(int dim);

// tmX: ln as {C, W, H, N} with box [64, kFfnHW, kFfnHH, 1], 128-byte swizzle.
cudaError_t launch_ffn(const CUtensorMap& tmX, const FfnArgs& a, int grid, cudaStream_t stream);

}  // namespace zjai
