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
//  - the hidden channels go in slices of 32 gated channels (k .. k + 31 and their multipliers
//    hidden + k ..): per slice one N = 64 UMMA chain per subtile into TMEM (K = dim), issued by
//    the project_in warp;
//  - two groups of 8 compute warps take alternate slices: a group drains its slice's
//    accumulator to its own f16 halo image in shared memory (the unfused path's f16
//    intermediate), then runs the depthwise 3x3 + ELU gate on CUDA cores, writing the slice's
//    gated 192 x 32 block in the UMMA operand layout, while the other group drains or
//    computes the neighbouring slice (accumulators, halo images and gated blocks are double
//    buffered, one per group);
//  - the project_out warp accumulates each gated block times W_out[:, k .. k + 31] into a
//    second TMEM accumulator (N = dim), in slice order;
//  - after the last slice, group 1 (which holds it) adds the residual (its rows prefetched
//    into L2 by the producer a tile earlier) and stores x in place, while group 0 starts the
//    next tile.
// Weights stream from L2 by bulk copies into small rings. Every wait is bounded.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cstddef>
#include <cstdint>

namespace zjai {

constexpr int kFfnTW = 16, kFfnTH = 12;  // output tile
constexpr int kFfnHW = kFfnTW + 2, kFfnHH = kFfnTH + 2;
constexpr int kFfnHalo = kFfnHW * kFfnHH;  // 252 halo pixels (<= 256 rows of two subtiles)
// warp 0 TMA producer, warp 1 project_in issuer, warps 2 .. 17 two compute groups of 8,
// warp 18 project_out issuer
constexpr int kFfnGroupWarps = 8;
constexpr int kFfnOutWarp = 2 + 2 * kFfnGroupWarps;
constexpr int kFfnThreads = 32 * (kFfnOutWarp + 1);

struct FfnArgs {
  int n_img, h, w;
  int dim;     // 64 or 128 (K of project_in, N of project_out)
  int nslice;  // hidden / 32 (even)
  int tiles_x, tiles_y, num_tiles;
  // W_in blocks [nslice][dim / 64][64 rows][64 halves]: rows 0..31 are output channels
  // 32 c + r (the ELU operands), rows 32..63 channels hidden + 32 c + r - 32 (their
  // multipliers), 128-byte swizzled rows (16-byte chunk j of row r at j ^ (r & 7)); W_out
  // blocks [nslice][dim rows][32 halves] (columns 32 c ..), 64-byte swizzled rows (chunk j
  // of row r at j ^ ((r / 2) & 3)); both f16 of the weights times a power-of-two scale
  const __half* win;
  const __half* wout;
  // depthwise weights [nslice][9 taps][16 pairs] x {elu 2j, 2j + 1, multipliers 2j, 2j + 1}
  // f32 (gated channels 32 c + 2j ..)
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
