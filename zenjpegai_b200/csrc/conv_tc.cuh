// Implicit-GEMM convolution on sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// GEMM view: M = output pixels (a tile of bh x bw = 128 pixels of one picture), N = packed
// output columns, K = taps x input channels. Activations are NHWC f16; per K step one TMA
// box [kc channels, bw, bh] of the input is loaded at the tap's offset (out-of-range
// coordinates read zeros, which is the convolution's zero padding; a crop is a smaller
// tensor-map extent over the same memory). Weights are packed [tap][N][Cin] f16 and loaded
// as [kc, bn] boxes. One thread per M subtile issues kind::f16 UMMAs into f32 accumulators in
// TMEM (two accumulator sets, so the epilogue of one tile overlaps the main loop of the next).
//
// Epilogue: TMEM -> registers -> scale/bias/activation -> shared staging -> a second pass in
// output order applies the pixel-shuffle remap (column n = phase * cph + channel, phase =
// dy * R + dx) and the residual ops (add, ResAU gate, CAB sigmoid-mul-add), then stores NHWC
// f16 (optionally also relu6 of it) or planar f32 (final layers: denormalize, crop to the
// tile core, chroma subsampling).
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace zjai {

enum Act : int { ACT_NONE = 0, ACT_RELU = 1, ACT_LEAKY = 2, ACT_SIGMOID = 3, ACT_RELU6 = 4 };
enum EpiOp : int { OP_NONE = 0, OP_ADD = 1, OP_GATE = 2, OP_CAB = 3 };

constexpr int kMaxTapMasks = 8;

struct ConvArgs {
  // tile grid
  int tiles_x, tiles_y, n_img, n_tiles, num_tiles;
  int bw, bh;          // pixel subtile, bh * bw == 128 (one UMMA M)
  // M subtiles per tile (1 or 2): a tile is bw x (bh * msub) pixels; subtile s (rows s * bh ..)
  // accumulates into its own TMEM columns and the UMMAs of a K step alternate between the
  // subtiles, so two independent accumulation chains keep the tensor pipe busy (a chain into
  // one accumulator waits for the previous UMMA) and each weight block serves 256 pixels
  int msub;
  // K loop
  int kw, taps, pad_t, pad_l;
  int s2;              // 1: stride-2 conv through the 5-D (parity-split) input view
  const CUtensorMap* tmA_img;  // s2: per-picture tensor maps in device memory (64 B aligned)
  int cchunks, kc;     // channel chunks per tap; chunk width (16, 32 or 64)
  int bn;              // N tile (multiple of 16, <= 256)
  int stages;
  int tmem_cols;
  int oh, ow;          // conv output extent (pixels of the GEMM M space)
  // weights as contiguous K-step blocks [bn][kc] in the shared-memory (swizzled) image, block
  // index (tap * cchunks + cc) * n_tiles + n_tile: one bulk copy per K step
  const __half* wblk;
  long long wblk_img;  // per-picture weight sets: stride in halves (0: one set for all)
  // Sparse K: the K steps whose weight block is not all zero, for N tile nt at
  // klist[koff[nt] .. koff[nt + 1]) (device arrays; null: every K step of every tile), each
  // entry kidx | kx << 16 | ky << 21 | cc << 26 with kidx = (ky * kw + kx) * cchunks + cc.
  // Grouped convolutions (one N tile per group) and stride-2 transposed ones (phases that use
  // a subset of the taps) skip the rest.
  const uint32_t* klist;
  const int* koff;
  // Grouped convolution (grp_pc == 1, halo mode): the groups of a 64-channel chunk cc form one
  // pseudo-group (their weights block-diagonal) owning output columns [cc * grp_n, + grp_n); a
  // K step is grp_n-wide UMMAs into that slice, and the chunk's weight block is [grp_n][64]
  // instead of [bn][64] of the dense-ified layer.
  int grp_n, grp_pc;
  // Halo mode (stride-1 kh x kw conv, kc == 64, tile bw = 8 x bh = 16): per channel chunk one
  // TMA box of the tile plus its halo, [64, hw = bw + kw - 1, hh = bh + kh - 1] in the 128-byte
  // swizzle, serves every tap: tap (ky, kx) is the UMMA A operand starting at halo pixel
  // (ky, kx), rows 128 bytes apart, 8-row groups (one tile row of 8 pixels) hw * 128 bytes
  // apart. The swizzle is a function of the shared-memory address bits, the same for the TMA
  // write and the UMMA read, so a window that starts mid-pattern needs no descriptor base
  // offset. halo_bytes: one halo slot (1 KB multiple); hslots: slots in the halo ring (2 ..
  // kMaxHaloSlots: layers with little MMA work per halo keep more halos in flight).
  int halo, hw, hh, hslots;
  uint32_t halo_bytes;
  // Live taps of a halo-mode layer per N tile (bit tap of tmask[nt]; taps <= 32, n_tiles <=
  // kMaxTapMasks), or tmask_on == 0 when every tap of every tile is live: a stride-2 transposed
  // conv packed with whole phases per N tile uses only some taps of its window per phase, and
  // the dead taps' weight blocks are neither loaded nor multiplied (the halo window still
  // steps over them).
  int tmask_on;
  uint32_t tmask[8];
  // epilogue
  const float* bias;   // [n_tiles * bn] in packed column order, or null
  float scale;         // weight unscale (power of two)
  int act1, op, act2;
  int R, cph;          // pixel-shuffle factor (power of two) and channels per phase
  int lR, lbw;         // log2(R), log2(bw)
  // NHWC f16 output
  __half* out;
  long long out_pix, out_row, out_img;
  int out_h, out_w;    // output extent after the shuffle (crop)
  const __half* r1;
  long long r1_pix, r1_row, r1_img;
  const __half* r2;
  long long r2_pix, r2_row, r2_img;
  __half* out2;        // optional relu6(out)
  long long o2_pix, o2_row, o2_img;
  // shuffled NHWC output through TMA stores: per picture a 5-D map of the output viewed as
  // {C, R (dx), W / R, R (dy), H / R}, box [16, 1, bx, 1, 32 / bx] (device array, or null)
  const CUtensorMap* tmO_img;
  // Residual prefetch of the TMA-store epilogue: nres (0, 1 or 2) residual operands whose box
  // of the next work item each epilogue warp loads into shared memory while it finishes the
  // current one. tmR (device array): the maps of r1 then r2 with the output map's box, one
  // each (unshuffled output) or one per picture each (shuffled output: n_img maps of r1, then
  // n_img of r2).
  const CUtensorMap* tmR;
  int nres;
  // planar f32 output
  int planar, denorm;  // denorm 1: x * 128 + 127.5 clamped to [0, 255]; 2: not clamped
  float* pout;
  float* pout2;        // plane 1 (when not at pout + p_plane)
  long long p_plane, p_row, p_img;
  int py0, px0;        // picture coordinates of output pixel (0, 0)
  int cy0, cy1, cx0, cx1;
  // per-image {py0, px0, cy0, cy1, cx0, cx1, base} (device), or null: picture coordinates of the
  // image's output pixel (0, 0), the kept window, and the sample offset of its picture's planes
  const int* img_win;
  int sv, sh;
  int lsv, lsh;        // log2 of sv / sh when both are powers of two, else -1
  // fused output stage: qbytes 1 (uint8) or 2 (uint16) writes quantized samples
  // (quantize_plane_par to qmax = 2^depth - 1) instead of f32; pout / pout2 are then the
  // integer planes and the strides count samples
  int qbytes;
  float qmax;
  int* err;            // [0] wait status, [1] set when a residual / gate output left the f16 range
  // limit of the kernel's pipeline waits in SM cycles (0: the default of about 2 s); a wait
  // that runs out records DEV_TIMEOUT_* in *err and the CTA drains its copies and MMAs and ends
  long long wait_cycles;
};

// warp 0 TMA, warp 1 MMA issuer 0, then kEpiWarpgroups warpgroups of epilogue (warpgroup g
// takes the accumulator column chunks c with c % kEpiWarpgroups == g), then the warp of MMA
// issuer 1
constexpr int kEpiWarpgroups = 4;
constexpr int kEpiThreads = 128 * kEpiWarpgroups;
constexpr int kMma2Warp = 2 + kEpiThreads / 32;
constexpr int kConvThreads = 32 * (kMma2Warp + 1);
// 2 * stages + 5 + 2 * halo slots mbarriers, the TMEM slot / abort word, 2 residual
// mbarriers per epilogue warp
constexpr int kBarrierBytes = 1024;
constexpr int kMaxStages = 16;

// a stage: the A tiles of msub subtiles (128 rows each) + the B block of bn rows
__host__ __device__ inline uint32_t conv_stage_bytes(int kc, int bn, int msub) {
  uint32_t b = 128u * msub * kc * 2u + (uint32_t)bn * kc * 2u;
  return (b + 1023u) & ~1023u;
}
// Unshuffled NHWC outputs leave through TMA stores: each epilogue warp stages its 32 pixels x
// 16 columns (1 KB of f16) in one of two slots, then one lane stores the box [16, bx, 32/bx].
constexpr uint32_t kEpiSlotBytes = 1024u;
constexpr uint32_t kEpiStagingBytes = 2u * kEpiSlotBytes * (kEpiThreads / 32);

// 1 KB alignment slack + barriers/slots + the column table and the bias (4 + 4 bytes per column)
// + the epilogue staging slots when the output goes out through TMA stores, and as many again
// per prefetched residual operand
__host__ __device__ inline uint32_t conv_fixed_smem(int npad, bool staged, int nres) {
  return 1024u + kBarrierBytes + 8u * (uint32_t)npad +
         (staged ? (1u + (uint32_t)nres) * kEpiStagingBytes : 0u);
}
constexpr int kMaxHaloSlots = 6;
// a stage holding only the B block (halo mode)
__host__ __device__ inline uint32_t conv_bstage_bytes(int kc, int bn) {
  return ((uint32_t)bn * kc * 2u + 1023u) & ~1023u;
}
// The operand rings: `stages` stages of A tile + B block, or (halo_bytes > 0) stages of B
// blocks only plus hslots halo slots.
__host__ __device__ inline uint32_t conv_ring_bytes(int kc, int bn, int msub, int stages,
                                                    uint32_t halo_bytes, int hslots) {
  return halo_bytes ? stages * conv_bstage_bytes(kc, bn) + hslots * halo_bytes
                    : stages * conv_stage_bytes(kc, bn, msub);
}
__host__ __device__ inline uint32_t conv_smem_bytes(int kc, int bn, int msub, int stages,
                                                    int npad, bool staged, uint32_t halo_bytes,
                                                    int hslots, int nres) {
  return conv_ring_bytes(kc, bn, msub, stages, halo_bytes, hslots) +
         conv_fixed_smem(npad, staged, nres);
}

// The output leaves through the TMA-store epilogue (staging slots): unshuffled NHWC, or
// shuffled NHWC with per-picture phase maps.
__host__ __device__ inline bool conv_staged_output(const ConvArgs& a) {
  return !a.planar && (a.R == 1 || a.tmO_img != nullptr);
}

// tmO: the output tensor map (TMA-store epilogue, R == 1 NHWC output), unused otherwise.
// Returns the launch status; on an error `detail` (if given) describes the launch.
cudaError_t launch_conv(const CUtensorMap& tmA, const CUtensorMap& tmO, const ConvArgs& a,
                        int grid, cudaStream_t stream, char* detail, int detail_len);

}  // namespace zjai
