// Launchers of the attention-block kernels (kernels_attn.cu).
#pragma once
#include "engine.h"

namespace zjai {

void launch_layer_norm(const TView& x, const TView& y, const float* gamma, const float* beta,
                       cudaStream_t s);
// Depthwise 3x3 (weights [c][9] f32), with gate: y has c/2 channels, y[k] = elu(dw[k]) *
// dw[k + c/2]. Persistent kernels over ctx->sms multiprocessors; returns the launch status.
int launch_dw3x3(Ctx* ctx, const TView& x, const TView& y, const float* wt, bool gate,
                 cudaStream_t s);
// scratch: attention_scratch_floats(n, dim, heads, h * w, sms) floats of device memory
void launch_attention(const TView& qkv, const TView& out, int heads, const float* temp,
                      float* scratch, int sms, cudaStream_t s);
// Scratch of the attention of n pictures of npix pixels: the Gram kernel's partial slots
// (summed in a fixed order, so the result is independent of scheduling) and the matrices.
size_t attention_scratch_floats(int n_img, int dim, int heads, int npix, int sms);
// The attention up to its matrices A_n, then A folded into the following 1x1 projection
// W_o (f32 [dim][dim], device): writes n per-picture weight sets in the blocked layout of the
// packed layer L (which holds W_o), scaled by `wscale`, at wout (n * L.npad * L.cin_pad
// halves). Running L with w = wout, w_img = L.npad * L.cin_pad, scale = 1 / wscale on the v
// slice of qkv gives project_out(attention(qkv)).
void launch_attention_fold(const TView& qkv, int heads, const float* temp, const float* wo,
                           float wscale, const ConvLayer& L, __half* wout, float* scratch,
                           int sms, cudaStream_t s);
// Kernel launches launch_attention_fold makes (the Gram, then one fused reduce + softmax +
// fold kernel for heads of 16 or 32 channels, else three).
int attention_fold_launches(int dim, int heads, const ConvLayer& L);
void launch_gather_latent(const float* src, int C, int LH, int LW, const int* origin,
                          const TView& dst, cudaStream_t s);

}  // namespace zjai
