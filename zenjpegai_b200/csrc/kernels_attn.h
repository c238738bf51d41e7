// Launchers of the attention-block kernels (kernels_attn.cu).
#pragma once
#include "engine.h"

namespace zjai {

void launch_layer_norm(const TView& x, const TView& y, const float* gamma, const float* beta,
                       cudaStream_t s);
// sms: multiprocessor count of the device (the kernel is persistent, two CTAs per SM)
void launch_dw3x3(const TView& x, const TView& y, const float* wt, bool gate, int sms,
                  cudaStream_t s);
// scratch: attention_scratch_floats(n, dim, heads) floats of device memory
void launch_attention(const TView& qkv, const TView& out, int heads, const float* temp,
                      float* scratch, int sms, cudaStream_t s);
size_t attention_scratch_floats(int n_img, int dim, int heads);
void launch_gather_latent(const float* src, int C, int LH, int LW, const int* origin,
                          const TView& dst, cudaStream_t s);

}  // namespace zjai
