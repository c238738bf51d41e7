// Entry points whose kernels are not wired up yet report ZJAI_UNSUPPORTED.
#include "api_common.h"

using namespace zjai;

extern "C" {

int zjai_net_create(zjai_ctx*, int, int, const zjai_param*, int, zjai_net** out) {
  if (out) *out = nullptr;
  return fail(ZJAI_UNSUPPORTED, "zjai_net_create: not built yet");
}
int zjai_net_destroy(zjai_net*) { return ZJAI_OK; }
int zjai_synth_out_size(int, int, int, int, int*, int*) {
  return fail(ZJAI_UNSUPPORTED, "not built yet");
}
int zjai_synthesis_primary(zjai_net*, const float*, int, int, int, int, float*, int) {
  return fail(ZJAI_UNSUPPORTED, "not built yet");
}
int zjai_synthesis_secondary(zjai_net*, const float*, int, int, const float*, int, int, int, int,
                             float*, int) {
  return fail(ZJAI_UNSUPPORTED, "not built yet");
}
int zjai_analysis_primary(zjai_net*, const float*, int, int, float*, int) {
  return fail(ZJAI_UNSUPPORTED, "not built yet");
}
int zjai_analysis_secondary(zjai_net*, const float*, int, int, float*, int) {
  return fail(ZJAI_UNSUPPORTED, "not built yet");
}
int zjai_synthesis_tiles(int, int, int, int, int, int, zjai_tile*, int, int*) {
  return fail(ZJAI_UNSUPPORTED, "not built yet");
}
int zjai_synthesize(zjai_ctx*, zjai_net*, zjai_net*, const float*, const float*, int, int, int,
                    int, int, int, int, int, int, int, float*, float*, float*, int,
                    const volatile int*) {
  return fail(ZJAI_UNSUPPORTED, "not built yet");
}
int zjai_quantize_plane(zjai_ctx*, const float*, int64_t, int, void*, int) {
  return fail(ZJAI_UNSUPPORTED, "not built yet");
}
int zjai_yuv_to_rgb(zjai_ctx*, const float*, const float*, const float*, int, int, int, int, int,
                    void*, int) {
  return fail(ZJAI_UNSUPPORTED, "not built yet");
}
int zjai_layer_norm(zjai_ctx*, const float*, int, int, int, const float*, const float*, float*,
                    int) {
  return fail(ZJAI_UNSUPPORTED, "not built yet");
}
int zjai_channel_attention(zjai_ctx*, const float*, int, int, int, int, const float*, float*, int) {
  return fail(ZJAI_UNSUPPORTED, "not built yet");
}
int zjai_depthwise3x3(zjai_ctx*, const float*, int, int, int, const float*, float*, int) {
  return fail(ZJAI_UNSUPPORTED, "not built yet");
}

}  // extern "C"
