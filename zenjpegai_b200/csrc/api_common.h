// Shared helpers of the C-ABI translation units.
#pragma once
#include <vector>

#include "engine.h"

struct zjai_ctx : zjai::Ctx {};

namespace zjai {

const char* last_error_cstr();
int ctx_enter(zjai_ctx* ctx);
int ctx_check_status(Ctx* ctx);
int finish_call(Ctx* ctx, int mem);
// ZJAI_INVALID_ARGUMENT unless p is memory the context's GPU can address (its device memory,
// managed memory or mapped pinned host memory): caller buffers passed as ZJAI_MEM_DEVICE are
// checked before any kernel touches them.
int check_device_buffer(Ctx* ctx, const void* p, const char* what);
int stage_in(Ctx* ctx, const float* p, size_t n, int mem, const float** out);
int stage_out_alloc(Ctx* ctx, float* p, size_t n, int mem, float** dev);
int stage_out_finish(Ctx* ctx, float* host, const float* dev, size_t n, int mem);
int planar_to_tensor(Ctx* ctx, const float* d, int c, int h, int w, TView* out);
int fetch_host(const float* p, size_t n, int mem, std::vector<float>* buf, const float** out);

// Releases arena allocations made inside a call when the call returns.
struct ArenaScope {
  Ctx* ctx;
  size_t mark;
  explicit ArenaScope(Ctx* c) : ctx(c), mark(c->arena.mark()) {}
  ~ArenaScope() { ctx->arena.release(mark); }
};

struct LayerGuard {
  ConvLayer* L;
  explicit LayerGuard(ConvLayer* l) : L(l) {}
  ~LayerGuard() {
    cudaDeviceSynchronize();
    free_conv(L);
  }
};

}  // namespace zjai
