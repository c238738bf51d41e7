// Channel attention that allocates nothing (zjai_channel_attention_static).
//
// Some callers cannot allocate device memory at call time: code running under an external
// allocator or a memory budget that forbids new allocations, and embedders that only hand in
// pre-allocated buffers. This entry
// point works on the caller's device buffers alone: the per-call scratch of the transposed
// attention (the c x c Gram per head, the squared norms, the softmax rows) lives in one
// file-scope device array of fixed size, and the kernels read the planar f32 tensors in place
// (no layout copies). Host code resolves the array's device address once per device with
// cudaGetSymbolAddress; the array's name is not a device address in host code.
//
// Limits: dim = c3 / 3 <= 256 and per-head channels c = dim / heads <= 64. All calls on a GPU
// share the array and it keeps the previous call's contents; every call writes each scratch
// entry before reading it (nothing is accumulated across calls), but calls whose work overlaps
// on the GPU (different streams or contexts) race on it. The Gram is reduced in a fixed order
// (no atomics), so a call gives the same bits every time.
#include <mutex>

#include "api_common.h"

namespace zjai {

namespace {

constexpr int kStaticMaxDim = 256;
constexpr int kStaticMaxC = 64;
// gram: dim * c, squared norms: 2 * dim, softmax rows: dim * c
constexpr int kStaticScratchFloats = 2 * kStaticMaxDim * kStaticMaxC + 2 * kStaticMaxDim;

// held by every GPU that loads the library, until the process exits (33280 floats = 130 KiB)
static __device__ __align__(256) float g_attention_scratch[kStaticScratchFloats];

constexpr int kMaxDevices = 64;
float* g_scratch_ptr[kMaxDevices] = {nullptr};
std::mutex g_scratch_mu;

// Device address of the scratch array on the current device (resolved once per device).
int scratch_address(int device, float** out) {
  if (device < 0 || device >= kMaxDevices) return fail(ZJAI_UNSUPPORTED, "device index too large");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[device]) {
    void* p = nullptr;
    ZJAI_TRY(cuda_check(cudaGetSymbolAddress(&p, g_attention_scratch), "cudaGetSymbolAddress"));
    g_scratch_ptr[device] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[device];
  return ZJAI_OK;
}

// ZJAI_OK when `p` is device (or managed) memory usable on `device`, ZJAI_INVALID_ARGUMENT
// for host memory or another GPU's memory.
int device_buffer(int device, const void* p, const char* what) {
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();  // clear the error the query recorded
    return fail(ZJAI_INVALID_ARGUMENT,
                std::string("zjai_channel_attention_static: ") + what + " is not a device pointer");
  }
  if (at.type == cudaMemoryTypeManaged) return ZJAI_OK;
  if (at.type != cudaMemoryTypeDevice || at.device != device)
    return fail(ZJAI_INVALID_ARGUMENT, std::string("zjai_channel_attention_static: ") + what +
                                           " must be device memory of the context's GPU");
  return ZJAI_OK;
}

constexpr int kPix = 64;   // pixels per shared-memory chunk of the Gram kernel
constexpr int kGramRows = 16;  // Gram rows (query channels) per block

// gram[h][i][j] = sum_p q[h*c+i][p] * k[h*c+j][p] and the squared norms of the q and k rows,
// in a fixed order: block (row group, head) owns kGramRows rows i of the head's c x c Gram and
// walks every pixel of the picture in 64-pixel chunks; each thread keeps its (up to four)
// entries in registers and adds the chunks' partial sums in pixel order, so every call gives
// the same bits. Row group 0 also writes the head's k-row norms, every group its q-row norms.
__global__ void __launch_bounds__(256) static_gram_kernel(const float* __restrict__ qkv, int dim,
                                                          int c, long long npix, float* gram,
                                                          float* sq) {
  __shared__ float qs[kGramRows][kPix + 1];
  __shared__ float ks[kStaticMaxC][kPix + 1];
  const int hd = blockIdx.y, i0 = blockIdx.x * kGramRows;
  const int rows = min(kGramRows, c - i0);
  const float* q = qkv + ((long long)hd * c + i0) * npix;
  const float* k = qkv + ((long long)dim + (long long)hd * c) * npix;
  const int entries = rows * c;  // <= 16 * 64 = 1024 = 4 per thread
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  float sacc = 0.f;  // thread t < rows + c: squared norm of q row t (t < rows) or k row t - rows
  for (long long p0 = 0; p0 < npix; p0 += kPix) {
    __syncthreads();
    for (int t = threadIdx.x; t < (rows + c) * kPix; t += blockDim.x) {
      const int r = t / kPix, pp = t - r * kPix;
      const long long p = p0 + pp;
      float v = 0.f;
      if (p < npix) v = r < rows ? q[(long long)r * npix + p] : k[(long long)(r - rows) * npix + p];
      if (r < rows)
        qs[r][pp] = v;
      else
        ks[r - rows][pp] = v;
    }
    __syncthreads();
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int id = threadIdx.x + e * 256;
      if (id < entries) {
        const int i = id / c, j = id - (id / c) * c;
        float s = 0.f;
        for (int pp = 0; pp < kPix; ++pp) s = fmaf(qs[i][pp], ks[j][pp], s);
        acc[e] += s;
      }
    }
    if (threadIdx.x < rows + c) {
      const int r = threadIdx.x;
      const float* row = r < rows ? qs[r] : ks[r - rows];
      float s = 0.f;
      for (int pp = 0; pp < kPix; ++pp) s = fmaf(row[pp], row[pp], s);
      sacc += s;
    }
  }
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int id = threadIdx.x + e * 256;
    if (id < entries) gram[((long long)hd * c + i0) * c + id] = acc[e];
  }
  if (threadIdx.x < rows) sq[hd * c + i0 + threadIdx.x] = sacc;
  else if (blockIdx.x == 0 && threadIdx.x < rows + c)
    sq[dim + hd * c + (threadIdx.x - rows)] = sacc;
}

// Row softmax of the normalised Gram times the head's temperature (math.rs:549-570).
__global__ void static_softmax_kernel(const float* gram, const float* sq,
                                      const float* __restrict__ temp, float* attn, int dim, int c) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= dim) return;
  const int hd = row / c;
  const float nq = fmaxf(sqrtf(sq[row]), 1e-12f);
  const float* g = gram + (long long)row * c;
  float vals[kStaticMaxC];
  float mx = -INFINITY;
  for (int j = 0; j < c; ++j) {
    const float nk = fmaxf(sqrtf(sq[dim + hd * c + j]), 1e-12f);
    vals[j] = g[j] / (nq * nk) * temp[hd];
    mx = fmaxf(mx, vals[j]);
  }
  float sum = 0.f;
  for (int j = 0; j < c; ++j) {
    vals[j] = expf(vals[j] - mx);
    sum += vals[j];
  }
  for (int j = 0; j < c; ++j) attn[(long long)row * c + j] = vals[j] / sum;
}

// out[h*c+i][p] = sum_j attn[h][i][j] * v[h*c+j][p]; block (256 pixels, head).
__global__ void __launch_bounds__(256) static_apply_kernel(const float* __restrict__ qkv,
                                                           const float* attn, float* __restrict__ out,
                                                           int dim, int c, long long npix) {
  __shared__ float a_s[kStaticMaxC * kStaticMaxC];
  const int hd = blockIdx.y;
  for (int t = threadIdx.x; t < c * c; t += blockDim.x) a_s[t] = attn[(long long)hd * c * c + t];
  __syncthreads();
  const long long p = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= npix) return;
  const float* v = qkv + (2LL * dim + (long long)hd * c) * npix + p;
  float vj[kStaticMaxC];
  for (int j = 0; j < c; ++j) vj[j] = v[(long long)j * npix];
  for (int i = 0; i < c; ++i) {
    float s = 0.f;
    for (int j = 0; j < c; ++j) s = fmaf(a_s[i * c + j], vj[j], s);
    out[((long long)hd * c + i) * npix + p] = s;
  }
}

}  // namespace

}  // namespace zjai

using namespace zjai;

extern "C" int zjai_channel_attention_static(zjai_ctx* ctx, const float* qkv, int c3, int h,
                                             int w, int heads, const float* temperature,
                                             float* out) {
  ZJAI_TRY(ctx_enter(ctx));
  if (!qkv || !temperature || !out || heads <= 0 || c3 <= 0 || c3 % (3 * heads) || h <= 0 ||
      w <= 0)
    return fail(ZJAI_INVALID_ARGUMENT, "attention: channel / head counts");
  const int dim = c3 / 3, c = dim / heads;
  if (dim > kStaticMaxDim || c > kStaticMaxC)
    return fail(ZJAI_LIMIT_EXCEEDED,
                "zjai_channel_attention_static: dim " + std::to_string(dim) + " / head size " +
                    std::to_string(c) + " exceed the static scratch (dim <= 256, head <= 64)");
  // the kernels dereference these pointers: host memory (pageable or pinned) is refused here
  ZJAI_TRY(device_buffer(ctx->device, qkv, "qkv"));
  ZJAI_TRY(device_buffer(ctx->device, temperature, "temperature"));
  ZJAI_TRY(device_buffer(ctx->device, out, "out"));
  float* scratch = nullptr;
  ZJAI_TRY(scratch_address(ctx->device, &scratch));
  float* gram = scratch;
  float* sq = gram + (size_t)dim * c;
  float* attn = sq + 2 * (size_t)dim;
  const long long npix = (long long)h * w;
  cudaStream_t s = ctx->stream;
  dim3 g1((unsigned)((c + kGramRows - 1) / kGramRows), heads);
  static_gram_kernel<<<g1, 256, 0, s>>>(qkv, dim, c, npix, gram, sq);
  static_softmax_kernel<<<(dim + 127) / 128, 128, 0, s>>>(gram, sq, temperature, attn, dim, c);
  dim3 g3((unsigned)((npix + 255) / 256), heads);
  static_apply_kernel<<<g3, 256, 0, s>>>(qkv, attn, out, dim, c, npix);
  ctx->launches += 3;
  return cuda_check(cudaGetLastError(), "attention launch");
}
