// Device buffers shared between the processes of a multi-GPU job (CUDA IPC): the final gather
// of a sharded synthesis without a collective. The process that owns the picture exports its
// planes' allocation; every other rank maps it (over NVLink / NVSwitch on one box) and its
// final layers' epilogue stores the 8-bit cores straight into the owner's planes.
#include <map>
#include <mutex>

#include "api_common.h"

using namespace zjai;

namespace {

// cuMemGetAddressRange (driver API, reached like cuTensorMapEncodeTiled): the base and size of
// the allocation holding a device pointer
typedef CUresult (*AddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

std::mutex g_ipc_mu;
std::map<void*, void*> g_ipc_base;  // mapped pointer -> base address of its mapping

int allocation_base(const void* ptr, char** base) {
  static AddressRangeFn fn = nullptr;
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !f)
      return fail(ZJAI_DEVICE, "cuMemGetAddressRange entry point not available");
    fn = reinterpret_cast<AddressRangeFn>(f);
  }
  CUdeviceptr b = 0;
  size_t sz = 0;
  if (fn(&b, &sz, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(ZJAI_INVALID_ARGUMENT, "ipc: not a device allocation of this process");
  *base = reinterpret_cast<char*>(b);
  return ZJAI_OK;
}

}  // namespace

extern "C" {

int zjai_ipc_export(zjai_ctx* ctx, const void* ptr, void* handle, uint64_t* offset) {
  ZJAI_TRY(ctx_enter(ctx));
  if (!ptr || !handle || !offset) return fail(ZJAI_INVALID_ARGUMENT, "ipc export: null argument");
  char* base = nullptr;
  ZJAI_TRY(allocation_base(ptr, &base));
  cudaIpcMemHandle_t h;
  ZJAI_TRY(cuda_check(cudaIpcGetMemHandle(&h, base), "cudaIpcGetMemHandle"));
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  memcpy(handle, &h, sizeof h);
  *offset = (uint64_t)(static_cast<const char*>(ptr) - base);
  return ZJAI_OK;
}

int zjai_ipc_import(zjai_ctx* ctx, const void* handle, uint64_t offset, void** ptr) {
  ZJAI_TRY(ctx_enter(ctx));
  if (!handle || !ptr) return fail(ZJAI_INVALID_ARGUMENT, "ipc import: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof h);
  void* base = nullptr;
  ZJAI_TRY(cuda_check(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess),
                      "cudaIpcOpenMemHandle"));
  void* p = static_cast<char*>(base) + offset;
  std::lock_guard<std::mutex> lock(g_ipc_mu);
  g_ipc_base[p] = base;
  *ptr = p;
  return ZJAI_OK;
}

int zjai_ipc_close(zjai_ctx* ctx, void* ptr) {
  ZJAI_TRY(ctx_enter(ctx));
  void* base = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_ipc_mu);
    auto it = g_ipc_base.find(ptr);
    if (it == g_ipc_base.end()) return fail(ZJAI_INVALID_ARGUMENT, "ipc close: not an imported pointer");
    base = it->second;
    g_ipc_base.erase(it);
  }
  return cuda_check(cudaIpcCloseMemHandle(base), "cudaIpcCloseMemHandle");
}

}  // extern "C"
