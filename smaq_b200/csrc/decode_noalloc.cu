// smaq_decode_noalloc: the hybrid decode entry point for callers that must not allocate device
// memory (custom allocators that own all device memory, code running inside a framework's
// memory pool, or hosts whose only device calls go through this C ABI).  It is smaq_decode with
// the scratch workspace taken from a fixed array that lives in this library's device image.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace {

// Scratch for the decode plan and the per-CTA partial slots.  Every GPU that loads the library
// holds these bytes until the process exits.
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB
static __device__ __align__(256) unsigned char g_decode_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};
unsigned long long g_scratch_ctx[kMaxDevices] = {};  // id of the context the address belongs to

// Driver entry points, resolved through the runtime (the library does not link libcuda).
struct CtxFns {
  PFN_cuCtxGetCurrent_v4000 current = nullptr;
  PFN_cuCtxGetId_v12000 id = nullptr;
};
const CtxFns& ctx_fns() {
  static CtxFns f;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 4000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      f.current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
    if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      f.id = reinterpret_cast<PFN_cuCtxGetId_v12000>(p);
  });
  return f;
}

// Device address of g_decode_scratch on the current device.  It is looked up again whenever the
// current context is not the one the cached address came from (a device reset or a re-created
// primary context reloads the module, and the symbol can move).
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return smaq::cuda_status(e, "smaq_decode_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return smaq::fail(SMAQ_ERR_UNSUPPORTED, "smaq_decode_noalloc: device %d", dev);
  const CtxFns& fn = ctx_fns();
  if (!fn.current || !fn.id) return smaq::fail(SMAQ_ERR_CUDA, "smaq_decode_noalloc: driver context queries unavailable");
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (fn.current(&ctx) != CUDA_SUCCESS || !ctx) {
    // no context yet: the symbol lookup below creates the runtime's primary context
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess) return smaq::cuda_status(e, "smaq_decode_noalloc: cudaGetSymbolAddress");
    if (fn.current(&ctx) != CUDA_SUCCESS || !ctx)
      return smaq::fail(SMAQ_ERR_CUDA, "smaq_decode_noalloc: no current context");
  }
  if (fn.id(ctx, &id) != CUDA_SUCCESS) return smaq::fail(SMAQ_ERR_CUDA, "smaq_decode_noalloc: cuCtxGetId");
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[dev] || g_scratch_ctx[dev] != id) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess) return smaq::cuda_status(e, "smaq_decode_noalloc: cudaGetSymbolAddress");
    g_scratch_ptr[dev] = p;
    g_scratch_ctx[dev] = id;
  }
  *out = g_scratch_ptr[dev];
  return SMAQ_OK;
}

}  // namespace

extern "C" size_t smaq_decode_noalloc_max_workspace(void) { return kNoAllocScratchBytes; }

// Scratch address of the current device (used by smaq_decode_status for no-allocation calls).
int smaq_noalloc_scratch(void** out) { return scratch_address(out); }

extern "C" int smaq_decode_noalloc(const smaq_decode_args* args, void* stream) {
  if (!args) return smaq::fail(SMAQ_ERR_INVALID, "smaq_decode_noalloc: null args");
  void* scratch = nullptr;
  const int st = scratch_address(&scratch);
  if (st) return st;
  smaq_decode_args a = *args;
  a.workspace = scratch;
  a.workspace_bytes = kNoAllocScratchBytes;
  // smaq_decode checks the exact need for the grid it picks, before launching anything
  const int r = smaq_decode(&a, stream);
  if (r == SMAQ_ERR_WORKSPACE)
    return smaq::fail(SMAQ_ERR_WORKSPACE,
                      "smaq_decode_noalloc: these shapes need more than the fixed %zu-byte scratch; use "
                      "smaq_decode with a caller-provided workspace",
                      kNoAllocScratchBytes);
  return r;
}
