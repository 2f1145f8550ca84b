// smaq_decode_noalloc: the hybrid decode entry point for callers that must not allocate device
// memory (custom allocators that own all device memory, code running inside a framework's
// memory pool, or hosts whose only device calls go through this C ABI).  It is smaq_decode with
// the scratch workspace taken from a fixed array that lives in this library's device image.
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

// Device address of g_decode_scratch on the current device, looked up once per device.
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return smaq::cuda_status(e, "smaq_decode_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return smaq::fail(SMAQ_ERR_UNSUPPORTED, "smaq_decode_noalloc: device %d", dev);
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess) return smaq::cuda_status(e, "smaq_decode_noalloc: cudaGetSymbolAddress");
    g_scratch_ptr[dev] = p;
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
  const size_t need = smaq_decode_workspace_size(args->batch, args->n_q_heads, args->n_kv_heads,
                                                 args->head_dim, args->num_ctas);
  if (need == 0) return smaq::fail(SMAQ_ERR_INVALID, "smaq_decode_noalloc: bad head counts");
  if (need > kNoAllocScratchBytes)
    return smaq::fail(SMAQ_ERR_WORKSPACE,
                      "smaq_decode_noalloc: these shapes need %zu bytes of scratch, more than the fixed "
                      "%zu-byte array; use smaq_decode with a caller-provided workspace",
                      need, kNoAllocScratchBytes);
  void* scratch = nullptr;
  const int st = scratch_address(&scratch);
  if (st) return st;
  smaq_decode_args a = *args;
  a.workspace = scratch;
  a.workspace_bytes = kNoAllocScratchBytes;
  return smaq_decode(&a, stream);
}
