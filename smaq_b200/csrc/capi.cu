// C-ABI plumbing: error text, device queries, version.
#include <stdarg.h>
#include <stdio.h>

#include "common.cuh"

namespace smaq {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_status(cudaError_t e, const char* where) {
  if (e == cudaSuccess) return SMAQ_OK;
  return fail(SMAQ_ERR_CUDA, "%s: %s", where, cudaGetErrorString(e));
}

int num_sms() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  return n;
}

}  // namespace smaq

extern "C" int smaq_abi_version(void) { return SMAQ_ABI_VERSION; }
extern "C" size_t smaq_args_size(int which) {
  return which == 0 ? sizeof(smaq_append_args)
       : which == 1 ? sizeof(smaq_decode_args)
       : which == 2 ? sizeof(smaq_scores_args)
       : which == 3 ? sizeof(smaq_attend_args)
                    : 0;
}
extern "C" const char* smaq_last_error(void) { return smaq::g_err; }
