// Placeholder until the tcgen05 rotation kernel lands: the SIMT kernel serves bf16 keys.
#include "tc_rotate.cuh"

namespace smaq {
bool tc_rotate_enabled() { return false; }
int launch_scalar_keys_tc(const smaq_append_args&, cudaStream_t) {
  return fail(SMAQ_ERR_UNSUPPORTED, "tcgen05 rotation not built");
}
}  // namespace smaq
