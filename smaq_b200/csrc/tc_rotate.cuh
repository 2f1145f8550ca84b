// tcgen05 (5th-generation tensor core) path for the d x d metric transform of bf16 keys.
#pragma once
#include "common.cuh"

namespace smaq {
bool tc_rotate_enabled();
int launch_scalar_keys_tc(const smaq_append_args& a, cudaStream_t s);
}  // namespace smaq
