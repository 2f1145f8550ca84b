// tcgen05 (5th-generation tensor core) path for the d x d metric transform of bf16 scalar keys.
#pragma once
#include "common.cuh"

namespace smaq {
// True when the request can take the tensor-core kernel: bf16 keys, head_dim 128, n_heads
// dividing 128, 16-byte aligned input / code rows and 8-element-aligned strides.
bool tc_rotate_eligible(const smaq_append_args& a);
int launch_scalar_keys_tc(const smaq_append_args& a, cudaStream_t s);
}  // namespace smaq
