// Shared device helpers for the smaq_b200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/smaq_b200.h"

namespace smaq {

// ---------------------------------------------------------------- error text
void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);
int cuda_status(cudaError_t e, const char* where);
int num_sms();

// ---------------------------------------------------------------- dtype tags
struct F32 {
  using T = float;
  static constexpr int code = SMAQ_F32;
};
struct BF16 {
  using T = __nv_bfloat16;
  static constexpr int code = SMAQ_BF16;
};
struct F16 {
  using T = __half;
  static constexpr int code = SMAQ_F16;
};

__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f(__half x) { return __half2float(x); }

// Round an fp32 value to the storage type (round-to-nearest-even) and back.
// This is how torch evaluates every elementwise op on a bf16/fp16 tensor:
// fp32 arithmetic, then one rounding of the result.
template <class DT>
__device__ __forceinline__ float rnd(float x);
template <>
__device__ __forceinline__ float rnd<F32>(float x) { return x; }
template <>
__device__ __forceinline__ float rnd<BF16>(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
template <>
__device__ __forceinline__ float rnd<F16>(float x) { return __half2float(__float2half_rn(x)); }

template <class DT>
__device__ __forceinline__ typename DT::T from_f(float x);
template <>
__device__ __forceinline__ float from_f<F32>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<BF16>(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ __half from_f<F16>(float x) { return __float2half_rn(x); }

__device__ __forceinline__ float load_elem(const void* p, int dtype, int64_t i) {
  if (dtype == SMAQ_F32) return static_cast<const float*>(p)[i];
  if (dtype == SMAQ_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(static_cast<const __half*>(p)[i]);
}

__device__ __forceinline__ float round_dtype(float x, int dtype) {
  if (dtype == SMAQ_BF16) return __bfloat162float(__float2bfloat16_rn(x));
  if (dtype == SMAQ_F16) return __half2float(__float2half_rn(x));
  return x;
}

__device__ __forceinline__ void store_elem(void* p, int dtype, int64_t i, float x) {
  if (dtype == SMAQ_F32)
    static_cast<float*>(p)[i] = x;
  else if (dtype == SMAQ_BF16)
    static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(x);
  else
    static_cast<__half*>(p)[i] = __float2half_rn(x);
}

// Load EPL consecutive elements of type DT starting at p (p aligned to EPL*sizeof(T)).
template <class DT, int EPL>
__device__ __forceinline__ void load_vec(const typename DT::T* p, float (&x)[EPL]) {
  using T = typename DT::T;
  constexpr int BYTES = EPL * sizeof(T);
  if constexpr (BYTES == 16) {
    uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < EPL; ++i) x[i] = to_f(e[i]);
  } else if constexpr (BYTES == 8) {
    uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < EPL; ++i) x[i] = to_f(e[i]);
  } else if constexpr (BYTES == 4) {
    uint32_t u = __ldg(reinterpret_cast<const uint32_t*>(p));
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < EPL; ++i) x[i] = to_f(e[i]);
  } else {
#pragma unroll
    for (int i = 0; i < EPL; ++i) x[i] = to_f(p[i]);
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Store-row index of chunk token t, head h (see include/smaq_b200.h).
__device__ __forceinline__ int64_t store_row(const int64_t* slots, int64_t slot_offset,
                                             int64_t page_size, int n_heads, int64_t t, int h) {
  const int64_t s = slots ? slots[t] : slot_offset + t;
  const int64_t page = s / page_size;
  return (page * n_heads + h) * page_size + (s - page * page_size);
}

}  // namespace smaq
