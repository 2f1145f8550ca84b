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

// Two values rounded to the storage type at once (one packed conversion for bf16 / fp16).
template <class DT>
__device__ __forceinline__ void rnd2(float& a, float& b);
template <>
__device__ __forceinline__ void rnd2<F32>(float&, float&) {}
template <>
__device__ __forceinline__ void rnd2<BF16>(float& a, float& b) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
  a = __uint_as_float(r << 16);
  b = __uint_as_float(r & 0xFFFF0000u);
}
template <>
__device__ __forceinline__ void rnd2<F16>(float& a, float& b) {
  const float2 f = __half22float2(__floats2half2_rn(a, b));
  a = f.x;
  b = f.y;
}

// Correctly rounded x / d, kept out of line so that the rare exact-division paths below stay
// branches instead of being if-converted into every element.
static __device__ __noinline__ float div_exact(float x, float d) { return __fdiv_rn(x, d); }

// A quotient q with rnd<DT>(q) == rnd<DT>(x / d) for x, d values of DT, given rcp = 1/d
// rounded to nearest; x * rcp is within 2^-22 relative of x / d.
//  - bf16: a quotient of two bf16 values is never exactly a bf16 rounding midpoint
//    (X * 2^p = m * D has no solution with X, D 8-bit significands and m an odd 9-bit integer:
//    the odd part of the left side is at most 255), and otherwise lies at least
//    1 / (511 * 255) > 2^-17 relative from every midpoint, so x * rcp rounds like x / d.  Only a
//    quotient below 2^-126 (an fp32 subnormal product) can differ, by 2^-149; the callers
//    either clamp such values away (value scales and codes) or feed them to an fp32 contraction
//    whose rounding band is far wider (unit keys).
//  - fp16 (11-bit significands) has no such margin: x * rcp is used unless it lies within a few
//    fp32 ulps of an fp16 rounding midpoint or outside fp16's normal range, where the exact
//    division is evaluated.
//  - fp32 storage needs the exact quotient and always divides.
template <class DT>
__device__ __forceinline__ float quot(float x, float d, float rcp);
template <>
__device__ __forceinline__ float quot<F32>(float x, float d, float) { return __fdiv_rn(x, d); }
template <>
__device__ __forceinline__ float quot<BF16>(float x, float, float rcp) { return x * rcp; }
template <>
__device__ __forceinline__ float quot<F16>(float x, float d, float rcp) {
  const float q = x * rcp;
  const uint32_t u = __float_as_uint(q);
  const uint32_t ex = (u >> 23) & 0xFFu;  // fp16 normal range: biased fp32 exponent 113..142
  if (((u + 32u) & 0x1FC0u) == 0x1000u || (ex < 113u && (u << 1) != 0u) || ex > 142u) return div_exact(x, d);
  return q;
}

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

// n / d for 0 <= n < 2^31 by a multiply-high and a shift (Granlund & Montgomery, "Division by
// invariant integers using multiplication", 1994): l = ceil(log2 d), m = floor(2^32 (2^l - d) / d) + 1,
// n / d = (umulhi(n, m) + n) >> l.  d == 0 marks a divisor beyond 2^31 - 1 (callers divide in 64 bits).
struct FastDiv {
  uint32_t d, m, l;
};
inline FastDiv make_fastdiv(int64_t d) {
  FastDiv f{0u, 0u, 0u};
  if (d < 1 || d >= (int64_t(1) << 31)) return f;
  uint32_t l = 0;
  while ((uint64_t(1) << l) < uint64_t(d)) ++l;
  f.d = uint32_t(d);
  f.m = uint32_t(((uint64_t(1) << 32) * ((uint64_t(1) << l) - uint64_t(d))) / uint64_t(d) + 1);
  f.l = l;
  return f;
}

// Destination rows of an append (see include/smaq_b200.h): chunk row r = t * n_heads + h,
// token t lands in slot s = slots ? slots[t] : slot_offset + t, and
// row = (s / page_size * n_heads + h) * page_size + s % page_size.
struct RowMap {
  const int64_t* slots;
  int64_t slot_offset;
  int64_t page_size;
  int n_heads;
  FastDiv hdiv, pdiv;

  __device__ __forceinline__ void token_head(int64_t r, int64_t& t, int& h) const {
    if (r < (int64_t(1) << 31))
      t = int64_t((__umulhi(uint32_t(r), hdiv.m) + uint32_t(r)) >> hdiv.l);
    else
      t = r / n_heads;
    h = int(r - t * n_heads);
  }
  __device__ __forceinline__ int64_t row(int64_t t, int h) const {
    const int64_t s = slots ? slots[t] : slot_offset + t;
    int64_t page;
    if (pdiv.d != 0u && s >= 0 && s < (int64_t(1) << 31))
      page = int64_t((__umulhi(uint32_t(s), pdiv.m) + uint32_t(s)) >> pdiv.l);
    else
      page = s / page_size;
    return (page * n_heads + h) * page_size + (s - page * page_size);
  }
};

inline RowMap make_rowmap(const smaq_append_args& a) {
  RowMap m;
  m.slots = a.slots;
  m.slot_offset = a.slot_offset;
  m.page_size = a.page_size;
  m.n_heads = a.n_heads;
  m.hdiv = make_fastdiv(a.n_heads);
  m.pdiv = make_fastdiv(a.page_size);
  return m;
}

}  // namespace smaq
