// Append / quantize kernels: value codec, scalar metric-aware key codes, block-VQ key codes.
//
// Reference algorithm (gauravsaini/smaq):
//   values  smaq/kv_cache.py:50-91   group-asymmetric min/max quantization, storage-dtype arithmetic
//   keys    smaq/quantizer.py:138-145 norm -> k/(norm+1e-10) -> @E^T -> searchsorted -> pack
//   bvq     smaq/block_vq.py:216-244  per 8-dim block: @E_b^T -> cdist to the codebook -> argmin
//
// Bit-exactness: every elementwise step is computed in fp32 and rounded to the storage dtype
// exactly where torch rounds (one rounding per torch op).  Only the d x d contraction and the
// cdist dot products have a library-defined summation order; their results agree with the
// reference except for elements that sit within an fp32 rounding band of a decision boundary.
#include <math.h>

#include "common.cuh"
#include "ptx.cuh"
#include "tc_rotate.cuh"

namespace smaq {

// =====================================================================================
// values: one warp per row, EPL = head_dim / 32 consecutive elements per lane
// =====================================================================================
template <class DT, int EPL, int BITS>
__global__ void __launch_bounds__(256) value_quant_kernel(
    const typename DT::T* __restrict__ v, int64_t n_tokens, int n_heads, int64_t st, int64_t sh,
    const RowMap rm, int group_size,
    uint8_t* __restrict__ data, typename DT::T* __restrict__ scales, typename DT::T* __restrict__ zeros,
    int layout) {
  constexpr int D = 32 * EPL;
  constexpr int NL = (1 << BITS) - 1;
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  const int64_t n_rows = n_tokens * n_heads;
  const int lpg = group_size / EPL;  // lanes per group (power of two)
  const int ng = D / group_size;
  const float floor_ = rnd<DT>(1e-10f);
  for (int64_t r = warp; r < n_rows; r += nwarps) {
    int64_t t;
    int h;
    rm.token_head(r, t, h);
    float x[EPL];
    load_vec<DT, EPL>(v + t * st + h * sh + lane * EPL, x);
    float mn = x[0], mx = x[0];
#pragma unroll
    for (int i = 1; i < EPL; ++i) {
      mn = fminf(mn, x[i]);
      mx = fmaxf(mx, x[i]);
    }
    for (int o = 1; o < lpg; o <<= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    // scale = ((max - min) / n_levels).clamp(min=1e-10); zero = min   (kv_cache.py:78-83)
    float scale = rnd<DT>(quot<DT>(rnd<DT>(mx - mn), float(NL), 1.0f / float(NL)));
    if (scale < floor_) scale = floor_;
    const float rscale = __frcp_rn(scale);
    // ((v - zero) / scale).round().clamp(0, n_levels)   (kv_cache.py:85).  Clamping before the
    // round-half-even is the same as after it (the bounds are integers); the rounding is the
    // 1.5 * 2^23 addition, whose low mantissa bits are then the code.  NaN -> 0 like the
    // reference's uint8 cast.
    float d[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) d[i] = x[i] - mn;
#pragma unroll
    for (int i = 0; i < EPL; i += 2) rnd2<DT>(d[i], d[i + 1]);
#pragma unroll
    for (int i = 0; i < EPL; ++i) d[i] = quot<DT>(d[i], scale, rscale);
#pragma unroll
    for (int i = 0; i < EPL; i += 2) rnd2<DT>(d[i], d[i + 1]);
    uint32_t packed = 0;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const float q = fminf(fmaxf(d[i], 0.0f), float(NL)) + 12582912.0f;
      packed |= (__float_as_uint(q) - 0x4B400000u) << (i * BITS);
    }
    const int64_t row = rm.row(t, h);
    constexpr int LANE_BITS = EPL * BITS;
    uint8_t* dst = data + row * (D * BITS / 8);
    if constexpr (LANE_BITS >= 8) {
      constexpr int NB = LANE_BITS / 8;
      if constexpr (NB == 1) {
        // decode layout (2-bit, D = 128): reference byte 8j + g goes to byte 4g + j
        const int pos = layout == SMAQ_LAYOUT_DECODE ? 4 * (lane & 7) + (lane >> 3) : lane;
        dst[pos] = uint8_t(packed);
      } else if constexpr (NB == 2) {
        reinterpret_cast<uint16_t*>(dst)[lane] = uint16_t(packed);
      } else {
        reinterpret_cast<uint32_t*>(dst)[lane] = packed;
      }
    } else {  // 4 bits per lane: pair lanes into one byte
      const uint32_t hi = __shfl_down_sync(0xffffffffu, packed, 1);
      if ((lane & 1) == 0) dst[lane >> 1] = uint8_t(packed | (hi << 4));
    }
    if ((lane % lpg) == 0) {
      const int g = lane / lpg;
      scales[row * ng + g] = from_f<DT>(scale);
      zeros[row * ng + g] = from_f<DT>(mn);
    }
  }
}

// =====================================================================================
// values, bf16 / head_dim 128 / group 32 / 2 bits: one thread per group of 32 elements (four
// threads per row).  Every step is a packed bf16x2 operation where the reference's fp32-then-bf16
// rounding allows it: bf16 subtraction and min/max are exact-then-rounded; the division goes
// through the reciprocal (see quot<BF16>); round-half-even is the bf16 addition of 192, whose
// ulp is 1 on [128, 256), so the code is the low bits of the sum.
// =====================================================================================
__device__ __forceinline__ uint32_t bf2_sub(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t bf2_add(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t bf2_min(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("min.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t bf2_max(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t bf2_pack(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__global__ void __launch_bounds__(256) value_bf16_g32_kernel(
    const __nv_bfloat16* __restrict__ v, int64_t n_tokens, int n_heads, int64_t st, int64_t sh, const RowMap rm,
    uint8_t* __restrict__ data, __nv_bfloat16* __restrict__ scales, __nv_bfloat16* __restrict__ zeros, int layout,
    int after_keys) {
  const int64_t gid = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t n_rows = n_tokens * n_heads;
  const int64_t r = gid >> 2;
  const int g = int(gid & 3);
  const bool live = r < n_rows;
  int64_t t = 0;
  int h = 0;
  uint32_t x[16];
  if (live) {
    rm.token_head(r, t, h);
    const uint4* src = reinterpret_cast<const uint4*>(v + t * st + h * sh + 32 * g);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 u = __ldg(src + i);
      x[4 * i] = u.x; x[4 * i + 1] = u.y; x[4 * i + 2] = u.z; x[4 * i + 3] = u.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) x[i] = 0u;
  }
  // min / max over the group (NaN-ignoring, like fminf)
  uint32_t mn2 = x[0], mx2 = x[0];
#pragma unroll
  for (int i = 1; i < 16; ++i) {
    mn2 = bf2_min(mn2, x[i]);
    mx2 = bf2_max(mx2, x[i]);
  }
  const float mn = fminf(__uint_as_float(mn2 << 16), __uint_as_float(mn2 & 0xFFFF0000u));
  const float mx = fmaxf(__uint_as_float(mx2 << 16), __uint_as_float(mx2 & 0xFFFF0000u));
  // scale = ((max - min) / 3).clamp(min=1e-10); zero = min   (kv_cache.py:78-83)
  float scale = rnd<BF16>(quot<BF16>(rnd<BF16>(mx - mn), 3.0f, 1.0f / 3.0f));
  const float floor_ = rnd<BF16>(1e-10f);
  if (scale < floor_) scale = floor_;
  const float rscale = __frcp_rn(scale);
  const uint32_t mnb = __float_as_uint(mn) >> 16;
  const uint32_t mn_pair = mnb | (mnb << 16);
  // ((v - zero) / scale).round().clamp(0, 3)   (kv_cache.py:85); NaN -> 0
  const uint32_t zero2 = 0u, three2 = 0x40404040u, magic2 = 0x43404340u;  // bf16 pairs 0, 3, 192
  // q = 192 + code in each bf16 half: the code is bits 0-1 (element 2i) and 16-17 (element
  // 2i + 1), and 192's own low mantissa bits are 0.  Pairs i = 4k .. 4k + 3 collect their two
  // code fields at bits 4(i - 4k) and 16 + 4(i - 4k) of acc[k]; one shift-and-merge per acc[k]
  // then interleaves them into the packed order (element 2i at bit 4i, 2i + 1 at bit 4i + 2).
  uint32_t acc[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint32_t d = bf2_sub(x[i], mn_pair);
    uint32_t q = bf2_pack(__uint_as_float(d << 16) * rscale, __uint_as_float(d & 0xFFFF0000u) * rscale);
    q = bf2_add(bf2_min(bf2_max(q, zero2), three2), magic2);
    acc[i >> 2] |= (q & 0x00030003u) << (4 * (i & 3));
  }
  uint32_t half16[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) half16[k] = (acc[k] & 0x3333u) | ((acc[k] >> 14) & 0xCCCCu);
  uint32_t lo = half16[0] | (half16[1] << 16), hi = half16[2] | (half16[3] << 16);
  if (layout == SMAQ_LAYOUT_DECODE) {
    // byte 4 * b + g of the row holds reference byte 8 * g + b (b < 8): transpose the 4 x 8
    // byte matrix held by the row's four threads.  16-bit chunk c of thread g = bytes 2c, 2c+1.
    uint32_t send = (g & 2) ? lo : hi;
    uint32_t recv = __shfl_xor_sync(0xffffffffu, send, 2);
    if (g & 2) lo = recv; else hi = recv;
    // now lo = chunks {2*b1, 2*b1+1}... of sources with bit1 = 0, hi = of sources with bit1 = 1
    send = (g & 1) ? __byte_perm(lo, hi, 0x5410) : __byte_perm(lo, hi, 0x7632);
    recv = __shfl_xor_sync(0xffffffffu, send, 1);
    uint32_t c01, c23;  // chunk g of sources (0, 1) and (2, 3)
    if (g & 1) {
      c01 = __byte_perm(recv, lo, 0x7610);  // source 0 from partner (low), source 1 own (lo high)
      c23 = __byte_perm(recv, hi, 0x7632);  // source 2 from partner (high), source 3 own (hi high)
    } else {
      c01 = __byte_perm(lo, recv, 0x5410);  // source 0 own (lo low), source 1 from partner (low)
      c23 = __byte_perm(hi, recv, 0x7610);  // source 2 own (hi low), source 3 from partner (high)
    }
    lo = __byte_perm(c01, c23, 0x6420);  // byte 2g of sources 0..3
    hi = __byte_perm(c01, c23, 0x7531);  // byte 2g + 1 of sources 0..3
  }
  // launched overlapped with the key kernel of the same append: the last block waits for that
  // grid, so this grid completes (and the stream moves on) only after both
  if (after_keys && blockIdx.x == gridDim.x - 1) pdl_wait();
  if (!live) return;  // after the shuffles: whole rows are live or not, warps stay converged
  const int64_t row = rm.row(t, h);
  reinterpret_cast<uint2*>(data + row * 32)[g] = make_uint2(lo, hi);
  scales[row * 4 + g] = __float2bfloat16_rn(scale);
  zeros[row * 4 + g] = __float2bfloat16_rn(mn);
}

// =====================================================================================
// scalar keys (SIMT path): a warp quantizes R rows at a time; E^T and the k_unit rows are
// staged in shared memory.  Used for fp32/fp16 keys and for head_dim != 128; bf16 keys at
// head_dim 128 take the tcgen05 path in tc_rotate.cuh.
// =====================================================================================
constexpr int SQ_WARPS = 8;
constexpr int SQ_ROWS = 8;

template <class DT, int EPL, int BITS>
__global__ void __launch_bounds__(SQ_WARPS * 32) scalar_key_kernel(
    const typename DT::T* __restrict__ k, int64_t n_tokens, int n_heads, int64_t st, int64_t sh,
    const RowMap rm,
    const float* __restrict__ E, const float* __restrict__ bnd, uint8_t* __restrict__ codes,
    typename DT::T* __restrict__ norms, int layout) {
  constexpr int D = 32 * EPL;
  constexpr int NB = (1 << BITS) - 1;
  constexpr int VPB = (8 / BITS) > 0 ? 8 / BITS : 1;
  constexpr int PD = (D + VPB - 1) / VPB;
  extern __shared__ float smem[];
  float* ET = smem;                       // [D][D]: ET[i][j] = E[j][i]
  float* KU = ET + D * D;                 // [warps][R][D]
  __shared__ float sb[16];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int idx = threadIdx.x; idx < D * D; idx += blockDim.x) {
    const int j = idx / D, i = idx - j * D;
    ET[i * D + j] = E[idx];
  }
  if (threadIdx.x < NB) sb[threadIdx.x] = bnd[threadIdx.x];
  __syncthreads();
  float b[NB];
#pragma unroll
  for (int i = 0; i < NB; ++i) b[i] = sb[i];
  float* ku = KU + wid * SQ_ROWS * D;
  const int64_t n_rows = n_tokens * n_heads;
  const int64_t gw = int64_t(blockIdx.x) * SQ_WARPS + wid;
  const int64_t nw = int64_t(gridDim.x) * SQ_WARPS;
  for (int64_t r0 = gw * SQ_ROWS; r0 < n_rows; r0 += nw * SQ_ROWS) {
    float nrm[SQ_ROWS];
#pragma unroll
    for (int rr = 0; rr < SQ_ROWS; ++rr) {
      const int64_t r = r0 + rr;
      float x[EPL];
      if (r < n_rows) {
        int64_t t;
        int h;
        rm.token_head(r, t, h);
        load_vec<DT, EPL>(k + t * st + h * sh + lane * EPL, x);
      } else {
#pragma unroll
        for (int i = 0; i < EPL; ++i) x[i] = 0.f;
      }
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < EPL; ++i) ss = fmaf(x[i], x[i], ss);
      ss = warp_sum(ss);
      // norms = k.norm(-1) in the key dtype; k_unit = k / (norms + 1e-10)  (quantizer.py:140-141)
      const float n = rnd<DT>(sqrtf(ss));
      nrm[rr] = n;
      const float den = rnd<DT>(n + 1e-10f);
      const float rden = __frcp_rn(den);
#pragma unroll
      for (int i = 0; i < EPL; ++i) x[i] = quot<DT>(x[i], den, rden);
#pragma unroll
      for (int i = 0; i < EPL; i += 2) rnd2<DT>(x[i], x[i + 1]);
#pragma unroll
      for (int i = 0; i < EPL; ++i) ku[rr * D + lane * EPL + i] = x[i];
    }
    __syncwarp();
    // y = k_unit.float() @ E.T  (quantizer.py:142)
    float y[SQ_ROWS][EPL];
#pragma unroll
    for (int rr = 0; rr < SQ_ROWS; ++rr)
#pragma unroll
      for (int e = 0; e < EPL; ++e) y[rr][e] = 0.f;
#pragma unroll 4
    for (int i = 0; i < D; ++i) {
      float et[EPL];
      if constexpr (EPL == 4) {
        const float4 w = *reinterpret_cast<const float4*>(ET + i * D + lane * 4);
        et[0] = w.x; et[1] = w.y; et[2] = w.z; et[3] = w.w;
      } else {
#pragma unroll
        for (int e = 0; e < EPL; ++e) et[e] = ET[i * D + lane * EPL + e];
      }
#pragma unroll
      for (int rr = 0; rr < SQ_ROWS; ++rr) {
        const float a = ku[rr * D + i];
#pragma unroll
        for (int e = 0; e < EPL; ++e) y[rr][e] = fmaf(a, et[e], y[rr][e]);
      }
    }
    __syncwarp();
#pragma unroll
    for (int rr = 0; rr < SQ_ROWS; ++rr) {
      const int64_t r = r0 + rr;
      if (r >= n_rows) break;
      int64_t t;
      int h;
      rm.token_head(r, t, h);
      const int64_t row = rm.row(t, h);
      // searchsorted(decision_boundaries, y), right=False: count of boundaries < y  (:143)
      uint32_t c[EPL];
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        int cnt = 0;
#pragma unroll
        for (int i = 0; i < NB; ++i) cnt += (b[i] < y[rr][e]) ? 1 : 0;
        c[e] = isnan(y[rr][e]) ? uint32_t(NB) : uint32_t(cnt);
      }
      uint8_t* dst = codes + row * PD;
      // _pack_indices (quantizer.py:34-46): VPB codes per byte, LSB first
      if constexpr (VPB == 4) {       // 2-bit: EPL codes -> EPL/4 bytes (EPL is 2 or 4)
        if constexpr (EPL == 4) {
          dst[lane] = uint8_t(c[0] | (c[1] << 2) | (c[2] << 4) | (c[3] << 6));
        } else {
          const uint32_t p = c[0] | (c[1] << 2);
          const uint32_t hi = __shfl_down_sync(0xffffffffu, p, 1);
          if ((lane & 1) == 0) dst[lane >> 1] = uint8_t(p | (hi << 4));
        }
      } else {                        // 3- and 4-bit: two codes per byte at shifts 0 and BITS
#pragma unroll
        for (int e = 0; e < EPL; e += 2) {
          const int pb = (lane * EPL + e) / 2;
          // decode layout (3/4-bit, head_dim 128): reference byte p at 16 (p % 4) + p / 4
          dst[layout == SMAQ_LAYOUT_DECODE ? 16 * (pb & 3) + (pb >> 2) : pb] = uint8_t(c[e] | (c[e + 1] << BITS));
        }
      }
      if (lane == 0) norms[row] = from_f<DT>(nrm[rr]);
    }
    __syncwarp();
  }
}

// =====================================================================================
// block VQ keys: a warp encodes BQ_ROWS rows per pass; codebook and its squared norms live
// in shared memory.  Distances follow torch.cdist's matmul expansion
//   d2 = |x|^2 + |c|^2 - 2 x.c,  dist = sqrt(clamp(d2, 0)),  argmin (first index on ties).
// =====================================================================================
constexpr int BQ_WARPS = 16;
constexpr int BQ_ROWS = 4;

template <class DT, int EPL>
__global__ void __launch_bounds__(BQ_WARPS * 32) bvq_key_kernel(
    const typename DT::T* __restrict__ k, int64_t n_tokens, int n_heads, int64_t st, int64_t sh,
    const RowMap rm,
    const float* __restrict__ Eb, const float* __restrict__ cent, int nc, uint8_t* __restrict__ out,
    int layout) {
  constexpr int D = 32 * EPL;
  constexpr int BD = 8;
  constexpr int NBLK = D / BD;
  extern __shared__ float smem[];
  float* C = smem;                        // [NBLK][nc][8]
  float* CN = C + NBLK * nc * BD;         // [NBLK][nc]
  float* EB = CN + NBLK * nc;             // [NBLK][8][8]
  float* KS = EB + NBLK * BD * BD;        // [warps][BQ_ROWS][D]
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < NBLK * nc * BD; i += blockDim.x) C[i] = cent[i];
  for (int i = threadIdx.x; i < NBLK * BD * BD; i += blockDim.x) EB[i] = Eb[i];
  __syncthreads();
  for (int i = threadIdx.x; i < NBLK * nc; i += blockDim.x) {
    float s = 0.f;  // x2.pow(2).sum(-1)
#pragma unroll
    for (int j = 0; j < BD; ++j) s = fmaf(C[i * BD + j], C[i * BD + j], s);
    CN[i] = s;
  }
  __syncthreads();
  float* ks = KS + wid * BQ_ROWS * D;
  const int64_t n_rows = n_tokens * n_heads;
  const int64_t gw = int64_t(blockIdx.x) * BQ_WARPS + wid;
  const int64_t nw = int64_t(gridDim.x) * BQ_WARPS;
  for (int64_t r0 = gw * BQ_ROWS; r0 < n_rows; r0 += nw * BQ_ROWS) {
    // shaped keys: k_b.float() @ E_b^T per block   (block_vq.py:230-235)
#pragma unroll
    for (int rr = 0; rr < BQ_ROWS; ++rr) {
      const int64_t r = r0 + rr;
      float x[EPL];
      if (r < n_rows) {
        int64_t t;
        int h;
        rm.token_head(r, t, h);
        load_vec<DT, EPL>(k + t * st + h * sh + lane * EPL, x);
      } else {
#pragma unroll
        for (int i = 0; i < EPL; ++i) x[i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < EPL; ++i) ks[rr * D + lane * EPL + i] = x[i];
    }
    __syncwarp();
    float sh_[BQ_ROWS][EPL];
#pragma unroll
    for (int rr = 0; rr < BQ_ROWS; ++rr) {
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        const int j = lane * EPL + e, blk = j / BD, jj = j % BD;
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < BD; ++i) s = fmaf(ks[rr * D + blk * BD + i], EB[(blk * BD + jj) * BD + i], s);
        sh_[rr][e] = s;
      }
    }
    __syncwarp();
#pragma unroll
    for (int rr = 0; rr < BQ_ROWS; ++rr)
#pragma unroll
      for (int e = 0; e < EPL; ++e) ks[rr * D + lane * EPL + e] = sh_[rr][e];
    __syncwarp();
    for (int blk = 0; blk < NBLK; ++blk) {
      float xs[BQ_ROWS][BD], xn[BQ_ROWS];
#pragma unroll
      for (int rr = 0; rr < BQ_ROWS; ++rr) {
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < BD; ++j) {
          xs[rr][j] = ks[rr * D + blk * BD + j];
          s = fmaf(xs[rr][j], xs[rr][j], s);
        }
        xn[rr] = s;
      }
      float best[BQ_ROWS];
      int bi[BQ_ROWS];
#pragma unroll
      for (int rr = 0; rr < BQ_ROWS; ++rr) {
        best[rr] = INFINITY;
        bi[rr] = 0;
      }
      for (int c = lane; c < nc; c += 32) {
        const float4 c0 = *reinterpret_cast<const float4*>(C + (blk * nc + c) * BD);
        const float4 c1 = *reinterpret_cast<const float4*>(C + (blk * nc + c) * BD + 4);
        const float cv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
        const float cn = CN[blk * nc + c];
#pragma unroll
        for (int rr = 0; rr < BQ_ROWS; ++rr) {
          float dot = 0.f;
#pragma unroll
          for (int j = 0; j < BD; ++j) dot = fmaf(-2.0f * xs[rr][j], cv[j], dot);
          // squared distance, clamped at 0 as cdist does; its square root is monotone, so the
          // argmin is the same except where two squared distances one ulp apart share a square
          // root (a near-tie, resolved by the lower index in cdist)
          const float d = fmaxf(dot + xn[rr] + cn, 0.0f);
          if (d < best[rr]) {
            best[rr] = d;
            bi[rr] = c;
          }
        }
      }
#pragma unroll
      for (int rr = 0; rr < BQ_ROWS; ++rr) {
        float bv = best[rr];
        int bx = bi[rr];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int ox = __shfl_xor_sync(0xffffffffu, bx, o);
          if (ov < bv || (ov == bv && ox < bx)) {
            bv = ov;
            bx = ox;
          }
        }
        bi[rr] = bx;
      }
      if (lane == 0) {
#pragma unroll
        for (int rr = 0; rr < BQ_ROWS; ++rr) {
          const int64_t r = r0 + rr;
          if (r < n_rows) {
            int64_t t;
            int h;
            rm.token_head(r, t, h);
            const int64_t row = rm.row(t, h);
            int64_t off = row * NBLK + blk;
            if (layout == SMAQ_LAYOUT_DECODE)  // see include/smaq_b200.h
              off = row * NBLK + 2 * (4 * (blk >> 3) + (blk & 3)) + ((blk >> 2) & 1);
            out[off] = uint8_t(bi[rr]);
          }
        }
      }
    }
    __syncwarp();
  }
}

// =====================================================================================
// host side
// =====================================================================================
static int grid_for(int64_t warps_needed, int warps_per_block, int blocks_per_sm) {
  int64_t g = (warps_needed + warps_per_block - 1) / warps_per_block;
  const int64_t cap = int64_t(num_sms()) * blocks_per_sm;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return int(g);
}

template <class DT, int EPL>
static int launch_values_t(const smaq_append_args& a, cudaStream_t s) {
  const int64_t rows = a.n_tokens * a.n_heads;
  const int grid = grid_for(rows, 8, 8);
  using T = typename DT::T;
  if (a.value_bits == 2)
    value_quant_kernel<DT, EPL, 2><<<grid, 256, 0, s>>>(
        static_cast<const T*>(a.v), a.n_tokens, a.n_heads, a.v_stride_t, a.v_stride_h, make_rowmap(a),
        a.group_size, a.v_data, static_cast<T*>(a.v_scales),
        static_cast<T*>(a.v_zeros), a.layout);
  else
    value_quant_kernel<DT, EPL, 4><<<grid, 256, 0, s>>>(
        static_cast<const T*>(a.v), a.n_tokens, a.n_heads, a.v_stride_t, a.v_stride_h, make_rowmap(a),
        a.group_size, a.v_data, static_cast<T*>(a.v_scales),
        static_cast<T*>(a.v_zeros), SMAQ_LAYOUT_REFERENCE);
  return cuda_status(cudaGetLastError(), "value_quant_kernel");
}

// after_keys: the key kernel of the same append was launched just before on `s`; the fast bf16
// value kernel then starts as its programmatic dependent and runs beside it (the key kernel
// leaves room for one 128-thread block per SM).
template <class DT>
static int launch_values_d(const smaq_append_args& a, cudaStream_t s, int after_keys) {
  if constexpr (std::is_same<DT, BF16>::value) {
    if (a.head_dim == 128 && a.group_size == 32 && a.value_bits == 2 &&
        reinterpret_cast<uintptr_t>(a.v) % 16 == 0 && a.v_stride_t % 8 == 0 && a.v_stride_h % 8 == 0 &&
        reinterpret_cast<uintptr_t>(a.v_data) % 8 == 0) {
      // 128-thread blocks: beside the key kernel (18 warps at 96 registers, 5/5/4/4 per SM
      // sub-partition) only two sub-partitions have room, three 40-register warps each
      const int64_t threads = a.n_tokens * a.n_heads * 4;
      const int64_t blocks = (threads + 127) / 128;
      if (blocks <= 0) return SMAQ_OK;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(unsigned(blocks));
      cfg.blockDim = dim3(128);
      cfg.stream = s;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = after_keys ? 1 : 0;
      return cuda_status(
          cudaLaunchKernelEx(&cfg, value_bf16_g32_kernel, static_cast<const __nv_bfloat16*>(a.v), a.n_tokens,
                             a.n_heads, a.v_stride_t, a.v_stride_h, make_rowmap(a), a.v_data,
                             static_cast<__nv_bfloat16*>(a.v_scales), static_cast<__nv_bfloat16*>(a.v_zeros),
                             a.layout, after_keys),
          "value_bf16_g32_kernel");
    }
  }
  switch (a.head_dim) {
    case 64: return launch_values_t<DT, 2>(a, s);
    case 128: return launch_values_t<DT, 4>(a, s);
    case 256: return launch_values_t<DT, 8>(a, s);
  }
  return fail(SMAQ_ERR_UNSUPPORTED, "values: head_dim %d not in {64,128,256}", a.head_dim);
}

template <class DT, int EPL, int BITS>
static int launch_scalar_t(const smaq_append_args& a, cudaStream_t s) {
  constexpr int D = 32 * EPL;
  const size_t sm = sizeof(float) * (D * D + SQ_WARPS * SQ_ROWS * D);
  auto kern = scalar_key_kernel<DT, EPL, BITS>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm));
  if (e != cudaSuccess) return cuda_status(e, "scalar_key_kernel attr");
  const int64_t rows = a.n_tokens * a.n_heads;
  const int grid = grid_for((rows + SQ_ROWS - 1) / SQ_ROWS, SQ_WARPS, 2);
  using T = typename DT::T;
  kern<<<grid, SQ_WARPS * 32, sm, s>>>(static_cast<const T*>(a.k), a.n_tokens, a.n_heads, a.k_stride_t,
                                       a.k_stride_h, make_rowmap(a), a.E,
                                       a.boundaries, a.key_codes, static_cast<T*>(a.key_norms), a.layout);
  return cuda_status(cudaGetLastError(), "scalar_key_kernel");
}

template <class DT, int EPL>
static int launch_scalar_b(const smaq_append_args& a, cudaStream_t s) {
  switch (a.key_bits) {
    case 2: return launch_scalar_t<DT, EPL, 2>(a, s);
    case 3: return launch_scalar_t<DT, EPL, 3>(a, s);
    case 4: return launch_scalar_t<DT, EPL, 4>(a, s);
  }
  return fail(SMAQ_ERR_UNSUPPORTED, "scalar keys: bits %d not in {2,3,4}", a.key_bits);
}

template <class DT>
static int launch_scalar_d(const smaq_append_args& a, cudaStream_t s) {
  if constexpr (std::is_same<DT, BF16>::value) {
    if (tc_rotate_eligible(a)) return launch_scalar_keys_tc(a, s);
  }
  switch (a.head_dim) {
    case 64: return launch_scalar_b<DT, 2>(a, s);
    case 128: return launch_scalar_b<DT, 4>(a, s);
  }
  return fail(SMAQ_ERR_UNSUPPORTED, "scalar keys: head_dim %d not in {64,128}", a.head_dim);
}

// ---------------------------------------------------------------------------------------
// Block-VQ encode on the tensor cores (bf16 keys, D = 128, 8-dim blocks, <= 256 codes).
// argmin_c |k_b E_b^T - c|^2 = argmin_c (|c|^2 - 2 k_b . c'), c' = c E_b, so each block is a
// [rows x 8] x [8 x 256] product: mma.m16n8k8 with A = the raw bf16 key (exact) and B = c'
// split into three bf16 terms (hi + mid + lo hold c' to ~2^-24), fp32 accumulation.  Thread
// (gid, tig) holds rows gid, gid + 8 and codes 8n + 2tig, +1 of every n-tile; the running
// minimum per row is merged over the 4 tig lanes at the end of the block, ties to the lower
// code (cdist + argmin's first index; a difference against the reference can only be a
// near-tie, as |x|^2 is left out and the sum order differs).
constexpr int BM_WARPS = 16;
constexpr int BM_NT = 32;                         // n-tiles of 8 codes
constexpr int BM_BBYTES = 16 * BM_NT * 3 * 32 * 4;  // B fragments [blk][nt][split][lane]
constexpr int BM_SMEM = BM_BBYTES + 16 * 256 * 4;   // + |c|^2 [blk][code]

__device__ __forceinline__ uint32_t bm_pack_bf16(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ void bm_mma(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm("mma.sync.aligned.m16n8k8.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(b0));
}

__global__ void __launch_bounds__(BM_WARPS * 32, 1) bvq_mma_kernel(
    const __nv_bfloat16* __restrict__ k, int64_t n_tokens, int n_heads, int64_t st, int64_t sh, const RowMap rm,
    const float* __restrict__ Eb, const float* __restrict__ cent, int nc, uint8_t* __restrict__ out, int layout) {
  extern __shared__ __align__(16) uint8_t bm_smem[];
  uint32_t* Bf = reinterpret_cast<uint32_t*>(bm_smem);                  // [16][32][3][32]
  float* CN = reinterpret_cast<float*>(bm_smem + BM_BBYTES);             // [16][256]
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  // c' = c E_b per (block, code): fragment (nt, lane) holds c'[8nt + gid][2tig, 2tig+1]
  for (int i = threadIdx.x; i < 16 * BM_NT * 32; i += blockDim.x) {
    const int blk = i / (BM_NT * 32), r = i - blk * BM_NT * 32, nt = r >> 5, l = r & 31;
    const int code = 8 * nt + (l >> 2), d0 = 2 * (l & 3);
    float v[2] = {0.f, 0.f};
    if (code < nc) {
      const float* c = cent + (int64_t(blk) * nc + code) * 8;
      const float* E = Eb + blk * 64;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) acc = fmaf(c[j], E[j * 8 + d0 + e], acc);
        v[e] = acc;
      }
    }
    uint32_t* dst = Bf + ((blk * BM_NT + nt) * 3) * 32 + l;
#pragma unroll
    for (int sp = 0; sp < 3; ++sp) {
      const uint32_t h = bm_pack_bf16(v[0], v[1]);
      dst[sp * 32] = h;
      v[0] -= __uint_as_float(h << 16);
      v[1] -= __uint_as_float(h & 0xffff0000u);
    }
  }
  for (int i = threadIdx.x; i < 16 * 256; i += blockDim.x) {
    const int blk = i >> 8, code = i & 255;
    float sq = INFINITY;  // codes past nc never win
    if (code < nc) {
      const float* c = cent + (int64_t(blk) * nc + code) * 8;
      sq = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) sq = fmaf(c[j], c[j], sq);
    }
    CN[i] = sq;
  }
  __syncthreads();
  const int64_t n_rows = n_tokens * n_heads;
  const int64_t n_tiles = (n_rows + 15) / 16;
  for (int64_t tile = int64_t(blockIdx.x) * BM_WARPS + wid; tile < n_tiles; tile += int64_t(gridDim.x) * BM_WARPS) {
    const int64_t r0 = tile * 16 + gid, r1 = r0 + 8;
    // A fragments of all 16 blocks for rows r0, r1 (dims 8 blk + 2 tig, +1)
    uint32_t a0[16], a1[16];
    {
      int64_t t;
      int h;
      const uint32_t* p0 = nullptr;
      const uint32_t* p1 = nullptr;
      if (r0 < n_rows) { rm.token_head(r0, t, h); p0 = reinterpret_cast<const uint32_t*>(k + t * st + h * sh); }
      if (r1 < n_rows) { rm.token_head(r1, t, h); p1 = reinterpret_cast<const uint32_t*>(k + t * st + h * sh); }
#pragma unroll
      for (int b = 0; b < 16; ++b) {
        a0[b] = p0 ? __ldg(p0 + 4 * b + tig) : 0u;
        a1[b] = p1 ? __ldg(p1 + 4 * b + tig) : 0u;
      }
    }
    uint32_t best_idx0[4] = {0u, 0u, 0u, 0u}, best_idx1[4] = {0u, 0u, 0u, 0u};  // 4 blocks per word
#pragma unroll 1
    for (int b = 0; b < 16; ++b) {
      float v0 = INFINITY, v1 = INFINITY;
      int i0 = 0, i1 = 0;
      const uint32_t* bb = Bf + (b * BM_NT * 3) * 32 + lane;
      const float* cn = CN + b * 256 + 2 * tig;
#pragma unroll 4
      for (int nt = 0; nt < BM_NT; ++nt) {
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        bm_mma(d, a0[b], a1[b], bb[(nt * 3 + 2) * 32]);  // smallest term first
        bm_mma(d, a0[b], a1[b], bb[(nt * 3 + 1) * 32]);
        bm_mma(d, a0[b], a1[b], bb[(nt * 3 + 0) * 32]);
        const float2 c2 = *reinterpret_cast<const float2*>(cn + 8 * nt);
        const int code = 8 * nt + 2 * tig;
        const float s0 = fmaf(-2.f, d[0], c2.x), s1 = fmaf(-2.f, d[1], c2.y);
        const float s2 = fmaf(-2.f, d[2], c2.x), s3 = fmaf(-2.f, d[3], c2.y);
        if (s0 < v0) { v0 = s0; i0 = code; }
        if (s1 < v0) { v0 = s1; i0 = code + 1; }
        if (s2 < v1) { v1 = s2; i1 = code; }
        if (s3 < v1) { v1 = s3; i1 = code + 1; }
      }
#pragma unroll
      for (int o = 1; o <= 2; o <<= 1) {
        const float ov0 = __shfl_xor_sync(0xffffffffu, v0, o), ov1 = __shfl_xor_sync(0xffffffffu, v1, o);
        const int oi0 = __shfl_xor_sync(0xffffffffu, i0, o), oi1 = __shfl_xor_sync(0xffffffffu, i1, o);
        if (ov0 < v0 || (ov0 == v0 && oi0 < i0)) { v0 = ov0; i0 = oi0; }
        if (ov1 < v1 || (ov1 == v1 && oi1 < i1)) { v1 = ov1; i1 = oi1; }
      }
      best_idx0[b >> 2] |= uint32_t(i0) << (8 * (b & 3));
      best_idx1[b >> 2] |= uint32_t(i1) << (8 * (b & 3));
    }
    if (tig == 0) {
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        const int64_t r = rr ? r1 : r0;
        if (r >= n_rows) continue;
        const uint32_t* bi = rr ? best_idx1 : best_idx0;
        int64_t t;
        int h;
        rm.token_head(r, t, h);
        uint8_t* row = out + rm.row(t, h) * 16;
        uint32_t w[4];
        if (layout == SMAQ_LAYOUT_DECODE) {  // block b at byte 2 (4 (b / 8) + b % 4) + (b / 4) % 2
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            // bytes 4q..4q+3 hold blocks {2q', ...}: byte p <- block sigma^-1(p)
            uint32_t v = 0;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int p = 4 * q + e;
              const int hi8 = p >> 3, rem = p & 7, lo4 = rem >> 1, par = rem & 1;
              const int blk = 8 * hi8 + 4 * par + lo4;
              v |= ((bi[blk >> 2] >> (8 * (blk & 3))) & 0xffu) << (8 * e);
            }
            w[q] = v;
          }
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q) w[q] = bi[q];
        }
        *reinterpret_cast<uint4*>(row) = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  }
}

static int launch_bvq_mma(const smaq_append_args& a, cudaStream_t s) {
  cudaError_t e = cudaFuncSetAttribute(bvq_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, BM_SMEM);
  if (e != cudaSuccess) return cuda_status(e, "bvq_mma_kernel attr");
  const int64_t rows = a.n_tokens * a.n_heads;
  const int64_t tiles = (rows + 15) / 16;
  const int64_t want = (tiles + BM_WARPS - 1) / BM_WARPS;
  const int grid = int(want < num_sms() ? want : num_sms());
  bvq_mma_kernel<<<grid, BM_WARPS * 32, BM_SMEM, s>>>(static_cast<const __nv_bfloat16*>(a.k), a.n_tokens, a.n_heads,
                                                      a.k_stride_t, a.k_stride_h, make_rowmap(a), a.E_blocks,
                                                      a.centroids, a.n_centroids, a.key_codes, a.layout);
  return cuda_status(cudaGetLastError(), "bvq_mma_kernel");
}

template <class DT, int EPL>
static int launch_bvq_t(const smaq_append_args& a, cudaStream_t s) {
  constexpr int D = 32 * EPL;
  constexpr int NBLK = D / 8;
  const int nc = a.n_centroids;
  const size_t sm = sizeof(float) * (NBLK * nc * 8 + NBLK * nc + NBLK * 64 + BQ_WARPS * BQ_ROWS * D);
  auto kern = bvq_key_kernel<DT, EPL>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm));
  if (e != cudaSuccess) return cuda_status(e, "bvq_key_kernel attr");
  const int64_t rows = a.n_tokens * a.n_heads;
  const int grid = grid_for((rows + BQ_ROWS - 1) / BQ_ROWS, BQ_WARPS, 1);
  using T = typename DT::T;
  kern<<<grid, BQ_WARPS * 32, sm, s>>>(static_cast<const T*>(a.k), a.n_tokens, a.n_heads, a.k_stride_t,
                                       a.k_stride_h, make_rowmap(a), a.E_blocks,
                                       a.centroids, nc, a.key_codes, a.layout);
  return cuda_status(cudaGetLastError(), "bvq_key_kernel");
}

template <class DT>
static int launch_bvq_d(const smaq_append_args& a, cudaStream_t s) {
  // bf16 keys of D = 128 with 16-byte aligned rows: the tensor-core encode
  if (DT::code == SMAQ_BF16 && a.head_dim == 128 && a.n_centroids <= 256 &&
      ((reinterpret_cast<uintptr_t>(a.k) | uintptr_t(a.k_stride_t * 2) | uintptr_t(a.k_stride_h * 2)) & 15) == 0)
    return launch_bvq_mma(a, s);
  switch (a.head_dim) {
    case 64: return launch_bvq_t<DT, 2>(a, s);
    case 128: return launch_bvq_t<DT, 4>(a, s);
  }
  return fail(SMAQ_ERR_UNSUPPORTED, "bvq keys: head_dim %d not in {64,128}", a.head_dim);
}

template <template <class> class F>
static int by_dtype(int dtype, const smaq_append_args& a, cudaStream_t s, int after_keys = 0) {
  switch (dtype) {
    case SMAQ_F32: return F<F32>::run(a, s, after_keys);
    case SMAQ_BF16: return F<BF16>::run(a, s, after_keys);
    case SMAQ_F16: return F<F16>::run(a, s, after_keys);
  }
  return fail(SMAQ_ERR_INVALID, "unknown dtype %d", dtype);
}
template <class DT> struct RunValues { static int run(const smaq_append_args& a, cudaStream_t s, int after_keys) { return launch_values_d<DT>(a, s, after_keys); } };
template <class DT> struct RunScalar { static int run(const smaq_append_args& a, cudaStream_t s, int) { return launch_scalar_d<DT>(a, s); } };
template <class DT> struct RunBvq { static int run(const smaq_append_args& a, cudaStream_t s, int) { return launch_bvq_d<DT>(a, s); } };

static size_t dsize(int dtype) { return dtype == SMAQ_F32 ? 4 : 2; }

static int validate_append(const smaq_append_args& a) {
  if (a.n_tokens < 0 || a.n_heads <= 0 || a.head_dim <= 0)
    return fail(SMAQ_ERR_INVALID, "append: bad sizes n_tokens=%lld n_heads=%d head_dim=%d",
                (long long)a.n_tokens, a.n_heads, a.head_dim);
  if (a.page_size <= 0) return fail(SMAQ_ERR_INVALID, "append: page_size must be > 0");
  if (a.dtype != SMAQ_F32 && a.dtype != SMAQ_BF16 && a.dtype != SMAQ_F16)
    return fail(SMAQ_ERR_INVALID, "append: unknown dtype %d", a.dtype);
  const size_t es = dsize(a.dtype);
  const int epl = a.head_dim / 32;
  if (a.layout != SMAQ_LAYOUT_REFERENCE && a.layout != SMAQ_LAYOUT_DECODE)
    return fail(SMAQ_ERR_INVALID, "append: unknown layout %d", a.layout);
  if (a.layout == SMAQ_LAYOUT_DECODE) {
    if (a.head_dim != 128 || (a.v && a.value_bits != 2) || (a.k && a.key_format == SMAQ_KEYS_BVQ && a.block_dim != 8) ||
        (a.k && a.key_format == SMAQ_KEYS_SCALAR && a.key_bits != 3 && a.key_bits != 4))
      return fail(SMAQ_ERR_UNSUPPORTED,
                  "decode layout needs head_dim 128, 2-bit values, 8-dim VQ blocks, 3/4-bit scalar keys");
    if (a.page_size % 16) return fail(SMAQ_ERR_INVALID, "decode layout needs page_size %% 16 == 0");
  }
  if (a.v) {
    if (a.value_bits != 2 && a.value_bits != 4)
      return fail(SMAQ_ERR_INVALID, "values: bits %d not in {2,4}", a.value_bits);
    if (a.group_size <= 0 || a.head_dim % a.group_size)
      return fail(SMAQ_ERR_INVALID, "head_dim %d must be divisible by group_size %d", a.head_dim, a.group_size);
    const int lpg = a.group_size / (epl ? epl : 1);
    if (a.group_size % (epl ? epl : 1) || (lpg & (lpg - 1)) || lpg < 1 || lpg > 32)
      return fail(SMAQ_ERR_UNSUPPORTED, "values: group_size %d with head_dim %d", a.group_size, a.head_dim);
    if (!a.v_data || !a.v_scales || !a.v_zeros) return fail(SMAQ_ERR_INVALID, "values: null output");
    if ((reinterpret_cast<uintptr_t>(a.v) % (es * epl)) || (a.v_stride_t % epl) || (a.v_stride_h % epl))
      return fail(SMAQ_ERR_INVALID, "values: input must be aligned to %d elements", epl);
  }
  if (a.k) {
    if ((reinterpret_cast<uintptr_t>(a.k) % (es * epl)) || (a.k_stride_t % epl) || (a.k_stride_h % epl))
      return fail(SMAQ_ERR_INVALID, "keys: input must be aligned to %d elements", epl);
    if (a.key_format == SMAQ_KEYS_SCALAR) {
      if (a.key_bits < 2 || a.key_bits > 4) return fail(SMAQ_ERR_UNSUPPORTED, "scalar keys: bits %d", a.key_bits);
      if (!a.E || !a.boundaries || !a.key_codes || !a.key_norms)
        return fail(SMAQ_ERR_INVALID, "scalar keys: null table or output");
    } else if (a.key_format == SMAQ_KEYS_BVQ) {
      if (a.block_dim != 8) return fail(SMAQ_ERR_UNSUPPORTED, "bvq: block_dim %d (only 8)", a.block_dim);
      if (a.n_centroids < 1 || a.n_centroids > 256)
        return fail(SMAQ_ERR_UNSUPPORTED, "bvq: n_centroids %d not in [1,256]", a.n_centroids);
      if (!a.E_blocks || !a.centroids || !a.key_codes) return fail(SMAQ_ERR_INVALID, "bvq: null table or output");
    } else {
      return fail(SMAQ_ERR_INVALID, "keys given with key_format %d", a.key_format);
    }
  }
  return SMAQ_OK;
}

}  // namespace smaq

using namespace smaq;

extern "C" int smaq_append(const smaq_append_args* args, void* stream) {
  if (!args) return fail(SMAQ_ERR_INVALID, "append: null args");
  const smaq_append_args& a = *args;
  int st = validate_append(a);
  if (st) return st;
  if (a.n_tokens == 0) return SMAQ_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // keys first: the value kernel may then run beside the (compute-bound) key kernel
  if (a.k) {
    if (a.key_format == SMAQ_KEYS_SCALAR)
      st = by_dtype<RunScalar>(a.dtype, a, s);
    else
      st = by_dtype<RunBvq>(a.dtype, a, s);
    if (st) return st;
  }
  if (a.v) st = by_dtype<RunValues>(a.dtype, a, s, a.k ? 1 : 0);
  return st;
}

extern "C" int smaq_quantize_keys_scalar(const void* k, int dtype, int64_t n_rows, int head_dim,
                                         const float* E, const float* boundaries, int bits,
                                         uint8_t* codes_out, void* norms_out, void* stream) {
  smaq_append_args a = {};
  a.k = k;
  a.dtype = dtype;
  a.n_tokens = n_rows;
  a.n_heads = 1;
  a.head_dim = head_dim;
  a.k_stride_t = head_dim;
  a.page_size = n_rows > 0 ? n_rows : 1;
  a.key_format = SMAQ_KEYS_SCALAR;
  a.key_bits = bits;
  a.E = E;
  a.boundaries = boundaries;
  a.key_codes = codes_out;
  a.key_norms = norms_out;
  return smaq_append(&a, stream);
}

extern "C" int smaq_quantize_values(const void* v, int dtype, int64_t n_rows, int head_dim, int bits,
                                    int group_size, uint8_t* data_out, void* scales_out, void* zeros_out,
                                    void* stream) {
  smaq_append_args a = {};
  a.v = v;
  a.dtype = dtype;
  a.n_tokens = n_rows;
  a.n_heads = 1;
  a.head_dim = head_dim;
  a.v_stride_t = head_dim;
  a.page_size = n_rows > 0 ? n_rows : 1;
  a.value_bits = bits;
  a.group_size = group_size;
  a.v_data = data_out;
  a.v_scales = scales_out;
  a.v_zeros = zeros_out;
  return smaq_append(&a, stream);
}

extern "C" int smaq_quantize_keys_bvq(const void* k, int dtype, int64_t n_rows, int head_dim,
                                      const float* E_blocks, const float* centroids, int block_dim,
                                      int n_centroids, uint8_t* idx_out, void* stream) {
  smaq_append_args a = {};
  a.k = k;
  a.dtype = dtype;
  a.n_tokens = n_rows;
  a.n_heads = 1;
  a.head_dim = head_dim;
  a.k_stride_t = head_dim;
  a.page_size = n_rows > 0 ? n_rows : 1;
  a.key_format = SMAQ_KEYS_BVQ;
  a.E_blocks = E_blocks;
  a.centroids = centroids;
  a.block_dim = block_dim;
  a.n_centroids = n_centroids;
  a.key_codes = idx_out;
  return smaq_append(&a, stream);
}
