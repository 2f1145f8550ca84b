// tcgen05 path for scalar metric-aware key codes of bf16 keys at head_dim 128.
//
// Reference: SMAQQuantizer.quantize (smaq/quantizer.py:138-145) + _pack_indices (:34-46):
//   norms = k.norm(-1); k_unit = k / (norms + 1e-10); y = k_unit.float() @ E.T;
//   idx = searchsorted(decision_boundaries, y); pack LSB-first.
//
// The d x d contraction runs on the 5th-generation tensor cores in split precision.  k_unit is
// a bf16 tensor, so it is exact as the A operand.  E is fp32; it is split into three bf16
// matrices E = E_hi + E_mid + E_lo (each the bf16 rounding of what the previous ones leave),
// which holds E to ~2^-27 relative, and the three products accumulate in one fp32 TMEM
// accumulator: y = A E_lo^T + A E_mid^T + A E_hi^T.  The result agrees with the reference's fp32
// matmul up to fp32 accumulation-order differences, the band the SIMT kernel has as well.
//
// Persistent kernel, one CTA per SM, 128 token-head rows per tile, warp-specialised:
//   warp 16       TMA: two 3-D tensor loads (d 0..63, 64..127) of 128 rows into a shared-memory
//                 stage (128-byte swizzled);
//   warps 0-7     warp w holds rows 32 (w % 4) + lane, half w / 4 of each row: norm (in the SIMT
//                 kernel's summation order, halves exchanged through shared memory), k_unit
//                 (bf16) written to a TMEM A buffer with tcgen05.st, norm written out;
//   warp 17       one thread issues 3 x 8 tcgen05.mma (M=128, N=128, K=16, A from TMEM, B = E
//                 splits from shared memory) per tile into one of two TMEM accumulators;
//   warps 8-15    epilogue: tcgen05.ld of a 32-row x 64-column quarter-half each, searchsorted
//                 against the boundaries (table lookup), pack, 16-byte stores of the code row.
// TMEM columns: accumulators [0,128) and [128,256), A buffers [256,320) and [320,384).
// Every mbarrier wait is bounded; a wait that runs out sets g_tc_rotate_fault and the CTA drains.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "ptx.cuh"
#include "tc_rotate.cuh"

namespace smaq {

namespace {

constexpr int TR_ROWS = 128;                  // rows per tile (= UMMA M, = TMEM lanes)
constexpr int TR_D = 128;                     // head_dim (= UMMA N = K)
constexpr int TR_STAGES = 3;                  // raw key ring depth
constexpr int TR_ATOM = TR_ROWS * 128;        // one 64-wide K atom of a 128-row operand: 16 KiB
constexpr int TR_TILE = 2 * TR_ATOM;          // 32 KiB per 128 x 128 16-bit operand
constexpr int TR_B_BYTES = 3 * TR_TILE;       // E_hi, E_mid, E_lo
constexpr int TR_LUT = 256;                   // searchsorted table entries
constexpr int TR_XCH_BYTES = 2 * TR_ROWS * 2 * 32;  // norm partial-sum exchange, double-buffered
constexpr int TR_SMEM = TR_B_BYTES + TR_STAGES * TR_TILE + TR_XCH_BYTES + TR_LUT * 8 + 256 + 1024;
constexpr int TR_NORM_WARPS = 8, TR_EPI_WARPS = 8;
constexpr int TR_TMA_WARP = TR_NORM_WARPS + TR_EPI_WARPS;  // 16
constexpr int TR_MMA_WARP = TR_TMA_WARP + 1;               // 17
constexpr int TR_THREADS = (TR_MMA_WARP + 1) * 32;         // 576
constexpr uint32_t TR_TMEM_COLS = 512;
constexpr uint32_t TR_TMEM_A = 256;                        // first A-buffer column

__device__ unsigned int g_tc_rotate_fault;

struct TrBars {
  uint64_t a_full[TR_STAGES];   // TMA bytes landed
  uint64_t a_empty[TR_STAGES];  // raw stage read (256 arrivals)
  uint64_t at_ready[2];         // TMEM A buffer written (256 arrivals)
  uint64_t at_free[2];          // MMAs that read the A buffer finished (tcgen05.commit)
  uint64_t acc_full[2];         // accumulator complete (tcgen05.commit)
  uint64_t acc_empty[2];        // accumulator drained (256 arrivals)
  uint32_t tmem_base;
};

// ---------------------------------------------------------------- PTX wrappers
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void named_bar(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// UMMA shared-memory descriptor: K-major, SWIZZLE_128B, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  return uint64_t((saddr & 0x3FFFFu) >> 4) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// kind::f16 instruction descriptor: bf16 x bf16 -> f32, both K-major, M = 128, N = 128.
constexpr uint32_t kIdescBf16 = (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(TR_D >> 3) << 17) |
                                (uint32_t(TR_ROWS >> 4) << 24);

// D (TMEM) (+)= A (TMEM) * B (shared memory)^T
__device__ __forceinline__ void umma_bf16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(db), "r"(kIdescBf16), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Byte offset of the 16-byte chunk holding elements [8c, 8c+8) of row r in a 128-row
// K-major SWIZZLE_128B operand (two 64-element atoms of 128-byte rows, chunk index XOR row%8).
__device__ __forceinline__ uint32_t sw128_chunk(int r, int c) {
  return uint32_t((c >> 3) * TR_ATOM + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// Packed fp32 pairs (one instruction for two independent IEEE operations, same rounding as two
// scalar ones).
__device__ __forceinline__ uint64_t f32x2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float2 f32x2_split(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t mul_f32x2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// k_unit elements are bf16(fp32 x / den) with x and den bf16.  They are computed as
// x * (1/den), within 2^-22 relative of the exact quotient.  A quotient of two bf16 values is
// never exactly a bf16 rounding midpoint (X * 2^p = m * Dn has no solution with X, Dn 8-bit
// significands and m an odd 9-bit integer: the odd part of the left side is at most 255), and
// when it is not, it is at least 1 / (511 * 255) > 2^-17 relative away from every midpoint.
// So x * (1/den) rounds to the same bf16 value as the correctly rounded fp32 quotient.  The one
// exception is a quotient below 2^-126 (an fp32 subnormal product), where the element may be off
// by 2^-149; its contribution to y is far below the fp32 rounding band of the contraction.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// 0xFFFFFFFF when x > b or x is NaN (searchsorted places NaN after every boundary), else 0.
__device__ __forceinline__ uint32_t gtu_mask(float x, float b) {
  uint32_t r;
  asm("set.gtu.u32.f32 %0, %1, %2;" : "=r"(r) : "f"(x), "f"(b));
  return r;
}
// 0xFFFFFFFF when x > b (ordered: NaN gives 0), else 0.
__device__ __forceinline__ uint32_t gt_mask(float x, float b) {
  uint32_t r;
  asm("set.gt.u32.f32 %0, %1, %2;" : "=r"(r) : "f"(x), "f"(b));
  return r;
}
__device__ __forceinline__ float fma_sat(float a, float b, float c) {
  float r;
  asm("fma.rn.sat.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// searchsorted over the decision boundaries by table lookup.  A uniform grid of step
// gap_min / 3 runs from hi = b_last + 2 step down to lo <= b_0 - 2 step (G <= 254 cells).
// For a value x, k = round(G * sat((hi - x) / (G step))) differs from the cell holding x by at
// most one, so x lies in the window (hi - (k+1) step, hi - (k-1) step] (extended to +inf for
// k = 0 and -inf for k = G).  Entry k holds base = #{b <= window start - step/4} and the single
// boundary t in the window widened by step/4 on each side (+inf if none; the widened window is
// 2.5 steps < gap_min long), so code(x) = #{b < x} = base + (x > t).  NaN gives k = 0, whose
// entry is (NB, +inf): NaN sorts after every boundary, as searchsorted places it.  An entry is
// the 8-byte pair (t bits, base), read by one shared load.
struct SearchGrid {
  float neg_inv_span, c0, g, step, hi;
  int G;
  bool ok;
};
template <int NB>
__device__ __forceinline__ SearchGrid search_grid(const float* __restrict__ bnd, float sc) {
  SearchGrid sg;
  sg.ok = false;
  float gap = INFINITY;
#pragma unroll
  for (int j = 0; j + 1 < NB; ++j) gap = fminf(gap, __ldg(bnd + j + 1) * sc - __ldg(bnd + j) * sc);
  const float b0 = __ldg(bnd) * sc, bl = __ldg(bnd + NB - 1) * sc;
  if (NB == 1) gap = fmaxf(fabsf(b0), sc);
  if (!(gap > 0.f) || !(gap < INFINITY) || !(fabsf(b0) < INFINITY) || !(fabsf(bl) < INFINITY)) return sg;
  sg.step = gap / 3.0f;
  sg.hi = bl + 2.0f * sg.step;
  const float Gf = ceilf((sg.hi - (b0 - 2.0f * sg.step)) / sg.step);
  if (!(Gf <= float(TR_LUT - 2))) return sg;
  sg.G = int(Gf);
  const float span = Gf * sg.step;
  sg.neg_inv_span = -1.0f / span;
  sg.c0 = sg.hi / span;
  sg.g = Gf;
  sg.ok = true;
  return sg;
}
template <int NB>
__device__ __forceinline__ void search_entry(const float* __restrict__ bnd, float sc, const SearchGrid& sg, int k,
                                             uint2* lut) {
  const float eps = 0.25f * sg.step;
  const float lo_w = sg.hi - float(k + 1) * sg.step - eps, hi_w = sg.hi - float(k - 1) * sg.step + eps;
  uint32_t base = 0;
  float t = INFINITY;
#pragma unroll
  for (int j = 0; j < NB; ++j) {
    const float b = __ldg(bnd + j) * sc;
    if (b <= lo_w) ++base;
    else if (b <= hi_w || k == 0) t = b;
  }
  lut[k] = make_uint2(__float_as_uint(t), base);
}
// Shared address of entry k is lut + 8k.  f = 2^23 + k exactly (k in [0, G]), whose bits are
// 0x4B000000 + k, so the address is lut_adj + 8 * bits(f) in 32-bit arithmetic with
// lut_adj = lut - 8 * 0x4B000000 (mod 2^32): the subtraction of the exponent bits folds into
// the table base.
__device__ __forceinline__ uint32_t lut_base_adj(const uint2* lut) { return smem_u32(lut) - (0x4B000000u << 3); }
__device__ __forceinline__ uint32_t search_lut(float x, const SearchGrid& sg, uint32_t lut_adj) {
  const float f = fmaf(fma_sat(x, sg.neg_inv_span, sg.c0), sg.g, 8388608.0f);
  const uint32_t addr = lut_adj + (__float_as_uint(f) << 3);
  uint32_t t, b;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(t), "=r"(b) : "r"(addr));
  return b - gt_mask(x, __uint_as_float(t));
}

// Codes of 32 consecutive coordinates, packed LSB-first (2-bit: 4 per byte, 3/4-bit: 2 per
// byte) into 32 * BITS' / 8 bytes, BITS' = 2 or 4.
template <int BITS, bool LUT>
__device__ __forceinline__ void encode32(const float (&y)[32], uint32_t* w, const SearchGrid& sg, uint32_t lut_adj,
                                         const float* __restrict__ bnd, float sc) {
  constexpr int NB = (1 << BITS) - 1;
  constexpr int VPB = BITS == 2 ? 4 : 2;
#pragma unroll
  for (int k = 0; k < 32 / (4 * VPB); ++k) {
    uint32_t v = 0;
#pragma unroll
    for (int u = 0; u < 4 * VPB; ++u) {
      const float x = y[4 * VPB * k + u];
      uint32_t c;
      if constexpr (LUT) {
        c = search_lut(x, sg, lut_adj);
      } else {  // degenerate boundaries: count them (>u puts NaN after every boundary)
        c = 0;
#pragma unroll
        for (int j = 0; j < NB; ++j) c -= gtu_mask(x, __ldg(bnd + j) * sc);
      }
      v += c << ((u / VPB) * 8 + (u % VPB) * BITS);
    }
    w[k] = v;
  }
}

// ---------------------------------------------------------------- kernel
template <int BITS>
__global__ void __launch_bounds__(TR_THREADS, 1) tc_scalar_key_kernel(
    const __grid_constant__ CUtensorMap kmap, int64_t n_tokens, int n_heads, const RowMap rm,
    const float* __restrict__ E, const float* __restrict__ bnd, uint8_t* __restrict__ codes,
    __nv_bfloat16* __restrict__ norms, int layout) {
  constexpr int NB = (1 << BITS) - 1;
  constexpr int VPB = BITS == 2 ? 4 : 2;      // codes per byte (3-bit packs two per byte)
  constexpr int PD = TR_D / VPB;              // bytes per code row
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* Bs = smem;                                          // [2 splits][2 atoms][128 rows][128 B]
  uint8_t* Rs = smem + TR_B_BYTES;                             // [STAGES][2 atoms][128 rows][128 B]
  float* xch = reinterpret_cast<float*>(Rs + TR_STAGES * TR_TILE);  // [2][128 rows][2 halves][8]
  uint2* lut = reinterpret_cast<uint2*>(xch + TR_XCH_BYTES / 4);  // [TR_LUT] (t bits, base)
  TrBars* bars = reinterpret_cast<TrBars*>(lut + TR_LUT);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n_rows = n_tokens * n_heads;
  const int tok_per_tile = TR_ROWS / n_heads;
  // the append's value kernel (launched next, as a programmatic dependent) may start beside us
  pdl_launch_dependents();
  const int64_t n_tiles = (n_tokens + tok_per_tile - 1) / tok_per_tile;

  // ---- E = E_hi + E_mid + E_lo in bf16 (each the bf16 rounding of what the previous ones
  // leave), written in the swizzled B layout (row n = E[n, :])
  const float sc = 1.0f;  // boundaries in the accumulator's units
  for (int idx = threadIdx.x; idx < TR_D * (TR_D / 8); idx += blockDim.x) {
    const int n = idx >> 4, c = idx & 15;
    const float4 e0 = __ldg(reinterpret_cast<const float4*>(E + n * TR_D + c * 8));
    const float4 e1 = __ldg(reinterpret_cast<const float4*>(E + n * TR_D + c * 8 + 4));
    const float ev[8] = {e0.x, e0.y, e0.z, e0.w, e1.x, e1.y, e1.z, e1.w};
    uint32_t w[3][4];
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      float r0 = ev[j], r1 = ev[j + 1];
#pragma unroll
      for (int sp = 0; sp < 3; ++sp) {
        const uint32_t h = pack_bf16x2(r0, r1);
        w[sp][j / 2] = h;
        r0 -= bf_lo(h);
        r1 -= bf_hi(h);
      }
    }
#pragma unroll
    for (int sp = 0; sp < 3; ++sp)
      *reinterpret_cast<uint4*>(Bs + sp * TR_TILE + sw128_chunk(n, c)) = make_uint4(w[sp][0], w[sp][1], w[sp][2], w[sp][3]);
  }
  const SearchGrid sgrid = search_grid<NB>(bnd, sc);
  if (sgrid.ok)
    for (int k = threadIdx.x; k <= sgrid.G; k += blockDim.x) search_entry<NB>(bnd, sc, sgrid, k, lut);
  fence_async_smem();
  if (threadIdx.x == 0) {
    for (int s = 0; s < TR_STAGES; ++s) {
      mbar_init(&bars->a_full[s], 1);
      mbar_init(&bars->a_empty[s], TR_NORM_WARPS * 32);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->at_ready[b], TR_NORM_WARPS * 32);
      mbar_init(&bars->at_free[b], 1);
      mbar_init(&bars->acc_full[b], 1);
      mbar_init(&bars->acc_empty[b], TR_EPI_WARPS * 32);
    }
    fence_mbar_init();
  }
  if (warp == TR_TMA_WARP) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&bars->tmem_base)),
                 "r"(TR_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  bool failed = false;

  if (warp == TR_TMA_WARP) {
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&kmap)) : "memory");
      int i = 0;
      for (int64_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++i) {
        const int s = i % TR_STAGES;
        if (!mbar_wait(&bars->a_empty[s], ((i / TR_STAGES) & 1) ^ 1)) { failed = true; break; }
        mbar_arrive_expect_tx(&bars->a_full[s], TR_TILE);
        uint8_t* dst = Rs + s * TR_TILE;
        const int z = int(tile * tok_per_tile);
        tma_load_3d(dst, &kmap, 0, 0, z, &bars->a_full[s]);
        tma_load_3d(dst + TR_ATOM, &kmap, 64, 0, z, &bars->a_full[s]);
      }
    }
  } else if (warp < TR_NORM_WARPS) {
    // ---- k_unit = k / (norm + 1e-10).  Thread (warp w, lane) holds row t = 32 (w % 4) + lane
    // (its TMEM lane) and half hf = w / 4, which owns chunks {4hf..4hf+3, 8+4hf..8+4hf+3}, i.e.
    // the 4-element partial sums of SIMT lanes {8hf..8hf+7, 16+8hf..16+8hf+7}: the first level of
    // the warp_sum tree (lanes 16 apart) stays inside a thread, the second (8 apart) pairs the
    // two halves, whose warps swap 8 sums through shared memory.
    const int q = warp & 3, hf = warp >> 2;
    const int t = 32 * q + lane;
    int i = 0;
    for (int64_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++i) {
      const int s = i % TR_STAGES, ab = i & 1;
      if (!mbar_wait(&bars->a_full[s], (i / TR_STAGES) & 1)) { failed = true; break; }
      const uint8_t* R = Rs + s * TR_TILE;
      uint4 raw[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) raw[j] = *reinterpret_cast<const uint4*>(R + sw128_chunk(t, (j < 4 ? j : j + 4) + 4 * hf));
      // the stage may be refilled once every row is in registers; the refill is an async-proxy
      // (TMA) write, so the generic-proxy reads above are ordered before it by a proxy fence
      fence_async_smem();
      mbar_arrive(&bars->a_empty[s]);
      // sum of squares in the SIMT kernel's order: partials of 4 elements (fma chain) per SIMT
      // lane, then the xor-butterfly tree of warp_sum (lanes 16 apart, then 8, 4, 2, 1)
      float p[16];  // p[j] = partial of SIMT lane (j < 8 ? 8hf + j : 16 + 8hf + j - 8)
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t w[4] = {raw[j].x, raw[j].y, raw[j].z, raw[j].w};
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          float a = 0.f;
          a = fmaf(bf_lo(w[2 * hh]), bf_lo(w[2 * hh]), a);
          a = fmaf(bf_hi(w[2 * hh]), bf_hi(w[2 * hh]), a);
          a = fmaf(bf_lo(w[2 * hh + 1]), bf_lo(w[2 * hh + 1]), a);
          a = fmaf(bf_hi(w[2 * hh + 1]), bf_hi(w[2 * hh + 1]), a);
          p[2 * (j & 3) + hh + 8 * (j >> 2)] = a;
        }
      }
      // level 16: SIMT lane l (< 16) = p_l + p_{l+16}; this thread holds lanes 8hf + m, m < 8
      float s1[8];
#pragma unroll
      for (int m = 0; m < 8; ++m) s1[m] = p[m] + p[m + 8];
      float* mine = xch + ((ab * TR_ROWS + t) * 2 + hf) * 8;
      float* other = xch + ((ab * TR_ROWS + t) * 2 + (hf ^ 1)) * 8;
      reinterpret_cast<float4*>(mine)[0] = make_float4(s1[0], s1[1], s1[2], s1[3]);
      reinterpret_cast<float4*>(mine)[1] = make_float4(s1[4], s1[5], s1[6], s1[7]);
      named_bar(1 + q, 64);  // warps q and q + 4
      const float4 o0 = reinterpret_cast<const float4*>(other)[0], o1 = reinterpret_cast<const float4*>(other)[1];
      const float o[8] = {o0.x, o0.y, o0.z, o0.w, o1.x, o1.y, o1.z, o1.w};
      // level 8: lane m (< 8) = lane m + lane m + 8 (half 0 holds lanes 0..7, half 1 lanes 8..15)
      float s2[8];
#pragma unroll
      for (int m = 0; m < 8; ++m) s2[m] = hf ? o[m] + s1[m] : s1[m] + o[m];
#pragma unroll
      for (int oo = 4; oo > 0; oo >>= 1)
#pragma unroll
        for (int l = 0; l < oo; ++l) s2[l] = s2[l] + s2[l + oo];
      const float nrm = rnd<BF16>(sqrtf(s2[0]));
      const float den = rnd<BF16>(nrm + 1e-10f);
      const float rcp = __frcp_rn(den);
      // k_unit in bf16 (the reference's storage type); column j of the A buffer holds elements
      // 2j, 2j+1
      uint32_t cols[2][16];
      const uint64_t rcp2 = f32x2(rcp, rcp);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t w[4] = {raw[j].x, raw[j].y, raw[j].z, raw[j].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 u = f32x2_split(mul_f32x2(f32x2(bf_lo(w[e]), bf_hi(w[e])), rcp2));
          cols[j >> 2][(j & 3) * 4 + e] = pack_bf16x2(u.x, u.y);
        }
      }
      if (!mbar_wait(&bars->at_free[ab], ((i >> 1) & 1) ^ 1)) { failed = true; break; }
      tc_fence_after();
      const uint32_t ta = tmem + (uint32_t(32 * q) << 16) + TR_TMEM_A + uint32_t(ab * 64 + 16 * hf);
      tmem_st16(ta, cols[0]);        // elements 32hf .. 32hf+31
      tmem_st16(ta + 32, cols[1]);   // elements 64+32hf .. 64+32hf+31
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&bars->at_ready[ab]);
      const int64_t r = tile * TR_ROWS + t;
      if (hf == 0 && r < n_rows) {
        int64_t tok;
        int h;
        rm.token_head(r, tok, h);
        norms[rm.row(tok, h)] = __float2bfloat16_rn(nrm);
      }
    }
  } else if (warp == TR_MMA_WARP) {
    if (lane == 0) {
      const uint32_t b0 = smem_u32(Bs);
      int i = 0;
      for (int64_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++i) {
        const int ab = i & 1;
        if (!mbar_wait(&bars->at_ready[ab], (i >> 1) & 1)) { failed = true; break; }
        if (!mbar_wait(&bars->acc_empty[ab], ((i >> 1) & 1) ^ 1)) { failed = true; break; }
        tc_fence_after();
        const uint32_t d = tmem + uint32_t(ab * TR_D);
        const uint32_t a = tmem + TR_TMEM_A + uint32_t(ab * 64);
        uint32_t acc = 0;
#pragma unroll
        for (int sp = 2; sp >= 0; --sp) {  // smaller terms first
#pragma unroll
          for (int ks = 0; ks < TR_D / 16; ++ks) {
            const uint32_t off = uint32_t((ks >> 2) * TR_ATOM + (ks & 3) * 32);
            umma_bf16_ts(d, a + uint32_t(ks * 8), umma_desc_sw128(b0 + sp * TR_TILE + off), acc);
            acc = 1;
          }
        }
        umma_commit(&bars->at_free[ab]);
        umma_commit(&bars->acc_full[ab]);
      }
    }
  } else {
    // ---- epilogue: warp (8 + q + 4 * half) reads TMEM lanes 32q.. and columns 64 half..
    const int ew = warp - TR_NORM_WARPS;
    const int q = warp & 3, half = ew >> 2;
    const int t = 32 * q + lane;
    int i = 0;
    for (int64_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++i) {
      const int ab = i & 1;
      if (!mbar_wait(&bars->acc_full[ab], (i >> 1) & 1)) { failed = true; break; }
      tc_fence_after();
      // searchsorted(decision_boundaries, y), right=False, 32 columns at a time
      uint32_t w[PD / 8];  // this half's PD/2 bytes as words, codes LSB-first
      const uint32_t taddr = tmem + (uint32_t(32 * q) << 16) + uint32_t(ab * TR_D + half * 64);
#pragma unroll
      for (int part = 0; part < 2; ++part) {
        float y[32];
        tmem_ld32(taddr + 32 * part, y);
        tmem_ld_wait();
        if (part == 1) {
          tc_fence_before();
          mbar_arrive(&bars->acc_empty[ab]);
        }
        if (sgrid.ok)
          encode32<BITS, true>(y, w + part * (PD / 16), sgrid, lut_base_adj(lut), bnd, sc);
        else
          encode32<BITS, false>(y, w + part * (PD / 16), sgrid, 0u, bnd, sc);
      }
      const int64_t r = tile * TR_ROWS + t;
      if (r >= n_rows) continue;
      int64_t tok;
      int h;
      rm.token_head(r, tok, h);
      uint8_t* crow = codes + rm.row(tok, h) * PD;
      if (BITS != 2 && layout == SMAQ_LAYOUT_DECODE) {
        // decode layout: reference byte p at 16 (p % 4) + p / 4, i.e. byte t of this half's
        // word i goes to 16 t + 8 half + i
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const uint32_t sel = uint32_t(t) | (uint32_t(t + 4) << 4);
          const uint32_t lo = __byte_perm(__byte_perm(w[0], w[1], sel), __byte_perm(w[2], w[3], sel), 0x5410);
          const uint32_t hi = __byte_perm(__byte_perm(w[4 % (PD / 8)], w[5 % (PD / 8)], sel),
                                          __byte_perm(w[6 % (PD / 8)], w[7 % (PD / 8)], sel), 0x5410);
          *reinterpret_cast<uint2*>(crow + 16 * t + 8 * half) = make_uint2(lo, hi);
        }
      } else {
        uint4* dst = reinterpret_cast<uint4*>(crow + half * (PD / 2));
#pragma unroll
        for (int k = 0; k < PD / 32; ++k) dst[k] = make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
      }
    }
  }
  if (failed) atomicOr(&g_tc_rotate_fault, 1u);
  tc_fence_before();
  __syncthreads();
  if (warp == TR_TMA_WARP) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TR_TMEM_COLS) : "memory");
  }
}

// ---------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

}  // namespace

bool tc_rotate_eligible(const smaq_append_args& a) {
  if (a.dtype != SMAQ_BF16 || a.head_dim != TR_D || a.key_format != SMAQ_KEYS_SCALAR) return false;
  if (a.n_heads <= 0 || a.n_heads > TR_ROWS || TR_ROWS % a.n_heads) return false;
  if (reinterpret_cast<uintptr_t>(a.k) % 16 || reinterpret_cast<uintptr_t>(a.key_codes) % 16) return false;
  if (a.k_stride_h % 8 || a.k_stride_t % 8 || a.k_stride_h <= 0 || a.k_stride_t <= 0) return false;
  if (reinterpret_cast<uintptr_t>(a.E) % 16) return false;
  if (a.n_tokens > (int64_t(1) << 31) - TR_ROWS) return false;
  return encode_fn() != nullptr;
}

template <int BITS>
static int launch_bits(const smaq_append_args& a, const CUtensorMap& map, cudaStream_t s) {
  auto kern = tc_scalar_key_kernel<BITS>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, TR_SMEM);
  if (e != cudaSuccess) return cuda_status(e, "tc_scalar_key_kernel attr");
  const int tok_per_tile = TR_ROWS / a.n_heads;
  const int64_t tiles = (a.n_tokens + tok_per_tile - 1) / tok_per_tile;
  const int grid = int(tiles < num_sms() ? tiles : num_sms());
  kern<<<grid, TR_THREADS, TR_SMEM, s>>>(map, a.n_tokens, a.n_heads, make_rowmap(a), a.E,
                                         a.boundaries, a.key_codes, static_cast<__nv_bfloat16*>(a.key_norms), a.layout);
  return cuda_status(cudaGetLastError(), "tc_scalar_key_kernel");
}

int launch_scalar_keys_tc(const smaq_append_args& a, cudaStream_t s) {
  if (a.n_tokens == 0) return SMAQ_OK;
  CUtensorMap map;
  const cuuint64_t dims[3] = {cuuint64_t(TR_D), cuuint64_t(a.n_heads), cuuint64_t(a.n_tokens)};
  const cuuint64_t strides[2] = {cuuint64_t(a.k_stride_h) * 2, cuuint64_t(a.k_stride_t) * 2};
  const cuuint32_t box[3] = {64u, cuuint32_t(a.n_heads), cuuint32_t(TR_ROWS / a.n_heads)};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  const CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(a.k), dims, strides, box,
                                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SMAQ_ERR_INVALID, "keys: cuTensorMapEncodeTiled failed (%d)", int(r));
  switch (a.key_bits) {
    case 2: return launch_bits<2>(a, map, s);
    case 3: return launch_bits<3>(a, map, s);
    case 4: return launch_bits<4>(a, map, s);
  }
  return fail(SMAQ_ERR_UNSUPPORTED, "scalar keys: bits %d not in {2,3,4}", a.key_bits);
}

}  // namespace smaq

extern "C" int smaq_append_status(void* stream) {
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return smaq::cuda_status(e, "append status: stream");
  unsigned int word = 0, zero = 0;
  e = cudaMemcpyFromSymbol(&word, smaq::g_tc_rotate_fault, sizeof(word));
  if (e == cudaSuccess && word) e = cudaMemcpyToSymbol(smaq::g_tc_rotate_fault, &zero, sizeof(zero));
  if (e != cudaSuccess) return smaq::cuda_status(e, "append status: read");
  if (word) return smaq::fail(SMAQ_ERR_DEVICE, "append: a bounded device wait in the key kernel ran out");
  return SMAQ_OK;
}
