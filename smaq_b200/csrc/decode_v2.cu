// Fast hybrid decode for block-VQ keys (sm_100a): TMA-staged streams, shared-memory score
// tables, tensor-core P.V.
//
// Reference semantics: compute_hybrid_attention (smaq/score.py:23-72) with SMAQBlockVQ scores
// q . decoded_centroid[idx] * scale (smaq/block_vq.py:246-297) and 2-bit group-32 values
// dequantized as code * scale + zero (smaq/kv_cache.py:94-103).  Same work partition, partial
// slots and merge as the general kernel in decode.cu.
//
// Per CTA: WARPS warps, each streaming its own 32-token chunks of one (sequence, kv head)
// segment.
//  * Staging: lane 0 of each warp issues 1-D bulk async copies (TMA engine, no multicast) of a
//    chunk's index / value-code / scale / zero rows into a private STAGES-deep ring; an
//    mbarrier counts the bytes.  Rows use SMAQ_LAYOUT_DECODE (include/smaq_b200.h).
//  * Scores: LUT[c][b][g] = log2(e) * scale * (q_g[8b:8b+8] . decoded_centroid[b][c]) lives in
//    shared memory laid out [head/4][c][b][head%4]: the 32 lanes of a warp, mapped to
//    (head%4, b%8), hit 32 distinct banks whatever the indices are.  One 16-byte load gives a
//    lane the (b, b+8) index pair of eight tokens in an order XOR-swizzled by b%8, so the
//    eight per-lane partial sums are reduce-scattered across the 8 block lanes with 7 shuffles
//    and no selects.  Scores come out in the log2 domain (p = exp2(s - m)).
//  * Online softmax per head over each chunk; the score lane of (token, head) also forms the
//    P.V weights w = p * value_scale of the token's 4 value groups, as fp16, in shared memory.
//  * P.V on the tensor cores with mma.m16n8k16 (fp16 in, fp32 accumulate): A = value codes as
//    exact fp16 subnormals -- the 2-bit field of code r of a byte sits at mantissa bits 2r,
//    so one AND yields code * 4^r * 2^-24 with no unpacking -- and B = w.  The epilogue
//    multiplies by 2^24 / 4^r; sum_t p_t * zero_t is accumulated on the CUDA cores.  Rows of
//    the MMA are value dimensions ordered so that each thread's operand bits come from ONE
//    32-bit word per token.
#include <math.h>

#include "common.cuh"
#include "decode_common.cuh"
#include "ptx.cuh"

namespace smaq {

constexpr int CH = 32;  // tokens per chunk
constexpr int ST_IDX = 0, ST_V = CH * 16, ST_S = CH * 48, ST_Z = CH * 56, STAGE_BYTES = CH * 64;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

template <int NP>
struct V2Cfg {
  static constexpr int G4 = 4 * NP;
  static constexpr int WARPS = NP == 1 ? 16 : 12;
  static constexpr int THREADS = WARPS * 32;
  static constexpr int STAGES = NP == 1 ? 3 : 2;
  static constexpr int LUT_BYTES = NP * 256 * 16 * 4 * 4;
  static constexpr int Q_BYTES = G4 * 128 * 4;
  static constexpr int WB_GSTRIDE = 68;                         // words per head in wbuf (padded)
  static constexpr int WB_BYTES = G4 * WB_GSTRIDE * 4;          // fp16 weights [g][j][ks][slot]
  static constexpr int WARP_BYTES = STAGES * STAGE_BYTES + WB_BYTES + 256;  // ring | wbuf | alpha, z
  static constexpr int BAR_BYTES = WARPS * STAGES * 8;
  static constexpr int SMEM = LUT_BYTES + Q_BYTES + WARPS * WARP_BYTES + BAR_BYTES;
  static constexpr int RED_FLOATS = G4 * (128 + 2);            // per-warp merge record
  static_assert(RED_FLOATS * 4 <= STAGES * STAGE_BYTES + WB_BYTES, "merge record must fit");
  static_assert(SMEM <= 232448, "shared memory budget");
};

__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Issue the bulk copies of chunk `kc` of a history segment into `stage`.
__device__ __forceinline__ void v2_issue(const DecodeParams& p, int b, int h, int64_t t0, int64_t t1, int kc,
                                         uint8_t* stage, uint64_t* bar) {
  const int64_t tc = t0 + int64_t(kc) * CH;
  int64_t nv = t1 - tc;
  if (nv > CH) nv = CH;
  const int64_t ncopy = (nv + 15) & ~int64_t(15);
  mbar_arrive_expect_tx(bar, uint32_t(ncopy * 64));
  const int64_t ps = p.page_size;
  int64_t t = tc, done = 0;
  while (done < ncopy) {
    const int64_t pg = t / ps;
    const int64_t off = t - pg * ps;
    int64_t len = ps - off;
    if (len > ncopy - done) len = ncopy - done;
    const int64_t page = p.bt ? int64_t(p.bt[b * p.bt_stride + pg]) : int64_t(b);
    const int64_t row0 = (page * p.Hkv + h) * ps + off;
    const uint32_t n = uint32_t(len);
    bulk_g2s(stage + ST_IDX + done * 16, p.kcodes + row0 * 16, n * 16, bar);
    bulk_g2s(stage + ST_V + done * 32, p.vdata + row0 * 32, n * 32, bar);
    bulk_g2s(stage + ST_S + done * 8, static_cast<const uint8_t*>(p.vscales) + row0 * 8, n * 8, bar);
    bulk_g2s(stage + ST_Z + done * 8, static_cast<const uint8_t*>(p.vzeros) + row0 * 8, n * 8, bar);
    done += len;
    t += len;
  }
}

// Merge WARPS per-warp records (record of warp w at rec0 + w * rstride floats: acc[G4][D],
// then (m, l) pairs in natural-log units) into the partial slot.  Ends with a CTA barrier.
template <int G4, int WARPS>
__device__ __forceinline__ void v2_merge(const DecodeParams& p, const float* rec0, int rstride, int slot) {
  constexpr int D = 128;
  const int G = p.G;
  float* out = p.slots + int64_t(slot) * G * (D + 2);
  for (int k = threadIdx.x; k < G * D; k += blockDim.x) {
    const int g = k / D, d = k - g * D;
    float M = -INFINITY;
    for (int w = 0; w < WARPS; ++w) M = fmaxf(M, rec0[w * rstride + G4 * D + g * 2]);
    float a = 0.f, L = 0.f;
    for (int w = 0; w < WARPS; ++w) {
      const float* r = rec0 + w * rstride;
      const float mw = r[G4 * D + g * 2];
      const float f = (mw == -INFINITY) ? 0.f : expf(mw - M);
      a += r[g * D + d] * f;
      L += r[G4 * D + g * 2 + 1] * f;
    }
    out[g * D + d] = a;
    if (d == 0) {
      out[G * D + g * 2] = M;
      out[G * D + g * 2 + 1] = L;
    }
  }
  __syncthreads();
}

// One 32-token chunk of a history segment for one warp.  FULL: all 32 tokens valid.
template <int NP, bool FULL>
__device__ __forceinline__ void v2_chunk(const uint8_t* __restrict__ stage, const float* __restrict__ lut,
                                         uint16_t* __restrict__ wb, float* __restrict__ alph, int nv,
                                         float (&acc)[8][4], float (&mrun)[NP], float (&lrun)[NP],
                                         float (&zrun)[NP][4]) {
  using C = V2Cfg<NP>;
  constexpr int G4 = C::G4;
  const int lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int g4 = lane >> 3, b8 = lane & 7;

  // ---- scores (log2 domain): lane (g4, b8) ends with token 8*sb + b8 of head q*4 + g4
  float sc[NP][4];
#pragma unroll
  for (int sb = 0; sb < 4; ++sb) {
    const uint4 u = *reinterpret_cast<const uint4*>(stage + ST_IDX + sb * 128 + b8 * 16);
    const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int q = 0; q < NP; ++q) {
      const char* l0 = reinterpret_cast<const char*>(lut + q * (256 * 64) + b8 * 4 + g4);
      float part[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        // halfword k holds the pair of token (k ^ b8): (idx[b8], idx[b8 + 8])
        const uint32_t w = uw[k >> 1];
        const uint32_t o0 = __byte_perm(w, 0u, (k & 1) ? 0x4424 : 0x4404);  // idx[b8] * 256
        const uint32_t o1 = __byte_perm(w, 0u, (k & 1) ? 0x4434 : 0x4414);  // idx[b8+8] * 256
        part[k] = *reinterpret_cast<const float*>(l0 + o0) + *reinterpret_cast<const float*>(l0 + 128 + o1);
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) part[k] += __shfl_xor_sync(0xffffffffu, part[k + 4], 4);
#pragma unroll
      for (int k = 0; k < 2; ++k) part[k] += __shfl_xor_sync(0xffffffffu, part[k + 2], 2);
      part[0] += __shfl_xor_sync(0xffffffffu, part[1], 1);
      sc[q][sb] = (FULL || sb * 8 + b8 < nv) ? part[0] : -INFINITY;
    }
  }
  // ---- online softmax per head; w = p * scale (fp16) into wbuf, zero term on the CUDA cores
  uint32_t zw[4][2], sw[4][2];
#pragma unroll
  for (int sb = 0; sb < 4; ++sb) {
    const int t = sb * 8 + b8;
    const uint2 z2 = *reinterpret_cast<const uint2*>(stage + ST_Z + t * 8);
    const uint2 s2 = *reinterpret_cast<const uint2*>(stage + ST_S + t * 8);
    zw[sb][0] = z2.x; zw[sb][1] = z2.y;
    sw[sb][0] = s2.x; sw[sb][1] = s2.y;
  }
  bool rescale = false;
#pragma unroll
  for (int q = 0; q < NP; ++q) {
    float mx = fmaxf(fmaxf(sc[q][0], sc[q][1]), fmaxf(sc[q][2], sc[q][3]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
    const float mn = fmaxf(mrun[q], mx);
    const float alpha = fast_exp2(mrun[q] - mn);
    rescale |= (mn != mrun[q]);
    mrun[q] = mn;
    const int g = q * 4 + g4;
    float ls = 0.f, z0 = 0.f, z1 = 0.f, z2 = 0.f, z3 = 0.f;
#pragma unroll
    for (int sb = 0; sb < 4; ++sb) {
      const float pv = fast_exp2(sc[q][sb] - mn);  // 0 for masked tokens
      float s0 = bf16lo(sw[sb][0]), s1 = bf16hi(sw[sb][0]), s2 = bf16lo(sw[sb][1]), s3 = bf16hi(sw[sb][1]);
      float y0 = bf16lo(zw[sb][0]), y1 = bf16hi(zw[sb][0]), y2 = bf16lo(zw[sb][1]), y3 = bf16hi(zw[sb][1]);
      if (!FULL && !(pv > 0.f)) {  // rows past the end may hold anything: keep them out
        s0 = s1 = s2 = s3 = 0.f;
        y0 = y1 = y2 = y3 = 0.f;
      }
      ls += pv;
      z0 = fmaf(pv, y0, z0);
      z1 = fmaf(pv, y1, z1);
      z2 = fmaf(pv, y2, z2);
      z3 = fmaf(pv, y3, z3);
      // token t -> k-step ks, k-slot: t & 15 = 4u + v  ->  slot 2v + (u & 1) + 8 (u >> 1)
      const int t = sb * 8 + b8, ks = t >> 4, u = (t >> 2) & 3, v = t & 3;
      const int slot = 2 * v + (u & 1) + 8 * (u >> 1);
      uint16_t* dst = wb + g * (2 * C::WB_GSTRIDE) + ks * 16 + slot;
      dst[0] = __half_as_ushort(__float2half_rn(pv * s0));
      dst[32] = __half_as_ushort(__float2half_rn(pv * s1));
      dst[64] = __half_as_ushort(__float2half_rn(pv * s2));
      dst[96] = __half_as_ushort(__float2half_rn(pv * s3));
    }
    lrun[q] = lrun[q] * alpha + ls;
    zrun[q][0] = zrun[q][0] * alpha + z0;
    zrun[q][1] = zrun[q][1] * alpha + z1;
    zrun[q][2] = zrun[q][2] * alpha + z2;
    zrun[q][3] = zrun[q][3] * alpha + z3;
    if (b8 == 0) alph[g] = alpha;
  }
  __syncwarp();
  if (__any_sync(0xffffffffu, rescale)) {
    const float aa = 2 * tig < G4 ? alph[2 * tig] : 0.f;
    const float ab = 2 * tig + 1 < G4 ? alph[2 * tig + 1] : 0.f;
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      acc[m][0] *= aa; acc[m][1] *= ab; acc[m][2] *= aa; acc[m][3] *= ab;
    }
  }
  // ---- P.V on the tensor cores: rows = value dims, k = tokens, cols = heads
  const uint32_t* vw = reinterpret_cast<const uint32_t*>(stage + ST_V);
#pragma unroll
  for (int ks = 0; ks < 2; ++ks) {
    uint32_t b0[4], b1[4];
    if (gid < G4) {
      const uint32_t* wr = reinterpret_cast<const uint32_t*>(wb) + gid * C::WB_GSTRIDE + ks * 8 + tig;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        b0[j] = wr[j * 16];
        b1[j] = wr[j * 16 + 4];
      }
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) b0[j] = b1[j] = 0u;
    }
    const int ta = ks * 16 + tig;
    const uint32_t w0 = vw[ta * 8 + gid], w1 = vw[(ta + 4) * 8 + gid];
    const uint32_t w2 = vw[(ta + 8) * 8 + gid], w3 = vw[(ta + 12) * 8 + gid];
    const uint32_t u01 = __byte_perm(w0, w1, 0x5410), v01 = __byte_perm(w0, w1, 0x7632);
    const uint32_t u23 = __byte_perm(w2, w3, 0x5410), v23 = __byte_perm(w2, w3, 0x7632);
    const uint32_t x01[4] = {u01, u01 >> 8, v01, v01 >> 8};
    const uint32_t x23[4] = {u23, u23 >> 8, v23, v23 >> 8};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const uint32_t m0 = 0x00030003u << (4 * hh), m1 = 0x00030003u << (4 * hh + 2);
        const uint32_t a[4] = {x01[j] & m0, x01[j] & m1, x23[j] & m0, x23[j] & m1};
        mma_f16_16816(acc[2 * j + hh], a, b0[j], b1[j]);
      }
    }
  }
  __syncwarp();
}

template <int NP>
__global__ void __launch_bounds__(V2Cfg<NP>::THREADS, 1) decode_v2_kernel(DecodeParams p) {
  using C = V2Cfg<NP>;
  constexpr int D = 128;
  constexpr int G4 = C::G4;
  constexpr int ST = C::STAGES;
  constexpr int WARPS = C::WARPS;
  extern __shared__ __align__(128) uint8_t sm[];
  float* lut = reinterpret_cast<float*>(sm);
  float* qs = reinterpret_cast<float*>(sm + C::LUT_BYTES);
  uint8_t* wreg0 = sm + C::LUT_BYTES + C::Q_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(wreg0 + WARPS * C::WARP_BYTES);

  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  const int g4 = lane >> 3, b8 = lane & 7;
  const int G = p.G;
  uint8_t* wreg = wreg0 + wid * C::WARP_BYTES;                     // ring | wbuf | alpha, z
  uint16_t* wb = reinterpret_cast<uint16_t*>(wreg + ST * STAGE_BYTES);
  float* alph = reinterpret_cast<float*>(wreg + ST * STAGE_BYTES + C::WB_BYTES);
  float* rec = reinterpret_cast<float*>(wreg);                     // merge record (after the loop)
  uint64_t* wbar = bars + wid * ST;
  if (lane == 0) {
    for (int s = 0; s < ST; ++s) mbar_init(&wbar[s], 1);
    fence_mbar_init();
  }
  __syncwarp();
  uint32_t phase = 0;
  bool failed = false;

  const int64_t total = p.plan[p.n_seg];
  const int64_t per = p.plan[p.n_seg + 1];
  const int c = blockIdx.x;
  const int64_t lo = int64_t(c) * per, hi = min(lo + per, total);
  if (lo >= hi) return;
  int sa = 0, sb_ = p.n_seg - 1;
  while (sa < sb_) {
    const int mid = (sa + sb_) >> 1;
    if (p.plan[mid + 1] > lo) sb_ = mid; else sa = mid + 1;
  }
  const float lscale = p.scale * kLog2e;
  for (int s = sa; s < p.n_seg; ++s) {
    const int64_t S = p.plan[s];
    if (S >= hi) break;
    const int n = seg_tokens(p, s);
    if (n == 0) continue;
    const int cs = seg_cost(s);
    int64_t t0 = (lo <= S) ? 0 : (lo - S + cs - 1) / cs;
    int64_t t1 = (hi - S + cs - 1) / cs;
    if (t1 > n) t1 = n;
    if (t0 >= t1) continue;
    const int pair = s >> 1, b = pair / p.Hkv, h = pair - b * p.Hkv;
    for (int i = threadIdx.x; i < G4 * D; i += blockDim.x) {
      const int g = i / D, d = i - g * D;
      qs[i] = g < G ? load_elem(p.q, p.q_dtype, b * p.q_sb + int64_t(h * G + g) * p.q_sh + d) : 0.f;
    }
    if (s & 1) {
      // ---------------- exact recent window (SIMT; a few percent of the bytes)
      __syncthreads();
      WarpState<G4> st;
      st.init();
      const int64_t nch = (t1 - t0 + 31) / 32;
      for (int64_t ch = wid; ch < nch; ch += WARPS) {
        const int64_t tb = t0 + ch * 32;
        const int nvalid = int((t1 - tb) < 32 ? (t1 - tb) : 32);
        float sc[G4];
#pragma unroll
        for (int g = 0; g < G4; ++g) sc[g] = -INFINITY;
        if (lane < nvalid) {
          const int64_t rb = b * p.r_sb + (tb + lane) * p.r_st + h * p.r_sh;
          float a[G4];
#pragma unroll
          for (int g = 0; g < G4; ++g) a[g] = 0.f;
          if (p.r_dtype == SMAQ_BF16) {
            const uint4* kr = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p.rk) + rb);
#pragma unroll 4
            for (int i = 0; i < 16; ++i) {
              const uint4 kv = __ldg(kr + i);
              const uint32_t w[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float k0 = bf16lo(w[e]), k1 = bf16hi(w[e]);
#pragma unroll
                for (int g = 0; g < G4; ++g) {
                  const float2 qq = *reinterpret_cast<const float2*>(qs + g * D + i * 8 + e * 2);
                  a[g] = fmaf(qq.x, k0, a[g]);
                  a[g] = fmaf(qq.y, k1, a[g]);
                }
              }
            }
          } else {
            for (int d = 0; d < D; ++d) {
              const float kv = load_elem(p.rk, p.r_dtype, rb + d);
#pragma unroll
              for (int g = 0; g < G4; ++g) a[g] = fmaf(qs[g * D + d], kv, a[g]);
            }
          }
#pragma unroll
          for (int g = 0; g < G4; ++g) sc[g] = a[g] * p.scale;
        }
        st.softmax_chunk(sc, G4);
#pragma unroll
        for (int jb = 0; jb < 4; ++jb) {
          float v[8][4];
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            const int j = jb * 8 + jj;
            if (j < nvalid) {
              const int64_t rb = b * p.r_sb + (tb + j) * p.r_st + h * p.r_sh + lane * 4;
              if (p.r_dtype == SMAQ_BF16) {
                const uint2 u =
                    __ldg(reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(p.rv) + rb));
                v[jj][0] = bf16lo(u.x); v[jj][1] = bf16hi(u.x); v[jj][2] = bf16lo(u.y); v[jj][3] = bf16hi(u.y);
              } else {
#pragma unroll
                for (int e = 0; e < 4; ++e) v[jj][e] = load_elem(p.rv, p.r_dtype, rb + e);
              }
            } else {
#pragma unroll
              for (int e = 0; e < 4; ++e) v[jj][e] = 0.f;
            }
          }
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
#pragma unroll
            for (int g = 0; g < G4; ++g) {
              const float pj = __shfl_sync(0xffffffffu, sc[g], jb * 8 + jj);
#pragma unroll
              for (int e = 0; e < 4; ++e) st.acc[g][e] = fmaf(pj, v[jj][e], st.acc[g][e]);
            }
          }
        }
      }
      // warp records for the merge live in the per-warp regions
#pragma unroll
      for (int g = 0; g < G4; ++g) {
#pragma unroll
        for (int e = 0; e < 4; ++e) rec[g * D + lane * 4 + e] = st.acc[g][e];
        if (lane == 0) {
          rec[G4 * D + g * 2] = st.m[g];
          rec[G4 * D + g * 2 + 1] = st.l[g];
        }
      }
      __syncthreads();
      v2_merge<G4, WARPS>(p, reinterpret_cast<const float*>(wreg0), C::WARP_BYTES / 4, c + s);
      continue;
    }

    // ---------------- compressed history
    const int64_t nchunks = (t1 - t0 + CH - 1) / CH;
    const int mine = (wid < nchunks) ? int((nchunks - 1 - wid) / WARPS + 1) : 0;
    if (lane == 0) {
      for (int i = 0; i < ST && i < mine; ++i)
        v2_issue(p, b, h, t0, t1, wid + WARPS * i, wreg + i * STAGE_BYTES, &wbar[i]);
    }
    __syncthreads();  // qs complete
    // LUT[q][c][blk][g4] = log2(e) * scale * (q[q*4+g4][8blk:8blk+8] . decoded_centroid[blk][c])
    for (int i = threadIdx.x; i < 16 * 256; i += blockDim.x) {
      const int blk = i >> 8, cc = i & 255;
      if (cc < p.nc) {
        const float4 c0 = __ldg(reinterpret_cast<const float4*>(p.cent + int64_t(blk * p.nc + cc) * 8));
        const float4 c1 = __ldg(reinterpret_cast<const float4*>(p.cent + int64_t(blk * p.nc + cc) * 8 + 4));
#pragma unroll
        for (int q = 0; q < NP; ++q) {
          float r[4];
#pragma unroll
          for (int gg = 0; gg < 4; ++gg) {
            const float* qg = qs + (q * 4 + gg) * D + blk * 8;
            float a = qg[0] * c0.x;
            a = fmaf(qg[1], c0.y, a);
            a = fmaf(qg[2], c0.z, a);
            a = fmaf(qg[3], c0.w, a);
            a = fmaf(qg[4], c1.x, a);
            a = fmaf(qg[5], c1.y, a);
            a = fmaf(qg[6], c1.z, a);
            a = fmaf(qg[7], c1.w, a);
            r[gg] = a * lscale;
          }
          *reinterpret_cast<float4*>(lut + q * (256 * 64) + (cc * 16 + blk) * 4) = make_float4(r[0], r[1], r[2], r[3]);
        }
      }
    }
    __syncthreads();

    float acc[8][4];
#pragma unroll
    for (int m = 0; m < 8; ++m)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[m][e] = 0.f;
    float mrun[NP], lrun[NP], zrun[NP][4];
#pragma unroll
    for (int q = 0; q < NP; ++q) {
      mrun[q] = -INFINITY;
      lrun[q] = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) zrun[q][j] = 0.f;
    }
    for (int i = 0; i < mine; ++i) {
      const int stg = i % ST;
      uint8_t* stage = wreg + stg * STAGE_BYTES;
      if (!failed && !mbar_wait(&wbar[stg], (phase >> stg) & 1u)) failed = true;
      phase ^= 1u << stg;
      const int64_t tc = t0 + int64_t(wid + WARPS * i) * CH;
      const int nv = int((t1 - tc) < CH ? (t1 - tc) : CH);
      if (nv == CH)
        v2_chunk<NP, true>(stage, lut, wb, alph, nv, acc, mrun, lrun, zrun);
      else
        v2_chunk<NP, false>(stage, lut, wb, alph, nv, acc, mrun, lrun, zrun);
      if (lane == 0 && i + ST < mine) v2_issue(p, b, h, t0, t1, wid + WARPS * (i + ST), stage, &wbar[stg]);
    }

    // ---- warp epilogue: (m, l, zero term) per head, then the value sums, into the record
#pragma unroll
    for (int q = 0; q < NP; ++q) {
      float l = lrun[q], z[4] = {zrun[q][0], zrun[q][1], zrun[q][2], zrun[q][3]};
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) {
        l += __shfl_xor_sync(0xffffffffu, l, o);
#pragma unroll
        for (int j = 0; j < 4; ++j) z[j] += __shfl_xor_sync(0xffffffffu, z[j], o);
      }
      const int g = q * 4 + g4;
      if (b8 == 0) {
        rec[G4 * D + g * 2] = mine ? mrun[q] * kLn2 : -INFINITY;   // back to natural-log units
        rec[G4 * D + g * 2 + 1] = l;
#pragma unroll
        for (int j = 0; j < 4; ++j) alph[8 + g * 4 + j] = z[j];
      }
    }
    __syncwarp();
    {
      const int ga = 2 * tig, gb = 2 * tig + 1;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float za = ga < G4 ? alph[8 + ga * 4 + j] : 0.f;
        const float zb = gb < G4 ? alph[8 + gb * 4 + j] : 0.f;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int d0 = 32 * j + 4 * gid + 2 * hh;       // row gid -> code r = 2hh; row gid+8 -> 2hh+1
          const float s0 = hh ? 1048576.0f : 16777216.0f;  // 2^24 * 4^-r
          const float s1 = hh ? 262144.0f : 4194304.0f;    // 2^24 * 4^-(r+1)
          if (ga < G4) {
            rec[ga * D + d0] = fmaf(acc[2 * j + hh][0], s0, za);
            rec[ga * D + d0 + 1] = fmaf(acc[2 * j + hh][2], s1, za);
          }
          if (gb < G4) {
            rec[gb * D + d0] = fmaf(acc[2 * j + hh][1], s0, zb);
            rec[gb * D + d0 + 1] = fmaf(acc[2 * j + hh][3], s1, zb);
          }
        }
      }
    }
    __syncthreads();
    v2_merge<G4, WARPS>(p, reinterpret_cast<const float*>(wreg0), C::WARP_BYTES / 4, c + s);
  }
  if (failed && lane == 0) atomicExch(reinterpret_cast<int*>(p.plan + p.n_seg + 2), 1);
}

bool decode_v2_eligible(const DecodeParams& p, int key_format, int value_bits, int q_dtype) {
  (void)q_dtype;
  return key_format == SMAQ_KEYS_BVQ && value_bits == 2 && p.D == 128 && p.gs == 32 && p.G <= 8 &&
         p.layout == SMAQ_LAYOUT_DECODE && p.kv_dtype == SMAQ_BF16 && p.page_size % 16 == 0 &&
         (p.q_dtype == SMAQ_BF16 || p.q_dtype == SMAQ_F16) && p.nc <= 256;
}

template <int NP>
static int launch_v2_t(DecodeParams& p, int grid_req, cudaStream_t s, int* grid_out, bool query_only) {
  auto kern = decode_v2_kernel<NP>;
  const int sm = V2Cfg<NP>::SMEM;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
  if (e != cudaSuccess) return cuda_status(e, "decode_v2 attr");
  const int grid = grid_req > 0 ? grid_req : num_sms();
  *grid_out = grid;
  if (query_only) return SMAQ_OK;
  kern<<<grid, V2Cfg<NP>::THREADS, sm, s>>>(p);
  return cuda_status(cudaGetLastError(), "decode_v2_kernel");
}

int launch_decode_v2(DecodeParams& p, int grid_req, cudaStream_t s, int* grid_out, bool query_only) {
  if (p.G <= 4) return launch_v2_t<1>(p, grid_req, s, grid_out, query_only);
  return launch_v2_t<2>(p, grid_req, s, grid_out, query_only);
}

}  // namespace smaq
