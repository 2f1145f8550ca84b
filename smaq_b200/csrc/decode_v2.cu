// Fast hybrid decode for block-VQ keys with an fp16 codebook (sm_100a): TMA-staged streams,
// tensor-core scores and tensor-core P.V; the exact recent window in the same launch.
//
// Reference semantics: compute_hybrid_attention (smaq/score.py:23-72) with SMAQBlockVQ scores
// q . decoded_centroid[idx] * scale (smaq/block_vq.py:246-297) and 2-bit group-32 values
// dequantized as code * scale + zero (smaq/kv_cache.py:94-103).  Same work partition, partial
// slots and merge as the general kernel in decode.cu.
//
// Per CTA: WARPS warps; each warp streams its own 32-token chunks of one (sequence, kv head)
// segment.
//  * Staging: lane 0 of each warp issues 1-D bulk async copies (TMA engine, no multicast) of a
//    chunk's index / value-code / scale / zero rows into a private STAGES-deep ring; an
//    mbarrier counts the bytes.  Rows use SMAQ_LAYOUT_DECODE (include/smaq_b200.h).
//  * Scores on the tensor cores (mma.m16n8k16, fp16 in, fp32 accumulate).  The decoded
//    codebook is fp16-valued, so K_hat = decoded_centroid[idx] is exact in fp16 and each
//    thread gathers the operand straight from a 64 KB shared copy of the codebook with one
//    16-byte load per (token, block).  B columns are (token, half of the head dim), A rows are
//    (head, half), so the 8 lanes of every load phase touch 8 distinct 16-byte bank groups;
//    score(h, t) = D[(h,0),(t,0)] + D[(h,1),(t,1)] lands in the thread that owns head h and
//    token t for the P.V step -- no shared-memory round trip.  Scores are kept in the log2
//    domain (p = exp2(s - m)).
//  * P.V on the tensor cores (mma.m16n8k16): A = value codes as exact fp16 subnormals -- the
//    2-bit field of code r of a byte sits at mantissa bits 2r, so one AND yields
//    code * 4^r * 2^-24 with no unpacking -- and B = p * value_scale (fp16).  Rows of that MMA
//    are value dimensions ordered so each thread's bits come from ONE 32-bit word per token.
//    The epilogue multiplies by 2^24 / 4^r; sum_t p_t * zero_t runs on the CUDA cores.
#include <math.h>

#include "common.cuh"
#include "decode_common.cuh"
#include "ptx.cuh"

namespace smaq {

constexpr int CH = 32;  // tokens per chunk
constexpr int ST_IDX = 0, ST_V = CH * 16, ST_S = CH * 48, ST_Z = CH * 56, STAGE_BYTES = CH * 64;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
// History weights are p = 2^(s - m + kShift) <= 64: fp16 keeps them normal down to 2^-20 of the
// maximum, and p * scale stays finite for value scales below 1023.
constexpr float kShift = 6.f;

// Floats of shared scratch the final merge of a pair with nt slots needs (G query heads).
__host__ __device__ constexpr int final_scratch_floats(int G, int nt) { return 2 * G * nt + 2 * G + 3 + 512 * 8; }
// Row pitch of the exact window's staged key / value rows (bytes): 8 rows of one ldmatrix
// phase fall in 8 distinct 16-byte bank groups.
constexpr int WIN_ROW = 272;

template <int GM>
struct V3Cfg {
  static constexpr int WARPS = 16;
  static constexpr int THREADS = WARPS * 32;
  static constexpr int STAGES = 3;
  static constexpr int CTAS = 1;    // resident CTAs per SM
  static constexpr int CB_BYTES = 256 * 16 * 16;                 // fp16 codebook [c][block'][8]
  static constexpr int Q_BYTES = GM * 128 * 4;                   // fp32 query rows
  static constexpr int SZ_BYTES = 2 * 4 * CH * 2;                // fp16 scales | zeros [j][ks][slot]
  static constexpr int WARP_BYTES = STAGES * STAGE_BYTES + SZ_BYTES + 256;  // ring | s,z | misc
  static constexpr int BAR_BYTES = WARPS * STAGES * 8;
  static constexpr int MAX_FUSED_SEG = 2048;  // in-kernel partition table
  static constexpr int PLAN_BYTES = (MAX_FUSED_SEG + 4) * 8 + 33 * 8 + 16 + MAX_FUSED_SEG * 4 + 3 * 32 * 4;  // table | scan | flag | tokens | arrivals
  static constexpr int SMEM = CB_BYTES + Q_BYTES + WARPS * WARP_BYTES + BAR_BYTES + PLAN_BYTES;
  static_assert(GM * (128 + 2) * 4 <= STAGES * STAGE_BYTES, "merge record must fit in a ring");
  static_assert(16 * WIN_ROW <= STAGES * STAGE_BYTES, "window rows must fit in a ring");
  static_assert(SMEM <= (CTAS == 1 ? 232448 : 233472 / CTAS - 1024), "shared memory budget");
  static_assert(final_scratch_floats(GM, 2 * 512) * 4 <= WARPS * WARP_BYTES, "final-merge scratch");
};

__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Shared-memory accesses by 32-bit offset from the start of the dynamic shared window.  Plain C++
// accesses (not volatile asm) so the compiler may hoist independent loads ahead of the mma chains.
extern __shared__ __align__(128) uint8_t sm[];
__device__ __forceinline__ uint4 lds128(uint32_t off) { return *reinterpret_cast<const uint4*>(sm + off); }

// block b of the codebook lives at 16-byte slot sigma(b) of its 256-byte row (see the bank note)
__host__ __device__ constexpr int cb_sigma(int b) { return b < 8 ? b : 8 + ((b - 8 + 4) & 7); }

// Per-segment source description of one stream for the bulk copies.
struct V3Src {
  const uint8_t* base;  // contiguous store: this stream at token t0 of the segment; paged: stream base
  uint32_t row_bytes;   // 16 (indices), 32 (value codes), 8 (scales), 8 (zeros)
  uint32_t dst_off;     // offset of the stream inside a stage
};

// This lane's stream (lane & 3: indices, value codes, scales, zeros) of the history segment of
// (sequence b, kv head h) that starts at token t0.
__device__ __forceinline__ V3Src v3_src(const DecodeParams& p, int b, int h, int64_t t0) {
  V3Src src;
  const int k = threadIdx.x & 3;
  const uint8_t* base = k == 0 ? p.kcodes
                        : k == 1 ? p.vdata
                        : k == 2 ? static_cast<const uint8_t*>(p.vscales)
                                 : static_cast<const uint8_t*>(p.vzeros);
  src.row_bytes = k == 0 ? 16u : k == 1 ? 32u : 8u;
  src.dst_off = k == 0 ? uint32_t(ST_IDX) : k == 1 ? uint32_t(ST_V) : k == 2 ? uint32_t(ST_S) : uint32_t(ST_Z);
  src.base = p.bt ? base : base + ((int64_t(b) * p.Hkv + h) * p.page_size + t0) * src.row_bytes;
  return src;
}

// Lanes 0..3 each copy one stream of chunk `kc` (tokens t0 + 32kc ..) into `stage`; the
// mbarrier was initialised with 4 arrivals.  Paged stores split the copy at page boundaries.
__device__ __forceinline__ void v3_issue(const DecodeParams& p, const V3Src& src, int b, int h, int64_t t0,
                                         int nv, int kc, uint8_t* stage, uint64_t* bar) {
  const uint32_t ncopy = (uint32_t(nv) + 15u) & ~15u;
  const uint64_t pol = evict_first_policy();  // streamed once
  mbar_arrive_expect_tx(bar, ncopy * src.row_bytes);
  if (!p.bt) {
    bulk_g2s_hint(stage + src.dst_off, src.base + size_t(kc) * CH * src.row_bytes, ncopy * src.row_bytes, bar, pol);
    return;
  }
  const int64_t ps = p.page_size;
  int64_t t = t0 + int64_t(kc) * CH;
  uint32_t done = 0;
  while (done < ncopy) {
    const int64_t pg = t / ps, off = t - pg * ps;
    uint32_t len = ncopy - done;
    if (int64_t(len) > ps - off) len = uint32_t(ps - off);
    const int64_t r = (int64_t(p.bt[b * p.bt_stride + pg]) * p.Hkv + h) * ps + off;
    bulk_g2s_hint(stage + src.dst_off + done * src.row_bytes, src.base + r * src.row_bytes, len * src.row_bytes, bar, pol);
    done += len;
    t += len;
  }
}

// Merge WARPS per-warp records (record of warp w at rec0 + w * rstride floats: acc[GM][D],
// then (m, l) pairs in natural-log units) into the partial slot.  Ends with a CTA barrier.
template <int GM, int WARPS>
__device__ __forceinline__ void v3_merge(const DecodeParams& p, const float* rec0, int rstride, int slot) {
  constexpr int D = 128;
  const int G = p.G;
  float* out = p.slots + int64_t(slot) * G * (D + 2);
  for (int k = threadIdx.x; k < G * D; k += blockDim.x) {
    const int g = k / D, d = k - g * D;
    float M = -INFINITY;
    for (int w = 0; w < WARPS; ++w) M = fmaxf(M, rec0[w * rstride + GM * D + g * 2]);
    float a = 0.f, L = 0.f;
    for (int w = 0; w < WARPS; ++w) {
      const float* r = rec0 + w * rstride;
      const float mw = r[GM * D + g * 2];
      const float f = (mw == -INFINITY) ? 0.f : expf(mw - M);
      a += r[g * D + d] * f;
      L += r[GM * D + g * 2 + 1] * f;
    }
    out[g * D + d] = a;
    if (d == 0) {
      out[G * D + g * 2] = M;
      out[G * D + g * 2 + 1] = L;
    }
  }
  fence_proxy_async_smem();  // the records sit in the rings, which bulk copies refill next
  __syncthreads();
}

struct V3Lane {
  uint32_t sz_off;    // byte offset of token `lane`'s slot in the fp16 scale/zero arrays
  uint32_t idx_off;   // byte offset of this lane's index word inside a chunk (token gid>>1)
  uint32_t sel[2];    // byte_perm selectors building the codebook address for kp = 0, 1
  uint32_t base[2];   // sigma(block) * 16 for kp = 0, 1
};

// One 32-token chunk for one warp.  Thread (gid, tig): score/MMA-B role = head gid and the
// tokens t = 4i + tig; P.V A role = value word gid of those tokens.  FULL: all 32 tokens valid.
__device__ __forceinline__ uint32_t lds32(uint32_t off) { return *reinterpret_cast<const uint32_t*>(sm + off); }
__device__ __forceinline__ uint2 lds64(uint32_t off) { return *reinterpret_cast<const uint2*>(sm + off); }
__device__ __forceinline__ void sts16(uint32_t off, uint16_t v) { *reinterpret_cast<uint16_t*>(sm + off) = v; }
__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// p * scale as fp16 hi + lo (an exact two-product: lo = fma(p, s, -hi)).  The dequantized
// values cancel strongly around their zero points (|code * scale| ~ |zero| >> |output| for a
// long, nearly uniform history), so one fp16 rounding per term is too coarse there.
__device__ __forceinline__ uint32_t two_prod_lo(uint32_t p, uint32_t sc, uint32_t hi) {
  return hfma2(p, sc, hi ^ 0x80008000u);
}

// Fold one chunk's zero-point sums into acc and clear them.  zacc rows 0..3 are value groups,
// columns 2 tig, 2 tig + 1 heads; value row r of acc is in units of 2^-24 4^r (the fp16-subnormal
// codes).  Folding every chunk keeps acc at sum p * value: the tensor cores' fp32 accumulation
// never carries the two large cancelling sums (p * scale * code and p * zero) across a history.
// keep: this thread's acc columns take the fold (false for the lo columns of the G <= 4 path).
__device__ __forceinline__ void fold_zero(float (&acc)[8][4], float (&zacc)[4], bool keep) {
  const int lane = threadIdx.x & 31, tig = lane & 3;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float za = __shfl_sync(0xffffffffu, zacc[0], j * 4 + tig);
    float zb = __shfl_sync(0xffffffffu, zacc[1], j * 4 + tig);
    if (!keep) za = zb = 0.f;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const float k0 = hh ? 1.0f / 1048576.0f : 1.0f / 16777216.0f;   // 4^r 2^-24, r = 2 hh
      const float k1 = hh ? 1.0f / 262144.0f : 1.0f / 4194304.0f;     // r = 2 hh + 1
      acc[2 * j + hh][0] = fmaf(za, k0, acc[2 * j + hh][0]);
      acc[2 * j + hh][2] = fmaf(za, k1, acc[2 * j + hh][2]);
      acc[2 * j + hh][1] = fmaf(zb, k0, acc[2 * j + hh][1]);
      acc[2 * j + hh][3] = fmaf(zb, k1, acc[2 * j + hh][3]);
    }
  }
  zacc[0] = zacc[1] = zacc[2] = zacc[3] = 0.f;
}

// The chunk's value scales and zeros as fp16, in MMA k-slot order (one token per lane).
template <bool FULL>
__device__ __forceinline__ void stage_scales(uint32_t st, uint32_t szs, const V3Lane& L, int nv) {
  const int lane = threadIdx.x & 31;
  uint2 s2 = lds64(st + ST_S + lane * 8);
  uint2 z2 = lds64(st + ST_Z + lane * 8);
  if (!FULL && lane >= nv) s2 = z2 = make_uint2(0u, 0u);  // rows past the end may hold anything
  const uint32_t sp0 = pack_f16x2(bf16lo(s2.x), bf16hi(s2.x)), sp1 = pack_f16x2(bf16lo(s2.y), bf16hi(s2.y));
  const uint32_t zp0 = pack_f16x2(bf16lo(z2.x), bf16hi(z2.x)), zp1 = pack_f16x2(bf16lo(z2.y), bf16hi(z2.y));
  const uint32_t o = szs + L.sz_off;
  sts16(o + 0, uint16_t(sp0)); sts16(o + 64, uint16_t(sp0 >> 16));
  sts16(o + 128, uint16_t(sp1)); sts16(o + 192, uint16_t(sp1 >> 16));
  sts16(o + 256, uint16_t(zp0)); sts16(o + 320, uint16_t(zp0 >> 16));
  sts16(o + 384, uint16_t(zp1)); sts16(o + 448, uint16_t(zp1 >> 16));
}

// One 32-token chunk for one warp (G in 5..8).  Thread (gid, tig): score/MMA-B role = head gid
// and the tokens t = 4i + tig; P.V A role = value word gid of those tokens.  FULL: all 32 tokens
// valid.  Shared addresses are 32-bit: st = this stage, szs = fp16 scales [j][ks][slot] then
// zeros.  History weights are p = 2^(s - m + kShift).
template <bool FULL>
__device__ __forceinline__ void v3_chunk(uint32_t st, uint32_t cb_s, uint32_t szs, const V3Lane& L,
                                         const uint32_t (&qa)[4][4], int G, float lscale, int nv,
                                         float (&acc)[8][4], float (&zacc)[4], float& mrun, float& lrun) {
  const int lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  stage_scales<FULL>(st, szs, L, nv);
  // ---- scores: 8 n-tiles of 4 tokens; thread ends with s[i] = score(head gid, token 4i + tig)
  float s[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t w = lds32(st + ST_IDX + L.idx_off + i * 64);
    const uint4 e0 = lds128(cb_s + __byte_perm(w, L.base[0], L.sel[0]));
    const uint4 e1 = lds128(cb_s + __byte_perm(w, L.base[1], L.sel[1]));
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    mma_f16_16816(d, qa[0], e0.x, e0.y);
    mma_f16_16816(d, qa[1], e0.z, e0.w);
    mma_f16_16816(d, qa[2], e1.x, e1.y);
    mma_f16_16816(d, qa[3], e1.z, e1.w);
    const float sc = (d[0] + d[3]) * lscale;
    s[i] = (FULL || 4 * i + tig < nv) ? sc : -INFINITY;  // heads >= G score 0: harmless
  }
  // ---- online softmax for head gid over the 8 tokens of this thread and its 3 tig peers
  float mx = fmaxf(fmaxf(fmaxf(s[0], s[1]), fmaxf(s[2], s[3])), fmaxf(fmaxf(s[4], s[5]), fmaxf(s[6], s[7])));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
  const float mn = fmaxf(mrun, mx);
  const float alpha = fast_exp2(mrun - mn);  // first chunk: exp2(-inf) = 0
  const bool grew = mn != mrun;
  mrun = mn;
  float ls = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    s[i] = fast_exp2(s[i] - (mn - kShift));  // p; 0 for masked tokens
    ls += s[i];
  }
  lrun = lrun * alpha + ls;
  if (__any_sync(0xffffffffu, grew)) {
    // acc columns 2tig, 2tig+1 belong to heads 2tig, 2tig+1: fetch their alphas
    const float aa = __shfl_sync(0xffffffffu, alpha, (2 * tig) * 4);
    const float ab = __shfl_sync(0xffffffffu, alpha, (2 * tig + 1) * 4);
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      acc[m][0] *= aa; acc[m][1] *= ab; acc[m][2] *= aa; acc[m][3] *= ab;
    }
  }
  __syncwarp();  // fp16 scales / zeros visible to the warp
  // ---- P.V: k-step ks covers tokens 16ks + tig + 4u (u = 0..3) = this thread's s[4ks + u]
#pragma unroll
  for (int ks = 0; ks < 2; ++ks) {
    const uint32_t p01 = pack_f16x2(s[4 * ks + 0], s[4 * ks + 1]);   // k-slots 2tig, 2tig+1
    const uint32_t p23 = pack_f16x2(s[4 * ks + 2], s[4 * ks + 3]);   // k-slots 2tig+8, 2tig+9
    const uint32_t sb = szs + ks * 32 + tig * 4;
    // zero-point term on the tensor cores: rows = value groups, B = p
    {
      uint32_t az[4] = {0u, 0u, 0u, 0u};
      if (gid < 4) {
        az[0] = lds32(sb + 256 + gid * 64);
        az[2] = lds32(sb + 256 + gid * 64 + 16);
      }
      mma_f16_16816(zacc, az, p01, p23);
    }
    const uint32_t vb = st + ST_V + (16 * ks + tig) * 32 + gid * 4;
    const uint32_t w0 = lds32(vb), w1 = lds32(vb + 128), w2 = lds32(vb + 256), w3 = lds32(vb + 384);
    const uint32_t u01 = __byte_perm(w0, w1, 0x5410), v01 = __byte_perm(w0, w1, 0x7632);
    const uint32_t u23 = __byte_perm(w2, w3, 0x5410), v23 = __byte_perm(w2, w3, 0x7632);
    const uint32_t x01[4] = {u01, u01 >> 8, v01, v01 >> 8};
    const uint32_t x23[4] = {u23, u23 >> 8, v23, v23 >> 8};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t sc0 = lds32(sb + j * 64), sc1 = lds32(sb + j * 64 + 16);
      const uint32_t bh0 = hmul2(p01, sc0), bh1 = hmul2(p23, sc1);
      const uint32_t bl0 = two_prod_lo(p01, sc0, bh0), bl1 = two_prod_lo(p23, sc1, bh1);
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const uint32_t m0 = 0x00030003u << (4 * hh), m1 = 0x00030003u << (4 * hh + 2);
        const uint32_t a[4] = {x01[j] & m0, x01[j] & m1, x23[j] & m0, x23[j] & m1};
        mma_f16_16816(acc[2 * j + hh], a, bh0, bh1);
        mma_f16_16816(acc[2 * j + hh], a, bl0, bl1);
      }
    }
  }
  fold_zero(acc, zacc, true);
  fence_proxy_async_smem();  // the stage is refilled by a bulk copy after this barrier
  __syncwarp();
}

// G <= 4: scores from a per-pair lookup table instead of the tensor cores.  Entry (code c,
// block b) at shared offset c * 256 + b * 16 holds, for the four query heads,
// scale * log2(e) * q_g[8b .. 8b+8) . decoded_centroid[b][c] in fp32, so a token's score is the
// sum of its 16 entries.  Lane = token.  Lane L visits block j ^ (L & 15) at step j, so the
// eight lanes of every load phase hit eight distinct 16-byte bank groups.  The softmax keeps
// one reference maximum per head for the warp and rescales only when a score exceeds it.
// P.V: columns 0..3 of the MMA are the four heads with B = hi(p * scale), columns 4..7 the same
// heads with B = lo(p * scale); the epilogue adds column g + 4 to column g.
struct LutLane {
  uint32_t xl;     // (L & 15) << 4
  uint32_t sel;    // byte_perm selector: byte i <- byte i ^ (L & 3)
  bool swp8, swp4; // word-pair / word swaps of the XOR permutation
};

template <bool FULL>
__device__ __forceinline__ void v3_chunk_lut(uint32_t st, uint32_t szs, uint32_t pb, const V3Lane& L,
                                             const LutLane& X, int nv, float (&acc)[8][4], float (&zacc)[4],
                                             float (&mref)[4], float (&lsum)[4]) {
  const int lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  stage_scales<FULL>(st, szs, L, nv);
  // ---- scores of token `lane`
  const uint4 w = *reinterpret_cast<const uint4*>(sm + st + ST_IDX + lane * 16);
  // decode-layout byte order -> natural block order, then XOR-permute the bytes by (L & 15)
  uint32_t n0 = __byte_perm(w.x, w.y, 0x6420), n1 = __byte_perm(w.x, w.y, 0x7531);
  uint32_t n2 = __byte_perm(w.z, w.w, 0x6420), n3 = __byte_perm(w.z, w.w, 0x7531);
  if (X.swp8) { const uint32_t a = n0, b = n1; n0 = n2; n1 = n3; n2 = a; n3 = b; }
  if (X.swp4) { const uint32_t a = n0, b = n2; n0 = n1; n1 = a; n2 = n3; n3 = b; }
  const uint32_t r[4] = {__byte_perm(n0, 0, X.sel), __byte_perm(n1, 0, X.sel), __byte_perm(n2, 0, X.sel),
                         __byte_perm(n3, 0, X.sel)};
  // heads (0, 1) and (2, 3) accumulate as packed fp32 pairs (one add.f32x2 per pair)
  uint64_t s01 = 0ull, s23 = 0ull;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const uint32_t c256 = __byte_perm(r[j >> 2], 0, 0x4404 | ((j & 3) << 4));  // code * 256
    const ulonglong2 e = *reinterpret_cast<const ulonglong2*>(sm + (c256 | (X.xl ^ uint32_t(j << 4))));
    asm("add.rn.f32x2 %0, %0, %1;" : "+l"(s01) : "l"(e.x));
    asm("add.rn.f32x2 %0, %0, %1;" : "+l"(s23) : "l"(e.y));
  }
  float s[4] = {__uint_as_float(uint32_t(s01)), __uint_as_float(uint32_t(s01 >> 32)),
                __uint_as_float(uint32_t(s23)), __uint_as_float(uint32_t(s23 >> 32))};
  if (!FULL && lane >= nv) s[0] = s[1] = s[2] = s[3] = -INFINITY;
  // ---- softmax: p = exp2(s - mref + kShift); the reference maximum only moves up
  const bool grow = (s[0] > mref[0]) | (s[1] > mref[1]) | (s[2] > mref[2]) | (s[3] > mref[3]);
  if (__any_sync(0xffffffffu, grow)) {
    float al[4];
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const float mn = fmaxf(mref[g], warp_max(s[g]));
      al[g] = fast_exp2(mref[g] - mn);  // first chunk: exp2(-inf) = 0
      mref[g] = mn;
      lsum[g] *= al[g];
    }
    // acc columns 2tig, 2tig+1 belong to heads (2tig, 2tig+1) mod 4 (columns 4..7: lo parts)
    const float aa = (tig & 1) ? al[2] : al[0];
    const float ab = (tig & 1) ? al[3] : al[1];
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      acc[m][0] *= aa; acc[m][1] *= ab; acc[m][2] *= aa; acc[m][3] *= ab;
    }
  }
  // p in fp16, k-slot order per head (the B operand layout of the P.V MMA)
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const float pg = fast_exp2(s[g] - (mref[g] - kShift));  // 0 for masked tokens
    lsum[g] += pg;
    sts16(pb + g * 64 + L.sz_off, __half_as_ushort(__float2half_rn(pg)));
  }
  __syncwarp();  // p, fp16 scales / zeros visible to the warp
  // ---- P.V: k-step ks covers tokens 16ks + tig + 4u (u = 0..3)
  const bool lo_col = gid >= 4;
#pragma unroll
  for (int ks = 0; ks < 2; ++ks) {
    const uint32_t p01 = lds32(pb + (gid & 3) * 64 + ks * 32 + tig * 4);        // k-slots 2tig, 2tig+1
    const uint32_t p23 = lds32(pb + (gid & 3) * 64 + ks * 32 + tig * 4 + 16);   // k-slots 2tig+8, 2tig+9
    const uint32_t sb = szs + ks * 32 + tig * 4;
    uint32_t b0[4], b1[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t sc0 = lds32(sb + j * 64), sc1 = lds32(sb + j * 64 + 16);
      const uint32_t h0 = hmul2(p01, sc0), h1 = hmul2(p23, sc1);
      b0[j] = lo_col ? two_prod_lo(p01, sc0, h0) : h0;
      b1[j] = lo_col ? two_prod_lo(p23, sc1, h1) : h1;
    }
    {
      uint32_t az[4] = {0u, 0u, 0u, 0u};
      if (gid < 4) {
        az[0] = lds32(sb + 256 + gid * 64);
        az[2] = lds32(sb + 256 + gid * 64 + 16);
      }
      mma_f16_16816(zacc, az, p01, p23);
    }
    const uint32_t vb = st + ST_V + (16 * ks + tig) * 32 + gid * 4;
    const uint32_t w0 = lds32(vb), w1 = lds32(vb + 128), w2 = lds32(vb + 256), w3 = lds32(vb + 384);
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
  fold_zero(acc, zacc, tig < 2);
  fence_proxy_async_smem();  // the stage is refilled by a bulk copy after this barrier
  __syncwarp();
}

// One chunk of up to 8 exact recent-window tokens for one warp: lanes 4j..4j+3 score token j
// (quarter q of the lane holds dims [32q, 32q + 32)), fp32 against the bf16/fp16 keys; online
// softmax; then P.V with lane owning dims [4 lane, 4 lane + 4).  This is _exact_scores /
// _apply_weights of smaq/score.py:99-124 in the kernel's softmax units.
template <int GM>
__device__ __forceinline__ void v3_window_chunk(const DecodeParams& p, const float* qs, int b, int h, int64_t tb,
                                                int nvalid, WarpState<GM>& st) {
  constexpr int D = 128;
  const int lane = threadIdx.x & 31;
  const int G = p.G;
  const int tok = lane >> 2, qt = lane & 3;
  const bool valid = tok < nvalid;
  float a[GM];
#pragma unroll
  for (int g = 0; g < GM; ++g) a[g] = 0.f;
  if (valid) {
    const int64_t rb = b * p.r_sb + (tb + tok) * p.r_st + h * p.r_sh + 32 * qt;
    if (p.r_dtype == SMAQ_BF16 || p.r_dtype == SMAQ_F16) {
      const bool bf = p.r_dtype == SMAQ_BF16;
      const uint4* kr = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.rk) + rb);
      uint4 kw[4];
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) kw[c8] = __ldg(kr + c8);
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) {
        const uint32_t ws[4] = {kw[c8].x, kw[c8].y, kw[c8].z, kw[c8].w};
        float k[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if (bf) {
            k[2 * e] = bf16lo(ws[e]);
            k[2 * e + 1] = bf16hi(ws[e]);
          } else {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&ws[e]));
            k[2 * e] = f.x;
            k[2 * e + 1] = f.y;
          }
        }
#pragma unroll
        for (int g = 0; g < GM; ++g) {
          if (g >= G) break;
          const float* qg = qs + g * D + 32 * qt + c8 * 8;
#pragma unroll
          for (int e = 0; e < 8; ++e) a[g] = fmaf(qg[e], k[e], a[g]);
        }
      }
    } else {
      for (int d = 0; d < 32; ++d) {
        const float kv = load_elem(p.rk, p.r_dtype, rb + d);
#pragma unroll
        for (int g = 0; g < GM; ++g) {
          if (g >= G) break;
          a[g] = fmaf(qs[g * D + 32 * qt + d], kv, a[g]);
        }
      }
    }
  }
  // the chunk's value rows (lane owns dims [4 lane, 4 lane + 4)), loaded before the softmax
  float v[8][4];
  {
    const int64_t vb = b * p.r_sb + tb * p.r_st + h * p.r_sh + lane * 4;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int64_t rb = vb + int64_t(u < nvalid ? u : 0) * p.r_st;
      if (p.r_dtype == SMAQ_BF16) {
        const uint2 w = __ldg(reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(p.rv) + rb));
        v[u][0] = bf16lo(w.x); v[u][1] = bf16hi(w.x); v[u][2] = bf16lo(w.y); v[u][3] = bf16hi(w.y);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) v[u][e] = load_elem(p.rv, p.r_dtype, rb + e);
      }
    }
  }
  float sc[GM];
#pragma unroll
  for (int g = 0; g < GM; ++g) {
    float r = a[g] + __shfl_xor_sync(0xffffffffu, a[g], 1);
    r += __shfl_xor_sync(0xffffffffu, r, 2);
    sc[g] = (valid && qt == 0) ? r * p.scale : -INFINITY;
  }
  st.softmax_chunk(sc, G);
#pragma unroll
  for (int u = 0; u < 8; ++u) {
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      if (g >= G) break;
      float pj = __shfl_sync(0xffffffffu, sc[g], u * 4);
      if (u >= nvalid) pj = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) st.acc[g][e] = fmaf(pj, v[u][e], st.acc[g][e]);
    }
  }
}

// ---------------------------------------------------------------- exact window on tensor cores
// Used when the window rows are bf16 or fp16 of the query's dtype with 16-byte aligned rows.
// Warp w takes 8-token chunks w, w + WARPS, ... of the window segment.
//  * Scores: mma m16n8k16, A = query rows (head gid; rows 8-15 zero), B = key rows (token gid).
//    The contraction runs over the head dim in a permuted order so that lane tig reads dims
//    [32 tig, 32 tig + 32) of its token's key row with four 16-byte loads: k-step ks takes dims
//    32 tig + 4 ks + {0,1} as fragment slots (2 tig, 2 tig + 1) and + {2,3} as (2 tig + 8, +9);
//    the query fragments use the same order, so every dot product is the plain one.
//  * P.V: mma m16n8k8, A = the weights in the score fragment layout (head gid, tokens 2 tig,
//    2 tig + 1) split into hi + lo of the value dtype, B = the chunk's value rows staged in
//    shared memory (row pitch WIN_ROW: the 8 rows of one ldmatrix phase hit 8 distinct bank
//    groups) and read transposed by ldmatrix.
// This is _exact_scores / _apply_weights of smaq/score.py:99-124 in the kernel's softmax units
// (natural log, as the merge records expect).

__device__ __forceinline__ bool window_mma_ok(const DecodeParams& p) {
  return (p.r_dtype == SMAQ_BF16 || p.r_dtype == SMAQ_F16) && p.r_dtype == p.q_dtype &&
         ((reinterpret_cast<uintptr_t>(p.rk) | reinterpret_cast<uintptr_t>(p.rv)) & 15) == 0 &&
         ((p.r_sb | p.r_st | p.r_sh) & 7) == 0;
}

template <bool BF>
__device__ __forceinline__ uint32_t pack16x2(float lo, float hi) {
  uint32_t r;
  if constexpr (BF) asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  else asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

template <bool BF>
__device__ __forceinline__ float2 unpack16x2(uint32_t w) {
  if constexpr (BF) return make_float2(bf16lo(w), bf16hi(w));
  else return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

// D[16x8] = A[16x16] B[16x8] + D with A rows 8-15 zero: only D rows 0-7 (d0, d1) are kept.
template <bool BF>
__device__ __forceinline__ void mma_k16_top(float& d0, float& d1, uint32_t a0, uint32_t a2, uint32_t b0,
                                            uint32_t b1) {
  float x2, x3;
  const uint32_t z = 0u;
  const float zf = 0.f;
  if constexpr (BF)
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%10,%10};"
        : "+f"(d0), "+f"(d1), "=f"(x2), "=f"(x3)
        : "r"(a0), "r"(z), "r"(a2), "r"(z), "r"(b0), "r"(b1), "f"(zf));
  else
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%10,%10};"
        : "+f"(d0), "+f"(d1), "=f"(x2), "=f"(x3)
        : "r"(a0), "r"(z), "r"(a2), "r"(z), "r"(b0), "r"(b1), "f"(zf));
}

// D[16x8] = A[16x8] B[8x8] + D, A rows 8-15 zero.
template <bool BF>
__device__ __forceinline__ void mma_k8_top(float& d0, float& d1, uint32_t a0, uint32_t b0) {
  float x2, x3;
  const uint32_t z = 0u;
  const float zf = 0.f;
  if constexpr (BF)
    asm("mma.sync.aligned.m16n8k8.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%7,%7};"
        : "+f"(d0), "+f"(d1), "=f"(x2), "=f"(x3)
        : "r"(a0), "r"(z), "r"(b0), "f"(zf));
  else
    asm("mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%7,%7};"
        : "+f"(d0), "+f"(d1), "=f"(x2), "=f"(x3)
        : "r"(a0), "r"(z), "r"(b0), "f"(zf));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

// Stage window chunk ch (tokens t0 + 8 ch ..) of pair (b, h) into this warp's ring: 8 key rows
// then 8 value rows at pitch WIN_ROW, by cp.async, zero-filled past the window's end.
__device__ __forceinline__ void v3_window_stage(const DecodeParams& p, int b, int h, int64_t t0, int ntok, int ch,
                                                uint8_t* ring) {
  const int lane = threadIdx.x & 31;
  const int64_t tb = t0 + int64_t(ch) * 8;
  const int nvalid = min(8, ntok - ch * 8);
  const int64_t base = b * p.r_sb + h * p.r_sh;
  const uint32_t ks_s = smem_u32(ring);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int i = lane + 32 * k, tok = (i >> 4) & 7, c16 = i & 15;
    const uint16_t* row = static_cast<const uint16_t*>(k < 4 ? p.rk : p.rv) + base + (tb + min(tok, nvalid - 1)) * p.r_st;
    cp_async16(ks_s + (i >> 4) * WIN_ROW + c16 * 16, row + c16 * 8, tok < nvalid ? 16u : 0u);
  }
}

// The window tokens [t0, t0 + ntok) of pair (b, h) for this warp; writes the warp's merge record
// (acc[GM][D], then (m, l) per head, natural-log units) at rec.  ring: >= 16 * WIN_ROW bytes of
// this warp's shared memory, free for the duration.  Key and value rows go to shared memory by
// cp.async (zero-filled past the window's end), so no registers are held while they load; the
// caller has staged the warp's first chunk (v3_window_stage, chunk wid) before loading the query
// rows, so that the two loads overlap.
template <int GM, int WARPS, bool BF>
__device__ __forceinline__ void v3_window_mma(const DecodeParams& p, const float* qs, int b, int h, int64_t t0,
                                              int ntok, uint8_t* ring, float* rec) {
  constexpr int D = 128;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  const int G = p.G;
  float m = -INFINITY, l = 0.f;  // l: this lane's partial row sum
  float acc[16][2];
#pragma unroll
  for (int j = 0; j < 16; ++j) acc[j][0] = acc[j][1] = 0.f;
  const uint32_t ks_s = smem_u32(ring), vs_s = ks_s + 8 * WIN_ROW;  // shared-window addresses
  const uint32_t ks_o = uint32_t(ring - sm);                        // offset for lds64
  const float scale = p.scale;
  for (int ch = wid; ch * 8 < ntok; ch += WARPS) {
    const int nvalid = min(8, ntok - ch * 8);
    if (ch != wid) v3_window_stage(p, b, h, t0, ntok, ch, ring);  // (the first chunk: by the caller)
    cp_async_wait_all();
    __syncwarp();
    // scores of head gid for tokens 2 tig, 2 tig + 1
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      float4 q4 = make_float4(0.f, 0.f, 0.f, 0.f);
      if (gid < GM) q4 = *reinterpret_cast<const float4*>(qs + gid * D + 32 * tig + 4 * ks);
      const uint2 kb = lds64(ks_o + gid * WIN_ROW + 64 * tig + 8 * ks);
      mma_k16_top<BF>(s0, s1, pack16x2<BF>(q4.x, q4.y), pack16x2<BF>(q4.z, q4.w), kb.x, kb.y);
    }
    // online softmax (the 4 lanes of group gid hold head gid)
    const float x0 = (2 * tig < nvalid) ? s0 * scale : -INFINITY;
    const float x1 = (2 * tig + 1 < nvalid) ? s1 * scale : -INFINITY;
    float cm = fmaxf(x0, x1);
    cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 1));
    cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 2));
    const float mn = fmaxf(m, cm);
    const float alpha = expf(m - mn);
    const float p0 = expf(x0 - mn), p1 = expf(x1 - mn);
    m = mn;
    l = l * alpha + (p0 + p1);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      acc[j][0] *= alpha;
      acc[j][1] *= alpha;
    }
    const uint32_t phi = pack16x2<BF>(p0, p1);
    const float2 ph = unpack16x2<BF>(phi);
    const uint32_t plo = pack16x2<BF>(p0 - ph.x, p1 - ph.y);
#pragma unroll
    for (int j4 = 0; j4 < 4; ++j4) {
      uint32_t vb[4];
      ldsm_x4_trans(vs_s + (lane & 7) * WIN_ROW + (4 * j4 + (lane >> 3)) * 16, vb);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        mma_k8_top<BF>(acc[4 * j4 + u][0], acc[4 * j4 + u][1], phi, vb[u]);
        mma_k8_top<BF>(acc[4 * j4 + u][0], acc[4 * j4 + u][1], plo, vb[u]);
      }
    }
    __syncwarp();  // staging area free for the next chunk
  }
  l += __shfl_xor_sync(0xffffffffu, l, 1);
  l += __shfl_xor_sync(0xffffffffu, l, 2);
  if (gid < GM) {  // (the record overwrites the staging area: every lane is past its last read)
    const bool live = gid < G;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float2 v = make_float2(0.f, 0.f);
      if (live) v = make_float2(acc[j][0], acc[j][1]);
      *reinterpret_cast<float2*>(rec + gid * D + 8 * j + 2 * tig) = v;
    }
    if (tig == 0) {
      rec[GM * D + gid * 2] = live ? m : -INFINITY;
      rec[GM * D + gid * 2 + 1] = live ? l : 0.f;
    }
  }
}

// The stream-K partition (what decode_plan_kernel writes) computed by one CTA into shared
// memory: prefix cost of every segment, then total and per-CTA slice.  Block-wide scan.
__device__ void v3_plan(const DecodeParams& p, int64_t* plan, int64_t* scratch /* [33] */, int* ntab) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (threadIdx.x == 0) scratch[32] = 0;
  __syncthreads();
  for (int base = 0; base < p.n_seg; base += blockDim.x) {
    const int s = base + threadIdx.x;
    const int n = (s < p.n_seg) ? seg_tokens(p, s) : 0;
    if (s < p.n_seg) ntab[s] = n;
    const int64_t c = (int64_t(n) * seg_cost(s) + 15) & ~int64_t(15);
    int64_t x = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) scratch[wid] = x;
    __syncthreads();
    if (wid == 0) {
      int64_t w = lane < nw ? scratch[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int64_t y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      if (lane < nw) scratch[lane] = w;
    }
    __syncthreads();
    const int64_t excl = scratch[32] + x - c + (wid ? scratch[wid - 1] : 0);
    if (s < p.n_seg) plan[s] = excl;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) scratch[32] = excl + c;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const int64_t total = scratch[32];
    plan[p.n_seg] = total;
    int64_t per = (total + gridDim.x - 1) / gridDim.x;
    per = (per + 15) & ~int64_t(15);
    if (per < MIN_SLICE) per = MIN_SLICE;
    plan[p.n_seg + 1] = per;
  }
  __syncthreads();
}

// CTAs c0..c1 wrote a partial slot for segment s (none if c1 < c0).
// Tokens of segment s: from the in-kernel table in single-launch mode (ntab), else from global.
__device__ __forceinline__ int v3_ntok(const DecodeParams& p, const int* ntab, int s) {
  return ntab ? ntab[s] : seg_tokens(p, s);
}

__device__ __forceinline__ void v3_seg_ctas(const DecodeParams& p, const int64_t* plan, const int* ntab, int s, int& c0,
                                            int& c1) {
  const int64_t per = plan[p.n_seg + 1];
  const int n = v3_ntok(p, ntab, s);
  const int64_t S = plan[s];
  c0 = int(S / per);
  c1 = n ? int((S + int64_t(n - 1) * seg_cost(s)) / per) : c0 - 1;
}

// Merge every partial slot of pair (b, h) into the outputs (what decode_merge_kernel does for
// one pair), reading other CTAs' slots through L2.  Three passes, so that no thread waits on a
// chain of dependent loads: every slot's (m, l) into shared memory; per head (one warp each) the
// maximum M, the slot factors exp(m - M) and the sum L; then the value sums, each thread taking
// four dims of one head over a share of the slots (8-byte loads, all independent), the shares
// added through shared memory.  fsc: shared scratch of FINAL_SCRATCH(G, slots) floats, not
// touched when the pair has no slots.  All threads of the CTA; ends with a CTA barrier when the
// pair has slots.

__device__ void v3_final_merge(const DecodeParams& p, const int64_t* plan, const int* ntab, int pair, float* fsc) {
  constexpr int D = 128;
  const int b = pair / p.Hkv, h = pair - b * p.Hkv;
  const int G = p.G;
  const int slot_f = G * (D + 2);
  int c0[2], c1[2];
  for (int k = 0; k < 2; ++k) v3_seg_ctas(p, plan, ntab, pair * 2 + k, c0[k], c1[k]);
  const int nh = c1[0] - c0[0] + 1, nt = nh + (c1[1] - c0[1] + 1);
  if (nt == 0) {  // nobody attends this pair: zero output, empty partials
    for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
      const int g = i / D, d = i - g * D, hq = h * G + g;
      if (p.partial_out) {
        float* po = p.partial_out + (int64_t(b) * p.Hq + hq) * (2 * D + 2);
        po[d] = po[D + d] = 0.f;
        if (d == 0) {
          po[2 * D] = -INFINITY;
          po[2 * D + 1] = 0.f;
        }
      }
      if (p.out) store_elem(p.out, p.q_dtype, b * p.o_sb + hq * p.o_sh + d, 0.f);
    }
    return;
  }
  auto slot_ptr = [&](int j) -> const float* {
    const int k = j < nh ? 0 : 1;
    const int c = k ? c0[1] + (j - nh) : c0[0] + j;
    return p.slots + int64_t(c + pair * 2 + k) * slot_f;
  };
  float* fm = fsc;                  // [nt][G]: m, then exp(m - M)
  float* fl = fsc + nt * G;         // [nt][G]: l
  float* ML = fl + nt * G;          // [G] M, [G] L
  float* red = fsc + ((2 * G * (nt + 1) + 3) & ~3);  // [512][8]: per-thread value shares (4 history, 4 window)
  // value shares: quad q (head q / 32, dims 4 (q % 32) ..), slots j = part, part + R, ...; the
  // first 8 slots of every share are requested before the (m, l) pass, so both loads overlap
  const int quads = G * (D / 4);
  const int R = blockDim.x / quads;  // >= 2 for G <= 8; threads past R * quads only add up
  const bool sharer = int(threadIdx.x) < R * quads;
  const int q = threadIdx.x % quads, part = threadIdx.x / quads;
  const int g = q / (D / 4), d4 = (q - g * (D / 4)) * 4;
  float4 v[8];
  auto load_batch = [&](int j0) {
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int j = j0 + u * R;
      v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (sharer && j < nt) {  // a slot is 130 G floats: 8-byte aligned for every G, 16-byte only for even G
        const float2* sp = reinterpret_cast<const float2*>(slot_ptr(j) + g * D + d4);
        const float2 x = __ldcg(sp), y = __ldcg(sp + 1);
        v[u] = make_float4(x.x, x.y, y.x, y.y);
      }
    }
  };
  load_batch(part);
  for (int k = threadIdx.x; k < nt * G; k += blockDim.x) {
    const int j = k / G, gg = k - j * G;
    const float* sl = slot_ptr(j);
    fm[k] = __ldcg(sl + G * D + 2 * gg);
    fl[k] = __ldcg(sl + G * D + 2 * gg + 1);
  }
  __syncthreads();
  {
    const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int gg = wid; gg < G; gg += blockDim.x >> 5) {
      float M = -INFINITY;
      for (int j = lane; j < nt; j += 32) M = fmaxf(M, fm[j * G + gg]);
      M = warp_max(M);
      float L = 0.f;
      for (int j = lane; j < nt; j += 32) {
        const float m = fm[j * G + gg];
        const float f = (m == -INFINITY) ? 0.f : expf(m - M);
        L += fl[j * G + gg] * f;
        fm[j * G + gg] = f;
      }
      L = warp_sum(L);
      if (lane == 0) {
        ML[gg] = M;
        ML[G + gg] = L;
      }
    }
  }
  __syncthreads();
  if (sharer) {
    float4 ah = make_float4(0.f, 0.f, 0.f, 0.f), ar = ah;
    for (int j0 = part;;) {
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int j = j0 + u * R;
        if (j >= nt) break;
        const float f = fm[j * G + g];
        if (j < nh) {
          ah.x = fmaf(v[u].x, f, ah.x); ah.y = fmaf(v[u].y, f, ah.y);
          ah.z = fmaf(v[u].z, f, ah.z); ah.w = fmaf(v[u].w, f, ah.w);
        } else {
          ar.x = fmaf(v[u].x, f, ar.x); ar.y = fmaf(v[u].y, f, ar.y);
          ar.z = fmaf(v[u].z, f, ar.z); ar.w = fmaf(v[u].w, f, ar.w);
        }
      }
      j0 += 8 * R;
      if (j0 >= nt) break;
      load_batch(j0);
    }
    reinterpret_cast<float4*>(red + threadIdx.x * 8)[0] = ah;
    reinterpret_cast<float4*>(red + threadIdx.x * 8)[1] = ar;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i - g * D;
    const int q = g * (D / 4) + (d >> 2), e = d & 3;
    float acc[2] = {0.f, 0.f};
    for (int r = 0; r < R; ++r) {
      acc[0] += red[(r * quads + q) * 8 + e];
      acc[1] += red[(r * quads + q) * 8 + 4 + e];
    }
    const float M = ML[g], L = ML[G + g];
    const int hq = h * G + g;
    if (p.partial_out) {
      float* po = p.partial_out + (int64_t(b) * p.Hq + hq) * (2 * D + 2);
      po[d] = acc[0];
      po[D + d] = acc[1];
      if (d == 0) {
        po[2 * D] = M;
        po[2 * D + 1] = L;
      }
    }
    if (p.out) {
      float oh = 0.f, orr = 0.f;
      if (L > 0.f) {
        oh = acc[0] / L;
        orr = acc[1] / L;
      }
      // each part is cast to the query dtype, then the parts are summed in it (score.py:70-72)
      const float o = round_dtype(round_dtype(oh, p.q_dtype) + round_dtype(orr, p.q_dtype), p.q_dtype);
      store_elem(p.out, p.q_dtype, b * p.o_sb + hq * p.o_sh + d, o);
    }
  }
  __syncthreads();  // scratch free
}

// Slot arrivals of one CTA, deferred: the CTA notes (pair, slots finished) as it goes and counts
// them at the end of its slice (or when the list is full), one atomicAdd per pair, all pairs at
// once; the CTA whose count completes a pair merges it and resets the counter to 0.  Counter
// values carry the call's epoch (epoch << 32 | slots): every CTA first claims the counters of the
// pairs its slice touches for this call (v3_claim: a counter holding another epoch -- a stale
// or never-zeroed workspace -- restarts at 0; one holding this epoch is left alone), so that the
// arrivals need no compare-and-swap retries.  arr (shared): [0, MAX_ARR) pairs, [MAX_ARR,
// 2 MAX_ARR) counts, then last flags.
constexpr int MAX_ARR = 32;
// Largest grid of the single-launch kernels: the final merge's scratch for a pair with slots
// from every CTA must fit in the warp rings.
constexpr int MAX_GRID_FUSED = 512;

// Claim pair `pair`'s counter for this call (see v3_flush_arrivals): restart it at 0 unless it
// already carries this call's epoch.
__device__ __forceinline__ void v3_claim(const DecodeParams& p, int pair) {
  unsigned long long* cnt = reinterpret_cast<unsigned long long*>(p.pair_cnt + pair);
  unsigned long long old = *reinterpret_cast<volatile unsigned long long*>(cnt);
  while (uint32_t(old >> 32) != p.epoch) {
    const unsigned long long seen = atomicCAS(cnt, old, uint64_t(p.epoch) << 32);
    if (seen == old) break;
    old = seen;
  }
}

// Claim the counters of every pair whose segments meet this CTA's slice [lo, hi) (all threads).
__device__ __forceinline__ void v3_claim_slice(const DecodeParams& p, const int64_t* plan, int sa, int64_t hi) {
  int s0 = sa, s1 = p.n_seg - 1;  // last segment starting below hi
  while (s0 < s1) {
    const int mid = (s0 + s1 + 1) >> 1;
    if (plan[mid] < hi) s0 = mid; else s1 = mid - 1;
  }
  for (int pr = (sa >> 1) + int(threadIdx.x); pr <= (s0 >> 1); pr += blockDim.x) v3_claim(p, pr);
}

__device__ void v3_flush_arrivals(const DecodeParams& p, const int64_t* plan, const int* ntab, int* arr, int n,
                                  float* fsc) {
  __syncthreads();  // every slot store of this CTA, and the list, before the counts
  if (int(threadIdx.x) < n) {
    const int pair = arr[threadIdx.x];
    const uint32_t add = uint32_t(arr[MAX_ARR + threadIdx.x]);
    int expected = 0;
    for (int k = 0; k < 2; ++k) {
      int c0, c1;
      v3_seg_ctas(p, plan, ntab, pair * 2 + k, c0, c1);
      expected += c1 - c0 + 1;
    }
    __threadfence();  // the CTA's slot stores before the count
    unsigned long long* cnt = reinterpret_cast<unsigned long long*>(p.pair_cnt + pair);
    const unsigned long long old = atomicAdd(cnt, (unsigned long long)add);
    bool last = false;
    if (uint32_t(old >> 32) != p.epoch) {
      atomicExch(reinterpret_cast<int*>(p.plan + p.n_seg + 2), 1);  // unclaimed counter: report
    } else {
      last = int(uint32_t(old) + add) == expected;
      if (last) {
        *reinterpret_cast<volatile unsigned long long*>(cnt) = 0ull;
        __threadfence();  // every other slot store is visible before the merge reads them
      }
    }
    arr[2 * MAX_ARR + threadIdx.x] = last;
  }
  __syncthreads();
  for (int i = 0; i < n; ++i)
    if (arr[2 * MAX_ARR + i]) v3_final_merge(p, plan, ntab, arr[i], fsc);
  __syncthreads();  // the list is rewritten next
}

// Note one finished slot of `pair` (all threads, after the slot's CTA barrier).  fsc: shared
// scratch for a flush (the warp rings: free between segments).
__device__ __forceinline__ void v3_note(const DecodeParams& p, const int64_t* plan, const int* ntab, int pair,
                                        int* arr, int& narr, int& last_pair, float* fsc) {
  if (pair == last_pair) {
    if (threadIdx.x == 0) arr[MAX_ARR + narr - 1] += 1;
    return;
  }
  if (narr == MAX_ARR) {
    v3_flush_arrivals(p, plan, ntab, arr, narr, fsc);
    narr = 0;
  }
  if (threadIdx.x == 0) {
    arr[narr] = pair;
    arr[MAX_ARR + narr] = 1;
  }
  ++narr;
  last_pair = pair;
}

template <int GM>
__global__ void __launch_bounds__(V3Cfg<GM>::THREADS, V3Cfg<GM>::CTAS) decode_v3_kernel(DecodeParams p,
                                                                          const uint16_t* __restrict__ cb16) {
  using C = V3Cfg<GM>;
  constexpr int D = 128;
  constexpr int ST = C::STAGES;
  constexpr int WARPS = C::WARPS;
  uint8_t* cb = sm;
  float* qs = reinterpret_cast<float*>(sm + C::CB_BYTES);
  uint8_t* wreg0 = sm + C::CB_BYTES + C::Q_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(wreg0 + WARPS * C::WARP_BYTES);

  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  const int G = p.G;
  uint8_t* wreg = wreg0 + wid * C::WARP_BYTES;                       // ring | s,z | misc
  const uint32_t szs = uint32_t(wreg + ST * STAGE_BYTES - sm);
  float* misc = reinterpret_cast<float*>(wreg + ST * STAGE_BYTES + C::SZ_BYTES);
  float* rec = reinterpret_cast<float*>(wreg);                       // merge record (after the loop)
  uint64_t* wbar = bars + wid * ST;
  if (lane == 0) {
    for (int s = 0; s < ST; ++s) mbar_init(&wbar[s], 4);
    fence_mbar_init();
  }
  uint32_t phase = 0;
  bool failed = false;

  // partition: computed here in single-launch mode, else read from decode_plan_kernel's output
  int64_t* splan = reinterpret_cast<int64_t*>(reinterpret_cast<uint8_t*>(bars) + C::BAR_BYTES);
  int* arrive_flag = reinterpret_cast<int*>(splan + C::MAX_FUSED_SEG + 4 + 33);
  int* sntab = arrive_flag + 4;
  int* arr = sntab + C::MAX_FUSED_SEG;  // deferred slot arrivals
  int narr = 0, last_pair = -1;
  float* fsc = reinterpret_cast<float*>(wreg0);  // final-merge scratch (rings free between segments)
  const int64_t* plan = p.plan;
  const int* ntab = nullptr;
  if (p.fused) {
    // overlapped launch: the next launch on the stream may be scheduled now; its CTAs take an SM
    // only when one of ours has exited
    if (p.pdl) pdl_launch_dependents();
    v3_plan(p, splan, splan + C::MAX_FUSED_SEG + 4, sntab);
    plan = splan;
    ntab = sntab;
  }
  const int64_t total = plan[p.n_seg];
  const int64_t per = plan[p.n_seg + 1];
  const int c = blockIdx.x;
  const int64_t lo = int64_t(c) * per, hi = min(lo + per, total);
  int sa = 0;
  if (lo < hi) {
    int sb_ = p.n_seg - 1;
    while (sa < sb_) {
      const int mid = (sa + sb_) >> 1;
      if (plan[mid + 1] > lo) sb_ = mid; else sa = mid + 1;
    }
  }
  // Overlapped launch: the first history chunks of this CTA are requested before waiting for
  // the previous launch on the stream (the caller promises that launch writes neither the
  // history rows nor the lengths); queries, the window, outputs and the workspace only after.
  if (GM != 4 && lo < hi) {
    // codebook -> shared, entry (block b, code cc) at cc * 256 + sigma(b) * 16; a constant of
    // the launch, so copied before the dependency wait (published by the loop's first barrier)
    for (int u = threadIdx.x; u < 16 * 256; u += blockDim.x) {
      const int blk = u >> 8, cc = u & 255;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (cc < p.nc) v = __ldg(reinterpret_cast<const uint4*>(cb16) + blk * p.nc + cc);
      *reinterpret_cast<uint4*>(cb + cc * 256 + cb_sigma(blk) * 16) = v;
    }
  }
  int pre_s = -1;
  if (p.pdl) {
    if (lo < hi) {
      for (int s = sa; s < p.n_seg && plan[s] < hi; ++s) {
        const int n = v3_ntok(p, ntab, s);
        if (n == 0) continue;
        int64_t t0 = (lo <= plan[s]) ? 0 : (lo - plan[s] + seg_cost(s) - 1) / seg_cost(s);
        int64_t t1 = (hi - plan[s] + seg_cost(s) - 1) / seg_cost(s);
        if (t1 > n) t1 = n;
        if (t0 >= t1) continue;
        if (!(s & 1)) {
          const int pair = s >> 1, b = pair / p.Hkv, h = pair - b * p.Hkv;
          const int ntok = int(t1 - t0), nchunks = (ntok + CH - 1) / CH;
          const int mine = (wid < nchunks) ? (nchunks - 1 - wid) / WARPS + 1 : 0;
          const V3Src src = v3_src(p, b, h, t0);
          if (lane < 4)
            for (int i = 0; i < ST && i < mine; ++i) {
              const int kc = wid + WARPS * i;
              v3_issue(p, src, b, h, t0, min(CH, ntok - kc * CH), kc, wreg + i * STAGE_BYTES, &wbar[i]);
            }
          pre_s = s;
        }
        break;
      }
    }
    pdl_wait();
  }
  if (p.fused) {
    // device error word: cleared by CTA 0 at start; a bounded wait that runs out (seconds later)
    // sets it, and smaq_decode_status reports it
    if (blockIdx.x == 0 && threadIdx.x == 0) *reinterpret_cast<volatile int*>(p.plan + p.n_seg + 2) = 0;
    // pairs nobody attends (no usable history, no window): zero output, empty partials
    for (int pair = blockIdx.x; pair < p.B * p.Hkv; pair += gridDim.x) {
      int e = 0;
      for (int k = 0; k < 2; ++k) {
        int c0, c1;
        v3_seg_ctas(p, plan, ntab, pair * 2 + k, c0, c1);
        e += c1 - c0 + 1;
      }
      if (e == 0) v3_final_merge(p, plan, ntab, pair, fsc);  // (no slots: touches no shared memory)
    }
    if (lo < hi) v3_claim_slice(p, plan, sa, hi);
  }
  if (lo >= hi) return;

  // per-lane constants of the score gather (B column = (token gid>>1, half gid&1), block quad tig)
  V3Lane L;
  {
    const int half = gid & 1;
    L.idx_off = uint32_t((gid >> 1) * 16 + 4 * (2 * half + (tig >> 1)));
    // token t = lane -> k-step ks = t/16, t%16 = 4u + v -> slot 2v + (u&1) + 8(u>>1)
    const int ks = lane >> 4, u = (lane >> 2) & 3, v = lane & 3;
    L.sz_off = uint32_t(2 * (16 * ks + 2 * v + (u & 1) + 8 * (u >> 1)));
#pragma unroll
    for (int kp = 0; kp < 2; ++kp) {
      const int blk = 8 * half + 4 * kp + tig;
      L.base[kp] = uint32_t(cb_sigma(blk) * 16);
      L.sel[kp] = 0x6504u | (uint32_t((tig & 1) * 2 + kp) << 4);
    }
  }
  const uint32_t cb_s = uint32_t(cb - sm);
  const uint32_t ring_s = uint32_t(wreg - sm);
  __syncthreads();

  // warm L2 with what this CTA reads outside its bulk-copied streams (the streams of the whole
  // step do not fit in L2, so these lines would otherwise come from HBM at full load latency):
  // the score-table codebook, and the exact window rows of its window segments
  {
    if (GM == 4 && threadIdx.x < 16) {
      const char* cbase = reinterpret_cast<const char*>(cb16);
      const uint32_t bytes = uint32_t(p.nc) * 16u;  // one block's [nc][8] fp16 rows
      if ((reinterpret_cast<uintptr_t>(cbase) & 15) == 0)
        l2_prefetch(cbase + size_t(threadIdx.x) * bytes, bytes);
    }
    for (int s2 = sa; s2 < p.n_seg && plan[s2] < hi; ++s2) {
      if (threadIdx.x < G && !(s2 & 1)) {  // the pair's query rows
        const int pair = s2 >> 1, b2 = pair / p.Hkv, h2 = pair - b2 * p.Hkv;
        const size_t es = p.q_dtype == SMAQ_F32 ? 4 : 2;
        const char* qrow = static_cast<const char*>(p.q) + (b2 * p.q_sb + int64_t(h2 * G + threadIdx.x) * p.q_sh) * es;
        if ((reinterpret_cast<uintptr_t>(qrow) & 15) == 0) l2_prefetch(qrow, uint32_t(128 * es));
      }
      if (!(s2 & 1) || (p.r_dtype != SMAQ_BF16 && p.r_dtype != SMAQ_F16)) continue;
      const int n2 = v3_ntok(p, ntab, s2);
      if (n2 == 0) continue;
      const int64_t S2 = plan[s2];
      int64_t u0 = (lo <= S2) ? 0 : (lo - S2 + RECENT_COST - 1) / RECENT_COST;
      int64_t u1 = (hi - S2 + RECENT_COST - 1) / RECENT_COST;
      if (u1 > n2) u1 = n2;
      const int pair = s2 >> 1, b2 = pair / p.Hkv, h2 = pair - b2 * p.Hkv;
      for (int64_t i = threadIdx.x; i < 2 * (u1 - u0); i += blockDim.x) {
        const int64_t t = u0 + (i >> 1);
        const uint16_t* base = static_cast<const uint16_t*>((i & 1) ? p.rv : p.rk);
        const char* row = reinterpret_cast<const char*>(base + b2 * p.r_sb + t * p.r_st + h2 * p.r_sh);
        if ((reinterpret_cast<uintptr_t>(row) & 15) == 0) l2_prefetch(row, 256u);
      }
    }
  }
  const float lscale = p.scale * kLog2e;
  for (int s = sa; s < p.n_seg; ++s) {
    const int64_t S = plan[s];
    if (S >= hi) break;
    const int n = v3_ntok(p, ntab, s);
    if (n == 0) continue;
    const int cs = seg_cost(s);
    int64_t t0 = (lo <= S) ? 0 : (lo - S + cs - 1) / cs;
    int64_t t1 = (hi - S + cs - 1) / cs;
    if (t1 > n) t1 = n;
    if (t0 >= t1) continue;
    const int pair = s >> 1, b = pair / p.Hkv, h = pair - b * p.Hkv;
    if ((s & 1) && window_mma_ok(p) && (wid << 3) < int(t1 - t0))
      v3_window_stage(p, b, h, t0, int(t1 - t0), wid, wreg);  // the window rows load with the query rows
    for (int i = threadIdx.x; i < GM * D; i += blockDim.x) {
      const int g = i / D, d = i - g * D;
      qs[i] = g < G ? load_elem(p.q, p.q_dtype, b * p.q_sb + int64_t(h * G + g) * p.q_sh + d) : 0.f;
    }
    if (s & 1) {
      // ---------------- exact recent window: warp w takes 8-token chunks w, w + WARPS, ...
      __syncthreads();  // qs complete
      const int ntok = int(t1 - t0);
      WarpState<GM> ws;
      ws.init();
      // 8 tokens per warp and round: the window is short, so spreading it over every warp
      // keeps its latency (key row loads, then value row loads) to about one round
      if (window_mma_ok(p)) {
        if (p.r_dtype == SMAQ_BF16) v3_window_mma<GM, WARPS, true>(p, qs, b, h, t0, ntok, wreg, rec);
        else v3_window_mma<GM, WARPS, false>(p, qs, b, h, t0, ntok, wreg, rec);
      } else {
        for (int ch = wid; ch * 8 < ntok; ch += WARPS)
          v3_window_chunk<GM>(p, qs, b, h, t0 + int64_t(ch) * 8, min(8, ntok - ch * 8), ws);
#pragma unroll
        for (int g = 0; g < GM; ++g) {
#pragma unroll
          for (int e = 0; e < 4; ++e) rec[g * D + lane * 4 + e] = g < G ? ws.acc[g][e] : 0.f;
          if (lane == 0) {
            rec[GM * D + g * 2] = g < G ? ws.m[g] : -INFINITY;
            rec[GM * D + g * 2 + 1] = g < G ? ws.l[g] : 0.f;
          }
        }
      }
      __syncthreads();
      v3_merge<GM, WARPS>(p, reinterpret_cast<const float*>(wreg0), C::WARP_BYTES / 4, c + s);
      if (p.fused) v3_note(p, plan, ntab, s >> 1, arr, narr, last_pair, fsc);
      continue;
    }

    // ---------------- compressed history
    const int ntok = int(t1 - t0);
    const int nchunks = (ntok + CH - 1) / CH;
    const int mine = (wid < nchunks) ? (nchunks - 1 - wid) / WARPS + 1 : 0;
    const V3Src src = v3_src(p, b, h, t0);
    if (lane < 4 && s != pre_s) {  // (pre_s: already issued before the dependency wait)
      for (int i = 0; i < ST && i < mine; ++i) {
        const int kc = wid + WARPS * i;
        v3_issue(p, src, b, h, t0, min(CH, ntok - kc * CH), kc, wreg + i * STAGE_BYTES, &wbar[i]);
      }
    }
    if constexpr (GM == 4) {
      // this pair's score table (see v3_chunk_lut); built while the first chunks load.  Thread t
      // fills block t % 16 for codes t / 16 + 32 k; its fp16 codebook rows are requested before
      // the barrier that publishes the query rows.
      {
        constexpr int NK = 256 / (C::THREADS >> 4);
        const int blk = threadIdx.x & 15, c0 = threadIdx.x >> 4;
        const uint4* cb4 = reinterpret_cast<const uint4*>(cb16) + int64_t(blk) * p.nc;
        uint4 cw[NK];
#pragma unroll
        for (int k = 0; k < NK; ++k) {
          const int cc = c0 + k * (C::THREADS >> 4);
          cw[k] = cc < p.nc ? __ldg(cb4 + cc) : make_uint4(0u, 0u, 0u, 0u);
        }
        __syncthreads();  // qs complete
        float qv[4][8];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const float4 a0 = *reinterpret_cast<const float4*>(qs + g * D + blk * 8);
          const float4 a1 = *reinterpret_cast<const float4*>(qs + g * D + blk * 8 + 4);
          const float q8[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
          for (int e = 0; e < 8; ++e) qv[g][e] = q8[e] * lscale;
        }
#pragma unroll
        for (int k = 0; k < NK; ++k) {
          const int cc = c0 + k * (C::THREADS >> 4);
          const uint32_t hw[4] = {cw[k].x, cw[k].y, cw[k].z, cw[k].w};
          float x[8];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hw[e]));
            x[2 * e] = f.x;
            x[2 * e + 1] = f.y;
          }
          float r4[4];
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            float acc4 = qv[g][0] * x[0];
#pragma unroll
            for (int e = 1; e < 8; ++e) acc4 = fmaf(qv[g][e], x[e], acc4);
            r4[g] = acc4;
          }
          *reinterpret_cast<float4*>(cb + (cc * 16 + blk) * 16) = make_float4(r4[0], r4[1], r4[2], r4[3]);
        }
      }
    }
    __syncthreads();  // qs and codebook complete
    // A fragments of the score MMA: rows (head gid, half 0) and (head gid, half 1); k-step ks
    // covers dims 8*(8*half + 4*(ks>>1) + tig) + 4*(ks&1) + {0,1 | 2,3}
    uint32_t qa[4][4];
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      if constexpr (GM == 4) break;
      const int kp = ks >> 1, s4 = 4 * (ks & 1);
      const float* q0 = qs + gid * D + 8 * (4 * kp + tig) + s4;
      const float* q1 = qs + gid * D + 8 * (8 + 4 * kp + tig) + s4;
      qa[ks][0] = pack_f16x2(q0[0], q0[1]);
      qa[ks][1] = pack_f16x2(q1[0], q1[1]);
      qa[ks][2] = pack_f16x2(q0[2], q0[3]);
      qa[ks][3] = pack_f16x2(q1[2], q1[3]);
    }

    float acc[8][4];
#pragma unroll
    for (int m = 0; m < 8; ++m)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[m][e] = 0.f;
    float zacc[4] = {0.f, 0.f, 0.f, 0.f};
    float mrun = -INFINITY, lrun = 0.f;
    float mref[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY}, lsum[4] = {0.f, 0.f, 0.f, 0.f};
    const uint32_t pb = uint32_t(reinterpret_cast<uint8_t*>(misc) - sm);
    LutLane X;
    X.xl = uint32_t(lane & 15) << 4;
    X.sel = 0u;
#pragma unroll
    for (int i = 0; i < 4; ++i) X.sel |= uint32_t(i ^ (lane & 3)) << (4 * i);
    X.swp8 = (lane & 8) != 0;
    X.swp4 = (lane & 4) != 0;
    for (int i = 0; i < mine; ++i) {
      const int stg = i % ST;
      uint8_t* stage = wreg + stg * STAGE_BYTES;
      if (!failed && !mbar_wait(&wbar[stg], (phase >> stg) & 1u)) failed = true;
      phase ^= 1u << stg;
      const int nv = min(CH, ntok - (wid + WARPS * i) * CH);
      if constexpr (GM == 4) {
        if (nv == CH)
          v3_chunk_lut<true>(ring_s + stg * STAGE_BYTES, szs, pb, L, X, nv, acc, zacc, mref, lsum);
        else
          v3_chunk_lut<false>(ring_s + stg * STAGE_BYTES, szs, pb, L, X, nv, acc, zacc, mref, lsum);
      } else {
        if (nv == CH)
          v3_chunk<true>(ring_s + stg * STAGE_BYTES, cb_s, szs, L, qa, G, lscale, nv, acc, zacc, mrun, lrun);
        else
          v3_chunk<false>(ring_s + stg * STAGE_BYTES, cb_s, szs, L, qa, G, lscale, nv, acc, zacc, mrun, lrun);
      }
      if (lane < 4 && i + ST < mine) {
        const int kc = wid + WARPS * (i + ST);
        v3_issue(p, src, b, h, t0, min(CH, ntok - kc * CH), kc, stage, &wbar[stg]);
      }
    }

    // ---- warp epilogue: per head (m, l), then the value sums -> record (the zero-point terms
    // were folded into acc chunk by chunk)
    if constexpr (GM == 4) {
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        const float l = warp_sum(lsum[g]);
        if (lane == 0) {
          rec[GM * D + g * 2] = (mine && mref[g] != -INFINITY) ? (mref[g] - kShift) * kLn2 : -INFINITY;
          rec[GM * D + g * 2 + 1] = l;
        }
      }
      // columns 4..7 hold the lo parts of heads 0..3: add them to columns 0..3
#pragma unroll
      for (int m = 0; m < 8; ++m)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[m][e] += __shfl_xor_sync(0xffffffffu, acc[m][e], 2);
    } else {
      float l = lrun;
      l += __shfl_xor_sync(0xffffffffu, l, 1);
      l += __shfl_xor_sync(0xffffffffu, l, 2);
      if (tig == 0 && gid < GM) {
        rec[GM * D + gid * 2] = (mine && mrun != -INFINITY) ? (mrun - kShift) * kLn2 : -INFINITY;  // natural log
        rec[GM * D + gid * 2 + 1] = l;
      }
    }
    {
      const int ga = 2 * tig, gb = 2 * tig + 1;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int d0 = 32 * j + 4 * gid + 2 * hh;       // row gid -> code r = 2hh; row gid+8 -> 2hh+1
          const float s0 = hh ? 1048576.0f : 16777216.0f;  // 2^24 * 4^-r
          const float s1 = hh ? 262144.0f : 4194304.0f;    // 2^24 * 4^-(r+1)
          if (ga < GM) {
            rec[ga * D + d0] = acc[2 * j + hh][0] * s0;
            rec[ga * D + d0 + 1] = acc[2 * j + hh][2] * s1;
          }
          if (gb < GM) {
            rec[gb * D + d0] = acc[2 * j + hh][1] * s0;
            rec[gb * D + d0 + 1] = acc[2 * j + hh][3] * s1;
          }
        }
      }
    }
    __syncthreads();
    v3_merge<GM, WARPS>(p, reinterpret_cast<const float*>(wreg0), C::WARP_BYTES / 4, c + s);
    if (p.fused) v3_note(p, plan, ntab, s >> 1, arr, narr, last_pair, fsc);
  }
  if (p.fused && narr) v3_flush_arrivals(p, plan, ntab, arr, narr, fsc);
  if (failed && lane == 0) atomicExch(reinterpret_cast<int*>(p.plan + p.n_seg + 2), 1);
}

// =====================================================================================
// Scalar 3/4-bit keys (SMAQQuantizer.attention_score, smaq/quantizer.py:154-184: scores =
// (q @ E_inv^T) . centroids[codes] * norm * scale) with 2-bit group-32 values, decode layout,
// bf16/fp16 queries, G <= 8.  Same partition, window, slots and merge as decode_v3_kernel.
//  * Scores on the tensor cores (mma.m16n8k16, rows = 16 tokens, columns = 8 query heads,
//    k = 16 dims).  The rotated query is split q = q_hi + q_lo (fp16) and so is every centroid
//    value (c = c_hi + c_lo); three MMAs per k-step (q_hi c_hi + q_lo c_hi + q_hi c_lo) keep
//    the products to ~2^-21 relative, i.e. fp32-class scores.
//  * A operands come straight from the code bytes: one byte = two dims = one A register, looked
//    up in a shared 256-entry table of (c_hi pair, c_lo pair), replicated per lane so every
//    lookup is conflict-free.  The decode layout puts the 16 code bytes one lane needs
//    for a token next to each other.
//  * The norm, the softmax (reference maximum per head that only moves up) and P.V follow the
//    block-VQ kernel.
// =====================================================================================
constexpr int SK_STAGE = CH * 64 + CH * 32 + CH * 8 + CH * 8 + CH * 2;  // codes | values | scales | zeros | norms
constexpr int SK_V = CH * 64, SK_S = CH * 96, SK_Z = CH * 104, SK_N = CH * 112;

struct SCfg {
  static constexpr int WARPS = 16;
  static constexpr int THREADS = WARPS * 32;
  static constexpr int STAGES = 2;
  static constexpr int TAB_BYTES = 2 * 256 * 32 * 4;                 // c_hi, c_lo tables x 32 lanes
  static constexpr int Q_BYTES = 8 * 128 * 4;                       // fp32 query rows (rotation, window)
  static constexpr int B_BYTES = 8 * 32 * 16;                       // B fragments [ks][lane]
  static constexpr int SZ_BYTES = 2 * 4 * CH * 2;
  static constexpr int PB_BYTES = 8 * 64;                           // p, fp16, [head][k-slot]
  static constexpr int WARP_BYTES = STAGES * SK_STAGE + SZ_BYTES + PB_BYTES;
  static constexpr int BAR_BYTES = WARPS * STAGES * 8;
  static constexpr int MAX_FUSED_SEG = 1024;
  static constexpr int PLAN_BYTES = (MAX_FUSED_SEG + 4) * 8 + 33 * 8 + 16 + MAX_FUSED_SEG * 4 + 3 * 32 * 4;
  static constexpr int SMEM = TAB_BYTES + Q_BYTES + B_BYTES + WARPS * WARP_BYTES + BAR_BYTES + PLAN_BYTES;
  static_assert(8 * (128 + 2) * 4 <= STAGES * SK_STAGE, "merge record must fit in a ring");
  static_assert(16 * WIN_ROW <= STAGES * SK_STAGE, "window rows must fit in a ring");
  static_assert(final_scratch_floats(8, 2 * 512) * 4 <= WARPS * WARP_BYTES, "final-merge scratch");
  static_assert(SMEM <= 232448, "shared memory budget");
};

template <bool FULL>
__device__ __forceinline__ void sk_chunk(uint32_t st, uint32_t szs, uint32_t pb, uint32_t bfr, uint32_t tab_l,
                                         const V3Lane& L, int nv, float (&acc)[8][4], float (&zacc)[4],
                                         float (&mref)[2], float (&lsum)[2]) {
  const int lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  // ---- value scales / zeros as fp16 in k-slot order (one token per lane)
  {
    uint2 s2 = lds64(st + SK_S + lane * 8);
    uint2 z2 = lds64(st + SK_Z + lane * 8);
    if (!FULL && lane >= nv) s2 = z2 = make_uint2(0u, 0u);
    const uint32_t sp0 = pack_f16x2(bf16lo(s2.x), bf16hi(s2.x)), sp1 = pack_f16x2(bf16lo(s2.y), bf16hi(s2.y));
    const uint32_t zp0 = pack_f16x2(bf16lo(z2.x), bf16hi(z2.x)), zp1 = pack_f16x2(bf16lo(z2.y), bf16hi(z2.y));
    const uint32_t o = szs + L.sz_off;
    sts16(o + 0, uint16_t(sp0)); sts16(o + 64, uint16_t(sp0 >> 16));
    sts16(o + 128, uint16_t(sp1)); sts16(o + 192, uint16_t(sp1 >> 16));
    sts16(o + 256, uint16_t(zp0)); sts16(o + 320, uint16_t(zp0 >> 16));
    sts16(o + 384, uint16_t(zp1)); sts16(o + 448, uint16_t(zp1 >> 16));
  }
  // ---- scores: two 16-token tiles; thread holds tokens 16T + gid (+8), heads 2tig, 2tig+1
  float d[2][4];
#pragma unroll
  for (int T = 0; T < 2; ++T) {
    // code bytes of tokens 16T + gid and 16T + gid + 8 (the lane's 16 contiguous bytes each)
    const uint4 c0 = lds128(st + (16 * T + gid) * 64 + 16 * tig);
    const uint4 c1 = lds128(st + (16 * T + gid + 8) * 64 + 16 * tig);
#pragma unroll
    for (int e = 0; e < 4; ++e) d[T][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const uint4 bq = lds128(bfr + (ks * 32 + lane) * 16);  // b0 hi, b1 hi, b0 lo, b1 lo
      uint32_t ah[4], al[4];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const uint4& cw = r ? c1 : c0;
        const uint32_t wv = (ks >> 1) == 0 ? cw.x : (ks >> 1) == 1 ? cw.y : (ks >> 1) == 2 ? cw.z : cw.w;
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {  // byte 2ks + h2 of the lane's 16: dims 16ks + 8h2 + 2tig, +1
          const uint32_t b256 = __byte_perm(wv, 0, 0x4404 | (uint32_t(2 * (ks & 1) + h2) << 4));  // byte * 256
          const uint2 e2 = lds64(b256 | tab_l);   // (c_hi pair, c_lo pair)
          ah[r + 2 * h2] = e2.x;
          al[r + 2 * h2] = e2.y;
        }
      }
      mma_f16_16816(d[T], ah, bq.x, bq.y);   // q_hi . c_hi
      mma_f16_16816(d[T], ah, bq.z, bq.w);   // q_lo . c_hi
      mma_f16_16816(d[T], al, bq.x, bq.y);   // q_hi . c_lo
    }
  }
  // times the token's norm; masked tokens -inf
  float s[2][4];
#pragma unroll
  for (int T = 0; T < 2; ++T) {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int t = 16 * T + gid + 8 * r;
      const float nrm = __uint_as_float(uint32_t(*reinterpret_cast<const uint16_t*>(sm + st + SK_N + 2 * t)) << 16);
      const bool ok = FULL || t < nv;
      s[T][2 * r] = ok ? d[T][2 * r] * nrm : -INFINITY;
      s[T][2 * r + 1] = ok ? d[T][2 * r + 1] * nrm : -INFINITY;
    }
  }
  // ---- softmax for heads 2tig (c = 0) and 2tig + 1 (c = 1) over the warp's 32 tokens
  bool grow = false;
#pragma unroll
  for (int T = 0; T < 2; ++T)
#pragma unroll
    for (int e = 0; e < 4; ++e) grow |= s[T][e] > mref[e & 1];
  if (__any_sync(0xffffffffu, grow)) {
    float al2[2];
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      float mx = fmaxf(fmaxf(s[0][c], s[0][c + 2]), fmaxf(s[1][c], s[1][c + 2]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
      const float mn = fmaxf(mref[c], mx);
      al2[c] = fast_exp2(mref[c] - mn);
      mref[c] = mn;
      lsum[c] *= al2[c];
    }
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      acc[m][0] *= al2[0]; acc[m][1] *= al2[1]; acc[m][2] *= al2[0]; acc[m][3] *= al2[1];
    }
  }
  // p -> fp16 in the P.V B layout: row = head, k-slot of token t (see V3Lane::sz_off)
#pragma unroll
  for (int T = 0; T < 2; ++T) {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int t = 16 * T + gid + 8 * r;
      const int u = (t >> 2) & 3, v = t & 3;
      const uint32_t slot = uint32_t(2 * (16 * T + 2 * v + (u & 1) + 8 * (u >> 1)));
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const float pv = fast_exp2(s[T][2 * r + c] - (mref[c] - kShift));
        lsum[c] += pv;
        sts16(pb + (2 * tig + c) * 64 + slot, __half_as_ushort(__float2half_rn(pv)));
      }
    }
  }
  __syncwarp();
  // ---- P.V: as the block-VQ kernel, all 8 head columns live
#pragma unroll
  for (int ks = 0; ks < 2; ++ks) {
    const uint32_t p01 = lds32(pb + gid * 64 + ks * 32 + tig * 4);
    const uint32_t p23 = lds32(pb + gid * 64 + ks * 32 + tig * 4 + 16);
    const uint32_t sb = szs + ks * 32 + tig * 4;
    {
      uint32_t az[4] = {0u, 0u, 0u, 0u};
      if (gid < 4) {
        az[0] = lds32(sb + 256 + gid * 64);
        az[2] = lds32(sb + 256 + gid * 64 + 16);
      }
      mma_f16_16816(zacc, az, p01, p23);
    }
    const uint32_t vb = st + SK_V + (16 * ks + tig) * 32 + gid * 4;
    const uint32_t w0 = lds32(vb), w1 = lds32(vb + 128), w2 = lds32(vb + 256), w3 = lds32(vb + 384);
    const uint32_t u01 = __byte_perm(w0, w1, 0x5410), v01 = __byte_perm(w0, w1, 0x7632);
    const uint32_t u23 = __byte_perm(w2, w3, 0x5410), v23 = __byte_perm(w2, w3, 0x7632);
    const uint32_t x01[4] = {u01, u01 >> 8, v01, v01 >> 8};
    const uint32_t x23[4] = {u23, u23 >> 8, v23, v23 >> 8};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t sc0 = lds32(sb + j * 64), sc1 = lds32(sb + j * 64 + 16);
      const uint32_t bh0 = hmul2(p01, sc0), bh1 = hmul2(p23, sc1);
      const uint32_t bl0 = two_prod_lo(p01, sc0, bh0), bl1 = two_prod_lo(p23, sc1, bh1);
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const uint32_t m0 = 0x00030003u << (4 * hh), m1 = 0x00030003u << (4 * hh + 2);
        const uint32_t a[4] = {x01[j] & m0, x01[j] & m1, x23[j] & m0, x23[j] & m1};
        mma_f16_16816(acc[2 * j + hh], a, bh0, bh1);
        mma_f16_16816(acc[2 * j + hh], a, bl0, bl1);
      }
    }
  }
  fold_zero(acc, zacc, true);
  fence_proxy_async_smem();  // the stage is refilled by a bulk copy after this barrier
  __syncwarp();
}

__global__ void __launch_bounds__(SCfg::THREADS, 1) decode_s_kernel(DecodeParams p) {
  using C = SCfg;
  constexpr int D = 128, GM = 8;
  constexpr int ST = C::STAGES;
  constexpr int WARPS = C::WARPS;
  uint8_t* tab = sm;                                                   // [256][32] (hi, lo) fp16 pairs
  float* qs = reinterpret_cast<float*>(sm + C::TAB_BYTES);
  uint8_t* bfrag = sm + C::TAB_BYTES + C::Q_BYTES;
  uint8_t* wreg0 = bfrag + C::B_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(wreg0 + WARPS * C::WARP_BYTES);

  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  const int G = p.G;
  uint8_t* wreg = wreg0 + wid * C::WARP_BYTES;                       // ring | s,z | p
  const uint32_t szs = uint32_t(wreg + ST * SK_STAGE - sm);
  const uint32_t pbuf = szs + C::SZ_BYTES;
  float* misc = reinterpret_cast<float*>(sm + pbuf);                  // zero terms after the loop
  float* rec = reinterpret_cast<float*>(wreg);
  uint64_t* wbar = bars + wid * ST;
  if (lane == 0) {
    for (int s = 0; s < ST; ++s) mbar_init(&wbar[s], 5);
    fence_mbar_init();
  }
  uint32_t phase = 0;
  bool failed = false;

  int64_t* splan = reinterpret_cast<int64_t*>(reinterpret_cast<uint8_t*>(bars) + C::BAR_BYTES);
  int* arrive_flag = reinterpret_cast<int*>(splan + C::MAX_FUSED_SEG + 4 + 33);
  int* sntab = arrive_flag + 4;
  int* arr = sntab + C::MAX_FUSED_SEG;  // deferred slot arrivals
  int narr = 0, last_pair = -1;
  float* fsc = reinterpret_cast<float*>(wreg0);  // final-merge scratch (rings free between segments)
  const int64_t* plan = p.plan;
  const int* ntab = nullptr;
  if (p.fused) {
    // overlapped launch: the next launch on the stream may be scheduled now
    if (p.pdl) pdl_launch_dependents();
    v3_plan(p, splan, splan + C::MAX_FUSED_SEG + 4, sntab);
    plan = splan;
    ntab = sntab;
  }
  // code byte -> (c_hi[lo nibble], c_hi[hi nibble]) | (c_lo pair), replicated per lane so a
  // warp's 32 lookups hit 32 distinct bank pairs: entry (byte, lane) at byte * 256 + lane * 8
  {
    const int bits = p.nc == 8 ? 3 : 4;
    const uint32_t mask = (1u << bits) - 1u;
    for (int i = threadIdx.x; i < 256 * 32; i += blockDim.x) {
      const int by = i >> 5;
      const float c0v = __ldg(p.cent + (by & mask)), c1v = __ldg(p.cent + ((by >> bits) & mask));
      const __half h0 = __float2half_rn(c0v), h1 = __float2half_rn(c1v);
      const __half l0 = __float2half_rn(c0v - __half2float(h0)), l1 = __float2half_rn(c1v - __half2float(h1));
      *reinterpret_cast<uint2*>(tab + i * 8) =
          make_uint2(uint32_t(__half_as_ushort(h0)) | (uint32_t(__half_as_ushort(h1)) << 16),
                     uint32_t(__half_as_ushort(l0)) | (uint32_t(__half_as_ushort(l1)) << 16));
    }
  }
  // overlapped launch: partition and code table above overlap the previous kernel's end;
  // everything below may read its outputs
  if (p.pdl) pdl_wait();
  if (p.fused) {
    // device error word: cleared by CTA 0 at start; a bounded wait that runs out (seconds later)
    // sets it, and smaq_decode_status reports it
    if (blockIdx.x == 0 && threadIdx.x == 0) *reinterpret_cast<volatile int*>(p.plan + p.n_seg + 2) = 0;
    for (int pair = blockIdx.x; pair < p.B * p.Hkv; pair += gridDim.x) {
      int e = 0;
      for (int k = 0; k < 2; ++k) {
        int c0, c1;
        v3_seg_ctas(p, plan, ntab, pair * 2 + k, c0, c1);
        e += c1 - c0 + 1;
      }
      if (e == 0) v3_final_merge(p, plan, ntab, pair, fsc);  // (no slots: touches no shared memory)
    }
  }
  const int64_t total = plan[p.n_seg];
  const int64_t per = plan[p.n_seg + 1];
  const int c = blockIdx.x;
  const int64_t lo = int64_t(c) * per, hi = min(lo + per, total);
  if (lo >= hi) return;

  V3Lane L;
  {
    const int ks = lane >> 4, u = (lane >> 2) & 3, v = lane & 3;
    L.sz_off = uint32_t(2 * (16 * ks + 2 * v + (u & 1) + 8 * (u >> 1)));
  }
  const uint32_t tab_l = uint32_t(lane * 8);
  const uint32_t ring_s = uint32_t(wreg - sm);
  const uint32_t bfr = uint32_t(bfrag - sm);
  __syncthreads();

  int sa = 0, sb_ = p.n_seg - 1;
  while (sa < sb_) {
    const int mid = (sa + sb_) >> 1;
    if (plan[mid + 1] > lo) sb_ = mid; else sa = mid + 1;
  }
  if (p.fused) v3_claim_slice(p, plan, sa, hi);
  const float lscale = p.scale * kLog2e;
  for (int s = sa; s < p.n_seg; ++s) {
    const int64_t S = plan[s];
    if (S >= hi) break;
    const int n = v3_ntok(p, ntab, s);
    if (n == 0) continue;
    const int cs = seg_cost(s);
    int64_t t0 = (lo <= S) ? 0 : (lo - S + cs - 1) / cs;
    int64_t t1 = (hi - S + cs - 1) / cs;
    if (t1 > n) t1 = n;
    if (t0 >= t1) continue;
    const int pair = s >> 1, b = pair / p.Hkv, h = pair - b * p.Hkv;
    if ((s & 1) && window_mma_ok(p) && (wid << 3) < int(t1 - t0))
      v3_window_stage(p, b, h, t0, int(t1 - t0), wid, wreg);  // the window rows load with the query rows
    for (int i = threadIdx.x; i < 8 * D; i += blockDim.x) {
      const int g = i / D, d = i - g * D;
      qs[i] = g < G ? load_elem(p.q, p.q_dtype, b * p.q_sb + int64_t(h * G + g) * p.q_sh + d) : 0.f;
    }
    if (s & 1) {
      __syncthreads();  // qs complete
      const int ntok = int(t1 - t0);
      WarpState<GM> ws;
      ws.init();
      if (window_mma_ok(p)) {
        if (p.r_dtype == SMAQ_BF16) v3_window_mma<GM, WARPS, true>(p, qs, b, h, t0, ntok, wreg, rec);
        else v3_window_mma<GM, WARPS, false>(p, qs, b, h, t0, ntok, wreg, rec);
      } else {
        for (int ch = wid; ch * 8 < ntok; ch += WARPS)
          v3_window_chunk<GM>(p, qs, b, h, t0 + int64_t(ch) * 8, min(8, ntok - ch * 8), ws);
#pragma unroll
        for (int g = 0; g < GM; ++g) {
#pragma unroll
          for (int e = 0; e < 4; ++e) rec[g * D + lane * 4 + e] = g < G ? ws.acc[g][e] : 0.f;
          if (lane == 0) {
            rec[GM * D + g * 2] = g < G ? ws.m[g] : -INFINITY;
            rec[GM * D + g * 2 + 1] = g < G ? ws.l[g] : 0.f;
          }
        }
      }
      __syncthreads();
      v3_merge<GM, WARPS>(p, reinterpret_cast<const float*>(wreg0), C::WARP_BYTES / 4, c + s);
      if (p.fused) v3_note(p, plan, ntab, s >> 1, arr, narr, last_pair, fsc);
      continue;
    }

    // ---------------- compressed history
    const int ntok = int(t1 - t0);
    const int nchunks = (ntok + CH - 1) / CH;
    const int mine = (wid < nchunks) ? (nchunks - 1 - wid) / WARPS + 1 : 0;
    V3Src src;
    {
      const int k = lane < 5 ? lane : 0;
      const uint8_t* base = k == 0 ? p.kcodes
                            : k == 1 ? p.vdata
                            : k == 2 ? static_cast<const uint8_t*>(p.vscales)
                            : k == 3 ? static_cast<const uint8_t*>(p.vzeros)
                                     : static_cast<const uint8_t*>(p.knorms);
      src.row_bytes = k == 0 ? 64u : k == 1 ? 32u : k == 4 ? 2u : 8u;
      src.dst_off = k == 0 ? 0u : k == 1 ? uint32_t(SK_V) : k == 2 ? uint32_t(SK_S) : k == 3 ? uint32_t(SK_Z) : uint32_t(SK_N);
      src.base = p.bt ? base : base + ((int64_t(b) * p.Hkv + h) * p.page_size + t0) * src.row_bytes;
    }
    if (lane < 5) {
      for (int i = 0; i < ST && i < mine; ++i) {
        const int kc = wid + WARPS * i;
        v3_issue(p, src, b, h, t0, min(CH, ntok - kc * CH), kc, wreg + i * SK_STAGE, &wbar[i]);
      }
    }
    __syncthreads();  // qs complete
    // rotated, scaled query q_r[g][j] = scale log2(e) sum_k q[g][k] E_inv[j][k], as fp16 hi + lo,
    // in B-fragment order: entry (ks, lane) = {b0 hi, b1 hi, b0 lo, b1 lo} for head gid, dims
    // 16 ks + 2 tig (+1) and 16 ks + 8 + 2 tig (+1)
    {
      for (int o = threadIdx.x; o < 8 * 32 * 4; o += blockDim.x) {
        // o -> (ks, ln, word): each thread computes the four dims of one B word pair
        const int ks = o >> 7, ln = (o >> 2) & 31, wsel = o & 3;
        const int g = ln >> 2, tg = ln & 3;
        const int dj = 16 * ks + 8 * (wsel & 1) + 2 * tg;  // first of the two dims of this word
        uint32_t word = 0u;
        if (g < G) {
          float r2[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float4* er = reinterpret_cast<const float4*>(p.E_inv + (dj + e) * D);
            const float* qg = qs + g * D;
            float a = 0.f;
#pragma unroll 8
            for (int k4 = 0; k4 < D / 4; ++k4) {
              const float4 ev = __ldg(er + k4);
              a = fmaf(qg[4 * k4], ev.x, a);
              a = fmaf(qg[4 * k4 + 1], ev.y, a);
              a = fmaf(qg[4 * k4 + 2], ev.z, a);
              a = fmaf(qg[4 * k4 + 3], ev.w, a);
            }
            r2[e] = a * lscale;
          }
          if (wsel < 2) {
            word = pack_f16x2(r2[0], r2[1]);
          } else {
            const float h0 = __half2float(__float2half_rn(r2[0])), h1 = __half2float(__float2half_rn(r2[1]));
            word = pack_f16x2(r2[0] - h0, r2[1] - h1);
          }
        }
        *reinterpret_cast<uint32_t*>(bfrag + (ks * 32 + ln) * 16 + wsel * 4) = word;
      }
    }
    __syncthreads();  // B fragments complete

    float acc[8][4];
#pragma unroll
    for (int m = 0; m < 8; ++m)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[m][e] = 0.f;
    float zacc[4] = {0.f, 0.f, 0.f, 0.f};
    float mref[2] = {-INFINITY, -INFINITY}, lsum[2] = {0.f, 0.f};
    for (int i = 0; i < mine; ++i) {
      const int stg = i % ST;
      uint8_t* stage = wreg + stg * SK_STAGE;
      if (!failed && !mbar_wait(&wbar[stg], (phase >> stg) & 1u)) failed = true;
      phase ^= 1u << stg;
      const int nv = min(CH, ntok - (wid + WARPS * i) * CH);
      if (nv == CH)
        sk_chunk<true>(ring_s + stg * SK_STAGE, szs, pbuf, bfr, tab_l, L, nv, acc, zacc, mref, lsum);
      else
        sk_chunk<false>(ring_s + stg * SK_STAGE, szs, pbuf, bfr, tab_l, L, nv, acc, zacc, mref, lsum);
      if (lane < 5 && i + ST < mine) {
        const int kc = wid + WARPS * (i + ST);
        v3_issue(p, src, b, h, t0, min(CH, ntok - kc * CH), kc, stage, &wbar[stg]);
      }
    }
    // ---- warp epilogue: heads 2tig, 2tig+1 -> (m, l); zero terms; value sums -> record
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      float l = lsum[cc];
      l += __shfl_xor_sync(0xffffffffu, l, 4);
      l += __shfl_xor_sync(0xffffffffu, l, 8);
      l += __shfl_xor_sync(0xffffffffu, l, 16);
      if (gid == 0) {
        const int g = 2 * tig + cc;
        rec[GM * D + g * 2] = (mine && mref[cc] != -INFINITY) ? (mref[cc] - kShift) * kLn2 : -INFINITY;
        rec[GM * D + g * 2 + 1] = l;
      }
    }
    __syncwarp();  // p buffer reads done before the zero terms reuse it
    if (gid < 4) {
      misc[(2 * tig) * 4 + gid] = zacc[0];
      misc[(2 * tig + 1) * 4 + gid] = zacc[1];
    }
    __syncwarp();
    {
      const int ga = 2 * tig, gb = 2 * tig + 1;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float za = misc[ga * 4 + j], zb = misc[gb * 4 + j];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int d0 = 32 * j + 4 * gid + 2 * hh;
          const float s0 = hh ? 1048576.0f : 16777216.0f;
          const float s1 = hh ? 262144.0f : 4194304.0f;
          rec[ga * D + d0] = fmaf(acc[2 * j + hh][0], s0, za);
          rec[ga * D + d0 + 1] = fmaf(acc[2 * j + hh][2], s1, za);
          rec[gb * D + d0] = fmaf(acc[2 * j + hh][1], s0, zb);
          rec[gb * D + d0 + 1] = fmaf(acc[2 * j + hh][3], s1, zb);
        }
      }
    }
    __syncthreads();
    v3_merge<GM, WARPS>(p, reinterpret_cast<const float*>(wreg0), C::WARP_BYTES / 4, c + s);
    if (p.fused) v3_note(p, plan, ntab, s >> 1, arr, narr, last_pair, fsc);
  }
  if (p.fused && narr) v3_flush_arrivals(p, plan, ntab, arr, narr, fsc);
  if (failed && lane == 0) atomicExch(reinterpret_cast<int*>(p.plan + p.n_seg + 2), 1);
}

bool decode_s_eligible(const DecodeParams& p, int key_bits, int value_bits) {
  return (key_bits == 3 || key_bits == 4) && value_bits == 2 && p.D == 128 && p.gs == 32 && p.G <= 8 &&
         p.layout == SMAQ_LAYOUT_DECODE && p.kv_dtype == SMAQ_BF16 && p.page_size % 16 == 0 &&
         (p.q_dtype == SMAQ_BF16 || p.q_dtype == SMAQ_F16) && p.n_seg <= SCfg::MAX_FUSED_SEG && p.E_inv != nullptr;
}

int launch_decode_s(DecodeParams& p, int grid_req, cudaStream_t s, int* grid_out, bool query_only) {
  auto kern = decode_s_kernel;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SCfg::SMEM);
  if (e != cudaSuccess) return cuda_status(e, "decode_s attr");
  const int grid = min(grid_req > 0 ? grid_req : num_sms(), MAX_GRID_FUSED);
  *grid_out = grid;
  if (query_only) return SMAQ_OK;
  if (!p.pdl) {
    kern<<<grid, SCfg::THREADS, SCfg::SMEM, s>>>(p);
    return cuda_status(cudaGetLastError(), "decode_s_kernel");
  }
  // programmatic dependent launch: may start while the previous kernel on `s` finishes
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(SCfg::THREADS);
  cfg.dynamicSmemBytes = SCfg::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, p), "decode_s_kernel (overlapped)");
}

bool decode_v2_eligible(const DecodeParams& p, int key_format, int value_bits, int q_dtype) {
  (void)q_dtype;
  return key_format == SMAQ_KEYS_BVQ && value_bits == 2 && p.D == 128 && p.gs == 32 && p.G <= 8 &&
         p.layout == SMAQ_LAYOUT_DECODE && p.kv_dtype == SMAQ_BF16 && p.page_size % 16 == 0 &&
         (p.q_dtype == SMAQ_BF16 || p.q_dtype == SMAQ_F16) && p.nc <= 256 && p.cent16 != nullptr;
}

template <int GM>
static int launch_v3_t(DecodeParams& p, int grid_req, cudaStream_t s, int* grid_out, bool query_only) {
  auto kern = decode_v3_kernel<GM>;
  const int sm = V3Cfg<GM>::SMEM;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
  if (e != cudaSuccess) return cuda_status(e, "decode_v3 attr");
  const int grid = min(grid_req > 0 ? grid_req : num_sms() * V3Cfg<GM>::CTAS, MAX_GRID_FUSED);
  *grid_out = grid;
  if (query_only) return SMAQ_OK;
  if (!p.pdl) {
    kern<<<grid, V3Cfg<GM>::THREADS, sm, s>>>(p, p.cent16);
    return cuda_status(cudaGetLastError(), "decode_v3_kernel");
  }
  // programmatic dependent launch: may start while the previous kernel on `s` finishes
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(V3Cfg<GM>::THREADS);
  cfg.dynamicSmemBytes = sm;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, p, p.cent16), "decode_v3_kernel (overlapped)");
}

int decode_v2_max_fused_segments(int G) { return G <= 4 ? V3Cfg<4>::MAX_FUSED_SEG : V3Cfg<8>::MAX_FUSED_SEG; }


int launch_decode_v2(DecodeParams& p, int grid_req, cudaStream_t s, int* grid_out, bool query_only) {
  if (p.G <= 4) return launch_v3_t<4>(p, grid_req, s, grid_out, query_only);
  return launch_v3_t<8>(p, grid_req, s, grid_out, query_only);
}

}  // namespace smaq
