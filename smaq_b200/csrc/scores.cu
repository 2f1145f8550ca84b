// Standalone scores against compressed history keys, and weighted sums of compressed history
// values (sm_100a): the two halves of an HF-style cache's attention (SMAQKVCache.attention_scores
// / attend, smaq/kv_cache.py:218-267) when the caller applies its own softmax.
//
// Both are HBM-bound streams over the history rows with a few query rows:
//  * key_scores: one thread per token.  Scalar keys: the CTA first rotates its query rows
//    (qr = q @ E_inv^T, smaq/quantizer.py:176-180) into shared memory; a token's score is then
//    norm * sum_d qr[d] * centroids[code_d], every thread reading the same qr[d] (a broadcast).
//    Block-VQ keys: the CTA builds the table q_block . decoded_centroid[block][c] for every
//    block and code (smaq/block_vq.py:273-297), and a token's score is the sum of its blocks'
//    entries.
//  * attend_values: one warp per token of a CTA's token range, lane l owning dims
//    [D/32 l, D/32 (l+1)), so a warp reads each value row in one coalesced pass; the dequantized
//    value is code * scale + zero in fp32 (two roundings, as smaq/kv_cache.py:94-103 does), the
//    weights are broadcast loads.  Token ranges are split over CTAs; the per-split partial sums go
//    to the workspace and a second kernel adds them in split order.
#include "common.cuh"

namespace smaq {

namespace {

constexpr int SC_THREADS = 256;
constexpr int SC_TOK = 4;  // tokens per thread

template <int BITS>
constexpr int codes_per_byte() { return BITS == 3 ? 2 : 8 / BITS; }

// Query rows q0 .. q0 + QC of group g into shared memory as fp32 (rows past nq are zero).
template <int QC>
__device__ void stage_queries(const smaq_scores_args& a, int64_t g, int q0, int nq, float* qs) {
  const int D = a.head_dim;
  for (int i = threadIdx.x; i < QC * D; i += blockDim.x) {
    const int q = i / D, d = i - q * D;
    qs[i] = q < nq ? load_elem(a.q, a.q_dtype, g * a.q_stride_g + int64_t(q0 + q) * a.q_stride_q + d) : 0.f;
  }
}

template <int BITS, int QC, int D>
__global__ void __launch_bounds__(SC_THREADS) key_scores_scalar_kernel(smaq_scores_args a, int q0, int nq) {
  extern __shared__ float sh[];
  float* qs = sh;                 // [QC][D] query rows
  float* qr = sh + QC * D;        // [QC][D] rotated (when the caller did not rotate)
  float* cent = qr + QC * D;      // [2^BITS]
  const int64_t g = blockIdx.y;
  stage_queries<QC>(a, g, q0, nq, qs);
  if (threadIdx.x < (1 << BITS)) cent[threadIdx.x] = a.centroids[threadIdx.x];
  __syncthreads();
  if (!a.q_rotated) {
    for (int i = threadIdx.x; i < QC * D; i += blockDim.x) {
      const int q = i / D, d = i - q * D;
      const float* e = a.E_inv + int64_t(d) * D;
      float s = 0.f;
      for (int j = 0; j < D; ++j) s = fmaf(qs[q * D + j], __ldg(e + j), s);
      qr[i] = s;
    }
    __syncthreads();
  }
  const float* R = a.q_rotated ? qs : qr;
  constexpr int VPB = codes_per_byte<BITS>();
  constexpr int RB = D / VPB;          // bytes per code row
  constexpr int NW = RB / 16;          // 16-byte words per row
  const int64_t tbase = int64_t(blockIdx.x) * SC_THREADS * SC_TOK;
  // token k + 1's row is requested before token k is scored (double buffer)
  auto load_row = [&](int64_t t, uint4 (&w)[NW], float& nrm) {
    const bool ok = t < a.n_tokens;
    const uint4* row = reinterpret_cast<const uint4*>(a.key_codes + g * a.codes_stride_g + (ok ? t : 0) * RB);
#pragma unroll
    for (int j = 0; j < NW; ++j) w[j] = ok ? __ldg(row + j) : make_uint4(0u, 0u, 0u, 0u);
    nrm = ok ? load_elem(a.key_norms, a.norms_dtype, g * a.norms_stride_g + t) * a.scale : 0.f;
  };
  uint4 cur[NW], nxt[NW];
  float ncur, nnxt;
  load_row(tbase + threadIdx.x, cur, ncur);
#pragma unroll 1
  for (int k = 0; k < SC_TOK; ++k) {
    const int64_t t = tbase + k * SC_THREADS + threadIdx.x;
    if (k + 1 < SC_TOK) load_row(t + SC_THREADS, nxt, nnxt);
    float acc[QC];
#pragma unroll
    for (int q = 0; q < QC; ++q) acc[q] = 0.f;
#pragma unroll
    for (int j = 0; j < NW; ++j) {
      const uint32_t ww[4] = {cur[j].x, cur[j].y, cur[j].z, cur[j].w};
#pragma unroll
      for (int c4 = 0; c4 < 4 * VPB; ++c4) {   // groups of 4 dims of this 16-byte word
        float cv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int code_i = c4 * 4 + e;                 // code index inside the word
          const int by = code_i / VPB, cc = code_i % VPB;
          cv[e] = cent[(ww[by >> 2] >> (8 * (by & 3) + BITS * cc)) & ((1u << BITS) - 1u)];
        }
        const int d = j * 16 * VPB + c4 * 4;
#pragma unroll
        for (int q = 0; q < QC; ++q) {
          const float4 r = *reinterpret_cast<const float4*>(R + q * D + d);
          acc[q] = fmaf(r.x, cv[0], fmaf(r.y, cv[1], fmaf(r.z, cv[2], fmaf(r.w, cv[3], acc[q]))));
        }
      }
    }
    if (t < a.n_tokens) {
#pragma unroll
      for (int q = 0; q < QC; ++q)
        if (q < nq) store_elem(a.out, a.out_dtype, g * a.out_stride_g + int64_t(q0 + q) * a.out_stride_q + t, acc[q] * ncur);
    }
#pragma unroll
    for (int j = 0; j < NW; ++j) cur[j] = nxt[j];
    ncur = nnxt;
  }
}

template <int QC, bool I64>
__global__ void __launch_bounds__(SC_THREADS) key_scores_bvq_kernel(smaq_scores_args a, int q0, int nq) {
  extern __shared__ float sh[];
  const int D = a.head_dim, bd = a.block_dim, nb = D / bd, nc = a.n_centroids;
  float* qs = sh;              // [QC][D]
  float* tab = sh + QC * D;    // [QC][nb][nc]
  const int64_t g = blockIdx.y;
  stage_queries<QC>(a, g, q0, nq, qs);
  __syncthreads();
  for (int i = threadIdx.x; i < QC * nb * nc; i += blockDim.x) {
    const int q = i / (nb * nc), r = i - q * nb * nc, blk = r / nc, c = r - blk * nc;
    const float* dc = a.decoded_centroids + (int64_t(blk) * nc + c) * bd;
    float s = 0.f;
    for (int e = 0; e < bd; ++e) s = fmaf(qs[q * D + blk * bd + e], __ldg(dc + e), s);
    tab[i] = s;
  }
  __syncthreads();
  const int64_t tbase = int64_t(blockIdx.x) * SC_THREADS * SC_TOK;
  for (int k = 0; k < SC_TOK; ++k) {
    const int64_t t = tbase + k * SC_THREADS + threadIdx.x;
    if (t >= a.n_tokens) break;
    float acc[QC];
#pragma unroll
    for (int q = 0; q < QC; ++q) acc[q] = 0.f;
    const int64_t base = g * a.idx_stride_g + t * nb;
    for (int blk = 0; blk < nb; ++blk) {
      const int c = I64 ? int(__ldg(static_cast<const long long*>(a.key_idx) + base + blk))
                        : int(__ldg(static_cast<const uint8_t*>(a.key_idx) + base + blk));
#pragma unroll
      for (int q = 0; q < QC; ++q) acc[q] += tab[(q * nb + blk) * nc + c];
    }
#pragma unroll
    for (int q = 0; q < QC; ++q)
      if (q < nq)
        store_elem(a.out, a.out_dtype, g * a.out_stride_g + int64_t(q0 + q) * a.out_stride_q + t, acc[q] * a.scale);
  }
}

// ------------------------------------------------------------------ attend
constexpr int AT_WARPS = 8;
constexpr int AT_QC = 4;           // query rows per launch
constexpr int AT_TOKENS_PER_WARP = 64;  // per split and warp: enough CTAs to keep loads in flight
constexpr int AT_UNROLL = 4;            // tokens a warp requests before using any

int attend_splits(int64_t n_groups, int n_queries, int64_t n_tokens) {
  const int64_t chunks = n_groups * ((n_queries + AT_QC - 1) / AT_QC);
  int64_t s = (n_tokens + AT_WARPS * AT_TOKENS_PER_WARP - 1) / (AT_WARPS * AT_TOKENS_PER_WARP);
  const int64_t cap = (16 * int64_t(num_sms()) + chunks - 1) / (chunks > 1 ? chunks : 1);  // ~16 CTAs per SM
  if (s > cap) s = cap;
  if (s < 1) s = 1;
  return int(s);
}

template <int DPL>
__host__ __device__ constexpr int attend_red_bytes() { return AT_WARPS * AT_QC * 32 * DPL * 4; }
template <int BITS, int DPL>
__host__ __device__ constexpr int attend_warp_bytes() {
  return (32 * (32 * DPL * BITS / 8 + 4) + 2 * 32 * DPL * 4 + AT_QC * 32 * 4 + 15) / 16 * 16;
}
template <int BITS, int DPL>
__host__ __device__ constexpr int attend_smem_bytes() { return attend_red_bytes<DPL>() + AT_WARPS * attend_warp_bytes<BITS, DPL>(); }

// Per warp: blocks of 32 tokens are staged in shared memory with wide loads (lane = token: its
// code row as 16-byte pieces, its scale / zero, its weights), then lane l accumulates dims
// [DPL l, DPL (l+1)) over the 32 staged tokens.
template <int BITS, int DPL>
__global__ void __launch_bounds__(AT_WARPS * 32) attend_values_kernel(smaq_attend_args a, int q0, int nq, int splits,
                                                                      float* partial) {
  constexpr int D = 32 * DPL;
  constexpr int RB = D * BITS / 8;              // code bytes per token
  constexpr int RBP = RB + 4;                   // padded shared row (words spread over banks)
  extern __shared__ __align__(16) uint8_t at_smem[];
  // [red: AT_WARPS][AT_QC][D] | per warp: codes [32][RBP] | scale, zero [2][32][DPL] | weights [AT_QC][32]
  float (*red)[AT_QC][D] = reinterpret_cast<float (*)[AT_QC][D]>(at_smem);
  uint8_t* wbase = at_smem + attend_red_bytes<DPL>() + (threadIdx.x >> 5) * attend_warp_bytes<BITS, DPL>();
  uint8_t* scode_w = wbase;
  float (*ssz_w)[32][DPL] = reinterpret_cast<float (*)[32][DPL]>(wbase + 32 * RBP);
  float (*sw_w)[32] = reinterpret_cast<float (*)[32]>(wbase + 32 * RBP + 2 * 32 * DPL * 4);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int64_t g = blockIdx.y;
  const int split = blockIdx.x;
  const int64_t per = (a.n_tokens + splits - 1) / splits;
  const int64_t t0 = split * per, t1 = min(a.n_tokens, t0 + per);
  const int ng = D / a.group_size;
  const int d0 = lane * DPL, grp = d0 / a.group_size;
  const int bit0 = d0 * BITS;
  float acc[AT_QC][DPL];
#pragma unroll
  for (int q = 0; q < AT_QC; ++q)
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[q][i] = 0.f;
  for (int64_t tb = t0 + int64_t(wid) * 32; tb < t1; tb += int64_t(AT_WARPS) * 32) {
    const int64_t t = tb + lane;
    const bool ok = t < t1;
    const int64_t tt = ok ? t : tb;
    // ---- stage (lane = token)
    {
      const uint8_t* row = a.v_data + g * a.data_stride_g + tt * RB;
      uint8_t* dst = scode_w + lane * RBP;
      if constexpr (RB % 4 == 0) {
        if ((reinterpret_cast<uintptr_t>(row) & 3) == 0) {
#pragma unroll
          for (int j = 0; j < RB / 4; ++j)
            reinterpret_cast<uint32_t*>(dst)[j] = ok ? __ldg(reinterpret_cast<const uint32_t*>(row) + j) : 0u;
        } else {
          for (int j = 0; j < RB; ++j) dst[j] = ok ? __ldg(row + j) : 0;
        }
      } else {
        for (int j = 0; j < RB; ++j) dst[j] = ok ? __ldg(row + j) : 0;
      }
      const int64_t sz = g * a.sz_stride_g + tt * ng;
      for (int k = 0; k < ng; ++k) {
        ssz_w[0][lane][k] = ok ? load_elem(a.v_scales, a.sz_dtype, sz + k) : 0.f;
        ssz_w[1][lane][k] = ok ? load_elem(a.v_zeros, a.sz_dtype, sz + k) : 0.f;
      }
#pragma unroll
      for (int q = 0; q < AT_QC; ++q)
        sw_w[q][lane] = (ok && q < nq) ? load_elem(a.w, a.w_dtype, g * a.w_stride_g + int64_t(q0 + q) * a.w_stride_q + t) : 0.f;
    }
    __syncwarp();
    // ---- accumulate (lane = dims)
    const int nt = t1 - tb < 32 ? int(t1 - tb) : 32;
    for (int u = 0; u < nt; ++u) {
      const uint8_t* row = scode_w + u * RBP + (bit0 >> 3);
      uint32_t bits = row[0];
      if ((bit0 & 7) + DPL * BITS > 8) bits |= uint32_t(row[1]) << 8;
      if ((bit0 & 7) + DPL * BITS > 16) bits |= uint32_t(row[2]) << 16 | uint32_t(row[3]) << 24;
      bits >>= (bit0 & 7);
      const float s = ssz_w[0][u][grp], z = ssz_w[1][u][grp];
#pragma unroll
      for (int i = 0; i < DPL; ++i) {
        const float v = __fadd_rn(__fmul_rn(float((bits >> (BITS * i)) & ((1u << BITS) - 1u)), s), z);
#pragma unroll
        for (int q = 0; q < AT_QC; ++q) acc[q][i] = fmaf(sw_w[q][u], v, acc[q][i]);
      }
    }
    __syncwarp();
  }
#pragma unroll
  for (int q = 0; q < AT_QC; ++q)
#pragma unroll
    for (int i = 0; i < DPL; ++i) red[wid][q][d0 + i] = acc[q][i];
  __syncthreads();
  for (int k = threadIdx.x; k < AT_QC * D; k += blockDim.x) {
    const int q = k / D, d = k - q * D;
    if (q >= nq) continue;
    float sum = 0.f;
    for (int w = 0; w < AT_WARPS; ++w) sum += red[w][q][d];
    if (splits == 1)
      store_elem(a.out, a.out_dtype, g * a.out_stride_g + int64_t(q0 + q) * a.out_stride_q + d, sum);
    else
      partial[((int64_t(split) * a.n_groups + g) * AT_QC + q) * D + d] = sum;
  }
}

__global__ void attend_reduce_kernel(smaq_attend_args a, int q0, int nq, int splits, const float* partial) {
  const int D = a.head_dim;
  const int64_t n = a.n_groups * AT_QC * D;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t g = i / (AT_QC * D);
    const int r = int(i - g * AT_QC * D), q = r / D, d = r - q * D;
    if (q >= nq) continue;
    float sum = 0.f;
    for (int s = 0; s < splits; ++s) sum += partial[int64_t(s) * n + i];
    store_elem(a.out, a.out_dtype, g * a.out_stride_g + int64_t(q0 + q) * a.out_stride_q + d, sum);
  }
}

bool dtype_ok(int dt) { return dt == SMAQ_F32 || dt == SMAQ_BF16 || dt == SMAQ_F16; }

}  // namespace

// ------------------------------------------------------------------ host entry points
template <int QC, typename K>
static int launch_scores_chunks(const smaq_scores_args& a, K kern, size_t smem, cudaStream_t s, const char* name) {
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return cuda_status(e, name);
  }
  const dim3 grid(unsigned((a.n_tokens + SC_THREADS * SC_TOK - 1) / (SC_THREADS * SC_TOK)), unsigned(a.n_groups));
  for (int q0 = 0; q0 < a.n_queries; q0 += QC) {
    kern<<<grid, SC_THREADS, smem, s>>>(a, q0, min(QC, a.n_queries - q0));
    const int st = cuda_status(cudaGetLastError(), name);
    if (st) return st;
  }
  return SMAQ_OK;
}

}  // namespace smaq

using namespace smaq;

extern "C" int smaq_key_scores(const smaq_scores_args* args, void* stream) {
  if (!args) return fail(SMAQ_ERR_INVALID, "key_scores: null args");
  const smaq_scores_args& a = *args;
  const int D = a.head_dim;
  if (D <= 0 || D % 32 || D > 256 || a.n_groups <= 0 || a.n_queries <= 0 || a.n_tokens < 0 || a.n_groups > 65535)
    return fail(SMAQ_ERR_INVALID, "key_scores: bad shape (D %d, groups %lld, queries %d, tokens %lld)", D,
                (long long)a.n_groups, a.n_queries, (long long)a.n_tokens);
  if (!a.q || !a.out || !dtype_ok(a.q_dtype) || !dtype_ok(a.out_dtype))
    return fail(SMAQ_ERR_INVALID, "key_scores: null query/output or bad dtype");
  if (a.n_tokens == 0) return SMAQ_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a.key_format == SMAQ_KEYS_SCALAR) {
    if (!a.key_codes || !a.key_norms || !a.E_inv || !a.centroids || !dtype_ok(a.norms_dtype))
      return fail(SMAQ_ERR_INVALID, "key_scores: scalar keys need codes, norms, E_inv and centroids");
    if (a.key_bits < 2 || a.key_bits > 4)
      return fail(SMAQ_ERR_UNSUPPORTED, "key_scores: key_bits %d (2, 3 or 4)", a.key_bits);
    if (D != 64 && D != 128 && D != 256) return fail(SMAQ_ERR_UNSUPPORTED, "key_scores: scalar keys, head_dim %d", D);
    if ((reinterpret_cast<uintptr_t>(a.key_codes) | uintptr_t(a.codes_stride_g)) & 15)
      return fail(SMAQ_ERR_INVALID, "key_scores: code rows must be 16-byte aligned");
    // one query row per launch when there is one (the HF decode case), else chunks of 8
#define SMAQ_SC(B, Q, DD) \
  launch_scores_chunks<Q>(a, key_scores_scalar_kernel<B, Q, DD>, sizeof(float) * (2 * Q * DD + 16), s, "key_scores_scalar")
#define SMAQ_SC_D(B, Q) (D == 64 ? SMAQ_SC(B, Q, 64) : D == 128 ? SMAQ_SC(B, Q, 128) : SMAQ_SC(B, Q, 256))
#define SMAQ_SC_Q(B) (a.n_queries == 1 ? SMAQ_SC_D(B, 1) : SMAQ_SC_D(B, 8))
    const int r = a.key_bits == 2 ? SMAQ_SC_Q(2) : a.key_bits == 3 ? SMAQ_SC_Q(3) : SMAQ_SC_Q(4);
#undef SMAQ_SC_Q
#undef SMAQ_SC_D
#undef SMAQ_SC
    return r;
  }
  if (a.key_format == SMAQ_KEYS_BVQ) {
    if (!a.key_idx || !a.decoded_centroids || a.block_dim <= 0 || D % a.block_dim || a.n_centroids <= 0 ||
        a.n_centroids > 256)
      return fail(SMAQ_ERR_INVALID, "key_scores: bvq keys need indices, decoded centroids, block_dim | D, nc <= 256");
    constexpr int QC = 4;
    const size_t smem = sizeof(float) * (QC * D + size_t(QC) * (D / a.block_dim) * a.n_centroids);
    if (smem > 227 * 1024) return fail(SMAQ_ERR_UNSUPPORTED, "key_scores: bvq table of %zu bytes", smem);
    return a.idx_is_int64 ? launch_scores_chunks<QC>(a, key_scores_bvq_kernel<QC, true>, smem, s, "key_scores_bvq")
                          : launch_scores_chunks<QC>(a, key_scores_bvq_kernel<QC, false>, smem, s, "key_scores_bvq");
  }
  return fail(SMAQ_ERR_INVALID, "key_scores: key_format %d", a.key_format);
}

extern "C" size_t smaq_attend_workspace_size(int64_t n_groups, int n_queries, int64_t n_tokens, int head_dim) {
  const int sp = attend_splits(n_groups, n_queries, n_tokens);
  return sp > 1 ? sizeof(float) * size_t(sp) * size_t(n_groups) * AT_QC * size_t(head_dim) : 0;
}

extern "C" int smaq_attend_values(const smaq_attend_args* args, void* stream) {
  if (!args) return fail(SMAQ_ERR_INVALID, "attend_values: null args");
  const smaq_attend_args& a = *args;
  const int D = a.head_dim;
  if (D <= 0 || D % 32 || D > 256 || a.n_groups <= 0 || a.n_groups > 65535 || a.n_queries <= 0 || a.n_tokens < 0)
    return fail(SMAQ_ERR_INVALID, "attend_values: bad shape");
  if (!a.w || !a.out || !a.v_data || !a.v_scales || !a.v_zeros || !dtype_ok(a.w_dtype) || !dtype_ok(a.out_dtype) ||
      !dtype_ok(a.sz_dtype))
    return fail(SMAQ_ERR_INVALID, "attend_values: null pointer or bad dtype");
  if ((a.value_bits != 2 && a.value_bits != 4) || a.group_size <= 0 || a.group_size % (D / 32) ||
      D % a.group_size)
    return fail(SMAQ_ERR_UNSUPPORTED, "attend_values: bits %d, group %d", a.value_bits, a.group_size);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int dpl = D / 32;
  int splits = a.n_tokens ? attend_splits(a.n_groups, a.n_queries, a.n_tokens) : 1;
  float* partial = nullptr;
  if (splits > 1) {
    const size_t need = smaq_attend_workspace_size(a.n_groups, a.n_queries, a.n_tokens, D);
    if (!a.workspace || a.workspace_bytes < need)
      return fail(SMAQ_ERR_WORKSPACE, "attend_values: workspace %zu bytes < %zu needed", a.workspace_bytes, need);
    partial = static_cast<float*>(a.workspace);
  }
  for (int q0 = 0; q0 < a.n_queries; q0 += AT_QC) {
    const int nq = min(AT_QC, a.n_queries - q0);
    const dim3 grid(unsigned(splits), unsigned(a.n_groups));
    const int t = AT_WARPS * 32;
#define SMAQ_ATTEND(B, P)                                                                                \
  do {                                                                                                    \
    constexpr int sm_ = attend_smem_bytes<B, P>();                                                       \
    if (sm_ > 48 * 1024)                                                                                   \
      cudaFuncSetAttribute(attend_values_kernel<B, P>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm_); \
    attend_values_kernel<B, P><<<grid, t, sm_, s>>>(a, q0, nq, splits, partial);                          \
  } while (0)
    if (a.value_bits == 2) {
      if (dpl == 1) SMAQ_ATTEND(2, 1); else if (dpl == 2) SMAQ_ATTEND(2, 2);
      else if (dpl == 4) SMAQ_ATTEND(2, 4); else if (dpl == 8) SMAQ_ATTEND(2, 8);
      else return fail(SMAQ_ERR_UNSUPPORTED, "attend_values: head_dim %d", D);
    } else {
      if (dpl == 1) SMAQ_ATTEND(4, 1); else if (dpl == 2) SMAQ_ATTEND(4, 2);
      else if (dpl == 4) SMAQ_ATTEND(4, 4); else if (dpl == 8) SMAQ_ATTEND(4, 8);
      else return fail(SMAQ_ERR_UNSUPPORTED, "attend_values: head_dim %d", D);
    }
#undef SMAQ_ATTEND
    int st = cuda_status(cudaGetLastError(), "attend_values_kernel");
    if (st) return st;
    if (splits > 1) {
      const int64_t n = a.n_groups * AT_QC * D;
      const int64_t nblk = (n + 255) / 256;
      const int blocks = int(nblk < 4 * num_sms() ? nblk : 4 * num_sms());
      attend_reduce_kernel<<<blocks, 256, 0, s>>>(a, q0, nq, splits, partial);
      st = cuda_status(cudaGetLastError(), "attend_reduce_kernel");
      if (st) return st;
    }
  }
  return SMAQ_OK;
}
