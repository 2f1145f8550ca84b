// Shared definitions of the decode kernels (work partition and store addressing).
#pragma once
#include "common.cuh"

namespace smaq {

constexpr int DEC_WARPS = 8;
constexpr int DEC_THREADS = DEC_WARPS * 32;
// Partition weight of one exact-window token in units of one compressed token-head.  The window
// of a pair is latency-bound (its K+V rows are read at full load latency), and the CTA holding it
// is the one that usually arrives last at the pair and runs the pair's final merge, so the weight
// covers the window's time plus most of a merge: at 40 the window CTAs finish their slices early
// and a history CTA merges.  Measured best over 12..64 for the single-launch kernels (long-context
// block-VQ at 1/2/4/8-way head shards, the 32K block-VQ batch and the paged scalar batch).
#ifndef SMAQ_RECENT_COST
#define SMAQ_RECENT_COST 40
#endif
constexpr int RECENT_COST = SMAQ_RECENT_COST;
// Shortest CTA slice (cost units, a multiple of 16).  A slice at least one window token long
// holds the start of every window token range it meets but the last, so every CTA between the
// first and the last CTA of a segment attends at least one of its tokens and writes its slot.
constexpr int64_t MIN_SLICE = (int64_t(RECENT_COST) + 15) & ~int64_t(15);
static_assert(MIN_SLICE >= RECENT_COST && MIN_SLICE >= 16, "slice floor");
constexpr int DEC_MAX_CTAS_PER_SM = 8;  // grid cap when the caller lets the library choose

struct DecodeParams {
  const void* q;
  int q_dtype;
  int64_t q_sb, q_sh;
  int B, Hq, Hkv, G, D;
  float scale;
  const float* E_inv;
  const float* cent;
  int nc;
  const uint8_t* kcodes;
  const void* knorms;
  int kv_dtype;
  const uint8_t* vdata;
  const void* vscales;
  const void* vzeros;
  int gs;
  const int32_t* bt;
  int64_t bt_stride;
  int64_t page_size;
  const int32_t* hist_len;
  const int32_t* hist_total;
  int min_hist;
  const void* rk;
  const void* rv;
  int r_dtype;
  int64_t r_sb, r_st, r_sh;
  const int32_t* recent_len;
  int n_seg;
  int64_t* plan;    // [n_seg + 1] prefix costs, then [per] at index n_seg + 1
  float* slots;     // [(grid + n_seg)][G][D + 2]
  int grid;
  int layout;
  const uint16_t* cent16;  // bvq: fp16 copy of the decoded centroids (exact), or null
  // single-launch mode of the tensor-core kernel: the partition is computed in every CTA and
  // the last CTA to finish a (sequence, kv head) pair merges its slots into the outputs
  int fused;
  int pdl;  // overlapped launch (smaq_decode_args.overlap_prior, single-launch kernels only)
  uint32_t epoch;          // nonzero, different for consecutive calls (tags pair_cnt values)
  uint64_t* pair_cnt;      // [B * Hkv] (epoch << 32 | slots written), reset by the merging CTA
  void* out;
  int64_t o_sb, o_sh;
  float* partial_out;
};

__device__ __forceinline__ int seg_tokens(const DecodeParams& p, int s) {
  const int pair = s >> 1, b = pair / p.Hkv;
  if ((s & 1) == 0) {
    const int tot = p.hist_total ? p.hist_total[b] : p.hist_len[b];
    return tot >= p.min_hist ? p.hist_len[b] : 0;
  }
  return p.recent_len ? p.recent_len[b] : 0;
}
__device__ __forceinline__ int seg_cost(int s) { return (s & 1) ? RECENT_COST : 1; }
// Segment cost padded to a multiple of 16 units so that every CTA slice and every history
// token range starts on a 16-token boundary (16-byte aligned bulk copies of every stream).
__device__ __forceinline__ int64_t seg_span(const DecodeParams& p, int s) {
  return (int64_t(seg_tokens(p, s)) * seg_cost(s) + 15) & ~int64_t(15);
}

__device__ __forceinline__ int64_t hist_row(const DecodeParams& p, int b, int h, int64_t t) {
  const int64_t ps = p.page_size;
  const int64_t pg = t / ps;
  const int64_t page = p.bt ? int64_t(p.bt[b * p.bt_stride + pg]) : int64_t(b);
  return (page * p.Hkv + h) * ps + (t - pg * ps);
}


// Online-softmax state of one warp for G query heads; lane owns dims [4*lane, 4*lane+4).
template <int GM>
struct WarpState {
  float m[GM], l[GM], acc[GM][4];
  __device__ __forceinline__ void init() {
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      m[g] = -INFINITY;
      l[g] = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[g][e] = 0.f;
    }
  }
  // fold one chunk of scores (lane = token, -inf for absent lanes); returns p per head in s
  __device__ __forceinline__ void softmax_chunk(float (&s)[GM], int G) {
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      if (g >= G) break;
      const float cm = warp_max(s[g]);
      const float mn = fmaxf(m[g], cm);
      const float alpha = expf(m[g] - mn);
      const float pv = expf(s[g] - mn);
      l[g] = l[g] * alpha + warp_sum(pv);
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[g][e] *= alpha;
      m[g] = mn;
      s[g] = pv;
    }
  }
};

// Merge per-warp states already written to `red` (warp w at red + w * GM * (D + 2): acc[GM][D],
// then (m, l) pairs) into one partial slot.  Ends with a CTA barrier.
template <int GM>
__device__ void cta_merge_red(const DecodeParams& p, const float* red, int slot) {
  const int G = p.G, D = p.D;
  const int stride = GM * (D + 2);
  float* out = p.slots + int64_t(slot) * G * (D + 2);
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i - g * D;
    float M = -INFINITY;
    for (int w = 0; w < DEC_WARPS; ++w) M = fmaxf(M, red[w * stride + GM * D + g * 2]);
    float a = 0.f, L = 0.f;
    for (int w = 0; w < DEC_WARPS; ++w) {
      const float mw = red[w * stride + GM * D + g * 2];
      const float f = (mw == -INFINITY) ? 0.f : expf(mw - M);
      a += red[w * stride + g * D + d] * f;
      L += red[w * stride + GM * D + g * 2 + 1] * f;
    }
    out[g * D + d] = a;
    if (d == 0) {
      out[G * D + g * 2] = M;
      out[G * D + g * 2 + 1] = L;
    }
  }
  __syncthreads();
}

// Write this warp's state (lane owns dims [4*lane, 4*lane+4)) to `red` and merge the CTA.
template <int GM>
__device__ void cta_flush(const DecodeParams& p, WarpState<GM>& st, float* red, int slot) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int G = p.G, D = p.D;
  float* mine = red + wid * GM * (D + 2);
#pragma unroll
  for (int g = 0; g < GM; ++g) {
    if (g >= G) break;
#pragma unroll
    for (int e = 0; e < 4; ++e) mine[g * D + lane * 4 + e] = st.acc[g][e];
    if (lane == 0) {
      mine[GM * D + g * 2] = st.m[g];
      mine[GM * D + g * 2 + 1] = st.l[g];
    }
  }
  __syncthreads();
  cta_merge_red<GM>(p, red, slot);
}

// Fast path (block-VQ keys, decode layout, 2-bit values, head_dim 128): see decode_v2.cu.
bool decode_v2_eligible(const DecodeParams& p, int key_format, int value_bits, int q_dtype);
int launch_decode_v2(DecodeParams& p, int grid_req, cudaStream_t s, int* grid_out, bool query_only);
int decode_v2_max_fused_segments(int G);
// Scalar 3/4-bit keys, decode layout: tensor-core kernel (decode_v2.cu); always single-launch.
bool decode_s_eligible(const DecodeParams& p, int key_bits, int value_bits);
int launch_decode_s(DecodeParams& p, int grid_req, cudaStream_t s, int* grid_out, bool query_only);

}  // namespace smaq
