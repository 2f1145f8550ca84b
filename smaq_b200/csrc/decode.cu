// Hybrid decode attention over compressed history + exact recent window (SIMT path).
//
// Reference: compute_hybrid_attention, smaq/score.py:23-72.
//   logits = [q.k_hat * scale  (history, fp32) || q.k * scale (recent, fp32)]   score.py:61-64
//   w      = softmax(logits)                                                   score.py:64
//   out    = (w_hist @ V_hat).to(qdtype) + (w_recent @ V_recent).to(qdtype)     score.py:70-72
// History shorter than min_history (16) is ignored (score.py:37).  Scalar history scores are
// (q @ E_inv^T) . centroids[codes] * norm * scale (quantizer.py:131-136, :176-183); block-VQ
// history scores are q . decoded_centroids[idx] * scale (block_vq.py:246-297).
//
// Work partition ("stream-K" over tokens): the (batch, kv-head, {history, recent}) segments are
// laid end to end in cost units (one unit per history token, RECENT_COST per exact token) and
// every CTA takes an equal slice.  A CTA therefore builds the per-query score tables of at most
// a few segments, all SMs stay busy regardless of batch size or length skew, and each
// (CTA, segment) intersection writes one fp32 partial (running max, sum, accumulator) into slot
// cta + segment -- unique because the intersections form a monotone staircase.  A merge kernel
// then combines the partials of each (batch, kv-head) with a log-sum-exp rescale.
#include <math.h>

#include <atomic>

#include "common.cuh"
#include "decode_common.cuh"
#include "ptx.cuh"

namespace smaq {

// One CTA: prefix sums of segment costs and the per-CTA slice length.
__global__ void decode_plan_kernel(DecodeParams p) {
  __shared__ int64_t carry;
  __shared__ int64_t wsum[32];
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int base = 0; base < p.n_seg; base += blockDim.x) {
    const int s = base + threadIdx.x;
    int64_t c = (s < p.n_seg) ? seg_span(p, s) : 0;
    int64_t x = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) wsum[wid] = x;
    __syncthreads();
    if (wid == 0) {
      int64_t w = lane < nw ? wsum[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int64_t y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      if (lane < nw) wsum[lane] = w;
    }
    __syncthreads();
    const int64_t excl = carry + x - c + (wid ? wsum[wid - 1] : 0);
    if (s < p.n_seg) p.plan[s] = excl;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = excl + c;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const int64_t total = carry;
    p.plan[p.n_seg] = total;
    int64_t per = (total + p.grid - 1) / p.grid;
    per = (per + 15) & ~int64_t(15);
    if (per < MIN_SLICE) per = MIN_SLICE;
    p.plan[p.n_seg + 1] = per;
    p.plan[p.n_seg + 2] = 0;  // error word (set by a kernel whose bounded wait ran out)
  }
}

template <int GM, int KB, int VB>
__global__ void __launch_bounds__(DEC_THREADS) decode_kernel(DecodeParams p) {
  constexpr int D = 128;
  constexpr int NBLK = D / 8;
  extern __shared__ float smem[];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int G = p.G;
  // shared layout: qs [GM][D] | table | warp-merge buffer
  float* qs = smem;
  float* tab = qs + GM * D;
  const int tab_floats = (KB == 0) ? GM * NBLK * p.nc : GM * D + 16;
  float* red = tab + tab_floats;

  const int64_t total = p.plan[p.n_seg];
  const int64_t per = p.plan[p.n_seg + 1];
  const int c = blockIdx.x;
  const int64_t lo = int64_t(c) * per, hi = min(lo + per, total);
  if (lo >= hi) return;
  // first segment whose cost range ends after lo
  int sa = 0, sb = p.n_seg - 1;
  while (sa < sb) {
    const int mid = (sa + sb) >> 1;
    if (p.plan[mid + 1] > lo) sb = mid; else sa = mid + 1;
  }
  for (int s = sa; s < p.n_seg; ++s) {
    const int64_t S = p.plan[s];
    if (S >= hi) break;
    const int n = seg_tokens(p, s);
    if (n == 0) continue;
    const int cs = seg_cost(s);
    int64_t t0 = (lo - S + cs - 1) / cs;
    if (lo <= S) t0 = 0;
    int64_t t1 = (hi - S + cs - 1) / cs;
    if (t1 > n) t1 = n;
    if (t0 >= t1) continue;
    const int pair = s >> 1, b = pair / p.Hkv, h = pair - b * p.Hkv;
    const bool recent = (s & 1);
    // ---- per-segment setup: the G query rows of this kv head
    for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
      const int g = i / D, d = i - g * D;
      qs[i] = load_elem(p.q, p.q_dtype, b * p.q_sb + int64_t(h * G + g) * p.q_sh + d);
    }
    __syncthreads();
    if (!recent) {
      if constexpr (KB == 0) {
        // LUT[g][blk][c] = q_g[blk] . decoded_centroid[blk][c]
        for (int i = threadIdx.x; i < NBLK * p.nc; i += blockDim.x) {
          const int blk = i / p.nc;
          const float4 c0 = __ldg(reinterpret_cast<const float4*>(p.cent + int64_t(i) * 8));
          const float4 c1 = __ldg(reinterpret_cast<const float4*>(p.cent + int64_t(i) * 8 + 4));
#pragma unroll
          for (int g = 0; g < GM; ++g) {
            if (g >= G) break;
            const float* qg = qs + g * D + blk * 8;
            float a = qg[0] * c0.x;
            a = fmaf(qg[1], c0.y, a);
            a = fmaf(qg[2], c0.z, a);
            a = fmaf(qg[3], c0.w, a);
            a = fmaf(qg[4], c1.x, a);
            a = fmaf(qg[5], c1.y, a);
            a = fmaf(qg[6], c1.z, a);
            a = fmaf(qg[7], c1.w, a);
            tab[g * NBLK * p.nc + i] = a;
          }
        }
      } else {
        // q_rot = q @ E_inv^T (quantizer.py:136) and the centroid table
        for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
          const int g = i / D, j = i - g * D;
          const float* er = p.E_inv + j * D;
          float a = 0.f;
          for (int k = 0; k < D; ++k) a = fmaf(qs[g * D + k], __ldg(er + k), a);
          tab[g * D + j] = a;
        }
        if (threadIdx.x < (1 << KB)) tab[GM * D + threadIdx.x] = p.cent[threadIdx.x];
      }
      __syncthreads();
    }
    WarpState<GM> st;
    st.init();
    const int64_t nchunks = (t1 - t0 + 31) / 32;
    for (int64_t ch = wid; ch < nchunks; ch += DEC_WARPS) {
      const int64_t tb = t0 + ch * 32;
      const int64_t t = tb + lane;
      const bool valid = t < t1;
      const int nvalid = int((t1 - tb) < 32 ? (t1 - tb) : 32);
      float sc[GM];
#pragma unroll
      for (int g = 0; g < GM; ++g) sc[g] = -INFINITY;
      if (!recent) {
        if (valid) {
          const int64_t row = hist_row(p, b, h, t);
          if constexpr (KB == 0) {
            uint4 iv;
            uint8_t* ibw = reinterpret_cast<uint8_t*>(&iv);
            if (p.layout == SMAQ_LAYOUT_DECODE) {
              const uint8_t* rb = p.kcodes + row * NBLK;
#pragma unroll
              for (int blk = 0; blk < NBLK; ++blk) ibw[blk] = rb[2 * (4 * (blk >> 3) + (blk & 3)) + ((blk >> 2) & 1)];
            } else {
              iv = __ldg(reinterpret_cast<const uint4*>(p.kcodes + row * NBLK));
            }
            const uint8_t* ib = ibw;
#pragma unroll
            for (int g = 0; g < GM; ++g) {
              if (g >= G) break;
              const float* lt = tab + g * NBLK * p.nc;
              float a = 0.f;
#pragma unroll
              for (int blk = 0; blk < NBLK; ++blk) a += lt[blk * p.nc + ib[blk]];
              sc[g] = a * p.scale;
            }
          } else {
            constexpr int VPB = (8 / KB) > 0 ? 8 / KB : 1;
            constexpr int PD = (D + VPB - 1) / VPB;
            constexpr int MASK = (1 << KB) - 1;
            const float* cent = tab + GM * D;
            float a[GM];
#pragma unroll
            for (int g = 0; g < GM; ++g) a[g] = 0.f;
            const uint8_t* crow = p.kcodes + row * PD;
            uint4 wrow[PD / 16];
#pragma unroll
            for (int q4 = 0; q4 < PD / 16; ++q4) wrow[q4] = __ldg(reinterpret_cast<const uint4*>(crow + q4 * 16));
            const uint8_t* rowb = reinterpret_cast<const uint8_t*>(wrow);
            // SMAQ_LAYOUT_DECODE (3/4-bit, 64-byte rows): reference byte pb sits at 16 (pb % 4) + pb / 4
            const bool perm = PD == 64 && p.layout == SMAQ_LAYOUT_DECODE;
#pragma unroll
            for (int q4 = 0; q4 < PD / 16; ++q4) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int pb = q4 * 16 + j;
                const uint32_t byv = perm ? rowb[(16 * (pb & 3) + (pb >> 2)) & (PD - 1)] : rowb[pb];
#pragma unroll
                for (int v = 0; v < VPB; ++v) {
                  const int d = (q4 * 16 + j) * VPB + v;
                  const float cv = cent[(byv >> (v * KB)) & MASK];
#pragma unroll
                  for (int g = 0; g < GM; ++g) {
                    if (g >= G) break;
                    a[g] = fmaf(tab[g * D + d], cv, a[g]);
                  }
                }
              }
            }
            const float nrm = load_elem(p.knorms, p.kv_dtype, row);
#pragma unroll
            for (int g = 0; g < GM; ++g) sc[g] = (a[g] * nrm) * p.scale;
          }
        }
      } else if (valid) {
        const int64_t rb = b * p.r_sb + t * p.r_st + h * p.r_sh;
        float a[GM];
#pragma unroll
        for (int g = 0; g < GM; ++g) a[g] = 0.f;
        for (int d = 0; d < D; ++d) {
          const float kv = load_elem(p.rk, p.r_dtype, rb + d);
#pragma unroll
          for (int g = 0; g < GM; ++g) {
            if (g >= G) break;
            a[g] = fmaf(qs[g * D + d], kv, a[g]);
          }
        }
#pragma unroll
        for (int g = 0; g < GM; ++g) sc[g] = a[g] * p.scale;
      }
      st.softmax_chunk(sc, G);
      // P @ V : lane owns dims [4*lane, 4*lane + 4)
      for (int j = 0; j < nvalid; ++j) {
        const int64_t tj = tb + j;
        float v[4];
        if (!recent) {
          const int64_t row = hist_row(p, b, h, tj);
          const int ng = D / p.gs;
          const int grp = (lane * 4) / p.gs;
          const float sc_ = load_elem(p.vscales, p.kv_dtype, row * ng + grp);
          const float zr = load_elem(p.vzeros, p.kv_dtype, row * ng + grp);
          if constexpr (VB == 2) {
            const int pos = p.layout == SMAQ_LAYOUT_DECODE ? 4 * (lane & 7) + (lane >> 3) : lane;
            const uint32_t by = p.vdata[row * (D / 4) + pos];
#pragma unroll
            for (int e = 0; e < 4; ++e) v[e] = fmaf(float((by >> (2 * e)) & 3u), sc_, zr);
          } else {
            const uint32_t by = *reinterpret_cast<const uint16_t*>(p.vdata + row * (D / 2) + lane * 2);
#pragma unroll
            for (int e = 0; e < 4; ++e) v[e] = fmaf(float((by >> (4 * e)) & 15u), sc_, zr);
          }
        } else {
          const int64_t rb = b * p.r_sb + tj * p.r_st + h * p.r_sh + lane * 4;
#pragma unroll
          for (int e = 0; e < 4; ++e) v[e] = load_elem(p.rv, p.r_dtype, rb + e);
        }
#pragma unroll
        for (int g = 0; g < GM; ++g) {
          if (g >= G) break;
          const float pj = __shfl_sync(0xffffffffu, sc[g], j);
#pragma unroll
          for (int e = 0; e < 4; ++e) st.acc[g][e] = fmaf(pj, v[e], st.acc[g][e]);
        }
      }
    }
    cta_flush<GM>(p, st, red, c + s);
  }
}

// Merge the partial slots of every (b, kv-head) into the output and/or the fp32 partials.
__global__ void decode_merge_kernel(DecodeParams p, void* out, int64_t o_sb, int64_t o_sh,
                                    float* partial_out) {
  const int pair = blockIdx.x;
  const int b = pair / p.Hkv, h = pair - b * p.Hkv;
  const int G = p.G, D = p.D;
  const int64_t per = p.plan[p.n_seg + 1];
  const int slot_f = G * (D + 2);
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i - g * D;
    float M = -INFINITY;
    int c0[2], c1[2], nn[2];
    for (int k = 0; k < 2; ++k) {
      const int s = pair * 2 + k;
      nn[k] = seg_tokens(p, s);
      const int64_t S = p.plan[s];
      c0[k] = int(S / per);
      c1[k] = nn[k] ? int((S + int64_t(nn[k] - 1) * seg_cost(s)) / per) : c0[k] - 1;
      for (int c = c0[k]; c <= c1[k]; ++c)
        M = fmaxf(M, p.slots[int64_t(c + s) * slot_f + G * D + g * 2]);
    }
    float L = 0.f, acc[2] = {0.f, 0.f};
    for (int k = 0; k < 2; ++k) {
      const int s = pair * 2 + k;
      for (int c = c0[k]; c <= c1[k]; ++c) {
        const float* sl = p.slots + int64_t(c + s) * slot_f;
        const float f = expf(sl[G * D + g * 2] - M);
        acc[k] += sl[g * D + d] * f;
        L += sl[G * D + g * 2 + 1] * f;
      }
    }
    const int hq = h * G + g;
    if (partial_out) {
      float* po = partial_out + (int64_t(b) * p.Hq + hq) * (2 * D + 2);
      po[d] = acc[0];
      po[D + d] = acc[1];
      if (d == 0) {
        po[2 * D] = M;
        po[2 * D + 1] = L;
      }
    }
    if (out) {
      float oh = 0.f, orr = 0.f;
      if (L > 0.f) {
        oh = acc[0] / L;
        orr = acc[1] / L;
      }
      // each part is cast to the query dtype, then the parts are summed in it (score.py:70-72)
      const float o = round_dtype(round_dtype(oh, p.q_dtype) + round_dtype(orr, p.q_dtype), p.q_dtype);
      store_elem(out, p.q_dtype, b * o_sb + hq * o_sh + d, o);
    }
  }
}

__global__ void merge_partials_kernel(const float* __restrict__ parts, int R, int B, int Hq, int D,
                                      void* out, int out_dtype, int64_t o_sb, int64_t o_sh) {
  const int bh = blockIdx.x;
  const int b = bh / Hq, hq = bh - b * Hq;
  const int64_t stride = int64_t(B) * Hq * (2 * D + 2);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float M = -INFINITY;
    for (int r = 0; r < R; ++r) M = fmaxf(M, parts[r * stride + int64_t(bh) * (2 * D + 2) + 2 * D]);
    float L = 0.f, a0 = 0.f, a1 = 0.f;
    for (int r = 0; r < R; ++r) {
      const float* po = parts + r * stride + int64_t(bh) * (2 * D + 2);
      const float mr = po[2 * D];
      const float f = (mr == -INFINITY) ? 0.f : expf(mr - M);
      a0 += po[d] * f;
      a1 += po[D + d] * f;
      L += po[2 * D + 1] * f;
    }
    float oh = 0.f, orr = 0.f;
    if (L > 0.f) {
      oh = a0 / L;
      orr = a1 / L;
    }
    const float o = round_dtype(round_dtype(oh, out_dtype) + round_dtype(orr, out_dtype), out_dtype);
    store_elem(out, out_dtype, b * o_sb + hq * o_sh + d, o);
  }
}

// ---------------------------------------------------------------- host
static size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// [n_seg] prefix costs, total, per-CTA slice, device error word | per-pair arrival counters
static size_t plan_table_bytes(int n_seg) { return align_up(sizeof(int64_t) * (n_seg + 4), 256); }
static size_t plan_bytes(int n_seg) { return plan_table_bytes(n_seg) + align_up(sizeof(uint64_t) * (n_seg / 2), 256); }

static size_t dec_smem(int GM, int KB, int nc) {
  const int D = 128;
  const int tab = (KB == 0) ? GM * (D / 8) * nc : GM * D + 16;
  return sizeof(float) * (GM * D + tab + DEC_WARPS * GM * (D + 2));
}

template <int GM, int KB, int VB>
static int launch_decode_t(DecodeParams& p, int grid_req, cudaStream_t s, int* grid_out, bool query_only) {
  auto kern = decode_kernel<GM, KB, VB>;
  const size_t sm = dec_smem(GM, KB, p.nc);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm));
  if (e != cudaSuccess) return cuda_status(e, "decode_kernel attr");
  int grid = grid_req;
  if (grid <= 0) {
    int occ = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, DEC_THREADS, sm);
    if (e != cudaSuccess) return cuda_status(e, "decode occupancy");
    if (occ < 1) occ = 1;
    if (occ > DEC_MAX_CTAS_PER_SM) occ = DEC_MAX_CTAS_PER_SM;
    grid = num_sms() * occ;
  }
  *grid_out = grid;
  if (query_only) return SMAQ_OK;
  kern<<<grid, DEC_THREADS, sm, s>>>(p);
  return cuda_status(cudaGetLastError(), "decode_kernel");
}

template <int GM>
static int launch_decode_g(DecodeParams& p, int kb, int vb, int grid_req, cudaStream_t s, int* grid_out,
                           bool query_only) {
  if (vb == 2) {
    switch (kb) {
      case 0: return launch_decode_t<GM, 0, 2>(p, grid_req, s, grid_out, query_only);
      case 2: return launch_decode_t<GM, 2, 2>(p, grid_req, s, grid_out, query_only);
      case 3: return launch_decode_t<GM, 3, 2>(p, grid_req, s, grid_out, query_only);
      case 4: return launch_decode_t<GM, 4, 2>(p, grid_req, s, grid_out, query_only);
    }
  } else {
    switch (kb) {
      case 0: return launch_decode_t<GM, 0, 4>(p, grid_req, s, grid_out, query_only);
      case 2: return launch_decode_t<GM, 2, 4>(p, grid_req, s, grid_out, query_only);
      case 3: return launch_decode_t<GM, 3, 4>(p, grid_req, s, grid_out, query_only);
      case 4: return launch_decode_t<GM, 4, 4>(p, grid_req, s, grid_out, query_only);
    }
  }
  return fail(SMAQ_ERR_UNSUPPORTED, "decode: key bits %d / value bits %d", kb, vb);
}

static int dispatch_decode(DecodeParams& p, int kb, int vb, int grid_req, cudaStream_t s, int* grid_out,
                           bool query_only) {
  if (kb != 0 && decode_s_eligible(p, kb, vb)) return launch_decode_s(p, grid_req, s, grid_out, query_only);
  if (kb == 0 && decode_v2_eligible(p, SMAQ_KEYS_BVQ, vb, p.q_dtype))
    return launch_decode_v2(p, grid_req, s, grid_out, query_only);
  if (p.G <= 1) return launch_decode_g<1>(p, kb, vb, grid_req, s, grid_out, query_only);
  if (p.G <= 2) return launch_decode_g<2>(p, kb, vb, grid_req, s, grid_out, query_only);
  if (p.G <= 4) return launch_decode_g<4>(p, kb, vb, grid_req, s, grid_out, query_only);
  if (p.G <= 8) return launch_decode_g<8>(p, kb, vb, grid_req, s, grid_out, query_only);
  return fail(SMAQ_ERR_UNSUPPORTED, "decode: %d query heads per kv head (max 8)", p.G);
}

}  // namespace smaq

using namespace smaq;

extern "C" size_t smaq_decode_workspace_size(int batch, int n_q_heads, int n_kv_heads, int head_dim,
                                             int num_ctas) {
  if (batch <= 0 || n_kv_heads <= 0 || n_q_heads % n_kv_heads) return 0;
  const int n_seg = 2 * batch * n_kv_heads;
  const int G = n_q_heads / n_kv_heads;
  const int grid = num_ctas > 0 ? num_ctas : num_sms() * DEC_MAX_CTAS_PER_SM;
  return plan_bytes(n_seg) + sizeof(float) * size_t(grid + n_seg) * G * (head_dim + 2);
}

namespace smaq {
// Validate the arguments and fill the kernel parameters (no CUDA call).
static int decode_params(const smaq_decode_args* args, DecodeParams& p, int& kb) {
  if (!args) return fail(SMAQ_ERR_INVALID, "decode: null args");
  const smaq_decode_args& a = *args;
  if (a.batch <= 0 || a.n_q_heads <= 0 || a.n_kv_heads <= 0 || a.n_q_heads % a.n_kv_heads)
    return fail(SMAQ_ERR_INVALID, "decode: bad head counts B=%d Hq=%d Hkv=%d", a.batch, a.n_q_heads,
                a.n_kv_heads);
  if (a.head_dim != 128) return fail(SMAQ_ERR_UNSUPPORTED, "decode: head_dim %d (only 128)", a.head_dim);
  if (!a.out && !a.partial_out) return fail(SMAQ_ERR_INVALID, "decode: no output");
  if (!a.q || !a.hist_len) return fail(SMAQ_ERR_INVALID, "decode: null query or hist_len");
  if (a.page_size <= 0) return fail(SMAQ_ERR_INVALID, "decode: page_size must be > 0");
  kb = 0;
  if (a.key_format == SMAQ_KEYS_SCALAR) {
    if (a.key_bits < 2 || a.key_bits > 4) return fail(SMAQ_ERR_UNSUPPORTED, "decode: key bits %d", a.key_bits);
    if (!a.E_inv || !a.centroids || !a.key_codes || !a.key_norms)
      return fail(SMAQ_ERR_INVALID, "decode: scalar key tables missing");
    kb = a.key_bits;
  } else if (a.key_format == SMAQ_KEYS_BVQ) {
    if (a.block_dim != 8 || a.n_centroids < 1 || a.n_centroids > 256)
      return fail(SMAQ_ERR_UNSUPPORTED, "decode: bvq block_dim %d n_centroids %d", a.block_dim, a.n_centroids);
    if (!a.centroids || !a.key_codes) return fail(SMAQ_ERR_INVALID, "decode: bvq tables missing");
  } else {
    return fail(SMAQ_ERR_INVALID, "decode: key_format %d", a.key_format);
  }
  if (a.value_bits != 2 && a.value_bits != 4) return fail(SMAQ_ERR_UNSUPPORTED, "decode: value bits %d", a.value_bits);
  if (a.group_size <= 0 || 128 % a.group_size || a.group_size % 4)
    return fail(SMAQ_ERR_UNSUPPORTED, "decode: group_size %d", a.group_size);
  if (!a.v_data || !a.v_scales || !a.v_zeros) return fail(SMAQ_ERR_INVALID, "decode: value streams missing");
  if (a.recent_len && (!a.recent_k || !a.recent_v)) return fail(SMAQ_ERR_INVALID, "decode: recent K/V missing");
  if ((reinterpret_cast<uintptr_t>(a.key_codes) & 15) || (reinterpret_cast<uintptr_t>(a.v_data) & 3))
    return fail(SMAQ_ERR_INVALID, "decode: key codes must be 16-byte aligned");

  p = DecodeParams{};
  p.q = a.q;
  p.q_dtype = a.q_dtype;
  p.q_sb = a.q_stride_b;
  p.q_sh = a.q_stride_h;
  p.B = a.batch;
  p.Hq = a.n_q_heads;
  p.Hkv = a.n_kv_heads;
  p.G = a.n_q_heads / a.n_kv_heads;
  p.D = a.head_dim;
  p.scale = a.scale;
  p.E_inv = a.E_inv;
  p.cent = a.centroids;
  p.nc = a.key_format == SMAQ_KEYS_BVQ ? a.n_centroids : (1 << a.key_bits);
  p.kcodes = a.key_codes;
  p.knorms = a.key_norms;
  p.kv_dtype = a.kv_dtype;
  p.vdata = a.v_data;
  p.vscales = a.v_scales;
  p.vzeros = a.v_zeros;
  p.gs = a.group_size;
  p.bt = a.block_table;
  p.bt_stride = a.bt_stride;
  p.page_size = a.page_size;
  p.hist_len = a.hist_len;
  p.hist_total = a.hist_total;
  p.min_hist = a.min_history;
  p.rk = a.recent_k;
  p.rv = a.recent_v;
  p.r_dtype = a.recent_dtype;
  p.r_sb = a.r_stride_b;
  p.r_st = a.r_stride_t;
  p.r_sh = a.r_stride_h;
  p.recent_len = a.recent_len;
  p.n_seg = 2 * a.batch * a.n_kv_heads;
  p.layout = a.layout;
  p.cent16 = a.key_format == SMAQ_KEYS_BVQ ? static_cast<const uint16_t*>(a.centroids_f16) : nullptr;
  return SMAQ_OK;
}

// Which kernel path smaq_decode takes for these arguments (see smaq_decode_kernel_path).
static int decode_path(const DecodeParams& p, int kb, int value_bits) {
  if (kb == 0 && decode_v2_eligible(p, SMAQ_KEYS_BVQ, value_bits, p.q_dtype) &&
      p.n_seg <= decode_v2_max_fused_segments(p.G))
    return SMAQ_PATH_FUSED_BVQ;
  if (kb != 0 && decode_s_eligible(p, kb, value_bits)) return SMAQ_PATH_FUSED_SCALAR;
  return SMAQ_PATH_GENERAL;
}
}  // namespace smaq

extern "C" int smaq_decode_kernel_path(const smaq_decode_args* args) {
  DecodeParams p;
  int kb = 0;
  const int st = decode_params(args, p, kb);
  return st ? -st : decode_path(p, kb, args->value_bits);
}

extern "C" int smaq_decode(const smaq_decode_args* args, void* stream) {
  DecodeParams p;
  int kb = 0;
  int st = decode_params(args, p, kb);
  if (st) return st;
  const smaq_decode_args& a = *args;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int grid = 0;
  st = dispatch_decode(p, kb, a.value_bits, a.num_ctas, s, &grid, true);
  if (st) return st;
  const size_t need = plan_bytes(p.n_seg) + sizeof(float) * size_t(grid + p.n_seg) * p.G * (p.D + 2);
  if (!a.workspace || a.workspace_bytes < need)
    return fail(SMAQ_ERR_WORKSPACE, "decode: workspace %zu bytes < %zu needed", a.workspace_bytes, need);
  p.plan = static_cast<int64_t*>(a.workspace);
  p.pair_cnt = reinterpret_cast<uint64_t*>(static_cast<char*>(a.workspace) + plan_table_bytes(p.n_seg));
  p.slots = reinterpret_cast<float*>(static_cast<char*>(a.workspace) + plan_bytes(p.n_seg));
  p.grid = grid;
  if (decode_path(p, kb, a.value_bits) != SMAQ_PATH_GENERAL) {
    // one launch: partition, history, window and the per-pair merge in the tensor-core kernel
    static std::atomic<uint32_t> epochs{0};
    uint32_t e = ++epochs;
    if (e == 0) e = ++epochs;
    p.fused = 1;
    p.pdl = a.overlap_prior ? 1 : 0;
    p.epoch = e;
    p.out = a.out;
    p.o_sb = a.o_stride_b;
    p.o_sh = a.o_stride_h;
    p.partial_out = a.partial_out;
    return dispatch_decode(p, kb, a.value_bits, grid, s, &grid, false);
  }
  decode_plan_kernel<<<1, 1024, 0, s>>>(p);
  st = cuda_status(cudaGetLastError(), "decode_plan_kernel");
  if (st) return st;
  st = dispatch_decode(p, kb, a.value_bits, grid, s, &grid, false);
  if (st) return st;
  decode_merge_kernel<<<a.batch * a.n_kv_heads, 256, 0, s>>>(p, a.out, a.o_stride_b, a.o_stride_h, a.partial_out);
  return cuda_status(cudaGetLastError(), "decode_merge_kernel");
}

extern "C" int smaq_merge_partials(const float* partials, int n_parts, int batch, int n_q_heads, int head_dim,
                                   void* out, int out_dtype, int64_t o_stride_b, int64_t o_stride_h,
                                   void* stream) {
  if (!partials || !out || n_parts <= 0 || batch <= 0 || n_q_heads <= 0 || head_dim <= 0)
    return fail(SMAQ_ERR_INVALID, "merge_partials: bad arguments");
  merge_partials_kernel<<<batch * n_q_heads, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      partials, n_parts, batch, n_q_heads, head_dim, out, out_dtype, o_stride_b, o_stride_h);
  return cuda_status(cudaGetLastError(), "merge_partials_kernel");
}

// ---------------------------------------------------------------- device status
namespace smaq {
__global__ void selftest_wait_kernel(uint32_t limit, int* status) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);  // one arrival expected, none ever comes
    fence_mbar_init();
  }
  __syncthreads();
  const bool done = mbar_wait(&bar, 0, limit);
  if (threadIdx.x == 0) *status = done ? 0 : 1;
  __syncthreads();
  if (threadIdx.x == 0) mbar_arrive_expect_tx(&bar, 0);  // complete the phase before the CTA exits
}
__device__ int g_selftest_status;
}  // namespace smaq

int smaq_noalloc_scratch(void** out);  // decode_noalloc.cu

extern "C" int smaq_decode_status(const void* workspace, int batch, int n_kv_heads, void* stream) {
  if (batch <= 0 || n_kv_heads <= 0) return smaq::fail(SMAQ_ERR_INVALID, "decode status: bad sizes");
  const int n_seg = 2 * batch * n_kv_heads;
  const void* ws = workspace;
  if (!ws) {  // the no-allocation entry point's scratch on the current device
    void* p = nullptr;
    const int st = smaq_noalloc_scratch(&p);
    if (st) return st;
    ws = p;
  }
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return smaq::cuda_status(e, "decode status: stream");
  int word = 0;
  e = cudaMemcpy(&word, static_cast<const int64_t*>(ws) + n_seg + 2, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return smaq::cuda_status(e, "decode status: read");
  if (word) return smaq::fail(SMAQ_ERR_DEVICE, "decode: a bounded device wait ran out (stream data never arrived)");
  return SMAQ_OK;
}

extern "C" int smaq_selftest_wait_timeout(unsigned int spin_limit, void* stream) {
  int* st = nullptr;
  cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&st), smaq::g_selftest_status);
  if (e != cudaSuccess) return smaq::cuda_status(e, "selftest: symbol");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  smaq::selftest_wait_kernel<<<1, 32, 0, s>>>(spin_limit, st);
  e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return smaq::cuda_status(e, "selftest: kernel");
  int word = -1;
  e = cudaMemcpy(&word, st, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return smaq::cuda_status(e, "selftest: read");
  if (word) return smaq::fail(SMAQ_ERR_DEVICE, "selftest: the wait ran out after %u polls and returned", spin_limit);
  return SMAQ_OK;
}
