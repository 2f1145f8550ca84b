// Device k-means for block-VQ calibration (sm_100a): k-means++ seeding then Lloyd iterations,
// every block of the head dim at once, with no host round trip per centre or per iteration.
//
// Same algorithm as SMAQBlockVQ's calibration (smaq/block_vq.py:37-79): first centre uniform,
// every further centre drawn with probability proportional to the squared distance to the
// nearest chosen centre, then Lloyd steps (nearest centre, first index on ties; mean of the
// assigned points; an empty cluster keeps its centre).  The random draws come from a
// counter-based generator (splitmix64 of seed, block and step), not torch's generator, so a
// seed gives a codebook of the same quality but not the reference's exact codebook.
//  * Seeding: one CTA per block keeps the nearest-centre squared distance of every point in
//    global scratch and updates it with each new centre (O(n) per centre instead of a full
//    distance matrix); the draw is a block-wide prefix sum over per-thread contiguous chunks.
//  * Assignment: one thread per point, the block's centres in shared memory.
//  * Update: one warp per centre sums its points in index order (ballot + fixed-order warp
//    reduction), so the result is deterministic.
#include "common.cuh"

namespace smaq {
namespace {

constexpr int KM_SEED_THREADS = 1024;
constexpr int KM_MAX_D = 16;

__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

// Uniform in [0, 1) with 53 random bits, draw `step` of block `b`.
__device__ __forceinline__ double uniform01(uint64_t seed, int b, int step) {
  const uint64_t r = splitmix64(seed * 0x100000001B3ull ^ (uint64_t(b) << 40) ^ uint64_t(step));
  return double(r >> 11) * (1.0 / 9007199254740992.0);
}

__device__ __forceinline__ float sqdist(const float* x, const float* c, int d) {
  float s = 0.f;
  for (int e = 0; e < d; ++e) {
    const float t = x[e] - c[e];
    s = fmaf(t, t, s);
  }
  return s;
}

__global__ void __launch_bounds__(KM_SEED_THREADS) kmeans_seed_kernel(const float* __restrict__ data, int64_t n, int d,
                                                                     int k, uint64_t seed, float* __restrict__ cent,
                                                                     float* __restrict__ dmin) {
  __shared__ double part[KM_SEED_THREADS];
  __shared__ float cur[KM_MAX_D];
  __shared__ int64_t pick;
  const int b = blockIdx.x, tid = threadIdx.x;
  const float* x = data + int64_t(b) * n * d;
  float* c = cent + int64_t(b) * k * d;
  float* dm = dmin + int64_t(b) * n;
  const int64_t chunk = (n + KM_SEED_THREADS - 1) / KM_SEED_THREADS;
  const int64_t i0 = min(n, tid * chunk), i1 = min(n, i0 + chunk);
  if (tid == 0) {
    const int64_t p0 = int64_t(uniform01(seed, b, 0) * double(n));
    pick = p0 < n ? p0 : n - 1;
  }
  __syncthreads();
  for (int j = 0; j < k; ++j) {
    if (tid < d) {
      cur[tid] = x[pick * d + tid];
      c[int64_t(j) * d + tid] = cur[tid];
    }
    __syncthreads();
    if (j == k - 1) break;
    // nearest-centre squared distances and this thread's chunk sum (fp64, fixed order)
    double s = 0.0;
    for (int64_t i = i0; i < i1; ++i) {
      const float dd = sqdist(x + i * d, cur, d);
      const float v = j == 0 ? dd : fminf(dm[i], dd);
      dm[i] = v;
      s += double(v);
    }
    part[tid] = s;
    __syncthreads();
    // inclusive scan of the chunk sums (Hillis-Steele in shared memory)
    for (int off = 1; off < KM_SEED_THREADS; off <<= 1) {
      const double add = tid >= off ? part[tid - off] : 0.0;
      __syncthreads();
      part[tid] += add;
      __syncthreads();
    }
    const double tot = part[KM_SEED_THREADS - 1];
    const double u = uniform01(seed, b, j + 1);
    if (!(tot > 0.0)) {
      if (tid == 0) {
        const int64_t p0 = int64_t(u * double(n));
        pick = p0 < n ? p0 : n - 1;
      }
    } else {
      const double target = u * tot;
      const double lo = tid ? part[tid - 1] : 0.0;
      if (target >= lo && (target < part[tid] || tid == KM_SEED_THREADS - 1) && i0 < i1) {
        double acc = lo;
        int64_t p = i1 - 1;
        for (int64_t i = i0; i < i1; ++i) {
          acc += double(dm[i]);
          if (acc > target) {
            p = i;
            break;
          }
        }
        pick = p;
      }
    }
    __syncthreads();
  }
}

__global__ void kmeans_assign_kernel(const float* __restrict__ data, int64_t n, int d, int k,
                                     const float* __restrict__ cent, int* __restrict__ assign) {
  extern __shared__ float cs[];  // [k][d]
  const int b = blockIdx.y;
  for (int i = threadIdx.x; i < k * d; i += blockDim.x) cs[i] = cent[int64_t(b) * k * d + i];
  __syncthreads();
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float xv[KM_MAX_D];
  const float* x = data + (int64_t(b) * n + i) * d;
  for (int e = 0; e < d; ++e) xv[e] = x[e];
  float best = INFINITY;
  int arg = 0;
  for (int c = 0; c < k; ++c) {
    const float dd = sqdist(xv, cs + c * d, d);
    if (dd < best) {
      best = dd;
      arg = c;
    }
  }
  assign[int64_t(b) * n + i] = arg;
}

__global__ void kmeans_update_kernel(const float* __restrict__ data, int64_t n, int d, int k,
                                     const int* __restrict__ assign, float* __restrict__ cent) {
  const int lane = threadIdx.x & 31;
  const int c = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int b = blockIdx.y;
  if (c >= k) return;
  const int* as = assign + int64_t(b) * n;
  const float* x = data + int64_t(b) * n * d;
  float sum[KM_MAX_D];
  for (int e = 0; e < KM_MAX_D; ++e) sum[e] = 0.f;
  int cnt = 0;
  for (int64_t base = 0; base < n; base += 32) {
    const int64_t i = base + lane;
    const bool mine = i < n && as[i] == c;
    unsigned m = __ballot_sync(0xffffffffu, mine);
    while (m) {  // the matching points in index order, every lane adds the same values
      const int src = __ffs(m) - 1;
      m &= m - 1;
      const float* p = x + (base + src) * d;
      for (int e = 0; e < d; ++e) sum[e] += p[e];
      ++cnt;
    }
  }
  if (lane < d && cnt > 0) cent[(int64_t(b) * k + c) * d + lane] = sum[lane] / float(cnt);
}

}  // namespace
}  // namespace smaq

using namespace smaq;

extern "C" size_t smaq_kmeans_workspace_size(int n_blocks, int64_t n_points) {
  return size_t(n_blocks) * size_t(n_points) * sizeof(float);
}

extern "C" int smaq_kmeans(const float* data, int n_blocks, int64_t n_points, int dim, int n_centroids, int n_iters,
                           uint64_t seed, float* centroids, void* workspace, size_t workspace_bytes, void* stream) {
  if (!data || !centroids || n_blocks <= 0 || n_blocks > 65535 || n_points <= 0 || dim <= 0 || dim > KM_MAX_D ||
      n_centroids <= 0 || n_centroids > 4096 || n_iters < 0)
    return fail(SMAQ_ERR_INVALID, "kmeans: bad arguments (blocks %d, points %lld, dim %d, centroids %d, iters %d)",
                n_blocks, (long long)n_points, dim, n_centroids, n_iters);
  if (n_points < n_centroids)
    return fail(SMAQ_ERR_INVALID, "kmeans: %lld points < %d centroids", (long long)n_points, n_centroids);
  const size_t need = smaq_kmeans_workspace_size(n_blocks, n_points);
  if (!workspace || workspace_bytes < need)
    return fail(SMAQ_ERR_WORKSPACE, "kmeans: workspace %zu bytes < %zu needed", workspace_bytes, need);
  const size_t smem = sizeof(float) * size_t(n_centroids) * dim;
  if (smem > 227 * 1024) return fail(SMAQ_ERR_UNSUPPORTED, "kmeans: %zu bytes of centroids", smem);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* dmin = static_cast<float*>(workspace);
  kmeans_seed_kernel<<<n_blocks, KM_SEED_THREADS, 0, s>>>(data, n_points, dim, n_centroids, seed, centroids, dmin);
  int st = cuda_status(cudaGetLastError(), "kmeans_seed_kernel");
  if (st || n_iters == 0) return st;
  // the assignment array reuses the distance scratch (same size)
  int* assign = static_cast<int*>(workspace);
  if (smem > 48 * 1024) {
    st = cuda_status(cudaFuncSetAttribute(kmeans_assign_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          int(smem)), "kmeans attr");
    if (st) return st;
  }
  const dim3 ga(unsigned((n_points + 255) / 256), unsigned(n_blocks));
  const dim3 gu(unsigned((n_centroids + 7) / 8), unsigned(n_blocks));
  for (int it = 0; it < n_iters; ++it) {
    kmeans_assign_kernel<<<ga, 256, smem, s>>>(data, n_points, dim, n_centroids, centroids, assign);
    kmeans_update_kernel<<<gu, 256, 0, s>>>(data, n_points, dim, n_centroids, assign, centroids);
  }
  return cuda_status(cudaGetLastError(), "kmeans lloyd");
}
