/*
 * smaq_b200 -- C ABI of the B200-native SMAQ compressed-KV hot path.
 *
 * Every entry point takes plain device pointers, sizes, strides and a
 * cudaStream_t (passed as void*), enqueues work on that stream without a host
 * synchronisation, and returns an int status (SMAQ_OK == 0).  A non-zero
 * status leaves a message for smaq_last_error() (thread-local).  Nothing here
 * allocates device memory except where a function says so; scratch space is
 * caller-provided ("workspace").
 *
 * Reference interfaces replaced (gauravsaini/smaq, file:line):
 *   smaq_quantize_keys_scalar  <- SMAQQuantizer.quantize          smaq/quantizer.py:138-145
 *                                 (+ _pack_indices                smaq/quantizer.py:34-46)
 *   smaq_quantize_values       <- quantize_values                 smaq/kv_cache.py:50-91
 *   smaq_quantize_keys_bvq     <- SMAQBlockVQ.quantize            smaq/block_vq.py:216-244
 *   smaq_append                <- CompressedKVStore.append_chunk  smaq/store.py:83-95
 *                                 (keys + values in one pass, written straight into the
 *                                  store's preallocated / paged rows)
 *   smaq_decode                <- compute_hybrid_attention        smaq/score.py:23-72
 *                                 (+ _quantized_scores / _exact_scores / _apply_weights
 *                                  smaq/score.py:75-124, SMAQQuantizer.attention_score
 *                                  smaq/quantizer.py:154-184, SMAQBlockVQ.attention_score
 *                                  smaq/block_vq.py:273-297, dequantize_values
 *                                  smaq/kv_cache.py:94-103)
 *   smaq_key_scores            <- SMAQQuantizer.attention_score   smaq/quantizer.py:154-184,
 *                                 SMAQBlockVQ.attention_score     smaq/block_vq.py:273-297
 *   smaq_attend_values         <- SMAQKVCache.attend (history)    smaq/kv_cache.py:243-267
 *   smaq_kmeans                <- _kmeans (block-VQ calibration)  smaq/block_vq.py:37-79
 *   smaq_merge_partials        <- (new) log-sum-exp combine of sequence-split partials;
 *                                 the reference has no multi-GPU path.
 *
 * Store layout ("rows").  All compressed streams of a layer share one row
 * index.  The store is [n_pages, n_kv_heads, page_size] rows; row r of a
 * stream lives at base + r * row_bytes.  Token t of a chunk lands in slot
 *   s = slots ? slots[t] : slot_offset + t,   page = s / page_size,
 *   row = (page * n_kv_heads + h) * page_size + s % page_size.
 * A contiguous per-head store [n_kv_heads, capacity] is page_size = capacity
 * with one page (SMAQ_LAYOUT_DECODE stores need page_size % 16 == 0).  Decode reads token t of
 * sequence b from page = block_table ? block_table[b * bt_stride + t / page_size] : b.
 *
 * SMAQ_LAYOUT_DECODE permutes bytes inside rows (same bits, same row sizes):
 *   block-VQ indices (16 blocks): byte 2 * (4 * (b / 8) + b % 4) + (b / 4) % 2 of a row holds
 *     the index of block b, so the pair of blocks (b, b + 4) a tensor-core lane gathers for
 *     one token sits in one 16-bit half of one 32-bit word;
 *   2-bit values (head_dim 128): byte 4 * g + j of a row holds reference byte 8 * j + g
 *     (g < 8, j < 4), so each 32-bit word carries one byte of every value group;
 *   3/4-bit scalar key codes (head_dim 128, 64-byte rows): byte 16 * (p % 4) + p / 4 holds
 *     reference byte p, so the 16 bytes a tensor-core lane needs for one token are contiguous.
 * Reference-layout bytes are recovered by the inverse permutation.
 */
#ifndef SMAQ_B200_H_
#define SMAQ_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SMAQ_ABI_VERSION 2

/* element types */
enum { SMAQ_F32 = 0, SMAQ_BF16 = 1, SMAQ_F16 = 2 };
/* key formats */
enum { SMAQ_KEYS_NONE = 0, SMAQ_KEYS_SCALAR = 1, SMAQ_KEYS_BVQ = 2 };
/* store row layouts */
enum {
  SMAQ_LAYOUT_REFERENCE = 0, /* bytes exactly as the reference packs them */
  SMAQ_LAYOUT_DECODE = 1     /* decode-friendly byte order inside each row group (see below) */
};
/* status codes */
enum {
  SMAQ_OK = 0,
  SMAQ_ERR_INVALID = 1,      /* bad pointer / shape / stride / alignment */
  SMAQ_ERR_UNSUPPORTED = 2,  /* valid request outside the compiled configurations */
  SMAQ_ERR_CUDA = 3,         /* a CUDA runtime call failed */
  SMAQ_ERR_WORKSPACE = 4,    /* workspace too small */
  SMAQ_ERR_DEVICE = 5,       /* the device reported an error word */
  SMAQ_ERR_TIMEOUT = 6,      /* a collective made no progress before its deadline (a peer is missing) */
  SMAQ_ERR_PEER = 7          /* a collective failed (remote or NCCL error); the communicator is aborted */
};

int smaq_abi_version(void);
/* No counterpart in the reference.  sizeof(smaq_append_args) for which = 0, sizeof(smaq_decode_args)
 * for which = 1, sizeof(smaq_scores_args) for 2, sizeof(smaq_attend_args) for 3, else 0: a binding
 * compares its own mirror of the structs with these. */
size_t smaq_args_size(int which);
const char* smaq_last_error(void);

/* ------------------------------------------------------------------ append */

typedef struct smaq_append_args {
  /* Input chunk, element (t, h, d) at ptr + t*stride_t + h*stride_h + d
   * (elements of `dtype`).  k or v may be NULL to skip that half. */
  const void* k;
  const void* v;
  int dtype;
  int64_t n_tokens;
  int n_heads;
  int head_dim;
  int64_t k_stride_t, k_stride_h;
  int64_t v_stride_t, v_stride_h;
  /* destination rows (see the layout note above) */
  const int64_t* slots; /* nullable, [n_tokens] */
  int64_t slot_offset;
  int64_t page_size;
  /* key format */
  int key_format;            /* SMAQ_KEYS_SCALAR or SMAQ_KEYS_BVQ */
  int key_bits;              /* scalar: 2, 3 or 4 */
  const float* E;            /* scalar: [D, D] row-major fp32, y = k_unit @ E^T */
  const float* boundaries;   /* scalar: [2^bits - 1] ascending fp32 */
  const float* E_blocks;     /* bvq: [D/bd, bd, bd] fp32 */
  const float* centroids;    /* bvq: [D/bd, n_centroids, bd] fp32 (encode space) */
  int block_dim;             /* bvq: 8 */
  int n_centroids;           /* bvq: <= 256 */
  uint8_t* key_codes;        /* scalar: rows of ceil(D / (8/bits)) bytes; bvq: rows of D/bd bytes */
  void* key_norms;           /* scalar: rows of one `dtype` element */
  /* value format */
  int value_bits;            /* 2 or 4 */
  int group_size;            /* 32, 64 or 128 */
  uint8_t* v_data;           /* rows of D*bits/8 bytes */
  void* v_scales;            /* rows of D/group_size `dtype` elements */
  void* v_zeros;             /* rows of D/group_size `dtype` elements */
  int layout;                /* SMAQ_LAYOUT_REFERENCE or SMAQ_LAYOUT_DECODE */
} smaq_append_args;

/* Quantize a chunk of keys and/or values straight into store rows. */
int smaq_append(const smaq_append_args* args, void* stream);

/* Reference-shaped helpers (dense rows in, dense rows out, n_rows = prod(leading dims)). */
int smaq_quantize_keys_scalar(const void* k, int dtype, int64_t n_rows, int head_dim,
                              const float* E, const float* boundaries, int bits,
                              uint8_t* codes_out, void* norms_out, void* stream);
int smaq_quantize_values(const void* v, int dtype, int64_t n_rows, int head_dim, int bits,
                         int group_size, uint8_t* data_out, void* scales_out, void* zeros_out,
                         void* stream);
int smaq_quantize_keys_bvq(const void* k, int dtype, int64_t n_rows, int head_dim,
                           const float* E_blocks, const float* centroids, int block_dim,
                           int n_centroids, uint8_t* idx_out, void* stream);

/* ------------------------------------------------------------------ decode */

typedef struct smaq_decode_args {
  /* queries [B, Hq, D]: element (b, h, d) at q + b*q_stride_b + h*q_stride_h + d */
  const void* q;
  int q_dtype;
  int64_t q_stride_b, q_stride_h;
  int batch, n_q_heads, n_kv_heads, head_dim;
  float scale;
  /* compressed history (store rows, see the layout note) */
  int key_format;            /* SMAQ_KEYS_SCALAR / SMAQ_KEYS_BVQ / SMAQ_KEYS_NONE */
  int key_bits;
  const float* E_inv;        /* scalar: [D, D] fp32, q_rot = q @ E_inv^T */
  const float* centroids;    /* scalar: [2^bits] fp32; bvq: decoded centroids [D/bd, nc, bd] fp32 */
  int block_dim, n_centroids;
  const uint8_t* key_codes;
  const void* key_norms;     /* scalar only, `kv_dtype` */
  int kv_dtype;              /* dtype of norms / value scales / value zeros */
  const uint8_t* v_data;
  const void* v_scales;
  const void* v_zeros;
  int value_bits, group_size;
  const int32_t* block_table; /* nullable: [B, bt_stride] page ids */
  int64_t bt_stride;
  int64_t page_size;
  const int32_t* hist_len;    /* [B] device */
  const int32_t* hist_total;  /* nullable [B]: history length of the whole sequence (for the
                                  minimum-history rule when the history is split across GPUs) */
  int min_history;            /* 16 in the reference */
  /* exact recent window: element (b, t, h, d) at r + b*r_stride_b + t*r_stride_t + h*r_stride_h + d */
  const void* recent_k;
  const void* recent_v;
  int recent_dtype;
  int64_t r_stride_b, r_stride_t, r_stride_h;
  const int32_t* recent_len; /* nullable [B] device */
  /* outputs: either the final attention output (query dtype) ... */
  void* out;
  int64_t o_stride_b, o_stride_h;
  /* ... and/or fp32 partials [B, Hq, 2*D + 2] (acc_hist[D], acc_recent[D], m, l) for a
   * cross-GPU merge with smaq_merge_partials.  Either pointer may be NULL, not both. */
  float* partial_out;
  /* scratch */
  void* workspace;
  size_t workspace_bytes;
  int num_ctas;              /* 0: one wave over the device's SMs */
  int layout;                /* row layout of the history streams */
  /* bvq only, nullable: the decoded centroids as fp16 [D/bd, nc, bd].  The caller promises
   * they equal `centroids` exactly (an fp16-valued codebook); with SMAQ_LAYOUT_DECODE rows,
   * bf16/fp16 queries, 2-bit values and group 32 this selects the tensor-core kernel. */
  const void* centroids_f16;
  /* Nonzero: launch the single-launch kernels with programmatic dependent launch, so that their
   * partition and first history copies overlap the end of the previous kernel on the stream.
   * The caller promises that kernel writes none of: key_codes / key_norms / v_data / v_scales /
   * v_zeros rows, block_table, hist_len, hist_total, recent_len, and the codebooks (centroids,
   * centroids_f16, E_inv).  Queries, the window, outputs
   * and the workspace are read or written only after that kernel has completed.  Ignored by the
   * multi-launch path.  Zero gives plain stream ordering. */
  int overlap_prior;
} smaq_decode_args;

/* Bytes of workspace smaq_decode needs for these shapes (host-only computation). */
size_t smaq_decode_workspace_size(int batch, int n_q_heads, int n_kv_heads, int head_dim,
                                  int num_ctas);
int smaq_decode(const smaq_decode_args* args, void* stream);

/* No counterpart in the reference (it has one implementation).  The kernel path smaq_decode
 * takes for these arguments, without launching anything: SMAQ_PATH_FUSED_BVQ (one launch,
 * block-VQ keys, tensor-core scores and P.V), SMAQ_PATH_FUSED_SCALAR (one launch, 3/4-bit
 * scalar keys, tensor-core scores and P.V) or SMAQ_PATH_GENERAL (partition, SIMT decode and
 * merge launches: every other supported format); a negative status for invalid arguments. */
enum { SMAQ_PATH_GENERAL = 0, SMAQ_PATH_FUSED_BVQ = 1, SMAQ_PATH_FUSED_SCALAR = 2 };
int smaq_decode_kernel_path(const smaq_decode_args* args);

/* No counterpart in the reference.  smaq_decode without a caller workspace, for callers that
 * cannot allocate device memory (all device memory owned by another allocator or pool, or a
 * host that reaches the GPU only through this ABI).  Scratch comes from a fixed 8 MiB array in
 * the library's device image (held on every GPU that loads the library until exit; its size is
 * smaq_decode_noalloc_max_workspace()).  Shapes whose workspace need, for the grid the call
 * picks, exceeds it are rejected with SMAQ_ERR_WORKSPACE before anything is launched.
 * args->workspace / workspace_bytes are ignored.  The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress) with that device current, and again whenever the current
 * context changes (a device reset reloads the module), so make the first call -- and the first
 * after a reset -- before any stream capture.  Every call shares the one array
 * and fully rewrites what it reads, so nothing carries over between calls; calls that can
 * overlap on the GPU (different streams, or several threads) race on it -- serialise them. */
int smaq_decode_noalloc(const smaq_decode_args* args, void* stream);
size_t smaq_decode_noalloc_max_workspace(void);

/* Merge R partial sets [R, B, Hq, 2*D+2] (as written to partial_out) into the
 * final output [B, Hq, D] (element (b, h, d) at out + b*o_stride_b + h*o_stride_h + d). */
int smaq_merge_partials(const float* partials, int n_parts, int batch, int n_q_heads, int head_dim,
                        void* out, int out_dtype, int64_t o_stride_b, int64_t o_stride_h,
                        void* stream);

/* Failure detection.  Every device-side wait (mbarrier, cross-CTA counter) polls a bounded
 * number of times; one that runs out records an error word and the kernel returns instead of
 * hanging, so the context stays usable.  These calls synchronise `stream` and read that word.
 *   smaq_decode_status: the word of the smaq_decode call that used `workspace` for a
 *     (batch, n_kv_heads) shape (NULL = the smaq_decode_noalloc scratch of the current device).
 *   smaq_append_status: the key kernel's word; reading clears it.
 * Both return SMAQ_OK, or SMAQ_ERR_DEVICE with a message for smaq_last_error().
 *   smaq_selftest_wait_timeout: launches one warp that waits on an mbarrier nothing arrives at,
 *     polling `spin_limit` times, and returns SMAQ_ERR_DEVICE once the wait has run out and the
 *     kernel has returned (the failure path, exercised without any device fault). */
int smaq_decode_status(const void* workspace, int batch, int n_kv_heads, void* stream);
int smaq_append_status(void* stream);
int smaq_selftest_wait_timeout(unsigned int spin_limit, void* stream);


/* ------------------------------------------------------------------ standalone scores / attend */

/* Scores of query rows against compressed history keys, without a softmax:
 *   out[g, q, t] = scale * q[g, q] . k_hat[g, t]          (in out_dtype)
 * Replaces SMAQQuantizer.attention_score (smaq/quantizer.py:154-184), SMAQBlockVQ.attention_score
 * (smaq/block_vq.py:273-297) and the history half of SMAQKVCache.attention_scores
 * (smaq/kv_cache.py:218-241).  Keys in the reference layout:
 *   scalar: the packed row of token (g, t) at key_codes + g*codes_stride_g + t*ceil(D/(8/bits))
 *           bytes, its norm at key_norms + g*norms_stride_g + t (norms_dtype); k_hat =
 *           (centroids[codes] @ E_inv) * norm, computed as (q @ E_inv^T) . centroids[codes] * norm;
 *   bvq:    index (g, t, block) at key_idx + g*idx_stride_g + t*(D/block_dim) + block (uint8, or
 *           int64 when idx_is_int64); k_hat = decoded_centroids[block][index] ([D/bd, nc, bd] fp32).
 * Queries: element (g, q, d) at q + g*q_stride_g + q*q_stride_q + d.  D % 32 == 0, D <= 256. */
typedef struct smaq_scores_args {
  const void* q;
  int q_dtype;
  int64_t q_stride_g, q_stride_q;
  int64_t n_groups;
  int n_queries;
  int64_t n_tokens;
  int head_dim;
  int key_format;                  /* SMAQ_KEYS_SCALAR or SMAQ_KEYS_BVQ */
  const uint8_t* key_codes;        /* scalar */
  int64_t codes_stride_g;          /* bytes */
  const void* key_norms;           /* scalar */
  int norms_dtype;
  int64_t norms_stride_g;          /* elements */
  int key_bits;                    /* scalar: 2, 3 or 4 */
  const float* E_inv;              /* scalar: [D, D] */
  const float* centroids;          /* scalar: [2^bits] */
  const void* key_idx;             /* bvq */
  int idx_is_int64;
  int64_t idx_stride_g;            /* elements */
  int block_dim;                   /* bvq */
  int n_centroids;                 /* bvq: <= 256 */
  const float* decoded_centroids;  /* bvq */
  float scale;
  void* out;
  int out_dtype;
  int64_t out_stride_g, out_stride_q;  /* element (g, q, t) at out + g*.. + q*.. + t */
  int q_rotated;                   /* scalar: nonzero when q already holds q @ E_inv^T (E_inv unused) */
} smaq_scores_args;
int smaq_key_scores(const smaq_scores_args* args, void* stream);

/* Weighted sum of compressed history values (caller-given weights, e.g. a softmax):
 *   out[g, q, :] = sum_t w[g, q, t] * (code[g, t, :] * scale[g, t, grp] + zero[g, t, grp])
 * Replaces the history half of SMAQKVCache.attend (smaq/kv_cache.py:243-267) with
 * dequantize_values (smaq/kv_cache.py:94-103) fused in.  Value rows in the reference layout:
 * row (g, t) at v_data + g*data_stride_g + t*D*bits/8 bytes; scale / zero (g, t, grp) at
 * v_scales / v_zeros + g*sz_stride_g + t*(D/group_size) + grp.  Weights: element (g, q, t) at
 * w + g*w_stride_g + q*w_stride_q + t.  The token range is split over CTAs; the partial sums go
 * to the workspace (smaq_attend_workspace_size bytes) and are added in a fixed order. */
typedef struct smaq_attend_args {
  const void* w;
  int w_dtype;
  int64_t w_stride_g, w_stride_q;
  int64_t n_groups;
  int n_queries;
  int64_t n_tokens;
  int head_dim;
  const uint8_t* v_data;
  int64_t data_stride_g;           /* bytes */
  const void* v_scales;
  const void* v_zeros;
  int sz_dtype;
  int64_t sz_stride_g;             /* elements */
  int value_bits;                  /* 2 or 4 */
  int group_size;
  void* out;
  int out_dtype;
  int64_t out_stride_g, out_stride_q;  /* element (g, q, d) */
  void* workspace;
  size_t workspace_bytes;
} smaq_attend_args;
size_t smaq_attend_workspace_size(int64_t n_groups, int n_queries, int64_t n_tokens, int head_dim);
int smaq_attend_values(const smaq_attend_args* args, void* stream);


/* ------------------------------------------------------------------ collectives */

/* All-gather of sequence-split decode partials inside one split group (no counterpart in the
 * reference, which has no multi-GPU path; the partials are what smaq_merge_partials combines).
 * One communicator per split group, NCCL underneath, created NON-BLOCKING: every call returns
 * within its deadline.  A peer that never arrives gives SMAQ_ERR_TIMEOUT, a remote or NCCL
 * error SMAQ_ERR_PEER; both abort the communicator (ncclCommAbort), after which every call on
 * it fails and the caller destroys it.  The CUDA device of the communicator is the current
 * device at smaq_comm_init.  Sequence of a step: smaq_comm_allgather (enqueue on `stream`),
 * then smaq_comm_wait (host waits for the exchange, polling NCCL's asynchronous error state)
 * before the merged output is used. */
#define SMAQ_COMM_ID_BYTES 128
typedef struct smaq_comm* smaq_comm_t;
/* Calls the communicator uses, each returning an ncclResult_t value (0 success, 7 in
 * progress).  Default: NCCL from libnccl.so.2 (dlopen on first use; a process that loaded NCCL
 * already shares it).  A host with its own NCCL build, or a test, installs its own table;
 * NULL restores NCCL. */
typedef struct smaq_comm_backend {
  int (*unique_id)(uint8_t* id);
  int (*init_rank)(void** handle, int n_ranks, const uint8_t* id, int rank);  /* non-blocking */
  int (*async_error)(void* handle);
  int (*all_gather)(const void* send, void* recv, size_t bytes_per_rank, void* handle, void* stream);
  int (*abort_comm)(void* handle);
  int (*finalize)(void* handle);
  int (*destroy)(void* handle);
} smaq_comm_backend;
int smaq_comm_set_backend(const smaq_comm_backend* backend);
/* Rank 0 of the split group makes the id and hands it to the others (any host channel). */
int smaq_comm_unique_id(uint8_t* id /* SMAQ_COMM_ID_BYTES */);
int smaq_comm_init(smaq_comm_t* comm, int n_ranks, int rank, const uint8_t* id, double timeout_s);
/* recv[r * bytes .. (r+1) * bytes) <- rank r's send buffer, on `stream`. */
int smaq_comm_allgather(smaq_comm_t comm, const void* send, void* recv, size_t bytes, void* stream,
                        double timeout_s);
int smaq_comm_wait(smaq_comm_t comm, void* stream, double timeout_s);
/* Non-blocking poll of the asynchronous error state (aborts on an error). */
int smaq_comm_status(smaq_comm_t comm);
int smaq_comm_abort(smaq_comm_t comm);
/* Finalize (bounded by timeout_s, abort past it) and free; accepts an aborted communicator. */
int smaq_comm_destroy(smaq_comm_t comm, double timeout_s);

/* ------------------------------------------------------------------ calibration */

/* Block-VQ calibration k-means on the device (SMAQBlockVQ.fit's _kmeans, smaq/block_vq.py:37-79):
 * k-means++ seeding and n_iters Lloyd steps for n_blocks independent point sets at once.
 * data [n_blocks][n_points][dim] fp32 (dim <= 16), centroids [n_blocks][n_centroids][dim] fp32
 * out.  The draws come from a counter-based generator seeded with `seed`, not torch's, so the
 * codebook matches the reference's in quality, not bit for bit.  Deterministic for a seed.
 * Workspace: smaq_kmeans_workspace_size(n_blocks, n_points) bytes. */
size_t smaq_kmeans_workspace_size(int n_blocks, int64_t n_points);
int smaq_kmeans(const float* data, int n_blocks, int64_t n_points, int dim, int n_centroids, int n_iters,
                uint64_t seed, float* centroids, void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SMAQ_B200_H_ */
