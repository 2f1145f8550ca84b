// Partials exchange for sequence-split decode: an NCCL communicator driven in non-blocking mode
// with host-side deadlines.
//
// The reference runs on one device and has no collective layer.  When a long context is split
// over GPUs (sequence splits of one KV-head group), each rank all-gathers the fp32 decode
// partials of its split group and merges them with smaq_merge_partials.  This file owns that
// all-gather:
//  * the communicator is created non-blocking (ncclConfig_t.blocking = 0), so neither the
//    init nor an enqueue can block the host inside NCCL;
//  * every step is polled with ncclCommGetAsyncError against a wall-clock deadline; a peer
//    that never arrives (or a remote error) ends in ncclCommAbort and a status code
//    (SMAQ_ERR_TIMEOUT / SMAQ_ERR_PEER), never in a hang;
//  * smaq_comm_wait also watches a CUDA event recorded after the collective, so a rank learns
//    that its partner died while the all-gather kernel is still waiting for it.
// NCCL is loaded with dlopen("libnccl.so.2") on first use: a process that already loaded NCCL
// (torch does) shares that copy, and the library itself does not link against NCCL.  Callers
// that bring their own NCCL build, or a test double, install a smaq_comm_backend table.
#include <dlfcn.h>
#include <nccl.h>
#include <string.h>

#include <chrono>
#include <mutex>
#include <thread>

#include "common.cuh"

struct smaq_comm {
  void* handle;
  const smaq_comm_backend* be;
  int n_ranks, rank;
  int aborted;
  cudaEvent_t done;  // created on the first wait
};

namespace smaq {
namespace {

constexpr int kNcclSuccess = ncclSuccess, kNcclInProgress = ncclInProgress;

struct NcclCalls {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRankConfig) init_rank_config = nullptr;
  decltype(&ncclCommGetAsyncError) get_async_error = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclCommAbort) abort_comm = nullptr;
  decltype(&ncclCommFinalize) finalize = nullptr;
  decltype(&ncclCommDestroy) destroy = nullptr;
};

NcclCalls g_nccl;
std::mutex g_mu;
const smaq_comm_backend* g_backend = nullptr;  // nullptr: NCCL

bool load_nccl() {
  static bool tried = false, ok = false;
  if (tried) return ok;
  tried = true;
  void* so = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!so) so = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
  if (!so) return false;
#define SMAQ_SYM(field, name) g_nccl.field = reinterpret_cast<decltype(g_nccl.field)>(dlsym(so, name))
  SMAQ_SYM(get_unique_id, "ncclGetUniqueId");
  SMAQ_SYM(init_rank_config, "ncclCommInitRankConfig");
  SMAQ_SYM(get_async_error, "ncclCommGetAsyncError");
  SMAQ_SYM(all_gather, "ncclAllGather");
  SMAQ_SYM(abort_comm, "ncclCommAbort");
  SMAQ_SYM(finalize, "ncclCommFinalize");
  SMAQ_SYM(destroy, "ncclCommDestroy");
#undef SMAQ_SYM
  ok = g_nccl.get_unique_id && g_nccl.init_rank_config && g_nccl.get_async_error && g_nccl.all_gather &&
       g_nccl.abort_comm && g_nccl.finalize && g_nccl.destroy;
  return ok;
}

int nccl_unique_id(uint8_t* id) {
  ncclUniqueId u;
  const int r = g_nccl.get_unique_id(&u);
  if (r == kNcclSuccess) memcpy(id, u.internal, NCCL_UNIQUE_ID_BYTES);
  return r;
}
int nccl_init_rank(void** handle, int n_ranks, const uint8_t* id, int rank) {
  ncclUniqueId u;
  memcpy(u.internal, id, NCCL_UNIQUE_ID_BYTES);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclComm_t c = nullptr;
  const int r = g_nccl.init_rank_config(&c, n_ranks, u, rank, &cfg);
  *handle = c;
  return r;
}
int nccl_async_error(void* handle) {
  ncclResult_t st = ncclSuccess;
  const int r = g_nccl.get_async_error(static_cast<ncclComm_t>(handle), &st);
  return r != kNcclSuccess ? r : int(st);
}
int nccl_all_gather(const void* send, void* recv, size_t bytes, void* handle, void* stream) {
  return g_nccl.all_gather(send, recv, bytes, ncclUint8, static_cast<ncclComm_t>(handle),
                           static_cast<cudaStream_t>(stream));
}
int nccl_abort(void* handle) { return g_nccl.abort_comm(static_cast<ncclComm_t>(handle)); }
int nccl_finalize(void* handle) { return g_nccl.finalize(static_cast<ncclComm_t>(handle)); }
int nccl_destroy(void* handle) { return g_nccl.destroy(static_cast<ncclComm_t>(handle)); }

const smaq_comm_backend kNccl = {nccl_unique_id, nccl_init_rank, nccl_async_error, nccl_all_gather,
                                 nccl_abort,     nccl_finalize,  nccl_destroy};

int backend(const smaq_comm_backend** out) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_backend) {
    *out = g_backend;
    return SMAQ_OK;
  }
  if (!load_nccl()) return fail(SMAQ_ERR_UNSUPPORTED, "smaq_comm: libnccl.so.2 could not be loaded");
  *out = &kNccl;
  return SMAQ_OK;
}

using Clock = std::chrono::steady_clock;

Clock::time_point deadline_of(double timeout_s) {
  if (!(timeout_s > 0.0)) timeout_s = 0.0;
  if (timeout_s > 1e6) timeout_s = 1e6;
  return Clock::now() + std::chrono::duration_cast<Clock::duration>(std::chrono::duration<double>(timeout_s));
}

// Poll sleeps grow from 1 us to 1 ms: short exchanges finish in a few polls, long waits cost
// little host time.
void backoff(int& us) {
  std::this_thread::sleep_for(std::chrono::microseconds(us));
  if (us < 1000) us *= 2;
}

void abort_comm(smaq_comm* c) {
  if (c->aborted) return;
  c->aborted = 1;
  if (c->handle) c->be->abort_comm(c->handle);
}

// Wait until the communicator leaves ncclInProgress.  Anything but success within the deadline
// aborts the communicator.
int settle(smaq_comm* c, Clock::time_point deadline, const char* what) {
  int us = 1;
  for (;;) {
    const int r = c->be->async_error(c->handle);
    if (r == kNcclSuccess) return SMAQ_OK;
    if (r != kNcclInProgress) {
      abort_comm(c);
      return fail(SMAQ_ERR_PEER, "smaq_comm rank %d/%d: %s failed with NCCL status %d; communicator aborted",
                  c->rank, c->n_ranks, what, r);
    }
    if (Clock::now() >= deadline) {
      abort_comm(c);
      return fail(SMAQ_ERR_TIMEOUT, "smaq_comm rank %d/%d: %s made no progress before the deadline; "
                  "communicator aborted", c->rank, c->n_ranks, what);
    }
    backoff(us);
  }
}

int usable(smaq_comm* c, const char* what) {
  if (!c) return fail(SMAQ_ERR_INVALID, "%s: NULL communicator", what);
  if (c->aborted) return fail(SMAQ_ERR_PEER, "%s: the communicator was aborted", what);
  return SMAQ_OK;
}

}  // namespace
}  // namespace smaq

using namespace smaq;

extern "C" int smaq_comm_set_backend(const smaq_comm_backend* be) {
  if (be && !(be->unique_id && be->init_rank && be->async_error && be->all_gather && be->abort_comm &&
              be->finalize && be->destroy))
    return fail(SMAQ_ERR_INVALID, "smaq_comm_set_backend: every call of the table must be set");
  std::lock_guard<std::mutex> lk(g_mu);
  g_backend = be;
  return SMAQ_OK;
}

extern "C" int smaq_comm_unique_id(uint8_t* id) {
  if (!id) return fail(SMAQ_ERR_INVALID, "smaq_comm_unique_id: NULL id buffer");
  const smaq_comm_backend* be = nullptr;
  if (int st = backend(&be)) return st;
  const int r = be->unique_id(id);
  if (r != kNcclSuccess) return fail(SMAQ_ERR_PEER, "smaq_comm_unique_id: NCCL status %d", r);
  return SMAQ_OK;
}

extern "C" int smaq_comm_init(smaq_comm_t* out, int n_ranks, int rank, const uint8_t* id, double timeout_s) {
  if (!out || !id) return fail(SMAQ_ERR_INVALID, "smaq_comm_init: NULL argument");
  *out = nullptr;
  if (n_ranks < 1 || rank < 0 || rank >= n_ranks)
    return fail(SMAQ_ERR_INVALID, "smaq_comm_init: rank %d outside [0, %d)", rank, n_ranks);
  const smaq_comm_backend* be = nullptr;
  if (int st = backend(&be)) return st;
  smaq_comm* c = new smaq_comm{nullptr, be, n_ranks, rank, 0, nullptr};
  const int r = be->init_rank(&c->handle, n_ranks, id, rank);
  if (r != kNcclSuccess && r != kNcclInProgress) {
    if (c->handle) be->abort_comm(c->handle);
    delete c;
    return fail(SMAQ_ERR_PEER, "smaq_comm_init rank %d/%d: NCCL status %d", rank, n_ranks, r);
  }
  if (!c->handle) {
    delete c;
    return fail(SMAQ_ERR_PEER, "smaq_comm_init rank %d/%d: no communicator returned", rank, n_ranks);
  }
  if (int st = settle(c, deadline_of(timeout_s), "init")) {
    delete c;  // already aborted
    return st;
  }
  *out = c;
  return SMAQ_OK;
}

extern "C" int smaq_comm_allgather(smaq_comm_t c, const void* send, void* recv, size_t bytes, void* stream,
                                   double timeout_s) {
  if (int st = usable(c, "smaq_comm_allgather")) return st;
  if ((!send || !recv) && bytes) return fail(SMAQ_ERR_INVALID, "smaq_comm_allgather: NULL buffer");
  const int r = c->be->all_gather(send, recv, bytes, c->handle, stream);
  if (r != kNcclSuccess && r != kNcclInProgress) {
    abort_comm(c);
    return fail(SMAQ_ERR_PEER, "smaq_comm_allgather rank %d/%d: NCCL status %d; communicator aborted", c->rank,
                c->n_ranks, r);
  }
  return settle(c, deadline_of(timeout_s), "all-gather enqueue");
}

extern "C" int smaq_comm_wait(smaq_comm_t c, void* stream, double timeout_s) {
  if (int st = usable(c, "smaq_comm_wait")) return st;
  const auto deadline = deadline_of(timeout_s);
  bool recorded = false;
  int us = 1;
  for (;;) {
    const int r = c->be->async_error(c->handle);
    if (r != kNcclSuccess && r != kNcclInProgress) {
      abort_comm(c);
      return fail(SMAQ_ERR_PEER, "smaq_comm_wait rank %d/%d: NCCL status %d; communicator aborted", c->rank,
                  c->n_ranks, r);
    }
    if (!recorded) {
      if (!c->done) {
        if (int st = cuda_status(cudaEventCreateWithFlags(&c->done, cudaEventDisableTiming), "smaq_comm_wait"))
          return st;
      }
      if (int st = cuda_status(cudaEventRecord(c->done, static_cast<cudaStream_t>(stream)), "smaq_comm_wait"))
        return st;
      recorded = true;
    }
    const cudaError_t q = cudaEventQuery(c->done);
    if (q == cudaSuccess && r == kNcclSuccess) return SMAQ_OK;
    if (q != cudaSuccess && q != cudaErrorNotReady) return cuda_status(q, "smaq_comm_wait");
    if (Clock::now() >= deadline) {
      abort_comm(c);
      return fail(SMAQ_ERR_TIMEOUT, "smaq_comm_wait rank %d/%d: the exchange did not complete before the "
                  "deadline (a peer is missing); communicator aborted", c->rank, c->n_ranks);
    }
    backoff(us);
  }
}

extern "C" int smaq_comm_status(smaq_comm_t c) {
  if (int st = usable(c, "smaq_comm_status")) return st;
  const int r = c->be->async_error(c->handle);
  if (r == kNcclSuccess || r == kNcclInProgress) return SMAQ_OK;
  abort_comm(c);
  return fail(SMAQ_ERR_PEER, "smaq_comm_status rank %d/%d: NCCL status %d; communicator aborted", c->rank,
              c->n_ranks, r);
}

extern "C" int smaq_comm_abort(smaq_comm_t c) {
  if (!c) return fail(SMAQ_ERR_INVALID, "smaq_comm_abort: NULL communicator");
  abort_comm(c);
  return SMAQ_OK;
}

extern "C" int smaq_comm_destroy(smaq_comm_t c, double timeout_s) {
  if (!c) return SMAQ_OK;
  int st = SMAQ_OK;
  if (!c->aborted) {
    const int r = c->be->finalize(c->handle);
    if (r != kNcclSuccess && r != kNcclInProgress) {
      abort_comm(c);
      st = fail(SMAQ_ERR_PEER, "smaq_comm_destroy: finalize returned NCCL status %d; communicator aborted", r);
    } else {
      st = settle(c, deadline_of(timeout_s), "finalize");  // aborts on failure
    }
    if (!c->aborted) c->be->destroy(c->handle);
  }
  if (c->done) cudaEventDestroy(c->done);
  delete c;
  return st;
}
