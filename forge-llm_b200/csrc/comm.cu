// Data-parallel gradient exchange behind the C-ABI: NCCL communicators over
// NVLink / NVSwitch, one per GPU (one process or host thread per GPU).
//
// The reference trains on one CPU thread, so this has no counterpart there;
// it is what a data-parallel host wraps around Adam.step
// (src/L2/autograd.js:214-244): the flat gradient buffer, averaged over the
// ranks bucket by bucket while the backward continues, then the identical
// Adam step on every rank (or, for ZeRO-1, a reduce-scatter, an Adam step on
// this rank's slices and an all-gather of the parameters).
//
// Design:
//   - NCCL is loaded at run time (dlopen "libnccl.so.2", or the path in
//     FORGECU_NCCL_LIB), so the library has no link-time NCCL dependency and
//     shares the NCCL a host process has already loaded.
//   - Communicators are non-blocking (ncclConfig_t.blocking = 0).  Every
//     NCCL call that answers ncclInProgress is polled with
//     ncclCommGetAsyncError against a deadline; a communicator that misses
//     its deadline (a rank that never joined, a peer that died) is aborted
//     (ncclCommAbort, which also ends its kernels in flight) and the call
//     returns FCU_ERR_TIMEOUT.  Nothing in this file waits without a bound.
//   - Each communicator owns a CUDA stream.  A collective first makes that
//     stream wait for the work already queued on the context's stream (an
//     event), so it starts when the bucket's gradients are final and runs
//     beside whatever the context launches next; fcu_comm_join makes the
//     context's stream wait for every collective launched so far.  This
//     fork / join is legal inside CUDA stream capture, so a captured
//     training step replays its collectives.
#include <dlfcn.h>
#include <nccl.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include <mutex>
#include <vector>

#include "common.cuh"

namespace {

struct NcclApi {
  void *handle = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*AllReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*ReduceScatter)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t,
                                ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  const char *(*GetErrorString)(ncclResult_t) = nullptr;
  ncclResult_t (*GetVersion)(int *) = nullptr;
};

NcclApi g_nccl;
std::mutex g_nccl_mu;

template <typename F>
bool bind(void *h, const char *name, F &fn) {
  fn = reinterpret_cast<F>(dlsym(h, name));
  return fn != nullptr;
}

int nccl_api(const NcclApi **out) {
  std::lock_guard<std::mutex> lock(g_nccl_mu);
  if (!g_nccl.handle) {
    const char *env = getenv("FORGECU_NCCL_LIB");
    const char *path = env && env[0] ? env : "libnccl.so.2";
    void *h = dlopen(path, RTLD_NOW | RTLD_LOCAL);
    if (!h) {
      fcu::set_error("cannot load NCCL (%s): %s", path, dlerror());
      return FCU_ERR_UNSUPPORTED;
    }
    NcclApi a;
    a.handle = h;
    bool ok = bind(h, "ncclGetUniqueId", a.GetUniqueId) &&
              bind(h, "ncclCommInitRankConfig", a.CommInitRankConfig) &&
              bind(h, "ncclCommGetAsyncError", a.CommGetAsyncError) &&
              bind(h, "ncclCommAbort", a.CommAbort) && bind(h, "ncclCommFinalize", a.CommFinalize) &&
              bind(h, "ncclCommDestroy", a.CommDestroy) && bind(h, "ncclAllReduce", a.AllReduce) &&
              bind(h, "ncclReduceScatter", a.ReduceScatter) && bind(h, "ncclAllGather", a.AllGather) &&
              bind(h, "ncclGetErrorString", a.GetErrorString) && bind(h, "ncclGetVersion", a.GetVersion);
    if (!ok) {
      fcu::set_error("NCCL at %s lacks a required entry point (needs NCCL >= 2.18)", path);
      dlclose(h);
      return FCU_ERR_UNSUPPORTED;
    }
    g_nccl = a;
  }
  *out = &g_nccl;
  return FCU_OK;
}

double now_s() {
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

void pause_briefly() {
  timespec ts = {0, 20000};   // 20 us between polls
  nanosleep(&ts, nullptr);
}

}  // namespace

// One profiled collective (or join): when its inputs were ready on the
// context's stream, when it started and ended on the communicator's stream.
struct CommProf {
  cudaEvent_t ready = nullptr, start = nullptr, end = nullptr;
  int kind = 0;
  int64_t bytes = 0;
};

struct fcu_comm {
  const NcclApi *api = nullptr;
  ncclComm_t nc = nullptr;
  int device = -1, nranks = 0, rank = 0;   // device -1: set by the first collective
  double timeout_s = 0;
  bool aborted = false;
  int pending = 0;   // collectives launched since the last fcu_comm_poll
  cudaStream_t stream = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr, done = nullptr;
  std::vector<CommProf> prof;   // fcu_comm_profile: timing events, prof_used of them recorded
  int prof_used = 0;
};

namespace {

int do_abort(fcu_comm *c) {
  if (c->aborted) return FCU_OK;
  c->aborted = true;
  if (c->nc) {
    ncclResult_t r = c->api->CommAbort(c->nc);
    c->nc = nullptr;
    if (r != ncclSuccess) {
      fcu::set_error("ncclCommAbort: %s", c->api->GetErrorString(r));
      return FCU_ERR_NCCL;
    }
  }
  return FCU_OK;
}

// Waits (bounded) until the communicator has no NCCL operation in progress.
// On a deadline miss or an asynchronous error the communicator is aborted.
int wait_ready(fcu_comm *c, double timeout_s, const char *what) {
  const double t0 = now_s();
  while (true) {
    ncclResult_t st = ncclInProgress;
    ncclResult_t r = c->api->CommGetAsyncError(c->nc, &st);
    if (r != ncclSuccess) st = r;
    if (st == ncclSuccess) return FCU_OK;
    if (st != ncclInProgress) {
      const char *msg = c->api->GetErrorString(st);
      do_abort(c);
      fcu::set_error("%s: NCCL error %d (%s); communicator aborted", what, (int)st, msg);
      return FCU_ERR_NCCL;
    }
    if (now_s() - t0 > timeout_s) {
      do_abort(c);
      fcu::set_error("%s: not complete within %.3g s (a rank missing or stalled); communicator aborted",
                     what, timeout_s);
      return FCU_ERR_TIMEOUT;
    }
    pause_briefly();
  }
}

// Checks the result of an enqueuing NCCL call (non-blocking: ncclInProgress
// means "still being enqueued"; it must finish before the next NCCL call).
int nccl_result(fcu_comm *c, ncclResult_t r, const char *what) {
  if (r == ncclSuccess) return FCU_OK;
  if (r == ncclInProgress) return wait_ready(c, c->timeout_s, what);
  const char *msg = c->api->GetErrorString(r);
  do_abort(c);
  fcu::set_error("%s: NCCL error %d (%s); communicator aborted", what, (int)r, msg);
  return FCU_ERR_NCCL;
}

int comm_usable(fcu_comm *c, const char *what) {
  FCU_REQUIRE(c != nullptr, "%s: null fcu_comm", what);
  if (c->aborted) {
    fcu::set_error("%s: the communicator was aborted", what);
    return FCU_ERR_NCCL;
  }
  return FCU_OK;
}

// The communicator's stream and events, created on first use on its device.
int comm_streams(fcu_comm *c) {
  if (c->stream) return FCU_OK;
  FCU_CHECK_CUDA(cudaSetDevice(c->device));
  FCU_CHECK_CUDA(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
  FCU_CHECK_CUDA(cudaEventCreateWithFlags(&c->fork, cudaEventDisableTiming));
  FCU_CHECK_CUDA(cudaEventCreateWithFlags(&c->join, cudaEventDisableTiming));
  FCU_CHECK_CUDA(cudaEventCreateWithFlags(&c->done, cudaEventDisableTiming));
  return FCU_OK;
}

// The communicator's stream waits for everything queued on ctx's stream.
int fork_from(fcu_ctx *ctx, fcu_comm *c, const char *what) {
  int rc = comm_usable(c, what);
  if (rc) return rc;
  FCU_REQUIRE(ctx != nullptr, "%s: null fcu_ctx", what);
  if (c->device < 0) c->device = ctx->device;   // created on "the current device"
  FCU_REQUIRE(ctx->device == c->device, "%s: context on device %d, communicator on device %d", what,
              ctx->device, c->device);
  rc = comm_streams(c);
  if (rc) return rc;
  FCU_CHECK_CUDA(cudaEventRecord(c->fork, ctx->stream));
  FCU_CHECK_CUDA(cudaStreamWaitEvent(c->stream, c->fork, 0));
  return FCU_OK;
}

// Profiling (fcu_comm_profile): timing events around a collective, outside
// stream capture only.  prof_begin runs after fork_from, prof_end after the
// NCCL call; a record is kept only if both were placed.
bool prof_on(fcu_comm *c, fcu_ctx *ctx) {
  if (c->prof_used >= (int)c->prof.size()) return false;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(ctx->stream, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) return false;
  return true;
}

int prof_begin(fcu_comm *c, fcu_ctx *ctx, int kind, int64_t bytes, bool *on) {
  *on = prof_on(c, ctx);
  if (!*on) return FCU_OK;
  CommProf &r = c->prof[c->prof_used];
  r.kind = kind;
  r.bytes = bytes;
  FCU_CHECK_CUDA(cudaEventRecord(r.ready, ctx->stream));
  FCU_CHECK_CUDA(cudaEventRecord(r.start, c->stream));
  return FCU_OK;
}

int prof_end(fcu_comm *c, bool on) {
  if (!on) return FCU_OK;
  FCU_CHECK_CUDA(cudaEventRecord(c->prof[c->prof_used].end, c->stream));
  c->prof_used++;
  return FCU_OK;
}

}  // namespace

extern "C" {

int fcu_comm_unique_id(void *id_out) {
  FCU_REQUIRE(id_out != nullptr, "fcu_comm_unique_id: null output");
  static_assert(sizeof(ncclUniqueId) == FCU_COMM_ID_BYTES, "NCCL unique id size");
  const NcclApi *api = nullptr;
  int rc = nccl_api(&api);
  if (rc) return rc;
  ncclUniqueId id;
  ncclResult_t r = api->GetUniqueId(&id);
  if (r != ncclSuccess) {
    fcu::set_error("ncclGetUniqueId: %s", api->GetErrorString(r));
    return FCU_ERR_NCCL;
  }
  memcpy(id_out, &id, sizeof id);
  return FCU_OK;
}

int fcu_comm_init(int device, const void *id, int nranks, int rank, double timeout_s, fcu_comm **out) {
  FCU_REQUIRE(out != nullptr && id != nullptr, "fcu_comm_init: null argument");
  FCU_REQUIRE(nranks >= 1 && rank >= 0 && rank < nranks, "fcu_comm_init: rank %d of %d", rank, nranks);
  FCU_REQUIRE(timeout_s > 0 && timeout_s <= 86400, "fcu_comm_init: timeout %.3g s out of range",
              timeout_s);
  *out = nullptr;
  const NcclApi *api = nullptr;
  int rc = nccl_api(&api);
  if (rc) return rc;
  // NCCL binds the communicator to the calling thread's current device.
  if (device >= 0) FCU_CHECK_CUDA(cudaSetDevice(device));
  fcu_comm *c = new fcu_comm;
  c->api = api;
  c->device = device;
  c->nranks = nranks;
  c->rank = rank;
  c->timeout_s = timeout_s;
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof uid);
  ncclResult_t r = api->CommInitRankConfig(&c->nc, nranks, uid, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    fcu::set_error("ncclCommInitRankConfig: %s", api->GetErrorString(r));
    if (c->nc) api->CommAbort(c->nc);
    delete c;
    return FCU_ERR_NCCL;
  }
  rc = wait_ready(c, timeout_s, "fcu_comm_init");
  if (rc) {
    delete c;   // wait_ready aborted it
    return rc;
  }
  *out = c;
  return FCU_OK;
}

int fcu_comm_abort(fcu_comm *comm) {
  FCU_REQUIRE(comm != nullptr, "fcu_comm_abort: null fcu_comm");
  return do_abort(comm);
}

int fcu_comm_destroy(fcu_comm *comm) {
  if (!comm) return FCU_OK;
  int rc = FCU_OK;
  if (!comm->aborted && comm->nc) {
    rc = nccl_result(comm, comm->api->CommFinalize(comm->nc), "ncclCommFinalize");
    if (rc == FCU_OK) {
      ncclResult_t r = comm->api->CommDestroy(comm->nc);
      if (r != ncclSuccess) {
        fcu::set_error("ncclCommDestroy: %s", comm->api->GetErrorString(r));
        rc = FCU_ERR_NCCL;
      }
      comm->nc = nullptr;
    }
  }
  if (comm->stream) {
    cudaSetDevice(comm->device);
    for (CommProf &r : comm->prof) {
      cudaEventDestroy(r.ready);
      cudaEventDestroy(r.start);
      cudaEventDestroy(r.end);
    }
    cudaEventDestroy(comm->fork);
    cudaEventDestroy(comm->join);
    cudaEventDestroy(comm->done);
    cudaStreamDestroy(comm->stream);
  }
  delete comm;
  return rc;
}

int fcu_comm_info(const fcu_comm *comm, int *nranks, int *rank, int *device) {
  FCU_REQUIRE(comm != nullptr, "fcu_comm_info: null fcu_comm");
  if (nranks) *nranks = comm->nranks;
  if (rank) *rank = comm->rank;
  if (device) *device = comm->device;
  return comm->aborted ? FCU_ERR_NCCL : FCU_OK;
}

int fcu_allreduce_grads(fcu_ctx *ctx, fcu_comm *comm, float *buf, int64_t n) {
  FCU_REQUIRE(n >= 0 && (n == 0 || buf), "fcu_allreduce_grads: bad buffer");
  int rc = fork_from(ctx, comm, "fcu_allreduce_grads");
  if (rc || n == 0) return rc;
  bool on = false;
  if ((rc = prof_begin(comm, ctx, 0, 4 * n, &on))) return rc;
  rc = nccl_result(comm, comm->api->AllReduce(buf, buf, (size_t)n, ncclFloat32, ncclAvg, comm->nc,
                                              comm->stream),
                   "fcu_allreduce_grads");
  if (rc == FCU_OK) rc = prof_end(comm, on);
  if (rc == FCU_OK) comm->pending++;
  return rc;
}

int fcu_reduce_scatter_grads(fcu_ctx *ctx, fcu_comm *comm, float *buf, int64_t n) {
  FCU_REQUIRE(n >= 0 && (n == 0 || buf), "fcu_reduce_scatter_grads: bad buffer");
  int rc = fork_from(ctx, comm, "fcu_reduce_scatter_grads");
  if (rc || n == 0) return rc;
  FCU_REQUIRE(n % comm->nranks == 0, "fcu_reduce_scatter_grads: %lld values do not split over %d ranks",
              (long long)n, comm->nranks);
  bool on = false;
  if ((rc = prof_begin(comm, ctx, 1, 4 * n, &on))) return rc;
  const int64_t per = n / comm->nranks;
  rc = nccl_result(comm, comm->api->ReduceScatter(buf, buf + (int64_t)comm->rank * per, (size_t)per,
                                                  ncclFloat32, ncclAvg, comm->nc, comm->stream),
                   "fcu_reduce_scatter_grads");
  if (rc == FCU_OK) rc = prof_end(comm, on);
  if (rc == FCU_OK) comm->pending++;
  return rc;
}

int fcu_allgather_params(fcu_ctx *ctx, fcu_comm *comm, void *buf, int64_t n, int elem_bytes) {
  FCU_REQUIRE(n >= 0 && (n == 0 || buf), "fcu_allgather_params: bad buffer");
  FCU_REQUIRE(elem_bytes == 4 || elem_bytes == 2, "fcu_allgather_params: elem_bytes %d (4: fp32, 2: bf16)",
              elem_bytes);
  int rc = fork_from(ctx, comm, "fcu_allgather_params");
  if (rc || n == 0) return rc;
  FCU_REQUIRE(n % comm->nranks == 0, "fcu_allgather_params: %lld values do not split over %d ranks",
              (long long)n, comm->nranks);
  bool on = false;
  if ((rc = prof_begin(comm, ctx, 2, (int64_t)elem_bytes * n, &on))) return rc;
  const int64_t per = n / comm->nranks;
  char *base = (char *)buf;
  rc = nccl_result(comm, comm->api->AllGather(base + (int64_t)comm->rank * per * elem_bytes, buf,
                                              (size_t)per, elem_bytes == 4 ? ncclFloat32 : ncclBfloat16,
                                              comm->nc, comm->stream),
                   "fcu_allgather_params");
  if (rc == FCU_OK) rc = prof_end(comm, on);
  if (rc == FCU_OK) comm->pending++;
  return rc;
}

int fcu_allreduce_sum_f64(fcu_ctx *ctx, fcu_comm *comm, double *buf, int64_t n) {
  FCU_REQUIRE(n >= 0 && (n == 0 || buf), "fcu_allreduce_sum_f64: bad buffer");
  int rc = fork_from(ctx, comm, "fcu_allreduce_sum_f64");
  if (rc || n == 0) return rc;
  bool on = false;
  if ((rc = prof_begin(comm, ctx, 3, 8 * n, &on))) return rc;
  rc = nccl_result(comm, comm->api->AllReduce(buf, buf, (size_t)n, ncclFloat64, ncclSum, comm->nc,
                                              comm->stream),
                   "fcu_allreduce_sum_f64");
  if (rc == FCU_OK) rc = prof_end(comm, on);
  if (rc == FCU_OK) comm->pending++;
  return rc;
}

int fcu_comm_join(fcu_ctx *ctx, fcu_comm *comm) {
  int rc = comm_usable(comm, "fcu_comm_join");
  if (rc) return rc;
  FCU_REQUIRE(ctx != nullptr, "fcu_comm_join: null fcu_ctx");
  if (!comm->stream) return FCU_OK;   // nothing launched yet
  FCU_REQUIRE(ctx->device == comm->device, "fcu_comm_join: context on device %d, communicator on %d",
              ctx->device, comm->device);
  const bool on = prof_on(comm, ctx);
  if (on) {
    CommProf &r = comm->prof[comm->prof_used];
    r.kind = 4;
    r.bytes = 0;
    FCU_CHECK_CUDA(cudaEventRecord(r.ready, ctx->stream));
  }
  FCU_CHECK_CUDA(cudaEventRecord(comm->join, comm->stream));
  FCU_CHECK_CUDA(cudaStreamWaitEvent(ctx->stream, comm->join, 0));
  if (on) {
    CommProf &r = comm->prof[comm->prof_used++];
    FCU_CHECK_CUDA(cudaEventRecord(r.start, ctx->stream));
    FCU_CHECK_CUDA(cudaEventRecord(r.end, ctx->stream));
  }
  return FCU_OK;
}

int fcu_comm_profile(fcu_comm *comm, int max_records) {
  int rc = comm_usable(comm, "fcu_comm_profile");
  if (rc) return rc;
  FCU_REQUIRE(max_records >= 0 && max_records <= 65536, "fcu_comm_profile: %d records", max_records);
  FCU_REQUIRE(comm->device >= 0, "fcu_comm_profile: the communicator's device is not known yet");
  if ((rc = comm_streams(comm))) return rc;
  FCU_CHECK_CUDA(cudaSetDevice(comm->device));
  FCU_CHECK_CUDA(cudaStreamSynchronize(comm->stream));   // no recorded event is still pending
  while ((int)comm->prof.size() < max_records) {
    CommProf r;
    FCU_CHECK_CUDA(cudaEventCreate(&r.ready));
    FCU_CHECK_CUDA(cudaEventCreate(&r.start));
    FCU_CHECK_CUDA(cudaEventCreate(&r.end));
    comm->prof.push_back(r);
  }
  while ((int)comm->prof.size() > max_records) {
    CommProf &r = comm->prof.back();
    cudaEventDestroy(r.ready);
    cudaEventDestroy(r.start);
    cudaEventDestroy(r.end);
    comm->prof.pop_back();
  }
  comm->prof_used = 0;
  return FCU_OK;
}

int fcu_comm_profile_read(fcu_comm *comm, double *out, int max_records, int *n_out) {
  FCU_REQUIRE(comm != nullptr && n_out != nullptr && (out != nullptr || max_records == 0),
              "fcu_comm_profile_read: null argument");
  *n_out = 0;
  if (comm->prof_used == 0) return FCU_OK;
  FCU_CHECK_CUDA(cudaSetDevice(comm->device));
  for (int i = 0; i < comm->prof_used; i++) FCU_CHECK_CUDA(cudaEventSynchronize(comm->prof[i].end));
  const int n = comm->prof_used < max_records ? comm->prof_used : max_records;
  const cudaEvent_t t0 = comm->prof[0].ready;
  for (int i = 0; i < n; i++) {
    const CommProf &r = comm->prof[i];
    float a = 0, b = 0, e = 0;
    FCU_CHECK_CUDA(cudaEventElapsedTime(&a, t0, r.ready));
    FCU_CHECK_CUDA(cudaEventElapsedTime(&b, t0, r.start));
    FCU_CHECK_CUDA(cudaEventElapsedTime(&e, t0, r.end));
    double *o = out + 5 * (int64_t)i;
    o[0] = r.kind;
    o[1] = (double)r.bytes;
    o[2] = a;
    o[3] = b;
    o[4] = e;
  }
  *n_out = n;
  return FCU_OK;
}

int fcu_comm_poll(fcu_comm *comm, double timeout_s) {
  int rc = comm_usable(comm, "fcu_comm_poll");
  if (rc) return rc;
  FCU_REQUIRE(timeout_s >= 0 && timeout_s <= 86400, "fcu_comm_poll: timeout %.3g s out of range",
              timeout_s);
  // an error another thread or a peer already raised
  ncclResult_t st = ncclSuccess;
  ncclResult_t r = comm->api->CommGetAsyncError(comm->nc, &st);
  if (r != ncclSuccess) st = r;
  if (st != ncclSuccess && st != ncclInProgress) {
    const char *msg = comm->api->GetErrorString(st);
    do_abort(comm);
    fcu::set_error("fcu_comm_poll: NCCL error %d (%s); communicator aborted", (int)st, msg);
    return FCU_ERR_NCCL;
  }
  if (!comm->stream || comm->pending == 0) return FCU_OK;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  FCU_CHECK_CUDA(cudaStreamIsCapturing(comm->stream, &cap));
  FCU_REQUIRE(cap == cudaStreamCaptureStatusNone, "fcu_comm_poll: not allowed during stream capture");
  FCU_CHECK_CUDA(cudaEventRecord(comm->done, comm->stream));
  const double t0 = now_s();
  while (true) {
    cudaError_t e = cudaEventQuery(comm->done);
    if (e == cudaSuccess) break;
    if (e != cudaErrorNotReady) return fcu::cuda_fail(e, "cudaEventQuery", __FILE__, __LINE__);
    st = ncclSuccess;
    r = comm->api->CommGetAsyncError(comm->nc, &st);
    if (r != ncclSuccess) st = r;
    if (st != ncclSuccess && st != ncclInProgress) {
      const char *msg = comm->api->GetErrorString(st);
      do_abort(comm);
      fcu::set_error("fcu_comm_poll: NCCL error %d (%s); communicator aborted", (int)st, msg);
      return FCU_ERR_NCCL;
    }
    if (now_s() - t0 > timeout_s) {
      do_abort(comm);
      fcu::set_error("fcu_comm_poll: collectives not finished within %.3g s; communicator aborted",
                     timeout_s);
      return FCU_ERR_TIMEOUT;
    }
    pause_briefly();
  }
  comm->pending = 0;
  return FCU_OK;
}

}  // extern "C"
