/* A stand-in for libnccl.so.2 used only by tests/test_comm_cpu.py: it lets the
 * CPU tests drive libforgecu's communicator code (fcu_comm_*) through every
 * failure path without GPUs or peers.  Behaviour is set with
 * fake_nccl_set_mode():
 *   0  healthy: init and finalize report ncclInProgress for a few polls,
 *      then success;
 *   1  a rank never joins: init stays ncclInProgress forever;
 *   2  init fails at once (ncclSystemError);
 *   3  a peer failed after init: ncclCommGetAsyncError reports
 *      ncclRemoteError.
 * Counters record the calls the tests check (aborts, destroys, ...). */
#include <nccl.h>
#include <string.h>

static int g_mode = 0, g_polls = 0;
static int g_aborts = 0, g_destroys = 0, g_finalizes = 0, g_inits = 0;
static int g_comm_token;

void fake_nccl_set_mode(int m) { g_mode = m; g_polls = 0; }
int fake_nccl_aborts(void) { return g_aborts; }
int fake_nccl_destroys(void) { return g_destroys; }
int fake_nccl_finalizes(void) { return g_finalizes; }
int fake_nccl_inits(void) { return g_inits; }

ncclResult_t ncclGetUniqueId(ncclUniqueId *id) {
  for (int i = 0; i < NCCL_UNIQUE_ID_BYTES; i++) id->internal[i] = (char)(i * 7 + 1);
  return ncclSuccess;
}

ncclResult_t ncclCommInitRankConfig(ncclComm_t *comm, int nranks, ncclUniqueId id, int rank,
                                    ncclConfig_t *config) {
  (void)nranks; (void)rank;
  g_inits++;
  if (config->blocking != 0) return ncclInvalidArgument;   /* the library must ask for non-blocking */
  if (id.internal[1] != 8) return ncclInvalidArgument;      /* the id from ncclGetUniqueId */
  if (g_mode == 2) return ncclSystemError;
  *comm = (ncclComm_t)&g_comm_token;
  g_polls = 0;
  return ncclInProgress;
}

ncclResult_t ncclCommGetAsyncError(ncclComm_t comm, ncclResult_t *st) {
  (void)comm;
  if (g_mode == 1) { *st = ncclInProgress; return ncclSuccess; }
  if (g_mode == 3) { *st = ncclRemoteError; return ncclSuccess; }
  *st = ++g_polls < 3 ? ncclInProgress : ncclSuccess;
  return ncclSuccess;
}

ncclResult_t ncclCommAbort(ncclComm_t comm) { (void)comm; g_aborts++; return ncclSuccess; }
ncclResult_t ncclCommFinalize(ncclComm_t comm) { (void)comm; g_finalizes++; g_polls = 0; return ncclInProgress; }
ncclResult_t ncclCommDestroy(ncclComm_t comm) { (void)comm; g_destroys++; return ncclSuccess; }

ncclResult_t ncclAllReduce(const void *s, void *r, size_t n, ncclDataType_t t, ncclRedOp_t op,
                           ncclComm_t c, cudaStream_t st) {
  (void)s; (void)r; (void)n; (void)t; (void)op; (void)c; (void)st;
  return ncclInternalError;
}
ncclResult_t ncclReduceScatter(const void *s, void *r, size_t n, ncclDataType_t t, ncclRedOp_t op,
                               ncclComm_t c, cudaStream_t st) {
  (void)s; (void)r; (void)n; (void)t; (void)op; (void)c; (void)st;
  return ncclInternalError;
}
ncclResult_t ncclAllGather(const void *s, void *r, size_t n, ncclDataType_t t, ncclComm_t c,
                           cudaStream_t st) {
  (void)s; (void)r; (void)n; (void)t; (void)c; (void)st;
  return ncclInternalError;
}

const char *ncclGetErrorString(ncclResult_t r) {
  switch (r) {
    case ncclSuccess: return "fake: success";
    case ncclInProgress: return "fake: in progress";
    case ncclRemoteError: return "fake: remote error";
    case ncclSystemError: return "fake: system error";
    default: return "fake: other error";
  }
}

ncclResult_t ncclGetVersion(int *v) { *v = 22703; return ncclSuccess; }
