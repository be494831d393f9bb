// Data parallelism over NCCL (NVLink 5 / NVSwitch), one process per GPU.
//
// The reference is single-device (no collective call sites anywhere); this is
// the exchange step of the data-parallel training step: gradients of every
// parameter are averaged across ranks in buckets on a dedicated communication
// stream, ordered after the backward kernels that finished them by events, so
// the reduction of late layers overlaps the backward of earlier ones.
//
// Every wait is bounded: communicator set-up polls ncclCommGetAsyncError with a
// deadline and aborts the communicator when it expires.
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <thread>

#include "common.h"

namespace {

struct DpState {
  ncclComm_t comm = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};

DpState *state(tx_ctx *ctx) { return reinterpret_cast<DpState *>(ctx->nccl); }

int nccl_fail(tx_ctx *ctx, ncclResult_t r, const char *what) {
  char buf[256];
  snprintf(buf, sizeof buf, "NCCL error %d (%s) in %s", (int)r, ncclGetErrorString(r), what);
  return tx_fail(ctx, TX_ERR_NCCL, buf);
}

// Wait for a non-blocking NCCL operation to leave ncclInProgress.
int nccl_wait(tx_ctx *ctx, ncclComm_t comm, uint64_t timeout_ms, const char *what) {
  auto start = std::chrono::steady_clock::now();
  while (true) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t r = ncclCommGetAsyncError(comm, &st);
    if (r != ncclSuccess) return nccl_fail(ctx, r, what);
    if (st == ncclSuccess) return TX_OK;
    if (st != ncclInProgress) return nccl_fail(ctx, st, what);
    auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                  std::chrono::steady_clock::now() - start)
                  .count();
    if (timeout_ms && (uint64_t)ms > timeout_ms) {
      ncclCommAbort(comm);
      return tx_fail(ctx, TX_ERR_TIMEOUT, std::string(what) + " timed out; communicator aborted");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
}

}  // namespace

extern "C" int tx_dp_unique_id(uint8_t *out128) {
  if (!out128) return TX_ERR_INVALID;
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId size");
  ncclUniqueId id;
  if (ncclGetUniqueId(&id) != ncclSuccess) return TX_ERR_NCCL;
  memcpy(out128, &id, 128);
  return TX_OK;
}

extern "C" int tx_dp_init(tx_ctx *ctx, int world, int rank, const uint8_t *id128, uint64_t timeout_ms) {
  if (!ctx || !id128 || world < 1 || rank < 0 || rank >= world) return TX_ERR_INVALID;
  if (ctx->nccl) return tx_fail(ctx, TX_ERR_INVALID, "data parallelism already initialised");
  TX_CUDA(ctx, cudaSetDevice(ctx->device));
  ncclUniqueId id;
  memcpy(&id, id128, 128);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  DpState *s = new DpState();
  ncclResult_t r = ncclCommInitRankConfig(&s->comm, world, id, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    if (s->comm) ncclCommAbort(s->comm);
    delete s;
    return nccl_fail(ctx, r, "ncclCommInitRankConfig");
  }
  int rc = nccl_wait(ctx, s->comm, timeout_ms, "communicator initialisation");
  if (rc != TX_OK) {
    // nccl_wait aborts the communicator itself when its deadline expires
    if (rc != TX_ERR_TIMEOUT) ncclCommAbort(s->comm);
    delete s;
    return rc;
  }
  cudaError_t e = cudaEventCreateWithFlags(&s->fork, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s->join, cudaEventDisableTiming);
  if (e != cudaSuccess) {
    if (s->fork) cudaEventDestroy(s->fork);
    ncclCommAbort(s->comm);
    delete s;
    return tx_cuda_fail(ctx, e, "tx_dp_init: event creation");
  }
  ctx->nccl = s;
  ctx->world = world;
  ctx->rank = rank;
  ctx->dp_timeout_ms = timeout_ms;
  return TX_OK;
}

int tx_dp_shutdown(tx_ctx *ctx) {
  DpState *s = state(ctx);
  if (!s) return TX_OK;
  if (s->comm) {
    ncclCommFinalize(s->comm);
    nccl_wait(ctx, s->comm, ctx->dp_timeout_ms, "communicator finalisation");
    ncclCommDestroy(s->comm);
  }
  if (s->fork) cudaEventDestroy(s->fork);
  if (s->join) cudaEventDestroy(s->join);
  delete s;
  ctx->nccl = nullptr;
  ctx->world = 1;
  ctx->rank = 0;
  return TX_OK;
}

extern "C" int tx_dp_destroy(tx_ctx *ctx) {
  if (!ctx) return TX_ERR_INVALID;
  cudaStreamSynchronize(ctx->stream);
  cudaStreamSynchronize(ctx->comm);
  return tx_dp_shutdown(ctx);
}

int dp_event_fork(tx_ctx *ctx) {
  DpState *s = state(ctx);
  if (!s) return tx_fail(ctx, TX_ERR_INVALID, "data parallelism is not initialised");
  TX_CUDA(ctx, cudaEventRecord(s->fork, ctx->stream));
  TX_CUDA(ctx, cudaStreamWaitEvent(ctx->comm, s->fork, 0));
  return TX_OK;
}

int dp_event_join(tx_ctx *ctx) {
  DpState *s = state(ctx);
  if (!s) return TX_OK;
  TX_CUDA(ctx, cudaEventRecord(s->join, ctx->comm));
  TX_CUDA(ctx, cudaStreamWaitEvent(ctx->stream, s->join, 0));
  return TX_OK;
}

int dp_allreduce_range(tx_ctx *ctx, float *buf, int64_t n) {
  DpState *s = state(ctx);
  if (!s) return tx_fail(ctx, TX_ERR_INVALID, "data parallelism is not initialised");
  if (n <= 0) return TX_OK;
  ncclResult_t r = ncclAllReduce(buf, buf, (size_t)n, ncclFloat32, ncclAvg, s->comm, ctx->comm);
  if (r != ncclSuccess && r != ncclInProgress) return nccl_fail(ctx, r, "ncclAllReduce");
  // a non-blocking communicator takes its next call only once this one has
  // left ncclInProgress (the enqueue, not the reduction itself)
  if (r == ncclInProgress) return nccl_wait(ctx, s->comm, ctx->dp_timeout_ms, "ncclAllReduce");
  return TX_OK;
}

extern "C" int tx_dp_allreduce(tx_ctx *ctx, float *buf, int64_t n, int average) {
  if (!ctx) return TX_ERR_INVALID;
  DpState *s = state(ctx);
  if (!s) return tx_fail(ctx, TX_ERR_INVALID, "data parallelism is not initialised");
  TX_TRY(dp_event_fork(ctx));
  ncclResult_t r = ncclAllReduce(buf, buf, (size_t)n, ncclFloat32, average ? ncclAvg : ncclSum,
                                 s->comm, ctx->comm);
  if (r != ncclSuccess && r != ncclInProgress) return nccl_fail(ctx, r, "ncclAllReduce");
  if (r == ncclInProgress) TX_TRY(nccl_wait(ctx, s->comm, ctx->dp_timeout_ms, "ncclAllReduce"));
  return dp_event_join(ctx);
}
