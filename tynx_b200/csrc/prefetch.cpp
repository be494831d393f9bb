// Upload ring for input batches: host-to-device copies run on a copy stream
// beside the context's compute stream, so the next batches upload while the
// current step runs.
//
// The ring owns `depth` device buffers (allocated once, outside the context's
// stream-ordered pool: a block recycled by that pool may still be read by
// compute work in flight, which a copy on another stream would not wait for).
// put n queues batch n's copy into buffer n % depth; get hands out the oldest
// queued batch, recording a mark on the compute stream (everything enqueued
// before this get has been issued, which includes the readers of the batch
// handed out by the previous get) and ordering the compute stream after that
// batch's copy.  Batch n's copy waits for the mark of get n - depth + 1, after
// which nothing reads the batch that buffer held before.  So a batch handed
// out by get g is valid for work issued before get g + 1, while batches
// g + 1 .. g + depth - 1 upload into the other buffers.
#include <vector>

#include "common.h"

struct tx_prefetch {
  tx_ctx *ctx = nullptr;
  size_t bytes = 0;
  int depth = 0;
  uint64_t puts = 0, gets = 0;
  cudaStream_t copy = nullptr;
  std::vector<void *> bufs;
  std::vector<cudaEvent_t> marks;   // compute-stream mark of get g, at g % depth
  std::vector<cudaEvent_t> copied;  // completion of put n, at n % depth
};

extern "C" int tx_prefetch_destroy(tx_prefetch *p) {
  if (!p) return TX_OK;
  if (p->copy) cudaStreamSynchronize(p->copy);
  if (p->ctx) cudaStreamSynchronize(p->ctx->stream);
  for (void *b : p->bufs)
    if (b) cudaFree(b);
  for (cudaEvent_t e : p->marks)
    if (e) cudaEventDestroy(e);
  for (cudaEvent_t e : p->copied)
    if (e) cudaEventDestroy(e);
  if (p->copy) cudaStreamDestroy(p->copy);
  delete p;
  return TX_OK;
}

extern "C" int tx_prefetch_create(tx_ctx *ctx, size_t bytes, int depth, tx_prefetch **out) {
  if (!ctx || !out || depth < 2 || depth > 16 || bytes == 0) return TX_ERR_INVALID;
  *out = nullptr;
  if (ctx->capturing) return tx_fail(ctx, TX_ERR_CAPTURE, "tx_prefetch_create during a capture");
  tx_prefetch *p = new tx_prefetch;
  p->ctx = ctx;
  p->bytes = bytes;
  p->depth = depth;
  p->bufs.assign(depth, nullptr);
  p->marks.assign(depth, nullptr);
  p->copied.assign(depth, nullptr);
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e == cudaSuccess && device != ctx->device) e = cudaSetDevice(ctx->device);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&p->copy, cudaStreamNonBlocking);
  for (int i = 0; i < depth && e == cudaSuccess; ++i) {
    e = cudaMalloc(&p->bufs[i], bytes);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->marks[i], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->copied[i], cudaEventDisableTiming);
  }
  if (device != ctx->device) cudaSetDevice(device);
  if (e != cudaSuccess) {
    tx_prefetch_destroy(p);
    return tx_cuda_fail(ctx, e, "tx_prefetch_create");
  }
  *out = p;
  return TX_OK;
}

extern "C" int tx_prefetch_put(tx_prefetch *p, const void *h_src, size_t bytes) {
  if (!p || !h_src) return TX_ERR_INVALID;
  tx_ctx *ctx = p->ctx;
  if (bytes > p->bytes) return tx_fail(ctx, TX_ERR_SHAPE, "tx_prefetch_put: batch larger than the ring's buffers");
  if (ctx->capturing) return tx_fail(ctx, TX_ERR_CAPTURE, "tx_prefetch_put during a capture");
  const uint64_t n = p->puts;
  if (n >= p->gets + (uint64_t)p->depth)
    return tx_fail(ctx, TX_ERR_INVALID, "tx_prefetch_put: every buffer holds a batch not yet taken by tx_prefetch_get");
  if (n >= (uint64_t)p->depth) {
    // buffer n % depth held batch n - depth, read by work enqueued before get n - depth + 1
    const uint64_t g = n - p->depth + 1;
    if (g >= p->gets)
      return tx_fail(ctx, TX_ERR_INVALID, "tx_prefetch_put: the buffer's previous batch has not been released by a later get");
    TX_CUDA(ctx, cudaStreamWaitEvent(p->copy, p->marks[g % p->depth], 0));
  }
  const int k = (int)(n % (uint64_t)p->depth);
  if (bytes) TX_CUDA(ctx, cudaMemcpyAsync(p->bufs[k], h_src, bytes, cudaMemcpyHostToDevice, p->copy));
  TX_CUDA(ctx, cudaEventRecord(p->copied[k], p->copy));
  p->puts = n + 1;
  return TX_OK;
}

extern "C" int tx_prefetch_get(tx_prefetch *p, void **d_out) {
  if (!p || !d_out) return TX_ERR_INVALID;
  tx_ctx *ctx = p->ctx;
  if (ctx->capturing) return tx_fail(ctx, TX_ERR_CAPTURE, "tx_prefetch_get during a capture");
  const uint64_t g = p->gets;
  if (g >= p->puts) return tx_fail(ctx, TX_ERR_INVALID, "tx_prefetch_get: no batch has been put");
  const int k = (int)(g % (uint64_t)p->depth);
  TX_CUDA(ctx, cudaEventRecord(p->marks[k], ctx->stream));
  TX_CUDA(ctx, cudaStreamWaitEvent(ctx->stream, p->copied[k], 0));
  p->gets = g + 1;
  *d_out = p->bufs[k];
  return TX_OK;
}
