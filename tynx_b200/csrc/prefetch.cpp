// Upload ring for input batches: the next batch's host-to-device copy runs on
// a copy stream beside the context's compute stream, so it overlaps the step
// that is running instead of preceding the next one.
//
// The ring owns `depth` device buffers (allocated once, outside the context's
// stream-ordered pool: a block recycled by that pool may still be read by
// compute work in flight, which a copy on another stream would not wait for).
// Put n copies into buffer n % depth after the compute stream has finished
// the work issued before put n - depth + 1 (the last reader of that buffer's
// previous batch ran before it), then orders the compute stream after the copy.
#include <vector>

#include "common.h"

struct tx_prefetch {
  tx_ctx *ctx = nullptr;
  size_t bytes = 0;
  int depth = 0;
  uint64_t count = 0;
  cudaStream_t copy = nullptr;
  std::vector<void *> bufs;
  std::vector<cudaEvent_t> issued;  // compute-stream marks, one per put (ring of depth)
  std::vector<cudaEvent_t> copied;  // copy completion, one per buffer
};

extern "C" int tx_prefetch_destroy(tx_prefetch *p) {
  if (!p) return TX_OK;
  if (p->copy) cudaStreamSynchronize(p->copy);
  if (p->ctx) cudaStreamSynchronize(p->ctx->stream);
  for (void *b : p->bufs)
    if (b) cudaFree(b);
  for (cudaEvent_t e : p->issued)
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
  p->issued.assign(depth, nullptr);
  p->copied.assign(depth, nullptr);
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e == cudaSuccess && device != ctx->device) e = cudaSetDevice(ctx->device);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&p->copy, cudaStreamNonBlocking);
  for (int i = 0; i < depth && e == cudaSuccess; ++i) {
    e = cudaMalloc(&p->bufs[i], bytes);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->issued[i], cudaEventDisableTiming);
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

extern "C" int tx_prefetch_put(tx_prefetch *p, const void *h_src, size_t bytes, void **d_out) {
  if (!p || !h_src || !d_out) return TX_ERR_INVALID;
  tx_ctx *ctx = p->ctx;
  if (bytes > p->bytes) return tx_fail(ctx, TX_ERR_SHAPE, "tx_prefetch_put: batch larger than the ring's buffers");
  if (ctx->capturing) return tx_fail(ctx, TX_ERR_CAPTURE, "tx_prefetch_put during a capture");
  const uint64_t n = p->count;
  const int k = (int)(n % (uint64_t)p->depth);
  // the buffer's previous batch (put n - depth) was read by compute work
  // issued before put n - depth + 1
  if (n >= (uint64_t)p->depth)
    TX_CUDA(ctx, cudaStreamWaitEvent(p->copy, p->issued[(n - p->depth + 1) % p->depth], 0));
  TX_CUDA(ctx, cudaEventRecord(p->issued[k], ctx->stream));
  if (bytes) TX_CUDA(ctx, cudaMemcpyAsync(p->bufs[k], h_src, bytes, cudaMemcpyHostToDevice, p->copy));
  TX_CUDA(ctx, cudaEventRecord(p->copied[k], p->copy));
  TX_CUDA(ctx, cudaStreamWaitEvent(ctx->stream, p->copied[k], 0));
  p->count = n + 1;
  *d_out = p->bufs[k];
  return TX_OK;
}
