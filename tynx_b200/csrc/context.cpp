// Context, caching allocator, host<->device copies, errors and CUDA-graph capture.
//
// Replaces the device plumbing of the reference: default_device / synchronize /
// take_device_error (crates/tynx/src/device.rs:55-227) and the tensor storage
// Burn owns behind DynTensor (crates/tynx/src/tensor.rs:156-185).
#include <chrono>
#include <cstdio>
#include <cstring>
#include <thread>

#include "common.h"

// ----------------------------------------------------------------------------
// errors
// ----------------------------------------------------------------------------
int tx_fail(tx_ctx *ctx, int code, const std::string &msg) {
  if (ctx && ctx->err_code == 0) {
    ctx->err_code = code;
    ctx->err_msg = msg;
  }
  return code;
}

int tx_cuda_fail(tx_ctx *ctx, cudaError_t err, const char *what) {
  char buf[512];
  snprintf(buf, sizeof buf, "CUDA error %d (%s) in %s", (int)err, cudaGetErrorString(err), what);
  return tx_fail(ctx, err == cudaErrorMemoryAllocation ? TX_ERR_OOM : TX_ERR_CUDA, buf);
}

extern "C" int tx_abi_version(void) { return TYNX_CUDA_ABI_VERSION; }

extern "C" int tx_device_count(int *out) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) n = 0;
  *out = n;
  return TX_OK;
}

extern "C" int tx_ctx_create(int device, int math_mode, tx_ctx **out) {
  if (!out) return TX_ERR_INVALID;
  *out = nullptr;
  if (math_mode < TX_MATH_TF32 || math_mode > TX_MATH_TF32_TRUNC) return TX_ERR_INVALID;
  if (cudaSetDevice(device) != cudaSuccess) return TX_ERR_CUDA;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return TX_ERR_CUDA;
  if (prop.major != 10) {
    // The kernels are compiled for sm_100a only.
    return TX_ERR_UNSUPPORTED;
  }
  tx_ctx *ctx = new tx_ctx();
  ctx->device = device;
  ctx->math = math_mode;
  ctx->num_sms = prop.multiProcessorCount;
  if (cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaStreamCreateWithFlags(&ctx->comm, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&ctx->d_err, 4 * sizeof(int)) != cudaSuccess ||
      cudaMemset(ctx->d_err, 0, 4 * sizeof(int)) != cudaSuccess ||
      cudaMalloc(&ctx->d_rng, sizeof(uint64_t)) != cudaSuccess ||
      cudaMemset(ctx->d_rng, 0, sizeof(uint64_t)) != cudaSuccess) {
    cudaFree(ctx->d_err);
    cudaFree(ctx->d_rng);
    delete ctx;
    return TX_ERR_CUDA;
  }
  *out = ctx;
  return TX_OK;
}

extern "C" int tx_ctx_set_math(tx_ctx *ctx, int math_mode) {
  if (!ctx || math_mode < TX_MATH_TF32 || math_mode > TX_MATH_TF32_TRUNC) return TX_ERR_INVALID;
  ctx->math = math_mode;
  return TX_OK;
}

extern "C" int tx_ctx_get_math(tx_ctx *ctx, int *out) {
  if (!ctx || !out) return TX_ERR_INVALID;
  *out = ctx->math;
  return TX_OK;
}

extern "C" int tx_last_error(tx_ctx *ctx, char *buf, size_t n) {
  if (!ctx) return TX_ERR_INVALID;
  int code = ctx->err_code;
  if (buf && n) {
    size_t len = ctx->err_msg.size() < n - 1 ? ctx->err_msg.size() : n - 1;
    memcpy(buf, ctx->err_msg.data(), len);
    buf[len] = 0;
  }
  ctx->err_code = 0;
  ctx->err_msg.clear();
  return code;
}

static int check_device_flag(tx_ctx *ctx) {
  int flag[4] = {0, 0, 0, 0};
  TX_CUDA(ctx, cudaMemcpy(flag, ctx->d_err, sizeof flag, cudaMemcpyDeviceToHost));
  if (flag[0] == DEVERR_NONE) return TX_OK;
  TX_CUDA(ctx, cudaMemset(ctx->d_err, 0, sizeof flag));
  char buf[256];
  switch (flag[0]) {
    case DEVERR_INDEX:
      snprintf(buf, sizeof buf, "index %d is out of range for an axis of size %d", flag[1], flag[2]);
      return tx_fail(ctx, TX_ERR_INDEX, buf);
    case DEVERR_LABEL:
      snprintf(buf, sizeof buf, "class target %d is out of range for %d classes", flag[1], flag[2]);
      return tx_fail(ctx, TX_ERR_INDEX, buf);
    case DEVERR_TIMEOUT:
      snprintf(buf, sizeof buf, "a device-side wait expired (site %d)", flag[1]);
      return tx_fail(ctx, TX_ERR_TIMEOUT, buf);
    default:
      snprintf(buf, sizeof buf, "device error flag %d", flag[0]);
      return tx_fail(ctx, TX_ERR_DEVICE, buf);
  }
}

extern "C" int tx_sync(tx_ctx *ctx, uint64_t timeout_ms) {
  if (!ctx) return TX_ERR_INVALID;
  if (ctx->capturing) return tx_fail(ctx, TX_ERR_CAPTURE, "tx_sync is not allowed during capture");
  auto start = std::chrono::steady_clock::now();
  cudaStream_t streams[2] = {ctx->stream, ctx->comm};
  for (cudaStream_t s : streams) {
    while (true) {
      cudaError_t q = cudaStreamQuery(s);
      if (q == cudaSuccess) break;
      if (q != cudaErrorNotReady) return tx_cuda_fail(ctx, q, "stream synchronisation");
      if (timeout_ms) {
        auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                      std::chrono::steady_clock::now() - start)
                      .count();
        if ((uint64_t)ms > timeout_ms)
          return tx_fail(ctx, TX_ERR_TIMEOUT, "device synchronisation timed out");
      }
      std::this_thread::yield();
    }
  }
  if (ctx->err_code) return ctx->err_code;
  return check_device_flag(ctx);
}

extern "C" int tx_stream(tx_ctx *ctx, void **out) {
  if (!ctx || !out) return TX_ERR_INVALID;
  *out = (void *)ctx->stream;
  return TX_OK;
}

// ----------------------------------------------------------------------------
// allocator
// ----------------------------------------------------------------------------
static size_t size_class(size_t bytes) {
  if (bytes == 0) bytes = 1;
  if (bytes <= (1u << 20)) return (bytes + 511) & ~size_t(511);
  return (bytes + (2u << 20) - 1) & ~size_t((2u << 20) - 1);
}

static void *arena_alloc(tx_ctx *ctx, tx_arena *arena, size_t bytes) {
  size_t need = (bytes + 255) & ~size_t(255);
  if (arena->chunks.empty() || arena->offset + need > arena->chunks.back().second) {
    size_t chunk = need > (64u << 20) ? need : (64u << 20);
    void *p = nullptr;
    if (cudaMalloc(&p, chunk) != cudaSuccess) {
      cudaGetLastError();
      tx_fail(ctx, TX_ERR_OOM, "capture arena allocation failed");
      return nullptr;
    }
    arena->chunks.push_back({(char *)p, chunk});
    arena->offset = 0;
  }
  char *p = arena->chunks.back().first + arena->offset;
  arena->offset += need;
  arena->blocks.insert(p);
  ctx->alloc.arena_owner[p] = arena;
  return p;
}

static void release_cached(tx_ctx *ctx) {
  cudaStreamSynchronize(ctx->stream);
  for (auto &kv : ctx->alloc.free_blocks)
    for (void *p : kv.second) cudaFree(p);
  ctx->alloc.free_blocks.clear();
  ctx->alloc.cached = 0;
}

void *tx_alloc_raw(tx_ctx *ctx, size_t bytes) {
  tx_allocator &A = ctx->alloc;
  if (A.arena) return arena_alloc(ctx, A.arena, bytes);
  size_t cls = size_class(bytes);
  auto it = A.free_blocks.find(cls);
  if (it != A.free_blocks.end() && !it->second.empty()) {
    void *p = it->second.back();
    it->second.pop_back();
    A.cached -= cls;
    A.live[p] = cls;
    A.in_use += cls;
    return p;
  }
  void *p = nullptr;
  if (cudaMalloc(&p, cls) != cudaSuccess) {
    cudaGetLastError();
    release_cached(ctx);
    if (cudaMalloc(&p, cls) != cudaSuccess) {
      cudaGetLastError();
      char buf[128];
      snprintf(buf, sizeof buf, "device allocation of %zu bytes failed", cls);
      tx_fail(ctx, TX_ERR_OOM, buf);
      return nullptr;
    }
  }
  A.live[p] = cls;
  A.in_use += cls;
  return p;
}

void tx_free_raw(tx_ctx *ctx, void *p) {
  if (!p) return;
  tx_allocator &A = ctx->alloc;
  if (A.arena_owner.count(p)) return;  // arena memory lives as long as its exec
  auto it = A.live.find(p);
  if (it == A.live.end()) return;
  size_t cls = it->second;
  A.live.erase(it);
  A.in_use -= cls;
  if (A.arena) {  // the graph being captured may still reference this block
    A.quarantine.push_back(p);
    return;
  }
  A.free_blocks[cls].push_back(p);
  A.cached += cls;
}

extern "C" int tx_alloc(tx_ctx *ctx, size_t bytes, void **d_out) {
  if (!ctx || !d_out) return TX_ERR_INVALID;
  *d_out = tx_alloc_raw(ctx, bytes);
  return *d_out ? TX_OK : TX_ERR_OOM;
}

extern "C" int tx_free(tx_ctx *ctx, void *d_ptr) {
  if (!ctx) return TX_ERR_INVALID;
  tx_free_raw(ctx, d_ptr);
  return TX_OK;
}

extern "C" int tx_mem_stats(tx_ctx *ctx, uint64_t *in_use, uint64_t *cached) {
  if (!ctx) return TX_ERR_INVALID;
  if (in_use) *in_use = ctx->alloc.in_use;
  if (cached) *cached = ctx->alloc.cached;
  return TX_OK;
}

extern "C" int tx_h2d(tx_ctx *ctx, void *d_dst, const void *h_src, size_t bytes) {
  if (!ctx) return TX_ERR_INVALID;
  if (!bytes) return TX_OK;
  if (ctx->capturing && ctx->alloc.arena) {
    // A recorded copy re-reads its source on every replay: stage the bytes in
    // pinned memory that lives as long as the captured graph.
    void *stage = nullptr;
    TX_CUDA(ctx, cudaMallocHost(&stage, bytes));
    memcpy(stage, h_src, bytes);
    ctx->alloc.arena->pinned.push_back(stage);
    h_src = stage;
  }
  TX_CUDA(ctx, cudaMemcpyAsync(d_dst, h_src, bytes, cudaMemcpyHostToDevice, ctx->stream));
  return TX_OK;
}

extern "C" int tx_d2h(tx_ctx *ctx, void *h_dst, const void *d_src, size_t bytes) {
  if (!ctx) return TX_ERR_INVALID;
  if (ctx->capturing)
    return tx_fail(ctx, TX_ERR_CAPTURE, "reading device data on the host is not capturable");
  if (bytes) {
    TX_CUDA(ctx, cudaMemcpyAsync(h_dst, d_src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
    TX_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  }
  return check_device_flag(ctx);
}

extern "C" int tx_d2d(tx_ctx *ctx, void *d_dst, const void *d_src, size_t bytes) {
  if (!ctx) return TX_ERR_INVALID;
  if (!bytes || d_dst == d_src) return TX_OK;
  TX_CUDA(ctx, cudaMemcpyAsync(d_dst, d_src, bytes, cudaMemcpyDeviceToDevice, ctx->stream));
  return TX_OK;
}

extern "C" int tx_memset(tx_ctx *ctx, void *d_ptr, int value, size_t bytes) {
  if (!ctx) return TX_ERR_INVALID;
  if (!bytes) return TX_OK;
  TX_CUDA(ctx, cudaMemsetAsync(d_ptr, value, bytes, ctx->stream));
  return TX_OK;
}

extern "C" int tx_host_alloc(size_t bytes, void **h_out) {
  if (!h_out) return TX_ERR_INVALID;
  return cudaMallocHost(h_out, bytes ? bytes : 1) == cudaSuccess ? TX_OK : TX_ERR_OOM;
}

extern "C" int tx_host_free(void *h_ptr) {
  if (h_ptr) cudaFreeHost(h_ptr);
  return TX_OK;
}

// ----------------------------------------------------------------------------
// capture
// ----------------------------------------------------------------------------
extern "C" int tx_capture_begin(tx_ctx *ctx) {
  if (!ctx) return TX_ERR_INVALID;
  if (ctx->capturing) return tx_fail(ctx, TX_ERR_CAPTURE, "a capture is already active");
  TX_CUDA(ctx, cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeRelaxed));
  ctx->alloc.arena = new tx_arena();
  ctx->capturing = true;
  return TX_OK;
}

static void drop_arena(tx_ctx *ctx, tx_arena *arena) {
  if (!arena) return;
  for (void *b : arena->blocks) ctx->alloc.arena_owner.erase(b);
  for (auto &c : arena->chunks) cudaFree(c.first);
  for (void *h : arena->pinned) cudaFreeHost(h);
  delete arena;
}

extern "C" int tx_capture_end(tx_ctx *ctx, tx_exec **out) {
  if (!ctx || !out) return TX_ERR_INVALID;
  *out = nullptr;
  if (!ctx->capturing) return tx_fail(ctx, TX_ERR_CAPTURE, "no capture is active");
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamEndCapture(ctx->stream, &graph);
  tx_arena *arena = ctx->alloc.arena;
  ctx->alloc.arena = nullptr;
  ctx->capturing = false;
  if (e != cudaSuccess || ctx->err_code) {
    if (graph) cudaGraphDestroy(graph);
    drop_arena(ctx, arena);
    cudaGetLastError();
    if (ctx->err_code) return ctx->err_code;
    return tx_cuda_fail(ctx, e, "cudaStreamEndCapture");
  }
  cudaGraphExec_t exec = nullptr;
  e = cudaGraphInstantiate(&exec, graph, 0);
  if (e != cudaSuccess) {
    cudaGraphDestroy(graph);
    drop_arena(ctx, arena);
    return tx_cuda_fail(ctx, e, "cudaGraphInstantiate");
  }
  tx_exec *x = new tx_exec();
  x->ctx = ctx;
  x->graph = graph;
  x->exec = exec;
  x->arena = arena;
  *out = x;
  return TX_OK;
}

extern "C" int tx_capture_abort(tx_ctx *ctx) {
  if (!ctx) return TX_ERR_INVALID;
  if (!ctx->capturing) return TX_OK;
  cudaGraph_t graph = nullptr;
  cudaStreamEndCapture(ctx->stream, &graph);
  cudaGetLastError();
  if (graph) cudaGraphDestroy(graph);
  drop_arena(ctx, ctx->alloc.arena);
  ctx->alloc.arena = nullptr;
  ctx->capturing = false;
  return TX_OK;
}

extern "C" int tx_capture_active(tx_ctx *ctx, int *out) {
  if (!ctx || !out) return TX_ERR_INVALID;
  *out = ctx->capturing ? 1 : 0;
  return TX_OK;
}

extern "C" int tx_exec_launch(tx_exec *x) {
  if (!x) return TX_ERR_INVALID;
  TX_CUDA(x->ctx, cudaGraphLaunch(x->exec, x->ctx->stream));
  return TX_OK;
}

extern "C" int tx_exec_node_count(tx_exec *x, int64_t *kernels, int64_t *total) {
  if (!x) return TX_ERR_INVALID;
  size_t n = 0;
  TX_CUDA(x->ctx, cudaGraphGetNodes(x->graph, nullptr, &n));
  std::vector<cudaGraphNode_t> nodes(n);
  if (n) TX_CUDA(x->ctx, cudaGraphGetNodes(x->graph, nodes.data(), &n));
  int64_t k = 0;
  for (auto node : nodes) {
    cudaGraphNodeType t;
    if (cudaGraphNodeGetType(node, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) ++k;
  }
  if (kernels) *kernels = k;
  if (total) *total = (int64_t)n;
  return TX_OK;
}

extern "C" int tx_exec_destroy(tx_exec *x) {
  if (!x) return TX_OK;
  cudaStreamSynchronize(x->ctx->stream);
  cudaGraphExecDestroy(x->exec);
  cudaGraphDestroy(x->graph);
  drop_arena(x->ctx, x->arena);
  delete x;
  return TX_OK;
}

int tx_dp_shutdown(tx_ctx *ctx);  // dp.cu

extern "C" int tx_ctx_destroy(tx_ctx *ctx) {
  if (!ctx) return TX_OK;
  cudaStreamSynchronize(ctx->stream);
  cudaStreamSynchronize(ctx->comm);
  tx_dp_shutdown(ctx);
  for (auto &kv : ctx->alloc.free_blocks)
    for (void *p : kv.second) cudaFree(p);
  for (auto &kv : ctx->alloc.live) cudaFree(kv.first);
  for (void *p : ctx->alloc.quarantine) cudaFree(p);
  cudaFree(ctx->d_err);
  cudaFree(ctx->d_rng);
  cudaStreamDestroy(ctx->stream);
  cudaStreamDestroy(ctx->comm);
  delete ctx;
  return TX_OK;
}
