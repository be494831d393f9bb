// Internal declarations shared by the libtynx_cuda translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <map>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "../../include/tynx_cuda.h"

// Device-side error codes written into ctx->d_err[0] by kernels.  Kernels never
// trap: they record the first problem, skip the offending access and return.
enum { DEVERR_NONE = 0, DEVERR_INDEX = 1, DEVERR_TIMEOUT = 2, DEVERR_LABEL = 3 };

struct tx_arena {
  std::vector<std::pair<char *, size_t>> chunks;
  size_t offset = 0;  // within chunks.back()
  std::unordered_set<void *> blocks;
  std::vector<void *> pinned;  // host staging for copies recorded during capture
};

struct tx_allocator {
  // size class (bytes) -> cached device blocks, reused in stream order
  std::map<size_t, std::vector<void *>> free_blocks;
  std::unordered_map<void *, size_t> live;
  uint64_t in_use = 0, cached = 0;
  tx_arena *arena = nullptr;  // non-null while capturing
  std::unordered_map<void *, tx_arena *> arena_owner;
  std::vector<void *> quarantine;  // eager blocks freed during a capture
};

struct tx_ctx {
  int device = 0;
  int math = TX_MATH_TF32;
  int num_sms = 148;
  cudaStream_t stream = nullptr;  // compute
  cudaStream_t comm = nullptr;    // collectives
  tx_allocator alloc;
  int err_code = 0;
  std::string err_msg;
  int *d_err = nullptr;  // device error flag [4]
  uint64_t *d_rng = nullptr;  // call counter of the dropout stream
  bool capturing = false;
  // data parallel
  void *nccl = nullptr;
  int world = 1, rank = 0;
  uint64_t dp_timeout_ms = 60000;
};

struct tx_exec {
  tx_ctx *ctx = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  tx_arena *arena = nullptr;
};

// ---- error helpers ---------------------------------------------------------
int tx_fail(tx_ctx *ctx, int code, const std::string &msg);
int tx_cuda_fail(tx_ctx *ctx, cudaError_t err, const char *what);
#define TX_CUDA(ctx, expr)                                    \
  do {                                                        \
    cudaError_t _e = (expr);                                  \
    if (_e != cudaSuccess) return tx_cuda_fail(ctx, _e, #expr); \
  } while (0)
#define TX_LAUNCHED(ctx, name)                                      \
  do {                                                              \
    cudaError_t _e = cudaGetLastError();                            \
    if (_e != cudaSuccess) return tx_cuda_fail(ctx, _e, name);      \
  } while (0)
#define TX_TRY(expr)             \
  do {                           \
    int _rc = (expr);            \
    if (_rc != TX_OK) return _rc; \
  } while (0)

// ---- allocation (stream ordered on ctx->stream) -----------------------------
void *tx_alloc_raw(tx_ctx *ctx, size_t bytes);
void tx_free_raw(tx_ctx *ctx, void *p);

// RAII scratch buffer from the context allocator.
struct Scratch {
  tx_ctx *ctx;
  void *ptr = nullptr;
  Scratch(tx_ctx *c, size_t bytes) : ctx(c) { ptr = bytes ? tx_alloc_raw(c, bytes) : nullptr; }
  ~Scratch() {
    if (ptr) tx_free_raw(ctx, ptr);
  }
  template <class T>
  T *as() const { return reinterpret_cast<T *>(ptr); }
  Scratch(const Scratch &) = delete;
  Scratch &operator=(const Scratch &) = delete;
};

// ---- GEMM internals -----------------------------------------------------------
// Fused column sums (tx_gemm_desc::colsum).  gemm_dispatch provides a partial
// buffer of ceil(M / 32) x N floats; a kernel path that can fuse the sums
// writes `rows` partial rows of unrounded column sums and sets fused.  A path
// that cannot fuse stores C unrounded (it ignores TX_GEMM_ROUND_OUT) and the
// dispatcher sums C afterwards.
struct FusedSum {
  float *part = nullptr;
  int64_t rows = 0;
  bool fused = false;
};

int gemm_simt(tx_ctx *ctx, const tx_gemm_desc &d);
int colsum_finish(tx_ctx *ctx, const float *part, int64_t np, int64_t cols, float *out, float scale, int acc);
// Returns TX_ERR_UNSUPPORTED (without latching) when the shape/layout cannot use
// the tensor-core path; the dispatcher then uses the SIMT kernel.
int gemm_tcgen05(tx_ctx *ctx, const tx_gemm_desc &d, int mode, FusedSum *fs = nullptr);
// `rounded` (optional) tells whether C was stored TF32-rounded.
int gemm_dispatch(tx_ctx *ctx, const tx_gemm_desc &d, bool *rounded = nullptr);
// Bandwidth-shaped kernels for K <= 32, N <= 16 or M <= 16; TX_ERR_UNSUPPORTED
// (not latched) for every other shape.
int gemm_skinny(tx_ctx *ctx, const tx_gemm_desc &d, FusedSum *fs = nullptr);
bool skinny_shape(const tx_gemm_desc &d);
int gemm_split_reduce(tx_ctx *ctx, const tx_gemm_desc &d, const float *part, int splits);

// N-d bandwidth kernels on canonicalised shapes (nd.cu).  Strides in elements,
// 0 = broadcast; outputs are contiguous.  nd_reduce returns TX_ERR_UNSUPPORTED
// (not latched) for layouts that are not [outer, reduced, inner].
int nd_binary(tx_ctx *ctx, int op, const float *A, const int64_t *sa, const float *B, const int64_t *sb,
              float *out, const int64_t *shape, int ndim);
// out[b][c][r] (+)= in[b][r][c]: batched transpose of [R, Cc] fp32 matrices
// through shared-memory tiles (engine.cu).
int batched_transpose(tx_ctx *ctx, const float *in, float *out, int64_t B, int64_t R, int64_t Cc, int acc);
int nd_copy(tx_ctx *ctx, const void *src, const int64_t *ss, void *out, const int64_t *shape, int ndim,
            int elem_bytes, float scale, int acc);
int nd_reduce(tx_ctx *ctx, const float *x, const int64_t *in_shape, const int64_t *out_shape, int ndim,
              float *y, float scale, int acc);
// out[os] (+)= src (contiguous over `shape`): a strided destination.
int nd_scatter(tx_ctx *ctx, const float *src, float *out, const int64_t *os, const int64_t *shape, int ndim,
               int acc);
// out (contiguous over `shape`) = dy * d(A op B)/d(operand `which`) for op MAX / MIN / POW.
int nd_binary_grad(tx_ctx *ctx, int op, int which, const float *A, const int64_t *sa, const float *B,
                   const int64_t *sb, const float *dy, float *out, const int64_t *shape, int ndim);
// y[o][i] = max / min over r of x[o][r][i] (contiguous x), arg (or null) the
// first r attaining it; the backward routes dy there
int reduce_maxmin(tx_ctx *ctx, const float *x, float *y, int32_t *arg, int64_t outer, int64_t red, int64_t inner,
                  bool is_max);
int reduce_maxmin_bwd(tx_ctx *ctx, const float *dy, const int32_t *arg, float *dx, int64_t outer, int64_t red,
                      int64_t inner, int acc);

// Softmax over rows; y32 (may be null, not with log): a second copy of y
// rounded to TF32 for the contractions that read it, while the backward
// reads the exact y.  The backward's round stores dx rounded to TF32.
int softmax_fwd(tx_ctx *ctx, const float *x, float *y, float *y32, int64_t rows, int64_t cols, int log);
int softmax_bwd(tx_ctx *ctx, const float *y, const float *dy, float *dx, int64_t rows, int64_t cols, int log,
                int acc, bool round);
// LayerNorm forward; round_tf32 stores y rounded to TF32 (for an output that
// only feeds contractions; the backward reads x, mean and rstd, not y).
int layernorm_fwd(tx_ctx *ctx, const float *x, const float *gamma, const float *beta, float *y, float *mean,
                  float *rstd, int64_t rows, int64_t cols, float eps, bool round_tf32);

// Direct convolution for short filters (conv_direct.cu): C * KH * KW < 32 and
// OC <= 64.  geom = {N, C, H, W, KH, KW, OH, OW, sh, sw, pt, pl, dh, dw}; x is
// NCHW; y NCHW or channels-last; dz channels-last [N * OH * OW][OC]; dw is
// [OC][C][KH][KW], db (or null) [OC].  TX_ERR_UNSUPPORTED for other shapes.
bool conv_direct_ok(int C, int KH, int KW, int OC);
int conv_direct_fwd(tx_ctx *ctx, const float *x, const float *w, const float *bias, float *y, const int *geom, int OC,
                    int act, bool nhwc_out);
int conv_direct_wgrad(tx_ctx *ctx, const float *x, const float *dz, const int *geom, int OC, float *dw, float *db,
                      int acc_w, int acc_b);

// grid sizing helper
inline unsigned grid_for(int64_t n, int threads, int64_t max_blocks = 148 * 16) {
  int64_t b = (n + threads - 1) / threads;
  if (b < 1) b = 1;
  if (b > max_blocks) b = max_blocks;
  return (unsigned)b;
}
