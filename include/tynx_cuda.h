/*
 * tynx_cuda.h -- C ABI of libtynx_cuda.so, the B200 (sm_100a) training-step
 * engine for imported ONNX graphs.
 *
 * The reference (blaind/tynx) runs every tensor operation through Burn
 * (burn-flex on CPU, burn-autodiff for backward rules, CubeCL/wgpu on GPUs);
 * there is no C ABI upstream.  This header is the drop-in boundary a
 * `tynx-cuda-sys` crate binds with `extern "C"` (crates/tynx-cuda-sys in this
 * repository holds that block as Rust source).  Each
 * group names the reference function or type it replaces (path:line inside
 * the reference project).
 *
 * Conventions
 *   - Every function returns int: 0 (TX_OK) on success, a TX_ERR_* code
 *     otherwise.  The message of the first error is latched per context and
 *     read with tx_last_error(), the analogue of LAST_DEVICE_ERROR /
 *     take_device_error (crates/tynx/src/device.rs:55-81).
 *   - Pointers named d_* are device pointers; h_* are host pointers.
 *   - Tensors are dense row-major.  float tensors are IEEE fp32; index
 *     tensors are int64 (ONNX/Flex semantics).
 *   - All work is enqueued on the context's compute stream in call order.
 *     Functions that return host data (tx_d2h, tx_sync) synchronise.
 *   - A context is confined to the host thread that created it, matching
 *     Tynx's thread confinement (crates/tynx-python/src/tensor.rs:54-92).
 */
#ifndef TYNX_CUDA_H
#define TYNX_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TYNX_CUDA_ABI_VERSION 2

/* ---- status codes (TynxError, crates/tynx/src/error.rs:1-122) ----------- */
enum {
  TX_OK = 0,
  TX_ERR_INVALID = 1,      /* bad argument (TynxError::TypeMismatch / InvalidModel) */
  TX_ERR_SHAPE = 2,        /* shape mismatch (TynxError::Shape) */
  TX_ERR_INDEX = 3,        /* index outside [-size, size) (normalize_indices, tensor.rs:2504) */
  TX_ERR_OOM = 4,          /* device allocation failed */
  TX_ERR_CUDA = 5,         /* CUDA runtime error (TynxError::AsynchronousDevice, error.rs:54-55) */
  TX_ERR_TIMEOUT = 6,      /* bounded wait expired (TynxError::DeviceSynchronization, error.rs:58-59) */
  TX_ERR_UNSUPPORTED = 7,  /* operator or attribute not implemented on this device */
  TX_ERR_DEVICE = 8,       /* a kernel raised the context's device error flag */
  TX_ERR_NCCL = 9,         /* collective failure */
  TX_ERR_CAPTURE = 10      /* operation not allowed while capturing a CUDA graph */
};

/* ---- math modes for fp32 contractions (TYNX_CUDA_MATH) ------------------ */
enum {
  TX_MATH_TF32 = 0,      /* tcgen05 kind::tf32, operands rounded to nearest TF32 in shared
                            memory, fp32 accumulate (rel 1e-3 class) */
  TX_MATH_3XTF32 = 1,    /* split-operand 3xTF32 on tcgen05 (fp32 class, 1e-5) */
  TX_MATH_FP32 = 2,      /* SIMT FFMA, exact fp32 products */
  TX_MATH_TF32_TRUNC = 3 /* kind::tf32 on raw fp32 operands: the tensor core drops the
                            13 low mantissa bits (truncation; fastest, biased) */
};

typedef struct tx_ctx tx_ctx;
typedef struct tx_graph tx_graph;
typedef struct tx_record tx_record;
typedef struct tx_exec tx_exec;
typedef struct tx_optim tx_optim;

/* =========================================================================
 * Context, placement, synchronisation
 * replaces: Device selection and errors -- default_device (crates/tynx/src/device.rs:214-227),
 *           synchronize (device.rs:84-90), take_device_error (device.rs:79-81),
 *           PyDevice::py_new (crates/tynx-python/src/device.rs:50-61)
 * ========================================================================= */
int tx_abi_version(void);
int tx_device_count(int *out);
int tx_ctx_create(int device, int math_mode, tx_ctx **out);
int tx_ctx_destroy(tx_ctx *ctx);
int tx_ctx_set_math(tx_ctx *ctx, int math_mode);
int tx_ctx_get_math(tx_ctx *ctx, int *out);
/* Copy the latched first error message (NUL-terminated) and clear it.
 * Returns the latched code (0 if none). */
int tx_last_error(tx_ctx *ctx, char *buf, size_t n);
/* Wait for all work on the context's streams; gives up after timeout_ms
 * (0 = no limit) with TX_ERR_TIMEOUT.  Surfaces device-side error flags. */
int tx_sync(tx_ctx *ctx, uint64_t timeout_ms);
/* The compute stream as a cudaStream_t, for interop with other libraries. */
int tx_stream(tx_ctx *ctx, void **out);

/* =========================================================================
 * Device memory (replaces Burn tensor storage behind DynTensor,
 * crates/tynx/src/tensor.rs:156-185).  Stream-ordered caching allocator.
 * ========================================================================= */
int tx_alloc(tx_ctx *ctx, size_t bytes, void **d_out);
int tx_free(tx_ctx *ctx, void *d_ptr);
int tx_h2d(tx_ctx *ctx, void *d_dst, const void *h_src, size_t bytes);
int tx_d2h(tx_ctx *ctx, void *h_dst, const void *d_src, size_t bytes);
int tx_d2d(tx_ctx *ctx, void *d_dst, const void *d_src, size_t bytes);
int tx_memset(tx_ctx *ctx, void *d_ptr, int value, size_t bytes);
int tx_fill_f32(tx_ctx *ctx, float *d_ptr, int64_t n, float value);
int tx_host_alloc(size_t bytes, void **h_out); /* pinned host memory */

/* Upload ring for input batches (no counterpart in the reference, which reads
 * its inputs from host memory on every step).  `depth` (2..16) device buffers
 * of `bytes` each and a copy stream beside the compute stream.
 * tx_prefetch_put queues the copy of `bytes` from h_src (pinned, for the copy
 * to overlap; unchanged until the copy has run) into the next buffer; it does
 * not order the compute stream.  tx_prefetch_get returns the buffer of the
 * oldest queued batch and orders all compute work issued after it behind that
 * batch's copy.  A buffer is refilled only after the compute work issued
 * before the get that followed its previous batch: a batch returned by get
 * stays valid for the device work issued before the next get (work issued
 * after that get may see the buffer refilled), while up to depth - 1 further
 * batches upload beside it.  With depth 3: put batches 0 and 1,
 * then per step get, launch the step, put the batch two ahead, read the loss.
 * put fails (TX_ERR_INVALID) when it would run more than depth - 1 batches
 * ahead of get.  Neither call is allowed during a capture. */
typedef struct tx_prefetch tx_prefetch;
int tx_prefetch_create(tx_ctx *ctx, size_t bytes, int depth, tx_prefetch **out);
int tx_prefetch_put(tx_prefetch *p, const void *h_src, size_t bytes);
int tx_prefetch_get(tx_prefetch *p, void **d_out);
int tx_prefetch_destroy(tx_prefetch *p);
int tx_host_free(void *h_ptr);
/* Bytes currently held by the allocator (in use, cached). */
int tx_mem_stats(tx_ctx *ctx, uint64_t *in_use, uint64_t *cached);

/* =========================================================================
 * Whole-step capture (replaces Graph::run_values replay,
 * crates/tynx-capture/src/lib.rs:747-882, and CompiledFunction,
 * crates/tynx-python/python/tynx/compiler.py:131-205).
 * Between begin and end, all work issued on the context is recorded into a
 * CUDA graph; allocations come from an arena owned by the resulting exec.
 * ========================================================================= */
int tx_capture_begin(tx_ctx *ctx);
int tx_capture_end(tx_ctx *ctx, tx_exec **out);
int tx_capture_abort(tx_ctx *ctx);
int tx_capture_active(tx_ctx *ctx, int *out);
int tx_exec_launch(tx_exec *exec);
int tx_exec_destroy(tx_exec *exec);
/* Number of kernel nodes (and all nodes) recorded in a captured graph. */
int tx_exec_node_count(tx_exec *exec, int64_t *kernels, int64_t *total);

/* =========================================================================
 * Kernels behind the DynTensor method surface (crates/tynx/src/tensor.rs).
 * These are the eager-op entry points used by Tensor and by the loss code.
 * ========================================================================= */

/* Dense fp32 contraction C = alpha * op(A) @ op(B) (+ beta * C) (+ bias) with
 * an optional fused activation epilogue.
 * replaces: DynTensor::matmul (tensor.rs:1715-1786), execute_gemm + add_bias
 * (crates/tynx-train/src/imported_model/executor.rs:499-524, 606-613) and
 * Burn's matmul backward (dA = dY B^T, dB = A^T dY). */
enum { TX_ACT_NONE = 0, TX_ACT_RELU = 1, TX_ACT_TANH = 2, TX_ACT_GELU = 3 };
typedef struct tx_gemm_desc {
  int64_t M, N, K;
  const float *A; int64_t lda; int32_t trans_a; /* A: MxK row-major, or KxM when trans_a */
  const float *B; int64_t ldb; int32_t trans_b; /* B: KxN row-major, or NxK when trans_b */
  float *C; int64_t ldc;                       /* C: MxN row-major */
  float alpha, beta;                           /* beta != 0 reads C before writing */
  const float *bias; float bias_scale;         /* optional per-column bias, length N */
  int32_t act;                                 /* TX_ACT_* applied after bias */
  float *preact; int64_t ld_preact;            /* optional: store value before act */
  /* optional dgrad fusion: multiply the result by act'(src) where src is the
   * saved forward output (relu, tanh) or pre-activation (gelu) */
  const float *dact_src; int64_t ld_dact; int32_t dact;
  int64_t batch; int64_t stride_a, stride_b, stride_c; /* strided batch (batch<=1: single) */
  int32_t flags;                               /* TX_GEMM_* below; 0 = none */
  /* optional fused column sum (the bias gradient of the layer whose
   * pre-activation gradient this product is): colsum[n] (+)= colsum_scale *
   * sum over rows of C[:, n], taken before any TF32 output rounding;
   * colsum_acc != 0 adds to colsum.  batch must be 1. */
  float *colsum; float colsum_scale; int32_t colsum_acc;
  /* optional, TX_MATH_TF32 only: the TF32 tail of B (B_lo = rna(B0 - B) for
   * the weights B0 whose TF32 head rna(B0) is B), same layout as B; the
   * product becomes op(A) (B + B_lo), fp32-class in B */
  const float *B_lo;
} tx_gemm_desc;
/* flags: in TX_MATH_TF32 (round-to-nearest) mode the contraction rounds each
 * operand element to TF32 (cvt.rna).  An operand whose buffer already holds
 * such values (A_TF32 / B_TF32) is used as is; ROUND_OUT stores C rounded the
 * same way, for a result that only feeds further contractions.  EXACT asks
 * for fp32-class accuracy in that mode (3xTF32: each operand split into a
 * TF32 head and a TF32 tail, three products per k-block); it overrides
 * A_TF32 / B_TF32, so both operands must hold unrounded values.  The graph
 * engine sets it on forward contractions whose result passes through a ReLU,
 * whose mask is discontinuous: a TF32 rounding of the pre-activation flips it
 * wherever the value lies within ~2^-11 of zero, and every flip moves a whole
 * gradient entry.  Other math modes ignore the flags, except A_SHARED: a
 * batched product (batch > 1) whose A is one matrix for every batch entry
 * (stride_a must be 0), as when sibling projections of one input run as one
 * launch over weights stored back to back. */
enum { TX_GEMM_A_TF32 = 1, TX_GEMM_B_TF32 = 2, TX_GEMM_ROUND_OUT = 4, TX_GEMM_EXACT = 8, TX_GEMM_A_SHARED = 16 };
int tx_gemm(tx_ctx *ctx, const tx_gemm_desc *desc);
/* dst[i] = src[i] rounded to TF32 (round to nearest, ties away from zero;
 * dst may equal src).  The operand shadow of TX_GEMM_A_TF32 / B_TF32. */
int tx_round_tf32(tx_ctx *ctx, const float *d_src, float *d_dst, int64_t n);
/* d_hi[i] = rna(src[i]) and d_lo[i] = rna(src[i] - d_hi[i]) (TF32 head and
 * tail: hi + lo equals src to about 2^-22 relative).  The graph engine splits
 * its parameters so every forward contraction multiplies by the weights to
 * fp32-class accuracy (tx_gemm_desc.B_lo). */
int tx_split_tf32(tx_ctx *ctx, const float *d_src, float *d_hi, float *d_lo, int64_t n);

/* Elementwise.  replaces: DynTensor activations (tensor.rs:2002-2240) and
 * broadcast arithmetic (tensor.rs:1637-1700). */
enum {
  TX_UN_NEG = 0, TX_UN_EXP = 1, TX_UN_LOG = 2, TX_UN_RELU = 3, TX_UN_TANH = 4,
  TX_UN_GELU = 5, TX_UN_SIGMOID = 6, TX_UN_CLAMP = 7, TX_UN_SQRT = 8, TX_UN_ABS = 9,
  TX_UN_SCALE = 10, /* y = a*x + b */
  TX_UN_POW = 11,   /* y = x^a */
  TX_UN_ERF = 12, TX_UN_LEAKYRELU = 13 /* slope a */, TX_UN_SOFTPLUS = 14, TX_UN_ELU = 15 /* alpha a */,
  TX_UN_HARDSIGMOID = 16 /* max(0, min(1, a*x + b)) */, TX_UN_SOFTSIGN = 17, TX_UN_RECIPROCAL = 18
};
int tx_unary(tx_ctx *ctx, int op, const float *d_x, float *d_y, int64_t n, float a, float b);
/* dx (+)= dy * op'(x or y).  `src` is y for EXP/TANH/SIGMOID/RELU, x otherwise. */
int tx_unary_bwd(tx_ctx *ctx, int op, const float *d_src, const float *d_dy, float *d_dx,
                 int64_t n, float a, float b, int accumulate);

enum {
  TX_BIN_ADD = 0, TX_BIN_SUB = 1, TX_BIN_MUL = 2, TX_BIN_DIV = 3, TX_BIN_MIN = 4,
  TX_BIN_MAX = 5, TX_BIN_LE = 6, /* 1.0f where a<=b else 0 */
  TX_BIN_GE = 7, TX_BIN_POW = 8
};
#define TX_MAX_DIMS 8
/* out[i] = a[i] op b[i] with numpy broadcasting expressed as element strides
 * (0 on broadcast axes) over the output shape. */
int tx_binary(tx_ctx *ctx, int op, const float *d_a, const int64_t *a_strides,
              const float *d_b, const int64_t *b_strides, float *d_out,
              const int64_t *out_shape, int ndim);
/* Sum (mean when `mean`) of x over every axis where out_shape[i]==1 and
 * in_shape[i]>1 (out has the same rank; broadcast-gradient reduction). */
int tx_reduce_to(tx_ctx *ctx, const float *d_x, const int64_t *in_shape, float *d_out,
                 const int64_t *out_shape, int ndim, int mean, int accumulate);
/* Copy with arbitrary element strides (transpose / expand materialisation). */
int tx_strided_copy(tx_ctx *ctx, const void *d_src, const int64_t *src_strides, void *d_dst,
                    const int64_t *shape, int ndim, int elem_bytes);
/* Training-mode dropout: mask[i] = 0 with probability p, else 1 / (1 - p),
 * y = x * mask, drawn from a counter-based stream keyed by `seed` and the
 * device counter *d_counter, which the call advances (so a replayed CUDA graph
 * draws a new mask each time); d_counter = NULL uses the context's own counter
 * (zero when the context is created).  replaces: the Dropout of the capture IR
 * (crates/tynx-capture/src/lib.rs, UnaryOp::Dropout). */
int tx_dropout_fwd(tx_ctx *ctx, const float *d_x, float *d_y, float *d_mask, int64_t n, float p, uint64_t seed,
                   uint64_t *d_counter);
/* dst[dst_strides] (+)= src (contiguous over `shape`): the gradient of a
 * strided view (slicing), Concat's slabs. */
int tx_strided_scatter(tx_ctx *ctx, const float *d_src, float *d_dst, const int64_t *dst_strides,
                       const int64_t *shape, int ndim, int accumulate);

/* Softmax / log-softmax over the last axis of a [rows, cols] view.
 * replaces: softmax / log_softmax (crates/tynx/src/interpreter/softmax.rs:9-17,
 * tensor.rs:2234-2242) and their Burn backward rules. */
int tx_softmax_fwd(tx_ctx *ctx, const float *d_x, float *d_y, int64_t rows, int64_t cols, int log);
int tx_softmax_bwd(tx_ctx *ctx, const float *d_y, const float *d_dy, float *d_dx,
                   int64_t rows, int64_t cols, int log, int accumulate);

/* Fused softmax cross-entropy: loss = -mean_r log_softmax(z)[r, y_r] and
 * (when d_dlogits is non-null) dlogits = scale * (softmax(z) - onehot(y)) / rows,
 * where scale is read from the device scalar d_scale (null = 1).
 * Labels outside [0, cols) raise the device error flag (TX_ERR_INDEX).
 * replaces: nn.functional.cross_entropy (crates/tynx-python/python/tynx/nn/functional.py:133-145)
 * = log_softmax -> gather -> squeeze -> neg -> mean and its taped backward. */
int tx_softmax_xent_fwd(tx_ctx *ctx, const float *d_logits, const int64_t *d_labels,
                        int64_t rows, int64_t cols, float *d_loss);
int tx_softmax_xent_bwd(tx_ctx *ctx, const float *d_logits, const int64_t *d_labels,
                        int64_t rows, int64_t cols, const float *d_scale, float *d_dlogits,
                        int accumulate);
/* Same result as tx_softmax_xent_fwd, for callers that cannot allocate device
 * memory: a host runtime that reserves all of the GPU's memory for its own
 * allocator and lends libraries only the buffers it passes in, or a
 * latency-bound loop that cannot afford the device-wide synchronisation a
 * cudaMalloc or cudaFree implies.  It has no counterpart in the reference.
 * The per-row losses go to a fixed 1 MiB device array built into the library
 * (held on every GPU that loads it until the process exits), so rows must be
 * at most 262144; larger inputs fail with TX_ERR_SHAPE.  Nothing is allocated:
 * the first call on a device looks up that array's device address (make that
 * first call before any stream capture).  All calls share the array, so calls
 * whose work overlaps on the GPU (other streams, other host threads) race; calls
 * issued in order on one context's stream do not. */
int tx_softmax_xent_fwd_noalloc(tx_ctx *ctx, const float *d_logits, const int64_t *d_labels,
                                int64_t rows, int64_t cols, float *d_loss);

/* LayerNormalization over the trailing `cols` elements of each row.
 * replaces: layer_normalization_values (crates/tynx/src/interpreter/normalization.rs:135-190). */
int tx_layernorm_fwd(tx_ctx *ctx, const float *d_x, const float *d_gamma, const float *d_beta,
                     float *d_y, float *d_mean, float *d_rstd, int64_t rows, int64_t cols,
                     float eps);
int tx_layernorm_bwd(tx_ctx *ctx, const float *d_x, const float *d_gamma, const float *d_mean,
                     const float *d_rstd, const float *d_dy, float *d_dx, float *d_dgamma,
                     float *d_dbeta, int64_t rows, int64_t cols, int accumulate_dx,
                     int accumulate_params);

/* BatchNormalization with its running statistics fixed (the only training
 * form the reference accepts: one output, mean / var are buffers):
 * y = ((x - mean) / sqrt(var + eps)) * scale + bias over x viewed as
 * [N][C][L] (L = product of the spatial dims, 1 for rank 2).  The backward
 * writes dx = (dy * scale) / sqrt(var + eps) (when d_dx is non-null) and the
 * affine gradients dscale = sum dy * xhat, dbias = sum dy over N and L (when
 * non-null; both or neither).
 * replaces: execute_batch_normalization
 * (crates/tynx-train/src/imported_model/executor.rs:371-448), batch_normalization
 * (crates/tynx/src/interpreter/normalization.rs:20-58) and their Burn backward. */
int tx_batchnorm_fwd(tx_ctx *ctx, const float *d_x, const float *d_scale, const float *d_bias,
                     const float *d_mean, const float *d_var, float *d_y, int64_t N, int64_t C,
                     int64_t L, float eps);
int tx_batchnorm_bwd(tx_ctx *ctx, const float *d_x, const float *d_dy, const float *d_scale,
                     const float *d_mean, const float *d_var, float *d_dx, float *d_dscale,
                     float *d_dbias, int64_t N, int64_t C, int64_t L, float eps, int accumulate_dx,
                     int accumulate_params);
/* GroupNormalization over x viewed as [N][groups][C / groups][L], per-channel
 * scale and bias [C]; InstanceNormalization is groups == C.  The forward saves
 * each (n, group) row's mean and sqrt(var + eps) (d_mean, d_sdev: N * groups).
 * replaces: group_normalization_values / instance_normalization_values
 * (crates/tynx/src/interpreter/normalization.rs:73-106, 213-273) and their Burn
 * backward. */
int tx_groupnorm_fwd(tx_ctx *ctx, const float *d_x, const float *d_scale, const float *d_bias,
                     float *d_y, float *d_mean, float *d_sdev, int64_t N, int64_t C, int64_t L,
                     int64_t groups, float eps);
int tx_groupnorm_bwd(tx_ctx *ctx, const float *d_x, const float *d_dy, const float *d_scale,
                     const float *d_mean, const float *d_sdev, float *d_dx, float *d_dscale,
                     float *d_dbias, int64_t N, int64_t C, int64_t L, int64_t groups,
                     int accumulate_dx, int accumulate_params);
/* PRelu y = x >= 0 ? x : slope * x with slope broadcast to `shape` through
 * slope_strides (0 on broadcast axes).  The backward writes dx (when non-null)
 * and, into d_dslope_full (shape `shape`, when non-null), dy * x where x < 0,
 * which the caller sums down to the slope's shape.
 * replaces: DynTensor::prelu (crates/tynx/src/tensor.rs:1911-1934). */
int tx_prelu_fwd(tx_ctx *ctx, const float *d_x, const float *d_slope, const int64_t *slope_strides,
                 float *d_y, const int64_t *shape, int ndim);
int tx_prelu_bwd(tx_ctx *ctx, const float *d_x, const float *d_slope, const int64_t *slope_strides,
                 const float *d_dy, float *d_dx, float *d_dslope_full, const int64_t *shape, int ndim,
                 int accumulate_dx);
/* 2-D max pooling over `planes` (= N * C) planes of H x W; geom = {kh, kw,
 * sh, sw, pad_top, pad_left, dil_h, dil_w, out_h, out_w}.  Taps outside the
 * input count as -inf.  d_argmax (int32, one per output) records the chosen
 * tap (h * W + w; the first maximal one in window order); the backward routes
 * each output gradient there, summing in a fixed order.
 * replaces: max_pool2d (crates/tynx/src/interpreter/pooling.rs:360-426) and Burn's
 * max_pool2d backward. */
int tx_maxpool2d_fwd(tx_ctx *ctx, const float *d_x, float *d_y, int32_t *d_argmax, int64_t planes,
                     int64_t H, int64_t W, const int64_t *geom);
int tx_maxpool2d_bwd(tx_ctx *ctx, const float *d_dy, const int32_t *d_argmax, float *d_dx,
                     int64_t planes, int64_t H, int64_t W, const int64_t *geom, int accumulate);
/* ONNX AveragePool over [planes][H][W]: geom as tx_maxpool2d_fwd followed by
 * the bottom and right padding; the divisor counts the taps inside the input,
 * or with count_include_pad inside the padded input.  replaces: the
 * AveragePool arm of crates/tynx/src/interpreter/pooling.rs. */
int tx_avgpool2d_fwd(tx_ctx *ctx, const float *d_x, float *d_y, int64_t planes, int64_t H, int64_t W,
                     const int64_t *geom, int count_include_pad);
int tx_avgpool2d_bwd(tx_ctx *ctx, const float *d_dy, float *d_dx, int64_t planes, int64_t H, int64_t W,
                     const int64_t *geom, int count_include_pad, int accumulate);

/* Fused multi-head attention over the merged layout: q, k, v, out (and dout,
 * dq, dk, dv) are [batch * seq, ld] row-major with head h in columns
 * h * head_dim .. h * head_dim + head_dim - 1.  out = softmax(scale * q k^T) v
 * per (sequence, head); the backward writes dq, dk, dv (flags bit 1:
 * accumulate into them; bit 2: store them rounded to TF32).  Forward flags:
 * bit 0 the inputs already hold TF32 values (else they are rounded to nearest
 * on chip), bit 1 store out rounded to TF32.  head_dim 64, seq 1..128; TF32
 * tensor-core products, fp32 softmax.  One CTA per (sequence, head): no
 * score, probability or head-split tensor is written to device memory.
 * replaces: the attention block of an imported graph (MatMul
 * crates/tynx/src/interpreter/matrix.rs:238-255, Softmax softmax.rs:9-17 and
 * the Reshape / Transpose head split and merge, shape.rs:118-152) and its
 * Burn backward. */
int tx_attention_fwd(tx_ctx *ctx, const float *d_q, const float *d_k, const float *d_v, int64_t ld_in,
                     float *d_out, int64_t ld_out, int64_t batch, int64_t seq, int64_t heads,
                     int64_t head_dim, float scale, int flags);
int tx_attention_bwd(tx_ctx *ctx, const float *d_q, const float *d_k, const float *d_v, int64_t ld_in,
                     const float *d_dout, int64_t ld_dout, float *d_dq, float *d_dk, float *d_dv,
                     int64_t ld_grad, int64_t batch, int64_t seq, int64_t heads, int64_t head_dim,
                     float scale, int flags);

/* Clipped-surrogate PPO objective over [rows, cols] policy logits (cols <=
 * 64), per-row value estimates, int64 actions, behaviour log-probabilities,
 * advantages and returns:
 *   loss = -mean(min(r A, clamp(r, 1 - clip, 1 + clip) A))
 *          + value_coef * mean((value - ret)^2) - entropy_coef * mean(entropy)
 * with r = exp(log_softmax(logits)[action] - old_log_prob) and the entropy of
 * the row's categorical distribution.  The backward writes d logits and (when
 * d_dvalues is non-null) d values, scaled by the upstream gradient *d_dloss.
 * Out-of-range actions raise the device index flag.
 * replaces: the composed objective of crates/tynx-python/tests/test_ppo.py:53-64
 * (Categorical, crates/tynx-python/python/tynx/distributions.py:47-104; mse_loss,
 * crates/tynx-python/python/tynx/nn/functional.py:126-130), about twenty taped ops. */
int tx_ppo_loss_fwd(tx_ctx *ctx, const float *d_logits, int64_t rows, int64_t cols, const float *d_values,
                    const int64_t *d_actions, const float *d_old_log_prob, const float *d_advantages,
                    const float *d_returns, float clip, float value_coef, float entropy_coef, float *d_loss);
int tx_ppo_loss_bwd(tx_ctx *ctx, const float *d_logits, int64_t rows, int64_t cols, const float *d_values,
                    const int64_t *d_actions, const float *d_old_log_prob, const float *d_advantages,
                    const float *d_returns, float clip, float value_coef, float entropy_coef,
                    const float *d_dloss, float *d_dlogits, float *d_dvalues, int accumulate_logits,
                    int accumulate_values);

/* Row gather out[i, :] = table[idx[i], :] (negative indices wrap once) and its
 * backward scatter-add.  replaces: gather_values (crates/tynx/src/interpreter/gather.rs:18-58),
 * DynTensor::select (tensor.rs:1450) and Burn select_assign. */
int tx_gather_rows(tx_ctx *ctx, const float *d_table, int64_t rows, int64_t width,
                   const int64_t *d_idx, int64_t n_idx, float *d_out);
int tx_scatter_add_rows(tx_ctx *ctx, float *d_table, int64_t rows, int64_t width,
                        const int64_t *d_idx, int64_t n_idx, const float *d_src);
/* out[r] = x[r, idx[r]] for a [rows, cols] x (Tensor.gather on the last axis,
 * crates/tynx-python/src/tensor.rs:1769) and its backward. */
int tx_take_last(tx_ctx *ctx, const float *d_x, const int64_t *d_idx, float *d_out,
                 int64_t rows, int64_t cols);
int tx_take_last_bwd(tx_ctx *ctx, const int64_t *d_idx, const float *d_dout, float *d_dx,
                     int64_t rows, int64_t cols, int accumulate);

/* Column sum db[n] (+)= sum_m dy[m, n] (bias gradient, Gemm `dC = sum_rows dY * beta`). */
int tx_bias_grad(tx_ctx *ctx, const float *d_dy, float *d_db, int64_t M, int64_t N, float scale,
                 int accumulate);

/* =========================================================================
 * Optimizers (replaces AdamEngine::step_parameters,
 * crates/tynx-train/src/optimizer/adam.rs:431-527; Sgd::step_parameters,
 * crates/tynx-train/src/optimizer.rs:310-356).  One multi-tensor launch per
 * step; per-tensor step counters live on the device so a captured step
 * replays with correct bias corrections.
 * ========================================================================= */
typedef struct tx_optim_cfg {
  int32_t kind;        /* 0 = Adam (coupled L2), 1 = AdamW (decoupled), 2 = SGD */
  double lr, beta1, beta2, eps, weight_decay;
  int32_t amsgrad;
  double momentum, dampening; int32_t nesterov; /* SGD */
} tx_optim_cfg;
int tx_optim_create(tx_ctx *ctx, const tx_optim_cfg *cfg, int n_tensors, float *const *d_values,
                    float *const *d_grads, const int64_t *numel, tx_optim **out);
int tx_optim_set_lr(tx_optim *opt, double lr);
int tx_optim_set_hparams(tx_optim *opt, const tx_optim_cfg *cfg);
/* One step over the tensors whose active[i] != 0 (tensors without a gradient
 * are skipped, adam.rs:439-441). */
int tx_optim_step(tx_optim *opt, const uint8_t *active);
/* Read or write per-tensor state: which = 0 m, 1 v, 2 vmax, 3 momentum. */
int tx_optim_state_ptr(tx_optim *opt, int tensor, int which, float **d_out);
int tx_optim_get_steps(tx_optim *opt, int64_t *h_steps);
int tx_optim_set_steps(tx_optim *opt, const int64_t *h_steps);
int tx_optim_destroy(tx_optim *opt);

/* =========================================================================
 * Imported-graph engine (replaces ImportedModel::run_with_tracking /
 * executor::run, crates/tynx-train/src/imported_model.rs:109-113,
 * imported_model/executor.rs:107-161, the Burn autodiff tape walked by
 * backward_parameters, crates/tynx-train/src/autograd.rs:56-95, and
 * ParameterSlot value/grad storage, crates/tynx-train/src/parameter.rs:88-333).
 * ========================================================================= */
enum {
  TX_OP_GEMM = 1, TX_OP_MATMUL, TX_OP_CONV, TX_OP_GATHER, TX_OP_LAYERNORM, TX_OP_ADD,
  TX_OP_SUB, TX_OP_MUL, TX_OP_DIV, TX_OP_RELU, TX_OP_TANH, TX_OP_GELU, TX_OP_SIGMOID,
  TX_OP_EXP, TX_OP_LOG, TX_OP_NEG, TX_OP_SOFTMAX, TX_OP_LOGSOFTMAX, TX_OP_REDUCEMEAN,
  TX_OP_REDUCESUM, TX_OP_GAP, TX_OP_RESHAPE, TX_OP_TRANSPOSE, TX_OP_FLATTEN,
  TX_OP_SQUEEZE, TX_OP_UNSQUEEZE, TX_OP_IDENTITY, TX_OP_CLIP, TX_OP_PRELU,
  TX_OP_BATCHNORM, TX_OP_GROUPNORM, TX_OP_MAXPOOL,
  /* iattr[0] a TX_UN_* code, fattr[0..1] its a, b: Sqrt, Abs, Reciprocal, Erf,
   * LeakyRelu, Softplus, Elu, HardSigmoid, Softsign, Pow by a constant */
  TX_OP_UNARY,
  /* iattr[0] TX_BIN_MAX / MIN / POW, broadcasting (Max, Min, Pow) */
  TX_OP_BINARY,
  TX_OP_CONCAT,     /* iattr[0] axis; up to 6 inputs */
  TX_OP_SLICE,      /* ints: n_axes, axes[n], starts[n], ends[n], steps[n] (n <= 3) */
  TX_OP_SPLIT,      /* iattr[0] axis; ints: the outputs' sizes (up to 3 outputs) */
  TX_OP_EXPAND,     /* ints: the target shape (numpy broadcasting) */
  TX_OP_AVGPOOL,    /* as TX_OP_MAXPOOL; iattr[2] count_include_pad */
  TX_OP_REDUCEMAX,  /* ints: axes (none: all); iattr[0] keepdims; inference only */
  TX_OP_REDUCEMIN
};
enum { TX_VAL_INPUT = 0, TX_VAL_PARAM = 1, TX_VAL_CONST = 2, TX_VAL_ACT = 3 };
enum { TX_DT_F32 = 0, TX_DT_I64 = 1 };
typedef struct tx_value_desc {
  int32_t kind;       /* TX_VAL_* */
  int32_t dtype;      /* TX_DT_* */
  int32_t ndim;       /* for PARAM/CONST: static rank; INPUT: -1 if unknown */
  int64_t shape[TX_MAX_DIMS];
  const void *h_data; /* PARAM/CONST initial contents (host), else NULL */
} tx_value_desc;
typedef struct tx_node_desc {
  int32_t op;                /* TX_OP_* */
  int32_t n_in, n_out;
  int32_t in[6], out[3];     /* value ids; -1 for an absent optional input */
  int64_t iattr[8];          /* op-specific integers */
  double fattr[4];           /* op-specific reals */
  int32_t n_ints; int64_t ints[16]; /* list attributes (perm, pads, strides, axes, shape) */
} tx_node_desc;
int tx_graph_create(tx_ctx *ctx, const tx_value_desc *values, int n_values,
                    const tx_node_desc *nodes, int n_nodes, const int32_t *outputs,
                    int n_outputs, tx_graph **out);
int tx_graph_destroy(tx_graph *g);
/* Parameter slots in value-id order of TX_VAL_PARAM entries. */
int tx_graph_param_count(tx_graph *g, int *out);
int tx_graph_param(tx_graph *g, int index, int32_t *value_id, float **d_value, float **d_grad,
                   int64_t *numel);
/* Device storage of a parameter or constant value (the BatchNorm running
 * statistics are constants the forward reads from here: writing them changes
 * the next forward, as ImportedModel buffers do in the reference). */
int tx_graph_value_ptr(tx_graph *g, int value_id, void **d_out);
int tx_graph_grad_defined(tx_graph *g, int index, int *out);
int tx_graph_set_grad_defined(tx_graph *g, int index, int defined);
/* Shape inference for given input shapes; fills output ranks and shapes. */
int tx_graph_infer(tx_graph *g, const int64_t *in_shapes, const int32_t *in_ndims,
                   int64_t *out_shapes, int32_t *out_ndims);
/* Forward.  Writes outputs into caller-provided buffers.  With tracking, a
 * record holding the saved activations is returned for backward. */
int tx_graph_forward(tx_graph *g, const void *const *d_inputs, const int64_t *in_shapes,
                     const int32_t *in_ndims, void *const *d_outputs, int tracking,
                     tx_record **rec_out);
/* Backward through one record: d_outputs[i] may be NULL (zero gradient).
 * Parameter gradients accumulate into the slots (grad += new, or = new when
 * the slot has no gradient yet, parameter.rs:300-333).  d_inputs[i] non-NULL
 * requests the input gradient (written, not accumulated). */
int tx_graph_backward(tx_graph *g, tx_record *rec, const float *const *d_outputs,
                      float *const *d_inputs);
int tx_record_free(tx_record *rec);

/* =========================================================================
 * Data parallelism over NCCL (no counterpart in the reference, which is
 * single-device; §e of the engine design).  One process per GPU.
 * ========================================================================= */
int tx_dp_unique_id(uint8_t *out128);
int tx_dp_init(tx_ctx *ctx, int world, int rank, const uint8_t *id128, uint64_t timeout_ms);
int tx_dp_destroy(tx_ctx *ctx);
/* Average every parameter gradient of g across ranks inside backward, in
 * buckets of about bucket_bytes on the communication stream, overlapped with
 * the remaining backward.  0 disables. */
int tx_graph_set_dp(tx_graph *g, int enabled, int64_t bucket_bytes);
int tx_dp_allreduce(tx_ctx *ctx, float *d_buf, int64_t n, int average);

#ifdef __cplusplus
}
#endif
#endif /* TYNX_CUDA_H */
