//! Raw bindings to `libtynx_cuda.so`, the B200 (sm_100a) training-step
//! engine for imported ONNX graphs: one `extern "C"` declaration per function
//! of `include/tynx_cuda.h`, the structs it passes by pointer, and its enum
//! constants.  This crate is the only place in the workspace that allows
//! `unsafe`; the engine behind `Device::Cuda` wraps it in owned handles
//! (`Drop` -> `tx_ctx_destroy` / `tx_graph_destroy` / `tx_free`) and turns
//! status codes into `TynxError` (`TX_ERR_SHAPE` -> `Shape`, `TX_ERR_INDEX` ->
//! index errors, `TX_ERR_TIMEOUT` -> `DeviceSynchronization`, others ->
//! `AsynchronousDevice`, crates/tynx/src/error.rs:54-59).
//!
//! Call sites in the reference that switch to these functions:
//! `executor::run` (crates/tynx-train/src/imported_model/executor.rs:107-161) ->
//! `tx_graph_forward`; `backward_parameters` (crates/tynx-train/src/autograd.rs:56-95)
//! -> `tx_graph_backward`; `AdamEngine::step_parameters`
//! (crates/tynx-train/src/optimizer/adam.rs:431-527) -> `tx_optim_step`;
//! `Graph::run_values` (crates/tynx-capture/src/lib.rs:747-882) -> `tx_exec_launch`;
//! `PyDevice::py_new` (crates/tynx-python/src/device.rs:50-61) -> `tx_ctx_create`.
//!
//! The declarations are checked against the header by the repository's host
//! tests (every header function appears here with the same parameter count).
#![allow(non_camel_case_types, non_snake_case)]
#![no_std]

use core::ffi::{c_char, c_int, c_void};

pub const TYNX_CUDA_ABI_VERSION: c_int = 2;
pub const TX_MAX_DIMS: usize = 8;

pub const TX_OK: c_int = 0;
pub const TX_ERR_INVALID: c_int = 1;
pub const TX_ERR_SHAPE: c_int = 2;
pub const TX_ERR_INDEX: c_int = 3;
pub const TX_ERR_OOM: c_int = 4;
pub const TX_ERR_CUDA: c_int = 5;
pub const TX_ERR_TIMEOUT: c_int = 6;
pub const TX_ERR_UNSUPPORTED: c_int = 7;
pub const TX_ERR_DEVICE: c_int = 8;
pub const TX_ERR_NCCL: c_int = 9;
pub const TX_ERR_CAPTURE: c_int = 10;
pub const TX_MATH_TF32: c_int = 0;
pub const TX_MATH_3XTF32: c_int = 1;
pub const TX_MATH_FP32: c_int = 2;
pub const TX_MATH_TF32_TRUNC: c_int = 3;
pub const TX_ACT_NONE: c_int = 0;
pub const TX_ACT_RELU: c_int = 1;
pub const TX_ACT_TANH: c_int = 2;
pub const TX_ACT_GELU: c_int = 3;
pub const TX_GEMM_A_TF32: c_int = 1;
pub const TX_GEMM_B_TF32: c_int = 2;
pub const TX_GEMM_ROUND_OUT: c_int = 4;
pub const TX_GEMM_EXACT: c_int = 8;
pub const TX_GEMM_A_SHARED: c_int = 16;
pub const TX_UN_NEG: c_int = 0;
pub const TX_UN_EXP: c_int = 1;
pub const TX_UN_LOG: c_int = 2;
pub const TX_UN_RELU: c_int = 3;
pub const TX_UN_TANH: c_int = 4;
pub const TX_UN_GELU: c_int = 5;
pub const TX_UN_SIGMOID: c_int = 6;
pub const TX_UN_CLAMP: c_int = 7;
pub const TX_UN_SQRT: c_int = 8;
pub const TX_UN_ABS: c_int = 9;
pub const TX_UN_SCALE: c_int = 10;
pub const TX_UN_POW: c_int = 11;
pub const TX_UN_ERF: c_int = 12;
pub const TX_UN_LEAKYRELU: c_int = 13;
pub const TX_UN_SOFTPLUS: c_int = 14;
pub const TX_UN_ELU: c_int = 15;
pub const TX_UN_HARDSIGMOID: c_int = 16;
pub const TX_UN_SOFTSIGN: c_int = 17;
pub const TX_UN_RECIPROCAL: c_int = 18;
pub const TX_BIN_ADD: c_int = 0;
pub const TX_BIN_SUB: c_int = 1;
pub const TX_BIN_MUL: c_int = 2;
pub const TX_BIN_DIV: c_int = 3;
pub const TX_BIN_MIN: c_int = 4;
pub const TX_BIN_MAX: c_int = 5;
pub const TX_BIN_LE: c_int = 6;
pub const TX_BIN_GE: c_int = 7;
pub const TX_BIN_POW: c_int = 8;
pub const TX_OP_GEMM: c_int = 1;
pub const TX_OP_MATMUL: c_int = 2;
pub const TX_OP_CONV: c_int = 3;
pub const TX_OP_GATHER: c_int = 4;
pub const TX_OP_LAYERNORM: c_int = 5;
pub const TX_OP_ADD: c_int = 6;
pub const TX_OP_SUB: c_int = 7;
pub const TX_OP_MUL: c_int = 8;
pub const TX_OP_DIV: c_int = 9;
pub const TX_OP_RELU: c_int = 10;
pub const TX_OP_TANH: c_int = 11;
pub const TX_OP_GELU: c_int = 12;
pub const TX_OP_SIGMOID: c_int = 13;
pub const TX_OP_EXP: c_int = 14;
pub const TX_OP_LOG: c_int = 15;
pub const TX_OP_NEG: c_int = 16;
pub const TX_OP_SOFTMAX: c_int = 17;
pub const TX_OP_LOGSOFTMAX: c_int = 18;
pub const TX_OP_REDUCEMEAN: c_int = 19;
pub const TX_OP_REDUCESUM: c_int = 20;
pub const TX_OP_GAP: c_int = 21;
pub const TX_OP_RESHAPE: c_int = 22;
pub const TX_OP_TRANSPOSE: c_int = 23;
pub const TX_OP_FLATTEN: c_int = 24;
pub const TX_OP_SQUEEZE: c_int = 25;
pub const TX_OP_UNSQUEEZE: c_int = 26;
pub const TX_OP_IDENTITY: c_int = 27;
pub const TX_OP_CLIP: c_int = 28;
pub const TX_OP_PRELU: c_int = 29;
pub const TX_OP_BATCHNORM: c_int = 30;
pub const TX_OP_GROUPNORM: c_int = 31;
pub const TX_OP_MAXPOOL: c_int = 32;
pub const TX_OP_UNARY: c_int = 33;
pub const TX_OP_BINARY: c_int = 34;
pub const TX_OP_CONCAT: c_int = 35;
pub const TX_OP_SLICE: c_int = 36;
pub const TX_OP_SPLIT: c_int = 37;
pub const TX_OP_EXPAND: c_int = 38;
pub const TX_OP_AVGPOOL: c_int = 39;
pub const TX_OP_REDUCEMAX: c_int = 40;
pub const TX_OP_REDUCEMIN: c_int = 41;
pub const TX_VAL_INPUT: c_int = 0;
pub const TX_VAL_PARAM: c_int = 1;
pub const TX_VAL_CONST: c_int = 2;
pub const TX_VAL_ACT: c_int = 3;
pub const TX_DT_F32: c_int = 0;
pub const TX_DT_I64: c_int = 1;

#[repr(C)]
pub struct tx_ctx {
    _opaque: [u8; 0],
}
#[repr(C)]
pub struct tx_graph {
    _opaque: [u8; 0],
}
#[repr(C)]
pub struct tx_record {
    _opaque: [u8; 0],
}
#[repr(C)]
pub struct tx_exec {
    _opaque: [u8; 0],
}
#[repr(C)]
pub struct tx_optim {
    _opaque: [u8; 0],
}
#[repr(C)]
pub struct tx_prefetch {
    _opaque: [u8; 0],
}

#[repr(C)]
#[derive(Clone, Copy)]
pub struct tx_gemm_desc {
    pub M: i64,
    pub N: i64,
    pub K: i64,
    pub A: *const f32,
    pub lda: i64,
    pub trans_a: i32,
    pub B: *const f32,
    pub ldb: i64,
    pub trans_b: i32,
    pub C: *mut f32,
    pub ldc: i64,
    pub alpha: f32,
    pub beta: f32,
    pub bias: *const f32,
    pub bias_scale: f32,
    pub act: i32,
    pub preact: *mut f32,
    pub ld_preact: i64,
    pub dact_src: *const f32,
    pub ld_dact: i64,
    pub dact: i32,
    pub batch: i64,
    pub stride_a: i64,
    pub stride_b: i64,
    pub stride_c: i64,
    pub flags: i32,
    pub colsum: *mut f32,
    pub colsum_scale: f32,
    pub colsum_acc: i32,
    pub B_lo: *const f32,
}

#[repr(C)]
#[derive(Clone, Copy)]
pub struct tx_optim_cfg {
    pub kind: i32,
    pub lr: f64,
    pub beta1: f64,
    pub beta2: f64,
    pub eps: f64,
    pub weight_decay: f64,
    pub amsgrad: i32,
    pub momentum: f64,
    pub dampening: f64,
    pub nesterov: i32,
}

#[repr(C)]
#[derive(Clone, Copy)]
pub struct tx_value_desc {
    pub kind: i32,
    pub dtype: i32,
    pub ndim: i32,
    pub shape: [i64; TX_MAX_DIMS],
    pub h_data: *const c_void,
}

#[repr(C)]
#[derive(Clone, Copy)]
pub struct tx_node_desc {
    pub op: i32,
    pub n_in: i32,
    pub n_out: i32,
    pub inp: [i32; 6],
    pub out: [i32; 3],
    pub iattr: [i64; 8],
    pub fattr: [f64; 4],
    pub n_ints: i32,
    pub ints: [i64; 16],
}

#[link(name = "tynx_cuda")]
extern "C" {
    pub fn tx_abi_version() -> c_int;
    pub fn tx_device_count(out: *mut c_int) -> c_int;
    pub fn tx_ctx_create(device: c_int, math_mode: c_int, out: *mut *mut tx_ctx) -> c_int;
    pub fn tx_ctx_destroy(ctx: *mut tx_ctx) -> c_int;
    pub fn tx_ctx_set_math(ctx: *mut tx_ctx, math_mode: c_int) -> c_int;
    pub fn tx_ctx_get_math(ctx: *mut tx_ctx, out: *mut c_int) -> c_int;
    pub fn tx_last_error(ctx: *mut tx_ctx, buf: *mut c_char, n: usize) -> c_int;
    pub fn tx_sync(ctx: *mut tx_ctx, timeout_ms: u64) -> c_int;
    pub fn tx_stream(ctx: *mut tx_ctx, out: *mut *mut c_void) -> c_int;
    pub fn tx_alloc(ctx: *mut tx_ctx, bytes: usize, d_out: *mut *mut c_void) -> c_int;
    pub fn tx_free(ctx: *mut tx_ctx, d_ptr: *mut c_void) -> c_int;
    pub fn tx_h2d(ctx: *mut tx_ctx, d_dst: *mut c_void, h_src: *const c_void, bytes: usize) -> c_int;
    pub fn tx_d2h(ctx: *mut tx_ctx, h_dst: *mut c_void, d_src: *const c_void, bytes: usize) -> c_int;
    pub fn tx_d2d(ctx: *mut tx_ctx, d_dst: *mut c_void, d_src: *const c_void, bytes: usize) -> c_int;
    pub fn tx_memset(ctx: *mut tx_ctx, d_ptr: *mut c_void, value: c_int, bytes: usize) -> c_int;
    pub fn tx_fill_f32(ctx: *mut tx_ctx, d_ptr: *mut f32, n: i64, value: f32) -> c_int;
    pub fn tx_host_alloc(bytes: usize, h_out: *mut *mut c_void) -> c_int;
    pub fn tx_prefetch_create(ctx: *mut tx_ctx, bytes: usize, depth: c_int, out: *mut *mut tx_prefetch) -> c_int;
    pub fn tx_prefetch_put(p: *mut tx_prefetch, h_src: *const c_void, bytes: usize) -> c_int;
    pub fn tx_prefetch_get(p: *mut tx_prefetch, d_out: *mut *mut c_void) -> c_int;
    pub fn tx_prefetch_destroy(p: *mut tx_prefetch) -> c_int;
    pub fn tx_host_free(h_ptr: *mut c_void) -> c_int;
    pub fn tx_mem_stats(ctx: *mut tx_ctx, in_use: *mut u64, cached: *mut u64) -> c_int;
    pub fn tx_capture_begin(ctx: *mut tx_ctx) -> c_int;
    pub fn tx_capture_end(ctx: *mut tx_ctx, out: *mut *mut tx_exec) -> c_int;
    pub fn tx_capture_abort(ctx: *mut tx_ctx) -> c_int;
    pub fn tx_capture_active(ctx: *mut tx_ctx, out: *mut c_int) -> c_int;
    pub fn tx_exec_launch(exec: *mut tx_exec) -> c_int;
    pub fn tx_exec_destroy(exec: *mut tx_exec) -> c_int;
    pub fn tx_exec_node_count(exec: *mut tx_exec, kernels: *mut i64, total: *mut i64) -> c_int;
    pub fn tx_gemm(ctx: *mut tx_ctx, desc: *const tx_gemm_desc) -> c_int;
    pub fn tx_round_tf32(ctx: *mut tx_ctx, d_src: *const f32, d_dst: *mut f32, n: i64) -> c_int;
    pub fn tx_split_tf32(ctx: *mut tx_ctx, d_src: *const f32, d_hi: *mut f32, d_lo: *mut f32, n: i64) -> c_int;
    pub fn tx_unary(ctx: *mut tx_ctx, op: c_int, d_x: *const f32, d_y: *mut f32, n: i64, a: f32, b: f32) -> c_int;
    pub fn tx_unary_bwd(ctx: *mut tx_ctx, op: c_int, d_src: *const f32, d_dy: *const f32, d_dx: *mut f32, n: i64, a: f32, b: f32, accumulate: c_int) -> c_int;
    pub fn tx_binary(ctx: *mut tx_ctx, op: c_int, d_a: *const f32, a_strides: *const i64, d_b: *const f32, b_strides: *const i64, d_out: *mut f32, out_shape: *const i64, ndim: c_int) -> c_int;
    pub fn tx_reduce_to(ctx: *mut tx_ctx, d_x: *const f32, in_shape: *const i64, d_out: *mut f32, out_shape: *const i64, ndim: c_int, mean: c_int, accumulate: c_int) -> c_int;
    pub fn tx_strided_copy(ctx: *mut tx_ctx, d_src: *const c_void, src_strides: *const i64, d_dst: *mut c_void, shape: *const i64, ndim: c_int, elem_bytes: c_int) -> c_int;
    pub fn tx_dropout_fwd(ctx: *mut tx_ctx, d_x: *const f32, d_y: *mut f32, d_mask: *mut f32, n: i64, p: f32, seed: u64, d_counter: *mut u64) -> c_int;
    pub fn tx_strided_scatter(ctx: *mut tx_ctx, d_src: *const f32, d_dst: *mut f32, dst_strides: *const i64, shape: *const i64, ndim: c_int, accumulate: c_int) -> c_int;
    pub fn tx_softmax_fwd(ctx: *mut tx_ctx, d_x: *const f32, d_y: *mut f32, rows: i64, cols: i64, log: c_int) -> c_int;
    pub fn tx_softmax_bwd(ctx: *mut tx_ctx, d_y: *const f32, d_dy: *const f32, d_dx: *mut f32, rows: i64, cols: i64, log: c_int, accumulate: c_int) -> c_int;
    pub fn tx_softmax_xent_fwd(ctx: *mut tx_ctx, d_logits: *const f32, d_labels: *const i64, rows: i64, cols: i64, d_loss: *mut f32) -> c_int;
    pub fn tx_softmax_xent_bwd(ctx: *mut tx_ctx, d_logits: *const f32, d_labels: *const i64, rows: i64, cols: i64, d_scale: *const f32, d_dlogits: *mut f32, accumulate: c_int) -> c_int;
    pub fn tx_softmax_xent_fwd_noalloc(ctx: *mut tx_ctx, d_logits: *const f32, d_labels: *const i64, rows: i64, cols: i64, d_loss: *mut f32) -> c_int;
    pub fn tx_layernorm_fwd(ctx: *mut tx_ctx, d_x: *const f32, d_gamma: *const f32, d_beta: *const f32, d_y: *mut f32, d_mean: *mut f32, d_rstd: *mut f32, rows: i64, cols: i64, eps: f32) -> c_int;
    pub fn tx_layernorm_bwd(ctx: *mut tx_ctx, d_x: *const f32, d_gamma: *const f32, d_mean: *const f32, d_rstd: *const f32, d_dy: *const f32, d_dx: *mut f32, d_dgamma: *mut f32, d_dbeta: *mut f32, rows: i64, cols: i64, accumulate_dx: c_int, accumulate_params: c_int) -> c_int;
    pub fn tx_batchnorm_fwd(ctx: *mut tx_ctx, d_x: *const f32, d_scale: *const f32, d_bias: *const f32, d_mean: *const f32, d_var: *const f32, d_y: *mut f32, N: i64, C: i64, L: i64, eps: f32) -> c_int;
    pub fn tx_batchnorm_bwd(ctx: *mut tx_ctx, d_x: *const f32, d_dy: *const f32, d_scale: *const f32, d_mean: *const f32, d_var: *const f32, d_dx: *mut f32, d_dscale: *mut f32, d_dbias: *mut f32, N: i64, C: i64, L: i64, eps: f32, accumulate_dx: c_int, accumulate_params: c_int) -> c_int;
    pub fn tx_groupnorm_fwd(ctx: *mut tx_ctx, d_x: *const f32, d_scale: *const f32, d_bias: *const f32, d_y: *mut f32, d_mean: *mut f32, d_sdev: *mut f32, N: i64, C: i64, L: i64, groups: i64, eps: f32) -> c_int;
    pub fn tx_groupnorm_bwd(ctx: *mut tx_ctx, d_x: *const f32, d_dy: *const f32, d_scale: *const f32, d_mean: *const f32, d_sdev: *const f32, d_dx: *mut f32, d_dscale: *mut f32, d_dbias: *mut f32, N: i64, C: i64, L: i64, groups: i64, accumulate_dx: c_int, accumulate_params: c_int) -> c_int;
    pub fn tx_prelu_fwd(ctx: *mut tx_ctx, d_x: *const f32, d_slope: *const f32, slope_strides: *const i64, d_y: *mut f32, shape: *const i64, ndim: c_int) -> c_int;
    pub fn tx_prelu_bwd(ctx: *mut tx_ctx, d_x: *const f32, d_slope: *const f32, slope_strides: *const i64, d_dy: *const f32, d_dx: *mut f32, d_dslope_full: *mut f32, shape: *const i64, ndim: c_int, accumulate_dx: c_int) -> c_int;
    pub fn tx_maxpool2d_fwd(ctx: *mut tx_ctx, d_x: *const f32, d_y: *mut f32, d_argmax: *mut i32, planes: i64, H: i64, W: i64, geom: *const i64) -> c_int;
    pub fn tx_maxpool2d_bwd(ctx: *mut tx_ctx, d_dy: *const f32, d_argmax: *const i32, d_dx: *mut f32, planes: i64, H: i64, W: i64, geom: *const i64, accumulate: c_int) -> c_int;
    pub fn tx_avgpool2d_fwd(ctx: *mut tx_ctx, d_x: *const f32, d_y: *mut f32, planes: i64, H: i64, W: i64, geom: *const i64, count_include_pad: c_int) -> c_int;
    pub fn tx_avgpool2d_bwd(ctx: *mut tx_ctx, d_dy: *const f32, d_dx: *mut f32, planes: i64, H: i64, W: i64, geom: *const i64, count_include_pad: c_int, accumulate: c_int) -> c_int;
    pub fn tx_attention_fwd(ctx: *mut tx_ctx, d_q: *const f32, d_k: *const f32, d_v: *const f32, ld_in: i64, d_out: *mut f32, ld_out: i64, batch: i64, seq: i64, heads: i64, head_dim: i64, scale: f32, flags: c_int) -> c_int;
    pub fn tx_attention_bwd(ctx: *mut tx_ctx, d_q: *const f32, d_k: *const f32, d_v: *const f32, ld_in: i64, d_dout: *const f32, ld_dout: i64, d_dq: *mut f32, d_dk: *mut f32, d_dv: *mut f32, ld_grad: i64, batch: i64, seq: i64, heads: i64, head_dim: i64, scale: f32, flags: c_int) -> c_int;
    pub fn tx_ppo_loss_fwd(ctx: *mut tx_ctx, d_logits: *const f32, rows: i64, cols: i64, d_values: *const f32, d_actions: *const i64, d_old_log_prob: *const f32, d_advantages: *const f32, d_returns: *const f32, clip: f32, value_coef: f32, entropy_coef: f32, d_loss: *mut f32) -> c_int;
    pub fn tx_ppo_loss_bwd(ctx: *mut tx_ctx, d_logits: *const f32, rows: i64, cols: i64, d_values: *const f32, d_actions: *const i64, d_old_log_prob: *const f32, d_advantages: *const f32, d_returns: *const f32, clip: f32, value_coef: f32, entropy_coef: f32, d_dloss: *const f32, d_dlogits: *mut f32, d_dvalues: *mut f32, accumulate_logits: c_int, accumulate_values: c_int) -> c_int;
    pub fn tx_gather_rows(ctx: *mut tx_ctx, d_table: *const f32, rows: i64, width: i64, d_idx: *const i64, n_idx: i64, d_out: *mut f32) -> c_int;
    pub fn tx_scatter_add_rows(ctx: *mut tx_ctx, d_table: *mut f32, rows: i64, width: i64, d_idx: *const i64, n_idx: i64, d_src: *const f32) -> c_int;
    pub fn tx_take_last(ctx: *mut tx_ctx, d_x: *const f32, d_idx: *const i64, d_out: *mut f32, rows: i64, cols: i64) -> c_int;
    pub fn tx_take_last_bwd(ctx: *mut tx_ctx, d_idx: *const i64, d_dout: *const f32, d_dx: *mut f32, rows: i64, cols: i64, accumulate: c_int) -> c_int;
    pub fn tx_bias_grad(ctx: *mut tx_ctx, d_dy: *const f32, d_db: *mut f32, M: i64, N: i64, scale: f32, accumulate: c_int) -> c_int;
    pub fn tx_optim_create(ctx: *mut tx_ctx, cfg: *const tx_optim_cfg, n_tensors: c_int, d_values: *const *mut f32, d_grads: *const *mut f32, numel: *const i64, out: *mut *mut tx_optim) -> c_int;
    pub fn tx_optim_set_lr(opt: *mut tx_optim, lr: f64) -> c_int;
    pub fn tx_optim_set_hparams(opt: *mut tx_optim, cfg: *const tx_optim_cfg) -> c_int;
    pub fn tx_optim_step(opt: *mut tx_optim, active: *const u8) -> c_int;
    pub fn tx_optim_state_ptr(opt: *mut tx_optim, tensor: c_int, which: c_int, d_out: *mut *mut f32) -> c_int;
    pub fn tx_optim_get_steps(opt: *mut tx_optim, h_steps: *mut i64) -> c_int;
    pub fn tx_optim_set_steps(opt: *mut tx_optim, h_steps: *const i64) -> c_int;
    pub fn tx_optim_destroy(opt: *mut tx_optim) -> c_int;
    pub fn tx_graph_create(ctx: *mut tx_ctx, values: *const tx_value_desc, n_values: c_int, nodes: *const tx_node_desc, n_nodes: c_int, outputs: *const i32, n_outputs: c_int, out: *mut *mut tx_graph) -> c_int;
    pub fn tx_graph_destroy(g: *mut tx_graph) -> c_int;
    pub fn tx_graph_param_count(g: *mut tx_graph, out: *mut c_int) -> c_int;
    pub fn tx_graph_param(g: *mut tx_graph, index: c_int, value_id: *mut i32, d_value: *mut *mut f32, d_grad: *mut *mut f32, numel: *mut i64) -> c_int;
    pub fn tx_graph_value_ptr(g: *mut tx_graph, value_id: c_int, d_out: *mut *mut c_void) -> c_int;
    pub fn tx_graph_grad_defined(g: *mut tx_graph, index: c_int, out: *mut c_int) -> c_int;
    pub fn tx_graph_set_grad_defined(g: *mut tx_graph, index: c_int, defined: c_int) -> c_int;
    pub fn tx_graph_infer(g: *mut tx_graph, in_shapes: *const i64, in_ndims: *const i32, out_shapes: *mut i64, out_ndims: *mut i32) -> c_int;
    pub fn tx_graph_forward(g: *mut tx_graph, d_inputs: *const *const c_void, in_shapes: *const i64, in_ndims: *const i32, d_outputs: *const *mut c_void, tracking: c_int, rec_out: *mut *mut tx_record) -> c_int;
    pub fn tx_graph_backward(g: *mut tx_graph, rec: *mut tx_record, d_outputs: *const *const f32, d_inputs: *const *mut f32) -> c_int;
    pub fn tx_record_free(rec: *mut tx_record) -> c_int;
    pub fn tx_dp_unique_id(out128: *mut u8) -> c_int;
    pub fn tx_dp_init(ctx: *mut tx_ctx, world: c_int, rank: c_int, id128: *const u8, timeout_ms: u64) -> c_int;
    pub fn tx_dp_destroy(ctx: *mut tx_ctx) -> c_int;
    pub fn tx_graph_set_dp(g: *mut tx_graph, enabled: c_int, bucket_bytes: i64) -> c_int;
    pub fn tx_dp_allreduce(ctx: *mut tx_ctx, d_buf: *mut f32, n: i64, average: c_int) -> c_int;
}
