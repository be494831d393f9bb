// Bandwidth-bound kernels of the training step (sm_100a).
//
// Each kernel restates the arithmetic of the Burn operator the reference calls
// through DynTensor (crates/tynx/src/tensor.rs) so that results agree with the
// Flex CPU backend within fp32 rounding.  Rows are handled one warp per row with
// shuffle reductions; elementwise work is vectorised to 128-bit accesses where
// alignment allows; every reduction across blocks is two-phase (partials to a
// scratch buffer, then a fixed-order sum) so results are deterministic.
#include <math.h>

#include <initializer_list>
#include <mutex>

#include "common.h"
#include "epilogue.cuh"

namespace {

constexpr int kWarp = 32;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ void raise_flag(int *flag, int code, int a, int b) {
  if (atomicCAS(flag, 0, code) == 0) {
    flag[1] = a;
    flag[2] = b;
  }
}

// ---- activations (erf GELU as in crates/tynx/src/interpreter/unary.rs:234; the
// GEMM epilogues' form, so fused and standalone GELU give the same bits) --------
__device__ __forceinline__ float gelu_f(float x) { return tx_epi::gelu(x); }
__device__ __forceinline__ float gelu_grad(float x) { return tx_epi::gelu_grad(x); }

__device__ __forceinline__ float unary_f(int op, float x, float a, float b) {
  switch (op) {
    case TX_UN_NEG: return -x;
    case TX_UN_EXP: return expf(x);
    case TX_UN_LOG: return logf(x);
    case TX_UN_RELU: return x > 0.f ? x : 0.f;
    case TX_UN_TANH: return tanhf(x);
    case TX_UN_GELU: return gelu_f(x);
    case TX_UN_SIGMOID: return 1.0f / (1.0f + expf(-x));
    case TX_UN_CLAMP: return fminf(fmaxf(x, a), b);
    case TX_UN_SQRT: return sqrtf(x);
    case TX_UN_ABS: return fabsf(x);
    case TX_UN_SCALE: return a * x + b;
    case TX_UN_POW: return powf(x, a);
    case TX_UN_ERF: return erff(x);
    case TX_UN_LEAKYRELU: return x >= 0.f ? x : a * x;
    case TX_UN_SOFTPLUS: return x > 20.f ? x : log1pf(expf(x));  // ln(1 + e^x), e^x beyond fp32 past 20
    case TX_UN_ELU: return x > 0.f ? x : a * (expf(x) - 1.f);
    case TX_UN_HARDSIGMOID: return fminf(fmaxf(a * x + b, 0.f), 1.f);
    case TX_UN_SOFTSIGN: return x / (1.f + fabsf(x));
    case TX_UN_RECIPROCAL: return 1.f / x;
  }
  return x;
}

// derivative factor; `s` is the saved forward output for EXP/TANH/SIGMOID/RELU
// and the forward input otherwise
__device__ __forceinline__ float unary_grad(int op, float s, float a, float b) {
  switch (op) {
    case TX_UN_NEG: return -1.f;
    case TX_UN_EXP: return s;
    case TX_UN_LOG: return 1.0f / s;
    case TX_UN_RELU: return s > 0.f ? 1.f : 0.f;
    case TX_UN_TANH: return 1.f - s * s;
    case TX_UN_GELU: return gelu_grad(s);
    case TX_UN_SIGMOID: return s * (1.f - s);
    case TX_UN_CLAMP: return (s >= a && s <= b) ? 1.f : 0.f;
    case TX_UN_SQRT: return 0.5f / sqrtf(s);
    case TX_UN_ABS: return s > 0.f ? 1.f : (s < 0.f ? -1.f : 0.f);
    case TX_UN_SCALE: return a;
    case TX_UN_POW: return a * powf(s, a - 1.f);
    case TX_UN_ERF: return 1.1283791670955126f * expf(-s * s);  // 2 / sqrt(pi) e^(-x^2)
    case TX_UN_LEAKYRELU: return s >= 0.f ? 1.f : a;
    case TX_UN_SOFTPLUS: return 1.f / (1.f + expf(-s));
    case TX_UN_ELU: return s > 0.f ? 1.f : a * expf(s);
    case TX_UN_HARDSIGMOID: {
      const float t = a * s + b;
      return (t > 0.f && t < 1.f) ? a : 0.f;
    }
    case TX_UN_SOFTSIGN: {
      const float d = 1.f + fabsf(s);
      return 1.f / (d * d);
    }
    case TX_UN_RECIPROCAL: return -1.f / (s * s);
  }
  return 1.f;
}

__global__ void k_fill(float *y, int64_t n, float v) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    y[i] = v;
}

__global__ void k_unary(int op, const float *__restrict__ x, float *__restrict__ y, int64_t n,
                        float a, float b) {
  int64_t n4 = n >> 2;
  const float4 *x4 = reinterpret_cast<const float4 *>(x);
  float4 *y4 = reinterpret_cast<float4 *>(y);
  bool vec = ((((uintptr_t)x) | ((uintptr_t)y)) & 15) == 0;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t start = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (vec) {
    for (int64_t i = start; i < n4; i += stride) {
      float4 v = x4[i];
      v.x = unary_f(op, v.x, a, b);
      v.y = unary_f(op, v.y, a, b);
      v.z = unary_f(op, v.z, a, b);
      v.w = unary_f(op, v.w, a, b);
      y4[i] = v;
    }
    for (int64_t i = (n4 << 2) + start; i < n; i += stride) y[i] = unary_f(op, x[i], a, b);
  } else {
    for (int64_t i = start; i < n; i += stride) y[i] = unary_f(op, x[i], a, b);
  }
}

__global__ void k_unary_bwd(int op, const float *__restrict__ s, const float *__restrict__ dy,
                            float *__restrict__ dx, int64_t n, float a, float b, int acc) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float g = dy[i] * unary_grad(op, s[i], a, b);
    dx[i] = acc ? dx[i] + g : g;
  }
}





// Reduction of x (shape `in`) to `out` (same rank, 1 on reduced axes).
struct RDims {
  int64_t in[TX_MAX_DIMS];
  int64_t out[TX_MAX_DIMS];
  int64_t in_stride[TX_MAX_DIMS];
};

__device__ __forceinline__ int64_t out_to_in_base(const RDims &d, int ndim, int64_t o) {
  int64_t base = 0;
  for (int k = ndim - 1; k >= 0; --k) {
    int64_t c = o % d.out[k];
    o /= d.out[k];
    base += c * d.in_stride[k];
  }
  return base;
}

__device__ __forceinline__ int64_t red_offset(const RDims &d, int ndim, int64_t r) {
  int64_t off = 0;
  for (int k = ndim - 1; k >= 0; --k) {
    if (d.out[k] == 1 && d.in[k] > 1) {
      int64_t c = r % d.in[k];
      r /= d.in[k];
      off += c * d.in_stride[k];
    }
  }
  return off;
}

// one thread per output element
__global__ void k_reduce_thread(const float *__restrict__ x, float *__restrict__ y, RDims d,
                                int ndim, int64_t n_out, int64_t n_red, float scale, int acc) {
  for (int64_t o = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; o < n_out;
       o += (int64_t)gridDim.x * blockDim.x) {
    int64_t base = out_to_in_base(d, ndim, o);
    float s = 0.f;
    for (int64_t r = 0; r < n_red; ++r) s += x[base + red_offset(d, ndim, r)];
    s *= scale;
    y[o] = acc ? y[o] + s : s;
  }
}

// one block per output element (tree reduction)
__global__ void k_reduce_block(const float *__restrict__ x, float *__restrict__ y, RDims d,
                               int ndim, int64_t n_out, int64_t n_red, float scale, int acc) {
  __shared__ float part[32];
  for (int64_t o = blockIdx.x; o < n_out; o += gridDim.x) {
    int64_t base = out_to_in_base(d, ndim, o);
    float s = 0.f;
    for (int64_t r = threadIdx.x; r < n_red; r += blockDim.x) s += x[base + red_offset(d, ndim, r)];
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
      float v = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.f;
      v = warp_sum(v);
      if (threadIdx.x == 0) {
        v *= scale;
        y[o] = acc ? y[o] + v : v;
      }
    }
    __syncthreads();
  }
}



// ---- softmax over the last axis: one warp per row ---------------------------------
__global__ void k_softmax_fwd(const float *__restrict__ x, float *__restrict__ y, int64_t rows,
                              int64_t cols, int log_mode) {
  int64_t warps = (int64_t)gridDim.x * (blockDim.x / kWarp);
  int lane = threadIdx.x & 31;
  for (int64_t r = blockIdx.x * (int64_t)(blockDim.x / kWarp) + threadIdx.x / kWarp; r < rows;
       r += warps) {
    const float *xr = x + r * cols;
    float *yr = y + r * cols;
    float m = -INFINITY;
    for (int64_t c = lane; c < cols; c += kWarp) m = fmaxf(m, xr[c]);
    m = warp_max(m);
    float s = 0.f;
    for (int64_t c = lane; c < cols; c += kWarp) s += expf(xr[c] - m);
    s = warp_sum(s);
    if (log_mode) {
      float lse = logf(s);
      for (int64_t c = lane; c < cols; c += kWarp) yr[c] = (xr[c] - m) - lse;
    } else {
      float inv = 1.0f / s;
      for (int64_t c = lane; c < cols; c += kWarp) yr[c] = expf(xr[c] - m) * inv;
    }
  }
}

__global__ void k_softmax_bwd(const float *__restrict__ y, const float *__restrict__ dy,
                              float *__restrict__ dx, int64_t rows, int64_t cols, int log_mode,
                              int acc, int round) {
  int64_t warps = (int64_t)gridDim.x * (blockDim.x / kWarp);
  int lane = threadIdx.x & 31;
  for (int64_t r = blockIdx.x * (int64_t)(blockDim.x / kWarp) + threadIdx.x / kWarp; r < rows;
       r += warps) {
    const float *yr = y + r * cols;
    const float *gr = dy + r * cols;
    float *dr = dx + r * cols;
    float s = 0.f;
    if (log_mode) {
      for (int64_t c = lane; c < cols; c += kWarp) s += gr[c];
    } else {
      for (int64_t c = lane; c < cols; c += kWarp) s += gr[c] * yr[c];
    }
    s = warp_sum(s);
    for (int64_t c = lane; c < cols; c += kWarp) {
      float g = log_mode ? gr[c] - expf(yr[c]) * s : yr[c] * (gr[c] - s);
      g = acc ? dr[c] + g : g;
      dr[c] = round ? tx_epi::round_tf32(g) : g;
    }
  }
}

// Register-resident softmax for rows of VPL * 128 floats: a warp per row,
// one HBM read of x (and of y, dy in the backward).  y32 (softmax only, may be
// null): a second copy of y rounded to TF32, for contractions that read y.
template <int VPL>
__global__ void k_softmax_fwd_v(const float *__restrict__ x, float *__restrict__ y, float *__restrict__ y32,
                                int64_t rows, int log_mode) {
  constexpr int cols = VPL * 128;
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / kWarp);
  for (int64_t r = blockIdx.x * (int64_t)(blockDim.x / kWarp) + threadIdx.x / kWarp; r < rows; r += warps) {
    const float4 *xr = reinterpret_cast<const float4 *>(x + r * cols);
    float4 v[VPL];
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      v[j] = xr[j * 32 + lane];
      m = fmaxf(m, fmaxf(fmaxf(v[j].x, v[j].y), fmaxf(v[j].z, v[j].w)));
    }
    m = warp_max(m);
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; ++j)
      s += expf(v[j].x - m) + expf(v[j].y - m) + expf(v[j].z - m) + expf(v[j].w - m);
    s = warp_sum(s);
    float4 *yr = reinterpret_cast<float4 *>(y + r * cols);
    if (log_mode) {
      const float lse = logf(s);
#pragma unroll
      for (int j = 0; j < VPL; ++j)
        yr[j * 32 + lane] = make_float4((v[j].x - m) - lse, (v[j].y - m) - lse, (v[j].z - m) - lse, (v[j].w - m) - lse);
    } else {
      const float inv = 1.0f / s;
      float4 *yq = y32 ? reinterpret_cast<float4 *>(y32 + r * cols) : nullptr;
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        const float4 p = make_float4(expf(v[j].x - m) * inv, expf(v[j].y - m) * inv, expf(v[j].z - m) * inv,
                                     expf(v[j].w - m) * inv);
        yr[j * 32 + lane] = p;
        if (yq)
          yq[j * 32 + lane] = make_float4(tx_epi::round_tf32(p.x), tx_epi::round_tf32(p.y),
                                          tx_epi::round_tf32(p.z), tx_epi::round_tf32(p.w));
      }
    }
  }
}

template <int VPL>
__global__ void k_softmax_bwd_v(const float *__restrict__ y, const float *__restrict__ dy, float *__restrict__ dx,
                                int64_t rows, int log_mode, int acc, int round) {
  constexpr int cols = VPL * 128;
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / kWarp);
  for (int64_t r = blockIdx.x * (int64_t)(blockDim.x / kWarp) + threadIdx.x / kWarp; r < rows; r += warps) {
    const float4 *yr = reinterpret_cast<const float4 *>(y + r * cols);
    const float4 *gr = reinterpret_cast<const float4 *>(dy + r * cols);
    float4 yv[VPL], gv[VPL];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      yv[j] = yr[j * 32 + lane];
      gv[j] = gr[j * 32 + lane];
      s += log_mode ? gv[j].x + gv[j].y + gv[j].z + gv[j].w
                    : gv[j].x * yv[j].x + gv[j].y * yv[j].y + gv[j].z * yv[j].z + gv[j].w * yv[j].w;
    }
    s = warp_sum(s);
    float4 *dr = reinterpret_cast<float4 *>(dx + r * cols);
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      float4 o;
      if (log_mode) {
        o = make_float4(gv[j].x - expf(yv[j].x) * s, gv[j].y - expf(yv[j].y) * s, gv[j].z - expf(yv[j].z) * s,
                        gv[j].w - expf(yv[j].w) * s);
      } else {
        o = make_float4(yv[j].x * (gv[j].x - s), yv[j].y * (gv[j].y - s), yv[j].z * (gv[j].z - s),
                        yv[j].w * (gv[j].w - s));
      }
      if (acc) {
        const float4 p = dr[j * 32 + lane];
        o.x += p.x;
        o.y += p.y;
        o.z += p.z;
        o.w += p.w;
      }
      if (round)
        o = make_float4(tx_epi::round_tf32(o.x), tx_epi::round_tf32(o.y), tx_epi::round_tf32(o.z),
                        tx_epi::round_tf32(o.w));
      dr[j * 32 + lane] = o;
    }
  }
}

// ---- fused softmax cross-entropy ----------------------------------------------------
// phase 1: per-row loss = logsumexp(z) - z[y]
__global__ void k_xent_rows(const float *__restrict__ z, const int64_t *__restrict__ labels,
                            float *__restrict__ row_loss, int64_t rows, int64_t cols, int *flag) {
  int64_t warps = (int64_t)gridDim.x * (blockDim.x / kWarp);
  int lane = threadIdx.x & 31;
  for (int64_t r = blockIdx.x * (int64_t)(blockDim.x / kWarp) + threadIdx.x / kWarp; r < rows;
       r += warps) {
    const float *zr = z + r * cols;
    float m = -INFINITY;
    for (int64_t c = lane; c < cols; c += kWarp) m = fmaxf(m, zr[c]);
    m = warp_max(m);
    float s = 0.f;
    for (int64_t c = lane; c < cols; c += kWarp) s += expf(zr[c] - m);
    s = warp_sum(s);
    if (lane == 0) {
      int64_t y = labels[r];
      if (y < 0 || y >= cols) {
        raise_flag(flag, DEVERR_LABEL, (int)y, (int)cols);
        row_loss[r] = 0.f;
      } else {
        // -log_softmax(z)[y] = -( (z_y - m) - log(s) )
        row_loss[r] = -((zr[y] - m) - logf(s));
      }
    }
  }
}

// phase 2: fixed-order mean over rows (single block)
__global__ void k_mean_rows(const float *__restrict__ v, int64_t n, float *__restrict__ out) {
  __shared__ float part[32];
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) s += v[i];
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) out[0] = t / (float)n;
  }
}

__global__ void k_xent_bwd(const float *__restrict__ z, const int64_t *__restrict__ labels,
                           const float *__restrict__ scale_ptr, float *__restrict__ dz,
                           int64_t rows, int64_t cols, int acc) {
  int64_t warps = (int64_t)gridDim.x * (blockDim.x / kWarp);
  int lane = threadIdx.x & 31;
  float scale = (scale_ptr ? scale_ptr[0] : 1.f) / (float)rows;
  for (int64_t r = blockIdx.x * (int64_t)(blockDim.x / kWarp) + threadIdx.x / kWarp; r < rows;
       r += warps) {
    const float *zr = z + r * cols;
    float *dr = dz + r * cols;
    float m = -INFINITY;
    for (int64_t c = lane; c < cols; c += kWarp) m = fmaxf(m, zr[c]);
    m = warp_max(m);
    float s = 0.f;
    for (int64_t c = lane; c < cols; c += kWarp) s += expf(zr[c] - m);
    s = warp_sum(s);
    float inv = 1.0f / s;
    int64_t y = labels[r];
    for (int64_t c = lane; c < cols; c += kWarp) {
      float p = expf(zr[c] - m) * inv;
      float g = scale * (p - (c == y ? 1.f : 0.f));
      dr[c] = acc ? dr[c] + g : g;
    }
  }
}

// ---- LayerNorm over trailing `cols` (normalization.rs:135-190) ---------------------------
__global__ void k_layernorm_fwd(const float *__restrict__ x, const float *__restrict__ gamma,
                                const float *__restrict__ beta, float *__restrict__ y,
                                float *__restrict__ mean_out, float *__restrict__ rstd_out,
                                int64_t rows, int64_t cols, float eps, int round_tf32) {
  int64_t warps = (int64_t)gridDim.x * (blockDim.x / kWarp);
  int lane = threadIdx.x & 31;
  for (int64_t r = blockIdx.x * (int64_t)(blockDim.x / kWarp) + threadIdx.x / kWarp; r < rows;
       r += warps) {
    const float *xr = x + r * cols;
    float s = 0.f;
    for (int64_t c = lane; c < cols; c += kWarp) s += xr[c];
    float mu = warp_sum(s) / (float)cols;
    float q = 0.f;
    for (int64_t c = lane; c < cols; c += kWarp) {
      float d = xr[c] - mu;
      q += d * d;
    }
    float var = warp_sum(q) / (float)cols;
    float rstd = 1.0f / sqrtf(var + eps);  // (var + eps)^(-1/2)
    float *yr = y + r * cols;
    for (int64_t c = lane; c < cols; c += kWarp) {
      float v = (xr[c] - mu) * rstd * gamma[c];
      if (beta) v += beta[c];
      yr[c] = round_tf32 ? tx_epi::round_tf32(v) : v;
    }
    if (lane == 0) {
      if (mean_out) mean_out[r] = mu;
      if (rstd_out) rstd_out[r] = rstd;
    }
  }
}

// Register-resident variants for rows of VPL * 128 floats (cols % 128 == 0,
// up to 1024): a warp per row, each lane holding VPL float4 of it, so the row
// is read from HBM once.  Same formulas as the scalar kernels
// (normalization.rs:135-190): mean, biased variance of the centred values,
// rstd = (var + eps)^-1/2.
template <int VPL>
__global__ void k_layernorm_fwd_v(const float *__restrict__ x, const float *__restrict__ gamma,
                                  const float *__restrict__ beta, float *__restrict__ y,
                                  float *__restrict__ mean_out, float *__restrict__ rstd_out, int64_t rows,
                                  float eps, int round_tf32) {
  constexpr int cols = VPL * 128;
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / kWarp);
  for (int64_t r = blockIdx.x * (int64_t)(blockDim.x / kWarp) + threadIdx.x / kWarp; r < rows; r += warps) {
    const float4 *xr = reinterpret_cast<const float4 *>(x + r * cols);
    float4 v[VPL];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      v[j] = xr[j * 32 + lane];
      s += v[j].x + v[j].y + v[j].z + v[j].w;
    }
    const float mu = warp_sum(s) / (float)cols;
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const float a = v[j].x - mu, b = v[j].y - mu, c = v[j].z - mu, e = v[j].w - mu;
      q += a * a + b * b + c * c + e * e;
    }
    const float var = warp_sum(q) / (float)cols;
    const float rstd = 1.0f / sqrtf(var + eps);
    float4 *yr = reinterpret_cast<float4 *>(y + r * cols);
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int c4 = j * 32 + lane;
      const float4 gm = reinterpret_cast<const float4 *>(gamma)[c4];
      const float4 bt = beta ? reinterpret_cast<const float4 *>(beta)[c4] : make_float4(0.f, 0.f, 0.f, 0.f);
      float4 o;
      o.x = (v[j].x - mu) * rstd * gm.x + bt.x;
      o.y = (v[j].y - mu) * rstd * gm.y + bt.y;
      o.z = (v[j].z - mu) * rstd * gm.z + bt.z;
      o.w = (v[j].w - mu) * rstd * gm.w + bt.w;
      if (round_tf32) {
        o.x = tx_epi::round_tf32(o.x);
        o.y = tx_epi::round_tf32(o.y);
        o.z = tx_epi::round_tf32(o.z);
        o.w = tx_epi::round_tf32(o.w);
      }
      yr[c4] = o;
    }
    if (lane == 0) {
      if (mean_out) mean_out[r] = mu;
      if (rstd_out) rstd_out[r] = rstd;
    }
  }
}

// Backward, 8 warps per block: dx per row from registers; each lane keeps the
// dgamma / dbeta partial sums of its columns over the rows its warp visits,
// and the 8 warps are combined in a fixed order into one partial row per block.
template <int VPL>
__global__ void __launch_bounds__(256) k_layernorm_bwd_v(const float *__restrict__ x, const float *__restrict__ gamma,
                                  const float *__restrict__ mean_in, const float *__restrict__ rstd_in,
                                  const float *__restrict__ dy, float *__restrict__ dx,
                                  float *__restrict__ part_g, float *__restrict__ part_b, int64_t rows,
                                  int acc_dx) {
  constexpr int cols = VPL * 128;
  __shared__ float4 sg[8][VPL * 32], sb[8][VPL * 32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  float4 pg[VPL], pb[VPL], gm[VPL];
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    pg[j] = pb[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    gm[j] = reinterpret_cast<const float4 *>(gamma)[j * 32 + lane];
  }
  for (int64_t r = blockIdx.x * (int64_t)8 + w; r < rows; r += (int64_t)gridDim.x * 8) {
    const float4 *xr = reinterpret_cast<const float4 *>(x + r * cols);
    const float4 *gr = reinterpret_cast<const float4 *>(dy + r * cols);
    const float mu = mean_in[r], rs = rstd_in[r];
    float4 xh[VPL], g[VPL];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const float4 xv = xr[j * 32 + lane], dv = gr[j * 32 + lane];
      xh[j] = make_float4((xv.x - mu) * rs, (xv.y - mu) * rs, (xv.z - mu) * rs, (xv.w - mu) * rs);
      g[j] = make_float4(dv.x * gm[j].x, dv.y * gm[j].y, dv.z * gm[j].z, dv.w * gm[j].w);
      s1 += g[j].x + g[j].y + g[j].z + g[j].w;
      s2 += g[j].x * xh[j].x + g[j].y * xh[j].y + g[j].z * xh[j].z + g[j].w * xh[j].w;
      pg[j].x += dv.x * xh[j].x;
      pg[j].y += dv.y * xh[j].y;
      pg[j].z += dv.z * xh[j].z;
      pg[j].w += dv.w * xh[j].w;
      pb[j].x += dv.x;
      pb[j].y += dv.y;
      pb[j].z += dv.z;
      pb[j].w += dv.w;
    }
    s1 = warp_sum(s1) / (float)cols;
    s2 = warp_sum(s2) / (float)cols;
    if (dx) {
      float4 *dr = reinterpret_cast<float4 *>(dx + r * cols);
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        float4 o = make_float4(rs * (g[j].x - s1 - xh[j].x * s2), rs * (g[j].y - s1 - xh[j].y * s2),
                               rs * (g[j].z - s1 - xh[j].z * s2), rs * (g[j].w - s1 - xh[j].w * s2));
        if (acc_dx) {
          const float4 p = dr[j * 32 + lane];
          o.x += p.x;
          o.y += p.y;
          o.z += p.z;
          o.w += p.w;
        }
        dr[j * 32 + lane] = o;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    sg[w][j * 32 + lane] = pg[j];
    sb[w][j * 32 + lane] = pb[j];
  }
  __syncthreads();
  for (int c4 = threadIdx.x; c4 < VPL * 32; c4 += blockDim.x) {
    float4 a = sg[0][c4], b = sb[0][c4];
#pragma unroll
    for (int i = 1; i < 8; ++i) {
      const float4 u = sg[i][c4], t = sb[i][c4];
      a.x += u.x; a.y += u.y; a.z += u.z; a.w += u.w;
      b.x += t.x; b.y += t.y; b.z += t.z; b.w += t.w;
    }
    reinterpret_cast<float4 *>(part_g + blockIdx.x * (int64_t)cols)[c4] = a;
    reinterpret_cast<float4 *>(part_b + blockIdx.x * (int64_t)cols)[c4] = b;
  }
}

// dx per row; per-block partial column sums of dy*xhat and dy for dgamma/dbeta
__global__ void k_layernorm_bwd(const float *__restrict__ x, const float *__restrict__ gamma,
                                const float *__restrict__ mean_in, const float *__restrict__ rstd_in,
                                const float *__restrict__ dy, float *__restrict__ dx,
                                float *__restrict__ part_g, float *__restrict__ part_b, int64_t rows,
                                int64_t cols, int acc_dx) {
  extern __shared__ float sm[];  // [warps][cols] for dgamma partial, then dbeta partial
  int nw = blockDim.x / kWarp;
  int w = threadIdx.x / kWarp;
  int lane = threadIdx.x & 31;
  float *pg = sm;
  float *pb = sm + (int64_t)nw * cols;
  for (int64_t c = lane; c < cols; c += kWarp) {
    pg[w * cols + c] = 0.f;
    pb[w * cols + c] = 0.f;
  }
  for (int64_t r = blockIdx.x * (int64_t)nw + w; r < rows; r += (int64_t)gridDim.x * nw) {
    const float *xr = x + r * cols;
    const float *gr = dy + r * cols;
    float mu = mean_in[r], rs = rstd_in[r];
    float s1 = 0.f, s2 = 0.f;
    for (int64_t c = lane; c < cols; c += kWarp) {
      float xh = (xr[c] - mu) * rs;
      float g = gr[c] * gamma[c];
      s1 += g;
      s2 += g * xh;
      pg[w * cols + c] += gr[c] * xh;
      pb[w * cols + c] += gr[c];
    }
    s1 = warp_sum(s1) / (float)cols;
    s2 = warp_sum(s2) / (float)cols;
    if (dx) {
      float *dr = dx + r * cols;
      for (int64_t c = lane; c < cols; c += kWarp) {
        float xh = (xr[c] - mu) * rs;
        float v = rs * (gr[c] * gamma[c] - s1 - xh * s2);
        dr[c] = acc_dx ? dr[c] + v : v;
      }
    }
  }
  __syncthreads();
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
    float a = 0.f, b = 0.f;
    for (int i = 0; i < nw; ++i) {
      a += pg[i * cols + c];
      b += pb[i * cols + c];
    }
    part_g[blockIdx.x * cols + c] = a;
    part_b[blockIdx.x * cols + c] = b;
  }
}

// out[c] (+)= scale * sum_p part[p, c]   (fixed order)

// Final column reduction of a [np, cols] partial-sum matrix: out = scale * sum
// (+ out when acc).  Block (32, 32): lane x owns column 32 * blockIdx.x + x,
// the 32 row groups take partial rows ty, ty + 32, ... in order with eight
// loads in flight, and the groups are combined in a fixed order.  blockIdx.y
// = 1 reduces a second matrix stored right after the first into out1.
__global__ void __launch_bounds__(1024) k_colsum_final(const float *__restrict__ part, int64_t np,
                                                       int64_t cols, float *__restrict__ out,
                                                       float *__restrict__ out1, float scale, int acc) {
  __shared__ float sm[32][33];
  if (blockIdx.y) {
    part += np * cols;
    out = out1;
  }
  const int64_t c = (int64_t)blockIdx.x * 32 + threadIdx.x;
  float s = 0.f;
  if (c < cols) {
    int64_t p = threadIdx.y;
    for (; p + 7 * 32 < np; p += 8 * 32) {
      float v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = part[(p + 32 * i) * cols + c];
#pragma unroll
      for (int i = 0; i < 8; ++i) s += v[i];
    }
    for (; p < np; p += 32) s += part[p * cols + c];
  }
  sm[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y == 0 && c < cols) {
    float t = sm[0][threadIdx.x];
#pragma unroll
    for (int i = 1; i < 32; ++i) t += sm[i][threadIdx.x];
    t *= scale;
    out[c] = acc ? out[c] + t : t;
  }
}


// ---- TF32 operand shadow ---------------------------------------------------------------
__global__ void k_round_tf32(const float *__restrict__ src, float *__restrict__ dst, int64_t n) {
  const int64_t n4 = n / 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const bool vec = ((((uintptr_t)src) | ((uintptr_t)dst)) & 15) == 0;
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (vec) {
    for (; i < n4; i += stride) {
      const float4 v = reinterpret_cast<const float4 *>(src)[i];
      reinterpret_cast<float4 *>(dst)[i] =
          make_float4(tx_epi::round_tf32(v.x), tx_epi::round_tf32(v.y), tx_epi::round_tf32(v.z),
                      tx_epi::round_tf32(v.w));
    }
    for (i = n4 * 4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride)
      dst[i] = tx_epi::round_tf32(src[i]);
  } else {
    for (; i < n; i += stride) dst[i] = tx_epi::round_tf32(src[i]);
  }
}

// TF32 head and tail: hi = rna(x), lo = rna(x - hi) (x - hi is exact in fp32)
__global__ void k_split_tf32(const float *__restrict__ src, float *__restrict__ hi, float *__restrict__ lo,
                             int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
    const float x = src[i];
    const float h = tx_epi::round_tf32(x);
    hi[i] = h;
    lo[i] = tx_epi::round_tf32(x - h);
  }
}

// ---- gather / scatter (gather.rs:18-58; select / select_assign) -------------------------
__global__ void k_gather_rows(const float *__restrict__ table, int64_t rows, int64_t width,
                              const int64_t *__restrict__ idx, int64_t n, float *__restrict__ out,
                              int *flag) {
  int64_t total = n * width;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = i / width, c = i - r * width;
    int64_t k = idx[r];
    if (k < 0) k += rows;
    if (k < 0 || k >= rows) {
      if (c == 0) raise_flag(flag, DEVERR_INDEX, (int)idx[r], (int)rows);
      out[i] = 0.f;
    } else {
      out[i] = table[k * width + c];
    }
  }
}

__global__ void k_gather_rows4(const float4 *__restrict__ table, int64_t rows, int64_t w4,
                               const int64_t *__restrict__ idx, int64_t n, float4 *__restrict__ out,
                               int *flag) {
  int64_t total = n * w4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = i / w4, c = i - r * w4;
    int64_t k = idx[r];
    if (k < 0) k += rows;
    if (k < 0 || k >= rows) {
      if (c == 0) raise_flag(flag, DEVERR_INDEX, (int)idx[r], (int)rows);
      out[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    } else {
      out[i] = table[k * w4 + c];
    }
  }
}

__global__ void k_scatter_add_rows(float *__restrict__ table, int64_t rows, int64_t width,
                                   const int64_t *__restrict__ idx, int64_t n,
                                   const float *__restrict__ src) {
  int64_t total = n * width;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = i / width, c = i - r * width;
    int64_t k = idx[r];
    if (k < 0) k += rows;
    if (k >= 0 && k < rows) atomicAdd(&table[k * width + c], src[i]);
  }
}

__global__ void k_take_last(const float *__restrict__ x, const int64_t *__restrict__ idx,
                            float *__restrict__ out, int64_t rows, int64_t cols, int *flag) {
  for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < rows;
       r += (int64_t)gridDim.x * blockDim.x) {
    int64_t k = idx[r];
    if (k < 0) k += cols;
    if (k < 0 || k >= cols) {
      raise_flag(flag, DEVERR_INDEX, (int)idx[r], (int)cols);
      out[r] = 0.f;
    } else {
      out[r] = x[r * cols + k];
    }
  }
}

__global__ void k_take_last_bwd(const int64_t *__restrict__ idx, const float *__restrict__ dout,
                                float *__restrict__ dx, int64_t rows, int64_t cols, int acc) {
  int64_t total = rows * cols;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = i / cols, c = i - r * cols;
    int64_t k = idx[r];
    if (k < 0) k += cols;
    float g = (c == k) ? dout[r] : 0.f;
    dx[i] = acc ? dx[i] + g : g;
  }
}

// ---- column sums (bias gradient) --------------------------------------------------------
// block (32, 8): 32 columns x 8 row lanes, rows [blockIdx.y*rows_per, ...)
// float4 columns (N % 4 == 0, 16-byte aligned rows): block (32, 8) covers 128
// columns; each thread sums rows r0 + ty, r0 + ty + 8, ... in order with four
// loads in flight, then the 8 row groups are combined in a fixed order.
__global__ void k_colsum_partial4(const float *__restrict__ dy, int64_t M, int64_t N,
                                  int64_t rows_per, float *__restrict__ part) {
  __shared__ float4 sm[8][32];
  const int64_t c = ((int64_t)blockIdx.x * 32 + threadIdx.x) * 4;
  const int64_t r0 = blockIdx.y * rows_per;
  const int64_t r1 = r0 + rows_per < M ? r0 + rows_per : M;
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  if (c < N) {
    int64_t r = r0 + threadIdx.y;
    for (; r + 24 < r1; r += 32) {
      float4 v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = *reinterpret_cast<const float4 *>(dy + (r + 8 * j) * N + c);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        s.x += v[j].x;
        s.y += v[j].y;
        s.z += v[j].z;
        s.w += v[j].w;
      }
    }
    for (; r < r1; r += 8) {
      const float4 v = *reinterpret_cast<const float4 *>(dy + r * N + c);
      s.x += v.x;
      s.y += v.y;
      s.z += v.z;
      s.w += v.w;
    }
  }
  sm[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y == 0 && c < N) {
    float4 t = sm[0][threadIdx.x];
#pragma unroll
    for (int i = 1; i < 8; ++i) {
      const float4 u = sm[i][threadIdx.x];
      t.x += u.x;
      t.y += u.y;
      t.z += u.z;
      t.w += u.w;
    }
    *reinterpret_cast<float4 *>(part + blockIdx.y * N + c) = t;
  }
}

__global__ void k_colsum_partial(const float *__restrict__ dy, int64_t M, int64_t N,
                                 int64_t rows_per, float *__restrict__ part) {
  __shared__ float sm[8][33];
  int64_t c = blockIdx.x * 32 + threadIdx.x;
  int64_t r0 = blockIdx.y * rows_per;
  int64_t r1 = r0 + rows_per < M ? r0 + rows_per : M;
  float s = 0.f;
  if (c < N)
    for (int64_t r = r0 + threadIdx.y; r < r1; r += 8) s += dy[r * N + c];
  sm[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y == 0 && c < N) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) t += sm[i][threadIdx.x];
    part[blockIdx.y * N + c] = t;
  }
}

// ---- multi-tensor optimizers (adam.rs:431-527, optimizer.rs:310-356) ---------------------
struct OptTensor {
  float *w;
  const float *g;
  float *m;
  float *v;
  float *vmax;
  int64_t n;
};
struct OptChunk {
  int32_t tensor;
  int64_t start, len;
};
struct OptHparams {
  float lr, beta1, beta2, eps, wd, one_minus_b1, one_minus_b2, decay_factor;
  double beta1_d, beta2_d;
  float momentum, one_minus_dampening;
};

// Adam / AdamW: one block per chunk.  Step counters: t = steps[i] + 1 for the
// math; the last block to finish (atomic ticket) commits the increments.
// The bias corrections of each tensor's next update, bc[2i] = 1 - beta1^t and
// bc[2i+1] = 1 - beta2^t (in double, rounded to f32 as mul_scalar /
// div_scalar(f64) on f32 data round them), live in device memory: written by
// k_adam_bc when the step counters or the betas are set, and by the last block
// of each step for the tensors it advanced, so no block evaluates pow().
__global__ void k_adam_bc(const int64_t *__restrict__ steps, float *__restrict__ bc, int n, double beta1,
                          double beta2) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const double t = (double)(steps[i] + 1);
    bc[2 * i] = (float)(1.0 - pow(beta1, t));
    bc[2 * i + 1] = (float)(1.0 - pow(beta2, t));
  }
}

constexpr int64_t kChunk_ = 4096;   // elements per optimizer chunk (kChunk below)
constexpr int64_t kAdamSub = 2048;  // elements per CTA piece: two float4 per thread (256 threads)

// At most 64 registers, so several CTAs share an SM.
__global__ void __launch_bounds__(256, 4)
    k_adam(const OptTensor *__restrict__ tensors, const OptChunk *__restrict__ chunks, int n_chunks,
           const OptHparams *__restrict__ hp_ptr, int64_t *steps, float *__restrict__ bc,
           const int32_t *__restrict__ active_list, int n_active, int kind, int amsgrad, unsigned *ticket) {
  const OptHparams hp = *hp_ptr;
  float bc1 = 1.f, bc2 = 1.f;  // the current piece's tensor's bias corrections
  const bool coupled = (kind == 0) && hp.wd != 0.f;
  const bool decoupled = (kind == 1) && hp.wd != 0.f;
  // one element, in the order of adam.rs:458-509 (no FMA contraction)
  auto update = [&](float &w, float d, float &m, float &v, float *vmax_slot) {
    if (coupled) d = __fadd_rn(d, __fmul_rn(w, hp.wd));
    m = __fadd_rn(__fmul_rn(m, hp.beta1), __fmul_rn(d, hp.one_minus_b1));
    v = __fadd_rn(__fmul_rn(v, hp.beta2), __fmul_rn(__fmul_rn(d, d), hp.one_minus_b2));
    float den = v;
    if (amsgrad) {
      den = fmaxf(*vmax_slot, v);
      *vmax_slot = den;
    }
    float mh = __fdiv_rn(m, bc1);
    float vh = __fdiv_rn(den, bc2);
    float upd = __fmul_rn(__fdiv_rn(mh, __fadd_rn(__fsqrt_rn(vh), hp.eps)), hp.lr);
    if (decoupled) w = __fmul_rn(w, hp.decay_factor);
    w = __fsub_rn(w, upd);
  };
  // One wave of CTAs walks the kAdamSub-element pieces of the chunks in order
  // (piece p: chunk p / subs, part p % subs): no partial last wave, and the
  // next piece's chunk entry is fetched before this piece is updated, so the
  // dependent descriptor loads overlap the stream.
  constexpr int subs = (int)(kChunk_ / kAdamSub);
  const int total = n_chunks * subs;
  int p = blockIdx.x;
  OptChunk ch_next = p < total ? chunks[p / subs] : OptChunk{0, 0, 0};
  for (; p < total; p += gridDim.x) {
  const OptChunk ch = ch_next;
  if (p + (int)gridDim.x < total) ch_next = chunks[(p + gridDim.x) / subs];
  const OptTensor t = tensors[ch.tensor];
  bc1 = bc[2 * ch.tensor];
  bc2 = bc[2 * ch.tensor + 1];
  const int64_t end = ch.start + ch.len;
  const int64_t lo = ch.start + (int64_t)(p % subs) * kAdamSub;
  const int64_t hi = lo + kAdamSub < end ? lo + kAdamSub : end;
  const bool vec = !amsgrad && (lo & 3) == 0 &&
                   ((((uintptr_t)t.w) | ((uintptr_t)t.g) | ((uintptr_t)t.m) | ((uintptr_t)t.v)) & 15) == 0;
  if (vec) {
    // both of a thread's float4 groups are loaded before either is updated,
    // so each thread keeps 128 bytes of loads in flight
    const int64_t i0 = lo + threadIdx.x * 4, i1 = i0 + (int64_t)blockDim.x * 4;
    const bool h0 = i0 + 3 < hi, h1 = i1 + 3 < hi;
    float4 w0, g0, m0, v0, w1, g1, m1, v1;
    if (h0) {
      w0 = *reinterpret_cast<float4 *>(t.w + i0);
      g0 = *reinterpret_cast<const float4 *>(t.g + i0);
      m0 = *reinterpret_cast<float4 *>(t.m + i0);
      v0 = *reinterpret_cast<float4 *>(t.v + i0);
    }
    if (h1) {
      w1 = *reinterpret_cast<float4 *>(t.w + i1);
      g1 = *reinterpret_cast<const float4 *>(t.g + i1);
      m1 = *reinterpret_cast<float4 *>(t.m + i1);
      v1 = *reinterpret_cast<float4 *>(t.v + i1);
    }
    if (h0) {
      update(w0.x, g0.x, m0.x, v0.x, nullptr);
      update(w0.y, g0.y, m0.y, v0.y, nullptr);
      update(w0.z, g0.z, m0.z, v0.z, nullptr);
      update(w0.w, g0.w, m0.w, v0.w, nullptr);
      *reinterpret_cast<float4 *>(t.w + i0) = w0;
      *reinterpret_cast<float4 *>(t.m + i0) = m0;
      *reinterpret_cast<float4 *>(t.v + i0) = v0;
    }
    if (h1) {
      update(w1.x, g1.x, m1.x, v1.x, nullptr);
      update(w1.y, g1.y, m1.y, v1.y, nullptr);
      update(w1.z, g1.z, m1.z, v1.z, nullptr);
      update(w1.w, g1.w, m1.w, v1.w, nullptr);
      *reinterpret_cast<float4 *>(t.w + i1) = w1;
      *reinterpret_cast<float4 *>(t.m + i1) = m1;
      *reinterpret_cast<float4 *>(t.v + i1) = v1;
    }
    // ragged tail of the last chunk of a tensor (past the last multiple of 4)
    const int64_t tail = (hi & ~int64_t(3)) > lo ? (hi & ~int64_t(3)) : lo;
    for (int64_t j = tail + threadIdx.x; j < hi; j += blockDim.x) {
      float w = t.w[j], m = t.m[j], v = t.v[j];
      update(w, t.g[j], m, v, nullptr);
      t.w[j] = w;
      t.m[j] = m;
      t.v[j] = v;
    }
  } else {
    for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
      float w = t.w[i], m = t.m[i], v = t.v[i];
      update(w, t.g[i], m, v, amsgrad ? t.vmax + i : nullptr);
      t.w[i] = w;
      t.m[i] = m;
      t.v[i] = v;
    }
  }
  }
  __shared__ int s_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    s_last = atomicAdd(ticket, 1u) == (unsigned)(gridDim.x * gridDim.y) - 1;
  }
  __syncthreads();
  if (s_last) {  // every block has read the step counters and corrections: advance them
    for (int i = threadIdx.x; i < n_active; i += blockDim.x) {
      const int k = active_list[i];
      const int64_t done = steps[k] + 1;
      steps[k] = done;
      bc[2 * k] = (float)(1.0 - pow(hp.beta1_d, (double)(done + 1)));
      bc[2 * k + 1] = (float)(1.0 - pow(hp.beta2_d, (double)(done + 1)));
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      *ticket = 0u;
    }
  }
}

__global__ void k_sgd(const OptTensor *__restrict__ tensors, const OptChunk *__restrict__ chunks,
                      const OptHparams *__restrict__ hp_ptr, int64_t *steps, int n_chunks,
                      const int32_t *__restrict__ active_list, int n_active, int nesterov,
                      unsigned *ticket) {
  const OptHparams hp = *hp_ptr;
  const OptChunk ch = chunks[blockIdx.x];
  const OptTensor t = tensors[ch.tensor];
  const bool first = steps[ch.tensor] == 0;
  for (int64_t i = ch.start + threadIdx.x; i < ch.start + ch.len; i += blockDim.x) {
    float w = t.w[i];
    float d = t.g[i];
    if (hp.wd != 0.f) d = __fadd_rn(d, __fmul_rn(w, hp.wd));
    if (hp.momentum != 0.f) {
      float buf = first ? d
                        : __fadd_rn(__fmul_rn(t.m[i], hp.momentum), __fmul_rn(d, hp.one_minus_dampening));
      t.m[i] = buf;
      d = nesterov ? __fadd_rn(d, __fmul_rn(buf, hp.momentum)) : buf;
    }
    t.w[i] = __fsub_rn(w, __fmul_rn(d, hp.lr));
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    unsigned done = atomicAdd(ticket, 1u);
    if (done == (unsigned)n_chunks - 1) {
      for (int i = 0; i < n_active; ++i) steps[active_list[i]] += 1;
      __threadfence();
      *ticket = 0u;
    }
  }
}

}  // namespace

int colsum_finish(tx_ctx *ctx, const float *part, int64_t np, int64_t cols, float *out, float scale,
                  int acc) {
  const int64_t blocks = (cols + 31) / 32;
  if (blocks > 0x7fffffff) return tx_fail(ctx, TX_ERR_UNSUPPORTED, "column reduction too wide");
  k_colsum_final<<<(unsigned)blocks, dim3(32, 32), 0, ctx->stream>>>(part, np, cols, out, nullptr, scale, acc);
  TX_LAUNCHED(ctx, "k_colsum_final");
  return TX_OK;
}

// Two column reductions in one launch: [np, cols] partials at part into out0
// and the next [np, cols] into out1 (either output may be null: then one)
static int colsum_finish2(tx_ctx *ctx, const float *part, int64_t np, int64_t cols, float *out0, float *out1,
                          float scale, int acc) {
  if (!out0 || !out1) {
    if (out0) TX_TRY(colsum_finish(ctx, part, np, cols, out0, scale, acc));
    if (out1) TX_TRY(colsum_finish(ctx, part + np * cols, np, cols, out1, scale, acc));
    return TX_OK;
  }
  const int64_t blocks = (cols + 31) / 32;
  if (blocks > 0x7fffffff) return tx_fail(ctx, TX_ERR_UNSUPPORTED, "column reduction too wide");
  k_colsum_final<<<dim3((unsigned)blocks, 2), dim3(32, 32), 0, ctx->stream>>>(part, np, cols, out0, out1, scale,
                                                                              acc);
  TX_LAUNCHED(ctx, "k_colsum_final");
  return TX_OK;
}

// ============================================================================
// host entry points
// ============================================================================
static inline unsigned rows_grid(int64_t rows, int warps_per_block) {
  int64_t b = (rows + warps_per_block - 1) / warps_per_block;
  if (b < 1) b = 1;
  if (b > 148 * 32) b = 148 * 32;
  return (unsigned)b;
}

extern "C" int tx_fill_f32(tx_ctx *ctx, float *y, int64_t n, float v) {
  if (!ctx) return TX_ERR_INVALID;
  if (n <= 0) return TX_OK;
  k_fill<<<grid_for(n, 256), 256, 0, ctx->stream>>>(y, n, v);
  TX_LAUNCHED(ctx, "k_fill");
  return TX_OK;
}

extern "C" int tx_unary(tx_ctx *ctx, int op, const float *x, float *y, int64_t n, float a, float b) {
  if (!ctx || op < 0 || op > TX_UN_RECIPROCAL) return TX_ERR_INVALID;
  if (n <= 0) return TX_OK;
  k_unary<<<grid_for((n + 3) / 4, 256), 256, 0, ctx->stream>>>(op, x, y, n, a, b);
  TX_LAUNCHED(ctx, "k_unary");
  return TX_OK;
}

extern "C" int tx_unary_bwd(tx_ctx *ctx, int op, const float *s, const float *dy, float *dx,
                            int64_t n, float a, float b, int acc) {
  if (!ctx || op < 0 || op > TX_UN_RECIPROCAL) return TX_ERR_INVALID;
  if (n <= 0) return TX_OK;
  k_unary_bwd<<<grid_for(n, 256), 256, 0, ctx->stream>>>(op, s, dy, dx, n, a, b, acc);
  TX_LAUNCHED(ctx, "k_unary_bwd");
  return TX_OK;
}

extern "C" int tx_binary(tx_ctx *ctx, int op, const float *A, const int64_t *sa, const float *B,
                         const int64_t *sb, float *out, const int64_t *shape, int ndim) {
  if (!ctx || ndim < 0 || ndim > TX_MAX_DIMS || op < 0 || op > TX_BIN_POW) return TX_ERR_INVALID;
  return nd_binary(ctx, op, A, sa, B, sb, out, shape, ndim);
}

extern "C" int tx_reduce_to(tx_ctx *ctx, const float *x, const int64_t *in_shape, float *y,
                            const int64_t *out_shape, int ndim, int mean, int acc) {
  if (!ctx || ndim < 0 || ndim > TX_MAX_DIMS) return TX_ERR_INVALID;
  RDims d;
  int64_t n_out = 1, n_red = 1, stride = 1;
  for (int k = ndim - 1; k >= 0; --k) {
    d.in[k] = in_shape[k];
    d.out[k] = out_shape[k];
    d.in_stride[k] = stride;
    stride *= in_shape[k];
    if (out_shape[k] != in_shape[k] && out_shape[k] != 1)
      return tx_fail(ctx, TX_ERR_SHAPE, "tx_reduce_to: output extent must equal input or be 1");
    n_out *= out_shape[k];
    if (out_shape[k] == 1) n_red *= in_shape[k];
  }
  if (n_out <= 0) return TX_OK;
  float scale = mean ? 1.0f / (float)(n_red > 0 ? n_red : 1) : 1.0f;
  if (n_red == 1) return nd_copy(ctx, x, d.in_stride, y, out_shape, ndim, 4, scale, acc);
  const int rc = nd_reduce(ctx, x, in_shape, out_shape, ndim, y, scale, acc);
  if (rc != TX_ERR_UNSUPPORTED) return rc;
  if (n_out >= 4096 || n_red <= 32) {
    k_reduce_thread<<<grid_for(n_out, 256), 256, 0, ctx->stream>>>(x, y, d, ndim, n_out, n_red,
                                                                   scale, acc);
  } else {
    unsigned blocks = n_out < 148 * 8 ? (unsigned)n_out : 148 * 8;
    k_reduce_block<<<blocks, 256, 0, ctx->stream>>>(x, y, d, ndim, n_out, n_red, scale, acc);
  }
  TX_LAUNCHED(ctx, "k_reduce");
  return TX_OK;
}

extern "C" int tx_strided_copy(tx_ctx *ctx, const void *src, const int64_t *ss, void *dst,
                               const int64_t *shape, int ndim, int elem_bytes) {
  if (!ctx || ndim < 0 || ndim > TX_MAX_DIMS || (elem_bytes != 4 && elem_bytes != 8)) return TX_ERR_INVALID;
  return nd_copy(ctx, src, ss, dst, shape, ndim, elem_bytes, 1.f, 0);
}

// ---- training-mode dropout (the capture IR's Dropout: a device random stream
// that advances with every call, so a replayed graph draws new masks) ----------
// u = the SplitMix64 finaliser (Steele, Lea and Flood, "Fast splittable
// pseudorandom number generators", OOPSLA 2014) of (seed, call counter, element)
// -> 24 uniform bits; the element is kept when u >= p and scaled by 1 / (1 - p).
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z ^= z >> 30;
  z *= 0xbf58476d1ce4e5b9ull;
  z ^= z >> 27;
  z *= 0x94d049bb133111ebull;
  z ^= z >> 31;
  return z;
}

__global__ void k_dropout(const float *__restrict__ x, float *__restrict__ y, float *__restrict__ mask, int64_t n,
                          float p, uint64_t seed, const uint64_t *__restrict__ counter) {
  const uint64_t ctr = *counter;
  const float keep_scale = 1.f / (1.f - p);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t h = mix64(seed ^ mix64(ctr * 0x9e3779b97f4a7c15ull + (uint64_t)i));
    const float u = (float)(h >> 40) * (1.f / 16777216.f);
    const float m = u >= p ? keep_scale : 0.f;
    mask[i] = m;
    y[i] = x[i] * m;
  }
}

__global__ void k_counter_add(uint64_t *counter) {
  if (threadIdx.x == 0 && blockIdx.x == 0) *counter += 1;
}

extern "C" int tx_dropout_fwd(tx_ctx *ctx, const float *x, float *y, float *mask, int64_t n, float p, uint64_t seed,
                              uint64_t *d_counter) {
  if (!ctx || !(p >= 0.f && p < 1.f)) return TX_ERR_INVALID;
  if (!d_counter) d_counter = ctx->d_rng;
  if (n > 0) {
    k_dropout<<<grid_for(n, 256), 256, 0, ctx->stream>>>(x, y, mask, n, p, seed, d_counter);
    TX_LAUNCHED(ctx, "k_dropout");
  }
  k_counter_add<<<1, 32, 0, ctx->stream>>>(d_counter);
  TX_LAUNCHED(ctx, "k_counter_add");
  return TX_OK;
}

extern "C" int tx_strided_scatter(tx_ctx *ctx, const float *src, float *dst, const int64_t *dst_strides,
                                  const int64_t *shape, int ndim, int acc) {
  if (!ctx || ndim < 0 || ndim > TX_MAX_DIMS) return TX_ERR_INVALID;
  return nd_scatter(ctx, src, dst, dst_strides, shape, ndim, acc);
}

// rows whose width is a multiple of 128 (up to 1024) on 16-byte aligned buffers
// take the register-resident float4 kernels
static bool ln_vec(int64_t cols, std::initializer_list<const void *> ptrs) {
  if (cols % 128 || cols > 1024) return false;
  for (const void *p : ptrs)
    if (((uintptr_t)p) & 15) return false;
  return true;
}

// y32 (may be null; not with log): also store y rounded to TF32 there
int softmax_fwd(tx_ctx *ctx, const float *x, float *y, float *y32, int64_t rows, int64_t cols, int log) {
  if (!ctx || (y32 && log)) return TX_ERR_INVALID;
  if (rows <= 0 || cols <= 0) return TX_OK;
  if (ln_vec(cols, {x, y}) && (!y32 || ln_vec(cols, {y32})) &&
      (cols == 128 || cols == 256 || cols == 512 || cols == 1024)) {
    const unsigned blocks = rows_grid(rows, 8);
    switch (cols) {
      case 128: k_softmax_fwd_v<1><<<blocks, 256, 0, ctx->stream>>>(x, y, y32, rows, log); break;
      case 256: k_softmax_fwd_v<2><<<blocks, 256, 0, ctx->stream>>>(x, y, y32, rows, log); break;
      case 512: k_softmax_fwd_v<4><<<blocks, 256, 0, ctx->stream>>>(x, y, y32, rows, log); break;
      default: k_softmax_fwd_v<8><<<blocks, 256, 0, ctx->stream>>>(x, y, y32, rows, log); break;
    }
    TX_LAUNCHED(ctx, "k_softmax_fwd_v");
    return TX_OK;
  }
  k_softmax_fwd<<<rows_grid(rows, 8), 256, 0, ctx->stream>>>(x, y, rows, cols, log);
  TX_LAUNCHED(ctx, "k_softmax_fwd");
  return y32 ? tx_round_tf32(ctx, y, y32, rows * cols) : TX_OK;
}

extern "C" int tx_softmax_fwd(tx_ctx *ctx, const float *x, float *y, int64_t rows, int64_t cols, int log) {
  return softmax_fwd(ctx, x, y, nullptr, rows, cols, log);
}

// round: store dx rounded to TF32 (for a gradient whose only readers are
// contractions that would round it anyway)
int softmax_bwd(tx_ctx *ctx, const float *y, const float *dy, float *dx, int64_t rows, int64_t cols, int log,
                int acc, bool round) {
  if (rows <= 0 || cols <= 0) return TX_OK;
  const int rt = round ? 1 : 0;
  if (ln_vec(cols, {y, dy, dx}) && (cols == 128 || cols == 256 || cols == 512 || cols == 1024)) {
    const unsigned blocks = rows_grid(rows, 8);
    switch (cols) {
      case 128: k_softmax_bwd_v<1><<<blocks, 256, 0, ctx->stream>>>(y, dy, dx, rows, log, acc, rt); break;
      case 256: k_softmax_bwd_v<2><<<blocks, 256, 0, ctx->stream>>>(y, dy, dx, rows, log, acc, rt); break;
      case 512: k_softmax_bwd_v<4><<<blocks, 256, 0, ctx->stream>>>(y, dy, dx, rows, log, acc, rt); break;
      default: k_softmax_bwd_v<8><<<blocks, 256, 0, ctx->stream>>>(y, dy, dx, rows, log, acc, rt); break;
    }
    TX_LAUNCHED(ctx, "k_softmax_bwd_v");
    return TX_OK;
  }
  k_softmax_bwd<<<rows_grid(rows, 8), 256, 0, ctx->stream>>>(y, dy, dx, rows, cols, log, acc, rt);
  TX_LAUNCHED(ctx, "k_softmax_bwd");
  return TX_OK;
}

extern "C" int tx_softmax_bwd(tx_ctx *ctx, const float *y, const float *dy, float *dx, int64_t rows,
                              int64_t cols, int log, int acc) {
  if (!ctx) return TX_ERR_INVALID;
  return softmax_bwd(ctx, y, dy, dx, rows, cols, log, acc, false);
}

extern "C" int tx_softmax_xent_fwd(tx_ctx *ctx, const float *z, const int64_t *labels, int64_t rows,
                                   int64_t cols, float *loss) {
  if (!ctx) return TX_ERR_INVALID;
  if (rows <= 0) return tx_fail(ctx, TX_ERR_SHAPE, "cross entropy over zero rows");
  Scratch rl(ctx, rows * sizeof(float));
  if (!rl.ptr) return TX_ERR_OOM;
  k_xent_rows<<<rows_grid(rows, 8), 256, 0, ctx->stream>>>(z, labels, rl.as<float>(), rows, cols,
                                                         ctx->d_err);
  TX_LAUNCHED(ctx, "k_xent_rows");
  k_mean_rows<<<1, 1024, 0, ctx->stream>>>(rl.as<float>(), rows, loss);
  TX_LAUNCHED(ctx, "k_mean_rows");
  return TX_OK;
}

// ---- allocation-free variant of tx_softmax_xent_fwd ------------------------------------
// The per-row losses live in a fixed file-scope device array instead of memory
// from the context allocator, for callers that must not allocate device memory.
// Every GPU that loads this library holds the array until the process exits.
static constexpr int64_t kXentNoAllocMaxRows = 1 << 18;  // 262144 rows = 1 MiB
static __device__ __align__(256) float g_xent_row_losses[kXentNoAllocMaxRows];
static float *g_xent_row_losses_addr[64] = {};  // per device, set on first use
static std::mutex g_xent_row_losses_mutex;

// The array's name is only a host-side stand-in in host code: its device
// address is resolved once per device, with that device current.
static int xent_noalloc_scratch(tx_ctx *ctx, float **out) {
  if (ctx->device < 0 || ctx->device >= 64)
    return tx_fail(ctx, TX_ERR_UNSUPPORTED, "device ordinal above 63");
  std::lock_guard<std::mutex> lock(g_xent_row_losses_mutex);
  if (!g_xent_row_losses_addr[ctx->device]) {
    int previous = 0;
    TX_CUDA(ctx, cudaGetDevice(&previous));
    TX_CUDA(ctx, cudaSetDevice(ctx->device));
    void *addr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&addr, g_xent_row_losses);
    cudaSetDevice(previous);
    if (e != cudaSuccess) return tx_cuda_fail(ctx, e, "cudaGetSymbolAddress(g_xent_row_losses)");
    g_xent_row_losses_addr[ctx->device] = (float *)addr;
  }
  *out = g_xent_row_losses_addr[ctx->device];
  return TX_OK;
}

extern "C" int tx_softmax_xent_fwd_noalloc(tx_ctx *ctx, const float *z, const int64_t *labels,
                                           int64_t rows, int64_t cols, float *loss) {
  if (!ctx) return TX_ERR_INVALID;
  if (rows <= 0) return tx_fail(ctx, TX_ERR_SHAPE, "cross entropy over zero rows");
  if (rows > kXentNoAllocMaxRows)
    return tx_fail(ctx, TX_ERR_SHAPE,
                   "tx_softmax_xent_fwd_noalloc handles at most 262144 rows; use tx_softmax_xent_fwd");
  float *scratch = nullptr;
  TX_TRY(xent_noalloc_scratch(ctx, &scratch));
  // every row in [0, rows) is written before it is read: nothing needs clearing
  k_xent_rows<<<rows_grid(rows, 8), 256, 0, ctx->stream>>>(z, labels, scratch, rows, cols,
                                                         ctx->d_err);
  TX_LAUNCHED(ctx, "k_xent_rows");
  k_mean_rows<<<1, 1024, 0, ctx->stream>>>(scratch, rows, loss);
  TX_LAUNCHED(ctx, "k_mean_rows");
  return TX_OK;
}

extern "C" int tx_softmax_xent_bwd(tx_ctx *ctx, const float *z, const int64_t *labels, int64_t rows,
                                   int64_t cols, const float *scale, float *dz, int acc) {
  if (!ctx) return TX_ERR_INVALID;
  if (rows <= 0) return TX_OK;
  k_xent_bwd<<<rows_grid(rows, 8), 256, 0, ctx->stream>>>(z, labels, scale, dz, rows, cols, acc);
  TX_LAUNCHED(ctx, "k_xent_bwd");
  return TX_OK;
}

int layernorm_fwd(tx_ctx *ctx, const float *x, const float *gamma, const float *beta, float *y, float *mean,
                  float *rstd, int64_t rows, int64_t cols, float eps, bool round_tf32) {
  if (rows <= 0) return TX_OK;
  if (ln_vec(cols, {x, gamma, beta, y})) {
    const unsigned blocks = rows_grid(rows, 8);
    const int rt = round_tf32 ? 1 : 0;
    switch (cols / 128) {
      case 1: k_layernorm_fwd_v<1><<<blocks, 256, 0, ctx->stream>>>(x, gamma, beta, y, mean, rstd, rows, eps, rt); break;
      case 2: k_layernorm_fwd_v<2><<<blocks, 256, 0, ctx->stream>>>(x, gamma, beta, y, mean, rstd, rows, eps, rt); break;
      case 4: k_layernorm_fwd_v<4><<<blocks, 256, 0, ctx->stream>>>(x, gamma, beta, y, mean, rstd, rows, eps, rt); break;
      case 8: k_layernorm_fwd_v<8><<<blocks, 256, 0, ctx->stream>>>(x, gamma, beta, y, mean, rstd, rows, eps, rt); break;
      default: goto scalar;
    }
    TX_LAUNCHED(ctx, "k_layernorm_fwd_v");
    return TX_OK;
  }
scalar:
  k_layernorm_fwd<<<rows_grid(rows, 8), 256, 0, ctx->stream>>>(x, gamma, beta, y, mean, rstd, rows,
                                                             cols, eps, round_tf32 ? 1 : 0);
  TX_LAUNCHED(ctx, "k_layernorm_fwd");
  return TX_OK;
}

extern "C" int tx_layernorm_fwd(tx_ctx *ctx, const float *x, const float *gamma, const float *beta,
                                float *y, float *mean, float *rstd, int64_t rows, int64_t cols,
                                float eps) {
  if (!ctx) return TX_ERR_INVALID;
  return layernorm_fwd(ctx, x, gamma, beta, y, mean, rstd, rows, cols, eps, false);
}

extern "C" int tx_layernorm_bwd(tx_ctx *ctx, const float *x, const float *gamma, const float *mean,
                                const float *rstd, const float *dy, float *dx, float *dgamma,
                                float *dbeta, int64_t rows, int64_t cols, int acc_dx, int acc_p) {
  if (!ctx) return TX_ERR_INVALID;
  if (rows <= 0) return TX_OK;
  const int vpl = (int)(cols / 128);
  if (ln_vec(cols, {x, gamma, dy, dx}) && (vpl == 1 || vpl == 2 || vpl == 4)) {
    int64_t blocks = (rows + 31) / 32;
    if (blocks > ctx->num_sms * 4) blocks = ctx->num_sms * 4;
    Scratch part(ctx, 2 * blocks * cols * sizeof(float));
    if (!part.ptr) return TX_ERR_OOM;
    float *pg = part.as<float>();
    float *pb = pg + blocks * cols;
    switch (vpl) {
      case 1: k_layernorm_bwd_v<1><<<(unsigned)blocks, 256, 0, ctx->stream>>>(x, gamma, mean, rstd, dy, dx, pg, pb, rows, acc_dx); break;
      case 2: k_layernorm_bwd_v<2><<<(unsigned)blocks, 256, 0, ctx->stream>>>(x, gamma, mean, rstd, dy, dx, pg, pb, rows, acc_dx); break;
      case 4: k_layernorm_bwd_v<4><<<(unsigned)blocks, 256, 0, ctx->stream>>>(x, gamma, mean, rstd, dy, dx, pg, pb, rows, acc_dx); break;
      default: k_layernorm_bwd_v<4><<<(unsigned)blocks, 256, 0, ctx->stream>>>(x, gamma, mean, rstd, dy, dx, pg, pb, rows, acc_dx); break;
    }
    TX_LAUNCHED(ctx, "k_layernorm_bwd_v");
    return colsum_finish2(ctx, pg, blocks, cols, dgamma, dbeta, 1.f, acc_p);  // pb follows pg
  }
  const int warps = 4;
  size_t smem = 2 * (size_t)warps * cols * sizeof(float);
  if (smem > 200 * 1024) return tx_fail(ctx, TX_ERR_UNSUPPORTED, "LayerNorm width too large");
  int64_t blocks = (rows + warps * 8 - 1) / (warps * 8);
  if (blocks > ctx->num_sms * 4) blocks = ctx->num_sms * 4;
  if (blocks < 1) blocks = 1;
  Scratch part(ctx, 2 * blocks * cols * sizeof(float));
  if (!part.ptr) return TX_ERR_OOM;
  float *pg = part.as<float>();
  float *pb = pg + blocks * cols;
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(k_layernorm_bwd, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  k_layernorm_bwd<<<(unsigned)blocks, warps * 32, smem, ctx->stream>>>(x, gamma, mean, rstd, dy, dx,
                                                                      pg, pb, rows, cols, acc_dx);
  TX_LAUNCHED(ctx, "k_layernorm_bwd");
  return colsum_finish2(ctx, pg, blocks, cols, dgamma, dbeta, 1.f, acc_p);  // pb follows pg
}

extern "C" int tx_gather_rows(tx_ctx *ctx, const float *table, int64_t rows, int64_t width,
                              const int64_t *idx, int64_t n, float *out) {
  if (!ctx) return TX_ERR_INVALID;
  if (n <= 0 || width <= 0) return TX_OK;
  bool vec = (width % 4 == 0) && ((((uintptr_t)table) | ((uintptr_t)out)) & 15) == 0;
  if (vec) {
    k_gather_rows4<<<grid_for(n * width / 4, 256), 256, 0, ctx->stream>>>(
        (const float4 *)table, rows, width / 4, idx, n, (float4 *)out, ctx->d_err);
  } else {
    k_gather_rows<<<grid_for(n * width, 256), 256, 0, ctx->stream>>>(table, rows, width, idx, n, out,
                                                                    ctx->d_err);
  }
  TX_LAUNCHED(ctx, "k_gather_rows");
  return TX_OK;
}

extern "C" int tx_scatter_add_rows(tx_ctx *ctx, float *table, int64_t rows, int64_t width,
                                   const int64_t *idx, int64_t n, const float *src) {
  if (!ctx) return TX_ERR_INVALID;
  if (n <= 0 || width <= 0) return TX_OK;
  k_scatter_add_rows<<<grid_for(n * width, 256), 256, 0, ctx->stream>>>(table, rows, width, idx, n, src);
  TX_LAUNCHED(ctx, "k_scatter_add_rows");
  return TX_OK;
}

extern "C" int tx_take_last(tx_ctx *ctx, const float *x, const int64_t *idx, float *out,
                            int64_t rows, int64_t cols) {
  if (!ctx) return TX_ERR_INVALID;
  if (rows <= 0) return TX_OK;
  k_take_last<<<grid_for(rows, 256), 256, 0, ctx->stream>>>(x, idx, out, rows, cols, ctx->d_err);
  TX_LAUNCHED(ctx, "k_take_last");
  return TX_OK;
}

extern "C" int tx_take_last_bwd(tx_ctx *ctx, const int64_t *idx, const float *dout, float *dx,
                                int64_t rows, int64_t cols, int acc) {
  if (!ctx) return TX_ERR_INVALID;
  if (rows <= 0) return TX_OK;
  k_take_last_bwd<<<grid_for(rows * cols, 256), 256, 0, ctx->stream>>>(idx, dout, dx, rows, cols, acc);
  TX_LAUNCHED(ctx, "k_take_last_bwd");
  return TX_OK;
}

extern "C" int tx_round_tf32(tx_ctx *ctx, const float *src, float *dst, int64_t n) {
  if (!ctx || (n > 0 && (!src || !dst))) return TX_ERR_INVALID;
  if (n <= 0) return TX_OK;
  k_round_tf32<<<grid_for((n + 3) / 4, 256), 256, 0, ctx->stream>>>(src, dst, n);
  TX_LAUNCHED(ctx, "k_round_tf32");
  return TX_OK;
}

extern "C" int tx_split_tf32(tx_ctx *ctx, const float *src, float *hi, float *lo, int64_t n) {
  if (!ctx || (n > 0 && (!src || !hi || !lo))) return TX_ERR_INVALID;
  if (n <= 0) return TX_OK;
  k_split_tf32<<<grid_for(n, 256), 256, 0, ctx->stream>>>(src, hi, lo, n);
  TX_LAUNCHED(ctx, "k_split_tf32");
  return TX_OK;
}

extern "C" int tx_bias_grad(tx_ctx *ctx, const float *dy, float *db, int64_t M, int64_t N,
                            float scale, int acc) {
  if (!ctx) return TX_ERR_INVALID;
  if (N <= 0) return TX_OK;
  if (M <= 0) {
    if (!acc) TX_CUDA(ctx, cudaMemsetAsync(db, 0, N * sizeof(float), ctx->stream));
    return TX_OK;
  }
  // split the rows so that the grid fills the machine
  const bool vec = (N % 4 == 0) && ((((uintptr_t)dy) & 15) == 0);
  int64_t col_blocks = vec ? (N + 127) / 128 : (N + 31) / 32;
  int64_t splits = (ctx->num_sms * 4 + col_blocks - 1) / col_blocks;
  int64_t max_splits = (M + 63) / 64;
  if (splits > max_splits) splits = max_splits;
  if (splits < 1) splits = 1;
  if (splits > 65535) splits = 65535;
  int64_t rows_per = (M + splits - 1) / splits;
  Scratch part(ctx, splits * N * sizeof(float));
  if (!part.ptr) return TX_ERR_OOM;
  if (vec)
    k_colsum_partial4<<<dim3((unsigned)col_blocks, (unsigned)splits), dim3(32, 8), 0, ctx->stream>>>(
        dy, M, N, rows_per, part.as<float>());
  else
    k_colsum_partial<<<dim3((unsigned)col_blocks, (unsigned)splits), dim3(32, 8), 0, ctx->stream>>>(
        dy, M, N, rows_per, part.as<float>());
  TX_LAUNCHED(ctx, "k_colsum_partial");
  TX_TRY(colsum_finish(ctx, part.as<float>(), splits, N, db, scale, acc));
  return TX_OK;
}

// ----------------------------------------------------------------------------
// optimizers
// ----------------------------------------------------------------------------
struct tx_optim {
  tx_ctx *ctx;
  tx_optim_cfg cfg;
  int n;
  std::vector<OptTensor> host_tensors;
  OptTensor *d_tensors = nullptr;
  int64_t *d_steps = nullptr;
  OptHparams *d_hp = nullptr;
  unsigned *d_ticket = nullptr;
  float *d_bc = nullptr;  // per tensor: the next update's two bias corrections (Adam)
  std::vector<float *> state;  // m, v, vmax per tensor (SGD: momentum in m)
  // chunk tables keyed by active mask
  std::map<std::vector<uint8_t>, std::pair<OptChunk *, int>> tables;
  std::map<std::vector<uint8_t>, std::pair<int32_t *, int>> active_lists;
};

// elements per optimizer block: 4 float4 per thread at 256 threads, and enough
// blocks (about 450 for 1.9 M parameters) to keep every SM streaming
static const int64_t kChunk = kChunk_;
static int build_table(tx_optim *o, const std::vector<uint8_t> &key);

// bias corrections of every tensor's next update from its step counter
static int refresh_bias_corrections(tx_optim *o) {
  if (o->cfg.kind == 2 || !o->d_bc) return TX_OK;
  k_adam_bc<<<grid_for(o->n, 128), 128, 0, o->ctx->stream>>>(o->d_steps, o->d_bc, o->n, o->cfg.beta1,
                                                             o->cfg.beta2);
  TX_LAUNCHED(o->ctx, "k_adam_bc");
  return TX_OK;
}

static int upload_hparams(tx_optim *o) {
  if (o->ctx->capturing)
    return tx_fail(o->ctx, TX_ERR_CAPTURE,
                   "optimizer hyper-parameters cannot change while a step is being captured");
  OptHparams h;
  const tx_optim_cfg &c = o->cfg;
  h.lr = (float)c.lr;
  h.beta1 = (float)c.beta1;
  h.beta2 = (float)c.beta2;
  h.eps = (float)c.eps;
  h.wd = (float)c.weight_decay;
  h.one_minus_b1 = (float)(1.0 - c.beta1);
  h.one_minus_b2 = (float)(1.0 - c.beta2);
  h.decay_factor = (float)(1.0 - c.lr * c.weight_decay);
  h.beta1_d = c.beta1;
  h.beta2_d = c.beta2;
  h.momentum = (float)c.momentum;
  h.one_minus_dampening = (float)(1.0 - c.dampening);
  // stream-ordered after earlier steps that read the old values
  TX_CUDA(o->ctx, cudaMemcpyAsync(o->d_hp, &h, sizeof h, cudaMemcpyHostToDevice, o->ctx->stream));
  TX_TRY(refresh_bias_corrections(o));
  TX_CUDA(o->ctx, cudaStreamSynchronize(o->ctx->stream));
  return TX_OK;
}

extern "C" int tx_optim_create(tx_ctx *ctx, const tx_optim_cfg *cfg, int n, float *const *values,
                               float *const *grads, const int64_t *numel, tx_optim **out) {
  if (!ctx || !cfg || !out || n <= 0) return TX_ERR_INVALID;
  if (ctx->capturing) return tx_fail(ctx, TX_ERR_CAPTURE, "optimizer creation is not capturable");
  tx_optim *o = new tx_optim();
  o->ctx = ctx;
  o->cfg = *cfg;
  o->n = n;
  for (int i = 0; i < n; ++i) {
    OptTensor t{values[i], grads[i], nullptr, nullptr, nullptr, numel[i]};
    size_t bytes = numel[i] * sizeof(float);
    int nstate = cfg->kind == 2 ? (cfg->momentum != 0.0 ? 1 : 0) : (cfg->amsgrad ? 3 : 2);
    float *bufs[3] = {nullptr, nullptr, nullptr};
    for (int s = 0; s < nstate; ++s) {
      if (cudaMalloc(&bufs[s], bytes ? bytes : 4) != cudaSuccess) {
        delete o;
        return tx_fail(ctx, TX_ERR_OOM, "optimizer state allocation failed");
      }
      cudaMemsetAsync(bufs[s], 0, bytes ? bytes : 4, ctx->stream);
    }
    t.m = bufs[0];
    t.v = bufs[1];
    t.vmax = bufs[2];
    o->state.push_back(bufs[0]);
    o->state.push_back(bufs[1]);
    o->state.push_back(bufs[2]);
    o->host_tensors.push_back(t);
  }
  TX_CUDA(ctx, cudaMalloc(&o->d_tensors, n * sizeof(OptTensor)));
  TX_CUDA(ctx, cudaMalloc(&o->d_steps, n * sizeof(int64_t)));
  TX_CUDA(ctx, cudaMalloc(&o->d_hp, sizeof(OptHparams)));
  TX_CUDA(ctx, cudaMalloc(&o->d_ticket, sizeof(unsigned)));
  TX_CUDA(ctx, cudaMalloc(&o->d_bc, 2 * n * sizeof(float)));
  TX_CUDA(ctx, cudaMemcpyAsync(o->d_tensors, o->host_tensors.data(), n * sizeof(OptTensor),
                               cudaMemcpyHostToDevice, ctx->stream));
  TX_CUDA(ctx, cudaMemsetAsync(o->d_steps, 0, n * sizeof(int64_t), ctx->stream));
  TX_CUDA(ctx, cudaMemsetAsync(o->d_ticket, 0, sizeof(unsigned), ctx->stream));
  int rc = upload_hparams(o);
  if (rc) {
    delete o;
    return rc;
  }
  *out = o;
  // the chunk table for "every tensor has a gradient" is built up front so a
  // captured step never has to create one
  std::vector<uint8_t> all(n, 1);
  return build_table(o, all);
}

extern "C" int tx_optim_set_hparams(tx_optim *o, const tx_optim_cfg *cfg) {
  if (!o || !cfg) return TX_ERR_INVALID;
  if (cfg->kind != o->cfg.kind || cfg->amsgrad != o->cfg.amsgrad)
    return tx_fail(o->ctx, TX_ERR_INVALID, "optimizer kind and amsgrad cannot change");
  o->cfg = *cfg;
  return upload_hparams(o);
}

extern "C" int tx_optim_set_lr(tx_optim *o, double lr) {
  if (!o) return TX_ERR_INVALID;
  o->cfg.lr = lr;
  return upload_hparams(o);
}

static int build_table(tx_optim *o, const std::vector<uint8_t> &key) {
  tx_ctx *ctx = o->ctx;
  const uint8_t *active = key.data();
  {
    std::vector<OptChunk> chunks;
    std::vector<int32_t> list;
    for (int i = 0; i < o->n; ++i) {
      if (!active[i]) continue;
      list.push_back(i);
      for (int64_t s = 0; s < o->host_tensors[i].n; s += kChunk) {
        int64_t len = o->host_tensors[i].n - s < kChunk ? o->host_tensors[i].n - s : kChunk;
        chunks.push_back({i, s, len});
      }
    }
    OptChunk *d_chunks = nullptr;
    int32_t *d_list = nullptr;
    if (!chunks.empty()) {
      TX_CUDA(ctx, cudaMalloc(&d_chunks, chunks.size() * sizeof(OptChunk)));
      TX_CUDA(ctx, cudaMalloc(&d_list, list.size() * sizeof(int32_t)));
      TX_CUDA(ctx, cudaMemcpy(d_chunks, chunks.data(), chunks.size() * sizeof(OptChunk),
                              cudaMemcpyHostToDevice));
      TX_CUDA(ctx, cudaMemcpy(d_list, list.data(), list.size() * sizeof(int32_t),
                              cudaMemcpyHostToDevice));
    }
    o->tables.emplace(key, std::make_pair(d_chunks, (int)chunks.size()));
    o->active_lists[key] = {d_list, (int)list.size()};
  }
  return TX_OK;
}

extern "C" int tx_optim_step(tx_optim *o, const uint8_t *active) {
  if (!o) return TX_ERR_INVALID;
  tx_ctx *ctx = o->ctx;
  std::vector<uint8_t> key(active, active + o->n);
  auto it = o->tables.find(key);
  if (it == o->tables.end()) {
    TX_TRY(build_table(o, key));
    it = o->tables.find(key);
  }
  int n_chunks = it->second.second;
  if (n_chunks == 0) return TX_OK;
  auto al = o->active_lists[key];
  if (o->cfg.kind == 2) {
    k_sgd<<<n_chunks, 256, 0, ctx->stream>>>(o->d_tensors, it->second.first, o->d_hp, o->d_steps,
                                             n_chunks, al.first, al.second, o->cfg.nesterov,
                                             o->d_ticket);
  } else {
    const int64_t pieces = (int64_t)n_chunks * (kChunk / kAdamSub);
    static int per_sm[64] = {};  // resident 256-thread CTAs per SM, per device
    if (!per_sm[ctx->device & 63]) {
      int nb = 0;
      TX_CUDA(ctx, cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, k_adam, 256, 0));
      per_sm[ctx->device & 63] = nb > 0 ? nb : 1;
    }
    const int64_t wave = (int64_t)ctx->num_sms * per_sm[ctx->device & 63];
    k_adam<<<(unsigned)(pieces < wave ? pieces : wave), 256, 0, ctx->stream>>>(
        o->d_tensors, it->second.first, n_chunks, o->d_hp, o->d_steps, o->d_bc, al.first, al.second,
        o->cfg.kind, o->cfg.amsgrad, o->d_ticket);
  }
  TX_LAUNCHED(ctx, "optimizer step");
  return TX_OK;
}

extern "C" int tx_optim_state_ptr(tx_optim *o, int tensor, int which, float **out) {
  if (!o || !out || tensor < 0 || tensor >= o->n || which < 0 || which > 3) return TX_ERR_INVALID;
  if (which == 3) which = 0;  // SGD momentum lives in slot 0
  *out = o->state[tensor * 3 + which];
  return *out ? TX_OK : TX_ERR_INVALID;
}

extern "C" int tx_optim_get_steps(tx_optim *o, int64_t *h) {
  if (!o || !h) return TX_ERR_INVALID;
  TX_CUDA(o->ctx, cudaMemcpyAsync(h, o->d_steps, o->n * sizeof(int64_t), cudaMemcpyDeviceToHost,
                                  o->ctx->stream));
  TX_CUDA(o->ctx, cudaStreamSynchronize(o->ctx->stream));
  return TX_OK;
}

extern "C" int tx_optim_set_steps(tx_optim *o, const int64_t *h) {
  if (!o || !h) return TX_ERR_INVALID;
  TX_CUDA(o->ctx, cudaMemcpyAsync(o->d_steps, h, o->n * sizeof(int64_t), cudaMemcpyHostToDevice,
                                  o->ctx->stream));
  TX_TRY(refresh_bias_corrections(o));
  TX_CUDA(o->ctx, cudaStreamSynchronize(o->ctx->stream));
  return TX_OK;
}

extern "C" int tx_optim_destroy(tx_optim *o) {
  if (!o) return TX_OK;
  cudaStreamSynchronize(o->ctx->stream);
  for (float *p : o->state)
    if (p) cudaFree(p);
  for (auto &kv : o->tables)
    if (kv.second.first) cudaFree(kv.second.first);
  for (auto &kv : o->active_lists)
    if (kv.second.first) cudaFree(kv.second.first);
  cudaFree(o->d_tensors);
  cudaFree(o->d_steps);
  cudaFree(o->d_hp);
  cudaFree(o->d_ticket);
  cudaFree(o->d_bc);
  delete o;
  return TX_OK;
}
