// Trainable operators beyond the five configurations: PRelu, BatchNormalization
// with fixed running statistics, Instance / GroupNormalization and 2-D MaxPool,
// forward and backward (the training registry of
// crates/tynx-train/src/backward_support.rs:106-179).
//
// All of them are bandwidth-bound: one pass over the input (plus the output)
// per kernel, 32-bit per-element index math where the sizes allow it, and
// fixed-order reductions so that a step is reproducible run to run.
//
// Arithmetic follows the composed Burn ops of the reference operation by
// operation (each f32 op rounded on its own: __fadd_rn / __fmul_rn / __fdiv_rn
// keep nvcc from contracting them into FMAs), so the forward results equal the
// reference's f32 values:
//   BatchNormalization  ((x - mean) / sqrt(var + eps)) * scale + bias
//                       (crates/tynx/src/interpreter/normalization.rs:20-58)
//   Instance / Group    centred = x - mean(x); var = mean(centred^2);
//                       (centred / sqrt(var + eps)) * scale + bias over each
//                       (sample, group) (normalization.rs:73-106, 213-273)
//   PRelu               x >= 0 ? x : slope * x (crates/tynx/src/tensor.rs:1911-1934)
//   MaxPool2d           max over the window of the -inf padded input
//                       (crates/tynx/src/interpreter/pooling.rs:360-426); the
//                       gradient goes to the first maximal tap in window order.
#include <cmath>

#include "common.h"

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float block_sum(float v, float *sh) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();  // sh may still be read by a previous call
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x < 32) {
    t = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.f;
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) sh[0] = t;
  }
  __syncthreads();
  return sh[0];
}

// ---- BatchNormalization with fixed statistics ------------------------------------------------
__global__ void k_bn_fwd(const float *__restrict__ x, const float *__restrict__ scale,
                         const float *__restrict__ bias, const float *__restrict__ mean,
                         const float *__restrict__ var, float *__restrict__ y, int64_t n, int64_t C,
                         int64_t L, float eps) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c = (i / L) % C;
    const float sd = __fsqrt_rn(__fadd_rn(var[c], eps));
    const float t = __fdiv_rn(__fsub_rn(x[i], mean[c]), sd);
    y[i] = __fadd_rn(__fmul_rn(t, scale[c]), bias[c]);
  }
}

// dx = (dy * scale) / sd; per (sample, channel) partial sums of dy * t and dy
// over the L positions, one warp per (n, c) row
__global__ void k_bn_bwd(const float *__restrict__ x, const float *__restrict__ dy,
                         const float *__restrict__ scale, const float *__restrict__ mean,
                         const float *__restrict__ var, float *__restrict__ dx, float *__restrict__ ps,
                         float *__restrict__ pb, int64_t rows, int64_t C, int64_t L, float eps, int acc) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    const int64_t c = r % C;
    const float sd = __fsqrt_rn(__fadd_rn(var[c], eps));
    const float m = mean[c], s = scale[c];
    float ss = 0.f, sb = 0.f;
    for (int64_t j = lane; j < L; j += 32) {
      const int64_t i = r * L + j;
      const float g = dy[i];
      if (dx) {
        const float v = __fdiv_rn(__fmul_rn(g, s), sd);
        dx[i] = acc ? __fadd_rn(dx[i], v) : v;
      }
      if (ps) {
        const float t = __fdiv_rn(__fsub_rn(x[i], m), sd);
        ss += g * t;
        sb += g;
      }
    }
    if (ps) {
      for (int o = 16; o > 0; o >>= 1) {
        ss += __shfl_xor_sync(0xffffffffu, ss, o);
        sb += __shfl_xor_sync(0xffffffffu, sb, o);
      }
      if (lane == 0) {
        ps[r] = ss;
        pb[r] = sb;
      }
    }
  }
}

// out[c] (+)= sum over n of part[n][c], in order of n
__global__ void k_sum_over_rows(const float *__restrict__ part, float *__restrict__ out, int64_t N, int64_t C,
                                int acc) {
  for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < C; c += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int64_t n = 0; n < N; ++n) s += part[n * C + c];
    out[c] = acc ? out[c] + s : s;
  }
}

// ---- Instance / Group normalization ----------------------------------------------------------
// x viewed as [N][G][cpg][L]; one block per (n, g) row of cpg * L elements.
__global__ void k_groupnorm_fwd(const float *__restrict__ x, const float *__restrict__ scale,
                                const float *__restrict__ bias, float *__restrict__ y, float *__restrict__ mean,
                                float *__restrict__ sdev, int64_t G, int64_t cpg, int64_t L, float eps) {
  __shared__ float sh[32];
  const int64_t row = blockIdx.x;
  const int64_t len = cpg * L;
  const float *xr = x + row * len;
  float s = 0.f;
  for (int64_t j = threadIdx.x; j < len; j += blockDim.x) s += xr[j];
  const float mu = __fdiv_rn(block_sum(s, sh), (float)len);
  float q = 0.f;
  for (int64_t j = threadIdx.x; j < len; j += blockDim.x) {
    const float c = __fsub_rn(xr[j], mu);
    q += c * c;
  }
  const float var = __fdiv_rn(block_sum(q, sh), (float)len);
  const float sd = __fsqrt_rn(__fadd_rn(var, eps));
  if (threadIdx.x == 0) {
    mean[row] = mu;
    sdev[row] = sd;
  }
  const int64_t g = row % G;
  float *yr = y + row * len;
  for (int64_t j = threadIdx.x; j < len; j += blockDim.x) {
    const int64_t ch = g * cpg + j / L;
    const float t = __fdiv_rn(__fsub_rn(xr[j], mu), sd);
    yr[j] = __fadd_rn(__fmul_rn(t, scale[ch]), bias[ch]);
  }
}

// dx = (dxh - mean(dxh) - xh * mean(dxh * xh)) / sd with dxh = dy * scale[ch];
// partial sums of dy * xh and dy per (n, channel) for the affine gradients.
__global__ void k_groupnorm_bwd(const float *__restrict__ x, const float *__restrict__ dy,
                                const float *__restrict__ scale, const float *__restrict__ mean,
                                const float *__restrict__ sdev, float *__restrict__ dx, float *__restrict__ ps,
                                float *__restrict__ pb, int64_t G, int64_t cpg, int64_t L, int acc) {
  __shared__ float sh[32];
  const int64_t row = blockIdx.x;
  const int64_t len = cpg * L;
  const int64_t g = row % G, n = row / G;
  const float mu = mean[row], sd = sdev[row];
  const float *xr = x + row * len, *dyr = dy + row * len;
  if (dx) {
    float a = 0.f, b = 0.f;
    for (int64_t j = threadIdx.x; j < len; j += blockDim.x) {
      const float xh = __fdiv_rn(__fsub_rn(xr[j], mu), sd);
      const float dxh = dyr[j] * scale[g * cpg + j / L];
      a += dxh;
      b += dxh * xh;
    }
    const float ma = block_sum(a, sh) / (float)len;
    const float mb = block_sum(b, sh) / (float)len;
    float *dxr = dx + row * len;
    for (int64_t j = threadIdx.x; j < len; j += blockDim.x) {
      const float xh = __fdiv_rn(__fsub_rn(xr[j], mu), sd);
      const float dxh = dyr[j] * scale[g * cpg + j / L];
      const float v = (dxh - ma - xh * mb) / sd;
      dxr[j] = acc ? dxr[j] + v : v;
    }
  }
  if (ps) {
    const int64_t C = G * cpg;
    for (int64_t k = 0; k < cpg; ++k) {
      float a = 0.f, b = 0.f;
      for (int64_t j = threadIdx.x; j < L; j += blockDim.x) {
        const int64_t i = k * L + j;
        const float xh = __fdiv_rn(__fsub_rn(xr[i], mu), sd);
        a += dyr[i] * xh;
        b += dyr[i];
      }
      a = block_sum(a, sh);
      b = block_sum(b, sh);
      if (threadIdx.x == 0) {
        ps[n * C + g * cpg + k] = a;
        pb[n * C + g * cpg + k] = b;
      }
    }
  }
}

// ---- PRelu --------------------------------------------------------------------------------------
struct Bcast {
  int64_t shape[TX_MAX_DIMS];
  int64_t s[TX_MAX_DIMS];  // slope strides over the output shape (0 = broadcast)
  int nd;
};

__device__ __forceinline__ int64_t bcast_index(const Bcast &b, int64_t i) {
  int64_t off = 0;
  for (int k = b.nd - 1; k >= 0; --k) {
    const int64_t e = b.shape[k];
    off += (i % e) * b.s[k];
    i /= e;
  }
  return off;
}

__global__ void k_prelu_fwd(const float *__restrict__ x, const float *__restrict__ slope, Bcast b,
                            float *__restrict__ y, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    y[i] = v >= 0.f ? v : __fmul_rn(v, slope[bcast_index(b, i)]);
  }
}

// dx = x >= 0 ? dy : dy * slope; tmp = x >= 0 ? 0 : dy * x (summed to the slope's shape after)
__global__ void k_prelu_bwd(const float *__restrict__ x, const float *__restrict__ slope, Bcast b,
                            const float *__restrict__ dy, float *__restrict__ dx, float *__restrict__ tmp,
                            int64_t n, int acc) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = x[i], g = dy[i];
    const bool pos = v >= 0.f;
    if (dx) {
      const float d = pos ? g : __fmul_rn(g, slope[bcast_index(b, i)]);
      dx[i] = acc ? __fadd_rn(dx[i], d) : d;
    }
    if (tmp) tmp[i] = pos ? 0.f : __fmul_rn(g, v);
  }
}

// ---- MaxPool2d --------------------------------------------------------------------------------
struct PoolGeom {
  int H, W, OH, OW, KH, KW, SH, SW, PT, PL, DH, DW;
};

__global__ void k_maxpool_fwd(const float *__restrict__ x, float *__restrict__ y, int32_t *__restrict__ arg,
                              PoolGeom p, int64_t planes) {
  const int64_t n = planes * p.OH * p.OW;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int ow = (int)(i % p.OW);
    const int oh = (int)((i / p.OW) % p.OH);
    const int64_t plane = i / ((int64_t)p.OW * p.OH);
    const float *xp = x + plane * (int64_t)p.H * p.W;
    float best = -INFINITY;
    int at = -1;
    for (int kh = 0; kh < p.KH; ++kh) {
      const int h = oh * p.SH - p.PT + kh * p.DH;
      if (h < 0 || h >= p.H) continue;
      for (int kw = 0; kw < p.KW; ++kw) {
        const int w = ow * p.SW - p.PL + kw * p.DW;
        if (w < 0 || w >= p.W) continue;
        const float v = xp[h * p.W + w];
        if (v > best || at < 0) {  // first maximal tap in window order; NaN never wins
          best = v;
          at = h * p.W + w;
        }
      }
    }
    y[i] = best;
    arg[i] = at;
  }
}

// Gather form: each input element sums the output gradients whose window chose
// it, in (kh, kw) order, so the result is deterministic.
__global__ void k_maxpool_bwd(const float *__restrict__ dy, const int32_t *__restrict__ arg,
                              float *__restrict__ dx, PoolGeom p, int64_t planes, int acc) {
  const int64_t n = planes * p.H * p.W;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int w = (int)(i % p.W);
    const int h = (int)((i / p.W) % p.H);
    const int64_t plane = i / ((int64_t)p.W * p.H);
    const int pos = h * p.W + w;
    const float *dyp = dy + plane * (int64_t)p.OH * p.OW;
    const int32_t *ap = arg + plane * (int64_t)p.OH * p.OW;
    float s = 0.f;
    for (int kh = 0; kh < p.KH; ++kh) {
      const int th = h + p.PT - kh * p.DH;
      if (th < 0 || th % p.SH) continue;
      const int oh = th / p.SH;
      if (oh >= p.OH) continue;
      for (int kw = 0; kw < p.KW; ++kw) {
        const int tw = w + p.PL - kw * p.DW;
        if (tw < 0 || tw % p.SW) continue;
        const int ow = tw / p.SW;
        if (ow >= p.OW) continue;
        if (ap[oh * p.OW + ow] == pos) s += dyp[oh * p.OW + ow];
      }
    }
    dx[i] = acc ? dx[i] + s : s;
  }
}

int check_launch(tx_ctx *ctx, const char *name) {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TX_OK : tx_cuda_fail(ctx, e, name);
}

}  // namespace

// ---- C ABI -------------------------------------------------------------------------------------

extern "C" int tx_batchnorm_fwd(tx_ctx *ctx, const float *x, const float *scale, const float *bias,
                                const float *mean, const float *var, float *y, int64_t N, int64_t C,
                                int64_t L, float eps) {
  if (!ctx || N < 0 || C <= 0 || L <= 0) return TX_ERR_INVALID;
  const int64_t n = N * C * L;
  if (n == 0) return TX_OK;
  k_bn_fwd<<<grid_for(n, kThreads), kThreads, 0, ctx->stream>>>(x, scale, bias, mean, var, y, n, C, L, eps);
  return check_launch(ctx, "k_bn_fwd");
}

extern "C" int tx_batchnorm_bwd(tx_ctx *ctx, const float *x, const float *dy, const float *scale,
                                const float *mean, const float *var, float *dx, float *dscale, float *dbias,
                                int64_t N, int64_t C, int64_t L, float eps, int acc_dx, int acc_params) {
  if (!ctx || N < 0 || C <= 0 || L <= 0 || ((dscale == nullptr) != (dbias == nullptr))) return TX_ERR_INVALID;
  const int64_t rows = N * C;
  if (rows == 0) {
    if (dscale && !acc_params) {
      TX_CUDA(ctx, cudaMemsetAsync(dscale, 0, C * 4, ctx->stream));
      TX_CUDA(ctx, cudaMemsetAsync(dbias, 0, C * 4, ctx->stream));
    }
    return TX_OK;
  }
  Scratch part(ctx, dscale ? (size_t)rows * 8 : 0);
  if (dscale && !part.ptr) return TX_ERR_OOM;
  float *ps = dscale ? part.as<float>() : nullptr, *pb = dscale ? part.as<float>() + rows : nullptr;
  k_bn_bwd<<<grid_for(rows * 32, kThreads), kThreads, 0, ctx->stream>>>(x, dy, scale, mean, var, dx, ps, pb,
                                                                        rows, C, L, eps, acc_dx);
  TX_TRY(check_launch(ctx, "k_bn_bwd"));
  if (dscale) {
    k_sum_over_rows<<<grid_for(C, kThreads), kThreads, 0, ctx->stream>>>(ps, dscale, N, C, acc_params);
    k_sum_over_rows<<<grid_for(C, kThreads), kThreads, 0, ctx->stream>>>(pb, dbias, N, C, acc_params);
    TX_TRY(check_launch(ctx, "k_sum_over_rows"));
  }
  return TX_OK;
}

extern "C" int tx_groupnorm_fwd(tx_ctx *ctx, const float *x, const float *scale, const float *bias, float *y,
                                float *mean, float *sdev, int64_t N, int64_t C, int64_t L, int64_t groups,
                                float eps) {
  if (!ctx || N < 0 || C <= 0 || L <= 0 || groups <= 0 || C % groups) return TX_ERR_INVALID;
  const int64_t rows = N * groups;
  if (rows == 0) return TX_OK;
  if (rows > 0x7fffffff) return tx_fail(ctx, TX_ERR_UNSUPPORTED, "GroupNormalization: too many rows");
  k_groupnorm_fwd<<<(unsigned)rows, kThreads, 0, ctx->stream>>>(x, scale, bias, y, mean, sdev, groups,
                                                                C / groups, L, eps);
  return check_launch(ctx, "k_groupnorm_fwd");
}

extern "C" int tx_groupnorm_bwd(tx_ctx *ctx, const float *x, const float *dy, const float *scale,
                                const float *mean, const float *sdev, float *dx, float *dscale, float *dbias,
                                int64_t N, int64_t C, int64_t L, int64_t groups, int acc_dx, int acc_params) {
  if (!ctx || N < 0 || C <= 0 || L <= 0 || groups <= 0 || C % groups ||
      ((dscale == nullptr) != (dbias == nullptr)))
    return TX_ERR_INVALID;
  const int64_t rows = N * groups;
  if (rows == 0) {
    if (dscale && !acc_params) {
      TX_CUDA(ctx, cudaMemsetAsync(dscale, 0, C * 4, ctx->stream));
      TX_CUDA(ctx, cudaMemsetAsync(dbias, 0, C * 4, ctx->stream));
    }
    return TX_OK;
  }
  if (rows > 0x7fffffff) return tx_fail(ctx, TX_ERR_UNSUPPORTED, "GroupNormalization: too many rows");
  Scratch part(ctx, dscale ? (size_t)N * C * 8 : 0);
  if (dscale && !part.ptr) return TX_ERR_OOM;
  float *ps = dscale ? part.as<float>() : nullptr, *pb = dscale ? part.as<float>() + N * C : nullptr;
  k_groupnorm_bwd<<<(unsigned)rows, kThreads, 0, ctx->stream>>>(x, dy, scale, mean, sdev, dx, ps, pb, groups,
                                                                C / groups, L, acc_dx);
  TX_TRY(check_launch(ctx, "k_groupnorm_bwd"));
  if (dscale) {
    k_sum_over_rows<<<grid_for(C, kThreads), kThreads, 0, ctx->stream>>>(ps, dscale, N, C, acc_params);
    k_sum_over_rows<<<grid_for(C, kThreads), kThreads, 0, ctx->stream>>>(pb, dbias, N, C, acc_params);
    TX_TRY(check_launch(ctx, "k_sum_over_rows"));
  }
  return TX_OK;
}

static int make_bcast(tx_ctx *ctx, const int64_t *shape, const int64_t *slope_strides, int ndim, Bcast *b,
                      int64_t *n) {
  if (ndim < 0 || ndim > TX_MAX_DIMS) return tx_fail(ctx, TX_ERR_INVALID, "PRelu rank above 8");
  b->nd = ndim;
  *n = 1;
  for (int i = 0; i < ndim; ++i) {
    if (shape[i] < 0) return TX_ERR_INVALID;
    b->shape[i] = shape[i] > 0 ? shape[i] : 1;
    b->s[i] = slope_strides[i];
    *n *= shape[i];
  }
  return TX_OK;
}

extern "C" int tx_prelu_fwd(tx_ctx *ctx, const float *x, const float *slope, const int64_t *slope_strides,
                            float *y, const int64_t *shape, int ndim) {
  if (!ctx || !shape || !slope_strides) return TX_ERR_INVALID;
  Bcast b;
  int64_t n;
  TX_TRY(make_bcast(ctx, shape, slope_strides, ndim, &b, &n));
  if (n == 0) return TX_OK;
  k_prelu_fwd<<<grid_for(n, kThreads), kThreads, 0, ctx->stream>>>(x, slope, b, y, n);
  return check_launch(ctx, "k_prelu_fwd");
}

extern "C" int tx_prelu_bwd(tx_ctx *ctx, const float *x, const float *slope, const int64_t *slope_strides,
                            const float *dy, float *dx, float *dslope_full, const int64_t *shape, int ndim,
                            int acc_dx) {
  if (!ctx || !shape || !slope_strides) return TX_ERR_INVALID;
  Bcast b;
  int64_t n;
  TX_TRY(make_bcast(ctx, shape, slope_strides, ndim, &b, &n));
  if (n == 0) return TX_OK;
  k_prelu_bwd<<<grid_for(n, kThreads), kThreads, 0, ctx->stream>>>(x, slope, b, dy, dx, dslope_full, n, acc_dx);
  return check_launch(ctx, "k_prelu_bwd");
}

// ---- average pooling (ONNX AveragePool; the inference arm of
// crates/tynx/src/interpreter/pooling.rs) --------------------------------------------------
// The divisor of a window is the number of its taps inside the input, or with
// count_include_pad the number inside the padded input [-PT, H + PB) x
// [-PL, W + PR) (a ceil-mode window that runs past the padding counts only
// what it covers).
__device__ __forceinline__ int avg_count(const PoolGeom &p, int oh, int ow, int pb, int pr, int include_pad) {
  const int lo_h = include_pad ? -p.PT : 0, hi_h = include_pad ? p.H + pb : p.H;
  const int lo_w = include_pad ? -p.PL : 0, hi_w = include_pad ? p.W + pr : p.W;
  int ch = 0, cw = 0;
  for (int kh = 0; kh < p.KH; ++kh) {
    const int h = oh * p.SH - p.PT + kh * p.DH;
    ch += h >= lo_h && h < hi_h;
  }
  for (int kw = 0; kw < p.KW; ++kw) {
    const int w = ow * p.SW - p.PL + kw * p.DW;
    cw += w >= lo_w && w < hi_w;
  }
  return ch * cw;
}

__global__ void k_avgpool_fwd(const float *__restrict__ x, float *__restrict__ y, PoolGeom p, int64_t planes,
                              int pb, int pr, int include_pad) {
  const int64_t n = planes * p.OH * p.OW;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int ow = (int)(i % p.OW);
    const int oh = (int)((i / p.OW) % p.OH);
    const int64_t plane = i / ((int64_t)p.OW * p.OH);
    const float *xp = x + plane * (int64_t)p.H * p.W;
    float sum = 0.f;
    for (int kh = 0; kh < p.KH; ++kh) {
      const int h = oh * p.SH - p.PT + kh * p.DH;
      if (h < 0 || h >= p.H) continue;
      for (int kw = 0; kw < p.KW; ++kw) {
        const int w = ow * p.SW - p.PL + kw * p.DW;
        if (w >= 0 && w < p.W) sum += xp[h * p.W + w];
      }
    }
    const int cnt = avg_count(p, oh, ow, pb, pr, include_pad);
    y[i] = cnt > 0 ? sum / (float)cnt : 0.f;
  }
}

// dx[h][w] (+)= sum over the windows that read (h, w) of dy / count (gather form)
__global__ void k_avgpool_bwd(const float *__restrict__ dy, float *__restrict__ dx, PoolGeom p, int64_t planes,
                              int pb, int pr, int include_pad, int acc) {
  const int64_t n = planes * p.H * p.W;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int w = (int)(i % p.W);
    const int h = (int)((i / p.W) % p.H);
    const int64_t plane = i / ((int64_t)p.W * p.H);
    const float *dp = dy + plane * (int64_t)p.OH * p.OW;
    float s = 0.f;
    for (int kh = 0; kh < p.KH; ++kh) {
      const int a = h + p.PT - kh * p.DH;
      if (a < 0 || a % p.SH) continue;
      const int oh = a / p.SH;
      if (oh >= p.OH) continue;
      for (int kw = 0; kw < p.KW; ++kw) {
        const int b = w + p.PL - kw * p.DW;
        if (b < 0 || b % p.SW) continue;
        const int ow = b / p.SW;
        if (ow >= p.OW) continue;
        const int cnt = avg_count(p, oh, ow, pb, pr, include_pad);
        if (cnt > 0) s += dp[oh * p.OW + ow] / (float)cnt;
      }
    }
    dx[i] = acc ? dx[i] + s : s;
  }
}

static int pool_geom(tx_ctx *ctx, int64_t H, int64_t W, const int64_t *g, PoolGeom *p) {
  // g: kh, kw, sh, sw, pt, pl, dh, dw, oh, ow
  for (int i = 0; i < 10; ++i)
    if (g[i] < 0 || g[i] > 0x3fffffff) return tx_fail(ctx, TX_ERR_INVALID, "MaxPool geometry out of range");
  if (g[0] == 0 || g[1] == 0 || g[2] == 0 || g[3] == 0 || g[6] == 0 || g[7] == 0 || H > 0x3fffffff ||
      W > 0x3fffffff || H * W > 0x7fffffff)
    return tx_fail(ctx, TX_ERR_INVALID, "MaxPool geometry out of range");
  *p = PoolGeom{(int)H, (int)W, (int)g[8], (int)g[9], (int)g[0], (int)g[1], (int)g[2],
                (int)g[3], (int)g[4], (int)g[5], (int)g[6], (int)g[7]};
  return TX_OK;
}

extern "C" int tx_maxpool2d_fwd(tx_ctx *ctx, const float *x, float *y, int32_t *argmax, int64_t planes,
                                int64_t H, int64_t W, const int64_t *geom) {
  if (!ctx || !geom || planes < 0) return TX_ERR_INVALID;
  PoolGeom p;
  TX_TRY(pool_geom(ctx, H, W, geom, &p));
  const int64_t n = planes * p.OH * p.OW;
  if (n == 0) return TX_OK;
  k_maxpool_fwd<<<grid_for(n, kThreads), kThreads, 0, ctx->stream>>>(x, y, argmax, p, planes);
  return check_launch(ctx, "k_maxpool_fwd");
}

extern "C" int tx_maxpool2d_bwd(tx_ctx *ctx, const float *dy, const int32_t *argmax, float *dx, int64_t planes,
                                int64_t H, int64_t W, const int64_t *geom, int acc) {
  if (!ctx || !geom || planes < 0) return TX_ERR_INVALID;
  PoolGeom p;
  TX_TRY(pool_geom(ctx, H, W, geom, &p));
  const int64_t n = planes * p.H * p.W;
  if (n == 0) return TX_OK;
  k_maxpool_bwd<<<grid_for(n, kThreads), kThreads, 0, ctx->stream>>>(dy, argmax, dx, p, planes, acc);
  return check_launch(ctx, "k_maxpool_bwd");
}

// geom: as tx_maxpool2d_fwd, then the bottom and right padding (pb, pr)
extern "C" int tx_avgpool2d_fwd(tx_ctx *ctx, const float *x, float *y, int64_t planes, int64_t H, int64_t W,
                                const int64_t *geom, int count_include_pad) {
  if (!ctx || !geom || planes < 0 || geom[10] < 0 || geom[11] < 0) return TX_ERR_INVALID;
  PoolGeom p;
  TX_TRY(pool_geom(ctx, H, W, geom, &p));
  const int64_t n = planes * p.OH * p.OW;
  if (n == 0) return TX_OK;
  k_avgpool_fwd<<<grid_for(n, kThreads), kThreads, 0, ctx->stream>>>(x, y, p, planes, (int)geom[10], (int)geom[11],
                                                                     count_include_pad);
  return check_launch(ctx, "k_avgpool_fwd");
}

extern "C" int tx_avgpool2d_bwd(tx_ctx *ctx, const float *dy, float *dx, int64_t planes, int64_t H, int64_t W,
                                const int64_t *geom, int count_include_pad, int acc) {
  if (!ctx || !geom || planes < 0 || geom[10] < 0 || geom[11] < 0) return TX_ERR_INVALID;
  PoolGeom p;
  TX_TRY(pool_geom(ctx, H, W, geom, &p));
  const int64_t n = planes * p.H * p.W;
  if (n == 0) return TX_OK;
  k_avgpool_bwd<<<grid_for(n, kThreads), kThreads, 0, ctx->stream>>>(dy, dx, p, planes, (int)geom[10],
                                                                     (int)geom[11], count_include_pad, acc);
  return check_launch(ctx, "k_avgpool_bwd");
}
