// Imported-graph engine: forward node loop, reverse tape, parameter slots.
//
// Replaces, for the CUDA placement:
//   * executor::run (crates/tynx-train/src/imported_model/executor.rs:107-161) -- the
//     topological node loop with live parameter slots (resolve_value 555-593);
//   * the Burn autodiff tape walked by backward_parameters
//     (crates/tynx-train/src/autograd.rs:56-95) -- here an explicit list of
//     backward rules, one per forward node, run in reverse order;
//   * ParameterSlot value/grad storage and accumulate_grad
//     (crates/tynx-train/src/parameter.rs:88-333).
// Parameters live in one flat device buffer (values) and one flat gradient
// buffer, laid out in the order their gradients become final during backward,
// so bucketed all-reduce ranges are contiguous.
//
// Fusions planned at build time:
//   * Gemm/MatMul followed by its only consumer Relu/Tanh/Gelu -> bias +
//     activation in the GEMM epilogue (Gelu also stores the pre-activation);
//   * in backward, the dgrad GEMM producing the gradient of such a fused
//     output multiplies by act' in its epilogue, handing the producer its
//     pre-activation gradient directly.
#include <math.h>

#include <algorithm>
#include <cstring>
#include <functional>
#include <memory>
#include <string>

#include "common.h"
#include "epilogue.cuh"
#include "gemm_tc.cuh"

extern "C" int tx_attention_fwd(tx_ctx *ctx, const float *q, const float *k, const float *v, int64_t ld_in,
                                float *out, int64_t ld_out, int64_t batch, int64_t seq, int64_t heads,
                                int64_t head_dim, float scale, int flags);  // attn.cu
extern "C" int tx_attention_bwd(tx_ctx *ctx, const float *q, const float *k, const float *v, int64_t ld_in,
                                const float *dout, int64_t ld_dout, float *dq, float *dk, float *dv,
                                int64_t ld_grad, int64_t batch, int64_t seq, int64_t heads, int64_t head_dim,
                                float scale, int flags);  // attn.cu
int dp_allreduce_range(tx_ctx *ctx, float *buf, int64_t n);  // dp.cu
int dp_event_fork(tx_ctx *ctx);                               // compute -> comm
int dp_event_join(tx_ctx *ctx);                               // comm -> compute

namespace {

using Shape = std::vector<int64_t>;

int64_t numel_of(const Shape &s) {
  int64_t n = 1;
  for (int64_t d : s) n *= d;
  return n;
}

std::string shape_str(const Shape &s) {
  std::string r = "[";
  for (size_t i = 0; i < s.size(); ++i) r += (i ? "," : "") + std::to_string(s[i]);
  return r + "]";
}

// ---- engine-only kernels -----------------------------------------------------------------
__global__ void k_gather_axis(const float *__restrict__ data, const int64_t *__restrict__ idx,
                              float *__restrict__ out, int64_t outer, int64_t axis_n, int64_t inner,
                              int64_t n_idx, int *flag) {
  int64_t total = outer * n_idx * inner;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t in_ = i % inner;
    int64_t t = i / inner;
    int64_t j = t % n_idx;
    int64_t o = t / n_idx;
    int64_t k = idx[j];
    if (k < 0) k += axis_n;
    if (k < 0 || k >= axis_n) {
      if (atomicCAS(flag, 0, DEVERR_INDEX) == 0) {
        flag[1] = (int)idx[j];
        flag[2] = (int)axis_n;
      }
      out[i] = 0.f;
    } else {
      out[i] = data[(o * axis_n + k) * inner + in_];
    }
  }
}

__global__ void k_gather_axis_bwd(float *__restrict__ ddata, const int64_t *__restrict__ idx,
                                  const float *__restrict__ dout, int64_t outer, int64_t axis_n,
                                  int64_t inner, int64_t n_idx) {
  int64_t total = outer * n_idx * inner;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t in_ = i % inner;
    int64_t t = i / inner;
    int64_t j = t % n_idx;
    int64_t o = t / n_idx;
    int64_t k = idx[j];
    if (k < 0) k += axis_n;
    if (k >= 0 && k < axis_n) atomicAdd(&ddata[(o * axis_n + k) * inner + in_], dout[i]);
  }
}

struct BDims {
  int64_t shape[TX_MAX_DIMS];
  int64_t s[TX_MAX_DIMS];
};


__global__ void k_axpy(float *__restrict__ y, const float *__restrict__ x, int64_t n, float a) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    y[i] += a * x[i];
}

// ---- convolution as a GEMM over channels-last columns ---------------------------------
// The ONNX tensors are NCHW; inside a convolution the activations are moved to
// NHWC so that an im2col column k = (kh * KW + kw) * C + c copies contiguous
// channel runs (float4 when C % 4 == 0), and the weights are permuted to the
// same (kh, kw, c) order once per forward.

// out[b][c][r] (+)= in[b][r][c] * act'(src[b][r][c]) (+ bias[c]): a batched
// transpose of [R, Cc] matrices through 32 x 32 shared-memory tiles, so both
// the loads and the stores are 128-byte row segments.  `src` (optional) is
// indexed like `in`.
__global__ void k_transpose_b(const float *__restrict__ in, float *__restrict__ out, int64_t R, int64_t Cc,
                              const float *__restrict__ bias, const float *__restrict__ src, int dact,
                              int acc) {
  __shared__ float tile[32][33];
  const int64_t b = blockIdx.z;
  const int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 32;
  const float *ib = in + b * R * Cc;
  const float *sb = src ? src + b * R * Cc : nullptr;
#pragma unroll
  for (int j = 0; j < 32; j += 8) {
    const int64_t r = r0 + threadIdx.y + j, c = c0 + threadIdx.x;
    float v = 0.f;
    if (r < R && c < Cc) {
      v = ib[r * Cc + c];
      if (sb) v *= tx_epi::dact(dact, sb[r * Cc + c]);
    }
    tile[threadIdx.y + j][threadIdx.x] = v;
  }
  __syncthreads();
  float *ob = out + b * R * Cc;
#pragma unroll
  for (int j = 0; j < 32; j += 8) {
    const int64_t c = c0 + threadIdx.y + j, r = r0 + threadIdx.x;
    if (r < R && c < Cc) {
      float v = tile[threadIdx.x][threadIdx.y + j];
      if (bias) v += bias[c];
      float *o = ob + c * R + r;
      *o = acc ? *o + v : v;
    }
  }
}

int transpose_b(tx_ctx *ctx, const float *in, float *out, int64_t B, int64_t R, int64_t Cc,
                const float *bias = nullptr, const float *src = nullptr, int dact = TX_ACT_NONE, int acc = 0) {
  if (B <= 0 || R <= 0 || Cc <= 0) return TX_OK;
  if (B > 65535 || (R + 31) / 32 > 65535) return tx_fail(ctx, TX_ERR_UNSUPPORTED, "transpose too large");
  dim3 grid((unsigned)((Cc + 31) / 32), (unsigned)((R + 31) / 32), (unsigned)B);
  k_transpose_b<<<grid, dim3(32, 8), 0, ctx->stream>>>(in, out, R, Cc, bias, src, dact, acc);
  TX_LAUNCHED(ctx, "k_transpose_b");
  return TX_OK;
}

struct ConvGeom {
  int N, C, H, W, KH, KW, OH, OW, sh, sw, pt, pl, dh, dw;
  int ldk;  // columns per im2col row (K = KH*KW*C rounded up to 4, zero padded)
  // grouped convolution: C is one group's channels; a pixel's channels-last
  // row holds ctot channels and the group's start at coff
  int groups = 1, ctot = 0, coff = 0;
};

// cols[m][(kh*KW + kw)*C + c] = xh[n][ih][iw][c] (0 outside the image and in
// the padding columns), m = (n*OH + oh)*OW + ow.  V = 4: float4 channel runs.
template <int V>
__global__ void k_im2col_nhwc(const float *__restrict__ xh, float *__restrict__ cols, ConvGeom g,
                              uint32_t units, int round_tf32) {
  const uint32_t per_row = (uint32_t)g.ldk / V;
  const uint32_t cv = (uint32_t)g.C / V;
  for (uint32_t u = blockIdx.x * blockDim.x + threadIdx.x; u < units; u += gridDim.x * blockDim.x) {
    const uint32_t m = u / per_row, kq = u - m * per_row;
    const uint32_t tap = kq / cv, c = (kq - tap * cv) * V;
    float v[V];
#pragma unroll
    for (int j = 0; j < V; ++j) v[j] = 0.f;
    if (tap < (uint32_t)(g.KH * g.KW)) {
      const uint32_t kh = tap / g.KW, kw = tap - kh * g.KW;
      const uint32_t ow = m % g.OW, t = m / g.OW, oh = t % g.OH, n = t / g.OH;
      const int ih = (int)oh * g.sh - g.pt + (int)kh * g.dh, iw = (int)ow * g.sw - g.pl + (int)kw * g.dw;
      if (ih >= 0 && ih < g.H && iw >= 0 && iw < g.W) {
        const float *p = xh + (((int64_t)n * g.H + ih) * g.W + iw) * g.ctot + g.coff + c;
        if (V == 4) {
          const float4 t4 = *reinterpret_cast<const float4 *>(p);
          v[0] = t4.x;
          v[V > 1 ? 1 : 0] = t4.y;
          v[V > 2 ? 2 : 0] = t4.z;
          v[V > 3 ? 3 : 0] = t4.w;
        } else {
          v[0] = *p;
        }
      }
    } else if (V == 1) {
      v[0] = 0.f;  // padding column
    }
#pragma unroll
    for (int j = 0; j < V; ++j)
      if (round_tf32) v[j] = tx_epi::round_tf32(v[j]);
    float *o = cols + (int64_t)u * V;
    if (V == 4)
      *reinterpret_cast<float4 *>(o) = make_float4(v[0], v[V > 1 ? 1 : 0], v[V > 2 ? 2 : 0], v[V > 3 ? 3 : 0]);
    else
      *o = v[0];
  }
}

// im2col for channel counts that are not multiples of 4 (the 3-channel input
// of a first convolution) and rows of at most 64 columns: each lane builds one
// row (its index decomposed once, taps walked in order) in shared memory, then
// the warp stores its 32 rows as one contiguous run.  The element-wise kernel
// spends four integer divisions per element and stores with a row stride.
constexpr int kIm2colRowsMaxLdk = 64;

__global__ void __launch_bounds__(128) k_im2col_rows(const float *__restrict__ xh, float *__restrict__ cols,
                                                     ConvGeom g, int64_t M, int round_tf32) {
  __shared__ float sm[4][32 * (kIm2colRowsMaxLdk + 1)];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ld = g.ldk + 1;  // odd row stride: the lanes' rows fall in different banks
  float *tile = sm[warp];
  for (int64_t m0 = ((int64_t)blockIdx.x * 4 + warp) * 32; m0 < M; m0 += (int64_t)gridDim.x * 128) {
    const int64_t m = m0 + lane;
    if (m < M) {
      float *row = tile + lane * ld;
      const int64_t ow = m % g.OW, t = m / g.OW, oh = t % g.OH, n = t / g.OH;
      int k = 0;
      for (int kh = 0; kh < g.KH; ++kh) {
        const int ih = (int)oh * g.sh - g.pt + kh * g.dh;
        for (int kw = 0; kw < g.KW; ++kw) {
          const int iw = (int)ow * g.sw - g.pl + kw * g.dw;
          const bool in = ih >= 0 && ih < g.H && iw >= 0 && iw < g.W;
          const float *p = xh + (((int64_t)n * g.H + ih) * g.W + iw) * g.ctot + g.coff;
          for (int c = 0; c < g.C; ++c, ++k) {
            const float v = in ? p[c] : 0.f;
            row[k] = round_tf32 ? tx_epi::round_tf32(v) : v;
          }
        }
      }
      for (; k < g.ldk; ++k) row[k] = 0.f;  // padding columns
    }
    __syncwarp();
    const int64_t nrows = M - m0 < 32 ? M - m0 : 32;
    float *dst = cols + m0 * g.ldk;
    for (int i = lane; i < nrows * g.ldk; i += 32) {
      const int r = i / g.ldk, k = i - r * g.ldk;
      dst[i] = tile[r * ld + k];
    }
    __syncwarp();
  }
}

// dxh[n][ih][iw][coff + c] = sum over the taps that read (ih, iw) of
// dcols[m][(kh*KW + kw)*C + c] (gather form: each input element is written
// once, no atomics).
// S: the stride when both strides equal it (1 or 2: the tap tests become masks
// and shifts instead of runtime divisions), 0 for any strides.
// act_src (or null): multiply each sum by act'(act_src) at the same index
// (the derivative of the activation fused into the convolution that produced
// a channels-last input).
template <int V, int S>
__global__ void k_col2im_nhwc(const float *__restrict__ dcols, float *__restrict__ dxh, ConvGeom g,
                              uint32_t units, const float *__restrict__ act_src, int act) {
  const uint32_t cv = (uint32_t)g.C / V;
  const int sh = S ? S : g.sh, sw = S ? S : g.sw;
  for (uint32_t u = blockIdx.x * blockDim.x + threadIdx.x; u < units; u += gridDim.x * blockDim.x) {
    const uint32_t pix = u / cv, c = (u - pix * cv) * V;
    const uint32_t iw = pix % g.W, t = pix / g.W, ih = t % g.H, n = t / g.H;
    float s[V];
#pragma unroll
    for (int j = 0; j < V; ++j) s[j] = 0.f;
    for (int kh = 0; kh < g.KH; ++kh) {
      const int a = (int)ih + g.pt - kh * g.dh;
      if (a < 0 || a % sh) continue;
      const int oh = a / sh;
      if (oh >= g.OH) continue;
      for (int kw = 0; kw < g.KW; ++kw) {
        const int b = (int)iw + g.pl - kw * g.dw;
        if (b < 0 || b % sw) continue;
        const int ow = b / sw;
        if (ow >= g.OW) continue;
        const float *p = dcols + (((int64_t)n * g.OH + oh) * g.OW + ow) * g.ldk + (kh * g.KW + kw) * g.C + c;
        if (V == 4) {
          const float4 t4 = *reinterpret_cast<const float4 *>(p);
          s[0] += t4.x;
          s[V > 1 ? 1 : 0] += t4.y;
          s[V > 2 ? 2 : 0] += t4.z;
          s[V > 3 ? 3 : 0] += t4.w;
        } else {
          s[0] += *p;
        }
      }
    }
    const int64_t at = (int64_t)pix * g.ctot + g.coff + c;  // the group's channels of this pixel
    if (act_src) {
      const float *a = act_src + at;
#pragma unroll
      for (int j = 0; j < V; ++j) s[j] *= tx_epi::dact(act, a[j]);
    }
    float *o = dxh + at;
    if (V == 4)
      *reinterpret_cast<float4 *>(o) = make_float4(s[0], s[V > 1 ? 1 : 0], s[V > 2 ? 2 : 0], s[V > 3 ? 3 : 0]);
    else
      *o = s[0];
  }
}

// wk[o][(kh*KW + kw)*C + c] = w[o][c][kh][kw], zero padded to ldk (optionally TF32-rounded)
__global__ void k_weight_to_khwc(const float *__restrict__ w, float *__restrict__ wk, int OC, int C, int KH,
                                 int KW, int ldk, int round_tf32) {
  const int64_t n = (int64_t)OC * ldk;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int o = (int)(i / ldk), k = (int)(i - (int64_t)o * ldk);
    float v = 0.f;
    if (k < KH * KW * C) {
      const int tap = k / C, c = k - tap * C, kh = tap / KW, kw = tap - kh * KW;
      v = w[(((int64_t)o * C + c) * KH + kh) * KW + kw];
    }
    wk[i] = round_tf32 ? tx_epi::round_tf32(v) : v;
  }
}

// dw[o][c][kh][kw] (+)= dwk[o][(kh*KW + kw)*C + c]
__global__ void k_weight_from_khwc(const float *__restrict__ dwk, float *__restrict__ dw, int OC, int C, int KH,
                                   int KW, int ldk, int acc) {
  const int64_t n = (int64_t)OC * C * KH * KW;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int kw = (int)(i % KW), kh = (int)((i / KW) % KH), c = (int)((i / (KW * KH)) % C),
              o = (int)(i / ((int64_t)KW * KH * C));
    const float v = dwk[(int64_t)o * ldk + (kh * KW + kw) * C + c];
    dw[i] = acc ? dw[i] + v : v;
  }
}

// wt[(t * C + c) * OC + o] = w[o][c][kh][kw], t = kh * KW + kw (optionally TF32-rounded):
// the data-gradient product's weight rows, one [C][OC] block per tap
__global__ void k_weight_to_tco(const float *__restrict__ w, float *__restrict__ wt, int OC, int C, int KH, int KW,
                                int round_tf32) {
  const int64_t n = (int64_t)OC * C * KH * KW;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int o = (int)(i % OC);
    const int64_t r = i / OC;
    const int c = (int)(r % C), t = (int)(r / C);
    const int kh = t / KW, kw = t - kh * KW;
    const float v = w[(((int64_t)o * C + c) * KH + kh) * KW + kw];
    wt[i] = round_tf32 ? tx_epi::round_tf32(v) : v;
  }
}

// ---- implicit-GEMM convolution ---------------------------------------------------------
// The tcgen05 product reads its activation operand straight from the
// channels-last tensor with shifted TMA boxes (tx_tc::GatherOp), so no im2col
// columns are written or read:
//   forward   Y[p][o]  = sum_(t,c) X[pixel(p) + tap(t)][c] Wk[o][(t, c)]   A gathered, 128 pixels per tile
//   wgrad     dWk[o][(t,c)] = sum_p dY[p][o] X[pixel(p) + tap(t)][c]         B gathered, 32 pixels per sub-tile
//   dgrad     for each phase (ph, pw) of the stride, the input pixels
//             (sh a + ph, sw b + pw) take the taps with (ph + pt - kh dh) % sh == 0:
//             dX[(a, b)][c] = sum_(t,o) dY[(a + dh_t, b + dw_t)][o] W[o][c][t]
//             with A gathered from dY (stride 1) and the output written
//             through a strided view of dX.
// A tile of R pixels is one box when it covers whole rows of one image (or
// whole images): R pixels of an OH x OW grid as {bw, bh, bn}.
bool pixel_box(int64_t OH, int64_t OW, int R, uint32_t &bw, uint32_t &bh, uint32_t &bn) {
  if (OH <= 0 || OW <= 0) return false;
  if (OW % R == 0) {
    bw = (uint32_t)R; bh = 1; bn = 1;
    return true;
  }
  if (R % OW != 0) return false;
  if (OH * OW >= R) {
    if (OH % (R / OW)) return false;
    bw = (uint32_t)OW; bh = (uint32_t)(R / OW); bn = 1;
    return true;
  }
  if (R % (OH * OW)) return false;
  bw = (uint32_t)OW; bh = (uint32_t)OH; bn = (uint32_t)(R / (OH * OW));
  return true;
}

// the tcgen05 operand mode for the context's math (as gemm_dispatch picks it)
int tc_mode(tx_ctx *ctx, tx_gemm_desc &q) {
  if (ctx->math != TX_MATH_TF32) q.flags = 0;
  if (ctx->math == TX_MATH_3XTF32) return 2;
  if (ctx->math == TX_MATH_TF32_TRUNC) return 0;
  if (q.flags & TX_GEMM_EXACT) {
    q.flags &= ~(TX_GEMM_A_TF32 | TX_GEMM_B_TF32);
    return 2;
  }
  return 1;
}

// the tap offsets of a forward / weight-gradient gather (every tap, in (kh, kw) order)
bool conv_gather_fwd(const ConvGeom &g, int R, tx_tc::ConvGemm &cv) {
  if (g.C % 32 || g.KH * g.KW > tx_tc::kGatherTaps || g.sh > 8 || g.sw > 8) return false;
  uint32_t bw, bh, bn;
  if (!pixel_box(g.OH, g.OW, R, bw, bh, bn)) return false;
  if (bw * g.sw > 256 || bh * g.sh > 256 || bn > 256) return false;
  memset(&cv, 0, sizeof cv);
  tx_tc::GatherOp &op = cv.op;
  op.cblocks = g.C / 32;
  op.ntaps = g.KH * g.KW;
  op.ohw = g.OH * g.OW;
  op.ow = g.OW;
  op.sw = g.sw;
  op.sh = g.sh;
  for (int kh = 0; kh < g.KH; ++kh)
    for (int kw = 0; kw < g.KW; ++kw) {
      const int t = kh * g.KW + kw;
      const int ox = kw * g.dw - g.pl, oy = kh * g.dh - g.pt;
      if (ox < -32768 || ox > 32767 || oy < -32768 || oy > 32767) return false;
      op.offx[t] = (int16_t)ox;
      op.offy[t] = (int16_t)oy;
      op.wtap[t] = (int16_t)t;
    }
  cv.box[0] = 32;
  cv.box[1] = bw * g.sw;
  cv.box[2] = bh * g.sh;
  cv.box[3] = bn;
  cv.estr_w = (uint32_t)g.sw;
  cv.estr_h = (uint32_t)g.sh;
  return true;
}

// A 1-D convolution ([N][C][L] input, [OC][C][K] weights) is the 2-D one
// over a unit height (the lowering writes unit height, stride and dilation
// and zero vertical padding); the memory layouts coincide.
ConvGeom conv_geom(const Shape &x, const Shape &w, const Shape &y, const tx_node_desc &d) {
  ConvGeom g;
  const bool one = x.size() == 3;
  g.N = (int)x[0]; g.C = (int)x[1]; g.H = one ? 1 : (int)x[2]; g.W = (int)x.back();
  g.KH = one ? 1 : (int)w[2]; g.KW = (int)w.back(); g.OH = one ? 1 : (int)y[2]; g.OW = (int)y.back();
  g.sh = (int)d.ints[0]; g.sw = (int)d.ints[1]; g.pt = (int)d.ints[2]; g.pl = (int)d.ints[3];
  g.dh = (int)d.ints[6]; g.dw = (int)d.ints[7];
  g.ldk = (g.KH * g.KW * g.C + 3) & ~3;
  g.ctot = g.C;
  return g;
}

// one group's geometry of a grouped convolution (C = that group's channels)
ConvGeom conv_group(const ConvGeom &all, int groups, int gi) {
  ConvGeom g = all;
  g.groups = groups;
  g.C = all.C / groups;
  g.ctot = all.C;
  g.coff = gi * g.C;
  g.ldk = (g.KH * g.KW * g.C + 3) & ~3;
  return g;
}

int im2col_nhwc(tx_ctx *ctx, const float *xh, float *cols, const ConvGeom &g, bool round_tf32) {
  const int64_t M = (int64_t)g.N * g.OH * g.OW;
  const bool vec = g.C % 4 == 0 && g.ctot % 4 == 0 && g.coff % 4 == 0;
  if (!vec && g.ldk <= kIm2colRowsMaxLdk) {
    int64_t blocks = (M + 127) / 128;
    if (blocks > (int64_t)ctx->num_sms * 16) blocks = (int64_t)ctx->num_sms * 16;
    k_im2col_rows<<<(unsigned)(blocks < 1 ? 1 : blocks), 128, 0, ctx->stream>>>(xh, cols, g, M, round_tf32);
    TX_LAUNCHED(ctx, "k_im2col_rows");
    return TX_OK;
  }
  const int64_t units = M * g.ldk / (vec ? 4 : 1);
  if (units >= (int64_t(1) << 32)) return tx_fail(ctx, TX_ERR_UNSUPPORTED, "im2col too large");
  if (vec)
    k_im2col_nhwc<4><<<grid_for(units, 256), 256, 0, ctx->stream>>>(xh, cols, g, (uint32_t)units, round_tf32);
  else
    k_im2col_nhwc<1><<<grid_for(units, 256), 256, 0, ctx->stream>>>(xh, cols, g, (uint32_t)units, round_tf32);
  TX_LAUNCHED(ctx, "k_im2col_nhwc");
  return TX_OK;
}

int col2im_nhwc(tx_ctx *ctx, const float *dcols, float *dxh, const ConvGeom &g, const float *act_src = nullptr,
                int act = TX_ACT_NONE) {
  const bool vec = g.C % 4 == 0 && g.ldk % 4 == 0 && g.ctot % 4 == 0 && g.coff % 4 == 0;
  const int64_t units = (int64_t)g.N * g.H * g.W * g.C / (vec ? 4 : 1);
  if (units >= (int64_t(1) << 32)) return tx_fail(ctx, TX_ERR_UNSUPPORTED, "col2im too large");
  const int S = g.sh == g.sw && (g.sh == 1 || g.sh == 2) ? g.sh : 0;
  const dim3 grid(grid_for(units, 256));
  if (vec) {
    if (S == 1) k_col2im_nhwc<4, 1><<<grid, 256, 0, ctx->stream>>>(dcols, dxh, g, (uint32_t)units, act_src, act);
    else if (S == 2) k_col2im_nhwc<4, 2><<<grid, 256, 0, ctx->stream>>>(dcols, dxh, g, (uint32_t)units, act_src, act);
    else k_col2im_nhwc<4, 0><<<grid, 256, 0, ctx->stream>>>(dcols, dxh, g, (uint32_t)units, act_src, act);
  } else {
    if (S == 1) k_col2im_nhwc<1, 1><<<grid, 256, 0, ctx->stream>>>(dcols, dxh, g, (uint32_t)units, act_src, act);
    else if (S == 2) k_col2im_nhwc<1, 2><<<grid, 256, 0, ctx->stream>>>(dcols, dxh, g, (uint32_t)units, act_src, act);
    else k_col2im_nhwc<1, 0><<<grid, 256, 0, ctx->stream>>>(dcols, dxh, g, (uint32_t)units, act_src, act);
  }
  TX_LAUNCHED(ctx, "k_col2im_nhwc");
  return TX_OK;
}

}  // namespace

int batched_transpose(tx_ctx *ctx, const float *in, float *out, int64_t B, int64_t R, int64_t Cc, int acc) {
  return transpose_b(ctx, in, out, B, R, Cc, nullptr, nullptr, TX_ACT_NONE, acc);
}

// ============================================================================
// graph structures
// ============================================================================
struct GValue {
  int kind = TX_VAL_ACT;
  int dtype = TX_DT_F32;
  Shape shape;                 // static shape (PARAM/CONST)
  void *dev = nullptr;         // PARAM: slice of flat values; CONST: own buffer
  float *grad = nullptr;       // PARAM: slice of flat grads
  int param_index = -1;
  bool grad_defined = false;
  std::vector<int> consumers;  // node indices
  int producer = -1;
  bool is_output = false;
  int input_index = -1;
  // TF32 mode: this value's gradient is written once, by a contraction of its
  // sole consumer, and read only as a contraction operand (by its producing
  // MatMul, directly or through reshapes and transposes), so the contraction
  // that writes it may store it rounded; set at graph creation
  bool grad_round = false;
};

struct GNode {
  tx_node_desc d;
  int fused_act = TX_ACT_NONE;  // GEMM/MATMUL: absorbed activation
  int fused_into = -1;          // activation node absorbed by node index
  int fused_out = -1;           // value written by the fused epilogue
  // TF32 mode: the epilogue may store its result rounded to TF32, because every
  // reader of it rounds it so anyway (GEMM operands) or only looks at its sign
  // (the relu mask); set at graph creation
  bool round_out = false;
  // Softmax whose output is read only as a contraction operand (attention
  // probabilities): in TF32 mode it also stores a rounded copy (the record's
  // extra for the node) that those contractions read without conversion; the
  // backward reads the exact output
  bool round_copy = false;
  // MatMul / Gemm whose sole consumer multiplies (or divides) it by a constant
  // scalar: the scale is folded into alpha and the result written to the
  // scaling node's output (scale_out); that node is skipped (scaled_into)
  float out_scale = 1.f;
  int scale_out = -1;
  int scaled_into = -1;
  // Conv -> Conv: the producer's (activated) output feeds only the consumer's
  // input, so it stays channels-last in HBM ([N][H][W][C], in the value's
  // buffer): the producer skips its output transpose and the consumer its
  // input transpose; in the backward the consumer's dX is written
  // channels-last and the producer applies act' elementwise
  bool nhwc_out = false;
  bool nhwc_in = false;
  // TF32 mode: a forward contraction whose result passes through a ReLU runs
  // to fp32-class accuracy (TX_GEMM_EXACT) on unrounded operands.  The mask
  // is discontinuous: a TF32 rounding of the pre-activation flips it wherever
  // the value lies within ~2^-11 of zero, and each flip moves a whole gradient
  // entry (on the MLP classifier at batch 4096 ~900 flips of 8M, a 2e-3
  // relative error of the first layer's weight gradient).  Its backward
  // products stay TF32.
  bool exact = false;
  // member of a fused attention block (tx_graph::attn index), or -1
  int attn = -1;
  // member of a group of sibling projections run as one batched product
  // (tx_graph::proj index), or -1
  int proj = -1;
};

// An attention block the fused kernels can run: q, k, v are [B, S, H * D]
// projection outputs; Reshape -> Transpose(0,2,1,3) (Transpose(0,2,3,1) for k)
// -> MatMul(qh, kh) (-> scale) -> Softmax -> MatMul(., vh) -> Transpose(0,2,1,3)
// -> Reshape produces `out` [B, S, H * D].  Every intermediate value has that
// one reader, so none of them is needed once the block runs fused.
struct AttnPlan {
  int q = -1, k = -1, v = -1, out = -1;
  int split_q = -1;             // the Reshape of q: its output shape gives H and D
  int first = -1, last = -1;    // node index range of the block
  float scale = 1.f;
  bool round_out = false;       // TF32 mode: out only feeds contractions
};

// Sibling projections of one input: MatMuls X @ W_z (z = 0, 1, 2) whose
// weights are parameters of one shape stored back to back (spacing elements
// apart) and whose results have no other writer (the q, k and v of a fused
// attention block).  They run as one batched product over the three weights
// with A shared, writing three consecutive slices of one allocation.
struct ProjGroup {
  int node[3] = {-1, -1, -1};   // in weight-offset order
  int out[3] = {-1, -1, -1};
  int weight0 = -1;             // value id of the lowest-offset weight
  int leader = -1;              // the first of the three nodes to run
  int64_t spacing = 0;          // elements between consecutive weights
};

struct tx_graph {
  tx_ctx *ctx = nullptr;
  std::vector<GValue> values;
  std::vector<GNode> nodes;
  std::vector<int> inputs;   // value ids of TX_VAL_INPUT in declaration order
  std::vector<bool> input_round;  // TF32 mode: input read only by contractions (rounded copy)
  std::vector<int> outputs;  // value ids
  std::vector<int> params;   // value ids in param-index order (declaration order)
  std::vector<int64_t> param_offset;  // offset in flat buffers
  float *flat_values = nullptr;
  float *flat_grads = nullptr;
  float *flat_tf32 = nullptr;  // TF32-rounded copy of flat_values (GEMM operands)
  float *flat_lo = nullptr;    // TF32 tail of flat_values (forward contractions: head + tail)
  int64_t flat_len = 0;
  // DP
  bool dp = false;
  int64_t bucket_bytes = 0;
  std::vector<int> grad_final_order;  // param indices in the order grads become final
  std::vector<AttnPlan> attn;          // fused attention blocks
  std::vector<ProjGroup> proj;         // batched sibling projections
};

struct tx_record {
  tx_graph *g = nullptr;
  std::vector<Shape> shapes;         // per value
  std::vector<void *> buf;           // per value device buffer
  std::vector<bool> owned;           // buffer owned by the record
  std::vector<void *> extra;         // per node saved extras
  std::vector<std::vector<void *>> extra2;
  std::vector<bool> tf32;  // per value: the buffer holds TF32-rounded values
  bool shadow = false;     // parameters read by GEMMs come from flat_tf32
  bool tracking = false;
  std::vector<uint8_t> attn_fused;  // per tx_graph::attn block: ran as the fused kernels
  std::vector<uint8_t> proj_done;   // per tx_graph::proj group: ran as one batched product
  std::vector<uint8_t> conv_implicit;  // per node: the convolution ran as an implicit GEMM (1;
                                       // extra holds its channels-last input, or null when
                                       // the input value is channels-last itself) or as the
                                       // direct short-filter kernel (2; it reads the NCHW input)
};

namespace {

int fail(tx_graph *g, int code, const std::string &msg) { return tx_fail(g->ctx, code, msg); }

// ---- shape inference ------------------------------------------------------------------------
bool broadcast_shapes(const Shape &a, const Shape &b, Shape &out) {
  size_t n = std::max(a.size(), b.size());
  out.assign(n, 1);
  for (size_t i = 0; i < n; ++i) {
    int64_t da = i < n - a.size() ? 1 : a[i - (n - a.size())];
    int64_t db = i < n - b.size() ? 1 : b[i - (n - b.size())];
    if (da != db && da != 1 && db != 1) return false;
    out[i] = da == 1 ? db : da;
  }
  return true;
}

// element strides of `s` broadcast to `out` (0 on broadcast axes)
void bstrides(const Shape &s, const Shape &out, int64_t *st) {
  size_t n = out.size();
  int64_t stride = 1;
  for (int64_t i = (int64_t)n - 1; i >= 0; --i) {
    int64_t j = i - (int64_t)(n - s.size());
    if (j < 0) {
      st[i] = 0;
      continue;
    }
    st[i] = s[j] == 1 && out[i] != 1 ? 0 : stride;
    stride *= s[j];
  }
}

int norm_axis(int64_t axis, int64_t rank) { return (int)(axis < 0 ? axis + rank : axis); }

// MaxPool geometry {kh, kw, sh, sw, pad_top, pad_left, dh, dw, oh, ow} from the
// node's attributes (ints: kh, kw, sh, sw, pt, pl, pb, pr, dh, dw; iattr[0]
// ceil_mode, iattr[1] auto_pad: 0 NOTSET, 1 VALID, 2 SAME_UPPER, 3 SAME_LOWER)
// and the input's spatial size.  Per axis it resolves the padding as
// crates/tynx/src/interpreter/spatial.rs:102-151 does (auto_pad, then the extra
// end padding that ceil_mode needs, the last window starting inside the input
// or its start padding); windows run over the -inf padded input.
// geom: kh, kw, sh, sw, pt, pl, dh, dw, oh, ow, then the end padding pb, pr
bool pool_geom(const tx_node_desc &d, int64_t H, int64_t W, int64_t geom[12]) {
  const int64_t in[2] = {H, W};
  int64_t start[2], out[2], endp[2];
  for (int a = 0; a < 2; ++a) {
    const int64_t k = d.ints[a], s = d.ints[2 + a], dil = d.ints[8 + a];
    if (k <= 0 || s <= 0 || dil <= 0) return false;
    const int64_t eff = (k - 1) * dil + 1;
    int64_t b = d.ints[4 + a], e = d.ints[6 + a];
    if (d.iattr[1] == 1) {
      b = e = 0;
    } else if (d.iattr[1] >= 2) {
      const int64_t o = (in[a] + s - 1) / s;
      int64_t total = (o - 1) * s + eff - in[a];
      if (total < 0) total = 0;
      const int64_t small = total / 2, large = total - small;
      b = d.iattr[1] == 3 ? large : small;
      e = d.iattr[1] == 3 ? small : large;
    }
    const int64_t padded = in[a] + b + e;
    if (padded < eff) return false;
    int64_t o = (padded - eff) / s + 1;
    if (d.iattr[0]) {
      o = (padded - eff + s - 1) / s + 1;
      if (o > 0 && (o - 1) * s >= in[a] + b) --o;
    }
    start[a] = b;
    out[a] = o;
    endp[a] = e;
  }
  const int64_t g[12] = {d.ints[0], d.ints[1], d.ints[2], d.ints[3], start[0], start[1],
                         d.ints[8], d.ints[9], out[0], out[1], endp[0], endp[1]};
  for (int i = 0; i < 12; ++i) geom[i] = g[i];
  return true;
}

// row-major element strides of a contiguous tensor of shape s
void cstrides(const Shape &s, int64_t *st) {
  int64_t acc = 1;
  for (int64_t i = (int64_t)s.size() - 1; i >= 0; --i) {
    st[i] = acc;
    acc *= s[i];
  }
}

// ONNX Slice on x: per axis the first element, the step and the count
// (negative starts / ends count from the end; both are clamped as the
// operator specifies for the step's sign).  ints: n, axes[n], starts[n],
// ends[n], steps[n].
bool slice_params(const tx_node_desc &d, const Shape &x, int64_t *first, int64_t *step, Shape &out) {
  const int n = (int)d.ints[0];
  const int64_t r = (int64_t)x.size();
  out = x;
  for (int64_t i = 0; i < r; ++i) {
    first[i] = 0;
    step[i] = 1;
  }
  for (int k = 0; k < n; ++k) {
    int64_t a = d.ints[1 + k];
    if (a < 0) a += r;
    if (a < 0 || a >= r) return false;
    const int64_t D = x[a];
    int64_t st = d.ints[1 + n + k], en = d.ints[1 + 2 * n + k], t = d.ints[1 + 3 * n + k];
    if (t == 0) return false;
    if (st < 0) st += D;
    if (en < 0) en += D;
    int64_t len;
    if (t > 0) {
      st = st < 0 ? 0 : st > D ? D : st;
      en = en < 0 ? 0 : en > D ? D : en;
      len = en > st ? (en - st + t - 1) / t : 0;
    } else {
      st = st < 0 ? 0 : st > D - 1 ? D - 1 : st;
      en = en < -1 ? -1 : en > D - 1 ? D - 1 : en;
      len = st > en ? (st - en + (-t) - 1) / (-t) : 0;
    }
    first[a] = st;
    step[a] = t;
    out[a] = len;
  }
  return true;
}

// [outer, reduced, inner] of a max / min reduction over `axes` (ints; none:
// all), when the reduced axes form one block after dropping unit axes
// the reduced axes of a max / min reduction: ints (none: all), or with
// iattr[1] the spatial axes 2.. (GlobalMaxPool)
bool maxmin_axes(const tx_node_desc &d, int64_t r, std::vector<bool> &rd) {
  rd.assign(r, d.n_ints == 0 && !d.iattr[1]);
  if (d.iattr[1]) {
    for (int64_t i = 2; i < r; ++i) rd[i] = true;
    return true;
  }
  for (int i = 0; i < d.n_ints; ++i) {
    int64_t a = d.ints[i];
    if (a < 0) a += r;
    if (a < 0 || a >= r) return false;
    rd[a] = true;
  }
  return true;
}

bool maxmin_block(const tx_node_desc &d, const Shape &x, int64_t *outer, int64_t *red, int64_t *inner) {
  const int64_t r = (int64_t)x.size();
  std::vector<bool> rd;
  if (!maxmin_axes(d, r, rd)) return false;
  int first = -1, last = -1;
  for (int64_t i = 0; i < r; ++i)
    if (rd[i] && x[i] != 1) {
      if (first < 0) first = (int)i;
      last = (int)i;
    }
  *outer = *red = *inner = 1;
  if (first < 0) {  // only unit axes reduced: a copy
    for (int64_t i = 0; i < r; ++i) *outer *= x[i];
    return true;
  }
  for (int i = first; i <= last; ++i)
    if (!rd[i] && x[i] != 1) return false;
  for (int64_t i = 0; i < r; ++i) {
    if (i < first) *outer *= x[i];
    else if (i <= last) *red *= x[i];
    else *inner *= x[i];
  }
  return true;
}

// [N][C][L] view of a rank >= 2 tensor (L = product of the dims after C).
void ncl(const Shape &x, int64_t *N, int64_t *C, int64_t *L) {
  *N = x[0];
  *C = x[1];
  int64_t l = 1;
  for (size_t i = 2; i < x.size(); ++i) l *= x[i];
  *L = l;
}

int infer_node(tx_graph *g, const GNode &n, std::vector<Shape> &S) {
  const tx_node_desc &d = n.d;
  auto in = [&](int i) -> const Shape & { return S[d.in[i]]; };
  Shape &out = S[d.out[0]];
  switch (d.op) {
    case TX_OP_GEMM: {
      const Shape &a = in(0), &b = in(1);
      if (a.size() != 2 || b.size() != 2) return fail(g, TX_ERR_SHAPE, "Gemm requires rank-2 inputs");
      int64_t M = d.iattr[0] ? a[1] : a[0], K = d.iattr[0] ? a[0] : a[1];
      int64_t K2 = d.iattr[1] ? b[1] : b[0], N = d.iattr[1] ? b[0] : b[1];
      if (K != K2) return fail(g, TX_ERR_SHAPE, "Gemm inner dimensions differ: " + shape_str(a) + " x " + shape_str(b));
      out = {M, N};
      return TX_OK;
    }
    case TX_OP_MATMUL: {
      Shape a = in(0), b = in(1);
      if (a.size() < 2 || b.size() < 2)
        return fail(g, TX_ERR_UNSUPPORTED, "MatMul with rank-1 operands is not supported on CUDA");
      if (a.back() != b[b.size() - 2])
        return fail(g, TX_ERR_SHAPE, "MatMul inner dimensions differ: " + shape_str(a) + " x " + shape_str(b));
      if (b.size() == 2) {
        out = a;
        out.back() = b[1];
        return TX_OK;
      }
      if (a.size() != b.size())
        return fail(g, TX_ERR_UNSUPPORTED, "MatMul batch broadcasting is not supported on CUDA");
      for (size_t i = 0; i + 2 < a.size(); ++i)
        if (a[i] != b[i]) return fail(g, TX_ERR_UNSUPPORTED, "MatMul batch broadcasting is not supported on CUDA");
      out = a;
      out.back() = b.back();
      return TX_OK;
    }
    case TX_OP_CONV: {
      const Shape &x = in(0), &w = in(1);
      if (!((x.size() == 4 && w.size() == 4) || (x.size() == 3 && w.size() == 3)))
        return fail(g, TX_ERR_UNSUPPORTED, "only 1-D and 2-D Conv are supported on CUDA");
      const int64_t groups = d.iattr[0];
      if (groups < 1 || x[1] != w[1] * groups || w[0] % groups)
        return fail(g, TX_ERR_SHAPE, "Conv channel mismatch: input " + shape_str(x) + ", weight " + shape_str(w) +
                                         ", " + std::to_string(groups) + " group(s)");
      const bool one = x.size() == 3;
      int64_t sh = d.ints[0], sw = d.ints[1], pt = d.ints[2], pl = d.ints[3], pb = d.ints[4],
              pr = d.ints[5], dh = d.ints[6], dw = d.ints[7];
      const int64_t H = one ? 1 : x[2], KH = one ? 1 : w[2];
      int64_t oh = (H + pt + pb - dh * (KH - 1) - 1) / sh + 1;
      int64_t ow = (x.back() + pl + pr - dw * (w.back() - 1) - 1) / sw + 1;
      if (oh < 1 || ow < 1) return fail(g, TX_ERR_SHAPE, "Conv kernel larger than its padded input");
      out = one ? Shape{x[0], w[0], ow} : Shape{x[0], w[0], oh, ow};
      return TX_OK;
    }
    case TX_OP_GATHER: {
      const Shape &x = in(0), &idx = in(1);
      int ax = norm_axis(d.iattr[0], (int64_t)x.size());
      out.clear();
      for (int i = 0; i < ax; ++i) out.push_back(x[i]);
      for (int64_t v : idx) out.push_back(v);
      for (size_t i = ax + 1; i < x.size(); ++i) out.push_back(x[i]);
      return TX_OK;
    }
    case TX_OP_LAYERNORM: {
      out = in(0);
      int ax = norm_axis(d.iattr[0], (int64_t)out.size());
      Shape st = out;
      for (size_t i = ax; i < st.size(); ++i) st[i] = 1;
      if (d.n_out > 1) S[d.out[1]] = st;
      if (d.n_out > 2) S[d.out[2]] = st;
      return TX_OK;
    }
    case TX_OP_ADD: case TX_OP_SUB: case TX_OP_MUL: case TX_OP_DIV:
      if (!broadcast_shapes(in(0), in(1), out))
        return fail(g, TX_ERR_SHAPE, "cannot broadcast " + shape_str(in(0)) + " with " + shape_str(in(1)));
      return TX_OK;
    case TX_OP_RELU: case TX_OP_TANH: case TX_OP_GELU: case TX_OP_SIGMOID: case TX_OP_EXP:
    case TX_OP_LOG: case TX_OP_NEG: case TX_OP_IDENTITY: case TX_OP_CLIP:
    case TX_OP_SOFTMAX: case TX_OP_LOGSOFTMAX:
      out = in(0);
      return TX_OK;
    case TX_OP_REDUCEMEAN: case TX_OP_REDUCESUM: {
      const Shape &x = in(0);
      std::vector<bool> red(x.size(), d.n_ints == 0);
      for (int i = 0; i < d.n_ints; ++i) red[norm_axis(d.ints[i], (int64_t)x.size())] = true;
      out.clear();
      for (size_t i = 0; i < x.size(); ++i) {
        if (!red[i]) out.push_back(x[i]);
        else if (d.iattr[0]) out.push_back(1);
      }
      return TX_OK;
    }
    case TX_OP_GAP: {
      out = in(0);
      for (size_t i = 2; i < out.size(); ++i) out[i] = 1;
      return TX_OK;
    }
    case TX_OP_PRELU: {
      const Shape &x = in(0), &sl = in(1);
      Shape b;
      if (sl.size() > x.size() || !broadcast_shapes(x, sl, b) || b != x)
        return fail(g, TX_ERR_SHAPE, "PRelu slope shape " + shape_str(sl) + " cannot broadcast to input shape " +
                                         shape_str(x));
      out = x;
      return TX_OK;
    }
    case TX_OP_BATCHNORM: case TX_OP_GROUPNORM: {
      const Shape &x = in(0);
      const bool bn = d.op == TX_OP_BATCHNORM;
      if (x.size() < (bn ? 2u : 3u))
        return fail(g, TX_ERR_SHAPE, std::string(bn ? "BatchNormalization" : "Instance/GroupNormalization") +
                                         " requires rank at least " + (bn ? "2" : "3") + ", got " + shape_str(x));
      const int64_t C = x[1];
      for (int k = 1; k < d.n_in; ++k) {
        if (d.in[k] < 0) return fail(g, TX_ERR_INVALID, "normalization inputs are required");
        if (numel_of(in(k)) != C || in(k).size() != 1)
          return fail(g, TX_ERR_SHAPE, "normalization input " + std::to_string(k) + " expects [" +
                                           std::to_string(C) + "], got " + shape_str(in(k)));
      }
      if (!bn) {
        const int64_t groups = d.iattr[0] > 0 ? d.iattr[0] : C;
        if (C % groups)
          return fail(g, TX_ERR_SHAPE, "GroupNormalization channels " + std::to_string(C) +
                                           " are not divisible by " + std::to_string(groups) + " groups");
      }
      out = x;
      return TX_OK;
    }
    case TX_OP_UNARY:
      if (d.iattr[0] < TX_UN_NEG || d.iattr[0] > TX_UN_RECIPROCAL) return fail(g, TX_ERR_INVALID, "unknown unary op");
      out = in(0);
      return TX_OK;
    case TX_OP_BINARY:
      if (d.iattr[0] != TX_BIN_MAX && d.iattr[0] != TX_BIN_MIN && d.iattr[0] != TX_BIN_POW)
        return fail(g, TX_ERR_INVALID, "unknown binary op");
      if (!broadcast_shapes(in(0), in(1), out))
        return fail(g, TX_ERR_SHAPE, "cannot broadcast " + shape_str(in(0)) + " with " + shape_str(in(1)));
      return TX_OK;
    case TX_OP_CONCAT: {
      const Shape &x = in(0);
      const int ax = norm_axis(d.iattr[0], (int64_t)x.size());
      out = x;
      for (int k = 1; k < d.n_in; ++k) {
        const Shape &o = in(k);
        if (o.size() != x.size()) return fail(g, TX_ERR_SHAPE, "Concat inputs differ in rank");
        for (size_t i = 0; i < x.size(); ++i)
          if ((int)i != ax && o[i] != x[i])
            return fail(g, TX_ERR_SHAPE, "Concat inputs " + shape_str(x) + " and " + shape_str(o) + " differ off axis");
        out[ax] += o[ax];
      }
      return TX_OK;
    }
    case TX_OP_SLICE: {
      int64_t first[TX_MAX_DIMS], step[TX_MAX_DIMS];
      if (!slice_params(d, in(0), first, step, out)) return fail(g, TX_ERR_SHAPE, "Slice axes or steps out of range");
      return TX_OK;
    }
    case TX_OP_SPLIT: {
      const Shape &x = in(0);
      const int ax = norm_axis(d.iattr[0], (int64_t)x.size());
      if (d.n_ints && d.n_ints != d.n_out) return fail(g, TX_ERR_SHAPE, "Split sizes and outputs differ in number");
      const int64_t part = (x[ax] + d.n_out - 1) / d.n_out;  // equal parts, the last one smaller
      int64_t total = 0;
      for (int k = 0; k < d.n_out; ++k) {
        Shape o = x;
        o[ax] = d.n_ints ? d.ints[k] : std::min(part, x[ax] - total);
        if (o[ax] < 0) return fail(g, TX_ERR_SHAPE, "Split sizes exceed the axis of " + shape_str(x));
        total += o[ax];
        S[d.out[k]] = o;
      }
      if (total != x[ax]) return fail(g, TX_ERR_SHAPE, "Split sizes do not add up to the axis of " + shape_str(x));
      return TX_OK;
    }
    case TX_OP_EXPAND: {
      Shape target(d.ints, d.ints + d.n_ints);
      if (!broadcast_shapes(in(0), target, out))
        return fail(g, TX_ERR_SHAPE, "cannot expand " + shape_str(in(0)) + " to " + shape_str(target));
      return TX_OK;
    }
    case TX_OP_REDUCEMAX: case TX_OP_REDUCEMIN: {
      const Shape &x = in(0);
      int64_t o, rd, inn;
      if (!maxmin_block(d, x, &o, &rd, &inn))
        return fail(g, TX_ERR_UNSUPPORTED, "ReduceMax / ReduceMin over non-adjacent axes is not supported on CUDA");
      std::vector<bool> red;
      maxmin_axes(d, (int64_t)x.size(), red);
      out.clear();
      for (size_t i = 0; i < x.size(); ++i) {
        if (!red[i]) out.push_back(x[i]);
        else if (d.iattr[0]) out.push_back(1);
      }
      return TX_OK;
    }
    case TX_OP_AVGPOOL:
    case TX_OP_MAXPOOL: {
      const Shape &x = in(0);
      if (x.size() != 4 && x.size() != 3)
        return fail(g, TX_ERR_UNSUPPORTED, "pooling on CUDA supports 1-D and 2-D windows, got " + shape_str(x));
      int64_t geom[12];
      const int64_t H = x.size() == 4 ? x[2] : 1, W = x.back();
      if (!pool_geom(d, H, W, geom)) return fail(g, TX_ERR_SHAPE, "MaxPool window larger than its padded input");
      out = x;
      if (x.size() == 4) out[2] = geom[8];
      out.back() = geom[9];
      return TX_OK;
    }
    case TX_OP_RESHAPE: {
      const Shape &x = in(0);
      out.clear();
      int64_t known = 1, infer = -1;
      for (int i = 0; i < d.n_ints; ++i) {
        int64_t s = d.ints[i];
        if (s == 0 && !d.iattr[0]) s = x[i];
        if (s == -1) {
          infer = i;
          s = 1;
        } else {
          known *= s;
        }
        out.push_back(s);
      }
      if (infer >= 0) out[infer] = known ? numel_of(x) / known : 0;
      if (numel_of(out) != numel_of(x))
        return fail(g, TX_ERR_SHAPE, "Reshape " + shape_str(x) + " -> " + shape_str(out));
      return TX_OK;
    }
    case TX_OP_FLATTEN: {
      const Shape &x = in(0);
      int ax = norm_axis(d.iattr[0], (int64_t)x.size());
      int64_t lead = 1;
      for (int i = 0; i < ax; ++i) lead *= x[i];
      out = {lead, numel_of(x) / (lead ? lead : 1)};
      return TX_OK;
    }
    case TX_OP_TRANSPOSE: {
      const Shape &x = in(0);
      out.assign(x.size(), 0);
      for (size_t i = 0; i < x.size(); ++i)
        out[i] = x[d.n_ints ? d.ints[i] : (int64_t)x.size() - 1 - (int64_t)i];
      return TX_OK;
    }
    case TX_OP_SQUEEZE: {
      const Shape &x = in(0);
      std::vector<bool> drop(x.size(), false);
      if (d.n_ints == 0)
        for (size_t i = 0; i < x.size(); ++i) drop[i] = x[i] == 1;
      for (int i = 0; i < d.n_ints; ++i) drop[norm_axis(d.ints[i], (int64_t)x.size())] = true;
      out.clear();
      for (size_t i = 0; i < x.size(); ++i)
        if (!drop[i]) out.push_back(x[i]);
      return TX_OK;
    }
    case TX_OP_UNSQUEEZE: {
      const Shape &x = in(0);
      int64_t r = (int64_t)x.size() + d.n_ints;
      std::vector<bool> ins(r, false);
      for (int i = 0; i < d.n_ints; ++i) ins[norm_axis(d.ints[i], r)] = true;
      out.clear();
      size_t j = 0;
      for (int64_t i = 0; i < r; ++i) out.push_back(ins[i] ? 1 : x[j++]);
      return TX_OK;
    }
  }
  return fail(g, TX_ERR_UNSUPPORTED, "operator " + std::to_string(d.op) + " is not supported on CUDA");
}

bool is_alias_op(int op) {
  return op == TX_OP_RESHAPE || op == TX_OP_FLATTEN || op == TX_OP_SQUEEZE ||
         op == TX_OP_UNSQUEEZE || op == TX_OP_IDENTITY;
}

int act_of_op(int op) {
  switch (op) {
    case TX_OP_RELU: return TX_ACT_RELU;
    case TX_OP_TANH: return TX_ACT_TANH;
    case TX_OP_GELU: return TX_ACT_GELU;
  }
  return TX_ACT_NONE;
}

int unary_code(int op) {
  switch (op) {
    case TX_OP_RELU: return TX_UN_RELU;
    case TX_OP_TANH: return TX_UN_TANH;
    case TX_OP_GELU: return TX_UN_GELU;
    case TX_OP_SIGMOID: return TX_UN_SIGMOID;
    case TX_OP_EXP: return TX_UN_EXP;
    case TX_OP_LOG: return TX_UN_LOG;
    case TX_OP_NEG: return TX_UN_NEG;
    case TX_OP_CLIP: return TX_UN_CLAMP;
  }
  return -1;
}

// forward output saved for the backward factor (true) or the input (false)
bool unary_uses_output(int op) {
  return op == TX_OP_RELU || op == TX_OP_TANH || op == TX_OP_SIGMOID || op == TX_OP_EXP;
}

}  // namespace

// ============================================================================
// build
// ============================================================================
extern "C" int tx_graph_create(tx_ctx *ctx, const tx_value_desc *vals, int n_values,
                               const tx_node_desc *nodes, int n_nodes, const int32_t *outputs,
                               int n_outputs, tx_graph **out) {
  if (!ctx || !out || n_values <= 0 || n_nodes < 0) return TX_ERR_INVALID;
  if (ctx->capturing) return tx_fail(ctx, TX_ERR_CAPTURE, "graph creation is not capturable");
  *out = nullptr;
  std::unique_ptr<tx_graph> g(new tx_graph());
  g->ctx = ctx;
  g->values.resize(n_values);
  for (int i = 0; i < n_values; ++i) {
    GValue &v = g->values[i];
    v.kind = vals[i].kind;
    v.dtype = vals[i].dtype;
    if (vals[i].ndim > TX_MAX_DIMS) return tx_fail(ctx, TX_ERR_INVALID, "value rank above 8");
    if (vals[i].ndim >= 0) v.shape.assign(vals[i].shape, vals[i].shape + vals[i].ndim);
    if (v.kind == TX_VAL_INPUT) {
      v.input_index = (int)g->inputs.size();
      g->inputs.push_back(i);
    }
    if (v.kind == TX_VAL_PARAM) {
      if (v.dtype != TX_DT_F32) return tx_fail(ctx, TX_ERR_INVALID, "parameters must be float32");
      v.param_index = (int)g->params.size();
      g->params.push_back(i);
    }
  }
  g->nodes.resize(n_nodes);
  for (int i = 0; i < n_nodes; ++i) {
    g->nodes[i].d = nodes[i];
    const tx_node_desc &d = nodes[i];
    if (d.n_in < 0 || d.n_in > 6 || d.n_out < 1 || d.n_out > 3 || d.n_ints < 0 || d.n_ints > 16)
      return tx_fail(ctx, TX_ERR_INVALID, "malformed node descriptor");
    for (int k = 0; k < d.n_in; ++k) {
      if (d.in[k] < -1 || d.in[k] >= n_values) return tx_fail(ctx, TX_ERR_INVALID, "node input id out of range");
      if (d.in[k] >= 0) g->values[d.in[k]].consumers.push_back(i);
    }
    for (int k = 0; k < d.n_out; ++k) {
      if (d.out[k] < 0 || d.out[k] >= n_values) return tx_fail(ctx, TX_ERR_INVALID, "node output id out of range");
      g->values[d.out[k]].producer = i;
    }
  }
  for (int i = 0; i < n_outputs; ++i) {
    if (outputs[i] < 0 || outputs[i] >= n_values) return tx_fail(ctx, TX_ERR_INVALID, "output id out of range");
    g->outputs.push_back(outputs[i]);
    g->values[outputs[i]].is_output = true;
  }

  // ---- fusion plan: Gemm / MatMul / Conv -> sole-consumer activation ------------------
  for (int i = 0; i < n_nodes; ++i) {
    GNode &n = g->nodes[i];
    if (n.d.op != TX_OP_GEMM && n.d.op != TX_OP_MATMUL && n.d.op != TX_OP_CONV) continue;
    GValue &y = g->values[n.d.out[0]];
    if (y.is_output || y.consumers.size() != 1) continue;
    GNode &a = g->nodes[y.consumers[0]];
    int act = act_of_op(a.d.op);
    if (act == TX_ACT_NONE || a.d.in[0] != n.d.out[0]) continue;
    // a convolution keeps no pre-activation: only activations whose
    // derivative follows from the output fuse into it
    if (n.d.op == TX_OP_CONV && act == TX_ACT_GELU) continue;
    n.fused_act = act;
    n.fused_out = a.d.out[0];
    a.fused_into = i;
  }

  // ---- exact forward products under a ReLU mask ----------------------------------------------
  for (int i = 0; i < n_nodes; ++i) {
    GNode &n = g->nodes[i];
    if (n.d.op != TX_OP_GEMM && n.d.op != TX_OP_MATMUL && n.d.op != TX_OP_CONV) continue;
    bool relu = n.fused_act == TX_ACT_RELU;
    for (int c : g->values[n.d.out[0]].consumers) relu |= g->nodes[c].d.op == TX_OP_RELU;
    n.exact = relu;
  }

  // ---- channels-last hand-off between consecutive convolutions --------------------------------
  for (int i = 0; i < n_nodes; ++i) {
    GNode &n = g->nodes[i];
    if (n.d.op != TX_OP_CONV) continue;
    const int yv = n.fused_act ? n.fused_out : n.d.out[0];
    const GValue &y = g->values[yv];
    if (y.is_output || y.consumers.size() != 1) continue;
    GNode &c = g->nodes[y.consumers[0]];
    if (c.d.op != TX_OP_CONV || c.d.in[0] != yv || c.d.in[1] == yv || (c.d.n_in > 2 && c.d.in[2] == yv))
      continue;
    n.nhwc_out = true;
    c.nhwc_in = true;
  }

  // ---- scalar scale folded into the producing contraction -------------------------------------
  for (int i = 0; i < n_nodes; ++i) {
    GNode &n = g->nodes[i];
    if ((n.d.op != TX_OP_GEMM && n.d.op != TX_OP_MATMUL) || n.fused_act) continue;
    const GValue &y = g->values[n.d.out[0]];
    if (y.is_output || y.consumers.size() != 1) continue;
    GNode &m = g->nodes[y.consumers[0]];
    if (m.d.op != TX_OP_MUL && m.d.op != TX_OP_DIV) continue;
    const int other = m.d.in[0] == n.d.out[0] ? m.d.in[1] : m.d.in[0];
    if (m.d.op == TX_OP_DIV && m.d.in[0] != n.d.out[0]) continue;  // c / y is not a scale
    if (other < 0 || other == n.d.out[0]) continue;
    const GValue &c = g->values[other];
    if (c.kind != TX_VAL_CONST || c.dtype != TX_DT_F32 || numel_of(c.shape) != 1 || !vals[other].h_data) continue;
    // the scale must not change the output shape (a rank-raising scalar would)
    if (c.shape.size() > y.shape.size() && !y.shape.empty()) continue;
    const float cv = *(const float *)vals[other].h_data;
    if (m.d.op == TX_OP_DIV && cv == 0.f) continue;
    n.out_scale = m.d.op == TX_OP_MUL ? cv : 1.f / cv;
    n.scale_out = m.d.out[0];
    m.scaled_into = i;
  }

  // ---- TF32 output rounding: results whose every reader is a contraction --------------------
  // (directly, or through reshapes and transposes, which move values unchanged)
  std::function<bool(int, int)> feeds_only_contractions = [&](int v, int depth) -> bool {
    const GValue &gv = g->values[v];
    if (gv.is_output || gv.consumers.empty() || depth > 8) return false;
    for (int c : gv.consumers) {
      const tx_node_desc &cd = g->nodes[c].d;
      if (cd.op == TX_OP_GEMM || cd.op == TX_OP_MATMUL) {
        if (g->nodes[c].exact) return false;  // reads the unrounded operand
        for (int k = 2; k < cd.n_in; ++k)
          if (cd.in[k] == v) return false;  // a bias is not a contraction operand
      } else if (is_alias_op(cd.op) || cd.op == TX_OP_TRANSPOSE) {
        if (cd.in[0] != v || !feeds_only_contractions(cd.out[0], depth + 1)) return false;
      } else {
        return false;
      }
    }
    return true;
  };
  for (int i = 0; i < n_nodes; ++i) {
    GNode &n = g->nodes[i];
    if (n.d.op == TX_OP_GEMM || n.d.op == TX_OP_MATMUL) {
      if (n.fused_act == TX_ACT_TANH) continue;  // tanh' reads the stored output
      n.round_out = feeds_only_contractions(
          n.fused_act ? n.fused_out : n.scale_out >= 0 ? n.scale_out : n.d.out[0], 0);
    } else if (n.d.op == TX_OP_LAYERNORM) {
      n.round_out = feeds_only_contractions(n.d.out[0], 0);
    } else if (n.d.op == TX_OP_SOFTMAX) {
      const GValue &y = g->values[n.d.out[0]];
      bool only = !y.is_output && !y.consumers.empty();
      for (int c : y.consumers) {
        const tx_node_desc &cd = g->nodes[c].d;
        if (cd.op != TX_OP_GEMM && cd.op != TX_OP_MATMUL) only = false;
        for (int k = 2; k < cd.n_in; ++k)
          if (cd.in[k] == n.d.out[0]) only = false;  // a bias is not a contraction operand
      }
      n.round_copy = only;
    }
  }
  // ---- fused attention blocks -------------------------------------------------------------------
  {
    auto single = [&](int v) {
      return v >= 0 && !g->values[v].is_output && g->values[v].consumers.size() == 1 &&
             g->values[v].kind == TX_VAL_ACT;
    };
    auto prod = [&](int v) { return v >= 0 ? g->values[v].producer : -1; };
    auto is_perm = [&](int ni, std::initializer_list<int> perm) {
      const tx_node_desc &t = g->nodes[ni].d;
      if (t.op != TX_OP_TRANSPOSE || t.n_ints != (int)perm.size()) return false;
      int i = 0;
      for (int p : perm)
        if (t.ints[i++] != p) return false;
      return true;
    };
    // value x = Transpose(perm)(Reshape(src)) with single readers on the way: returns src, or -1
    auto split_of = [&](int x, std::initializer_list<int> perm, int *reshape_node, std::vector<int> &nodes) {
      if (!single(x)) return -1;
      const int t = prod(x);
      if (t < 0 || !is_perm(t, perm)) return -1;
      const int y = g->nodes[t].d.in[0];
      if (!single(y)) return -1;
      const int rsh = prod(y);
      if (rsh < 0 || g->nodes[rsh].d.op != TX_OP_RESHAPE) return -1;
      const int src = g->nodes[rsh].d.in[0];
      if (!single(src)) return -1;
      nodes.push_back(t);
      nodes.push_back(rsh);
      *reshape_node = rsh;
      return src;
    };
    for (int si = 0; si < n_nodes; ++si) {
      GNode &sn = g->nodes[si];
      if (sn.d.op != TX_OP_SOFTMAX || (sn.d.iattr[0] != -1 && sn.d.iattr[0] != 3)) continue;
      std::vector<int> nodes{si};
      const int x = sn.d.in[0];
      if (!single(x)) continue;
      int m1 = -1;
      float scale = 1.f;
      const int px = prod(x);
      if (px < 0) continue;
      if (g->nodes[px].scaled_into >= 0) {
        m1 = g->nodes[px].scaled_into;
        scale = g->nodes[m1].out_scale;
        nodes.push_back(px);
      } else if (g->nodes[px].d.op == TX_OP_MATMUL && g->nodes[px].scale_out < 0) {
        m1 = px;
      }
      if (m1 < 0 || g->nodes[m1].d.op != TX_OP_MATMUL || g->nodes[m1].fused_act) continue;
      nodes.push_back(m1);
      int rq = -1, rk = -1, rv = -1;
      const int q = split_of(g->nodes[m1].d.in[0], {0, 2, 1, 3}, &rq, nodes);
      const int k = split_of(g->nodes[m1].d.in[1], {0, 2, 3, 1}, &rk, nodes);
      const int probs = sn.d.out[0];
      if (q < 0 || k < 0 || !single(probs)) continue;
      const int m2 = g->values[probs].consumers[0];
      GNode &mn = g->nodes[m2];
      if (mn.d.op != TX_OP_MATMUL || mn.d.in[0] != probs || mn.d.in[1] == probs || mn.fused_act ||
          mn.scale_out >= 0)
        continue;
      nodes.push_back(m2);
      const int v = split_of(mn.d.in[1], {0, 2, 1, 3}, &rv, nodes);
      const int ctxv = mn.d.out[0];
      if (v < 0 || !single(ctxv)) continue;
      const int to = g->values[ctxv].consumers[0];
      if (!is_perm(to, {0, 2, 1, 3}) || !single(g->nodes[to].d.out[0])) continue;
      const int ro = g->values[g->nodes[to].d.out[0]].consumers[0];
      if (g->nodes[ro].d.op != TX_OP_RESHAPE) continue;
      if (q == k || q == v || k == v) continue;
      bool taken = false;
      for (int ni : nodes) taken |= g->nodes[ni].attn >= 0;
      if (taken) continue;
      nodes.push_back(to);
      nodes.push_back(ro);
      AttnPlan a;
      a.q = q;
      a.k = k;
      a.v = v;
      a.out = g->nodes[ro].d.out[0];
      a.split_q = rq;
      a.scale = scale;
      a.first = *std::min_element(nodes.begin(), nodes.end());
      a.last = *std::max_element(nodes.begin(), nodes.end());
      a.round_out = feeds_only_contractions(a.out, 0);
      // the last member must run after q, k and v exist: every member reads
      // (through the chain) one of them, and the block ends at the merge
      for (int ni : nodes) g->nodes[ni].attn = (int)g->attn.size();
      g->attn.push_back(a);
    }
  }

  // ---- TF32 gradient rounding: gradients whose every reader is a contraction -----------------
  // The gradient of v is read by the backward of v's producer: a MatMul (no
  // fused activation, no bias) reads it only as an operand of its dgrad and
  // wgrad; a reshape or a transpose copies it unchanged to its own input's
  // gradient.  v must have one consumer that reads it once, so that its
  // gradient has one writer and is never summed.
  std::function<bool(int, int)> grad_feeds_only_contractions = [&](int v, int depth) -> bool {
    const GValue &gv = g->values[v];
    if (gv.kind != TX_VAL_ACT || gv.is_output || gv.producer < 0 || gv.consumers.size() != 1 || depth > 8)
      return false;
    const tx_node_desc &cd = g->nodes[gv.consumers[0]].d;
    int reads = 0;
    for (int k = 0; k < cd.n_in; ++k) reads += cd.in[k] == v;
    if (reads != 1) return false;
    // a contraction whose backward reads dY only as a dgrad / wgrad operand
    auto plain = [](const GNode &n) {
      return !n.fused_act && (n.d.op == TX_OP_MATMUL ||
                              (n.d.op == TX_OP_GEMM && (n.d.n_in <= 2 || n.d.in[2] < 0)));
    };
    const GNode &p = g->nodes[gv.producer];
    if (p.fused_into >= 0) return false;  // act' is applied elementwise to this gradient
    if (p.scaled_into >= 0) {             // the gradient of a folded scale's output
      const GNode &m = g->nodes[p.scaled_into];
      return m.scale_out == v && plain(m);
    }
    if (p.d.op == TX_OP_MATMUL || p.d.op == TX_OP_GEMM) return p.d.out[0] == v && p.scale_out < 0 && plain(p);
    if (is_alias_op(p.d.op) || p.d.op == TX_OP_TRANSPOSE)
      return p.d.out[0] == v && grad_feeds_only_contractions(p.d.in[0], depth + 1);
    return false;
  };
  for (int v = 0; v < (int)g->values.size(); ++v) g->values[v].grad_round = grad_feeds_only_contractions(v, 0);

  g->input_round.assign(g->inputs.size(), false);
  for (size_t i = 0; i < g->inputs.size(); ++i)
    g->input_round[i] = g->values[g->inputs[i]].dtype == TX_DT_F32 &&
                        feeds_only_contractions(g->inputs[i], 0);

  // ---- parameter storage: order = when gradients become final in backward -----------------
  std::vector<int> first_use(g->params.size(), n_nodes);
  for (int i = 0; i < n_nodes; ++i)
    for (int k = 0; k < g->nodes[i].d.n_in; ++k) {
      int v = g->nodes[i].d.in[k];
      if (v >= 0 && g->values[v].kind == TX_VAL_PARAM)
        first_use[g->values[v].param_index] = std::min(first_use[g->values[v].param_index], i);
    }
  std::vector<int> order(g->params.size());
  for (size_t i = 0; i < order.size(); ++i) order[i] = (int)i;
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return first_use[a] > first_use[b]; });
  g->grad_final_order = order;
  g->param_offset.assign(g->params.size(), 0);
  int64_t off = 0;
  for (int p : order) {
    g->param_offset[p] = off;
    int64_t n = numel_of(g->values[g->params[p]].shape);
    off += (n + 63) & ~int64_t(63);
  }
  g->flat_len = off;
  if (off > 0) {
    TX_CUDA(ctx, cudaMalloc(&g->flat_values, off * sizeof(float)));
    TX_CUDA(ctx, cudaMalloc(&g->flat_grads, off * sizeof(float)));
    TX_CUDA(ctx, cudaMemsetAsync(g->flat_grads, 0, off * sizeof(float), ctx->stream));
    TX_CUDA(ctx, cudaMemsetAsync(g->flat_values, 0, off * sizeof(float), ctx->stream));
  }
  // Every copy is ordered on the context's stream after the memsets above (the
  // stream is non-blocking: a legacy-stream cudaMemcpy could run before them).
  for (size_t p = 0; p < g->params.size(); ++p) {
    GValue &v = g->values[g->params[p]];
    v.dev = g->flat_values + g->param_offset[p];
    v.grad = g->flat_grads + g->param_offset[p];
    if (vals[g->params[p]].h_data)
      TX_CUDA(ctx, cudaMemcpyAsync(v.dev, vals[g->params[p]].h_data,
                                   numel_of(v.shape) * sizeof(float), cudaMemcpyHostToDevice,
                                   ctx->stream));
  }
  // ---- sibling projections of a fused attention block (needs the layout) ----------------------
  for (const AttnPlan &a : g->attn) {
    const int outs[3] = {a.q, a.k, a.v};
    int pn[3], w[3];
    int64_t off[3];
    bool ok = true;
    for (int z = 0; z < 3 && ok; ++z) {
      pn[z] = g->values[outs[z]].producer;
      if (pn[z] < 0) {
        ok = false;
        break;
      }
      const GNode &n = g->nodes[pn[z]];
      ok = n.d.op == TX_OP_MATMUL && n.d.n_in == 2 && n.fused_act == TX_ACT_NONE && n.scale_out < 0 &&
           !n.exact && n.out_scale == 1.f && n.attn < 0 && n.proj < 0 && n.d.out[0] == outs[z];
      if (!ok) break;
      w[z] = n.d.in[1];
      const GValue &wv = g->values[w[z]];
      ok = wv.kind == TX_VAL_PARAM && wv.shape.size() == 2 && n.d.in[0] == g->nodes[pn[0]].d.in[0] &&
           wv.shape == g->values[w[0]].shape && n.round_out == g->nodes[pn[0]].round_out &&
           g->values[outs[z]].shape == g->values[outs[0]].shape;
      if (ok) off[z] = g->param_offset[wv.param_index];
    }
    if (!ok) continue;
    int ord[3] = {0, 1, 2};
    std::sort(ord, ord + 3, [&](int x, int y) { return off[x] < off[y]; });
    const int64_t sp = off[ord[1]] - off[ord[0]];
    if (sp <= 0 || off[ord[2]] - off[ord[1]] != sp || (sp & 3)) continue;
    ProjGroup pg;
    for (int z = 0; z < 3; ++z) {
      pg.node[z] = pn[ord[z]];
      pg.out[z] = outs[ord[z]];
    }
    pg.weight0 = w[ord[0]];
    pg.leader = std::min(pn[0], std::min(pn[1], pn[2]));
    pg.spacing = sp;
    for (int z = 0; z < 3; ++z) g->nodes[pn[z]].proj = (int)g->proj.size();
    g->proj.push_back(pg);
  }
  for (int i = 0; i < n_values; ++i) {
    GValue &v = g->values[i];
    if (v.kind != TX_VAL_CONST) continue;
    size_t bytes = numel_of(v.shape) * (v.dtype == TX_DT_I64 ? 8 : 4);
    TX_CUDA(ctx, cudaMalloc(&v.dev, bytes ? bytes : 8));
    if (vals[i].h_data && bytes)
      TX_CUDA(ctx, cudaMemcpyAsync(v.dev, vals[i].h_data, bytes, cudaMemcpyHostToDevice,
                                   ctx->stream));
  }
  // the host arrays belong to the caller: finish reading them before returning
  TX_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  *out = g.release();
  return TX_OK;
}

extern "C" int tx_graph_destroy(tx_graph *g) {
  if (!g) return TX_OK;
  cudaStreamSynchronize(g->ctx->stream);
  for (GValue &v : g->values)
    if (v.kind == TX_VAL_CONST && v.dev) cudaFree(v.dev);
  if (g->flat_values) cudaFree(g->flat_values);
  if (g->flat_grads) cudaFree(g->flat_grads);
  if (g->flat_tf32) cudaFree(g->flat_tf32);
  if (g->flat_lo) cudaFree(g->flat_lo);
  delete g;
  return TX_OK;
}

extern "C" int tx_graph_param_count(tx_graph *g, int *out) {
  if (!g || !out) return TX_ERR_INVALID;
  *out = (int)g->params.size();
  return TX_OK;
}

extern "C" int tx_graph_param(tx_graph *g, int i, int32_t *vid, float **value, float **grad, int64_t *numel) {
  if (!g || i < 0 || i >= (int)g->params.size()) return TX_ERR_INVALID;
  GValue &v = g->values[g->params[i]];
  if (vid) *vid = g->params[i];
  if (value) *value = (float *)v.dev;
  if (grad) *grad = v.grad;
  if (numel) *numel = numel_of(v.shape);
  return TX_OK;
}

extern "C" int tx_graph_value_ptr(tx_graph *g, int value_id, void **out) {
  if (!g || !out || value_id < 0 || value_id >= (int)g->values.size()) return TX_ERR_INVALID;
  const GValue &v = g->values[value_id];
  if (v.kind != TX_VAL_CONST && v.kind != TX_VAL_PARAM)
    return tx_fail(g->ctx, TX_ERR_INVALID, "only parameters and constants have storage of their own");
  *out = v.dev;
  return TX_OK;
}

extern "C" int tx_graph_grad_defined(tx_graph *g, int i, int *out) {
  if (!g || !out || i < 0 || i >= (int)g->params.size()) return TX_ERR_INVALID;
  *out = g->values[g->params[i]].grad_defined ? 1 : 0;
  return TX_OK;
}

extern "C" int tx_graph_set_grad_defined(tx_graph *g, int i, int defined) {
  if (!g || i < 0 || i >= (int)g->params.size()) return TX_ERR_INVALID;
  g->values[g->params[i]].grad_defined = defined != 0;
  return TX_OK;
}

extern "C" int tx_graph_set_dp(tx_graph *g, int enabled, int64_t bucket_bytes) {
  if (!g) return TX_ERR_INVALID;
  if (enabled && g->ctx->world <= 1 && g->ctx->nccl == nullptr)
    return tx_fail(g->ctx, TX_ERR_INVALID, "data parallelism needs tx_dp_init first");
  g->dp = enabled != 0;
  g->bucket_bytes = bucket_bytes > 0 ? bucket_bytes : (8 << 20);
  return TX_OK;
}

static int infer_all(tx_graph *g, const int64_t *in_shapes, const int32_t *in_ndims,
                     std::vector<Shape> &S) {
  S.assign(g->values.size(), Shape());
  size_t off = 0;
  for (size_t i = 0; i < g->inputs.size(); ++i) {
    int nd = in_ndims[i];
    if (nd < 0 || nd > TX_MAX_DIMS) return fail(g, TX_ERR_INVALID, "input rank out of range");
    S[g->inputs[i]].assign(in_shapes + off, in_shapes + off + nd);
    off += nd;
    const GValue &v = g->values[g->inputs[i]];
    if (!v.shape.empty() && v.shape.size() != (size_t)nd)
      return fail(g, TX_ERR_SHAPE, "input " + std::to_string(i) + " has rank " + std::to_string(nd) +
                                       ", expected " + std::to_string(v.shape.size()));
  }
  for (size_t i = 0; i < g->values.size(); ++i)
    if (g->values[i].kind == TX_VAL_PARAM || g->values[i].kind == TX_VAL_CONST) S[i] = g->values[i].shape;
  for (const GNode &n : g->nodes) TX_TRY(infer_node(g, n, S));
  return TX_OK;
}

extern "C" int tx_graph_infer(tx_graph *g, const int64_t *in_shapes, const int32_t *in_ndims,
                              int64_t *out_shapes, int32_t *out_ndims) {
  if (!g) return TX_ERR_INVALID;
  std::vector<Shape> S;
  TX_TRY(infer_all(g, in_shapes, in_ndims, S));
  size_t off = 0;
  for (size_t i = 0; i < g->outputs.size(); ++i) {
    const Shape &s = S[g->outputs[i]];
    out_ndims[i] = (int32_t)s.size();
    for (int64_t v : s) out_shapes[off++] = v;
  }
  return TX_OK;
}

// ============================================================================
// forward
// ============================================================================
namespace {

// Pointer a contraction reads value v from, and whether those values are
// already TF32-rounded (TX_GEMM_A_TF32 / B_TF32): parameters come from the
// rounded shadow refreshed at the start of the forward.
const float *gemm_operand(tx_graph *g, tx_record *r, int v, bool *tf32, bool exact = false) {
  const GValue &gv = g->values[v];
  if (exact) {  // the unrounded values (parameters from the flat buffer itself)
    *tf32 = false;
    return (const float *)r->buf[v];
  }
  if (r->shadow && gv.kind == TX_VAL_PARAM) {
    *tf32 = true;
    return g->flat_tf32 + g->param_offset[gv.param_index];
  }
  if (gv.producer >= 0 && g->nodes[gv.producer].round_copy && r->extra[gv.producer]) {
    *tf32 = true;  // the softmax's rounded copy
    return (const float *)r->extra[gv.producer];
  }
  *tf32 = r->tf32[v];
  return (const float *)r->buf[v];
}

struct Fwd {
  tx_graph *g;
  tx_ctx *ctx;
  tx_record *r;

  float *F(int v) { return (float *)r->buf[v]; }
  const Shape &S(int v) { return r->shapes[v]; }

  int alloc_value(int v) {
    if (r->buf[v]) return TX_OK;
    size_t bytes = numel_of(r->shapes[v]) * (g->values[v].dtype == TX_DT_I64 ? 8 : 4);
    r->buf[v] = tx_alloc_raw(ctx, bytes ? bytes : 4);
    if (!r->buf[v]) return TX_ERR_OOM;
    r->owned[v] = true;
    return TX_OK;
  }

  // The leader of a projection group runs the three products as one batched
  // launch (A shared, the weights as a batch of three); TX_ERR_UNSUPPORTED
  // when the outputs already have buffers (each member then runs alone).
  int proj_forward(const ProjGroup &pg) {
    for (int z = 0; z < 3; ++z)
      if (r->buf[pg.out[z]]) return TX_ERR_UNSUPPORTED;
    const GNode &n0 = g->nodes[pg.node[0]];
    const Shape &a = S(n0.d.in[0]), &b = S(pg.weight0);
    const int64_t K = a.back(), N = b.back(), M = numel_of(a) / K;
    for (int z = 0; z < 3; ++z)
      if (numel_of(S(pg.out[z])) != M * N) return TX_ERR_UNSUPPORTED;
    float *blk = (float *)tx_alloc_raw(ctx, (size_t)(3 * M * N) * 4);
    if (!blk) return TX_ERR_OOM;
    for (int z = 0; z < 3; ++z) {
      r->buf[pg.out[z]] = blk + z * M * N;
      r->owned[pg.out[z]] = z == 0;  // the first slice's value frees the whole block
    }
    tx_gemm_desc q;
    memset(&q, 0, sizeof q);
    q.alpha = 1.f;
    q.bias_scale = 1.f;
    q.M = M;
    q.N = N;
    q.K = K;
    q.batch = 3;
    bool a32 = false, b32 = false;
    q.A = gemm_operand(g, r, n0.d.in[0], &a32);
    q.lda = K;
    q.stride_a = 0;
    q.B = gemm_operand(g, r, pg.weight0, &b32);
    q.ldb = N;
    q.stride_b = pg.spacing;
    q.C = blk;
    q.ldc = N;
    q.stride_c = M * N;
    q.flags = (a32 ? TX_GEMM_A_TF32 : 0) | (b32 ? TX_GEMM_B_TF32 : 0) | TX_GEMM_A_SHARED;
    if (r->shadow && b32) q.B_lo = g->flat_lo + g->param_offset[g->values[pg.weight0].param_index];
    if (n0.round_out && ctx->math == TX_MATH_TF32) {
      q.flags |= TX_GEMM_ROUND_OUT;
      for (int z = 0; z < 3; ++z) r->tf32[pg.out[z]] = true;
    }
    return gemm_dispatch(ctx, q);
  }

  int gemm_node(int ni) {
    GNode &n = g->nodes[ni];
    const tx_node_desc &d = n.d;
    if (n.proj >= 0) {
      if (r->proj_done[n.proj]) return TX_OK;
      const ProjGroup &pg = g->proj[n.proj];
      if (ni == pg.leader) {
        const int rc = proj_forward(pg);
        if (rc != TX_ERR_UNSUPPORTED) {
          if (rc == TX_OK) r->proj_done[n.proj] = 1;
          return rc;
        }
      }
    }
    int yv = n.fused_act ? n.fused_out : n.scale_out >= 0 ? n.scale_out : d.out[0];
    TX_TRY(alloc_value(yv));
    const Shape &a = S(d.in[0]), &b = S(d.in[1]);
    tx_gemm_desc q;
    memset(&q, 0, sizeof q);
    q.alpha = 1.f;
    q.batch = 1;
    q.act = n.fused_act;
    bool a32 = false, b32 = false;
    const bool ex = n.exact && ctx->math == TX_MATH_TF32;
    if (n.fused_act == TX_ACT_GELU) {
      r->extra[ni] = tx_alloc_raw(ctx, numel_of(S(yv)) * 4);
      if (!r->extra[ni]) return TX_ERR_OOM;
    }
    if (d.op == TX_OP_GEMM) {
      q.trans_a = (int)d.iattr[0];
      q.trans_b = (int)d.iattr[1];
      q.M = q.trans_a ? a[1] : a[0];
      q.K = q.trans_a ? a[0] : a[1];
      q.N = q.trans_b ? b[0] : b[1];
      q.A = gemm_operand(g, r, d.in[0], &a32, ex);
      q.lda = a[1];
      q.B = gemm_operand(g, r, d.in[1], &b32, ex);
      q.ldb = b[1];
      q.alpha = (float)d.fattr[0];
      if (d.n_in > 2 && d.in[2] >= 0) {
        const Shape &c = S(d.in[2]);
        int64_t cn = numel_of(c);
        if (!(cn == q.N && (c.size() == 1 || (c.size() == 2 && c[0] == 1))))
          return fail(g, TX_ERR_UNSUPPORTED, "Gemm bias must have shape [N] or [1, N] on CUDA");
        q.bias = F(d.in[2]);
        q.bias_scale = (float)d.fattr[1];
      }
    } else {  // MATMUL
      q.K = a.back();
      q.N = b.back();
      if (b.size() == 2) {
        q.M = numel_of(a) / q.K;
        q.A = gemm_operand(g, r, d.in[0], &a32, ex);
        q.lda = q.K;
        q.B = gemm_operand(g, r, d.in[1], &b32, ex);
        q.ldb = q.N;
      } else {
        q.M = a[a.size() - 2];
        q.batch = numel_of(a) / (q.M * q.K);
        q.A = gemm_operand(g, r, d.in[0], &a32, ex);
        q.lda = q.K;
        q.stride_a = q.M * q.K;
        q.B = gemm_operand(g, r, d.in[1], &b32, ex);
        q.ldb = q.N;
        q.stride_b = q.K * q.N;
        q.stride_c = q.M * q.N;
      }
    }
    q.C = F(yv);
    q.ldc = q.N;
    if (n.fused_act == TX_ACT_GELU) {
      q.preact = (float *)r->extra[ni];
      q.ld_preact = q.N;
    }
    q.alpha *= n.out_scale;
    q.flags = (a32 ? TX_GEMM_A_TF32 : 0) | (b32 ? TX_GEMM_B_TF32 : 0) | (ex ? TX_GEMM_EXACT : 0);
    // TF32 mode: a weight operand enters the forward product as head + tail
    // (fp32-class in the weights; the activation stays TF32).  Rounding the
    // weights is a systematic perturbation that the whole backward inherits:
    // on the transformer encoder it sets most of the TF32 gradient error
    // (1.2e-3 relative with rounded weights, 0.9e-3 with split ones, float64
    // emulation of every product).
    const GValue &wv = g->values[d.in[1]];
    if (!ex && r->shadow && b32 && wv.kind == TX_VAL_PARAM)
      q.B_lo = g->flat_lo + g->param_offset[wv.param_index];
    if (n.round_out && ctx->math == TX_MATH_TF32) {
      q.flags |= TX_GEMM_ROUND_OUT;
      r->tf32[yv] = true;
    }
    return gemm_dispatch(ctx, q);
  }

  // The forward as an implicit GEMM: A gathered from the channels-last input
  // (kept for the weight gradient), B the (kh, kw, c)-ordered weights.  In
  // TF32 mode the kernel rounds the gathered tiles in shared memory, as the
  // explicit columns were rounded.  TX_ERR_UNSUPPORTED: the geometry does not
  // fit the boxes, and the explicit path runs.
  int conv_forward_implicit(int ni, const ConvGeom &cg, bool ex, bool tf32) {
    GNode &n = g->nodes[ni];
    const tx_node_desc &d = n.d;
    tx_tc::ConvGemm cv;
    if (!conv_gather_fwd(cg, tx_tc::TC_BM, cv)) return TX_ERR_UNSUPPORTED;
    const int yv = n.fused_act ? n.fused_out : d.out[0];
    const int64_t M = (int64_t)cg.N * cg.OH * cg.OW, OC = S(d.in[1])[0];
    const int64_t K = (int64_t)cg.KH * cg.KW * cg.C;
    Scratch wk(ctx, (size_t)OC * K * 4), tmp(ctx, n.nhwc_out ? 0 : (size_t)M * OC * 4);
    if (!wk.ptr || (!n.nhwc_out && !tmp.ptr)) return TX_ERR_OOM;
    float *xh = nullptr;
    const float *xin = F(d.in[0]);
    if (!n.nhwc_in) {
      xh = (float *)tx_alloc_raw(ctx, (size_t)cg.N * cg.H * cg.W * cg.C * 4);
      if (!xh) return TX_ERR_OOM;
      r->extra[ni] = xh;  // the weight gradient gathers from it
      TX_TRY(transpose_b(ctx, F(d.in[0]), xh, cg.N, cg.C, (int64_t)cg.H * cg.W));
      xin = xh;
    }
    cv.op.a = 1;
    cv.src = {xin, cg.N, cg.H, cg.W, cg.C};
    k_weight_to_khwc<<<grid_for(OC * K, 256), 256, 0, ctx->stream>>>(F(d.in[1]), wk.as<float>(), (int)OC, cg.C,
                                                                    cg.KH, cg.KW, (int)K, tf32);
    TX_LAUNCHED(ctx, "k_weight_to_khwc");
    tx_gemm_desc q;
    memset(&q, 0, sizeof q);
    q.M = M; q.N = OC; q.K = K;
    q.A = xin; q.lda = K; q.trans_a = 0;
    q.B = wk.as<float>(); q.ldb = K; q.trans_b = 1;
    q.C = n.nhwc_out ? F(yv) : tmp.as<float>(); q.ldc = OC; q.alpha = 1.f; q.batch = 1;
    if (d.n_in > 2 && d.in[2] >= 0) {
      q.bias = F(d.in[2]);
      q.bias_scale = 1.f;
    }
    q.act = n.fused_act;
    q.flags = tf32 ? TX_GEMM_B_TF32 : ex ? TX_GEMM_EXACT : 0;
    const int mode = tc_mode(ctx, q);
    const int rc = gemm_conv_tc(ctx, q, mode, cv);
    if (rc == TX_ERR_UNSUPPORTED) {
      tx_free_raw(ctx, xh);
      r->extra[ni] = nullptr;
      return rc;
    }
    TX_TRY(rc);
    r->conv_implicit[ni] = 1;
    if (n.nhwc_out) return TX_OK;
    return transpose_b(ctx, tmp.as<float>(), F(yv), cg.N, (int64_t)cg.OH * cg.OW, OC);
  }

  int conv_node(int ni) {
    GNode &n = g->nodes[ni];
    const tx_node_desc &d = n.d;
    const Shape &x = S(d.in[0]), &w = S(d.in[1]);
    const int yv = n.fused_act ? n.fused_out : d.out[0];
    TX_TRY(alloc_value(yv));
    const Shape &y = S(d.out[0]);
    const ConvGeom cg = conv_geom(x, w, y, d);
    const int64_t M = (int64_t)cg.N * cg.OH * cg.OW, OC = w[0];
    const bool ex = n.exact && ctx->math == TX_MATH_TF32;
    const bool tf32 = ctx->math == TX_MATH_TF32 && !ex;
    const int G = d.iattr[0];
    if (G == 1 && !n.nhwc_in && conv_direct_ok(cg.C, cg.KH, cg.KW, (int)OC)) {
      const int geom[14] = {cg.N, cg.C, cg.H, cg.W, cg.KH, cg.KW, cg.OH, cg.OW, cg.sh, cg.sw, cg.pt, cg.pl, cg.dh, cg.dw};
      const float *bias = d.n_in > 2 && d.in[2] >= 0 ? F(d.in[2]) : nullptr;
      TX_TRY(conv_direct_fwd(ctx, F(d.in[0]), F(d.in[1]), bias, F(yv), geom, (int)OC, n.fused_act, n.nhwc_out));
      r->conv_implicit[ni] = 2;
      return TX_OK;
    }
    if (ctx->math != TX_MATH_FP32 && G == 1) {
      const int rc = conv_forward_implicit(ni, cg, ex, tf32);
      if (rc != TX_ERR_UNSUPPORTED) return rc;
    }
    // channels-last input, (kh, kw, c) columns per group, weights permuted to
    // match; in TF32 mode both operands are stored rounded, so the GEMM reads
    // them as is.  A grouped convolution runs one product per group over its
    // channel slice (columns [G][M][ldk_g], weights [OC][ldk_g]).
    const ConvGeom g0 = conv_group(cg, G, 0);
    const int64_t ldk = g0.ldk, OCg = OC / G;
    Scratch xh(ctx, n.nhwc_in ? 0 : (size_t)cg.N * cg.H * cg.W * cg.C * 4), wk(ctx, (size_t)OC * ldk * 4),
        tmp(ctx, n.nhwc_out ? 0 : (size_t)M * OC * 4);
    float *cols = (float *)tx_alloc_raw(ctx, (size_t)G * M * ldk * 4);
    if ((!n.nhwc_in && !xh.ptr) || !wk.ptr || (!n.nhwc_out && !tmp.ptr) || !cols) {
      tx_free_raw(ctx, cols);
      return TX_ERR_OOM;
    }
    r->extra[ni] = cols;  // saved for wgrad
    const float *xin = F(d.in[0]);  // channels-last already when the producer kept it so
    if (!n.nhwc_in) {
      TX_TRY(transpose_b(ctx, F(d.in[0]), xh.as<float>(), cg.N, cg.C, (int64_t)cg.H * cg.W));
      xin = xh.as<float>();
    }
    for (int gi = 0; gi < G; ++gi) TX_TRY(im2col_nhwc(ctx, xin, cols + gi * M * ldk, conv_group(cg, G, gi), tf32));
    k_weight_to_khwc<<<grid_for(OC * ldk, 256), 256, 0, ctx->stream>>>(F(d.in[1]), wk.as<float>(), (int)OC,
                                                                      g0.C, cg.KH, cg.KW, (int)ldk, tf32);
    TX_LAUNCHED(ctx, "k_weight_to_khwc");
    for (int gi = 0; gi < G; ++gi) {
      tx_gemm_desc q;
      memset(&q, 0, sizeof q);
      q.M = M; q.N = OCg; q.K = ldk;
      q.A = cols + gi * M * ldk; q.lda = ldk; q.trans_a = 0;
      q.B = wk.as<float>() + gi * OCg * ldk; q.ldb = ldk; q.trans_b = 1;
      q.C = (n.nhwc_out ? F(yv) : tmp.as<float>()) + gi * OCg; q.ldc = OC; q.alpha = 1.f; q.batch = 1;
      if (d.n_in > 2 && d.in[2] >= 0) {
        q.bias = F(d.in[2]) + gi * OCg;
        q.bias_scale = 1.f;
      }
      q.act = n.fused_act;
      q.flags = tf32 ? (TX_GEMM_A_TF32 | TX_GEMM_B_TF32) : ex ? TX_GEMM_EXACT : 0;
      TX_TRY(gemm_dispatch(ctx, q));
    }
    if (n.nhwc_out) return TX_OK;  // the next convolution reads [N][OH][OW][OC]
    return transpose_b(ctx, tmp.as<float>(), F(yv), cg.N, (int64_t)cg.OH * cg.OW, OC);
  }

  // The fused kernels take the block when the contractions run in TF32 and the
  // shapes fit them (q, k, v [B, S <= 128, H * 64]); otherwise its nodes run one
  // by one.
  bool attn_ok(const AttnPlan &a) {
    if (ctx->math != TX_MATH_TF32) return false;
    const Shape &q = S(a.q), &sp = S(g->nodes[a.split_q].d.out[0]);
    if (q.size() != 3 || S(a.k) != q || S(a.v) != q || sp.size() != 4) return false;
    return sp[0] == q[0] && sp[1] == q[1] && sp[3] == 64 && sp[2] * 64 == q[2] && q[1] >= 1 && q[1] <= 128;
  }

  int attn_forward(const AttnPlan &a) {
    TX_TRY(alloc_value(a.out));
    const Shape &q = S(a.q);
    const int64_t B = q[0], Sq = q[1], E = q[2];
    const int flags = ((r->tf32[a.q] && r->tf32[a.k] && r->tf32[a.v]) ? 1 : 0) | (a.round_out ? 2 : 0);
    if (a.round_out) r->tf32[a.out] = true;
    return tx_attention_fwd(ctx, F(a.q), F(a.k), F(a.v), E, F(a.out), E, B, Sq, E / 64, 64, a.scale, flags);
  }

  int node(int ni) {
    GNode &n = g->nodes[ni];
    const tx_node_desc &d = n.d;
    if (n.attn >= 0) {
      const AttnPlan &a = g->attn[n.attn];
      if (ni == a.first) r->attn_fused[n.attn] = attn_ok(a);
      if (r->attn_fused[n.attn]) return ni == a.last ? attn_forward(a) : TX_OK;
    }
    if (n.fused_into >= 0 || n.scaled_into >= 0) return TX_OK;  // done by the producing GEMM
    if (is_alias_op(d.op)) {
      r->buf[d.out[0]] = r->buf[d.in[0]];
      r->owned[d.out[0]] = false;
      r->tf32[d.out[0]] = r->tf32[d.in[0]];
      return TX_OK;
    }
    switch (d.op) {
      case TX_OP_GEMM: case TX_OP_MATMUL: return gemm_node(ni);
      case TX_OP_CONV: return conv_node(ni);
      default: break;
    }
    int yv = d.out[0];
    TX_TRY(alloc_value(yv));
    const Shape &y = S(yv);
    int64_t ny = numel_of(y);
    switch (d.op) {
      case TX_OP_GATHER: {
        const Shape &x = S(d.in[0]);
        int ax = norm_axis(d.iattr[0], (int64_t)x.size());
        int64_t outer = 1, inner = 1;
        for (int i = 0; i < ax; ++i) outer *= x[i];
        for (size_t i = ax + 1; i < x.size(); ++i) inner *= x[i];
        int64_t nidx = numel_of(S(d.in[1]));
        if (g->values[d.in[1]].dtype != TX_DT_I64) return fail(g, TX_ERR_INVALID, "Gather indices must be int64");
        if (ax == 0) return tx_gather_rows(ctx, F(d.in[0]), x[0], inner, (const int64_t *)r->buf[d.in[1]], nidx, F(yv));
        k_gather_axis<<<grid_for(ny, 256), 256, 0, ctx->stream>>>(F(d.in[0]), (const int64_t *)r->buf[d.in[1]], F(yv),
                                                                 outer, x[ax], inner, nidx, ctx->d_err);
        TX_LAUNCHED(ctx, "k_gather_axis");
        return TX_OK;
      }
      case TX_OP_LAYERNORM: {
        const Shape &x = S(d.in[0]);
        int ax = norm_axis(d.iattr[0], (int64_t)x.size());
        int64_t rows = 1;
        for (int i = 0; i < ax; ++i) rows *= x[i];
        int64_t cols = numel_of(x) / (rows ? rows : 1);
        float *mean = nullptr, *rstd = nullptr;
        if (d.n_out > 1) { TX_TRY(alloc_value(d.out[1])); mean = F(d.out[1]); }
        if (d.n_out > 2) { TX_TRY(alloc_value(d.out[2])); rstd = F(d.out[2]); }
        if (!mean) { mean = (float *)tx_alloc_raw(ctx, rows * 4); r->extra[ni] = mean; }
        if (!rstd) {
          rstd = (float *)tx_alloc_raw(ctx, rows * 4);
          r->extra2[ni].push_back(rstd);
        }
        const float *beta = (d.n_in > 2 && d.in[2] >= 0) ? F(d.in[2]) : nullptr;
        const bool rnd = g->nodes[ni].round_out && ctx->math == TX_MATH_TF32;
        if (rnd) r->tf32[yv] = true;
        return layernorm_fwd(ctx, F(d.in[0]), F(d.in[1]), beta, F(yv), mean, rstd, rows, cols,
                             (float)d.fattr[0], rnd);
      }
      case TX_OP_PRELU: {
        int64_t ss[TX_MAX_DIMS];
        bstrides(S(d.in[1]), y, ss);
        return tx_prelu_fwd(ctx, F(d.in[0]), F(d.in[1]), ss, F(yv), y.data(), (int)y.size());
      }
      case TX_OP_BATCHNORM: {
        int64_t N, C, L;
        ncl(S(d.in[0]), &N, &C, &L);
        return tx_batchnorm_fwd(ctx, F(d.in[0]), F(d.in[1]), F(d.in[2]), F(d.in[3]), F(d.in[4]), F(yv), N, C, L,
                                (float)d.fattr[0]);
      }
      case TX_OP_GROUPNORM: {
        int64_t N, C, L;
        ncl(S(d.in[0]), &N, &C, &L);
        const int64_t groups = d.iattr[0] > 0 ? d.iattr[0] : C;
        float *mean = (float *)tx_alloc_raw(ctx, (N * groups + 1) * 4);
        float *sdev = (float *)tx_alloc_raw(ctx, (N * groups + 1) * 4);
        r->extra[ni] = mean;
        if (sdev) r->extra2[ni].push_back(sdev);
        if (!mean || !sdev) return TX_ERR_OOM;
        return tx_groupnorm_fwd(ctx, F(d.in[0]), F(d.in[1]), F(d.in[2]), F(yv), mean, sdev, N, C, L, groups,
                                (float)d.fattr[0]);
      }
      case TX_OP_UNARY:
        return tx_unary(ctx, (int)d.iattr[0], F(d.in[0]), F(yv), ny, (float)d.fattr[0], (float)d.fattr[1]);
      case TX_OP_BINARY: {
        int64_t sa[TX_MAX_DIMS], sb[TX_MAX_DIMS];
        bstrides(S(d.in[0]), y, sa);
        bstrides(S(d.in[1]), y, sb);
        return tx_binary(ctx, (int)d.iattr[0], F(d.in[0]), sa, F(d.in[1]), sb, F(yv), y.data(), (int)y.size());
      }
      case TX_OP_CONCAT: {
        // each input into its slab of the output
        const int ax = norm_axis(d.iattr[0], (int64_t)y.size());
        int64_t ys[TX_MAX_DIMS];
        cstrides(y, ys);
        int64_t at = 0;
        for (int k = 0; k < d.n_in; ++k) {
          const Shape &xk = S(d.in[k]);
          TX_TRY(nd_scatter(ctx, F(d.in[k]), F(yv) + at * ys[ax], ys, xk.data(), (int)xk.size(), 0));
          at += xk[ax];
        }
        return TX_OK;
      }
      case TX_OP_SLICE: {
        const Shape &x = S(d.in[0]);
        int64_t first[TX_MAX_DIMS], step[TX_MAX_DIMS], xs[TX_MAX_DIMS], ss[TX_MAX_DIMS];
        Shape o;
        slice_params(d, x, first, step, o);
        cstrides(x, xs);
        int64_t base = 0;
        for (size_t i = 0; i < x.size(); ++i) {
          base += first[i] * xs[i];
          ss[i] = step[i] * xs[i];
        }
        return nd_copy(ctx, F(d.in[0]) + base, ss, F(yv), y.data(), (int)y.size(), 4, 1.f, 0);
      }
      case TX_OP_SPLIT: {
        const Shape &x = S(d.in[0]);
        const int ax = norm_axis(d.iattr[0], (int64_t)x.size());
        int64_t xs[TX_MAX_DIMS];
        cstrides(x, xs);
        int64_t at = 0;
        for (int k = 0; k < d.n_out; ++k) {
          if (k > 0) TX_TRY(alloc_value(d.out[k]));
          const Shape &ok = S(d.out[k]);
          TX_TRY(nd_copy(ctx, F(d.in[0]) + at * xs[ax], xs, F(d.out[k]), ok.data(), (int)ok.size(), 4, 1.f, 0));
          at += ok[ax];
        }
        return TX_OK;
      }
      case TX_OP_EXPAND: {
        int64_t sx[TX_MAX_DIMS];
        bstrides(S(d.in[0]), y, sx);
        return nd_copy(ctx, F(d.in[0]), sx, F(yv), y.data(), (int)y.size(), 4, 1.f, 0);
      }
      case TX_OP_REDUCEMAX: case TX_OP_REDUCEMIN: {
        int64_t o, rd, inn;
        maxmin_block(d, S(d.in[0]), &o, &rd, &inn);
        int32_t *arg = (int32_t *)tx_alloc_raw(ctx, ny * 4 + 4);
        r->extra[ni] = arg;
        if (!arg) return TX_ERR_OOM;
        return reduce_maxmin(ctx, F(d.in[0]), F(yv), arg, o, rd, inn, d.op == TX_OP_REDUCEMAX);
      }
      case TX_OP_AVGPOOL: {
        const Shape &x = S(d.in[0]);
        const int64_t H = x.size() == 4 ? x[2] : 1, W = x.back();
        int64_t geom[12];
        if (!pool_geom(d, H, W, geom)) return fail(g, TX_ERR_SHAPE, "AveragePool window larger than its padded input");
        return tx_avgpool2d_fwd(ctx, F(d.in[0]), F(yv), x[0] * x[1], H, W, geom, (int)d.iattr[2]);
      }
      case TX_OP_MAXPOOL: {
        const Shape &x = S(d.in[0]);
        const int64_t H = x.size() == 4 ? x[2] : 1, W = x.back();
        int64_t geom[12];
        if (!pool_geom(d, H, W, geom)) return fail(g, TX_ERR_SHAPE, "MaxPool window larger than its padded input");
        int32_t *arg = (int32_t *)tx_alloc_raw(ctx, ny * 4 + 4);
        r->extra[ni] = arg;
        if (!arg) return TX_ERR_OOM;
        return tx_maxpool2d_fwd(ctx, F(d.in[0]), F(yv), arg, x[0] * x[1], H, W, geom);
      }
      case TX_OP_ADD: case TX_OP_SUB: case TX_OP_MUL: case TX_OP_DIV: {
        int64_t sa[TX_MAX_DIMS], sb[TX_MAX_DIMS];
        bstrides(S(d.in[0]), y, sa);
        bstrides(S(d.in[1]), y, sb);
        int op = d.op == TX_OP_ADD ? TX_BIN_ADD : d.op == TX_OP_SUB ? TX_BIN_SUB : d.op == TX_OP_MUL ? TX_BIN_MUL : TX_BIN_DIV;
        return tx_binary(ctx, op, F(d.in[0]), sa, F(d.in[1]), sb, F(yv), y.data(), (int)y.size());
      }
      case TX_OP_RELU: case TX_OP_TANH: case TX_OP_GELU: case TX_OP_SIGMOID: case TX_OP_EXP:
      case TX_OP_LOG: case TX_OP_NEG:
        return tx_unary(ctx, unary_code(d.op), F(d.in[0]), F(yv), ny, 0.f, 0.f);
      case TX_OP_CLIP: {
        float lo = d.iattr[0] ? (float)d.fattr[0] : -INFINITY;
        float hi = d.iattr[1] ? (float)d.fattr[1] : INFINITY;
        return tx_unary(ctx, TX_UN_CLAMP, F(d.in[0]), F(yv), ny, lo, hi);
      }
      case TX_OP_SOFTMAX: case TX_OP_LOGSOFTMAX: {
        const Shape &x = S(d.in[0]);
        int ax = norm_axis(d.iattr[0], (int64_t)x.size());
        if (ax != (int)x.size() - 1) return fail(g, TX_ERR_UNSUPPORTED, "Softmax over a non-final axis is not supported on CUDA");
        int64_t cols = x.back();
        float *y32 = nullptr;
        if (n.round_copy && ctx->math == TX_MATH_TF32) {
          r->extra[ni] = y32 = (float *)tx_alloc_raw(ctx, ny * 4);
          if (!y32) return TX_ERR_OOM;
        }
        return softmax_fwd(ctx, F(d.in[0]), F(yv), y32, ny / cols, cols, d.op == TX_OP_LOGSOFTMAX);
      }
      case TX_OP_REDUCEMEAN: case TX_OP_REDUCESUM: case TX_OP_GAP: {
        const Shape &x = S(d.in[0]);
        Shape keep = x;
        if (d.op == TX_OP_GAP) {
          for (size_t i = 2; i < keep.size(); ++i) keep[i] = 1;
        } else if (d.n_ints == 0) {
          for (auto &k : keep) k = 1;
        } else {
          for (int i = 0; i < d.n_ints; ++i) keep[norm_axis(d.ints[i], (int64_t)x.size())] = 1;
        }
        return tx_reduce_to(ctx, F(d.in[0]), x.data(), F(yv), keep.data(), (int)x.size(),
                            d.op != TX_OP_REDUCESUM, 0);
      }
      case TX_OP_TRANSPOSE: {
        const Shape &x = S(d.in[0]);
        int nd = (int)x.size();
        int64_t xs[TX_MAX_DIMS], ss[TX_MAX_DIMS];
        int64_t st = 1;
        for (int i = nd - 1; i >= 0; --i) { xs[i] = st; st *= x[i]; }
        for (int i = 0; i < nd; ++i) ss[i] = xs[d.n_ints ? d.ints[i] : nd - 1 - i];
        r->tf32[yv] = r->tf32[d.in[0]];  // a transpose moves values unchanged
        return tx_strided_copy(ctx, F(d.in[0]), ss, F(yv), y.data(), nd, g->values[d.in[0]].dtype == TX_DT_I64 ? 8 : 4);
      }
    }
    return fail(g, TX_ERR_UNSUPPORTED, "operator " + std::to_string(d.op) + " has no CUDA forward");
  }
};

}  // namespace

extern "C" int tx_graph_forward(tx_graph *g, const void *const *d_inputs, const int64_t *in_shapes,
                                const int32_t *in_ndims, void *const *d_outputs, int tracking,
                                tx_record **rec_out) {
  if (!g) return TX_ERR_INVALID;
  if (rec_out) *rec_out = nullptr;
  tx_ctx *ctx = g->ctx;
  std::unique_ptr<tx_record> r(new tx_record());
  r->g = g;
  r->tracking = tracking != 0;
  TX_TRY(infer_all(g, in_shapes, in_ndims, r->shapes));
  size_t nv = g->values.size();
  r->buf.assign(nv, nullptr);
  r->owned.assign(nv, false);
  r->extra.assign(g->nodes.size(), nullptr);
  r->extra2.assign(g->nodes.size(), {});
  r->tf32.assign(nv, false);
  r->attn_fused.assign(g->attn.size(), 0);
  r->proj_done.assign(g->proj.size(), 0);
  r->conv_implicit.assign(g->nodes.size(), 0);
  if (ctx->math == TX_MATH_TF32 && g->flat_len > 0) {
    // the contractions of this forward (and of its backward) read parameters
    // from a TF32-rounded copy, refreshed here so that it always matches the
    // fp32 values whatever changed them since
    if (!g->flat_tf32) TX_CUDA(ctx, cudaMalloc(&g->flat_tf32, g->flat_len * sizeof(float)));
    if (!g->flat_lo) TX_CUDA(ctx, cudaMalloc(&g->flat_lo, g->flat_len * sizeof(float)));
    TX_TRY(tx_split_tf32(ctx, g->flat_values, g->flat_tf32, g->flat_lo, g->flat_len));
    r->shadow = true;
  }
  for (size_t i = 0; i < g->inputs.size(); ++i) {
    const int v = g->inputs[i];
    r->buf[v] = const_cast<void *>(d_inputs[i]);
    if (r->shadow && g->input_round[i] && numel_of(r->shapes[v]) >= (int64_t(1) << 20)) {
      // an input only contractions read is rounded once here, not in every
      // GEMM that reads it (the copy lives with the record: backward reads it)
      const int64_t n = numel_of(r->shapes[v]);
      void *copy = tx_alloc_raw(ctx, n * 4);
      int rc = copy ? tx_round_tf32(ctx, (const float *)d_inputs[i], (float *)copy, n) : TX_ERR_OOM;
      if (copy) {
        r->buf[v] = copy;
        r->owned[v] = true;
        r->tf32[v] = true;
      }
      if (rc != TX_OK) {
        tx_record_free(r.release());
        return rc;
      }
    }
  }
  for (size_t i = 0; i < nv; ++i)
    if (g->values[i].kind == TX_VAL_PARAM || g->values[i].kind == TX_VAL_CONST) r->buf[i] = g->values[i].dev;
  // outputs are written straight into the caller's buffers, unless an output
  // aliases another value (reshape of an input, an output listed twice...)
  for (size_t i = 0; i < g->outputs.size(); ++i) {
    int v = g->outputs[i];
    const GValue &gv = g->values[v];
    if (gv.kind != TX_VAL_ACT || gv.producer < 0) continue;
    const GNode &p = g->nodes[gv.producer];
    if (is_alias_op(p.d.op) || r->buf[v]) continue;
    r->buf[v] = d_outputs[i];
  }
  Fwd f{g, ctx, r.get()};
  int rc = TX_OK;
  for (size_t i = 0; i < g->nodes.size() && rc == TX_OK; ++i) rc = f.node((int)i);
  if (rc == TX_OK) {
    for (size_t i = 0; i < g->outputs.size(); ++i) {
      int v = g->outputs[i];
      if (r->buf[v] != d_outputs[i]) {
        size_t bytes = numel_of(r->shapes[v]) * (g->values[v].dtype == TX_DT_I64 ? 8 : 4);
        rc = tx_d2d(ctx, d_outputs[i], r->buf[v], bytes);
        if (rc) break;
      }
    }
  }
  if (rc != TX_OK || !tracking || !rec_out) {
    tx_record_free(r.release());
    return rc;
  }
  *rec_out = r.release();
  return TX_OK;
}

extern "C" int tx_record_free(tx_record *r) {
  if (!r) return TX_OK;
  tx_ctx *ctx = r->g->ctx;
  for (size_t i = 0; i < r->buf.size(); ++i)
    if (r->owned[i]) tx_free_raw(ctx, r->buf[i]);
  for (void *p : r->extra) tx_free_raw(ctx, p);
  for (auto &v : r->extra2)
    for (void *p : v) tx_free_raw(ctx, p);
  delete r;
  return TX_OK;
}

// ============================================================================
// backward
// ============================================================================
namespace {

struct Bwd {
  tx_graph *g;
  tx_ctx *ctx;
  tx_record *r;
  std::vector<float *> grad;       // per value gradient buffer
  std::vector<bool> grad_owned;
  std::vector<bool> grad_preact;   // gradient already multiplied by act' (fused dgrad)
  std::vector<bool> grad_tf32;     // gradient buffer holds TF32-rounded values
  std::vector<bool> bias_fused;    // per node: bias gradient already summed by a dgrad epilogue
  std::vector<bool> needs;         // value needs a gradient
  std::vector<float *> param_tmp;  // unused
  // DP bucketing
  std::vector<bool> param_done;
  size_t next_final = 0;      // index into g->grad_final_order
  int64_t bucket_start = 0;   // flat offset of the first not-yet-reduced element
  std::vector<int> param_pending;  // remaining contributions per param

  float *F(int v) { return (float *)r->buf[v]; }
  const Shape &S(int v) { return r->shapes[v]; }

  // Returns the buffer to write the gradient of value v into and whether the
  // write must accumulate.  Parameter slots honour grad_defined.
  int target(int v, float **out, int *acc) {
    GValue &gv = g->values[v];
    if (gv.kind == TX_VAL_PARAM) {
      *out = gv.grad;
      *acc = gv.grad_defined ? 1 : 0;
      return TX_OK;
    }
    if (grad[v]) {
      *out = grad[v];
      *acc = 1;
      return TX_OK;
    }
    grad[v] = (float *)tx_alloc_raw(ctx, numel_of(S(v)) * 4 + 4);
    if (!grad[v]) return TX_ERR_OOM;
    grad_owned[v] = true;
    *out = grad[v];
    *acc = 0;
    return TX_OK;
  }

  void wrote(int v) {
    GValue &gv = g->values[v];
    if (gv.kind == TX_VAL_PARAM) {
      gv.grad_defined = true;
      param_contribution_done(gv.param_index);
    }
  }

  // ---- DP: launch all-reduce for contiguous ranges of final gradients ----------
  void param_contribution_done(int p) {
    if (--param_pending[p] > 0) return;
    param_done[p] = true;
    if (!g->dp) return;
    int64_t end = bucket_start;
    while (next_final < g->grad_final_order.size() && param_done[g->grad_final_order[next_final]]) {
      int q = g->grad_final_order[next_final];
      int64_t n = numel_of(g->values[g->params[q]].shape);
      end = g->param_offset[q] + ((n + 63) & ~int64_t(63));
      ++next_final;
    }
    if ((end - bucket_start) * 4 >= g->bucket_bytes) flush(end);
  }

  int flush(int64_t end) {
    if (end <= bucket_start) return TX_OK;
    TX_TRY(dp_event_fork(ctx));
    TX_TRY(dp_allreduce_range(ctx, g->flat_grads + bucket_start, end - bucket_start));
    bucket_start = end;
    return TX_OK;
  }

  int gemm_backward(int ni) {
    GNode &n = g->nodes[ni];
    const tx_node_desc &d = n.d;
    int yv = n.fused_act ? n.fused_out : n.scale_out >= 0 ? n.scale_out : d.out[0];
    float *dy = grad[yv];
    if (!dy) return TX_OK;
    // gradient with respect to the pre-activation
    float *dz = dy;
    float *dz_tmp = nullptr;
    if (n.fused_act && !grad_preact[yv]) {
      int64_t ny = numel_of(S(yv));
      dz_tmp = (float *)tx_alloc_raw(ctx, ny * 4);
      if (!dz_tmp) return TX_ERR_OOM;
      if (n.fused_act == TX_ACT_GELU)
        TX_TRY(tx_unary_bwd(ctx, TX_UN_GELU, (const float *)r->extra[ni], dy, dz_tmp, ny, 0.f, 0.f, 0));
      else
        TX_TRY(tx_unary_bwd(ctx, n.fused_act == TX_ACT_RELU ? TX_UN_RELU : TX_UN_TANH, F(yv), dy, dz_tmp, ny, 0.f, 0.f, 0));
      dz = dz_tmp;
    }
    const Shape &a = S(d.in[0]), &b = S(d.in[1]);
    int rc = TX_OK;
    bool dz32 = dz == dy && grad_tf32[yv];  // dZ came TF32-rounded from a fused dgrad
    float *dz_rnd = nullptr;
    if (d.op == TX_OP_GEMM) {
      int ta = (int)d.iattr[0], tb = (int)d.iattr[1];
      int64_t M = ta ? a[1] : a[0], K = ta ? a[0] : a[1], N = tb ? b[0] : b[1];
      float alpha = (float)d.fattr[0] * n.out_scale;
      // bias (unless the dgrad that produced dZ already summed it)
      if (rc == TX_OK && d.n_in > 2 && d.in[2] >= 0 && needs[d.in[2]] && !bias_fused[ni]) {
        float *t; int acc;
        rc = target(d.in[2], &t, &acc);
        if (rc == TX_OK) rc = tx_bias_grad(ctx, dz, t, M, N, (float)d.fattr[1], acc);
        if (rc == TX_OK) wrote(d.in[2]);
      }
      // dB
      if (rc == TX_OK && needs[d.in[1]]) {
        float *t; int acc;
        rc = target(d.in[1], &t, &acc);
        tx_gemm_desc q; memset(&q, 0, sizeof q);
        q.alpha = alpha; q.beta = acc ? 1.f : 0.f; q.batch = 1;
        bool x32 = false;
        const float *x = gemm_operand(g, r, d.in[0], &x32);
        if (!tb) {  // dB[K,N] = op(A)^T dY
          q.M = K; q.N = N; q.K = M;
          q.A = x; q.lda = a[1]; q.trans_a = ta ? 0 : 1;
          q.B = dz; q.ldb = N; q.trans_b = 0;
          q.C = t; q.ldc = N;
          q.flags = (x32 ? TX_GEMM_A_TF32 : 0) | (dz32 ? TX_GEMM_B_TF32 : 0);
        } else {    // dB[N,K] = dY^T op(A)
          q.M = N; q.N = K; q.K = M;
          q.A = dz; q.lda = N; q.trans_a = 1;
          q.B = x; q.ldb = a[1]; q.trans_b = ta ? 1 : 0;
          q.C = t; q.ldc = K;
          q.flags = (x32 ? TX_GEMM_B_TF32 : 0) | (dz32 ? TX_GEMM_A_TF32 : 0);
        }
        round_grad(d.in[1], q);
        bool rounded = false;
        if (rc == TX_OK) rc = gemm_dispatch(ctx, q, &rounded);
        if (rc == TX_OK) {
          grad_tf32[d.in[1]] = rounded;
          wrote(d.in[1]);
        }
      }
      // dA
      if (rc == TX_OK && needs[d.in[0]]) {
        float *t; int acc;
        int fused_node = -1;
        rc = dgrad_target(d.in[0], &t, &acc);
        tx_gemm_desc q; memset(&q, 0, sizeof q);
        q.alpha = alpha; q.beta = acc ? 1.f : 0.f; q.batch = 1;
        bool w32 = false;
        const float *w = gemm_operand(g, r, d.in[1], &w32);
        if (!ta) {  // dA[M,K] = dY op(B)^T
          q.M = M; q.N = K; q.K = N;
          q.A = dz; q.lda = N; q.trans_a = 0;
          q.B = w; q.ldb = b[1]; q.trans_b = tb ? 0 : 1;
          q.C = t; q.ldc = K;
          q.flags = (w32 ? TX_GEMM_B_TF32 : 0) | (dz32 ? TX_GEMM_A_TF32 : 0);
          fused_node = fuse_dact(d.in[0], q);
        } else {    // dA[K,M] = op(B) dY^T
          q.M = K; q.N = M; q.K = N;
          q.A = w; q.lda = b[1]; q.trans_a = tb ? 1 : 0;
          q.B = dz; q.ldb = N; q.trans_b = 1;
          q.C = t; q.ldc = M;
          q.flags = (w32 ? TX_GEMM_A_TF32 : 0) | (dz32 ? TX_GEMM_B_TF32 : 0);
        }
        round_grad(d.in[0], q);
        bool rounded = false;
        if (rc == TX_OK) rc = gemm_dispatch(ctx, q, &rounded);
        if (rc == TX_OK) {
          fused_done(d.in[0], fused_node, rounded);
          wrote(d.in[0]);
        }
      }
    } else {  // MATMUL
      int64_t K = a.back(), N = b.back();
      bool weight2d = b.size() == 2;
      int64_t M = weight2d ? numel_of(a) / K : a[a.size() - 2];
      int64_t batch = weight2d ? 1 : numel_of(a) / (M * K);
      // TF32 mode: a dZ that the dgrad would round into scratch anyway (at
      // most half the size of dA, more 128 x 256 tiles of dA than SMs) is
      // rounded once here, and the wgrad reads the same copy without
      // conversion (the second MatMul of a 256 -> 1024 -> 256 FFN over 32768
      // rows: wgrad 53 -> 40 us)
      if (ctx->math == TX_MATH_TF32 && !dz32 && weight2d && needs[d.in[0]] && needs[d.in[1]] && 2 * N <= K &&
          M * K > (int64_t)ctx->num_sms * 128 * 256) {
        dz_rnd = (float *)tx_alloc_raw(ctx, M * N * 4);
        if (!dz_rnd) rc = TX_ERR_OOM;
        if (rc == TX_OK) rc = tx_round_tf32(ctx, dz, dz_rnd, M * N);
        if (rc == TX_OK) {
          dz = dz_rnd;
          dz32 = true;
        }
      }
      if (rc == TX_OK && needs[d.in[1]]) {  // dB = A^T dY
        float *t; int acc;
        rc = target(d.in[1], &t, &acc);
        tx_gemm_desc q; memset(&q, 0, sizeof q);
        q.alpha = n.out_scale; q.beta = acc ? 1.f : 0.f; q.batch = batch;
        q.M = K; q.N = N; q.K = M;
        bool x32 = false;
        q.A = gemm_operand(g, r, d.in[0], &x32); q.lda = K; q.trans_a = 1; q.stride_a = M * K;
        q.flags = (x32 ? TX_GEMM_A_TF32 : 0) | (dz32 ? TX_GEMM_B_TF32 : 0);
        q.B = dz; q.ldb = N; q.trans_b = 0; q.stride_b = M * N;
        q.C = t; q.ldc = N; q.stride_c = K * N;
        round_grad(d.in[1], q);
        bool rounded = false;
        if (rc == TX_OK) rc = gemm_dispatch(ctx, q, &rounded);
        if (rc == TX_OK) {
          grad_tf32[d.in[1]] = rounded;
          wrote(d.in[1]);
        }
      }
      if (rc == TX_OK && needs[d.in[0]]) {  // dA = dY B^T
        float *t; int acc;
        rc = dgrad_target(d.in[0], &t, &acc);
        tx_gemm_desc q; memset(&q, 0, sizeof q);
        q.alpha = n.out_scale; q.beta = acc ? 1.f : 0.f; q.batch = batch;
        q.M = M; q.N = K; q.K = N;
        q.A = dz; q.lda = N; q.trans_a = 0; q.stride_a = M * N;
        bool w32 = false;
        q.B = gemm_operand(g, r, d.in[1], &w32); q.ldb = N; q.trans_b = 1; q.stride_b = weight2d ? 0 : K * N;
        q.flags = (w32 ? TX_GEMM_B_TF32 : 0) | (dz32 ? TX_GEMM_A_TF32 : 0);
        q.C = t; q.ldc = K; q.stride_c = M * K;
        if (weight2d) { q.M = M; q.batch = 1; }
        const int fused_node = fuse_dact(d.in[0], q);
        round_grad(d.in[0], q);
        bool rounded = false;
        if (rc == TX_OK) rc = gemm_dispatch(ctx, q, &rounded);
        if (rc == TX_OK) {
          fused_done(d.in[0], fused_node, rounded);
          wrote(d.in[0]);
        }
      }
    }
    if (dz_tmp) tx_free_raw(ctx, dz_tmp);
    if (dz_rnd) tx_free_raw(ctx, dz_rnd);
    return rc;
  }

  int dgrad_target(int v, float **t, int *acc) { return target(v, t, acc); }

  // TF32 mode: a gradient that only contractions read (GValue::grad_round) is
  // stored rounded by the contraction that writes it, as those readers would
  // round it anyway; recorded in grad_tf32 from what gemm_dispatch reports
  void round_grad(int v, tx_gemm_desc &q) {
    if (ctx->math == TX_MATH_TF32 && q.beta == 0.f && !q.dact && !q.colsum && g->values[v].grad_round)
      q.flags |= TX_GEMM_ROUND_OUT;
  }

  // If v is the (sole-consumer) output of a fused Gemm+act, fold act' into this
  // dgrad epilogue so the producer receives its pre-activation gradient dZ.
  // When the producer is a Gemm whose bias needs a gradient, the same epilogue
  // also sums dZ's columns into it (the returned node's bias is then done);
  // and since the producer's backward reads dZ only as a contraction operand,
  // dZ is stored TF32-rounded in TF32 mode.  Returns the producer node whose
  // bias gradient was fused, or -1.
  int fuse_dact(int v, tx_gemm_desc &q) {
    const GValue &gv = g->values[v];
    if (gv.kind != TX_VAL_ACT || gv.producer < 0 || gv.is_output) return -1;
    const GNode &p = g->nodes[gv.producer];
    if (p.fused_into < 0 || gv.consumers.size() != 1 || q.beta != 0.f) return -1;
    const int pi = p.fused_into;
    const GNode &prod = g->nodes[pi];
    if (prod.fused_out != v) return -1;
    q.dact = prod.fused_act;
    q.dact_src = prod.fused_act == TX_ACT_GELU ? (const float *)r->extra[pi] : F(v);
    q.ld_dact = q.N;
    grad_preact[v] = true;
    if (prod.d.op != TX_OP_GEMM && prod.d.op != TX_OP_MATMUL) return -1;
    const bool has_bias = prod.d.op == TX_OP_GEMM && prod.d.n_in > 2 && prod.d.in[2] >= 0;
    int fused = -1;
    if (has_bias && needs[prod.d.in[2]] && q.batch <= 1) {
      float *t; int acc;
      if (target(prod.d.in[2], &t, &acc) == TX_OK) {
        q.colsum = t;
        q.colsum_scale = (float)prod.d.fattr[1];
        q.colsum_acc = acc;
        fused = pi;
      }
    }
    if (ctx->math == TX_MATH_TF32 && (fused >= 0 || !has_bias || !needs[prod.d.in[2]]))
      q.flags |= TX_GEMM_ROUND_OUT;
    return fused;
  }

  // after a dgrad launched with fuse_dact: record what it produced
  void fused_done(int v, int fused_node, bool rounded) {
    grad_tf32[v] = rounded;
    if (fused_node >= 0) {
      bias_fused[fused_node] = true;
      wrote(g->nodes[fused_node].d.in[2]);
    }
  }

  // dX = the outputs' gradients in their slabs (zeros where an output has none)
  int split_backward(int ni) {
    const tx_node_desc &d = g->nodes[ni].d;
    const int xv = d.in[0];
    if (!needs[xv]) return TX_OK;
    bool any = false;
    for (int k = 0; k < d.n_out; ++k) any |= grad[d.out[k]] != nullptr;
    if (!any) return TX_OK;
    const Shape &x = S(xv);
    const int ax = norm_axis(d.iattr[0], (int64_t)x.size());
    int64_t xs[TX_MAX_DIMS];
    cstrides(x, xs);
    float *t; int acc;
    TX_TRY(target(xv, &t, &acc));
    if (!acc) TX_CUDA(ctx, cudaMemsetAsync(t, 0, numel_of(x) * 4, ctx->stream));
    int64_t at = 0;
    for (int k = 0; k < d.n_out; ++k) {
      const Shape &ok = S(d.out[k]);
      if (grad[d.out[k]]) TX_TRY(nd_scatter(ctx, grad[d.out[k]], t + at * xs[ax], xs, ok.data(), (int)ok.size(), 1));
      at += ok[ax];
    }
    wrote(xv);
    return TX_OK;
  }

  // dX as one implicit GEMM per phase of the stride (see the implicit-GEMM
  // note above the kernels): A gathered from the channels-last dY with the
  // phase's tap shifts, B the taps' [C][OC] weight blocks, the output written
  // through a view of dX with the phase's origin and strides (and act' of a
  // channels-last producer applied there, as col2im applied it).
  // TX_ERR_UNSUPPORTED with `launched` false: nothing ran, and the columns path runs.
  int conv_dgrad_implicit(int ni, const ConvGeom &cg, const float *dz, float *t, int acc, bool &launched) {
    launched = false;
    GNode &n = g->nodes[ni];
    const tx_node_desc &d = n.d;
    const int64_t OC = S(d.in[1])[0];
    if (OC % 32 || cg.C % 4 || cg.H % cg.sh || cg.W % cg.sw || cg.KH * cg.KW > tx_tc::kGatherTaps) return TX_ERR_UNSUPPORTED;
    const int Hp = cg.H / cg.sh, Wp = cg.W / cg.sw;
    uint32_t bw, bh, bn;
    if (!pixel_box(Hp, Wp, tx_tc::TC_BM, bw, bh, bn) || bw > 256 || bh > 256 || bn > 256) return TX_ERR_UNSUPPORTED;
    if (!(Wp % 32 == 0 || 32 % Wp == 0)) return TX_ERR_UNSUPPORTED;
    // every phase must take at least one tap (else part of dX has no product)
    auto phase_taps = [&](int ph, int pw, tx_tc::GatherOp &op) {
      int nt = 0;
      for (int kh = 0; kh < cg.KH; ++kh) {
        const int a = ph + cg.pt - kh * cg.dh;
        if (((a % cg.sh) + cg.sh) % cg.sh) continue;
        for (int kw = 0; kw < cg.KW; ++kw) {
          const int b = pw + cg.pl - kw * cg.dw;
          if (((b % cg.sw) + cg.sw) % cg.sw) continue;
          op.offx[nt] = (int16_t)(b / cg.sw);  // exact quotients (b, a divisible)
          op.offy[nt] = (int16_t)(a / cg.sh);
          op.wtap[nt] = (int16_t)(kh * cg.KW + kw);
          ++nt;
        }
      }
      return nt;
    };
    for (int ph = 0; ph < cg.sh; ++ph)
      for (int pw = 0; pw < cg.sw; ++pw) {
        tx_tc::GatherOp probe;
        if (phase_taps(ph, pw, probe) == 0) return TX_ERR_UNSUPPORTED;
      }
    // the producer's act' against its channels-last output, when nothing accumulates
    const int xv = d.in[0];
    const GValue &xg = g->values[xv];
    int pc = xg.producer;
    if (pc >= 0 && g->nodes[pc].fused_into >= 0) pc = g->nodes[pc].fused_into;
    const GNode *pn = pc >= 0 ? &g->nodes[pc] : nullptr;
    const bool fuse = n.nhwc_in && !acc && pn && pn->d.op == TX_OP_CONV && pn->nhwc_out && pn->fused_act &&
                      (pn->fused_act == TX_ACT_RELU || pn->fused_act == TX_ACT_TANH) && pn->fused_out == xv;
    const bool tf32 = ctx->math == TX_MATH_TF32;
    const int64_t taps = (int64_t)cg.KH * cg.KW;
    Scratch wt(ctx, (size_t)taps * cg.C * OC * 4),
        dxh(ctx, n.nhwc_in ? 0 : (size_t)cg.N * cg.H * cg.W * cg.C * 4);
    if (!wt.ptr || (!n.nhwc_in && !dxh.ptr)) return TX_ERR_OOM;
    k_weight_to_tco<<<grid_for(taps * cg.C * OC, 256), 256, 0, ctx->stream>>>(F(d.in[1]), wt.as<float>(), (int)OC,
                                                                             cg.C, cg.KH, cg.KW, tf32);
    TX_LAUNCHED(ctx, "k_weight_to_tco");
    launched = true;  // from here a refusal is an error (part of dX may be written)
    float *dst = n.nhwc_in ? t : dxh.as<float>();
    for (int ph = 0; ph < cg.sh; ++ph)
      for (int pw = 0; pw < cg.sw; ++pw) {
        tx_tc::ConvGemm cv;
        memset(&cv, 0, sizeof cv);
        tx_tc::GatherOp &op = cv.op;
        op.ntaps = phase_taps(ph, pw, op);
        op.a = 1;
        op.b = 2;
        op.cblocks = (int)(OC / 32);
        op.ohw = Hp * Wp;
        op.ow = Wp;
        op.sw = 1;
        op.sh = 1;
        op.brows = cg.C;
        op.wsplit = Wp;
        cv.src = {dz, cg.N, cg.OH, cg.OW, OC};
        cv.box[0] = 32; cv.box[1] = bw; cv.box[2] = bh; cv.box[3] = bn;
        cv.estr_w = cv.estr_h = 1;
        cv.b_inner = OC;
        cv.b_rows = taps * cg.C;
        cv.out_rows = (int64_t)cg.N * Hp;
        cv.out_sw = (int64_t)cg.sw * cg.C;
        cv.out_sr = (int64_t)cg.sh * cg.W * cg.C;
        const int64_t origin = ((int64_t)ph * cg.W + pw) * cg.C;
        tx_gemm_desc q;
        memset(&q, 0, sizeof q);
        q.M = (int64_t)cg.N * Hp * Wp; q.N = cg.C; q.K = op.ntaps * OC;
        q.A = dz; q.lda = OC; q.trans_a = 0;
        q.B = wt.as<float>(); q.ldb = OC; q.trans_b = 1;
        q.C = dst + origin; q.ldc = cg.C; q.alpha = 1.f; q.batch = 1;
        if (n.nhwc_in && acc) q.beta = 1.f;
        if (fuse) {
          q.dact = pn->fused_act;
          q.dact_src = F(xv) + origin;
          q.ld_dact = cg.C;
        }
        q.flags = tf32 ? TX_GEMM_B_TF32 : 0;
        const int mode = tc_mode(ctx, q);
        const int rc = gemm_conv_tc(ctx, q, mode, cv);
        if (rc == TX_ERR_UNSUPPORTED) return tx_fail(ctx, rc, "implicit data gradient: the product was refused");
        TX_TRY(rc);
      }
    if (fuse) grad_preact[xv] = true;
    if (!n.nhwc_in)
      return transpose_b(ctx, dxh.as<float>(), t, cg.N, (int64_t)cg.H * cg.W, cg.C, nullptr, nullptr, TX_ACT_NONE,
                         acc);
    return TX_OK;
  }

  int conv_backward(int ni) {
    GNode &n = g->nodes[ni];
    const tx_node_desc &d = n.d;
    const int yv = n.fused_act ? n.fused_out : d.out[0];
    float *dy = grad[yv];
    if (!dy) return TX_OK;
    const Shape &x = S(d.in[0]), &w = S(d.in[1]), &y = S(d.out[0]);
    const ConvGeom cg = conv_geom(x, w, y, d);
    const int64_t M = (int64_t)cg.N * cg.OH * cg.OW, OC = w[0];
    const bool tf32 = ctx->math == TX_MATH_TF32;
    // dY (NCHW) -> [M, OC]; a fused activation's derivative is applied on the
    // way.  A channels-last output got its dY channels-last from the next
    // convolution: act' is then elementwise against the channels-last output.
    const bool apply_dact = n.fused_act && !grad_preact[yv];
    // a channels-last dY whose act' the next convolution applied is used as is
    const bool dy_ready = n.nhwc_out && !apply_dact;
    Scratch dyt(ctx, dy_ready ? 0 : (size_t)M * OC * 4);
    if (!dy_ready && !dyt.ptr) return TX_ERR_OOM;
    float *dz = dy_ready ? dy : dyt.as<float>();
    if (dy_ready) {
    } else if (n.nhwc_out) {
      TX_TRY(tx_unary_bwd(ctx, n.fused_act == TX_ACT_RELU ? TX_UN_RELU : TX_UN_TANH, F(yv), dy, dz, M * OC, 0.f,
                          0.f, 0));
    } else {
      TX_TRY(transpose_b(ctx, dy, dz, cg.N, OC, (int64_t)cg.OH * cg.OW, nullptr,
                         apply_dact ? F(yv) : nullptr, apply_dact ? n.fused_act : TX_ACT_NONE));
    }
    const bool direct = r->conv_implicit[ni] == 2;
    const bool bias_grad = d.n_in > 2 && d.in[2] >= 0 && needs[d.in[2]];
    if (direct && needs[d.in[1]]) {
      // weight and bias gradients in one pass over the NCHW input and dZ
      const int geom[14] = {cg.N, cg.C, cg.H, cg.W, cg.KH, cg.KW, cg.OH, cg.OW, cg.sh, cg.sw, cg.pt, cg.pl, cg.dh, cg.dw};
      float *tw, *tb = nullptr; int aw, ab = 0;
      TX_TRY(target(d.in[1], &tw, &aw));
      if (bias_grad) TX_TRY(target(d.in[2], &tb, &ab));
      TX_TRY(conv_direct_wgrad(ctx, F(d.in[0]), dz, geom, (int)OC, tw, tb, aw, ab));
      wrote(d.in[1]);
      if (bias_grad) wrote(d.in[2]);
    } else if (bias_grad) {
      float *t; int acc;
      TX_TRY(target(d.in[2], &t, &acc));
      TX_TRY(tx_bias_grad(ctx, dz, t, M, OC, 1.f, acc));
      wrote(d.in[2]);
    }
    // per group g (one group unless the convolution is grouped): columns
    // [M][ldk_g] of the channel slice, weights rows [g OCg, (g + 1) OCg)
    const int G = d.iattr[0];
    const ConvGeom g0 = conv_group(cg, G, 0);
    const int64_t ldk = g0.ldk, OCg = OC / G;
    if (!direct && needs[d.in[1]]) {  // dW_khwc[OC, ldk] = dY^T cols, then back to [OC, C, KH, KW]
      float *t; int acc;
      TX_TRY(target(d.in[1], &t, &acc));
      Scratch dwk(ctx, (size_t)OC * ldk * 4);
      if (!dwk.ptr) return TX_ERR_OOM;
      tx_gemm_desc q; memset(&q, 0, sizeof q);
      q.M = OC; q.N = ldk; q.K = M; q.alpha = 1.f; q.batch = 1;
      q.A = dz; q.lda = OC; q.trans_a = 1;
      q.C = dwk.as<float>(); q.ldc = ldk;
      if (r->conv_implicit[ni] == 1) {
        // B gathered from the channels-last input, 32 pixels per sub-tile;
        // without a fitting box the columns are built here after all
        const float *xin = r->extra[ni] ? (const float *)r->extra[ni] : F(d.in[0]);
        tx_tc::ConvGemm cv;
        int rc = TX_ERR_UNSUPPORTED;
        q.B = xin; q.ldb = ldk; q.trans_b = 0;
        if (conv_gather_fwd(cg, 32, cv)) {
          cv.op.b = 1;
          cv.src = {xin, cg.N, cg.H, cg.W, cg.C};
          tx_gemm_desc e = q;
          const int mode = tc_mode(ctx, e);
          rc = gemm_conv_tc(ctx, e, mode, cv);
        }
        Scratch cols(ctx, rc == TX_ERR_UNSUPPORTED ? (size_t)M * ldk * 4 : 0);
        if (rc == TX_ERR_UNSUPPORTED) {
          if (!cols.ptr) return TX_ERR_OOM;
          TX_TRY(im2col_nhwc(ctx, xin, cols.as<float>(), cg, tf32));
          q.B = cols.as<float>();
          q.flags = tf32 ? TX_GEMM_B_TF32 : 0;
          rc = gemm_dispatch(ctx, q);
        }
        TX_TRY(rc);
      } else {
        for (int gi = 0; gi < G; ++gi) {
          tx_gemm_desc e = q;
          e.M = OCg;
          e.A = dz + gi * OCg;
          e.B = (const float *)r->extra[ni] + gi * M * ldk; e.ldb = ldk; e.trans_b = 0;
          e.C = dwk.as<float>() + gi * OCg * ldk;
          e.flags = tf32 ? TX_GEMM_B_TF32 : 0;
          TX_TRY(gemm_dispatch(ctx, e));
        }
      }
      k_weight_from_khwc<<<grid_for(OC * g0.C * cg.KH * cg.KW, 256), 256, 0, ctx->stream>>>(
          dwk.as<float>(), t, (int)OC, g0.C, cg.KH, cg.KW, (int)ldk, acc);
      TX_LAUNCHED(ctx, "k_weight_from_khwc");
      wrote(d.in[1]);
    }
    if (needs[d.in[0]]) {  // dcols[M, ldk] = dY W_khwc ; dx = col2im(dcols) -> NCHW
      float *t; int acc;
      TX_TRY(target(d.in[0], &t, &acc));
      if (ctx->math != TX_MATH_FP32 && G == 1) {
        bool launched = false;
        const int rc = conv_dgrad_implicit(ni, cg, dz, t, acc, launched);
        if (rc != TX_ERR_UNSUPPORTED || launched) {
          TX_TRY(rc);
          wrote(d.in[0]);
          return TX_OK;
        }
      }
      Scratch wk(ctx, (size_t)OC * ldk * 4), dcols(ctx, (size_t)M * ldk * 4),
          dxh(ctx, (size_t)cg.N * cg.H * cg.W * cg.C * 4);
      if (!wk.ptr || !dcols.ptr || !dxh.ptr) return TX_ERR_OOM;
      k_weight_to_khwc<<<grid_for(OC * ldk, 256), 256, 0, ctx->stream>>>(F(d.in[1]), wk.as<float>(), (int)OC,
                                                                        g0.C, cg.KH, cg.KW, (int)ldk, tf32);
      TX_LAUNCHED(ctx, "k_weight_to_khwc");
      // the producer reads dX channels-last; its fused activation's
      // derivative is applied here, against its channels-last output
      const int xv = d.in[0];
      const GValue &xg = g->values[xv];
      int pc = xg.producer;
      if (pc >= 0 && g->nodes[pc].fused_into >= 0) pc = g->nodes[pc].fused_into;
      const GNode *pn = pc >= 0 ? &g->nodes[pc] : nullptr;
      const bool fuse = n.nhwc_in && !acc && pn && pn->d.op == TX_OP_CONV && pn->nhwc_out && pn->fused_act &&
                        (pn->fused_act == TX_ACT_RELU || pn->fused_act == TX_ACT_TANH) && pn->fused_out == xv;
      float *dst = (n.nhwc_in && !acc) ? t : dxh.as<float>();
      for (int gi = 0; gi < G; ++gi) {
        tx_gemm_desc q; memset(&q, 0, sizeof q);
        q.M = M; q.N = ldk; q.K = OCg; q.alpha = 1.f; q.batch = 1;
        q.A = dz + gi * OCg; q.lda = OC; q.trans_a = 0;
        q.B = wk.as<float>() + gi * OCg * ldk; q.ldb = ldk; q.trans_b = 0;
        q.C = dcols.as<float>(); q.ldc = ldk;
        q.flags = tf32 ? TX_GEMM_B_TF32 : 0;
        TX_TRY(gemm_dispatch(ctx, q));
        TX_TRY(col2im_nhwc(ctx, dcols.as<float>(), dst, conv_group(cg, G, gi), fuse ? F(xv) : nullptr,
                           fuse ? pn->fused_act : TX_ACT_NONE));
      }
      if (fuse) grad_preact[xv] = true;
      if (n.nhwc_in && acc) {
        const int64_t nx = (int64_t)cg.N * cg.H * cg.W * cg.C, one = 1;
        TX_TRY(nd_copy(ctx, dxh.as<float>(), &one, t, &nx, 1, 4, 1.f, acc));
      } else if (!n.nhwc_in) {
        TX_TRY(transpose_b(ctx, dxh.as<float>(), t, cg.N, (int64_t)cg.H * cg.W, cg.C, nullptr, nullptr,
                           TX_ACT_NONE, acc));
      }
      wrote(d.in[0]);
    }
    return TX_OK;
  }

  // dX (+)= reduce_to_shape(src) for broadcast binary backward
  // dst (+)= src over n elements
  int add_or_copy(float *dst, const float *src, int64_t n, int acc) {
    if (!acc) return tx_d2d(ctx, dst, src, n * 4);
    k_axpy<<<grid_for(n, 256), 256, 0, ctx->stream>>>(dst, src, n, 1.f);
    TX_LAUNCHED(ctx, "k_axpy");
    return TX_OK;
  }

  int reduce_into(int v, const float *src, const Shape &from, float scale) {
    float *t; int acc;
    TX_TRY(target(v, &t, &acc));
    Shape xs = S(v);
    Shape padded(from.size() - xs.size(), 1);
    padded.insert(padded.end(), xs.begin(), xs.end());
    int rc;
    if (numel_of(padded) == numel_of(from)) {
      if (scale == 1.f && !acc) rc = tx_d2d(ctx, t, src, numel_of(from) * 4);
      else if (!acc) rc = tx_unary(ctx, TX_UN_SCALE, src, t, numel_of(from), scale, 0.f);
      else {
        k_axpy<<<grid_for(numel_of(from), 256), 256, 0, ctx->stream>>>(t, src, numel_of(from), scale);
        TX_LAUNCHED(ctx, "k_axpy");
        rc = TX_OK;
      }
    } else {
      if (scale != 1.f) return fail(g, TX_ERR_UNSUPPORTED, "scaled broadcast reduction");
      rc = tx_reduce_to(ctx, src, from.data(), t, padded.data(), (int)from.size(), 0, acc);
    }
    if (rc == TX_OK) wrote(v);
    return rc;
  }

  int attn_backward(const AttnPlan &a) {
    const float *dout = grad[a.out];
    if (!dout) return TX_OK;
    const Shape &q = S(a.q);
    const int64_t B = q[0], Sq = q[1], E = q[2];
    float *t[3];
    int acc[3];
    const int vs[3] = {a.q, a.k, a.v};
    for (int i = 0; i < 3; ++i) TX_TRY(target(vs[i], &t[i], &acc[i]));
    const bool all_acc = acc[0] && acc[1] && acc[2];
    if (!all_acc && (acc[0] || acc[1] || acc[2]))  // one launch writes all three: accumulate into zeroed ones
      for (int i = 0; i < 3; ++i)
        if (!acc[i]) TX_CUDA(ctx, cudaMemsetAsync(t[i], 0, numel_of(q) * 4, ctx->stream));
    const bool any_acc = acc[0] || acc[1] || acc[2];
    const bool rnd = ctx->math == TX_MATH_TF32 && !any_acc && g->values[a.q].grad_round &&
                     g->values[a.k].grad_round && g->values[a.v].grad_round;
    const int flags = ((r->tf32[a.q] && r->tf32[a.k] && r->tf32[a.v] && grad_tf32[a.out]) ? 1 : 0) |
                      (any_acc ? 2 : 0) | (rnd ? 4 : 0);
    TX_TRY(tx_attention_bwd(ctx, F(a.q), F(a.k), F(a.v), E, dout, E, t[0], t[1], t[2], E, B, Sq, E / 64, 64,
                            a.scale, flags));
    for (int i = 0; i < 3; ++i) {
      grad_tf32[vs[i]] = rnd;
      wrote(vs[i]);
    }
    return TX_OK;
  }

  int node(int ni) {
    GNode &n = g->nodes[ni];
    const tx_node_desc &d = n.d;
    if (n.attn >= 0 && r->attn_fused[n.attn]) {
      const AttnPlan &a = g->attn[n.attn];
      return ni == a.last ? attn_backward(a) : TX_OK;
    }
    if (n.scaled_into >= 0) return TX_OK;  // scale folded into the producing contraction's alpha
    if (n.fused_into >= 0) {
      // activation folded into the producing GEMM: hand the gradient over
      int src = d.out[0];
      GNode &p = g->nodes[n.fused_into];
      (void)p;
      (void)src;
      return TX_OK;
    }
    bool any = false;
    for (int k = 0; k < d.n_in; ++k)
      if (d.in[k] >= 0 && needs[d.in[k]]) any = true;
    if (!any) return TX_OK;
    switch (d.op) {
      case TX_OP_GEMM: case TX_OP_MATMUL: return gemm_backward(ni);
      case TX_OP_CONV: return conv_backward(ni);
      default: break;
    }
    if (d.op == TX_OP_SPLIT) return split_backward(ni);
    int yv = d.out[0];
    float *dy = grad[yv];
    if (!dy) return TX_OK;
    const Shape &y = S(yv);
    int64_t ny = numel_of(y);
    int xv = d.in[0];
    if (is_alias_op(d.op)) {
      if (!needs[xv]) return TX_OK;
      GValue &gx = g->values[xv];
      if (gx.kind != TX_VAL_PARAM && !grad[xv] && grad_owned[yv]) {  // hand the buffer over
        grad[xv] = dy;
        grad_owned[xv] = true;
        grad_owned[yv] = false;
        grad_preact[xv] = grad_preact[yv];
        grad_tf32[xv] = grad_tf32[yv] && gx.grad_round;  // nothing else will add to it
        wrote(xv);
        return TX_OK;
      }
      float *t; int acc;
      TX_TRY(target(xv, &t, &acc));
      if (acc) {
        k_axpy<<<grid_for(ny, 256), 256, 0, ctx->stream>>>(t, dy, ny, 1.f);
        TX_LAUNCHED(ctx, "k_axpy");
      } else {
        TX_TRY(tx_d2d(ctx, t, dy, ny * 4));
      }
      grad_tf32[xv] = !acc && grad_tf32[yv] && gx.grad_round;
      wrote(xv);
      return TX_OK;
    }
    switch (d.op) {
      case TX_OP_GATHER: {
        if (!needs[xv]) return TX_OK;
        const Shape &x = S(xv);
        int ax = norm_axis(d.iattr[0], (int64_t)x.size());
        int64_t outer = 1, inner = 1;
        for (int i = 0; i < ax; ++i) outer *= x[i];
        for (size_t i = ax + 1; i < x.size(); ++i) inner *= x[i];
        int64_t nidx = numel_of(S(d.in[1]));
        float *t; int acc;
        TX_TRY(target(xv, &t, &acc));
        if (!acc) TX_CUDA(ctx, cudaMemsetAsync(t, 0, numel_of(x) * 4, ctx->stream));
        if (ax == 0) {
          TX_TRY(tx_scatter_add_rows(ctx, t, x[0], inner, (const int64_t *)r->buf[d.in[1]], nidx, dy));
        } else {
          k_gather_axis_bwd<<<grid_for(ny, 256), 256, 0, ctx->stream>>>(t, (const int64_t *)r->buf[d.in[1]], dy,
                                                                       outer, x[ax], inner, nidx);
          TX_LAUNCHED(ctx, "k_gather_axis_bwd");
        }
        wrote(xv);
        return TX_OK;
      }
      case TX_OP_LAYERNORM: {
        const Shape &x = S(xv);
        int ax = norm_axis(d.iattr[0], (int64_t)x.size());
        int64_t rows = 1;
        for (int i = 0; i < ax; ++i) rows *= x[i];
        int64_t cols = numel_of(x) / (rows ? rows : 1);
        const float *mean = d.n_out > 1 ? F(d.out[1]) : (const float *)r->extra[ni];
        const float *rstd = d.n_out > 2 ? F(d.out[2]) : (const float *)r->extra2[ni][0];
        float *dx = nullptr, *dg = nullptr, *db = nullptr;
        int ax_acc = 0, p_acc = 0;
        if (needs[xv]) TX_TRY(target(xv, &dx, &ax_acc));
        int gv = d.in[1], bv = (d.n_in > 2 ? d.in[2] : -1);
        int gacc = 0, bacc = 0;
        if (needs[gv]) TX_TRY(target(gv, &dg, &gacc));
        if (bv >= 0 && needs[bv]) TX_TRY(target(bv, &db, &bacc));
        // the kernel takes one accumulate flag for both parameter gradients
        float *dg_tmp = nullptr, *db_tmp = nullptr;
        p_acc = gacc;
        if (db && bacc != gacc) {
          db_tmp = (float *)tx_alloc_raw(ctx, cols * 4);
          TX_CUDA(ctx, cudaMemsetAsync(db_tmp, 0, cols * 4, ctx->stream));
          if (bacc) TX_CUDA(ctx, cudaMemcpyAsync(db_tmp, db, cols * 4, cudaMemcpyDeviceToDevice, ctx->stream));
        }
        TX_TRY(tx_layernorm_bwd(ctx, F(xv), F(gv), mean, rstd, dy, dx, dg, db_tmp ? db_tmp : db, rows, cols,
                                ax_acc, p_acc));
        if (db_tmp) {
          TX_CUDA(ctx, cudaMemcpyAsync(db, db_tmp, cols * 4, cudaMemcpyDeviceToDevice, ctx->stream));
          tx_free_raw(ctx, db_tmp);
        }
        (void)dg_tmp;
        if (dx) wrote(xv);
        if (dg) wrote(gv);
        if (db) wrote(bv);
        return TX_OK;
      }
      case TX_OP_PRELU: {
        const int xv0 = d.in[0], sv = d.in[1];
        float *dx = nullptr, *tmp = nullptr;
        int xacc = 0;
        if (needs[xv0]) TX_TRY(target(xv0, &dx, &xacc));
        if (needs[sv]) {
          tmp = (float *)tx_alloc_raw(ctx, ny * 4 + 4);
          if (!tmp) return TX_ERR_OOM;
        }
        int64_t ss[TX_MAX_DIMS];
        bstrides(S(sv), y, ss);
        int rc = tx_prelu_bwd(ctx, F(xv0), F(sv), ss, dy, dx, tmp, y.data(), (int)y.size(), xacc);
        if (rc == TX_OK && dx) wrote(xv0);
        if (rc == TX_OK && tmp) rc = reduce_into(sv, tmp, y, 1.f);
        tx_free_raw(ctx, tmp);
        return rc;
      }
      case TX_OP_BATCHNORM: case TX_OP_GROUPNORM: {
        const int xv0 = d.in[0], sv = d.in[1], bv = d.in[2];
        int64_t N, C, L;
        ncl(S(xv0), &N, &C, &L);
        float *dx = nullptr;
        int xacc = 0;
        if (needs[xv0]) TX_TRY(target(xv0, &dx, &xacc));
        // the affine gradients: both or neither (a missing one goes to scratch)
        const bool want = needs[sv] || needs[bv];
        float *ds = nullptr, *db = nullptr;
        int sacc = 0, bacc = 0;
        Scratch spare(ctx, want ? (size_t)C * 4 : 0);
        if (want) {
          if (needs[sv]) TX_TRY(target(sv, &ds, &sacc)); else ds = spare.as<float>();
          if (needs[bv]) TX_TRY(target(bv, &db, &bacc)); else db = spare.as<float>();
        }
        // one accumulate flag covers both affine outputs: accumulate into scratch when they differ
        Scratch tmp2(ctx, want && sacc != bacc ? (size_t)C * 8 : 0);
        float *ds_w = ds, *db_w = db;
        const int pacc = want && sacc == bacc ? sacc : 0;
        if (want && sacc != bacc) {
          ds_w = tmp2.as<float>();
          db_w = tmp2.as<float>() + C;
        }
        if (d.op == TX_OP_BATCHNORM) {
          TX_TRY(tx_batchnorm_bwd(ctx, F(xv0), dy, F(sv), F(d.in[3]), F(d.in[4]), dx, ds_w, db_w, N, C, L,
                                  (float)d.fattr[0], xacc, pacc));
        } else {
          const int64_t groups = d.iattr[0] > 0 ? d.iattr[0] : C;
          TX_TRY(tx_groupnorm_bwd(ctx, F(xv0), dy, F(sv), (const float *)r->extra[ni], (const float *)r->extra2[ni][0],
                                  dx, ds_w, db_w, N, C, L, groups, xacc, pacc));
        }
        if (want && sacc != bacc) {
          if (needs[sv]) TX_TRY(add_or_copy(ds, ds_w, C, sacc));
          if (needs[bv]) TX_TRY(add_or_copy(db, db_w, C, bacc));
        }
        if (dx) wrote(xv0);
        if (needs[sv]) wrote(sv);
        if (needs[bv]) wrote(bv);
        return TX_OK;
      }
      case TX_OP_UNARY: {
        if (!needs[xv]) return TX_OK;
        float *t; int acc;
        TX_TRY(target(xv, &t, &acc));
        TX_TRY(tx_unary_bwd(ctx, (int)d.iattr[0], F(xv), dy, t, ny, (float)d.fattr[0], (float)d.fattr[1], acc));
        wrote(xv);
        return TX_OK;
      }
      case TX_OP_BINARY: {
        int64_t sa[TX_MAX_DIMS], sb[TX_MAX_DIMS];
        bstrides(S(d.in[0]), y, sa);
        bstrides(S(d.in[1]), y, sb);
        for (int k = 0; k < 2; ++k) {
          if (!needs[d.in[k]]) continue;
          float *tmp = (float *)tx_alloc_raw(ctx, ny * 4 + 4);
          if (!tmp) return TX_ERR_OOM;
          int rc = nd_binary_grad(ctx, (int)d.iattr[0], k, F(d.in[0]), sa, F(d.in[1]), sb, dy, tmp, y.data(),
                                  (int)y.size());
          if (rc == TX_OK) rc = reduce_into(d.in[k], tmp, y, 1.f);
          tx_free_raw(ctx, tmp);
          TX_TRY(rc);
        }
        return TX_OK;
      }
      case TX_OP_CONCAT: {
        const int ax = norm_axis(d.iattr[0], (int64_t)y.size());
        int64_t ys[TX_MAX_DIMS];
        cstrides(y, ys);
        int64_t at = 0;
        for (int k = 0; k < d.n_in; ++k) {
          const Shape &xk = S(d.in[k]);
          if (needs[d.in[k]]) {
            float *t; int acc;
            TX_TRY(target(d.in[k], &t, &acc));
            TX_TRY(nd_copy(ctx, dy + at * ys[ax], ys, t, xk.data(), (int)xk.size(), 4, 1.f, acc));
            wrote(d.in[k]);
          }
          at += xk[ax];
        }
        return TX_OK;
      }
      case TX_OP_SLICE: {
        if (!needs[xv]) return TX_OK;
        const Shape &x = S(xv);
        int64_t first[TX_MAX_DIMS], step[TX_MAX_DIMS], xs[TX_MAX_DIMS], ss[TX_MAX_DIMS];
        Shape o;
        slice_params(d, x, first, step, o);
        cstrides(x, xs);
        int64_t base = 0;
        for (size_t i = 0; i < x.size(); ++i) {
          base += first[i] * xs[i];
          ss[i] = step[i] * xs[i];
        }
        float *t; int acc;
        TX_TRY(target(xv, &t, &acc));
        if (!acc) TX_CUDA(ctx, cudaMemsetAsync(t, 0, numel_of(x) * 4, ctx->stream));
        TX_TRY(nd_scatter(ctx, dy, t + base, ss, y.data(), (int)y.size(), 1));
        wrote(xv);
        return TX_OK;
      }
      case TX_OP_EXPAND:
        return needs[xv] ? reduce_into(xv, dy, y, 1.f) : TX_OK;
      case TX_OP_REDUCEMAX: case TX_OP_REDUCEMIN: {
        if (!needs[xv]) return TX_OK;
        int64_t o, rd, inn;
        maxmin_block(d, S(xv), &o, &rd, &inn);
        float *t; int acc;
        TX_TRY(target(xv, &t, &acc));
        TX_TRY(reduce_maxmin_bwd(ctx, dy, (const int32_t *)r->extra[ni], t, o, rd, inn, acc));
        wrote(xv);
        return TX_OK;
      }
      case TX_OP_AVGPOOL: {
        if (!needs[xv]) return TX_OK;
        const Shape &x = S(xv);
        const int64_t H = x.size() == 4 ? x[2] : 1, W = x.back();
        int64_t geom[12];
        if (!pool_geom(d, H, W, geom)) return fail(g, TX_ERR_SHAPE, "AveragePool window larger than its padded input");
        float *t; int acc;
        TX_TRY(target(xv, &t, &acc));
        TX_TRY(tx_avgpool2d_bwd(ctx, dy, t, x[0] * x[1], H, W, geom, (int)d.iattr[2], acc));
        wrote(xv);
        return TX_OK;
      }
      case TX_OP_MAXPOOL: {
        if (!needs[xv]) return TX_OK;
        const Shape &x = S(xv);
        const int64_t H = x.size() == 4 ? x[2] : 1, W = x.back();
        int64_t geom[12];
        if (!pool_geom(d, H, W, geom)) return fail(g, TX_ERR_SHAPE, "MaxPool window larger than its padded input");
        float *t; int acc;
        TX_TRY(target(xv, &t, &acc));
        TX_TRY(tx_maxpool2d_bwd(ctx, dy, (const int32_t *)r->extra[ni], t, x[0] * x[1], H, W, geom, acc));
        wrote(xv);
        return TX_OK;
      }
      case TX_OP_ADD: case TX_OP_SUB: {
        if (needs[d.in[0]]) TX_TRY(reduce_into(d.in[0], dy, y, 1.f));
        if (needs[d.in[1]]) {
          if (d.op == TX_OP_ADD) {
            TX_TRY(reduce_into(d.in[1], dy, y, 1.f));
          } else {
            float *neg = (float *)tx_alloc_raw(ctx, ny * 4);
            TX_TRY(tx_unary(ctx, TX_UN_NEG, dy, neg, ny, 0.f, 0.f));
            int rc = reduce_into(d.in[1], neg, y, 1.f);
            tx_free_raw(ctx, neg);
            TX_TRY(rc);
          }
        }
        return TX_OK;
      }
      case TX_OP_MUL: case TX_OP_DIV: {
        int64_t sa[TX_MAX_DIMS], sb[TX_MAX_DIMS], sy[TX_MAX_DIMS];
        const Shape &A = S(d.in[0]), &B = S(d.in[1]);
        bstrides(A, y, sa);
        bstrides(B, y, sb);
        bstrides(y, y, sy);
        float *tmp = (float *)tx_alloc_raw(ctx, ny * 4);
        if (!tmp) return TX_ERR_OOM;
        int rc = TX_OK;
        if (needs[d.in[0]]) {  // dA = dy * B  (or dy / B)
          rc = tx_binary(ctx, d.op == TX_OP_MUL ? TX_BIN_MUL : TX_BIN_DIV, dy, sy, F(d.in[1]), sb, tmp, y.data(), (int)y.size());
          if (rc == TX_OK) rc = reduce_into(d.in[0], tmp, y, 1.f);
        }
        if (rc == TX_OK && needs[d.in[1]]) {
          if (d.op == TX_OP_MUL) {  // dB = dy * A
            rc = tx_binary(ctx, TX_BIN_MUL, dy, sy, F(d.in[0]), sa, tmp, y.data(), (int)y.size());
          } else {  // dB = -dy * y / B
            rc = tx_binary(ctx, TX_BIN_MUL, dy, sy, F(yv), sy, tmp, y.data(), (int)y.size());
            if (rc == TX_OK) rc = tx_binary(ctx, TX_BIN_DIV, tmp, sy, F(d.in[1]), sb, tmp, y.data(), (int)y.size());
            if (rc == TX_OK) rc = tx_unary(ctx, TX_UN_NEG, tmp, tmp, ny, 0.f, 0.f);
          }
          if (rc == TX_OK) rc = reduce_into(d.in[1], tmp, y, 1.f);
        }
        tx_free_raw(ctx, tmp);
        return rc;
      }
      case TX_OP_RELU: case TX_OP_TANH: case TX_OP_GELU: case TX_OP_SIGMOID: case TX_OP_EXP:
      case TX_OP_LOG: case TX_OP_NEG: case TX_OP_CLIP: {
        if (!needs[xv]) return TX_OK;
        float *t; int acc;
        TX_TRY(target(xv, &t, &acc));
        const float *src = unary_uses_output(d.op) ? F(yv) : F(xv);
        float lo = 0.f, hi = 0.f;
        if (d.op == TX_OP_CLIP) {
          lo = d.iattr[0] ? (float)d.fattr[0] : -INFINITY;
          hi = d.iattr[1] ? (float)d.fattr[1] : INFINITY;
        }
        TX_TRY(tx_unary_bwd(ctx, unary_code(d.op), src, dy, t, ny, lo, hi, acc));
        wrote(xv);
        return TX_OK;
      }
      case TX_OP_SOFTMAX: case TX_OP_LOGSOFTMAX: {
        if (!needs[xv]) return TX_OK;
        float *t; int acc;
        TX_TRY(target(xv, &t, &acc));
        int64_t cols = y.back();
        // In TF32 mode the gradient of attention scores is read only by the
        // scores' own contraction (dgrad and wgrad operands, which round it):
        // store it rounded so that they run without operand conversion.
        bool rnd = false;
        const GValue &xg = g->values[xv];
        if (ctx->math == TX_MATH_TF32 && !acc && d.op == TX_OP_SOFTMAX && xg.kind == TX_VAL_ACT &&
            !xg.is_output && xg.consumers.size() == 1 && xg.producer >= 0) {
          const GNode &p = g->nodes[xg.producer];
          const GNode *c = nullptr;
          if (p.scaled_into >= 0) c = &g->nodes[p.scaled_into];
          else if ((p.d.op == TX_OP_GEMM || p.d.op == TX_OP_MATMUL) && !p.fused_act) c = &p;
          rnd = c && (c->d.op == TX_OP_GEMM || c->d.op == TX_OP_MATMUL) && !c->fused_act;
        }
        TX_TRY(softmax_bwd(ctx, F(yv), dy, t, ny / cols, cols, d.op == TX_OP_LOGSOFTMAX, acc, rnd));
        wrote(xv);
        grad_tf32[xv] = rnd;
        return TX_OK;
      }
      case TX_OP_REDUCEMEAN: case TX_OP_REDUCESUM: case TX_OP_GAP: {
        if (!needs[xv]) return TX_OK;
        const Shape &x = S(xv);
        Shape keep = x;
        if (d.op == TX_OP_GAP) {
          for (size_t i = 2; i < keep.size(); ++i) keep[i] = 1;
        } else if (d.n_ints == 0) {
          for (auto &k : keep) k = 1;
        } else {
          for (int i = 0; i < d.n_ints; ++i) keep[norm_axis(d.ints[i], (int64_t)x.size())] = 1;
        }
        int64_t nred = numel_of(x) / numel_of(keep);
        float scale = d.op == TX_OP_REDUCESUM ? 1.f : 1.f / (float)nred;
        BDims bd;
        int64_t st[TX_MAX_DIMS];
        bstrides(keep, x, st);
        for (size_t i = 0; i < x.size(); ++i) { bd.shape[i] = x[i]; bd.s[i] = st[i]; }
        float *t; int acc;
        TX_TRY(target(xv, &t, &acc));
        TX_TRY(nd_copy(ctx, dy, bd.s, t, x.data(), (int)x.size(), 4, scale, acc));
        wrote(xv);
        return TX_OK;
      }
      case TX_OP_TRANSPOSE: {
        if (!needs[xv]) return TX_OK;
        const Shape &x = S(xv);
        int nd = (int)x.size();
        // dX[perm^-1] : element of dx at index i corresponds to dy at permuted index
        int64_t ys[TX_MAX_DIMS], ss[TX_MAX_DIMS];
        int64_t st = 1;
        for (int i = nd - 1; i >= 0; --i) { ys[i] = st; st *= y[i]; }
        for (int i = 0; i < nd; ++i) {
          int p = (int)(d.n_ints ? d.ints[i] : nd - 1 - i);  // y axis i = x axis p
          ss[p] = ys[i];
        }
        float *t; int acc;
        TX_TRY(target(xv, &t, &acc));
        // a transpose moves values unchanged; the flag passes on where nothing else adds to dX
        grad_tf32[xv] = !acc && grad_tf32[yv] && g->values[xv].grad_round;
        if (!acc) {
          TX_TRY(tx_strided_copy(ctx, dy, ss, t, x.data(), nd, 4));
        } else {
          float *tmp = (float *)tx_alloc_raw(ctx, ny * 4);
          TX_TRY(tx_strided_copy(ctx, dy, ss, tmp, x.data(), nd, 4));
          k_axpy<<<grid_for(ny, 256), 256, 0, ctx->stream>>>(t, tmp, ny, 1.f);
          tx_free_raw(ctx, tmp);
        }
        wrote(xv);
        return TX_OK;
      }
    }
    return fail(g, TX_ERR_UNSUPPORTED, "operator " + std::to_string(d.op) + " has no CUDA backward");
  }
};

}  // namespace

extern "C" int tx_graph_backward(tx_graph *g, tx_record *r, const float *const *d_outputs,
                                 float *const *d_inputs) {
  if (!g || !r || r->g != g) return TX_ERR_INVALID;
  tx_ctx *ctx = g->ctx;
  size_t nv = g->values.size();
  Bwd b{g, ctx, r};
  b.grad.assign(nv, nullptr);
  b.grad_owned.assign(nv, false);
  b.grad_preact.assign(nv, false);
  b.grad_tf32.assign(nv, false);
  b.bias_fused.assign(g->nodes.size(), false);
  b.needs.assign(nv, false);
  b.param_done.assign(g->params.size(), false);
  b.param_pending.assign(g->params.size(), 0);
  // which values need gradients: parameters, requested inputs, and anything downstream
  for (size_t i = 0; i < nv; ++i)
    if (g->values[i].kind == TX_VAL_PARAM) b.needs[i] = true;
  for (size_t i = 0; i < g->inputs.size(); ++i)
    if (d_inputs && d_inputs[i]) b.needs[g->inputs[i]] = true;
  for (const GNode &n : g->nodes) {
    bool any = false;
    for (int k = 0; k < n.d.n_in; ++k)
      if (n.d.in[k] >= 0 && b.needs[n.d.in[k]]) any = true;
    if (any && n.d.op != TX_OP_GATHER)
      for (int k = 0; k < n.d.n_out; ++k) b.needs[n.d.out[k]] = true;
    if (n.d.op == TX_OP_GATHER && b.needs[n.d.in[0]]) b.needs[n.d.out[0]] = true;
  }
  // contributions per parameter (for DP bucket readiness)
  for (const GNode &n : g->nodes)
    for (int k = 0; k < n.d.n_in; ++k) {
      int v = n.d.in[k];
      if (v >= 0 && g->values[v].kind == TX_VAL_PARAM) b.param_pending[g->values[v].param_index]++;
    }
  if (g->dp) {
    for (size_t p = 0; p < g->params.size(); ++p)
      if (b.param_pending[p] == 0) b.param_pending[p] = 1;  // unused params still reduce
  }
  // seed output gradients
  for (size_t i = 0; i < g->outputs.size(); ++i) {
    int v = g->outputs[i];
    if (!d_outputs[i]) continue;
    int64_t nel = numel_of(r->shapes[v]);
    if (b.grad[v]) {  // output listed twice
      k_axpy<<<grid_for(nel, 256), 256, 0, ctx->stream>>>(b.grad[v], d_outputs[i], nel, 1.f);
      TX_LAUNCHED(ctx, "k_axpy");
    } else {
      // own copy: later accumulation must never write into the caller's tensor
      b.grad[v] = (float *)tx_alloc_raw(ctx, nel * 4 + 4);
      if (!b.grad[v]) return TX_ERR_OOM;
      b.grad_owned[v] = true;
      TX_TRY(tx_d2d(ctx, b.grad[v], d_outputs[i], nel * 4));
    }
  }
  // the value an absorbed activation produces is the one the GEMM backward reads
  int rc = TX_OK;
  for (int i = (int)g->nodes.size() - 1; i >= 0 && rc == TX_OK; --i) rc = b.node(i);
  if (rc == TX_OK && g->dp) {
    // parameters no node touched still take part in the reduction
    for (size_t p = 0; p < g->params.size(); ++p)
      if (!b.param_done[p]) {
        b.param_pending[p] = 1;
        GValue &gv = g->values[g->params[p]];
        if (!gv.grad_defined) {
          cudaMemsetAsync(gv.grad, 0, numel_of(gv.shape) * 4, ctx->stream);
          gv.grad_defined = true;
        }
        b.param_contribution_done((int)p);
      }
    rc = b.flush(g->flat_len);
    if (rc == TX_OK) rc = dp_event_join(ctx);
  }
  if (rc == TX_OK && d_inputs) {
    for (size_t i = 0; i < g->inputs.size(); ++i) {
      if (!d_inputs[i]) continue;
      int v = g->inputs[i];
      size_t bytes = numel_of(r->shapes[v]) * 4;
      if (b.grad[v]) rc = tx_d2d(ctx, d_inputs[i], b.grad[v], bytes);
      else rc = tx_memset(ctx, d_inputs[i], 0, bytes);
      if (rc) break;
    }
  }
  for (size_t i = 0; i < nv; ++i)
    if (b.grad_owned[i]) tx_free_raw(ctx, b.grad[i]);
  return rc;
}
