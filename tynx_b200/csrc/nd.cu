// N-dimensional bandwidth kernels on canonical shapes: broadcast binary ops,
// strided copies (transposes, head split/merge), broadcast-scale (the backward
// of a mean), and reductions to a broadcastable shape (ReduceMean / pooling /
// the gradient of a broadcast).
//
// Shapes are canonicalised on the host first: size-1 axes are dropped and
// adjacent axes that are contiguous with each other in every operand are
// merged, so that [256,128,4,64] -> [256,4,128,64] is a 3-axis copy with a
// 64-element contiguous inner run, a residual add is one axis, and a bias add
// is [rows, cols] with a zero row stride.  Kernels then decompose indices with
// 32-bit arithmetic when the element count allows and move float4 along the
// innermost axis when every operand is contiguous (or broadcast) there.
// Semantics follow the broadcast arithmetic of DynTensor (crates/tynx/src/
// tensor.rs:1637-1700), Transpose/Reshape (interpreter/shape.rs:118,152) and
// mean_dims / sum_dims (tensor.rs:1789-1825).
#include "common.h"

namespace {

constexpr int kNd = TX_MAX_DIMS;

struct Nd {
  int nd;
  int64_t shape[kNd];   // outermost first
  int64_t st[3][kNd];   // element strides of up to three operands
  // ceil(2^64 / shape[k]) (0 for an extent of 1): for a 32-bit index x,
  // x / shape[k] = mulhi64(x, rcp[k]) exactly (the error of the product is
  // below 2^-32 < 1 / shape[k]), a few instructions instead of a division
  uint64_t rcp[kNd];
};

// Drop size-1 axes and merge adjacent axes that are contiguous in every operand.
void canonicalize(int nd, const int64_t *shape, const int64_t *const *strides, int nops, Nd &c) {
  int64_t sh[kNd], s[3][kNd];
  int m = 0;
  for (int k = nd - 1; k >= 0; --k) {  // innermost first
    if (shape[k] == 1) continue;
    if (m > 0) {
      bool merge = true;
      for (int o = 0; o < nops; ++o)
        if (strides[o][k] != s[o][m - 1] * sh[m - 1]) merge = false;
      if (merge) {
        sh[m - 1] *= shape[k];
        continue;
      }
    }
    sh[m] = shape[k];
    for (int o = 0; o < nops; ++o) s[o][m] = strides[o][k];
    ++m;
  }
  if (m == 0) {  // a single element
    sh[0] = 1;
    for (int o = 0; o < nops; ++o) s[o][0] = 0;
    m = 1;
  }
  c.nd = m;
  for (int i = 0; i < m; ++i) {
    c.shape[i] = sh[m - 1 - i];
    for (int o = 0; o < nops; ++o) c.st[o][i] = s[o][m - 1 - i];
    c.rcp[i] = c.shape[i] >= 2 ? ~uint64_t(0) / (uint64_t)c.shape[i] + 1 : 0;
  }
}

// float4 along the innermost axis: its extent is a multiple of 4, every
// operand is contiguous (stride 1) or broadcast (stride 0) there, all outer
// strides are multiples of 4 and every base pointer is 16-byte aligned.
bool vectorizable(const Nd &c, int nops, const void *const *ptrs) {
  if (c.shape[c.nd - 1] % 4) return false;
  for (int o = 0; o < nops; ++o) {
    if (((uintptr_t)ptrs[o]) & 15) return false;
    const int64_t inner = c.st[o][c.nd - 1];
    if (inner != 0 && inner != 1) return false;
    for (int k = 0; k < c.nd - 1; ++k)
      if (c.st[o][k] % 4) return false;
  }
  return true;
}

__device__ __forceinline__ float bin_f(int op, float a, float b) {
  switch (op) {
    case TX_BIN_ADD: return a + b;
    case TX_BIN_SUB: return a - b;
    case TX_BIN_MUL: return a * b;
    case TX_BIN_DIV: return a / b;
    case TX_BIN_MIN: return a <= b ? a : b;
    case TX_BIN_MAX: return a >= b ? a : b;
    case TX_BIN_LE: return a <= b ? 1.f : 0.f;
    case TX_BIN_GE: return a >= b ? 1.f : 0.f;
    case TX_BIN_POW: return powf(a, b);
  }
  return 0.f;
}

// Offsets of element `i` (row-major over c.shape) in the first NOPS operands.
template <typename I, int NOPS>
__device__ __forceinline__ void offsets(const Nd &c, I i, int64_t (&off)[NOPS]) {
#pragma unroll
  for (int o = 0; o < NOPS; ++o) off[o] = 0;
  for (int k = c.nd - 1; k >= 0; --k) {
    const I ext = (I)c.shape[k];
    I q;
    if constexpr (sizeof(I) == 4)
      q = c.rcp[k] ? (I)__umul64hi((uint64_t)i, c.rcp[k]) : i;
    else
      q = i / ext;
    const I r = i - q * ext;
    i = q;
#pragma unroll
    for (int o = 0; o < NOPS; ++o) off[o] += (int64_t)r * c.st[o][k];
  }
}

__device__ __forceinline__ float4 ld_or_splat(const float *p, int64_t inner_stride) {
  if (inner_stride) return *reinterpret_cast<const float4 *>(p);
  const float v = *p;
  return make_float4(v, v, v, v);
}

// out (contiguous) = A op B; operands 0 = A, 1 = B.
template <typename I, bool VEC>
__global__ void k_binary_nd(int op, const float *__restrict__ A, const float *__restrict__ B,
                            float *__restrict__ out, Nd c, I n) {
  const I stride = (I)gridDim.x * blockDim.x;
  if (VEC) {
    const int64_t ia = c.st[0][c.nd - 1], ib = c.st[1][c.nd - 1];
    for (I j = blockIdx.x * (I)blockDim.x + threadIdx.x; j < n / 4; j += stride) {
      int64_t off[2];
      offsets<I, 2>(c, j * 4, off);
      const float4 a = ld_or_splat(A + off[0], ia);
      const float4 b = ld_or_splat(B + off[1], ib);
      reinterpret_cast<float4 *>(out)[j] =
          make_float4(bin_f(op, a.x, b.x), bin_f(op, a.y, b.y), bin_f(op, a.z, b.z), bin_f(op, a.w, b.w));
    }
  } else {
    for (I i = blockIdx.x * (I)blockDim.x + threadIdx.x; i < n; i += stride) {
      int64_t off[2];
      offsets<I, 2>(c, i, off);
      out[i] = bin_f(op, A[off[0]], B[off[1]]);
    }
  }
}

// out (contiguous) (+)= scale * src[strided]; with scale == 1 and !acc a copy.
template <typename T, typename I, bool VEC>
__global__ void k_copy_nd(const T *__restrict__ src, T *__restrict__ out, Nd c, I n, float scale, int acc) {
  const I stride = (I)gridDim.x * blockDim.x;
  if (VEC) {
    const int64_t is = c.st[0][c.nd - 1];
    for (I j = blockIdx.x * (I)blockDim.x + threadIdx.x; j < n / 4; j += stride) {
      int64_t off[1];
      offsets<I, 1>(c, j * 4, off);
      float4 v = ld_or_splat((const float *)src + off[0], is);
      if (scale != 1.f) {
        v.x *= scale;
        v.y *= scale;
        v.z *= scale;
        v.w *= scale;
      }
      float4 *o = reinterpret_cast<float4 *>(out) + j;
      if (acc) {
        const float4 p = *o;
        v.x += p.x;
        v.y += p.y;
        v.z += p.z;
        v.w += p.w;
      }
      *o = v;
    }
  } else {
    for (I i = blockIdx.x * (I)blockDim.x + threadIdx.x; i < n; i += stride) {
      int64_t off[1];
      offsets<I, 1>(c, i, off);
      if constexpr (sizeof(T) == 4) {
        float v = (float)src[off[0]] * scale;
        out[i] = acc ? out[i] + v : v;
      } else {
        out[i] = src[off[0]];
      }
    }
  }
}

// Reduction of the middle axis of a contiguous [outer, red, inner] tensor.
// Block (32, 8) over (columns, row groups); VEC: 4 columns per thread.  Each
// thread sums rows r0 + ty, r0 + ty + 8, ... of its split in order (four loads
// in flight) and the 8 groups are combined in a fixed order.  With one split
// the result (scaled, optionally accumulated) goes straight to y; otherwise
// raw partials go to part[outer][splits][inner].
template <bool VEC>
__global__ void k_reduce_mid(const float *__restrict__ x, int64_t red, int64_t inner, int64_t rows_per,
                             int splits, float *__restrict__ part, float *__restrict__ y, float scale,
                             int acc) {
  constexpr int W = VEC ? 4 : 1;
  __shared__ float sm[8][32 * W];
  const int64_t o = blockIdx.z;
  const int64_t c = ((int64_t)blockIdx.x * 32 + threadIdx.x) * W;
  const int64_t r0 = (int64_t)blockIdx.y * rows_per;
  const int64_t r1 = r0 + rows_per < red ? r0 + rows_per : red;
  const float *xo = x + o * red * inner;
  float s[W];
#pragma unroll
  for (int j = 0; j < W; ++j) s[j] = 0.f;
  if (c < inner) {
    int64_t r = r0 + threadIdx.y;
    for (; r + 24 < r1; r += 32) {
      float v[4][W];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float *p = xo + (r + 8 * i) * inner + c;
        if (VEC) {
          const float4 t = *reinterpret_cast<const float4 *>(p);
          v[i][0] = t.x;
          v[i][W > 1 ? 1 : 0] = t.y;
          v[i][W > 2 ? 2 : 0] = t.z;
          v[i][W > 3 ? 3 : 0] = t.w;
        } else {
          v[i][0] = *p;
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < W; ++j) s[j] += v[i][j];
    }
    for (; r < r1; r += 8)
#pragma unroll
      for (int j = 0; j < W; ++j) s[j] += xo[r * inner + c + j];
  }
#pragma unroll
  for (int j = 0; j < W; ++j) sm[threadIdx.y][threadIdx.x * W + j] = s[j];
  __syncthreads();
  if (threadIdx.y == 0 && c < inner) {
#pragma unroll
    for (int j = 0; j < W; ++j) {
      float t = sm[0][threadIdx.x * W + j];
#pragma unroll
      for (int i = 1; i < 8; ++i) t += sm[i][threadIdx.x * W + j];
      if (splits == 1) {
        t *= scale;
        float *yo = y + o * inner + c + j;
        *yo = acc ? *yo + t : t;
      } else {
        part[(o * splits + blockIdx.y) * inner + c + j] = t;
      }
    }
  }
}

// Sum of the split partials of k_reduce_mid, in split order.
__global__ void k_reduce_mid_final(const float *__restrict__ part, int64_t outer, int splits,
                                   int64_t inner, float *__restrict__ y, float scale, int acc) {
  const int64_t n = outer * inner;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = i / inner, c = i - o * inner;
    const float *p = part + o * splits * inner + c;
    float t = 0.f;
    int s = 0;
    for (; s + 4 <= splits; s += 4) {
      const float v0 = p[(int64_t)s * inner], v1 = p[(int64_t)(s + 1) * inner];
      const float v2 = p[(int64_t)(s + 2) * inner], v3 = p[(int64_t)(s + 3) * inner];
      t += v0;
      t += v1;
      t += v2;
      t += v3;
    }
    for (; s < splits; ++s) t += p[(int64_t)s * inner];
    t *= scale;
    y[i] = acc ? y[i] + t : t;
  }
}

// Reduction of the innermost axis of a contiguous [outer, red]: a warp per row
// (fixed butterfly order).
__global__ void k_reduce_rows(const float *__restrict__ x, int64_t outer, int64_t red,
                              float *__restrict__ y, float scale, int acc) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t o = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); o < outer; o += warps) {
    const float *row = x + o * red;
    float s = 0.f;
    for (int64_t r = lane; r < red; r += 32) s += row[r];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) {
      s *= scale;
      y[o] = acc ? y[o] + s : s;
    }
  }
}

template <typename T>
int launch_copy(tx_ctx *ctx, const T *src, T *out, const Nd &c, int64_t n, float scale, int acc, bool vec) {
  const bool small = n < (int64_t(1) << 31);
  const int64_t units = vec ? n / 4 : n;
  const unsigned blocks = grid_for(units, 256);
  if (vec) {
    if (small) k_copy_nd<T, uint32_t, true><<<blocks, 256, 0, ctx->stream>>>(src, out, c, (uint32_t)n, scale, acc);
    else k_copy_nd<T, uint64_t, true><<<blocks, 256, 0, ctx->stream>>>(src, out, c, (uint64_t)n, scale, acc);
  } else {
    if (small) k_copy_nd<T, uint32_t, false><<<blocks, 256, 0, ctx->stream>>>(src, out, c, (uint32_t)n, scale, acc);
    else k_copy_nd<T, uint64_t, false><<<blocks, 256, 0, ctx->stream>>>(src, out, c, (uint64_t)n, scale, acc);
  }
  TX_LAUNCHED(ctx, "k_copy_nd");
  return TX_OK;
}

}  // namespace

// out (contiguous, `shape`) = A[sa] op B[sb]; strides in elements, 0 = broadcast.
int nd_binary(tx_ctx *ctx, int op, const float *A, const int64_t *sa, const float *B, const int64_t *sb,
              float *out, const int64_t *shape, int ndim) {
  int64_t n = 1;
  for (int k = 0; k < ndim; ++k) n *= shape[k];
  if (n <= 0) return TX_OK;
  Nd c;
  const int64_t *st[2] = {sa, sb};
  canonicalize(ndim, shape, st, 2, c);
  const void *ptrs[3] = {A, B, out};
  const bool vec = vectorizable(c, 2, ptrs) && ((uintptr_t)out & 15) == 0;
  const bool small = n < (int64_t(1) << 31);
  const unsigned blocks = grid_for(vec ? n / 4 : n, 256);
  if (vec) {
    if (small) k_binary_nd<uint32_t, true><<<blocks, 256, 0, ctx->stream>>>(op, A, B, out, c, (uint32_t)n);
    else k_binary_nd<uint64_t, true><<<blocks, 256, 0, ctx->stream>>>(op, A, B, out, c, (uint64_t)n);
  } else {
    if (small) k_binary_nd<uint32_t, false><<<blocks, 256, 0, ctx->stream>>>(op, A, B, out, c, (uint32_t)n);
    else k_binary_nd<uint64_t, false><<<blocks, 256, 0, ctx->stream>>>(op, A, B, out, c, (uint64_t)n);
  }
  TX_LAUNCHED(ctx, "k_binary_nd");
  return TX_OK;
}

// out (contiguous, `shape`) (+)= scale * src[ss] (elem_bytes 4; 8 copies only).
int nd_copy(tx_ctx *ctx, const void *src, const int64_t *ss, void *out, const int64_t *shape, int ndim,
            int elem_bytes, float scale, int acc) {
  int64_t n = 1;
  for (int k = 0; k < ndim; ++k) n *= shape[k];
  if (n <= 0) return TX_OK;
  Nd c;
  const int64_t *st[1] = {ss};
  canonicalize(ndim, shape, st, 1, c);
  if (elem_bytes == 8) {
    if (scale != 1.f || acc) return TX_ERR_INVALID;
    return launch_copy<int64_t>(ctx, (const int64_t *)src, (int64_t *)out, c, n, 1.f, 0, false);
  }
  if (elem_bytes != 4) return TX_ERR_INVALID;
  // A copy that swaps the two inner merged axes of a contiguous [B][R][Cc]
  // source into [B][Cc][R] (attention's key transpose and its gradient) is a
  // batched matrix transpose: shared-memory tiles keep both sides coalesced
  // (element-wise, one side is strided by a whole row).
  if (scale == 1.f && (c.nd == 2 || c.nd == 3)) {
    const int o = c.nd - 2;  // [B?, Cc, R] in destination order
    const int64_t Cc = c.shape[o], R = c.shape[o + 1];
    const bool inner_swap = c.st[0][o] == 1 && c.st[0][o + 1] == Cc;
    const bool batch_ok = c.nd == 2 || c.st[0][0] == R * Cc;
    const int64_t B = c.nd == 3 ? c.shape[0] : 1;
    if (inner_swap && batch_ok && B <= 65535 && (R + 31) / 32 <= 65535)
      return batched_transpose(ctx, (const float *)src, (float *)out, B, R, Cc, acc);
  }
  const void *ptrs[2] = {src, out};
  const bool vec = vectorizable(c, 1, ptrs) && ((uintptr_t)out & 15) == 0;
  return launch_copy<float>(ctx, (const float *)src, (float *)out, c, n, scale, acc, vec);
}

// y (shape `out_shape`, 1 on reduced axes) (+)= scale * sum of contiguous x over
// the reduced axes.  Returns TX_ERR_UNSUPPORTED for layouts that are not
// [outer, red, inner] after canonicalisation (the caller's generic kernel).
int nd_reduce(tx_ctx *ctx, const float *x, const int64_t *in_shape, const int64_t *out_shape, int ndim,
              float *y, float scale, int acc) {
  // blocks of kept / reduced axes, innermost first; input is contiguous so
  // adjacent axes of the same kind always merge
  int64_t ext[kNd];
  bool redk[kNd];
  int m = 0;
  for (int k = ndim - 1; k >= 0; --k) {
    if (in_shape[k] == 1) continue;
    const bool r = out_shape[k] == 1;
    if (m > 0 && redk[m - 1] == r) {
      ext[m - 1] *= in_shape[k];
      continue;
    }
    ext[m] = in_shape[k];
    redk[m] = r;
    ++m;
  }
  int64_t outer = 1, red = 1, inner = 1;
  if (m == 0) return TX_ERR_UNSUPPORTED;
  // innermost-first blocks: [inner?] red [outer?]
  int i = 0;
  if (!redk[0]) inner = ext[i++];
  if (i >= m || !redk[i]) return TX_ERR_UNSUPPORTED;
  red = ext[i++];
  if (i < m) outer = ext[i++];
  if (i < m) return TX_ERR_UNSUPPORTED;
  if (inner == 1) {
    int64_t nb = (outer + 7) / 8;
    if (nb > 148 * 32) nb = 148 * 32;
    const unsigned blocks = (unsigned)(nb < 1 ? 1 : nb);
    k_reduce_rows<<<blocks, 256, 0, ctx->stream>>>(x, outer, red, y, scale, acc);
    TX_LAUNCHED(ctx, "k_reduce_rows");
    return TX_OK;
  }
  const bool vec = inner % 4 == 0 && ((uintptr_t)x & 15) == 0;
  const int64_t col_blocks = vec ? (inner + 127) / 128 : (inner + 31) / 32;
  if (outer > 65535 || col_blocks > 0x7fffffff) return TX_ERR_UNSUPPORTED;
  int64_t splits = (4 * (int64_t)ctx->num_sms + col_blocks * outer - 1) / (col_blocks * outer);
  const int64_t most = (red + 63) / 64;
  if (splits > most) splits = most;
  if (splits > 64) splits = 64;
  if (splits < 1) splits = 1;
  const int64_t rows_per = (red + splits - 1) / splits;
  splits = (red + rows_per - 1) / rows_per;
  Scratch part(ctx, splits > 1 ? (size_t)(outer * splits * inner) * sizeof(float) : 0);
  if (splits > 1 && !part.ptr) return TX_ERR_OOM;
  const dim3 grid((unsigned)col_blocks, (unsigned)splits, (unsigned)outer);
  if (vec)
    k_reduce_mid<true><<<grid, dim3(32, 8), 0, ctx->stream>>>(x, red, inner, rows_per, (int)splits,
                                                              part.as<float>(), y, scale, acc);
  else
    k_reduce_mid<false><<<grid, dim3(32, 8), 0, ctx->stream>>>(x, red, inner, rows_per, (int)splits,
                                                               part.as<float>(), y, scale, acc);
  TX_LAUNCHED(ctx, "k_reduce_mid");
  if (splits > 1) {
    k_reduce_mid_final<<<grid_for(outer * inner, 256), 256, 0, ctx->stream>>>(
        part.as<float>(), outer, (int)splits, inner, y, scale, acc);
    TX_LAUNCHED(ctx, "k_reduce_mid_final");
  }
  return TX_OK;
}

// ---- scatter, broadcast max / min / pow gradients, max / min reductions ----------------
// (Concat, Slice, Split and their gradients; Max / Min / Pow backward;
// ReduceMax / ReduceMin / GlobalMaxPool, crates/tynx/src/interpreter/
// reduction.rs and extrema.rs for the inference arms.)
namespace {

// out[off(i)] (+)= src[i]: a contiguous source into a strided destination
template <typename I>
__global__ void k_scatter_nd(const float *__restrict__ src, float *__restrict__ out, Nd c, I n, int acc) {
  for (I i = blockIdx.x * (I)blockDim.x + threadIdx.x; i < n; i += (I)gridDim.x * blockDim.x) {
    int64_t off[1];
    offsets<I, 1>(c, i, off);
    float *o = out + off[0];
    *o = acc ? *o + src[i] : src[i];
  }
}

// d out / d operand `which` of a broadcast MAX / MIN / POW, times dy, over the
// output shape (the caller reduces it to the operand's shape).  Ties go to A,
// as the forward takes A when a >= b (MAX) or a <= b (MIN).
template <typename I>
__global__ void k_binary_grad_nd(int op, int which, const float *__restrict__ A, const float *__restrict__ B,
                                 const float *__restrict__ dy, float *__restrict__ out, Nd c, I n) {
  for (I i = blockIdx.x * (I)blockDim.x + threadIdx.x; i < n; i += (I)gridDim.x * blockDim.x) {
    int64_t off[2];
    offsets<I, 2>(c, i, off);
    const float a = A[off[0]], b = B[off[1]], g = dy[i];
    float r = 0.f;
    if (op == TX_BIN_MAX || op == TX_BIN_MIN) {
      const bool take_a = op == TX_BIN_MAX ? a >= b : a <= b;
      r = (which == 0) == take_a ? g : 0.f;
    } else if (op == TX_BIN_POW) {
      r = which == 0 ? g * b * powf(a, b - 1.f) : g * powf(a, b) * logf(a);
    }
    out[i] = r;
  }
}

// y[o][i] = max (or min) over r of x[o][r][i], arg[o][i] = the first r that
// attains it (a NaN wins at its first occurrence)
__global__ void k_reduce_maxmin(const float *__restrict__ x, float *__restrict__ y, int32_t *__restrict__ arg,
                                int64_t outer, int64_t red, int64_t inner, int is_max) {
  const int64_t n = outer * inner;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = t / inner, i = t - o * inner;
    const float *p = x + o * red * inner + i;
    float m = p[0];
    int32_t at = 0;
    for (int64_t r = 1; r < red && m == m; ++r) {
      const float v = p[r * inner];
      if (v != v || (is_max ? v > m : v < m)) {
        m = v;
        at = (int32_t)r;
      }
    }
    y[t] = m;
    if (arg) arg[t] = at;
  }
}

// dx[o][arg[o][i]][i] += dy[o][i] (dx zeroed first unless accumulating)
__global__ void k_reduce_maxmin_bwd(const float *__restrict__ dy, const int32_t *__restrict__ arg,
                                    float *__restrict__ dx, int64_t outer, int64_t red, int64_t inner) {
  const int64_t n = outer * inner;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = t / inner, i = t - o * inner;
    dx[(o * red + arg[t]) * inner + i] += dy[t];
  }
}

}  // namespace

// out[os] (+)= src (contiguous, `shape`); os: the destination's element strides.
int nd_scatter(tx_ctx *ctx, const float *src, float *out, const int64_t *os, const int64_t *shape, int ndim,
               int acc) {
  int64_t n = 1;
  for (int k = 0; k < ndim; ++k) n *= shape[k];
  if (n <= 0) return TX_OK;
  Nd c;
  const int64_t *st[1] = {os};
  canonicalize(ndim, shape, st, 1, c);
  const unsigned blocks = grid_for(n, 256);
  if (n < (int64_t(1) << 31))
    k_scatter_nd<uint32_t><<<blocks, 256, 0, ctx->stream>>>(src, out, c, (uint32_t)n, acc);
  else
    k_scatter_nd<uint64_t><<<blocks, 256, 0, ctx->stream>>>(src, out, c, (uint64_t)n, acc);
  TX_LAUNCHED(ctx, "k_scatter_nd");
  return TX_OK;
}

int nd_binary_grad(tx_ctx *ctx, int op, int which, const float *A, const int64_t *sa, const float *B,
                   const int64_t *sb, const float *dy, float *out, const int64_t *shape, int ndim) {
  int64_t n = 1;
  for (int k = 0; k < ndim; ++k) n *= shape[k];
  if (n <= 0) return TX_OK;
  // dy and out are contiguous over `shape`: only A and B need strides
  Nd c;
  const int64_t *st[2] = {sa, sb};
  canonicalize(ndim, shape, st, 2, c);
  const unsigned blocks = grid_for(n, 256);
  if (n < (int64_t(1) << 31))
    k_binary_grad_nd<uint32_t><<<blocks, 256, 0, ctx->stream>>>(op, which, A, B, dy, out, c, (uint32_t)n);
  else
    k_binary_grad_nd<uint64_t><<<blocks, 256, 0, ctx->stream>>>(op, which, A, B, dy, out, c, (uint64_t)n);
  TX_LAUNCHED(ctx, "k_binary_grad_nd");
  return TX_OK;
}

int reduce_maxmin(tx_ctx *ctx, const float *x, float *y, int32_t *arg, int64_t outer, int64_t red, int64_t inner,
                  bool is_max) {
  if (outer * inner <= 0 || red <= 0) return TX_OK;
  k_reduce_maxmin<<<grid_for(outer * inner, 256), 256, 0, ctx->stream>>>(x, y, arg, outer, red, inner, is_max);
  TX_LAUNCHED(ctx, "k_reduce_maxmin");
  return TX_OK;
}

int reduce_maxmin_bwd(tx_ctx *ctx, const float *dy, const int32_t *arg, float *dx, int64_t outer, int64_t red,
                      int64_t inner, int acc) {
  if (outer * inner <= 0 || red <= 0) return TX_OK;
  if (!acc) TX_CUDA(ctx, cudaMemsetAsync(dx, 0, (size_t)outer * red * inner * sizeof(float), ctx->stream));
  k_reduce_maxmin_bwd<<<grid_for(outer * inner, 256), 256, 0, ctx->stream>>>(dy, arg, dx, outer, red, inner);
  TX_LAUNCHED(ctx, "k_reduce_maxmin_bwd");
  return TX_OK;
}
