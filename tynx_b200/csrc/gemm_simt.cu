// SIMT fp32 GEMM with the fused epilogue, and the GEMM dispatcher.
//
// The SIMT kernel is the exact-fp32 mode (TX_MATH_FP32: FFMA products, no
// operand rounding) and serves shapes the tensor-core kernel cannot take
// (strides that are not 16-byte multiples, tiny N such as 10-class heads).
// Semantics follow execute_gemm + add_bias
// (crates/tynx-train/src/imported_model/executor.rs:499-524, 606-613):
//   C = alpha * op(A) op(B) + bias_scale * bias   (then activation)
// plus beta * C for gradient accumulation (parameter.rs:300-333) and an
// optional act' multiply for backward (dgrad) fusion.
#include <math.h>

#include "common.h"
#include "epilogue.cuh"

namespace {

constexpr int BM = 64, BN = 64, BK = 16, TM = 4, TN = 4;

__device__ __forceinline__ float act_f(int act, float v) { return tx_epi::act(act, v); }
__device__ __forceinline__ float dact_f(int act, float s) { return tx_epi::dact(act, s); }

// split > 0: blockIdx.z is the K split; raw partial sums go to part[split][M][N]
__global__ void __launch_bounds__(256) k_gemm_simt(tx_gemm_desc d, int split_len, float *part) {
  __shared__ float As[BK][BM + 4];
  __shared__ float Bs[BK][BN + 4];
  const int64_t bz = part ? 0 : blockIdx.z;
  const float *A = d.A + bz * d.stride_a;
  const float *B = d.B + bz * d.stride_b;
  float *C = d.C + bz * d.stride_c;
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

  // Two-level accumulation: 256-deep partial sums are folded into `tot`, so a
  // long reduction (K = 4096 batch rows in a weight gradient) does not lose
  // precision to one running fp32 sum.
  float tot[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) tot[i][j] = 0.f;
  const int64_t k_begin = part ? (int64_t)blockIdx.z * split_len : 0;
  const int64_t k_end = part ? (k_begin + split_len < d.K ? k_begin + split_len : d.K) : d.K;
  for (int64_t k0 = k_begin; k0 < k_end; k0 += BK) {
    if (k0 != k_begin && ((k0 - k_begin) & 255) == 0) {
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) {
          tot[i][j] += acc[i][j];
          acc[i][j] = 0.f;
        }
    }
    // 64x16 A tile and 16x64 B tile: 1024 elements each, 4 per thread
    for (int e = threadIdx.x; e < BM * BK; e += 256) {
      int mm, kk;
      if (d.trans_a) { mm = e % BM; kk = e / BM; }  // A stored K x M: consecutive threads along m
      else { kk = e % BK; mm = e / BK; }
      int64_t gm = m0 + mm, gk = k0 + kk;
      float v = 0.f;
      if (gm < d.M && gk < k_end) v = d.trans_a ? A[gk * d.lda + gm] : A[gm * d.lda + gk];
      As[kk][mm] = v;
    }
    for (int e = threadIdx.x; e < BK * BN; e += 256) {
      int nn, kk;
      if (d.trans_b) { kk = e % BK; nn = e / BK; }  // B stored N x K
      else { nn = e % BN; kk = e / BN; }
      int64_t gn = n0 + nn, gk = k0 + kk;
      float v = 0.f;
      if (gn < d.N && gk < k_end) v = d.trans_b ? B[gn * d.ldb + gk] : B[gk * d.ldb + gn];
      Bs[kk][nn] = v;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[TM], b[TN];
#pragma unroll
      for (int i = 0; i < TM; ++i) a[i] = As[kk][ty * TM + i];
#pragma unroll
      for (int j = 0; j < TN; ++j) b[j] = Bs[kk][tx * TN + j];
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] += tot[i][j];
  if (part) {
    float *P = part + (int64_t)blockIdx.z * d.M * d.N;
#pragma unroll
    for (int i = 0; i < TM; ++i) {
      int64_t gm = m0 + ty * TM + i;
      if (gm >= d.M) continue;
#pragma unroll
      for (int j = 0; j < TN; ++j) {
        int64_t gn = n0 + tx * TN + j;
        if (gn < d.N) P[gm * d.N + gn] = acc[i][j];
      }
    }
    return;
  }
  // every load of the epilogue is issued before the first store (the stores
  // may alias the loaded tensors, so interleaving would serialise them)
  float cv[TM][TN], sv[TM][TN];
  const float *S = d.dact_src ? d.dact_src + bz * d.stride_c : nullptr;
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int64_t gm = m0 + ty * TM + i, gn = n0 + tx * TN + j;
      const bool ok = gm < d.M && gn < d.N;
      cv[i][j] = (ok && d.beta != 0.f) ? C[gm * d.ldc + gn] : 0.f;
      sv[i][j] = (ok && S) ? S[gm * d.ld_dact + gn] : 0.f;
    }
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    int64_t gm = m0 + ty * TM + i;
    if (gm >= d.M) continue;
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      int64_t gn = n0 + tx * TN + j;
      if (gn >= d.N) continue;
      float v = d.alpha * acc[i][j];
      if (d.bias) v += d.bias[gn] * d.bias_scale;
      if (d.beta != 0.f) v += d.beta * cv[i][j];
      if (d.preact) d.preact[bz * d.stride_c + gm * d.ld_preact + gn] = v;
      v = act_f(d.act, v);
      if (d.dact) v *= dact_f(d.dact, sv[i][j]);
      C[gm * d.ldc + gn] = (d.flags & TX_GEMM_ROUND_OUT) ? tx_epi::round_tf32(v) : v;
    }
  }
}

// Sum the split-K partials in a fixed order and apply the epilogue.  Block
// (32, 8): each thread owns up to 4 consecutive columns of one row.
__device__ __forceinline__ float split_epilogue(const tx_gemm_desc &d, float s, int64_t gm,
                                                int64_t gn) {
  float v = d.alpha * s;
  if (d.bias) v += d.bias[gn] * d.bias_scale;
  if (d.beta != 0.f) v += d.beta * d.C[gm * d.ldc + gn];
  if (d.preact) d.preact[gm * d.ld_preact + gn] = v;
  v = act_f(d.act, v);
  if (d.dact) v *= dact_f(d.dact, d.dact_src[gm * d.ld_dact + gn]);
  return (d.flags & TX_GEMM_ROUND_OUT) ? tx_epi::round_tf32(v) : v;
}

// Three blocks per SM (80 registers): at 96 registers two fitted and the
// grid of a 1024 x 1024 reduction ran in 3.5 waves (9.2 -> 6.6 us).
__global__ void __launch_bounds__(256, 3) k_gemm_split_reduce(tx_gemm_desc d, const float *__restrict__ part, int splits,
                                    int vec) {
  const int64_t gm = (int64_t)blockIdx.y * blockDim.y + threadIdx.y;
  const int64_t gn = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (gm >= d.M || gn >= d.N) return;
  const int64_t n = d.M * d.N;
  const float *src = part + gm * d.N + gn;
  if (vec && gn + 4 <= d.N) {
    // partials are added in split order (the first one starts the sum); up to
    // four loads are in flight before the adds (four blocks per SM)
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int p = 0; p < splits; p += 4) {
      float4 t[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (p + j < splits) t[j] = *reinterpret_cast<const float4 *>(src + (int64_t)(p + j) * n);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (p + j >= splits) break;
        if (p + j == 0) {
          s = t[0];
        } else {
          s.x += t[j].x;
          s.y += t[j].y;
          s.z += t[j].z;
          s.w += t[j].w;
        }
      }
    }
    float4 o = make_float4(split_epilogue(d, s.x, gm, gn), split_epilogue(d, s.y, gm, gn + 1),
                           split_epilogue(d, s.z, gm, gn + 2), split_epilogue(d, s.w, gm, gn + 3));
    if (((d.ldc & 3) == 0) && ((((uintptr_t)(d.C + gm * d.ldc + gn)) & 15) == 0)) {
      *reinterpret_cast<float4 *>(d.C + gm * d.ldc + gn) = o;
    } else {
      d.C[gm * d.ldc + gn] = o.x;
      d.C[gm * d.ldc + gn + 1] = o.y;
      d.C[gm * d.ldc + gn + 2] = o.z;
      d.C[gm * d.ldc + gn + 3] = o.w;
    }
    return;
  }
  for (int64_t c = gn; c < gn + 4 && c < d.N; ++c) {
    float s = 0.f;
    for (int p = 0; p < splits; ++p) s += part[(int64_t)p * n + gm * d.N + c];
    d.C[gm * d.ldc + c] = split_epilogue(d, s, gm, c);
  }
}

// Many splits of a small output: block (32, 8) covers 128 consecutive output
// elements (4 per thread, flattened row-major), its 8 row groups take splits
// ty, ty + 8, ... in order, and the groups are combined in a fixed order
// before the epilogue.  N % 4 == 0 so that 4 consecutive elements share a row.
__global__ void k_gemm_split_reduce_tree(tx_gemm_desc d, const float *__restrict__ part, int splits) {
  __shared__ float4 sm[8][32];
  const int64_t n = d.M * d.N;
  const int64_t e = ((int64_t)blockIdx.x * 32 + threadIdx.x) * 4;
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  if (e < n) {
    int p = threadIdx.y;
    for (; p + 24 < splits; p += 32) {
      float4 t[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) t[j] = *reinterpret_cast<const float4 *>(part + (int64_t)(p + 8 * j) * n + e);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        s.x += t[j].x;
        s.y += t[j].y;
        s.z += t[j].z;
        s.w += t[j].w;
      }
    }
    for (; p < splits; p += 8) {
      const float4 t = *reinterpret_cast<const float4 *>(part + (int64_t)p * n + e);
      s.x += t.x;
      s.y += t.y;
      s.z += t.z;
      s.w += t.w;
    }
  }
  sm[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y != 0 || e >= n) return;
  float4 t = sm[0][threadIdx.x];
#pragma unroll
  for (int i = 1; i < 8; ++i) {
    const float4 u = sm[i][threadIdx.x];
    t.x += u.x;
    t.y += u.y;
    t.z += u.z;
    t.w += u.w;
  }
  const int64_t gm = e / d.N, gn = e - gm * d.N;
  const float4 o = make_float4(split_epilogue(d, t.x, gm, gn), split_epilogue(d, t.y, gm, gn + 1),
                               split_epilogue(d, t.z, gm, gn + 2), split_epilogue(d, t.w, gm, gn + 3));
  float *c = d.C + gm * d.ldc + gn;
  if (((d.ldc & 3) == 0) && ((((uintptr_t)c) & 15) == 0)) {
    *reinterpret_cast<float4 *>(c) = o;
  } else {
    c[0] = o.x;
    c[1] = o.y;
    c[2] = o.z;
    c[3] = o.w;
  }
}

}  // namespace

// Sum `splits` raw [M, N] partial products in a fixed order (IEEE fp32 adds) and
// apply the epilogue of d.  Shared by the split-K paths of both GEMM kernels.
int gemm_split_reduce(tx_ctx *ctx, const tx_gemm_desc &d, const float *part, int splits) {
  const int vec = ((d.N & 3) == 0) && ((((uintptr_t)part) & 15) == 0);
  if (vec && splits >= 16 && d.M * d.N <= (int64_t)ctx->num_sms * 512) {
    const int64_t blocks = (d.M * d.N + 127) / 128;
    k_gemm_split_reduce_tree<<<(unsigned)blocks, dim3(32, 8), 0, ctx->stream>>>(d, part, splits);
    TX_LAUNCHED(ctx, "k_gemm_split_reduce_tree");
    return TX_OK;
  }
  dim3 block(32, 8);
  dim3 grid((unsigned)((d.N + 127) / 128), (unsigned)((d.M + 7) / 8));
  if (grid.y > 65535) return tx_fail(ctx, TX_ERR_UNSUPPORTED, "split-K reduce: M too large");
  k_gemm_split_reduce<<<grid, block, 0, ctx->stream>>>(d, part, splits, vec);
  TX_LAUNCHED(ctx, "k_gemm_split_reduce");
  return TX_OK;
}

int gemm_simt(tx_ctx *ctx, const tx_gemm_desc &d) {
  int64_t batch = d.batch > 1 ? d.batch : 1;
  if (batch > 65535) return tx_fail(ctx, TX_ERR_UNSUPPORTED, "GEMM batch above 65535");
  dim3 grid((unsigned)((d.N + BN - 1) / BN), (unsigned)((d.M + BM - 1) / BM), (unsigned)batch);
  if (grid.y > 65535) return tx_fail(ctx, TX_ERR_UNSUPPORTED, "GEMM M too large for SIMT grid");
  // Skinny outputs with a long reduction (the weight gradient of a 10-class head:
  // M = 10, N = 1024, K = batch) leave most SMs idle: split K across blocks.
  const int64_t tiles = (int64_t)grid.x * grid.y;
  if (batch == 1 && tiles < ctx->num_sms && d.K >= 8 * BK) {
    int64_t splits = (2 * ctx->num_sms + tiles - 1) / tiles;
    int64_t max_splits = d.K / (4 * BK);
    if (splits > max_splits) splits = max_splits;
    if (splits > 64) splits = 64;
    if (splits >= 2) {
      int64_t split_len = ((d.K + splits - 1) / splits + BK - 1) / BK * BK;
      splits = (d.K + split_len - 1) / split_len;
      Scratch part(ctx, (size_t)splits * d.M * d.N * sizeof(float));
      if (!part.ptr) return TX_ERR_OOM;
      grid.z = (unsigned)splits;
      k_gemm_simt<<<grid, 256, 0, ctx->stream>>>(d, (int)split_len, part.as<float>());
      TX_LAUNCHED(ctx, "k_gemm_simt(split)");
      return gemm_split_reduce(ctx, d, part.as<float>(), (int)splits);
    }
  }
  k_gemm_simt<<<grid, 256, 0, ctx->stream>>>(d, 0, nullptr);
  TX_LAUNCHED(ctx, "k_gemm_simt");
  return TX_OK;
}

int gemm_dispatch(tx_ctx *ctx, const tx_gemm_desc &desc, bool *rounded) {
  if (rounded) *rounded = false;
  tx_gemm_desc d = desc;
  if (ctx->math != TX_MATH_TF32) {
    d.flags &= TX_GEMM_A_SHARED;  // TF32 operand / output rounding only applies there
    d.B_lo = nullptr;
  }
  if (d.B_lo && d.M > 0 && d.N > 0) {
    // split weights: the persistent tcgen05 kernel takes the head and the
    // tail in one pass; any other path computes C = alpha A B_lo first, then
    // alpha A B + C with the epilogue (beta 1)
    if (d.colsum || d.beta != 0.f || (d.flags & TX_GEMM_EXACT))
      return tx_fail(ctx, TX_ERR_UNSUPPORTED, "split weights with beta, column sums or EXACT");
    // (skinny shapes take the FFMA kernels for both products)
    int rc = skinny_shape(d) ? TX_ERR_UNSUPPORTED : gemm_tcgen05(ctx, d, (d.flags & TX_GEMM_A_TF32) ? 0 : 1, nullptr);
    if (rc != TX_ERR_UNSUPPORTED) {
      if (rounded) *rounded = rc == TX_OK && (d.flags & TX_GEMM_ROUND_OUT);
      return rc;
    }
    tx_gemm_desc lo = d;
    lo.B = d.B_lo;
    lo.B_lo = nullptr;
    lo.bias = nullptr;
    lo.act = TX_ACT_NONE;
    lo.preact = nullptr;
    lo.dact = TX_ACT_NONE;
    lo.dact_src = nullptr;
    lo.flags &= ~TX_GEMM_ROUND_OUT;
    TX_TRY(gemm_dispatch(ctx, lo));
    tx_gemm_desc hi = d;
    hi.B_lo = nullptr;
    hi.beta = 1.f;
    return gemm_dispatch(ctx, hi, rounded);
  }
  if (d.M <= 0 || d.N <= 0) {
    if (d.colsum && d.N > 0 && !d.colsum_acc)
      TX_CUDA(ctx, cudaMemsetAsync(d.colsum, 0, d.N * sizeof(float), ctx->stream));
    return TX_OK;
  }
  const bool want = d.colsum != nullptr;
  if (want && (d.batch > 1 || d.ldc != d.N))
    return tx_fail(ctx, TX_ERR_UNSUPPORTED, "fused column sums need batch 1 and ldc == N");
  Scratch part(ctx, want ? (size_t)((d.M + 31) / 32) * d.N * sizeof(float) : 0);
  if (want && !part.ptr) return TX_ERR_OOM;
  FusedSum fs;
  fs.part = part.as<float>();
  FusedSum *pfs = want ? &fs : nullptr;
  int rc = gemm_skinny(ctx, d, pfs);
  if (rc == TX_ERR_UNSUPPORTED && ctx->math != TX_MATH_FP32) {
    int mode = ctx->math == TX_MATH_3XTF32 ? 2 : ctx->math == TX_MATH_TF32_TRUNC ? 0 : 1;
    tx_gemm_desc e = d;
    if (ctx->math == TX_MATH_TF32 && (d.flags & TX_GEMM_EXACT)) {
      // fp32-class product in TF32 mode: both operands are split in the kernel
      mode = 2;
      e.flags &= ~(TX_GEMM_A_TF32 | TX_GEMM_B_TF32);
    }
    rc = gemm_tcgen05(ctx, e, mode, pfs);
  }
  if (rc == TX_ERR_UNSUPPORTED) {
    tx_gemm_desc q = d;
    if (want) q.flags &= ~TX_GEMM_ROUND_OUT;
    rc = gemm_simt(ctx, q);
  }
  if (rc != TX_OK) return rc;
  if (want) {
    if (fs.fused)
      TX_TRY(colsum_finish(ctx, fs.part, fs.rows, d.N, d.colsum, d.colsum_scale, d.colsum_acc));
    else
      TX_TRY(tx_bias_grad(ctx, d.C, d.colsum, d.M, d.N, d.colsum_scale, d.colsum_acc));
  }
  if (rounded) *rounded = (d.flags & TX_GEMM_ROUND_OUT) && (!want || fs.fused);
  return TX_OK;
}

extern "C" int tx_gemm(tx_ctx *ctx, const tx_gemm_desc *desc) {
  if (!ctx || !desc) return TX_ERR_INVALID;
  const tx_gemm_desc &d = *desc;
  if (d.M < 0 || d.N < 0 || d.K < 0) return tx_fail(ctx, TX_ERR_SHAPE, "negative GEMM extent");
  if (d.act < 0 || d.act > TX_ACT_GELU || d.dact < 0 || d.dact > TX_ACT_GELU)
    return TX_ERR_INVALID;
  if (d.dact && !d.dact_src) return TX_ERR_INVALID;
  return gemm_dispatch(ctx, d);
}
