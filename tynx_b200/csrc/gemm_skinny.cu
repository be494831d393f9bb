// Skinny contractions: one extent is tiny, so the work is bound by HBM traffic,
// not by the tensor core.  These are the classifier / value heads of every
// workload and their gradients (a Gemm 1024 -> 10 gives a forward with N = 10,
// a dgrad with K = 10 and a wgrad with M = 10), and the first convolution of a
// CNN lowered to a GEMM (K = 3 * 3 * 3 = 27).  All three kernels accumulate in
// IEEE fp32 (FFMA) in a fixed order, so they are exact-fp32-class in every math
// mode, and apply the same epilogue as the other GEMM kernels
// (alpha, bias * bias_scale, beta * C, pre-activation store, act, act').
//
//   small K (K <= 32)   C = op(A) op(B): both operand tiles staged in shared
//                       memory, each thread owns 4 adjacent columns x 8 rows;
//                       float4 loads and stores of C and of the act' source.
//   small N (N <= 16)   A row-major (K contiguous): a warp per output row reads
//                       the row with float4 loads, op(B) sits in shared memory,
//                       and a butterfly shuffle reduces the N dot products.
//   small M (M <= 16)   B row-major (N contiguous): K is split across blocks,
//                       each lane owns 4 columns, warps split the block's K
//                       range, a fixed-order tree combines the warps, and the
//                       split-K reduction applies the epilogue.
// Semantics are those of execute_gemm + add_bias
// (crates/tynx-train/src/imported_model/executor.rs:499-524, 606-613).
#include "common.h"
#include "epilogue.cuh"

namespace {

constexpr int SK_KMAX = 32;
constexpr int kSmallMSmem = 96 * 1024;  // As[kc][MM] + red[8][MM][128]

struct EpiVals {
  float out, pre;
};

__device__ __forceinline__ EpiVals finish(const tx_gemm_desc &d, float acc, float bias_v,
                                          float c_old, float s) {
  float v = d.alpha * acc;
  if (d.bias) v += bias_v;
  if (d.beta != 0.f) v += d.beta * c_old;
  const float pre = v;
  v = tx_epi::act(d.act, v);
  if (d.dact) v *= tx_epi::dact(d.dact, s);
  if (d.flags & TX_GEMM_ROUND_OUT) v = tx_epi::round_tf32(v);
  return {v, pre};
}

__device__ __forceinline__ float4 ld4(const float *p, bool vec, int valid) {
  if (vec && valid >= 4) return *reinterpret_cast<const float4 *>(p);
  float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
  if (valid > 0) r.x = p[0];
  if (valid > 1) r.y = p[1];
  if (valid > 2) r.z = p[2];
  if (valid > 3) r.w = p[3];
  return r;
}

__device__ __forceinline__ void st4(float *p, float4 v, bool vec, int valid) {
  if (vec && valid >= 4) {
    *reinterpret_cast<float4 *>(p) = v;
    return;
  }
  if (valid > 0) p[0] = v.x;
  if (valid > 1) p[1] = v.y;
  if (valid > 2) p[2] = v.z;
  if (valid > 3) p[3] = v.w;
}

__host__ __device__ __forceinline__ bool vec_ok(const float *p, int64_t ld) {
  return p && ((ld & 3) == 0) && ((((uintptr_t)p) & 15) == 0);
}

// Epilogue of one thread's 8 rows x 4 columns.  ACT / DACT are compile-time so
// that the unrolled rows hold only the math they run (-1: runtime values, for
// the rare activation-and-act' combination).  Loads precede every store.
struct EpiRow {
  float *C;
  const float *S;  // act' source
  float *P;        // pre-activation
  int64_t gn;
};

template <int ACT, int DACT, int RG>
__device__ __forceinline__ void small_k_epilogue(const tx_gemm_desc &d, const EpiRow &er,
                                                 float (&acc)[8][4], int row_first) {
  const int act = ACT >= 0 ? ACT : d.act;
  const int dact = DACT >= 0 ? DACT : d.dact;
  const int64_t gn = er.gn;
  const int valid = d.N - gn >= 4 ? 4 : (int)(d.N - gn);
  const bool vc = vec_ok(er.C, d.ldc);
  const bool vs = vec_ok(er.S, d.ld_dact);
  const bool vp = vec_ok(er.P, d.ld_preact);
  const bool beta = d.beta != 0.f;
  float4 bias = make_float4(0.f, 0.f, 0.f, 0.f);
  if (d.bias) {
    bias = ld4(d.bias + gn, false, valid);
    bias.x *= d.bias_scale;
    bias.y *= d.bias_scale;
    bias.z *= d.bias_scale;
    bias.w *= d.bias_scale;
  }
  float4 cold[8], sv[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t gm = row_first + RG * i;
    const bool ok = gm < d.M;
    cold[i] = (ok && beta) ? ld4(er.C + gm * d.ldc + gn, vc, valid) : make_float4(0.f, 0.f, 0.f, 0.f);
    sv[i] = (ok && dact != TX_ACT_NONE) ? ld4(er.S + gm * d.ld_dact + gn, vs, valid)
                                        : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t gm = row_first + RG * i;
    if (gm >= d.M) continue;
    float4 pre = make_float4(d.alpha * acc[i][0], d.alpha * acc[i][1], d.alpha * acc[i][2],
                             d.alpha * acc[i][3]);
    float4 o;
    if (d.bias) {
      pre.x += bias.x;
      pre.y += bias.y;
      pre.z += bias.z;
      pre.w += bias.w;
    }
    if (beta) {
      pre.x += d.beta * cold[i].x;
      pre.y += d.beta * cold[i].y;
      pre.z += d.beta * cold[i].z;
      pre.w += d.beta * cold[i].w;
    }
    if (er.P) st4(er.P + gm * d.ld_preact + gn, pre, vp, valid);
    o.x = tx_epi::act(act, pre.x);
    o.y = tx_epi::act(act, pre.y);
    o.z = tx_epi::act(act, pre.z);
    o.w = tx_epi::act(act, pre.w);
    if (dact != TX_ACT_NONE) {
      o.x *= tx_epi::dact(dact, sv[i].x);
      o.y *= tx_epi::dact(dact, sv[i].y);
      o.z *= tx_epi::dact(dact, sv[i].z);
      o.w *= tx_epi::dact(dact, sv[i].w);
    }
    if (d.flags & TX_GEMM_ROUND_OUT) {
      o.x = tx_epi::round_tf32(o.x);
      o.y = tx_epi::round_tf32(o.y);
      o.z = tx_epi::round_tf32(o.z);
      o.w = tx_epi::round_tf32(o.w);
    }
    st4(er.C + gm * d.ldc + gn, o, vc, valid);
  }
}

// ---- small K ----------------------------------------------------------------------------
// TCOLS columns per block (TCOLS / 4 threads per row), 8 rows per thread.
template <int TCOLS>
__global__ void __launch_bounds__(256) k_gemm_small_k(const tx_gemm_desc d) {
  constexpr int TPR = TCOLS / 4;    // threads per row
  constexpr int RG = 256 / TPR;     // row groups
  constexpr int ROWS = RG * 8;      // rows per block
  __shared__ __align__(16) float Bs[SK_KMAX][TCOLS + 4];
  __shared__ float As[ROWS][SK_KMAX + 1];
  const int64_t bz = blockIdx.z;
  const float *A = d.A + bz * d.stride_a;
  const float *B = d.B + bz * d.stride_b;
  float *C = d.C + bz * d.stride_c;
  const int64_t m0 = (int64_t)blockIdx.y * ROWS, n0 = (int64_t)blockIdx.x * TCOLS;
  const int K = (int)d.K;
#pragma unroll 4
  for (int e = threadIdx.x; e < K * TCOLS; e += 256) {
    int k, n;
    if (d.trans_b) { k = e % K; n = e / K; }  // stored N x K
    else { n = e % TCOLS; k = e / TCOLS; }    // stored K x N
    const int64_t gn = n0 + n;
    Bs[k][n] = gn < d.N ? (d.trans_b ? B[gn * d.ldb + k] : B[(int64_t)k * d.ldb + gn]) : 0.f;
  }
#pragma unroll 4
  for (int e = threadIdx.x; e < K * ROWS; e += 256) {
    int k, m;
    if (d.trans_a) { m = e % ROWS; k = e / ROWS; }  // stored K x M
    else { k = e % K; m = e / K; }                  // stored M x K
    const int64_t gm = m0 + m;
    As[m][k] = gm < d.M ? (d.trans_a ? A[(int64_t)k * d.lda + gm] : A[gm * d.lda + k]) : 0.f;
  }
  __syncthreads();

  const int cg = threadIdx.x % TPR, rg = threadIdx.x / TPR;
  float acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  for (int k = 0; k < K; ++k) {
    const float4 b = *reinterpret_cast<const float4 *>(&Bs[k][cg * 4]);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float a = As[rg + RG * i][k];
      acc[i][0] = fmaf(a, b.x, acc[i][0]);
      acc[i][1] = fmaf(a, b.y, acc[i][1]);
      acc[i][2] = fmaf(a, b.z, acc[i][2]);
      acc[i][3] = fmaf(a, b.w, acc[i][3]);
    }
  }

  const int64_t gn = n0 + cg * 4;
  if (gn >= d.N) return;
  const EpiRow er{C, d.dact_src ? d.dact_src + bz * d.stride_c : nullptr,
                  d.preact ? d.preact + bz * d.stride_c : nullptr, gn};
  const int row_first = (int)(m0 + rg);
  if (!d.dact) {
    switch (d.act) {
      case TX_ACT_RELU: small_k_epilogue<TX_ACT_RELU, TX_ACT_NONE, RG>(d, er, acc, row_first); break;
      case TX_ACT_TANH: small_k_epilogue<TX_ACT_TANH, TX_ACT_NONE, RG>(d, er, acc, row_first); break;
      case TX_ACT_GELU: small_k_epilogue<TX_ACT_GELU, TX_ACT_NONE, RG>(d, er, acc, row_first); break;
      default: small_k_epilogue<TX_ACT_NONE, TX_ACT_NONE, RG>(d, er, acc, row_first); break;
    }
  } else if (d.act == TX_ACT_NONE) {
    switch (d.dact) {
      case TX_ACT_RELU: small_k_epilogue<TX_ACT_NONE, TX_ACT_RELU, RG>(d, er, acc, row_first); break;
      case TX_ACT_TANH: small_k_epilogue<TX_ACT_NONE, TX_ACT_TANH, RG>(d, er, acc, row_first); break;
      default: small_k_epilogue<TX_ACT_NONE, TX_ACT_GELU, RG>(d, er, acc, row_first); break;
    }
  } else {
    small_k_epilogue<-1, -1, RG>(d, er, acc, row_first);
  }
}

// Aligned fast path (N % 4 == 0, C / act' source / pre-activation 16-byte
// aligned with leading dimensions that are multiples of 4): the activation pair
// is a template parameter and every access is a float4, so the unrolled rows
// carry no alternative code; B is staged once per block and the block walks
// row tiles, so its instructions are reused instead of fetched once per warp.
template <int TCOLS, int ACT, int DACT>
__global__ void __launch_bounds__(256) k_gemm_small_k2(const tx_gemm_desc d, int row_tiles, float *col_part) {
  constexpr int TPR = TCOLS / 4;
  constexpr int RG = 256 / TPR;
  constexpr int ROWS = RG * 8;
  __shared__ __align__(16) float Bs[SK_KMAX][TCOLS + 4];
  __shared__ float As[ROWS][SK_KMAX + 1];
  __shared__ float red[RG][TCOLS];  // fused column sums: one row per row group
  const int64_t bz = blockIdx.z;
  const float *A = d.A + bz * d.stride_a;
  const float *B = d.B + bz * d.stride_b;
  float *C = d.C + bz * d.stride_c;
  const float *S = d.dact_src ? d.dact_src + bz * d.stride_c : nullptr;
  float *P = d.preact ? d.preact + bz * d.stride_c : nullptr;
  const int64_t n0 = (int64_t)blockIdx.x * TCOLS;
  const int K = (int)d.K;
  const int cg = threadIdx.x % TPR, rg = threadIdx.x / TPR;
  const int64_t gn = n0 + cg * 4;
  const bool col_ok = gn < d.N;  // N % 4 == 0: a group is all in or all out
  const bool beta = d.beta != 0.f;
  // epilogue inputs (C for beta, the act' source) of a row tile: they do not
  // depend on the products, so they are in flight while A and B are staged
  float4 cold[8], sv[8];
  auto load_epi = [&](int64_t m0) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t gm = m0 + rg + RG * i;
      const bool ok = col_ok && gm < d.M;
      cold[i] = (ok && beta) ? *reinterpret_cast<const float4 *>(C + gm * d.ldc + gn) : make_float4(0.f, 0.f, 0.f, 0.f);
      sv[i] = (ok && DACT != TX_ACT_NONE) ? *reinterpret_cast<const float4 *>(S + gm * d.ld_dact + gn)
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  if ((int)blockIdx.y < row_tiles) load_epi((int64_t)blockIdx.y * ROWS);
  for (int e = threadIdx.x; e < K * TCOLS; e += 256) {
    int k, n;
    if (d.trans_b) { k = e % K; n = e / K; }
    else { n = e % TCOLS; k = e / TCOLS; }
    const int64_t gbn = n0 + n;
    Bs[k][n] = gbn < d.N ? (d.trans_b ? B[gbn * d.ldb + k] : B[(int64_t)k * d.ldb + gbn]) : 0.f;
  }
  float4 bias = make_float4(0.f, 0.f, 0.f, 0.f);
  if (d.bias && col_ok) {
    bias = make_float4(d.bias[gn] * d.bias_scale, d.bias[gn + 1] * d.bias_scale, d.bias[gn + 2] * d.bias_scale,
                       d.bias[gn + 3] * d.bias_scale);
  }
  const bool round_out = (d.flags & TX_GEMM_ROUND_OUT) != 0;
#pragma unroll 1
  for (int rt = blockIdx.y; rt < row_tiles; rt += gridDim.y) {
    const int64_t m0 = (int64_t)rt * ROWS;
    if (rt != (int)blockIdx.y) load_epi(m0);  // the first tile's were issued above
    __syncthreads();  // the previous tile's readers of As are done
    for (int e = threadIdx.x; e < K * ROWS; e += 256) {
      int k, m;
      if (d.trans_a) { m = e % ROWS; k = e / ROWS; }
      else { k = e % K; m = e / K; }
      const int64_t gm = m0 + m;
      As[m][k] = gm < d.M ? (d.trans_a ? A[(int64_t)k * d.lda + gm] : A[gm * d.lda + k]) : 0.f;
    }
    __syncthreads();
    float acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    for (int k = 0; k < K; ++k) {
      const float4 b = *reinterpret_cast<const float4 *>(&Bs[k][cg * 4]);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float a = As[rg + RG * i][k];
        acc[i][0] = fmaf(a, b.x, acc[i][0]);
        acc[i][1] = fmaf(a, b.y, acc[i][1]);
        acc[i][2] = fmaf(a, b.z, acc[i][2]);
        acc[i][3] = fmaf(a, b.w, acc[i][3]);
      }
    }
    float csum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t gm = m0 + rg + RG * i;
      if (!col_ok || gm >= d.M) continue;
      float o[4];
      const float bb[4] = {bias.x, bias.y, bias.z, bias.w};
      const float cc[4] = {cold[i].x, cold[i].y, cold[i].z, cold[i].w};
      const float ss[4] = {sv[i].x, sv[i].y, sv[i].z, sv[i].w};
      float pre[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float x = d.alpha * acc[i][j];
        if (d.bias) x += bb[j];
        if (beta) x += d.beta * cc[j];
        pre[j] = x;
        x = tx_epi::act(ACT, x);
        if (DACT != TX_ACT_NONE) x *= tx_epi::dact(DACT, ss[j]);
        csum[j] += x;
        o[j] = round_out ? tx_epi::round_tf32(x) : x;
      }
      if (P) *reinterpret_cast<float4 *>(P + gm * d.ld_preact + gn) = make_float4(pre[0], pre[1], pre[2], pre[3]);
      *reinterpret_cast<float4 *>(C + gm * d.ldc + gn) = make_float4(o[0], o[1], o[2], o[3]);
    }
    if (col_part) {
      // this tile's column sums: the row groups combined in a fixed order
#pragma unroll
      for (int j = 0; j < 4; ++j) red[rg][cg * 4 + j] = csum[j];
      __syncthreads();
      if (rg == 0 && col_ok) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float t = red[0][cg * 4 + j];
#pragma unroll
          for (int g = 1; g < RG; ++g) t += red[g][cg * 4 + j];
          col_part[(int64_t)rt * d.N + gn + j] = t;
        }
      }
    }
  }
}

// ---- small N ----------------------------------------------------------------------------
// Dynamic shared memory: Bs[NN][kc] (op(B) transposed to N x K, zero padded),
// kc <= SN_KC.  Each lane holds 8 float4 of a row (K chunk <= 1024); the next
// row's loads are issued before the current row is reduced.
// part != nullptr: blockIdx.y is the K split and raw sums go to part[y][M][N].
constexpr int SN_KC = 1024;

// Two blocks per SM (at most 128 registers): the launch below sizes the grid
// for two, and at 176 registers one fitted and the grid ran in two waves.
template <int NN>
__global__ void __launch_bounds__(256, 2) k_gemm_small_n(const tx_gemm_desc d, int kc, float *part) {
  extern __shared__ __align__(16) float bsm[];
  const int64_t k0 = (int64_t)blockIdx.y * kc;
  const int klen = (int)(d.K - k0 < kc ? d.K - k0 : kc);
  if (d.trans_b && vec_ok(d.B, d.ldb)) {  // stored N x K: float4 along K
    const int kc4 = kc / 4;
#pragma unroll 4
    for (int e = threadIdx.x; e < NN * kc4; e += 256) {
      const int n = e / kc4, kk = (e % kc4) * 4;
      const float4 v = n < d.N ? ld4(d.B + (int64_t)n * d.ldb + k0 + kk, true, klen - kk)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
      *reinterpret_cast<float4 *>(&bsm[n * kc + kk]) = v;
    }
  } else {
#pragma unroll 4
    for (int e = threadIdx.x; e < NN * kc; e += 256) {
      int n, kk;
      if (d.trans_b) { kk = e % kc; n = e / kc; }  // stored N x K
      else { n = e % NN; kk = e / NN; }            // stored K x N
      float v = 0.f;
      if (n < d.N && kk < klen)
        v = d.trans_b ? d.B[(int64_t)n * d.ldb + k0 + kk] : d.B[(k0 + kk) * d.ldb + n];
      bsm[n * kc + kk] = v;
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool avec = vec_ok(d.A, d.lda);
  // two rows per warp: every W float4 read from shared memory feeds both
  const int64_t stride = (int64_t)gridDim.x * 16;
  for (int64_t m = ((int64_t)blockIdx.x * 8 + warp) * 2; m < d.M; m += stride) {
    const bool two = m + 1 < d.M;
    const float *a0p = d.A + m * d.lda + k0;
    const float *a1p = a0p + d.lda;
    float4 a0[8], a1[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int kk = lane * 4 + 128 * j;
      const bool in = kk < klen;
      a0[j] = in ? ld4(a0p + kk, avec, klen - kk) : make_float4(0.f, 0.f, 0.f, 0.f);
      a1[j] = (in && two) ? ld4(a1p + kk, avec, klen - kk) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float acc0[NN], acc1[NN];
#pragma unroll
    for (int n = 0; n < NN; ++n) acc0[n] = acc1[n] = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int kk = lane * 4 + 128 * j;
      if (kk < klen) {
#pragma unroll
        for (int n = 0; n < NN; ++n) {
          const float4 b = *reinterpret_cast<const float4 *>(&bsm[n * kc + kk]);
          float t = acc0[n], u = acc1[n];
          t = fmaf(a0[j].x, b.x, t);
          u = fmaf(a1[j].x, b.x, u);
          t = fmaf(a0[j].y, b.y, t);
          u = fmaf(a1[j].y, b.y, u);
          t = fmaf(a0[j].z, b.z, t);
          u = fmaf(a1[j].z, b.z, u);
          t = fmaf(a0[j].w, b.w, t);
          u = fmaf(a1[j].w, b.w, u);
          acc0[n] = t;
          acc1[n] = u;
        }
      }
    }
#pragma unroll
    for (int n = 0; n < NN; ++n) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        acc0[n] += __shfl_xor_sync(0xffffffffu, acc0[n], off);
        acc1[n] += __shfl_xor_sync(0xffffffffu, acc1[n], off);
      }
    }
    // lanes 0..N-1 finish row m, lanes 16..16+N-1 row m + 1
    const int col = lane & 15;
    const int64_t row = m + (lane >> 4);
    float v = 0.f;
#pragma unroll
    for (int n = 0; n < NN; ++n)
      if (n == col) v = (lane >> 4) ? acc1[n] : acc0[n];
    if (col >= d.N || row >= d.M) continue;
    if (part) {
      part[(int64_t)blockIdx.y * d.M * d.N + row * d.N + col] = v;
      continue;
    }
    const float bias_v = d.bias ? d.bias[col] * d.bias_scale : 0.f;
    const float c_old = d.beta != 0.f ? d.C[row * d.ldc + col] : 0.f;
    const float sv = d.dact ? d.dact_src[row * d.ld_dact + col] : 0.f;
    const EpiVals r = finish(d, v, bias_v, c_old, sv);
    if (d.preact) d.preact[row * d.ld_preact + col] = r.pre;
    d.C[row * d.ldc + col] = r.out;
  }
}

// ---- small M ----------------------------------------------------------------------------
// Block: 8 warps x 32 lanes; 128 columns (4 per lane); blockIdx.y = K split of
// kc rows, dealt to the warps round-robin.  Dynamic shared memory:
// As[kc][MM] then red[8][MM][128].
template <int MM>
__global__ void __launch_bounds__(256) k_gemm_small_m(const tx_gemm_desc d, int kc, float *part) {
  extern __shared__ __align__(16) float sm[];
  float *As = sm;
  float *red = sm + kc * MM;
  const int64_t k0 = (int64_t)blockIdx.y * kc;
  const int klen = (int)(d.K - k0 < kc ? d.K - k0 : kc);
#pragma unroll 4
  for (int e = threadIdx.x; e < kc * MM; e += 256) {
    int m, kk;
    if (d.trans_a) { m = e % MM; kk = e / MM; }  // stored K x M
    else { kk = e % kc; m = e / kc; }            // stored M x K
    float v = 0.f;
    if (m < d.M && kk < klen)
      v = d.trans_a ? d.A[(k0 + kk) * d.lda + m] : d.A[(int64_t)m * d.lda + k0 + kk];
    As[kk * MM + m] = v;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t gn = (int64_t)blockIdx.x * 128 + lane * 4;
  const int valid = d.N - gn >= 4 ? 4 : (int)(d.N - gn);
  const bool bvec = vec_ok(d.B, d.ldb);
  float acc[MM][4];
#pragma unroll
  for (int m = 0; m < MM; ++m) acc[m][0] = acc[m][1] = acc[m][2] = acc[m][3] = 0.f;
  if (valid > 0) {
    // rows warp, warp + 8, ... in order; four B rows in flight at a time
    int kk = warp;
    for (; kk + 24 < klen; kk += 32) {
      float4 b[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = ld4(d.B + (k0 + kk + 8 * j) * d.ldb + gn, bvec, valid);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int m = 0; m < MM; ++m) {
          const float a = As[(kk + 8 * j) * MM + m];
          acc[m][0] = fmaf(a, b[j].x, acc[m][0]);
          acc[m][1] = fmaf(a, b[j].y, acc[m][1]);
          acc[m][2] = fmaf(a, b[j].z, acc[m][2]);
          acc[m][3] = fmaf(a, b[j].w, acc[m][3]);
        }
      }
    }
    for (; kk < klen; kk += 8) {
      const float4 b = ld4(d.B + (k0 + kk) * d.ldb + gn, bvec, valid);
#pragma unroll
      for (int m = 0; m < MM; ++m) {
        const float a = As[kk * MM + m];
        acc[m][0] = fmaf(a, b.x, acc[m][0]);
        acc[m][1] = fmaf(a, b.y, acc[m][1]);
        acc[m][2] = fmaf(a, b.z, acc[m][2]);
        acc[m][3] = fmaf(a, b.w, acc[m][3]);
      }
    }
  }
#pragma unroll
  for (int m = 0; m < MM; ++m)
    *reinterpret_cast<float4 *>(&red[(warp * MM + m) * 128 + lane * 4]) =
        make_float4(acc[m][0], acc[m][1], acc[m][2], acc[m][3]);
  __syncthreads();
  // fixed-order combination of the 8 warps, then one partial per block
  float *out = part + (int64_t)blockIdx.y * d.M * d.N;
  for (int e = threadIdx.x; e < MM * 128; e += 256) {
    const int m = e / 128, c = e % 128;
    const int64_t n = (int64_t)blockIdx.x * 128 + c;
    float s = red[m * 128 + c];
#pragma unroll
    for (int w = 1; w < 8; ++w) s += red[(w * MM + m) * 128 + c];
    if (m < d.M && n < d.N) out[(int64_t)m * d.N + n] = s;
  }
}

template <int NN>
int launch_small_n(tx_ctx *ctx, const tx_gemm_desc &d) {
  // K chunk per block: the whole K when it fits 64 KB of shared memory
  int64_t kc = (d.K + 127) / 128 * 128;
  if (kc > SN_KC) kc = SN_KC;
  const int64_t splits = (d.K + kc - 1) / kc;
  if (splits > 65535) return TX_ERR_UNSUPPORTED;
  const size_t smem = (size_t)NN * kc * sizeof(float);
  static bool configured[64] = {};
  if (!configured[ctx->device & 63]) {
    TX_CUDA(ctx, cudaFuncSetAttribute(k_gemm_small_n<NN>, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024));
    configured[ctx->device & 63] = true;
  }
  // two blocks per SM: each stages op(B) once and walks many row pairs
  int64_t rows_blocks = (d.M + 15) / 16;
  int64_t cap = 2 * (int64_t)ctx->num_sms / splits;
  if (cap < 1) cap = 1;
  if (rows_blocks > cap) rows_blocks = cap;
  dim3 grid((unsigned)rows_blocks, (unsigned)splits);
  if (splits == 1) {
    k_gemm_small_n<NN><<<grid, 256, smem, ctx->stream>>>(d, (int)kc, nullptr);
    TX_LAUNCHED(ctx, "k_gemm_small_n");
    return TX_OK;
  }
  Scratch part(ctx, (size_t)splits * d.M * d.N * sizeof(float));
  if (!part.ptr) return TX_ERR_OOM;
  k_gemm_small_n<NN><<<grid, 256, smem, ctx->stream>>>(d, (int)kc, part.as<float>());
  TX_LAUNCHED(ctx, "k_gemm_small_n(split)");
  return gemm_split_reduce(ctx, d, part.as<float>(), (int)splits);
}

template <int MM>
int launch_small_m(tx_ctx *ctx, const tx_gemm_desc &d) {
  const int64_t col_blocks = (d.N + 127) / 128;
  if (col_blocks > 65535) return TX_ERR_UNSUPPORTED;
  // about two blocks per SM, at least 64 K rows (8 per warp) per block
  int64_t splits = (2 * (int64_t)ctx->num_sms + col_blocks - 1) / col_blocks;
  int64_t most = (d.K + 63) / 64;
  if (splits > most) splits = most;
  if (splits > 256) splits = 256;
  if (splits < 1) splits = 1;
  int64_t kc = (d.K + splits - 1) / splits;
  kc = (kc + 7) / 8 * 8;
  const int64_t kc_max = (kSmallMSmem / 4 - 8 * MM * 128) / MM;
  if (kc > kc_max) kc = kc_max / 8 * 8;
  splits = (d.K + kc - 1) / kc;
  if (splits > 65535) return TX_ERR_UNSUPPORTED;
  const size_t smem = ((size_t)kc * MM + 8 * MM * 128) * sizeof(float);
  static bool configured[64] = {};
  if (!configured[ctx->device & 63]) {
    TX_CUDA(ctx, cudaFuncSetAttribute(k_gemm_small_m<MM>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmallMSmem));
    configured[ctx->device & 63] = true;
  }
  Scratch part(ctx, (size_t)splits * d.M * d.N * sizeof(float));
  if (!part.ptr) return TX_ERR_OOM;
  dim3 grid((unsigned)col_blocks, (unsigned)splits);
  k_gemm_small_m<MM><<<grid, 256, smem, ctx->stream>>>(d, (int)kc, part.as<float>());
  TX_LAUNCHED(ctx, "k_gemm_small_m");
  return gemm_split_reduce(ctx, d, part.as<float>(), (int)splits);
}

template <int TCOLS, int ACT, int DACT>
int launch_small_k2(tx_ctx *ctx, const tx_gemm_desc &d, int64_t batch, FusedSum *fs) {
  constexpr int ROWS = (256 / (TCOLS / 4)) * 8;
  const int64_t col_tiles = (d.N + TCOLS - 1) / TCOLS, row_tiles = (d.M + ROWS - 1) / ROWS;
  int64_t gy = 3 * (int64_t)ctx->num_sms / (col_tiles * batch);
  if (gy < 1) gy = 1;
  if (gy > row_tiles) gy = row_tiles;
  if (col_tiles > 0x7fffffff || gy > 65535 || row_tiles > 0x7fffffff) return TX_ERR_UNSUPPORTED;
  dim3 grid((unsigned)col_tiles, (unsigned)gy, (unsigned)batch);
  float *col_part = nullptr;
  if (fs && batch == 1) {
    col_part = fs->part;  // row_tiles <= ceil(M / 32) partial rows
    fs->rows = row_tiles;
    fs->fused = true;
  }
  k_gemm_small_k2<TCOLS, ACT, DACT><<<grid, 256, 0, ctx->stream>>>(d, (int)row_tiles, col_part);
  TX_LAUNCHED(ctx, "k_gemm_small_k2");
  return TX_OK;
}

template <int TCOLS>
int launch_small_k2_act(tx_ctx *ctx, const tx_gemm_desc &d, int64_t batch, FusedSum *fs) {
  if (!d.dact) {
    switch (d.act) {
      case TX_ACT_RELU: return launch_small_k2<TCOLS, TX_ACT_RELU, TX_ACT_NONE>(ctx, d, batch, fs);
      case TX_ACT_TANH: return launch_small_k2<TCOLS, TX_ACT_TANH, TX_ACT_NONE>(ctx, d, batch, fs);
      case TX_ACT_GELU: return launch_small_k2<TCOLS, TX_ACT_GELU, TX_ACT_NONE>(ctx, d, batch, fs);
      default: return launch_small_k2<TCOLS, TX_ACT_NONE, TX_ACT_NONE>(ctx, d, batch, fs);
    }
  }
  if (d.act != TX_ACT_NONE) return TX_ERR_UNSUPPORTED;
  switch (d.dact) {
    case TX_ACT_RELU: return launch_small_k2<TCOLS, TX_ACT_NONE, TX_ACT_RELU>(ctx, d, batch, fs);
    case TX_ACT_TANH: return launch_small_k2<TCOLS, TX_ACT_NONE, TX_ACT_TANH>(ctx, d, batch, fs);
    default: return launch_small_k2<TCOLS, TX_ACT_NONE, TX_ACT_GELU>(ctx, d, batch, fs);
  }
}

bool small_k2_ok(const tx_gemm_desc &d, int64_t batch) {
  if (d.N % 4 || !vec_ok(d.C, d.ldc)) return false;
  if (d.dact && !vec_ok(d.dact_src, d.ld_dact)) return false;
  if (d.preact && !vec_ok(d.preact, d.ld_preact)) return false;
  if (batch > 1 && (d.stride_c % 4)) return false;
  return true;
}

template <int TCOLS>
int launch_small_k(tx_ctx *ctx, const tx_gemm_desc &desc, int64_t batch, FusedSum *fs) {
  constexpr int ROWS = (256 / (TCOLS / 4)) * 8;
  if (small_k2_ok(desc, batch)) {
    const int rc = launch_small_k2_act<TCOLS>(ctx, desc, batch, fs);
    if (rc != TX_ERR_UNSUPPORTED) return rc;
  }
  tx_gemm_desc d = desc;
  if (fs) d.flags &= ~TX_GEMM_ROUND_OUT;  // no fused sums here: C stays exact for the caller
  dim3 grid((unsigned)((d.N + TCOLS - 1) / TCOLS), (unsigned)((d.M + ROWS - 1) / ROWS), (unsigned)batch);
  if ((d.N + TCOLS - 1) / TCOLS > 0x7fffffff || (d.M + ROWS - 1) / ROWS > 65535)
    return TX_ERR_UNSUPPORTED;
  k_gemm_small_k<TCOLS><<<grid, 256, 0, ctx->stream>>>(d);
  TX_LAUNCHED(ctx, "k_gemm_small_k");
  return TX_OK;
}

}  // namespace

// Whether gemm_skinny takes a batch-1 product without fused column sums
// (the short-K rule aside, which it only narrows).
bool skinny_shape(const tx_gemm_desc &d) {
  if (d.K <= 0 || d.batch > 1) return false;
  if (d.K <= SK_KMAX) return true;
  return (d.N <= 16 && !d.trans_a) || (d.M <= 16 && !d.trans_b && d.N >= 64);
}

// Route the skinny shapes; TX_ERR_UNSUPPORTED leaves the shape to the
// tensor-core / SIMT kernels.
int gemm_skinny(tx_ctx *ctx, const tx_gemm_desc &desc, FusedSum *fs) {
  const int64_t batch = desc.batch > 1 ? desc.batch : 1;
  if (desc.K <= 0 || batch > 65535) return TX_ERR_UNSUPPORTED;
  // A short-K product with a large output whose operands are already TF32
  // values (a first convolution over im2col columns) runs on the tensor core
  // (persistent, no operand conversion) instead: its output dominates.
  if (desc.K <= SK_KMAX && desc.K >= 16 && batch == 1 && !fs && desc.M >= 65536 && desc.N >= 32 &&
      (desc.flags & TX_GEMM_A_TF32) && (desc.flags & TX_GEMM_B_TF32))
    return TX_ERR_UNSUPPORTED;
  if (desc.K <= SK_KMAX) {
    if (desc.N <= 32) return launch_small_k<32>(ctx, desc, batch, fs);
    if (desc.N <= 64) return launch_small_k<64>(ctx, desc, batch, fs);
    if (desc.N <= 128) return launch_small_k<128>(ctx, desc, batch, fs);
    return launch_small_k<256>(ctx, desc, batch, fs);
  }
  tx_gemm_desc d = desc;
  if (fs) d.flags &= ~TX_GEMM_ROUND_OUT;  // the remaining kernels do not sum columns
  if (batch != 1) return TX_ERR_UNSUPPORTED;
  if (d.N <= 16 && !d.trans_a) {
    if (d.N <= 2) return launch_small_n<2>(ctx, d);
    if (d.N <= 4) return launch_small_n<4>(ctx, d);
    if (d.N <= 8) return launch_small_n<8>(ctx, d);
    if (d.N <= 10) return launch_small_n<10>(ctx, d);
    return launch_small_n<16>(ctx, d);
  }
  if (d.M <= 16 && !d.trans_b && d.N >= 64) {
    if (d.M <= 2) return launch_small_m<2>(ctx, d);
    if (d.M <= 4) return launch_small_m<4>(ctx, d);
    if (d.M <= 8) return launch_small_m<8>(ctx, d);
    return launch_small_m<16>(ctx, d);
  }
  return TX_ERR_UNSUPPORTED;
}
