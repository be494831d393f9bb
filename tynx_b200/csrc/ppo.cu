// Fused clipped-surrogate PPO objective, forward and backward.
//
// The reference composes it from about twenty taped operations
// (crates/tynx-python/tests/test_ppo.py:53-64 with Categorical from
// crates/tynx-python/python/tynx/distributions.py:47-104 and mse_loss from
// crates/tynx-python/python/tynx/nn/functional.py:126-130):
//
//   logp    = log_softmax(logits)                 per row, over the classes
//   ratio   = exp(logp[action] - old_log_prob)
//   surr    = min(ratio * adv, clamp(ratio, 1 - clip, 1 + clip) * adv)
//   entropy = -sum_j exp(logp_j) * logp_j
//   loss    = -mean(surr) + value_coef * mean((value - ret)^2) - entropy_coef * mean(entropy)
//
// Here one thread owns one row (the class count is small: 16 for the PPO
// actor-critic): the forward computes the row's three terms and one block
// sum per term, a one-block kernel adds the block sums in a fixed order; the
// backward writes d logits and d value per row from the same row quantities
// and the upstream scalar gradient.  The gradient follows the composed
// operations: min sends the gradient to the first argument when surr1 <=
// surr2, clamp passes it inside [1 - clip, 1 + clip], and d logp feeds the
// log-softmax backward dz = dlogp - p * sum(dlogp).
#include <cmath>

#include "common.h"

namespace {

constexpr int kMaxCols = 64;
constexpr int kThreads = 256;

// log-softmax of a row as the reference computes it: shifted by the max,
// minus log(sum(exp(shifted))); MAXC bounds the class count at compile time
// so that the row stays in registers
template <int MAXC>
__device__ __forceinline__ void row_log_softmax(const float *z, int cols, float *logp) {
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < MAXC; ++j)
    if (j < cols) m = fmaxf(m, z[j]);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < MAXC; ++j)
    if (j < cols) s += expf(z[j] - m);
  const float lse = logf(s);
#pragma unroll
  for (int j = 0; j < MAXC; ++j) logp[j] = j < cols ? (z[j] - m) - lse : 0.f;
}

template <int MAXC>
__global__ void k_ppo_fwd(const float *__restrict__ logits, int64_t rows, int cols,
                          const float *__restrict__ values, const int64_t *__restrict__ actions,
                          const float *__restrict__ old_logp, const float *__restrict__ adv,
                          const float *__restrict__ ret, float lo, float hi, float *__restrict__ part,
                          int *err) {
  __shared__ float sh[3][kThreads / 32];
  float s_surr = 0.f, s_sq = 0.f, s_ent = 0.f;
  for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < rows; r += (int64_t)gridDim.x * blockDim.x) {
    float z[MAXC], logp[MAXC];
#pragma unroll
    for (int j = 0; j < MAXC; ++j) z[j] = j < cols ? logits[r * cols + j] : 0.f;
    row_log_softmax<MAXC>(z, cols, logp);
    int64_t a = actions[r];
    if (a < 0) a += cols;  // negative indices count from the end (normalize_indices)
    if (a < 0 || a >= cols) {
      atomicCAS(err, 0, DEVERR_INDEX);
      continue;
    }
    float lp = 0.f, ent = 0.f;
#pragma unroll
    for (int j = 0; j < MAXC; ++j) {
      if (j == a) lp = logp[j];
      if (j < cols) ent += expf(logp[j]) * logp[j];
    }
    const float ratio = expf(lp - old_logp[r]);
    const float A = adv[r];
    const float s1 = ratio * A, s2 = fminf(fmaxf(ratio, lo), hi) * A;
    s_surr += s1 <= s2 ? s1 : s2;
    const float e = values[r] - ret[r];
    s_sq += e * e;
    s_ent += -ent;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int o = 16; o > 0; o >>= 1) {
    s_surr += __shfl_xor_sync(0xffffffffu, s_surr, o);
    s_sq += __shfl_xor_sync(0xffffffffu, s_sq, o);
    s_ent += __shfl_xor_sync(0xffffffffu, s_ent, o);
  }
  if (lane == 0) {
    sh[0][warp] = s_surr;
    sh[1][warp] = s_sq;
    sh[2][warp] = s_ent;
  }
  __syncthreads();
  if (threadIdx.x < 3) {
    float t = 0.f;
    for (int w = 0; w < kThreads / 32; ++w) t += sh[threadIdx.x][w];
    part[blockIdx.x * 3 + threadIdx.x] = t;
  }
}

// loss = -(sum surr)/B + value_coef * (sum sq)/B - entropy_coef * (sum ent)/B, block sums in order
__global__ void k_ppo_finish(const float *__restrict__ part, int blocks, float inv_rows, float value_coef,
                             float entropy_coef, float *__restrict__ loss) {
  if (threadIdx.x != 0) return;
  float a = 0.f, b = 0.f, c = 0.f;
  for (int i = 0; i < blocks; ++i) {
    a += part[3 * i];
    b += part[3 * i + 1];
    c += part[3 * i + 2];
  }
  loss[0] = -(a * inv_rows) + (b * inv_rows) * value_coef - (c * inv_rows) * entropy_coef;
}

template <int MAXC>
__global__ void k_ppo_bwd(const float *__restrict__ logits, int64_t rows, int cols,
                          const float *__restrict__ values, const int64_t *__restrict__ actions,
                          const float *__restrict__ old_logp, const float *__restrict__ adv,
                          const float *__restrict__ ret, float lo, float hi, float inv_rows, float value_coef,
                          float entropy_coef, const float *__restrict__ dloss, float *__restrict__ dlogits,
                          float *__restrict__ dvalues, int acc_logits, int acc_values) {
  const float g = dloss[0];
  const float d_surr = -g * inv_rows;          // d loss / d surr_r
  const float d_ent = -g * entropy_coef * inv_rows;  // d loss / d entropy_r
  for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < rows; r += (int64_t)gridDim.x * blockDim.x) {
    float z[MAXC], logp[MAXC];
#pragma unroll
    for (int j = 0; j < MAXC; ++j) z[j] = j < cols ? logits[r * cols + j] : 0.f;
    row_log_softmax<MAXC>(z, cols, logp);
    int64_t a = actions[r];
    if (a < 0) a += cols;
    const bool ok = a >= 0 && a < cols;
    float lp = 0.f;
#pragma unroll
    for (int j = 0; j < MAXC; ++j)
      if (j == a) lp = logp[j];
    const float ratio = expf(lp - old_logp[r]);
    const float A = adv[r];
    const float s1 = ratio * A, s2 = fminf(fmaxf(ratio, lo), hi) * A;
    float dratio;
    if (s1 <= s2) dratio = d_surr * A;
    else dratio = (ratio >= lo && ratio <= hi) ? d_surr * A : 0.f;
    const float dlp = dratio * ratio;
    // d logp_j: the entropy term -sum exp(l) l gives -(p_j l_j + p_j) per unit of entropy
    float dl[MAXC];
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < MAXC; ++j) {
      const float p = expf(logp[j]);
      dl[j] = j < cols ? d_ent * -(p * logp[j] + p) + ((ok && j == a) ? dlp : 0.f) : 0.f;
      sum += dl[j];
    }
#pragma unroll
    for (int j = 0; j < MAXC; ++j) {
      if (j >= cols) continue;
      const float v = dl[j] - expf(logp[j]) * sum;
      float *o = dlogits + r * cols + j;
      *o = acc_logits ? *o + v : v;
    }
    if (dvalues) {
      const float dv = 2.f * (values[r] - ret[r]) * (g * value_coef * inv_rows);
      dvalues[r] = acc_values ? dvalues[r] + dv : dv;
    }
  }
}

unsigned ppo_blocks(int64_t rows) {
  int64_t b = (rows + kThreads - 1) / kThreads;
  return (unsigned)(b < 1 ? 1 : b > 148 * 4 ? 148 * 4 : b);
}

}  // namespace

extern "C" int tx_ppo_loss_fwd(tx_ctx *ctx, const float *logits, int64_t rows, int64_t cols, const float *values,
                               const int64_t *actions, const float *old_log_prob, const float *advantages,
                               const float *returns, float clip, float value_coef, float entropy_coef,
                               float *loss) {
  if (!ctx || rows <= 0 || cols <= 0) return TX_ERR_INVALID;
  if (cols > kMaxCols) return tx_fail(ctx, TX_ERR_UNSUPPORTED, "fused PPO loss: at most 64 classes");
  const unsigned blocks = ppo_blocks(rows);
  Scratch part(ctx, (size_t)blocks * 3 * sizeof(float));
  if (!part.ptr) return TX_ERR_OOM;
  auto fwd = cols <= 16 ? k_ppo_fwd<16> : cols <= 32 ? k_ppo_fwd<32> : k_ppo_fwd<64>;
  fwd<<<blocks, kThreads, 0, ctx->stream>>>(logits, rows, (int)cols, values, actions, old_log_prob, advantages,
                                            returns, 1.f - clip, 1.f + clip, part.as<float>(), ctx->d_err);
  TX_LAUNCHED(ctx, "k_ppo_fwd");
  k_ppo_finish<<<1, 32, 0, ctx->stream>>>(part.as<float>(), (int)blocks, 1.0f / (float)rows, value_coef,
                                          entropy_coef, loss);
  TX_LAUNCHED(ctx, "k_ppo_finish");
  return TX_OK;
}

extern "C" int tx_ppo_loss_bwd(tx_ctx *ctx, const float *logits, int64_t rows, int64_t cols, const float *values,
                               const int64_t *actions, const float *old_log_prob, const float *advantages,
                               const float *returns, float clip, float value_coef, float entropy_coef,
                               const float *dloss, float *dlogits, float *dvalues, int acc_logits,
                               int acc_values) {
  if (!ctx || rows <= 0 || cols <= 0 || !dloss || !dlogits) return TX_ERR_INVALID;
  if (cols > kMaxCols) return tx_fail(ctx, TX_ERR_UNSUPPORTED, "fused PPO loss: at most 64 classes");
  auto bwd = cols <= 16 ? k_ppo_bwd<16> : cols <= 32 ? k_ppo_bwd<32> : k_ppo_bwd<64>;
  bwd<<<ppo_blocks(rows), kThreads, 0, ctx->stream>>>(
      logits, rows, (int)cols, values, actions, old_log_prob, advantages, returns, 1.f - clip, 1.f + clip,
      1.0f / (float)rows, value_coef, entropy_coef, dloss, dlogits, dvalues, acc_logits, acc_values);
  TX_LAUNCHED(ctx, "k_ppo_bwd");
  return TX_OK;
}
