// Activation and activation-derivative math shared by every GEMM epilogue, so
// the fused forward (Gemm -> Relu/Tanh/Gelu) and the fused dgrad (dY * act')
// give the same bits whichever kernel a shape lands on.
//
// Relu / Tanh / exact-erf GELU follow the reference's unary ops
// (crates/tynx/src/tensor.rs:2002, 2012, 2229; the ONNX `approximate`
// attribute is not consulted there either).  Derivatives are taken from the
// saved tensor: Relu and Tanh use the forward output y (mask y > 0; 1 - y^2),
// GELU uses the pre-activation x (Phi(x) + x phi(x)).
#pragma once

#include <math.h>
#include <stdint.h>

#include "tynx_cuda.h"

namespace tx_epi {

// The normal CDF Phi(x) = (1 + erf(x / sqrt 2)) / 2 and the density phi(x)
// from one exponential.  erfc(z), z = |x| / sqrt 2 >= 0, follows Hastings'
// rational approximation as tabulated in Abramowitz and Stegun, Handbook of
// Mathematical Functions, formula 7.1.26: erfc(z) = t P(t) exp(-z^2) with
// t = 1 / (1 + p z) and P of degree 4, |error| <= 1.5e-7 on erf; exp(-z^2) =
// exp(-x^2 / 2) is also phi's exponential.  With the hardware reciprocal and
// exponential Phi and GELU' stay within ~2e-7 absolute of float64 (the test
// checks them); the GELU epilogues issue about half the instructions of an
// erff / expf pair.
__device__ __forceinline__ void norm_cdf_pdf(float x, float &cdf, float &pdf) {
  const float z = fabsf(x) * 0.70710678118654752f;
  const float t = __fdividef(1.0f, fmaf(0.3275911f, z, 1.0f));
  const float e = __expf(-0.5f * x * x);
  const float poly =
      t * fmaf(t, fmaf(t, fmaf(t, fmaf(t, 1.061405429f, -1.453152027f), 1.421413741f), -0.284496736f), 0.254829592f);
  const float half_erfc = 0.5f * poly * e;
  cdf = x >= 0.f ? 1.0f - half_erfc : half_erfc;
  pdf = e * 0.39894228040143268f;
}

__device__ __forceinline__ float gelu(float x) {
  float cdf, pdf;
  norm_cdf_pdf(x, cdf, pdf);
  return x * cdf;
}

__device__ __forceinline__ float gelu_grad(float x) {
  float cdf, pdf;
  norm_cdf_pdf(x, cdf, pdf);
  return fmaf(x, pdf, cdf);
}

__device__ __forceinline__ float act(int a, float v) {
  switch (a) {
    case TX_ACT_RELU: return v > 0.f ? v : 0.f;
    case TX_ACT_TANH: return tanhf(v);
    case TX_ACT_GELU: return gelu(v);
  }
  return v;
}

__device__ __forceinline__ float dact(int a, float s) {
  switch (a) {
    case TX_ACT_RELU: return s > 0.f ? 1.f : 0.f;
    case TX_ACT_TANH: return 1.f - s * s;
    case TX_ACT_GELU: return gelu_grad(s);
  }
  return 1.f;
}

// Round to TF32 (10-bit mantissa), to nearest with ties away from zero: the
// rounding the tensor-core path applies to its operands, used to store a
// result that only feeds further TF32 contractions.
__device__ __forceinline__ float round_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// Column sums of a 32 x 32 chunk held one row per lane (v[j] = column j):
// a reduce-scatter in five shuffle rounds (16 + 8 + 4 + 2 + 1 exchanges),
// after which lane l holds the sum of column l over the 32 rows.  The order of
// the additions is fixed, so the result is deterministic.
__device__ __forceinline__ float colsum32(float (&w)[32], int lane) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < o; ++i) {
      const float send = up ? w[i] : w[i + o];
      const float keep = up ? w[i + o] : w[i];
      w[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  return w[0];
}

}  // namespace tx_epi
