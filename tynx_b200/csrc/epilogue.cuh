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

__device__ __forceinline__ float act(int a, float v) {
  switch (a) {
    case TX_ACT_RELU: return v > 0.f ? v : 0.f;
    case TX_ACT_TANH: return tanhf(v);
    case TX_ACT_GELU: return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
  }
  return v;
}

__device__ __forceinline__ float dact(int a, float s) {
  switch (a) {
    case TX_ACT_RELU: return s > 0.f ? 1.f : 0.f;
    case TX_ACT_TANH: return 1.f - s * s;
    case TX_ACT_GELU: {
      float cdf = 0.5f * (1.0f + erff(s * 0.70710678118654752f));
      return cdf + s * expf(-0.5f * s * s) * 0.39894228040143268f;
    }
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
