// Shared declarations of the tcgen05 contraction: the tile constants, the
// tensor maps of one launch, and the launch entry points that the kernel
// translation units define (one per operand mode, the CTA pair and the
// persistent variant, so that they compile in parallel).
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.h"

namespace tx_tc {

constexpr int TC_BM = 128;
constexpr int TC_BK = 32;  // fp32 elements per 128-byte swizzle row

// Tensor maps of one launch: the operands, and for the TMA epilogue the
// output (also the beta * C input), the act' source and the pre-activation.
struct Maps {
  CUtensorMap a, b, c, s, p;
  CUtensorMap b2;  // the TF32 tail of B (tx_gemm_desc.B_lo), persistent kernel only
  int tma_epi = 0;
  int conv_mask = 3;  // MODE 1: operands to round in shared memory (bit 0 A, bit 1 B)
  float *col_part = nullptr;  // fused column sums, TMA epilogue only
};

// One-tile kernel, operand mode 0 / 1 / 2 (gemm_tc_m0.cu, gemm_tc_m1.cu,
// gemm_tc_m2.cu).  `z` = batch count, or the number of K splits when
// kb_per_cta > 0.
int launch_mode0(tx_ctx *ctx, int bn, const tx_gemm_desc &d, const Maps &m, int64_t z, int kb_per_cta);
int launch_mode1(tx_ctx *ctx, int bn, const tx_gemm_desc &d, const Maps &m, int64_t z, int kb_per_cta);
int launch_mode2(tx_ctx *ctx, int bn, const tx_gemm_desc &d, const Maps &m, int64_t z, int kb_per_cta);
// CTA pairs, BN = 256, mode 0 (gemm_tc_pair.cu)
int launch_pair(tx_ctx *ctx, const tx_gemm_desc &d, const Maps &m, int64_t z, int kb_per_cta);
// persistent, mode 0 (gemm_tc_pers.cu); TX_ERR_UNSUPPORTED when the stages
// would not fit next to the epilogue's tiles
int launch_persistent(tx_ctx *ctx, int bn, const tx_gemm_desc &d, const Maps &m, int64_t z, int kb_per,
                      int max_grid = 0);

}  // namespace tx_tc
