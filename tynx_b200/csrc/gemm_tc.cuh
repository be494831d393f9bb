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

// Implicit-GEMM convolution operands: tiles cut from a channels-last
// [n][h][w][c] fp32 tensor by shifted 4-D TMA boxes (element strides along w
// and h for a strided convolution) instead of read from a dense matrix, so
// the im2col columns never exist in HBM.  The GEMM's k-block kb reads tap
// kb / cblocks and channels (kb % cblocks) * 32 .. + 31 of that tap; a pixel p
// of the output grid is (n, oh, ow) = (p / ohw, (p % ohw) / ow, p % ow) and its
// box starts at (ow * sw + offx[tap], oh * sh + offy[tap], n).
constexpr int kGatherTaps = 64;
struct GatherOp {
  int a;        // 1: A's 128-row K-major tiles are boxes of 128 pixels
  int b;        // 1: B's MN-major 32 x 32 sub-tiles are boxes of 32 pixels (K = pixels,
                //    column group g = tap g / cblocks, channel block g % cblocks);
                // 2: B is K-major with the k-block's rows at wtap[tap] * brows + n0
  int cblocks;  // 32-channel blocks per tap
  int ntaps;
  int ohw, ow;  // output pixels per image and per row
  int sw, sh;   // box start step per output column / row
  int brows;    // b == 2: weight rows per tap
  int wsplit;   // > 0: the output-side maps are 3-D [rows][wsplit][N] views and
                //      output row y sits at (y % wsplit, y / wsplit)
  int16_t offx[kGatherTaps], offy[kGatherTaps], wtap[kGatherTaps];
  // dense MN-major operands (not gathered): 1 when the map is 4-D {32, K,
  // MN / 32, batch} and a tile's 32-column blocks come in one box instead of
  // one box each (the MN extent a multiple of 32)
  int amn, bmn;
  int ashared;  // 1: A is one matrix for every batch entry (loaded at batch 0)
};

// Tensor maps of one launch: the operands, and for the TMA epilogue the
// output (also the beta * C input), the act' source and the pre-activation.
struct Maps {
  CUtensorMap a, b, c, s, p;
  CUtensorMap b2;  // the TF32 tail of B (tx_gemm_desc.B_lo), persistent kernel only
  int tma_epi = 0;
  int conv_mask = 3;  // MODE 1: operands to round in shared memory (bit 0 A, bit 1 B)
  float *col_part = nullptr;  // fused column sums, TMA epilogue only
  GatherOp g;                 // gathered operands (all zero: dense operands)
};

// A channels-last activation tensor that a gathered operand is cut from.
struct ConvTensor {
  const float *base;
  int64_t n, h, w, c;
};

// An implicit-GEMM convolution product for gemm_conv_tc: the gather, the
// tensor it reads, the box (elements along c, w, h, n before the element
// strides) and, for a K-major weight operand read by tap (op.b == 2), the
// weight matrix's extents; for op.wsplit > 0 the output view's extents.
struct ConvGemm {
  GatherOp op;
  ConvTensor src;
  uint32_t box[4];
  uint32_t estr_w, estr_h;
  int64_t b_inner, b_rows;          // op.b == 2: B is [b_rows][b_inner] with row stride ldb
  int64_t out_rows, out_sw, out_sr; // op.wsplit > 0: [out_rows][wsplit][N] with element strides
                                    // out_sw (w) and out_sr (rows); the act' source and beta * C alike
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
// persistent with operand conversion in shared memory: TF32 rounding of the
// operands m.conv_mask selects (gemm_tc_pers1.cu), or the 3xTF32 split of
// both, tiles at most 128 wide (gemm_tc_pers2.cu)
int launch_persistent_round(tx_ctx *ctx, int bn, const tx_gemm_desc &d, const Maps &m, int64_t z, int kb_per);
int launch_persistent_split(tx_ctx *ctx, int bn, const tx_gemm_desc &d, const Maps &m, int64_t z, int kb_per);

}  // namespace tx_tc

// The tcgen05 product of d with gathered operands (gemm_tc.cu).  mode as for
// gemm_tcgen05; TX_ERR_UNSUPPORTED when a tensor map or a tile rule does not
// fit, and the caller takes the explicit columns instead.
int gemm_conv_tc(tx_ctx *ctx, const tx_gemm_desc &d, int mode, const tx_tc::ConvGemm &cv);

namespace tx_tc {

}  // namespace tx_tc
