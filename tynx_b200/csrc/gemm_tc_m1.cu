// Instantiations of the one-tile tcgen05 contraction for operand mode 1.
#include "gemm_tc_kern.cuh"

int tx_tc::launch_mode1(tx_ctx *ctx, int bn, const tx_gemm_desc &d, const Maps &m, int64_t z,
                          int kb_per_cta) {
  return launch_mode<1>(ctx, bn, d, m, z, kb_per_cta);
}
