// Instantiations of the persistent tcgen05 contraction without operand
// conversion (operands used as loaded).
#define TX_TC_PERSISTENT_TU
#include "gemm_tc_kern.cuh"

int tx_tc::launch_persistent(tx_ctx *ctx, int bn, const tx_gemm_desc &d, const Maps &m, int64_t z,
                             int kb_per, int max_grid) {
  return launch_persistent_impl<0>(ctx, bn, d, m, z, kb_per, max_grid);
}
