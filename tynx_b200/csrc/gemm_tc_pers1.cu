// Instantiations of the persistent tcgen05 contraction that rounds its
// operands to TF32 in shared memory.
#define TX_TC_PERSISTENT_TU
#include "gemm_tc_kern.cuh"

int tx_tc::launch_persistent_round(tx_ctx *ctx, int bn, const tx_gemm_desc &d, const Maps &m, int64_t z,
                                   int kb_per) {
  return launch_persistent_impl<1>(ctx, bn, d, m, z, kb_per, 0);
}
