// Instantiations of the persistent tcgen05 contraction that splits its
// operands into TF32 big and small halves in shared memory (3xTF32).
#define TX_TC_PERSISTENT_TU
#include "gemm_tc_kern.cuh"

int tx_tc::launch_persistent_split(tx_ctx *ctx, int bn, const tx_gemm_desc &d, const Maps &m, int64_t z,
                                   int kb_per) {
  return launch_persistent_impl<2>(ctx, bn, d, m, z, kb_per, 0);
}
