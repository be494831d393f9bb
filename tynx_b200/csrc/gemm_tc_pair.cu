// Instantiations of the CTA-pair tcgen05 contraction (256-row x 256-column tiles on two SMs).
#define TX_TC_PAIR_TU
#include "gemm_tc_kern.cuh"

int tx_tc::launch_pair(tx_ctx *ctx, const tx_gemm_desc &d, const Maps &m, int64_t z, int kb_per_cta) {
  return launch_pair_impl(ctx, d, m, z, kb_per_cta);
}
