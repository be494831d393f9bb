#pragma once
// tcgen05 / TMEM / TMA fp32 contraction for sm_100a (kind::tf32).
//
// One CTA computes a 128 x BN tile of C.  Warp roles (320 threads in the
// one-tile kernel, 192 or 320 in the persistent one):
//   warp 0      TMA producer: loads 128x32 A and BNx32 B fp32 tiles per stage
//               into a STAGES-deep shared-memory ring;
//   warp 1      allocates TMEM (BN fp32 columns x 128 lanes) and, from one
//               thread, issues tcgen05.mma.kind::tf32 (K = 8 per instruction,
//               4 per stage), committing each stage back to the producer;
//   warps 2..5  operand conversion during the main loop (see MODE);
//   warps 2..9  the epilogue, two warps per TMEM lane quadrant (warps 2..5 in
//               the persistent kernel unless its epilogue is a GELU or GELU'):
//               tcgen05.ld the accumulator, apply
//               alpha / bias / beta*C / activation / act', and store each
//               32x32 chunk through swizzled shared memory by TMA.
// MODE selects how fp32 operands become TF32:
//   0  raw: the tensor core reads fp32 and drops the 13 low mantissa bits
//      (truncation, biased toward zero);
//   1  round to nearest: warps 2..5 round each landed stage in place
//      (cvt.rna.tf32) before the MMA consumes it (unbiased; ~2^-11 relative);
//   2  3xTF32: each operand is split into big = rna(x) and small = rna(x - big)
//      and C += A_big B_big + A_big B_small + A_small B_big (fp32-class accuracy).
// Operands may be K-major or MN-major on either side, so the forward (X W^T),
// dgrad (dY W) and wgrad (dY^T X) products of a Gemm map onto the same kernel
// without transposes.  No TMA multicast is used anywhere.
//
// Every mbarrier wait is bounded (~2 s of %globaltimer).  On expiry the CTA
// raises the context's device error flag, stops issuing work, lets every role
// reach the final barrier (no named barriers that an early exit could strand),
// frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>

#include <cstring>

#include "epilogue.cuh"
#include "gemm_tc.cuh"


namespace {

using tx_tc::Maps;
using tx_tc::TC_BK;
using tx_tc::TC_BM;

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s
constexpr int kConvThreads = 128;                 // warps 2..5

// PAIR: a cluster of two CTAs (an SM pair) computes a 256 x BN tile with
// cta_group::2 MMAs; each CTA stages its own 128 rows of A and half of B's BN
// rows, and the MMA reads B from both, so every SM streams 128 x 32 + BN/2 x 32
// operand floats per k-block instead of 128 x 32 + BN x 32.
template <int BN, int MODE, bool PAIR = false>
struct TcCfg {
  static constexpr int A_BYTES = TC_BM * TC_BK * 4;
  static constexpr int B_BYTES = (PAIR ? BN / 2 : BN) * TC_BK * 4;
  // 3xTF32 keeps the small halves of both operands next to the big ones
  static constexpr int STAGE = (A_BYTES + B_BYTES) * (MODE == 2 ? 2 : 1);
  static constexpr int STAGES = (196 * 1024 / STAGE) > 8 ? 8 : (196 * 1024 / STAGE);
  // barriers, TMEM address and abort flag in the first 1 KB, then each of the
  // eight epilogue warps' copy of the tile's BN bias values
  static constexpr int TAIL = 1024 + 8 * BN * 4;
  static constexpr int SMEM = STAGES * STAGE + 1024 /*align*/ + TAIL;
  // The TMA epilogue reuses the drained stages: 48 tiles of 32 x 32 fp32,
  // six per warp when eight warps share the epilogue (two output tiles and
  // two each of the pre-activation, act'-source and C tiles in use), eight
  // per warp when four do.
  static_assert(STAGES * STAGE >= 48 * 4096, "epilogue tiles must fit in the stage memory");
  // The tensor core adds each MMA's products into the fp32 TMEM accumulator
  // with a biased (toward zero) rounding, so the error grows with the number
  // of MMAs in one chain.  k-blocks are dealt round-robin to NACC accumulators
  // (BN columns each, within the 512 TMEM columns) that the epilogue sums with
  // IEEE fp32 adds.
  static constexpr int NACC = MODE == 2 ? (512 / BN > 4 ? 4 : 512 / BN) : (512 / BN >= 2 ? 2 : 1);
  static constexpr int TMEM_COLS = BN * NACC;
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait.  Returns false (and raises the flags) when the limit expires
// or another role of the CTA has already given up.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag,
                                          int *err, int site) {
  if (mbar_try(bar, parity)) return true;
  uint64_t start = global_ns();
  while (true) {
    if (mbar_try(bar, parity)) return true;
    if (*abort_flag) return false;
    if (global_ns() - start > kWaitLimitNs) {
      *abort_flag = 1;
      if (atomicCAS(err, 0, DEVERR_TIMEOUT) == 0) err[1] = site;
      return false;
    }
  }
}

// Wait for a phase regardless of the abort flag (a copy in flight must land
// before its shared memory is released), still bounded in time.
__device__ __forceinline__ void mbar_drain(uint64_t *bar, uint32_t parity) {
  const uint64_t start = global_ns();
  while (!mbar_try(bar, parity) && global_ns() - start < kWaitLimitNs) {
  }
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, uint64_t *bar,
                                            int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap *map, uint64_t *bar, int c,
                                            int x, int y, int n) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(map), "r"(smem_u32(bar)), "r"(c), "r"(x), "r"(y), "r"(n)
      : "memory");
}

// An MN-major operand tile of nblk 32-column blocks (4 KB each, consecutive in
// shared memory) starting at column c0: one box of a 4-D map when `merged`,
// else one 3-D box per block.  TMA issue is serial per SM, so fewer boxes keep
// the producer ahead.
__device__ __forceinline__ void load_mn(uint32_t dst, const CUtensorMap *map, uint64_t *bar, int merged, int nblk,
                                        int c0, int k0, int z) {
  if (merged) {
    tma_load_4d(dst, map, bar, 0, k0, c0 / 32, z);
  } else {
#pragma unroll 1
    for (int j = 0; j < nblk; ++j) tma_load_3d(dst + j * 4096, map, bar, c0 + 32 * j, k0, z);
  }
}

// The box of the pixels from p of an implicit-GEMM operand (GatherOp), tap t,
// channel block cb.  Boxes that start outside the tensor read zeros there: the
// convolution's padding.
__device__ __forceinline__ void gather_box(uint32_t dst, const CUtensorMap *map, uint64_t *bar,
                                           const tx_tc::GatherOp &g, int64_t p, int t, int cb) {
  const int64_t n = p / g.ohw;
  const int r = (int)(p - n * g.ohw);
  const int oh = r / g.ow, ow = r - oh * g.ow;
  tma_load_4d(dst, map, bar, cb * 32, ow * g.sw + g.offx[t], oh * g.sh + g.offy[t], (int)n);
}

// Bytes of B one k-block brings: a gathered weight-gradient operand has no
// sub-tile past the last column group (those columns are never stored).
template <int BN>
__device__ __forceinline__ uint32_t gather_b_bytes(const tx_tc::GatherOp &g, int n0) {
  if (g.b != 1) return BN * TC_BK * 4;
  int groups = g.ntaps * g.cblocks - n0 / 32;
  groups = groups < 0 ? 0 : groups > BN / 32 ? BN / 32 : groups;
  return (uint32_t)groups * 4096u;
}

// The operand loads of global k-block kg of the tile at (m0, n0) for gathered
// operands (the dense ones are the caller's).
template <int BN>
__device__ __forceinline__ void gather_loads(const tx_tc::GatherOp &g, const CUtensorMap *mapA,
                                             const CUtensorMap *mapB, uint64_t *bar, uint32_t a_dst,
                                             uint32_t b_dst, int m0, int n0, int kg) {
  if (g.a) gather_box(a_dst, mapA, bar, g, m0, kg / g.cblocks, kg % g.cblocks);
  if (g.b == 1) {
    const int groups = g.ntaps * g.cblocks;
#pragma unroll 1
    for (int j = 0; j < BN / 32; ++j) {
      const int grp = n0 / 32 + j;
      if (grp < groups) gather_box(b_dst + j * 4096, mapB, bar, g, (int64_t)kg * TC_BK, grp / g.cblocks, grp % g.cblocks);
    }
  } else if (g.b == 2) {
    const int t = kg / g.cblocks;
    tma_load_3d(b_dst, mapB, bar, (kg % g.cblocks) * 32, g.wtap[t] * g.brows + n0, 0);
  }
}

// CTA-pair load: the copy lands in this CTA's shared memory and completes
// its bytes on the barrier at `bar_cluster` (a shared::cluster address, the
// leader CTA's barrier for both CTAs of the pair).
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap *map, uint32_t bar_cluster,
                                                 int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(map), "r"(bar_cluster), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d_pair(uint32_t dst, const CUtensorMap *map, uint32_t bar_cluster,
                                                 int c, int x, int y, int n) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(map), "r"(bar_cluster), "r"(c), "r"(x), "r"(y), "r"(n)
      : "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// shared::cluster address of this CTA's variable at `addr` in CTA `rank`
__device__ __forceinline__ uint32_t map_to_rank(uint32_t addr, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(addr), "r"(rank));
  return out;
}

// every thread of both CTAs of the cluster
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, uint32_t src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(map),
               "r"(src), "r"(x), "r"(y), "r"(z)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// A 32 x 32 fp32 tile as TMA writes and reads it with the 128-byte swizzle:
// row r is 128 bytes at r * 128, and its 16-byte chunk j sits at chunk
// j ^ (r & 7).  A thread that owns row r moves the row with 8 float4 accesses;
// the 8 lanes of one shared-memory phase hit 8 different chunks.
__device__ __forceinline__ void tile_row_load(const uint8_t *tile, int r, float (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 t = *reinterpret_cast<const float4 *>(tile + r * 128 + ((j ^ (r & 7)) << 4));
    v[4 * j] = t.x;
    v[4 * j + 1] = t.y;
    v[4 * j + 2] = t.z;
    v[4 * j + 3] = t.w;
  }
}
__device__ __forceinline__ void tile_row_store(uint8_t *tile, int r, const float (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 8; ++j)
    *reinterpret_cast<float4 *>(tile + r * 128 + ((j ^ (r & 7)) << 4)) =
        make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// arrive (once every earlier pair MMA of this thread has completed) on the
// barrier at a shared::cluster address, in either CTA of the pair
__device__ __forceinline__ void tc_commit_pair(uint32_t bar_cluster) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar_cluster)
               : "memory");
}

template <bool PAIR = false>
__device__ __forceinline__ void tc_mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  if (PAIR)
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  else
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ float to_tf32_rn(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// Shared-memory matrix descriptor (sm_100 layout, version 1).  K-major tiles
// use the 128-byte swizzle (layout 2: 8 rows x 128 B atoms); MN-major fp32 tiles
// use the 128-byte swizzle with 32-byte atomicity (layout 1: 4 rows x 128 B
// atoms), the only MN-major layout the tf32 MMA accepts.
constexpr uint32_t kLayoutSW128 = 2;
constexpr uint32_t kLayoutSW128Base32B = 1;

__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo,
                                              uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // version
  d |= (uint64_t)layout << 61;
  return d;
}

// descriptor of the k-th 8-deep slice of a staged operand tile
template <bool MN>
__device__ __forceinline__ uint64_t operand_desc(uint32_t base, int k) {
  // K-major: advance 32 bytes inside the swizzled 128-byte row (SBO = 8 rows).
  // MN-major: 8 K rows (1024 bytes) per instruction, LBO = the 4 KB stride
  // between 32-element MN blocks, SBO = 4 rows.
  return MN ? smem_desc(base + k * 1024, 4096, 512, kLayoutSW128Base32B)
            : smem_desc(base + k * 32, 16, 1024, kLayoutSW128);
}

// tcgen05.ld without the wait: the registers are valid after tmem_wait_ld()
// and reg_fence() (which keeps every use of them behind the wait)
__device__ __forceinline__ void tmem_ld32_issue(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void reg_fence(uint32_t (&r)[32]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
                 "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]),
                 "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]),
                 "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]),
                 "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]),
                 "+r"(r[31]));
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ float act_f(int act, float v) { return tx_epi::act(act, v); }
__device__ __forceinline__ float dact_f(int act, float s) { return tx_epi::dact(act, s); }

// Epilogue over one transposed 32x32 chunk: lane = column, rr walks rows.
// The common cases (no beta, no pre-activation store, no act') run a tight
// loop specialised on the activation; everything else takes the general path.
template <int ACT>
__device__ __forceinline__ void epi_rows_fast(const float *__restrict__ t, int lane,
                                              float *__restrict__ cp, int64_t ldc, int rows,
                                              float alpha, bool has_bias, float bias_v, bool round_out) {
#pragma unroll 8
  for (int rr = 0; rr < rows; ++rr) {
    float x = alpha * t[rr * 33 + lane];
    if (has_bias) x += bias_v;
    x = act_f(ACT, x);
    cp[rr * ldc] = round_out ? tx_epi::round_tf32(x) : x;
  }
}

// Epilogue arguments that stay in registers across the chunk loop.
struct EpiArgs {
  float alpha, beta;
  int act, dact;
  float *C;
  int64_t ldc;
  float *preact;
  int64_t ld_preact;
  const float *dact_src;
  int64_t ld_dact;
  bool round_out;
};

// Epilogue with beta * C, a pre-activation store or act', specialised on the
// activation pair so that the 32 unrolled rows hold only the math they run
// (a runtime switch inlined 32 times spreads each row's few instructions over
// tens of KB of code and the warps stall on instruction fetch).  All loads of
// the chunk's rows are issued before the first store: the stores may alias the
// loaded tensors, so interleaving them would cost one round trip per row.
template <int ACT, int DACT>
__device__ __forceinline__ void epi_rows_spec(const float *__restrict__ t, int lane, const EpiArgs &e,
                                              int64_t row0, int64_t gn, int rows, bool has_bias,
                                              float bias_v) {
  const bool beta = e.beta != 0.f;
  float cv[32], sv[32];
#pragma unroll
  for (int rr = 0; rr < 32; ++rr) {
    const bool ok = rr < rows;
    cv[rr] = (ok && beta) ? e.C[(row0 + rr) * e.ldc + gn] : 0.f;
    sv[rr] = (DACT != TX_ACT_NONE && ok) ? __ldg(e.dact_src + (row0 + rr) * e.ld_dact + gn) : 0.f;
  }
#pragma unroll
  for (int rr = 0; rr < 32; ++rr) {
    if (rr < rows) {
      float x = e.alpha * t[rr * 33 + lane];
      if (has_bias) x += bias_v;
      if (beta) x += e.beta * cv[rr];
      if (e.preact) e.preact[(row0 + rr) * e.ld_preact + gn] = x;
      x = act_f(ACT, x);
      if (DACT != TX_ACT_NONE) x *= dact_f(DACT, sv[rr]);
      e.C[(row0 + rr) * e.ldc + gn] = e.round_out ? tx_epi::round_tf32(x) : x;
    }
  }
}

// Both an activation and act' in one epilogue (no workload lowers to this):
// compact runtime loop.
__device__ __noinline__ void epi_rows_any(const float *__restrict__ t, int lane, const EpiArgs &e,
                                          int64_t row0, int64_t gn, int rows, bool has_bias,
                                          float bias_v) {
#pragma unroll 1
  for (int rr = 0; rr < rows; ++rr) {
    const int64_t gm = row0 + rr;
    float x = e.alpha * t[rr * 33 + lane];
    if (has_bias) x += bias_v;
    if (e.beta != 0.f) x += e.beta * e.C[gm * e.ldc + gn];
    if (e.preact) e.preact[gm * e.ld_preact + gn] = x;
    x = act_f(e.act, x);
    x *= dact_f(e.dact, e.dact_src[gm * e.ld_dact + gn]);
    e.C[gm * e.ldc + gn] = e.round_out ? tx_epi::round_tf32(x) : x;
  }
}

// Hint the rows of a tensor this CTA's epilogue will read into L2 while the
// main loop runs (bulk prefetch; in-bounds, 16-byte aligned spans only).
__device__ __forceinline__ void prefetch_rows_l2(const float *base, int64_t ld, int64_t row0,
                                                 int64_t rows, int64_t col0, int64_t cols, int lane) {
  if (!base || cols <= 0 || rows <= 0) return;
  const float *p0 = base + row0 * ld + col0;
  uint32_t bytes = (uint32_t)(cols * 4) & ~15u;
  if (((uintptr_t)p0 & 15) || (ld & 3) || bytes == 0) return;
  for (int64_t r = lane; r < rows; r += 32) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p0 + r * ld), "r"(bytes)
                 : "memory");
  }
}

// After the epilogue math of a chunk: the fused column sums of the unrounded
// values (one partial row per 32 output rows), then the optional TF32 rounding
// of what is stored.
__device__ __forceinline__ void chunk_finish(float (&v)[32], const tx_gemm_desc &d, float *col_part,
                                             int64_t row_tile, int64_t gn0, int lane) {
  // a 32-row group wholly past M (the last tile's lower quadrants) has no
  // partial row: the buffer holds ceil(M / 32)
  if (col_part && row_tile < d.M) {
    float w[32];
    const bool row_ok = row_tile + lane < d.M;
#pragma unroll
    for (int j = 0; j < 32; ++j) w[j] = row_ok ? v[j] : 0.f;
    const float cs = tx_epi::colsum32(w, lane);
    if (gn0 + lane < d.N) col_part[(row_tile / 32) * d.N + gn0 + lane] = cs;
  }
  if (d.flags & TX_GEMM_ROUND_OUT) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = tx_epi::round_tf32(v[j]);
  }
}

// ---- TMA epilogue of one warp ------------------------------------------------------------
// A warp owns the 32 accumulator rows of its TMEM lane quadrant.  Per 32 x 32
// chunk: tcgen05.ld of the chunk in every accumulator (one wait); the act'
// source / C tiles from an NS-slot ring that TMA fills ahead; alpha, the bias
// (staged in shared memory before the accumulator is ready), beta * C, act,
// act'; column sums and rounding; then a swizzled output (and pre-activation)
// tile that lane 0 stores with TMA from one of two slots.  Ring and output
// slots count across tiles, so a persistent CTA keeps one state per warp.
template <int NS>
struct EpiWarp {
  uint8_t *out_t;  // 2 output slots
  uint8_t *pre_t;  // 2 pre-activation slots (when stored)
  uint8_t *s_t;    // NS act'-source slots
  uint8_t *c_t;    // NS C slots
  uint64_t *bars;  // NS load barriers
  const CUtensorMap *map_c, *map_s, *map_p;
  uint32_t issued, consumed, seq;
  bool need_s, need_c, need_p;
  int wsplit;  // > 0: output row y sits at (y % wsplit, y / wsplit) of 3-D views (GatherOp)

  // the map coordinates of output row y, batch z
  __device__ __forceinline__ void rows(int y, int z, int &y2, int &z2) const {
    if (wsplit > 0) {
      y2 = y % wsplit;
      z2 = y / wsplit;
    } else {
      y2 = y;
      z2 = z;
    }
  }
  // act' / C tiles of the chunk at column x into the next ring slot
  __device__ __forceinline__ void issue(int x, int y, int z, int lane) {
    const int slot = (int)(issued % NS);
    if (lane == 0) {
      uint64_t *bar = &bars[slot];
      int y2, z2;
      rows(y, z, y2, z2);
      mbar_expect_tx(bar, (need_s ? 4096u : 0u) + (need_c ? 4096u : 0u));
      if (need_s) tma_load_3d(smem_u32(s_t + slot * 4096), map_s, bar, x, y2, z2);
      if (need_c) tma_load_3d(smem_u32(c_t + slot * 4096), map_c, bar, x, y2, z2);
    }
    ++issued;
  }
  // fill the free ring slots with this warp's next chunks of the tile (chunk
  // c0 + k * cstep for the k-th)
  template <int NCH>
  __device__ __forceinline__ void fill(int &next, int c0, int cstep, int n0, int row_tile, int z,
                                       int lane) {
    while (c0 + next * cstep < NCH && issued - consumed < (uint32_t)NS) {
      issue(n0 + 32 * (c0 + next * cstep), row_tile, z, lane);
      ++next;
    }
  }
  // before the shared memory is released: loads still in flight (after an
  // abort) land, and the stores have read their tiles
  __device__ __forceinline__ void drain(int lane) {
    for (uint32_t c = consumed; c < issued; ++c) mbar_drain(&bars[c % NS], (c / NS) & 1);
    if (lane == 0) bulk_wait_read<0>();
    __syncwarp();
  }
};

// Stage the tile's bias (times bias_scale; zero past N) for this warp.
template <int BN>
__device__ __forceinline__ void stage_bias(float *bias_w, const tx_gemm_desc &d, int n0, int lane) {
#pragma unroll
  for (int i = lane; i < BN; i += 32) {
    const int64_t gn = (int64_t)n0 + i;
    bias_w[i] = (d.bias && gn < d.N) ? d.bias[gn] * d.bias_scale : 0.f;
  }
  __syncwarp();
}

// One tile of this warp.  tbase: TMEM address of the warp's lanes at the
// tile's first accumulator column; `next`: chunks of the tile already issued
// into the ring.  bias_w: the tile's staged bias, or null to fetch it a chunk
// ahead into registers and pass each chunk's 32 values through bias_row (32
// floats of this warp).  release (or null): arrived on once the warp has read
// the tile's last accumulator chunk.  ACT / DACT compile-time, or -1 for the
// values in d; LOADS: an act' source or beta * C is read.  DUAL: the first two
// accumulators' loads are in flight together (32 more live registers).
template <int BN, int NACC, int NS, int ACT, int DACT, bool LOADS, bool DUAL>
__device__ __forceinline__ bool epi_tile(EpiWarp<NS> &e, const tx_gemm_desc &d, uint32_t tbase, int used_acc,
                                      const float *bias_w, float *bias_row, int n0, int row_tile, int z,
                                      float *col_part, int next, uint64_t *release, volatile int *abort_flag,
                                      int *err, int site, int lane, int c0, int cstep) {
  constexpr int NCH = BN / 32;
  const int act = ACT >= 0 ? ACT : d.act;
  const int dact = DACT >= 0 ? DACT : d.dact;
  const bool has_bias = d.bias != nullptr;
  const float alpha = d.alpha, beta = d.beta;
  auto bias_at = [&](int c) {
    const int64_t gn = (int64_t)n0 + 32 * c + lane;
    return (has_bias && gn < d.N) ? d.bias[gn] * d.bias_scale : 0.f;
  };
  float bnext = bias_w ? 0.f : bias_at(c0);
  if (LOADS) e.template fill<NCH>(next, c0, cstep, n0, row_tile, z, lane);
#pragma unroll 1
  for (int c = c0; c < NCH; c += cstep) {
    float v[32];
    {
      uint32_t r0[32];
      int a = 1;
      tmem_ld32_issue(tbase + (uint32_t)(c * 32), r0);
      if (DUAL && NACC > 1 && used_acc > 1) {
        uint32_t r1[32];
        tmem_ld32_issue(tbase + (uint32_t)(BN + c * 32), r1);
        tmem_wait_ld();
        reg_fence(r0);
        reg_fence(r1);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r0[j]) + __uint_as_float(r1[j]);
        a = 2;
      } else {
        tmem_wait_ld();
        reg_fence(r0);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r0[j]);
      }
#pragma unroll 1
      for (; a < used_acc; ++a) {  // accumulators loaded one at a time
        tmem_ld32_issue(tbase + (uint32_t)(a * BN + c * 32), r0);
        tmem_wait_ld();
        reg_fence(r0);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] += __uint_as_float(r0[j]);
      }
    }
    if (release && c + cstep >= NCH) {
      // this warp has read its rows of the accumulator: hand the buffer back
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(release);
    }
    float sv[32], cv[32];
    if (LOADS) {
      const uint32_t k = e.consumed;
      if (!mbar_wait(&e.bars[k % NS], (k / NS) & 1, abort_flag, err, site)) return false;
      ++e.consumed;
      if (e.need_s) {
        tile_row_load(e.s_t + (k % NS) * 4096, lane, sv);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) sv[j] = 0.f;
      }
      if (e.need_c) {
        tile_row_load(e.c_t + (k % NS) * 4096, lane, cv);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) cv[j] = 0.f;
      }
      __syncwarp();  // every lane has read the slot before it is refilled
      e.template fill<NCH>(next, c0, cstep, n0, row_tile, z, lane);
    }
    const int oslot = (int)(e.seq & 1);
    const float *bb = bias_w + c * 32;
    if (!bias_w) {
      bias_row[lane] = bnext;
      if (c + cstep < NCH) bnext = bias_at(c + cstep);  // lands while this chunk is processed
      bb = bias_row;
    }
    if (lane == 0 && e.seq >= 2) bulk_wait_read<1>();  // the tiles of chunk seq - 2 are free
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      float x = alpha * v[j];
      if (has_bias) x += bb[j];
      if (LOADS) x += beta * cv[j];
      v[j] = x;
    }
    uint8_t *pre_tile = e.need_p ? e.pre_t + oslot * 4096 : nullptr;
    if (pre_tile) tile_row_store(pre_tile, lane, v);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      float x = act_f(act, v[j]);
      if (LOADS && dact != TX_ACT_NONE) x *= dact_f(dact, sv[j]);
      v[j] = x;
    }
    chunk_finish(v, d, col_part, row_tile, (int64_t)n0 + 32 * c, lane);
    tile_row_store(e.out_t + oslot * 4096, lane, v);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> TMA reads
    __syncwarp();
    if (lane == 0) {
      int y2, z2;
      e.rows(row_tile, z, y2, z2);
      tma_store_3d(e.map_c, smem_u32(e.out_t + oslot * 4096), n0 + 32 * c, y2, z2);
      if (pre_tile) tma_store_3d(e.map_p, smem_u32(pre_tile), n0 + 32 * c, y2, z2);
      bulk_commit();
    }
    __syncwarp();
    ++e.seq;
  }
  return true;
}

// The epilogue variant for d: compile-time activation paths for every
// combination the engine produces (the runtime-valued path is several times
// slower: measured 46.8 against 6.6 us for a 32768 x 256 beta = 1 epilogue).
template <int BN, int NACC, int NS, bool DUAL>
__device__ __forceinline__ bool epi_any(EpiWarp<NS> &e, const tx_gemm_desc &d, uint32_t tbase, int used_acc,
                                        const float *bias_w, float *bias_row, int n0, int row_tile, int z,
                                        float *col_part, int next, uint64_t *release, volatile int *abort_flag,
                                        int *err, int site, int lane, int c0 = 0, int cstep = 1) {
#define TX_EPI(A, D, L)                                                                                 \
  epi_tile<BN, NACC, NS, A, D, L, DUAL>(e, d, tbase, used_acc, bias_w, bias_row, n0, row_tile, z, col_part, next, \
                                  release, abort_flag, err, site, lane, c0, cstep)
  if (!e.need_s && !e.need_c) {  // no act' source: dact is none
    switch (d.act) {
      case TX_ACT_RELU: return TX_EPI(TX_ACT_RELU, TX_ACT_NONE, false);
      case TX_ACT_TANH: return TX_EPI(TX_ACT_TANH, TX_ACT_NONE, false);
      case TX_ACT_GELU: return TX_EPI(TX_ACT_GELU, TX_ACT_NONE, false);
      default: return TX_EPI(TX_ACT_NONE, TX_ACT_NONE, false);
    }
  }
  if (d.dact == TX_ACT_NONE) {  // beta * C, with or without an activation
    switch (d.act) {
      case TX_ACT_RELU: return TX_EPI(TX_ACT_RELU, TX_ACT_NONE, true);
      case TX_ACT_TANH: return TX_EPI(TX_ACT_TANH, TX_ACT_NONE, true);
      case TX_ACT_GELU: return TX_EPI(TX_ACT_GELU, TX_ACT_NONE, true);
      default: return TX_EPI(TX_ACT_NONE, TX_ACT_NONE, true);
    }
  }
  if (d.act == TX_ACT_NONE) {  // act', with or without beta * C
    switch (d.dact) {
      case TX_ACT_RELU: return TX_EPI(TX_ACT_NONE, TX_ACT_RELU, true);
      case TX_ACT_TANH: return TX_EPI(TX_ACT_NONE, TX_ACT_TANH, true);
      default: return TX_EPI(TX_ACT_NONE, TX_ACT_GELU, true);
    }
  }
  // an activation and act' together (not produced by the engine): runtime
  // values, several times slower
  return TX_EPI(-1, -1, true);
#undef TX_EPI
}

// PAIR (MODE 0 only): launched as clusters of two CTAs along blockIdx.x; the
// even CTA (the leader) issues the MMAs for both, the odd one only loads its
// operand halves and runs its own epilogue on its own TMEM rows.
template <int BN, bool A_MN, bool B_MN, int MODE, bool PAIR = false>
__global__ void __launch_bounds__(320, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
              const __grid_constant__ CUtensorMap mapC, const __grid_constant__ CUtensorMap mapS,
              const __grid_constant__ CUtensorMap mapP, const tx_gemm_desc d, int *err, int kb_per_cta,
              int tma_epi, int conv_mask, float *col_part, const __grid_constant__ tx_tc::GatherOp gop) {
  static_assert(!PAIR || MODE == 0, "operand conversion is per CTA");
  using Cfg = TcCfg<BN, MODE, PAIR>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int NACC = Cfg::NACC;
  constexpr int A_BYTES = Cfg::A_BYTES, B_BYTES = Cfg::B_BYTES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t *full = (uint64_t *)(smem + STAGES * Cfg::STAGE);
  uint64_t *conv = full + STAGES;
  uint64_t *empty = conv + STAGES;
  uint64_t *accb = empty + STAGES;
  uint64_t *ebar = accb + 1;  // two act'/C tile-load slots per epilogue warp (eight warps)
  uint32_t *tmem_holder = (uint32_t *)(ebar + 16);
  volatile int *abort_flag = (volatile int *)(tmem_holder + 1);
  float *bias_all = reinterpret_cast<float *>(smem + STAGES * Cfg::STAGE + 1024);  // [8][BN]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // a CTA pair's two row tiles are neighbours along x (the cluster's x)
  const int m0 = (PAIR ? blockIdx.x : blockIdx.y) * TC_BM;
  const int n0 = (PAIR ? blockIdx.y : blockIdx.x) * BN;
  const int bz = blockIdx.z;
  // split-K (kb_per_cta > 0): blockIdx.z selects a range of k-blocks and a raw
  // partial output slice; the operands have no batch dimension then
  const int total_kb = (int)((d.K + TC_BK - 1) / TC_BK);
  const int kb_first = kb_per_cta > 0 ? bz * kb_per_cta : 0;
  const int num_k = kb_per_cta > 0 ? min(kb_per_cta, total_kb - kb_first) : total_kb;
  const int zc = kb_per_cta > 0 ? 0 : bz;
  const int used_acc = num_k < NACC ? num_k : NACC;
  const uint32_t rank = PAIR ? cluster_rank() : 0u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], kConvThreads);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accb, 1);
    for (int i = 0; i < 16; ++i) mbar_init(&ebar[i], 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    if (PAIR) {
      // both CTAs of the pair allocate together; the leader's MMAs write the
      // same columns of both
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_u32(tmem_holder)),
                   "r"(Cfg::TMEM_COLS));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_u32(tmem_holder)),
                   "r"(Cfg::TMEM_COLS));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
  }
  tc_fence_before();
  if (PAIR)
    cluster_sync_all();  // the peer's barriers are initialised before any copy or commit reaches them
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      for (int kb = 0; kb < num_k; ++kb) {
        const int s = kb % STAGES;
        const uint32_t round = kb / STAGES;
        if (!mbar_wait(&empty[s], (round & 1) ^ 1, abort_flag, err, 1)) break;
        const uint32_t a_dst = smem_u32(smem + s * Cfg::STAGE);
        const uint32_t b_dst = a_dst + A_BYTES;
        const int k0 = (kb_first + kb) * TC_BK;
        if (PAIR) {
          // both halves complete on the leader's full barrier; the leader
          // expects the bytes of both
          const uint32_t fb = map_to_rank(smem_u32(&full[s]), 0);
          if (rank == 0) mbar_expect_tx(&full[s], 2 * (A_BYTES + B_BYTES));
          if (A_MN && gop.amn) {
            tma_load_4d_pair(a_dst, &mapA, fb, 0, k0, m0 / 32, gop.ashared ? 0 : zc);
          } else if (A_MN) {
#pragma unroll
            for (int j = 0; j < TC_BM / 32; ++j)
              tma_load_3d_pair(a_dst + j * 4096, &mapA, fb, m0 + 32 * j, k0, gop.ashared ? 0 : zc);
          } else {
            tma_load_3d_pair(a_dst, &mapA, fb, k0, m0, gop.ashared ? 0 : zc);
          }
          const int nb = n0 + (int)rank * (BN / 2);
          if (B_MN && gop.bmn) {
            tma_load_4d_pair(b_dst, &mapB, fb, 0, k0, nb / 32, zc);
          } else if (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_3d_pair(b_dst + j * 4096, &mapB, fb, nb + 32 * j, k0, zc);
          } else {
            tma_load_3d_pair(b_dst, &mapB, fb, k0, nb, zc);
          }
          continue;
        }
        mbar_expect_tx(&full[s], A_BYTES + gather_b_bytes<BN>(gop, n0));
        if (gop.a || gop.b) gather_loads<BN>(gop, &mapA, &mapB, &full[s], a_dst, b_dst, m0, n0, kb_first + kb);
        if (gop.a) {
        } else if (A_MN) {
          load_mn(a_dst, &mapA, &full[s], gop.amn, TC_BM / 32, m0, k0, gop.ashared ? 0 : zc);
        } else {
          tma_load_3d(a_dst, &mapA, &full[s], k0, m0, gop.ashared ? 0 : zc);
        }
        if (gop.b) {
        } else if (B_MN) {
          load_mn(b_dst, &mapB, &full[s], gop.bmn, BN / 32, n0, k0, zc);
        } else {
          tma_load_3d(b_dst, &mapB, &full[s], k0, n0, zc);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      const uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((A_MN ? 1u : 0u) << 15) |
                             ((B_MN ? 1u : 0u) << 16) | ((uint32_t)(BN >> 3) << 17) |
                             ((uint32_t)((PAIR ? 2 : 1) * TC_BM >> 4) << 24);
      for (int kb = 0; kb < num_k; ++kb) {
        const int s = kb % STAGES;
        const uint32_t round = kb / STAGES;
        uint64_t *ready = MODE == 0 ? &full[s] : &conv[s];
        if (!mbar_wait(ready, round & 1, abort_flag, err, 2)) break;
        tc_fence_after();
        const uint32_t a_base = smem_u32(smem + s * Cfg::STAGE);
        const uint32_t b_base = a_base + A_BYTES;
        const uint32_t acc = tmem + (uint32_t)((kb % NACC) * BN);
        const bool fresh = kb < NACC;  // first k-block of this accumulator
#pragma unroll
        for (int k = 0; k < TC_BK / 8; ++k) {
          const uint64_t ad = operand_desc<A_MN>(a_base, k);
          const uint64_t bd = operand_desc<B_MN>(b_base, k);
          tc_mma_tf32<PAIR>(acc, ad, bd, idesc, (fresh && k == 0) ? 0u : 1u);
          if (MODE == 2) {
            const uint32_t sa = a_base + A_BYTES + B_BYTES, sb = sa + A_BYTES;
            tc_mma_tf32(acc, ad, operand_desc<B_MN>(sb, k), idesc, 1u);
            tc_mma_tf32(acc, operand_desc<A_MN>(sa, k), bd, idesc, 1u);
          }
        }
        if (PAIR) {
          // free the stage in both CTAs; the last STAGES stages are never
          // waited for, so no arrive is left in flight toward the peer at exit
          if (kb + STAGES < num_k) {
            tc_commit_pair(map_to_rank(smem_u32(&empty[s]), 0));
            tc_commit_pair(map_to_rank(smem_u32(&empty[s]), 1));
          }
        } else {
          tc_commit(&empty[s]);
        }
      }
      if (PAIR) {
        tc_commit_pair(map_to_rank(smem_u32(accb), 0));
        tc_commit_pair(map_to_rank(smem_u32(accb), 1));
      } else {
        tc_commit(accb);  // arrives once every MMA issued above has completed
      }
    }
  } else {
    const int ct = threadIdx.x - 64;  // 0..255; warps 2..5 (0..127) convert operands
    if (warp < 6) {
      // the epilogue's reads of C (beta) and of the act' source hit L2, not DRAM
      const int q = warp & 3;
      const int64_t r0 = (int64_t)m0 + q * 32;
      const int64_t nrows = d.M - r0 < 32 ? d.M - r0 : 32;
      const int64_t ncols = d.N - n0 < BN ? d.N - n0 : BN;
      const int64_t cb = (int64_t)bz * d.stride_c;
      if (d.dact) prefetch_rows_l2(d.dact_src + cb, d.ld_dact, r0, nrows, n0, ncols, lane);
      if (d.beta != 0.f) prefetch_rows_l2(d.C + cb, d.ldc, r0, nrows, n0, ncols, lane);
    }
    if (MODE != 0 && warp < 6) {
      // operand conversion, one stage behind the producer and one ahead of the MMA;
      // in MODE 1 an operand that already holds TF32 values (conv_mask bit clear)
      // is left alone
      constexpr int N4 = (A_BYTES + B_BYTES) / 16;
      const int i_begin = (MODE == 2 || (conv_mask & 1)) ? ct : A_BYTES / 16 + ct;
      const int i_end = (MODE == 2 || (conv_mask & 2)) ? N4 : A_BYTES / 16;
      for (int kb = 0; kb < num_k; ++kb) {
        const int s = kb % STAGES;
        const uint32_t round = kb / STAGES;
        if (!mbar_wait(&full[s], round & 1, abort_flag, err, 4)) break;
        float4 *p = reinterpret_cast<float4 *>(smem + s * Cfg::STAGE);
        float4 *q = reinterpret_cast<float4 *>(smem + s * Cfg::STAGE + A_BYTES + B_BYTES);
#pragma unroll 4
        for (int i = i_begin; i < i_end; i += kConvThreads) {
          float4 v = p[i];
          float4 big = make_float4(to_tf32_rn(v.x), to_tf32_rn(v.y), to_tf32_rn(v.z), to_tf32_rn(v.w));
          p[i] = big;
          if (MODE == 2)
            q[i] = make_float4(to_tf32_rn(v.x - big.x), to_tf32_rn(v.y - big.y),
                               to_tf32_rn(v.z - big.z), to_tf32_rn(v.w - big.w));
        }
        // make the generic-proxy writes visible to the tensor core (async proxy)
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive(&conv[s]);
      }
    }
    // epilogue warps 2..9 -> TMEM lane quadrants 2,3,0,1,2,3,0,1.  Two warps
    // share a quadrant and take alternate 32-column chunks, so two serial
    // chains (TMEM load, math, shared store, TMA store) run per scheduler;
    // when all of pre-activation, act' source and C are in use, warps 2..5
    // alone take every chunk (six tiles per warp would not hold them).
    const int ew = warp - 2;  // 0..7
    const int quad = warp & 3;
    const int half = ew >> 2;
    const bool need_s = d.dact != TX_ACT_NONE, need_c = d.beta != 0.f, need_p = d.preact != nullptr;
    const int tiles_w = 2 + (need_p ? 2 : 0) + (need_s ? 2 : 0) + (need_c ? 2 : 0);
    const bool wide = tiles_w <= 6;
    const bool active = wide || half == 0;
    float *bias_w = bias_all + ew * BN;
    if (active) stage_bias<BN>(bias_w, d, n0, lane);  // while the main loop runs
    const bool have = mbar_wait(accb, 0, abort_flag, err, 3);
    tc_fence_after();
    if (have && !*abort_flag && tma_epi) {
      if (active) {
        // TMA epilogue over the drained pipeline stages
        EpiWarp<2> e;
        uint8_t *eb = smem + ew * (wide ? 6 : 8) * 4096;
        e.need_s = need_s;
        e.need_c = need_c;
        e.need_p = need_p;
        e.out_t = eb;
        e.pre_t = eb + 2 * 4096;
        e.s_t = e.pre_t + (need_p ? 2 * 4096 : 0);
        e.c_t = e.s_t + (need_s ? 2 * 4096 : 0);
        e.bars = &ebar[ew * 2];
        e.map_c = &mapC;
        e.map_s = &mapS;
        e.map_p = &mapP;
        e.issued = e.consumed = e.seq = 0;
        e.wsplit = gop.wsplit;
        const uint32_t tbase = tmem + ((uint32_t)(quad * 32) << 16);
        epi_any<BN, NACC, 2, true>(e, d, tbase, used_acc, bias_w, nullptr, n0, m0 + quad * 32, bz, col_part,
                                   0, nullptr, abort_flag, err, 5, lane, wide ? half : 0, wide ? 2 : 1);
        e.drain(lane);
      }
    } else if (have && !*abort_flag && half == 0) {
      // TMEM gives each thread one row; global memory wants a warp per row.
      // Each 32x32 chunk is transposed through padded shared memory (the
      // drained pipeline stages), then lanes walk columns so every load and
      // store of the epilogue is a coalesced 128-byte row segment.
      float *tile = reinterpret_cast<float *>(smem) + quad * (32 * 33);
      const int64_t row0 = (int64_t)m0 + quad * 32;
      float *C = d.C + (int64_t)bz * d.stride_c;
      const int64_t cbase = bz * d.stride_c;
      const bool round_out = (d.flags & TX_GEMM_ROUND_OUT) != 0;
      const EpiArgs ea{d.alpha, d.beta, d.act, d.dact, C, d.ldc,
                       d.preact ? d.preact + cbase : nullptr, d.ld_preact,
                       d.dact_src ? d.dact_src + cbase : nullptr, d.ld_dact, round_out};
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        float v[32];
        const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)c;
        tmem_ld32(lane_base, v);
#pragma unroll 1
        for (int a = 1; a < used_acc; ++a) {
          float w[32];
          tmem_ld32(lane_base + (uint32_t)(a * BN), w);
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] += w[j];
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) tile[lane * 33 + j] = v[j];
        __syncwarp();
        const int64_t gn = (int64_t)n0 + c + lane;
        const bool col_ok = gn < d.N;
        const float bias_v = (d.bias && col_ok) ? d.bias[gn] * d.bias_scale : 0.f;
        int rows = d.M - row0 < 32 ? (int)(d.M - row0) : 32;
        if (!col_ok || rows < 0) rows = 0;
        if (d.beta == 0.f && !d.preact && !d.dact) {
          float *cp = C + row0 * d.ldc + gn;
          switch (d.act) {
            case TX_ACT_RELU: epi_rows_fast<TX_ACT_RELU>(tile, lane, cp, d.ldc, rows, d.alpha, d.bias != nullptr, bias_v, round_out); break;
            case TX_ACT_TANH: epi_rows_fast<TX_ACT_TANH>(tile, lane, cp, d.ldc, rows, d.alpha, d.bias != nullptr, bias_v, round_out); break;
            case TX_ACT_GELU: epi_rows_fast<TX_ACT_GELU>(tile, lane, cp, d.ldc, rows, d.alpha, d.bias != nullptr, bias_v, round_out); break;
            default: epi_rows_fast<TX_ACT_NONE>(tile, lane, cp, d.ldc, rows, d.alpha, d.bias != nullptr, bias_v, round_out); break;
          }
        } else if (!d.dact) {
          const bool hb = d.bias != nullptr;
          switch (d.act) {
            case TX_ACT_RELU: epi_rows_spec<TX_ACT_RELU, TX_ACT_NONE>(tile, lane, ea, row0, gn, rows, hb, bias_v); break;
            case TX_ACT_TANH: epi_rows_spec<TX_ACT_TANH, TX_ACT_NONE>(tile, lane, ea, row0, gn, rows, hb, bias_v); break;
            case TX_ACT_GELU: epi_rows_spec<TX_ACT_GELU, TX_ACT_NONE>(tile, lane, ea, row0, gn, rows, hb, bias_v); break;
            default: epi_rows_spec<TX_ACT_NONE, TX_ACT_NONE>(tile, lane, ea, row0, gn, rows, hb, bias_v); break;
          }
        } else if (d.act == TX_ACT_NONE) {
          const bool hb = d.bias != nullptr;
          switch (d.dact) {
            case TX_ACT_RELU: epi_rows_spec<TX_ACT_NONE, TX_ACT_RELU>(tile, lane, ea, row0, gn, rows, hb, bias_v); break;
            case TX_ACT_TANH: epi_rows_spec<TX_ACT_NONE, TX_ACT_TANH>(tile, lane, ea, row0, gn, rows, hb, bias_v); break;
            default: epi_rows_spec<TX_ACT_NONE, TX_ACT_GELU>(tile, lane, ea, row0, gn, rows, hb, bias_v); break;
          }
        } else {
          epi_rows_any(tile, lane, ea, row0, gn, rows, d.bias != nullptr, bias_v);
        }
        __syncwarp();
      }
    }
  }

  tc_fence_before();
  __syncwarp();
  if (PAIR)
    cluster_sync_all();  // neither CTA leaves while the other may still touch its memory
  else
    __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if (PAIR)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                   "r"(Cfg::TMEM_COLS));
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                   "r"(Cfg::TMEM_COLS));
  }
}

// ---- persistent variant ------------------------------------------------------------------
// For operands that need no conversion (TF32 mode with pre-rounded operands,
// or the truncating mode): one CTA per SM walks the output tiles (tile order:
// N fastest, so CTAs that run together share A rows in L2).  The TMA / MMA
// ring runs on across tiles, and TMEM holds two accumulator buffers, so the
// MMA warp fills one while the epilogue warps drain the other.  The epilogue
// has its own shared memory (the stages stay busy): per warp two output tiles
// plus two pre-activation, act'-source and C tiles when the GEMM uses them.
// EW epilogue warps: 4 (one per TMEM lane quadrant), or 8 for epilogues whose
// arithmetic outweighs a tile's main loop (GELU and its derivative): two warps
// per quadrant then take alternate 32-column chunks.
constexpr int kSmemMax = 232448;  // 227 KB opt-in
constexpr int kPTail = 2048;  // barriers, then each epilogue warp's 32 bias values (8 warps at most)

// BLO: B arrives as a TF32 head and tail (two tiles per stage) and each
// k-slice issues A B + A B_lo, so the weights enter the product to fp32-class
// accuracy while A stays TF32.
// MODE (as in the one-tile kernel): 0 operands used as loaded; 1 four
// conversion warps round each landed stage to TF32 in place; 2 they split
// both operands into big and small halves (the small ones in the stage's
// second half) and each k-slice issues three MMAs.  With conversion the tiles
// are at most 128 wide, so that each of the two TMEM buffers holds as many
// accumulators as the one-tile kernel keeps (the chains of truncating TMEM
// adds, and so the products' rounding, stay as short).
template <int BN, bool BLO = false, int MODE = 0>
struct PCfg {
  static_assert(MODE == 0 || BN <= 128, "persistent tiles with operand conversion are at most 128 wide");
  static constexpr int NACC = MODE == 2 ? (512 / (2 * BN) > 4 ? 4 : 512 / (2 * BN)) : (BN == 256 ? 1 : 2);
  static constexpr int ACC = BN * NACC;                 // columns per accumulator buffer
  static constexpr int TMEM_COLS = 2 * ACC < 256 ? 256 : 2 * ACC;
  static constexpr int A_BYTES = TC_BM * TC_BK * 4;
  static constexpr int B_BYTES = BN * TC_BK * 4;
  static constexpr int STAGE = (A_BYTES + B_BYTES * (BLO ? 2 : 1)) * (MODE == 2 ? 2 : 1);
  static constexpr int CONV_THREADS = MODE ? kConvThreads : 0;
};

struct PWork {
  int tiles_m, tiles_n, items;
  int total_kb, kb_per;  // kb_per > 0: split-K, the third item index is the split
  int stages;            // pipeline depth (runtime: the epilogue's tiles vary)
  int ep_stride;         // epilogue bytes per warp
  float *col_part;       // fused column sums (one row per 32 output rows) or null
  int conv_mask;         // MODE 1: operands to round (bit 0 A, bit 1 B)
};

template <int BN, bool A_MN, bool B_MN, int EW, bool BLO = false, int MODE = 0>
__global__ void __launch_bounds__(64 + 32 * EW + PCfg<BN, BLO, MODE>::CONV_THREADS, 1)
    k_gemm_tcp(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
               const __grid_constant__ CUtensorMap mapC, const __grid_constant__ CUtensorMap mapS,
               const __grid_constant__ CUtensorMap mapP, const __grid_constant__ CUtensorMap mapB2,
               const tx_gemm_desc d, int *err, PWork w, const __grid_constant__ tx_tc::GatherOp gop) {
  static_assert(MODE == 0 || !BLO, "split weights take no operand conversion");
  using Cfg = PCfg<BN, BLO, MODE>;
  constexpr int NACC = Cfg::NACC;
  constexpr int A_BYTES = Cfg::A_BYTES, B_BYTES = Cfg::B_BYTES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int stages = w.stages;
  uint8_t *ep = smem + stages * Cfg::STAGE;
  static_assert(EW == 4 || EW == 8, "one or two epilogue warps per TMEM lane quadrant");
  uint8_t *tail = ep + EW * w.ep_stride;
  uint64_t *full = (uint64_t *)tail;
  uint64_t *empty = full + 8;
  uint64_t *tfull = empty + 8;
  uint64_t *tempty = tfull + 2;
  uint64_t *ebar = tempty + 2;
  uint64_t *conv = ebar + 2 * EW;  // MODE >= 1: stage converted (kConvThreads arrivals)
  uint32_t *tmem_holder = (uint32_t *)(conv + 8);
  volatile int *abort_flag = (volatile int *)(tmem_holder + 1);
  float *bias_rows = reinterpret_cast<float *>(tail + 1024);  // [EW][32]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const bool split = w.kb_per > 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&conv[s], kConvThreads);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], EW);  // one arrival per epilogue warp
    }
    for (int i = 0; i < 2 * EW; ++i) mbar_init(&ebar[i], 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_holder)),
                 "r"(Cfg::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  // item -> (z, m tile, n tile) and its k-block range
  auto decode = [&](int item, int &m0, int &n0, int &z, int &kb_first, int &num_k) {
    const int nt = item % w.tiles_n;
    const int t = item / w.tiles_n;
    m0 = (t % w.tiles_m) * TC_BM;
    n0 = nt * BN;
    z = t / w.tiles_m;
    kb_first = split ? z * w.kb_per : 0;
    num_k = split ? min(w.kb_per, w.total_kb - kb_first) : w.total_kb;
  };

  if (warp == 0) {
    if (lane == 0) {
      uint32_t cnt = 0;
      for (int item = blockIdx.x; item < w.items && !*abort_flag; item += gridDim.x) {
        int m0, n0, z, kb_first, num_k;
        decode(item, m0, n0, z, kb_first, num_k);
        const int zc = split ? 0 : z;
        for (int kb = 0; kb < num_k; ++kb, ++cnt) {
          const int s = (int)(cnt % (uint32_t)stages);
          const uint32_t round = cnt / (uint32_t)stages;
          if (!mbar_wait(&empty[s], (round & 1) ^ 1, abort_flag, err, 11)) break;
          mbar_expect_tx(&full[s], A_BYTES + gather_b_bytes<BN>(gop, n0) + (BLO ? B_BYTES : 0));
          const uint32_t a_dst = smem_u32(smem + s * Cfg::STAGE);
          const uint32_t b_dst = a_dst + A_BYTES;
          const int k0 = (kb_first + kb) * TC_BK;
          if (gop.a || gop.b) gather_loads<BN>(gop, &mapA, &mapB, &full[s], a_dst, b_dst, m0, n0, kb_first + kb);
          if (gop.a) {
          } else if (A_MN) {
            load_mn(a_dst, &mapA, &full[s], gop.amn, TC_BM / 32, m0, k0, gop.ashared ? 0 : zc);
          } else {
            tma_load_3d(a_dst, &mapA, &full[s], k0, m0, gop.ashared ? 0 : zc);
          }
          if (gop.b) {
          } else if (B_MN) {
            load_mn(b_dst, &mapB, &full[s], gop.bmn, BN / 32, n0, k0, zc);
          } else {
            tma_load_3d(b_dst, &mapB, &full[s], k0, n0, zc);
          }
          if (BLO) {
            const uint32_t l_dst = b_dst + B_BYTES;
            if (B_MN) {
              load_mn(l_dst, &mapB2, &full[s], gop.bmn, BN / 32, n0, k0, zc);
            } else {
              tma_load_3d(l_dst, &mapB2, &full[s], k0, n0, zc);
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((A_MN ? 1u : 0u) << 15) |
                             ((B_MN ? 1u : 0u) << 16) | ((uint32_t)(BN >> 3) << 17) |
                             ((uint32_t)(TC_BM >> 4) << 24);
      uint32_t cnt = 0;
      int it = 0;
      for (int item = blockIdx.x; item < w.items && !*abort_flag; item += gridDim.x, ++it) {
        int m0, n0, z, kb_first, num_k;
        decode(item, m0, n0, z, kb_first, num_k);
        const int buf = it & 1;
        const uint32_t use = (uint32_t)it >> 1;
        if (!mbar_wait(&tempty[buf], (use & 1) ^ 1, abort_flag, err, 12)) break;
        tc_fence_after();
        bool ok = true;
        for (int kb = 0; kb < num_k; ++kb, ++cnt) {
          const int s = (int)(cnt % (uint32_t)stages);
          const uint32_t round = cnt / (uint32_t)stages;
          if (!mbar_wait(MODE == 0 ? &full[s] : &conv[s], round & 1, abort_flag, err, 13)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + s * Cfg::STAGE);
          const uint32_t b_base = a_base + A_BYTES;
          const uint32_t acc = tmem + (uint32_t)(buf * Cfg::ACC + (kb % NACC) * BN);
          const bool fresh = kb < NACC;
#pragma unroll
          for (int k = 0; k < TC_BK / 8; ++k) {
            const uint64_t ad = operand_desc<A_MN>(a_base, k);
            const uint64_t bd = operand_desc<B_MN>(b_base, k);
            tc_mma_tf32(acc, ad, bd, idesc, (fresh && k == 0) ? 0u : 1u);
            if (BLO) tc_mma_tf32(acc, ad, operand_desc<B_MN>(b_base + B_BYTES, k), idesc, 1u);
            if (MODE == 2) {
              const uint32_t sa = a_base + A_BYTES + B_BYTES, sb = sa + A_BYTES;
              tc_mma_tf32(acc, ad, operand_desc<B_MN>(sb, k), idesc, 1u);
              tc_mma_tf32(acc, operand_desc<A_MN>(sa, k), bd, idesc, 1u);
            }
          }
          tc_commit(&empty[s]);
        }
        if (!ok) break;
        tc_commit(&tfull[buf]);  // arrives when every MMA of this tile has completed
      }
    }
  } else if (MODE != 0 && warp >= 2 + EW) {
    // operand conversion, one stage behind the producer and one ahead of the
    // MMA, over the same k-block sequence
    const int ct = threadIdx.x - (64 + 32 * EW);  // 0 .. kConvThreads - 1
    constexpr int N4 = (A_BYTES + B_BYTES) / 16;
    const int i_begin = (MODE == 2 || (w.conv_mask & 1)) ? ct : A_BYTES / 16 + ct;
    const int i_end = (MODE == 2 || (w.conv_mask & 2)) ? N4 : A_BYTES / 16;
    uint32_t cnt = 0;
    bool alive = true;
    for (int item = blockIdx.x; item < w.items && alive; item += gridDim.x) {
      int m0, n0, z, kb_first, num_k;
      decode(item, m0, n0, z, kb_first, num_k);
      for (int kb = 0; kb < num_k; ++kb, ++cnt) {
        const int s = (int)(cnt % (uint32_t)stages);
        const uint32_t round = cnt / (uint32_t)stages;
        if (!mbar_wait(&full[s], round & 1, abort_flag, err, 16)) {
          alive = false;
          break;
        }
        float4 *pa = reinterpret_cast<float4 *>(smem + s * Cfg::STAGE);
        float4 *pq = reinterpret_cast<float4 *>(smem + s * Cfg::STAGE + A_BYTES + B_BYTES);
#pragma unroll 4
        for (int i = i_begin; i < i_end; i += kConvThreads) {
          const float4 v = pa[i];
          const float4 big = make_float4(to_tf32_rn(v.x), to_tf32_rn(v.y), to_tf32_rn(v.z), to_tf32_rn(v.w));
          pa[i] = big;
          if (MODE == 2)
            pq[i] = make_float4(to_tf32_rn(v.x - big.x), to_tf32_rn(v.y - big.y), to_tf32_rn(v.z - big.z),
                                to_tf32_rn(v.w - big.w));
        }
        // the generic-proxy writes become visible to the tensor core (async proxy)
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive(&conv[s]);
      }
    }
  } else {
    const int ew = warp - 2;        // 0 .. EW-1
    const int quad = warp & 3;      // the TMEM lane quadrant this warp may read
    const int c0 = ew >> 2;         // first chunk; then every cstep-th
    constexpr int cstep = EW / 4;
    uint8_t *eb = ep + ew * w.ep_stride;
    EpiWarp<2> e;
    e.need_s = d.dact != TX_ACT_NONE;
    e.need_c = d.beta != 0.f;
    e.need_p = d.preact != nullptr;
    // per-warp tile slots: out[2], then pre[2], s[2], c[2] when used
    e.out_t = eb;
    e.pre_t = eb + 8192;
    e.s_t = e.pre_t + (e.need_p ? 8192 : 0);
    e.c_t = e.s_t + (e.need_s ? 8192 : 0);
    e.bars = &ebar[ew * 2];
    e.map_c = &mapC;
    e.map_s = &mapS;
    e.map_p = &mapP;
    e.issued = e.consumed = e.seq = 0;
    e.wsplit = gop.wsplit;
    float *bias_row = bias_rows + ew * 32;
    int it = 0;
    bool alive = true;
    for (int item = blockIdx.x; item < w.items && alive; item += gridDim.x, ++it) {
      int m0, n0, z, kb_first, num_k;
      decode(item, m0, n0, z, kb_first, num_k);
      const int buf = it & 1;
      const uint32_t use = (uint32_t)it >> 1;
      const int row_tile = m0 + quad * 32;
      const int used_acc = num_k < NACC ? num_k : NACC;
      // the tile's first act' / C tiles, while its MMAs run
      int next = 0;
      if (e.need_s || e.need_c) e.template fill<BN / 32>(next, c0, cstep, n0, row_tile, z, lane);
      if (!mbar_wait(&tfull[buf], use & 1, abort_flag, err, 14)) break;
      tc_fence_after();
      const uint32_t tbase = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(buf * Cfg::ACC);
      alive = epi_any<BN, NACC, 2, false>(e, d, tbase, used_acc, nullptr, bias_row, n0, row_tile, z, w.col_part,
                                   next, &tempty[buf], abort_flag, err, 15, lane, c0, cstep);
    }
    e.drain(lane);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(Cfg::TMEM_COLS));
  }
}

// ---- launches ----------------------------------------------------------------------------
// `z` = batch count, or the number of K splits when kb_per_cta > 0
template <int BN, bool A_MN, bool B_MN, int MODE>
int launch_tc(tx_ctx *ctx, const tx_gemm_desc &d, const Maps &m, int64_t z, int kb_per_cta) {
  auto kern = k_gemm_tc<BN, A_MN, B_MN, MODE>;
  static bool configured[64] = {};
  int dev = ctx->device & 63;
  if (!configured[dev]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<BN, MODE>::SMEM);
    configured[dev] = true;
  }
  dim3 grid((unsigned)((d.N + BN - 1) / BN), (unsigned)((d.M + TC_BM - 1) / TC_BM), (unsigned)z);
  kern<<<grid, 320, TcCfg<BN, MODE>::SMEM, ctx->stream>>>(m.a, m.b, m.c, m.s, m.p, d, ctx->d_err,
                                                          kb_per_cta, m.tma_epi, m.conv_mask, m.col_part, m.g);
  TX_LAUNCHED(ctx, "k_gemm_tc");
  return TX_OK;
}

#ifdef TX_TC_PAIR_TU
// CTA pairs (BN = 256, no operand conversion): clusters of two CTAs along x
// (row tiles along x, column tiles along y), whose B maps box BN / 2 rows of
// a K-major B.
template <bool A_MN, bool B_MN>
int launch_tc_pair(tx_ctx *ctx, const tx_gemm_desc &d, const Maps &m, int64_t z, int kb_per_cta) {
  auto kern = k_gemm_tc<256, A_MN, B_MN, 0, true>;
  using Cfg = TcCfg<256, 0, true>;
  static bool configured[64] = {};
  const int dev = ctx->device & 63;
  if (!configured[dev]) {
    TX_CUDA(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
    configured[dev] = true;
  }
  const int64_t pairs_m = (d.M + 2 * TC_BM - 1) / (2 * TC_BM);
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof cfg);
  const int64_t tiles_n = (d.N + 255) / 256;
  if (tiles_n > 65535) return TX_ERR_UNSUPPORTED;
  cfg.gridDim = dim3((unsigned)(2 * pairs_m), (unsigned)tiles_n, (unsigned)z);
  cfg.blockDim = dim3(320, 1, 1);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  TX_CUDA(ctx, cudaLaunchKernelEx(&cfg, kern, m.a, m.b, m.c, m.s, m.p, d, ctx->d_err, kb_per_cta,
                                  m.tma_epi, m.conv_mask, m.col_part, m.g));
  TX_LAUNCHED(ctx, "k_gemm_tc");
  return TX_OK;
}

int launch_pair_impl(tx_ctx *ctx, const tx_gemm_desc &d, const Maps &m, int64_t z, int kb_per_cta) {
  const bool a_mn = d.trans_a != 0, b_mn = d.trans_b == 0;
  if (a_mn && b_mn) return launch_tc_pair<true, true>(ctx, d, m, z, kb_per_cta);
  if (a_mn) return launch_tc_pair<true, false>(ctx, d, m, z, kb_per_cta);
  if (b_mn) return launch_tc_pair<false, true>(ctx, d, m, z, kb_per_cta);
  return launch_tc_pair<false, false>(ctx, d, m, z, kb_per_cta);
}
#endif  // TX_TC_PAIR_TU

template <int BN, int MODE>
int launch_bn(tx_ctx *ctx, const tx_gemm_desc &d, const Maps &m, int64_t z, int kb_per_cta) {
  const bool a_mn = d.trans_a != 0, b_mn = d.trans_b == 0;
  if (a_mn && b_mn) return launch_tc<BN, true, true, MODE>(ctx, d, m, z, kb_per_cta);
  if (a_mn) return launch_tc<BN, true, false, MODE>(ctx, d, m, z, kb_per_cta);
  if (b_mn) return launch_tc<BN, false, true, MODE>(ctx, d, m, z, kb_per_cta);
  return launch_tc<BN, false, false, MODE>(ctx, d, m, z, kb_per_cta);
}

template <int MODE>
int launch_mode(tx_ctx *ctx, int bn, const tx_gemm_desc &d, const Maps &m, int64_t z, int kb_per_cta) {
  switch (bn) {
    case 256: return launch_bn<256, MODE>(ctx, d, m, z, kb_per_cta);
    case 64: return launch_bn<64, MODE>(ctx, d, m, z, kb_per_cta);
    default: return launch_bn<128, MODE>(ctx, d, m, z, kb_per_cta);
  }
}


#ifdef TX_TC_PERSISTENT_TU
template <int BN, bool A_MN, bool B_MN, int EW, bool BLO = false, int MODE = 0>
int launch_p(tx_ctx *ctx, const tx_gemm_desc &d, const Maps &m, const PWork &w, int smem, int max_grid) {
  auto kern = k_gemm_tcp<BN, A_MN, B_MN, EW, BLO, MODE>;
  static bool configured[64] = {};
  const int dev = ctx->device & 63;
  if (!configured[dev]) {
    TX_CUDA(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax));
    configured[dev] = true;
  }
  int grid = w.items < ctx->num_sms ? w.items : ctx->num_sms;
  if (max_grid > 0 && grid > max_grid) grid = max_grid;
  constexpr int threads = 64 + 32 * EW + PCfg<BN, BLO, MODE>::CONV_THREADS;
  kern<<<grid, threads, smem, ctx->stream>>>(m.a, m.b, m.c, m.s, m.p, m.b2, d, ctx->d_err, w, m.g);
  TX_LAUNCHED(ctx, "k_gemm_tcp");
  return TX_OK;
}

template <int BN, int EW, int MODE>
int launch_p_bn(tx_ctx *ctx, const tx_gemm_desc &d, const Maps &m, const PWork &w, int smem, int max_grid) {
  const bool a_mn = d.trans_a != 0, b_mn = d.trans_b == 0;
  if constexpr (MODE == 0) {
    if (d.B_lo) {  // split weights: forward layouts only (A K-major)
      if (a_mn) return TX_ERR_UNSUPPORTED;
      return b_mn ? launch_p<BN, false, true, EW, true>(ctx, d, m, w, smem, max_grid)
                  : launch_p<BN, false, false, EW, true>(ctx, d, m, w, smem, max_grid);
    }
  } else {
    if (d.B_lo) return TX_ERR_UNSUPPORTED;
  }
  if (a_mn && b_mn) return launch_p<BN, true, true, EW, false, MODE>(ctx, d, m, w, smem, max_grid);
  if (a_mn) return launch_p<BN, true, false, EW, false, MODE>(ctx, d, m, w, smem, max_grid);
  if (b_mn) return launch_p<BN, false, true, EW, false, MODE>(ctx, d, m, w, smem, max_grid);
  return launch_p<BN, false, false, EW, false, MODE>(ctx, d, m, w, smem, max_grid);
}

// Persistent launch of d (raw split partials when kb_per > 0, z = splits or
// batch) with operand mode MODE.  TX_ERR_UNSUPPORTED when the stages would
// not fit next to the epilogue's tiles (or a 3xTF32 tile is wider than 128).
// max_grid > 0 caps the CTA count (several tiles per CTA even when the tiles
// would fit one wave, so that one tile's epilogue overlaps the next's main loop).
template <int MODE>
int launch_persistent_impl(tx_ctx *ctx, int bn, const tx_gemm_desc &d, const Maps &m, int64_t z, int kb_per,
                           int max_grid) {
  if (MODE != 0 && bn > 128) return TX_ERR_UNSUPPORTED;
  const int stage = (TC_BM + bn * (d.B_lo ? 2 : 1)) * TC_BK * 4 * (MODE == 2 ? 2 : 1);
  const int kinds = 1 + (d.preact ? 1 : 0) + (d.dact ? 1 : 0) + (d.beta != 0.f ? 1 : 0);
  PWork w;
  w.ep_stride = kinds * 8192;
  w.col_part = m.col_part;
  w.conv_mask = m.conv_mask;
  // a GELU (or GELU') epilogue costs more than a 256-wide tile's main loop:
  // eight epilogue warps, when two stages still fit beside their tiles (also
  // for short reductions: with four warps on the K = 256 GELU' data gradients
  // the transformer step at batch 256 measured 4.34 against 4.21 ms)
  int ew = 4;
  if (MODE == 0 && bn == 256 && (d.act == TX_ACT_GELU || d.dact == TX_ACT_GELU) &&
      (kSmemMax - 1024 - kPTail - 8 * w.ep_stride) / stage >= 2)
    ew = 8;
  w.stages = (kSmemMax - 1024 - kPTail - ew * w.ep_stride) / stage;
  if (w.stages > 8) w.stages = 8;
  if (w.stages < 2) return TX_ERR_UNSUPPORTED;
  w.tiles_m = (int)((d.M + TC_BM - 1) / TC_BM);
  w.tiles_n = (int)((d.N + bn - 1) / bn);
  w.total_kb = (int)((d.K + TC_BK - 1) / TC_BK);
  w.kb_per = kb_per;
  const int64_t items = (int64_t)w.tiles_m * w.tiles_n * z;
  if (items > 0x7fffffff) return TX_ERR_UNSUPPORTED;
  w.items = (int)items;
  const int smem = 1024 + w.stages * stage + ew * w.ep_stride + kPTail;
  if constexpr (MODE != 0) {
    return bn == 64 ? launch_p_bn<64, 4, MODE>(ctx, d, m, w, smem, max_grid)
                    : launch_p_bn<128, 4, MODE>(ctx, d, m, w, smem, max_grid);
  } else {
    switch (bn) {
      case 256:
        return ew == 8 ? launch_p_bn<256, 8, MODE>(ctx, d, m, w, smem, max_grid)
                       : launch_p_bn<256, 4, MODE>(ctx, d, m, w, smem, max_grid);
      case 64: return launch_p_bn<64, 4, MODE>(ctx, d, m, w, smem, max_grid);
      default: return launch_p_bn<128, 4, MODE>(ctx, d, m, w, smem, max_grid);
    }
  }
}

#endif  // TX_TC_PERSISTENT_TU

}  // namespace
