// Fused multi-head attention on tcgen05 (kind::tf32), forward and backward.
//
// The transformer's attention block, as an imported graph states it
// (MatMul(Q, K^T) -> scale -> Softmax -> MatMul(., V) with the head split and
// merge as Reshape / Transpose around it, crates/tynx/src/interpreter/matrix.rs,
// softmax.rs:9-17), runs here as one kernel per direction, with one CTA per
// (sequence, head) and the whole sequence (<= 128 positions) in one tile:
//
//   forward   S = Q K^T (TMEM) -> P = softmax(scale * S) by rows (registers,
//             TF32-rounded into shared memory) -> O = P V (TMEM) -> O rows
//             stored into the merged [batch * seq, heads * dim] layout;
//   backward  S = Q K^T and dP = dO V^T (TMEM) -> P, D = rowsum(P * dP),
//             dS = P * (dP - D) * scale -> dV = P^T dO, dQ = dS K, dK = dS^T Q.
//
// Q, K, V, dO are read straight from the projections' [batch * seq, ld]
// row-major outputs (head h = columns h * 64 .. h * 64 + 63) by TMA, and dQ, dK,
// dV are written in the same layout, so no head split / merge copies, score,
// probability or score-gradient tensor ever reaches HBM (128 x 128 fp32 per
// head and layer: 64 MB per tensor at batch 256 x 4 heads).  P is recomputed
// by the backward from Q and K exactly as the forward computed it.
//
// Layouts in shared memory (all the UMMA descriptor forms of the tcgen05 GEMM
// in gemm_tc_kern.cuh): K-major operand tiles of 128 rows x 32 fp32 (128-byte
// swizzle: 16-byte chunk j of row r at chunk j ^ (r & 7)); MN-major tiles of
// 32 x 32 fp32 (128-byte swizzle with 32-byte atoms, as TMA writes them).  P
// and dS are written by the row-owning threads as K-major tiles; P^T and dS^T
// (the A operands of dV and dK, whose rows are keys) are written transposed,
// one fp32 per store, which a warp spreads over the 32 banks of one swizzled
// row.  Every mbarrier wait is bounded (~2 s); on expiry the CTA raises the
// context's error flag, skips the rest of its work and frees its TMEM.  No TMA
// multicast is used.
//
// Numerics (TF32 mode): operands are rounded to nearest TF32 (cvt.rna) in
// shared memory unless the caller states they already are; softmax is
// exp(x - max) * (1 / sum) in fp32 with the hardware exponential (__expf, a
// few ulp; the products around it are TF32).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.h"

namespace {

constexpr int kRows = 128;                        // sequence tile (queries and keys)
constexpr int kDim = 64;                          // head dimension
constexpr int kTile = kRows * kDim * 4;           // one [128 x 64] fp32 operand: 32 KB
constexpr int kSq = kRows * kRows * 4;            // one [128 x 128] fp32 tile: 64 KB
constexpr uint64_t kWaitNs = 2000000000ull;       // 2 s

__device__ __forceinline__ uint32_t su32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t gtime() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void bar_init(uint64_t *b, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(n));
}
__device__ __forceinline__ void bar_expect(uint64_t *b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bar_arrive(uint64_t *b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ bool bar_try(uint64_t *b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(su32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// bounded wait for phase 0 (every barrier here completes once)
__device__ __forceinline__ bool bar_wait(uint64_t *b, volatile int *abort_flag, int *err, int site) {
  if (bar_try(b, 0)) return true;
  const uint64_t t0 = gtime();
  while (true) {
    if (bar_try(b, 0)) return true;
    if (*abort_flag) return false;
    if (gtime() - t0 > kWaitNs) {
      *abort_flag = 1;
      if (atomicCAS(err, 0, DEVERR_TIMEOUT) == 0) err[1] = 100 + site;
      return false;
    }
  }
}
// wait regardless of the abort flag (copies in flight must land before the
// CTA's shared memory is released), still bounded
__device__ __forceinline__ void bar_drain(uint64_t *b) {
  const uint64_t t0 = gtime();
  while (!bar_try(b, 0) && gtime() - t0 < kWaitNs) {
  }
}

__device__ __forceinline__ void tma_2d(uint32_t dst, const CUtensorMap *map, uint64_t *b, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(map), "r"(su32(b)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void mma_commit(uint64_t *b) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(b))
               : "memory");
}

__device__ __forceinline__ void mma_tf32(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ float rn_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// UMMA shared-memory descriptor (version 1): K-major 128-byte swizzle (layout
// 2), MN-major 128-byte swizzle with 32-byte atoms (layout 1)
__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)layout << 61;
  return d;
}
// k-th 8-deep slice of a K-major [rows x 32] tile
__device__ __forceinline__ uint64_t kdesc(uint32_t base, int k) { return sdesc(base + k * 32, 16, 1024, 2); }
// k-th 8-deep slice of an MN-major [32 K x (n/32) blocks of 32] stage
__device__ __forceinline__ uint64_t ndesc(uint32_t base, int k) { return sdesc(base + k * 1024, 4096, 512, 1); }

// instruction descriptor: fp32 accumulate, tf32 A and B, M x N
__device__ __forceinline__ uint32_t idesc(int m, int n, bool a_mn, bool b_mn) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void tld32(uint32_t taddr, float (&v)[32]) {
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

// tcgen05.ld without the wait; the registers are valid after tld_wait() and
// regs_after_wait(), which keeps every use of them behind the wait
__device__ __forceinline__ void tld32_issue(uint32_t taddr, uint32_t (&r)[32]) {
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
__device__ __forceinline__ void tld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void regs_after_wait(uint32_t (&r)[32]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
                 "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]),
                 "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]),
                 "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]),
                 "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]),
                 "+r"(r[31]));
}
// a thread's whole 128-column row of a TMEM tile: four loads in flight, one wait
__device__ __forceinline__ void tld128(uint32_t trow, float (&v)[128]) {
  uint32_t r0[32], r1[32], r2[32], r3[32];
  tld32_issue(trow, r0);
  tld32_issue(trow + 32, r1);
  tld32_issue(trow + 64, r2);
  tld32_issue(trow + 96, r3);
  tld_wait();
  regs_after_wait(r0);
  regs_after_wait(r1);
  regs_after_wait(r2);
  regs_after_wait(r3);
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    v[j] = __uint_as_float(r0[j]);
    v[32 + j] = __uint_as_float(r1[j]);
    v[64 + j] = __uint_as_float(r2[j]);
    v[96 + j] = __uint_as_float(r3[j]);
  }
}
// 32 columns of a thread's TMEM row from registers (visible to later loads of
// this thread after tst_wait())
__device__ __forceinline__ void tst32(uint32_t taddr, const float *v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
      "%13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, "
      "%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}
__device__ __forceinline__ void tst_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Softmax of scale * row over its valid keys, in place: v becomes P (0 on
// masked keys and on rows past the sequence).  exp via the __expf intrinsic.
__device__ __forceinline__ void softmax_row(float (&v)[128], float scale, int seq, bool live) {
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < 128; ++j) {
    v[j] *= scale;
    if (j < seq) m = fmaxf(m, v[j]);
  }
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < 128; ++j) {
    v[j] = j < seq ? __expf(v[j] - m) : 0.f;
    sum += v[j];
  }
  const float inv = live ? 1.0f / sum : 0.f;
#pragma unroll
  for (int j = 0; j < 128; ++j) v[j] *= inv;
}

// Round `bytes` of shared memory to TF32 in place (nt threads, float4 steps).
__device__ __forceinline__ void round_region(uint8_t *p, int bytes, int t, int nt = 128) {
  float4 *q = reinterpret_cast<float4 *>(p);
  for (int i = t; i < bytes / 16; i += nt) {
    float4 v = q[i];
    q[i] = make_float4(rn_tf32(v.x), rn_tf32(v.y), rn_tf32(v.z), rn_tf32(v.w));
  }
}

// Row r's 32 values of K-block c into a K-major [128 x 32] tile (float4 stores).
__device__ __forceinline__ void put_row(uint8_t *tile, int r, const float (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 8; ++j)
    *reinterpret_cast<float4 *>(tile + r * 128 + ((j ^ (r & 7)) << 4)) =
        make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
}

// Column r (a query) of the transposed matrix: element (row = key 32c + j,
// k = query r) of a K-major tile set whose K blocks are 32 queries wide.
__device__ __forceinline__ void put_col(uint8_t *tiles, int r, int c, const float (&v)[32]) {
  uint8_t *t = tiles + (r >> 5) * (kRows * 128);
  const int q = r & 31, qc = q >> 2, qo = (q & 3) * 4;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int key = c * 32 + j;
    *reinterpret_cast<float *>(t + key * 128 + ((qc ^ (key & 7)) << 4) + qo) = v[j];
  }
}

// Store 32 columns of a thread's row of a TMEM accumulator (at taddr) to
// global memory (row < seq only; all lanes take part in the TMEM load).
__device__ __forceinline__ void store_chunk(uint32_t taddr, float *dst, bool live, bool acc, bool rnd) {
  float v[32];
  tld32(taddr, v);
  if (!live) return;
  float4 *d4 = reinterpret_cast<float4 *>(dst);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float4 w = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    if (acc) {
      const float4 o = d4[j];
      w.x += o.x;
      w.y += o.y;
      w.z += o.z;
      w.w += o.w;
    }
    if (rnd) w = make_float4(rn_tf32(w.x), rn_tf32(w.y), rn_tf32(w.z), rn_tf32(w.w));
    d4[j] = w;
  }
}

// Named barrier of the two epilogue warps that share a TMEM lane quadrant.
__device__ __forceinline__ void pair_sync(int quad) {
  asm volatile("bar.sync %0, 64;" ::"r"(1 + quad) : "memory");
}

// ---- forward --------------------------------------------------------------------------------
// smem: Q (K-major, 2 x 16 KB) | K (K-major) | V (MN-major, 4 key blocks x 2 x 4 KB) | tail;
// P (K-major, 4 key blocks x 16 KB) overlays Q and K once S has been computed.
constexpr int kFwdSmem = 3 * kTile + 1024 /*tail*/ + 1024 /*align*/;

__global__ void __launch_bounds__(192, 2)
    k_attn_fwd(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
               const __grid_constant__ CUtensorMap mv, float *__restrict__ out, int64_t ldo, int seq,
               int heads, float scale, int flags, int *err) {
  extern __shared__ uint8_t raw[];
  uint8_t *sm = (uint8_t *)(((uintptr_t)raw + 1023) & ~(uintptr_t)1023);
  uint8_t *sq = sm, *sk = sm + kTile, *sv = sm + 2 * kTile, *sp = sm;
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + 3 * kTile);
  uint64_t *b_ld = bars, *b_cv = bars + 1, *b_s = bars + 2, *b_p = bars + 3, *b_o = bars + 4;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 8);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x / heads, h = blockIdx.x % heads;
  const int row0 = b * seq, col0 = h * kDim;
  const bool rounded = flags & 1, round_out = flags & 2;

  if (threadIdx.x == 0) {
    bar_init(b_ld, 1);
    bar_init(b_cv, 128);
    bar_init(b_s, 1);
    bar_init(b_p, 128);
    bar_init(b_o, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_holder)),
                 "r"(256));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      bar_expect(b_ld, 3 * kTile);
      for (int j = 0; j < kDim / 32; ++j) {
        tma_2d(su32(sq + j * 16384), &mq, b_ld, col0 + 32 * j, row0);
        tma_2d(su32(sk + j * 16384), &mk, b_ld, col0 + 32 * j, row0);
      }
      for (int kb = 0; kb < 4; ++kb)
        for (int j = 0; j < kDim / 32; ++j)
          tma_2d(su32(sv + (kb * (kDim / 32) + j) * 4096), &mv, b_ld, col0 + 32 * j, row0 + 32 * kb);
      if (bar_wait(rounded ? b_ld : b_cv, abort_flag, err, 1)) {
        fence_after();
        const uint32_t ids = idesc(128, 128, false, false);
        for (int j = 0; j < kDim / 32; ++j)
          for (int k = 0; k < 4; ++k)
            mma_tf32(tmem, kdesc(su32(sq + j * 16384), k), kdesc(su32(sk + j * 16384), k), ids, (j | k) ? 1u : 0u);
        mma_commit(b_s);
        if (bar_wait(b_p, abort_flag, err, 2)) {
          fence_after();
          const uint32_t ido = idesc(128, kDim, false, true);
          for (int kb = 0; kb < 4; ++kb)
            for (int k = 0; k < 4; ++k)
              mma_tf32(tmem + 128, kdesc(su32(sp + kb * 16384), k),
                       ndesc(su32(sv + kb * (kDim / 32) * 4096), k), ido, (kb | k) ? 1u : 0u);
          mma_commit(b_o);
        }
      }
      bar_drain(b_ld);  // every copy has landed before the CTA can exit
    }
  } else if (warp >= 2) {
    const int t = threadIdx.x - 64;
    if (!rounded) {
      if (bar_wait(b_ld, abort_flag, err, 3)) round_region(sm, 3 * kTile, t);
      fence_async_smem();
      bar_arrive(b_cv);
    }
    const int quad = warp & 3, r = quad * 32 + lane;
    const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16);
    const bool ok_s = __all_sync(0xffffffffu, bar_wait(b_s, abort_flag, err, 4));
    fence_after();
    if (ok_s) {
      float p[128];
      tld128(trow, p);
      softmax_row(p, scale, seq, r < seq);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float q[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) q[j] = rn_tf32(p[c * 32 + j]);
        put_row(sp + c * 16384, r, q);
      }
    }
    fence_async_smem();
    bar_arrive(b_p);
    const bool ok_o = __all_sync(0xffffffffu, ok_s && bar_wait(b_o, abort_flag, err, 5));
    fence_after();
    if (ok_o) {
      float *dst = out + (int64_t)(row0 + r) * ldo + col0;
#pragma unroll 1
      for (int c = 0; c < kDim / 32; ++c) {
        float v[32];
        tld32(trow + 128 + c * 32, v);
        if (r >= seq) continue;
        float4 *d4 = reinterpret_cast<float4 *>(dst + c * 32);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float4 w = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          if (round_out) w = make_float4(rn_tf32(w.x), rn_tf32(w.y), rn_tf32(w.z), rn_tf32(w.w));
          d4[j] = w;
        }
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256));
  }
}

// ---- backward -------------------------------------------------------------------------------
// smem regions of 32 KB: R0 Q (K-major) | R1 K (K-major) | R2 dO (K-major) | R3 V (K-major) |
// R4 dO (MN-major; then Q MN-major) | R5 K (MN-major) | tail.  P^T (64 KB) overlays R0..R1
// after S and dP are computed; dS (64 KB) overlays R2..R3; dS^T overlays P^T once dV is done.
// TMEM columns: S 0..127 | dP 128..255 | dV 256..319 | dQ 320..383 | dK 384..447.
// Eight epilogue warps, two per TMEM lane quadrant: the warp of half h takes
// key columns 64h .. 64h + 63 of its 32 rows (score chunks 2h, 2h + 1) and
// output chunk h of dV, dQ and dK; the row max, row sum and rowsum(P * dP) of
// the two halves meet in the tail (3 x [2][128] floats after the barriers).
constexpr int kBwdEpi = 256;                      // epilogue threads
constexpr int kBwdTail = 4096;
constexpr int kBwdSmem = 6 * kTile + kBwdTail + 1024;

__global__ void __launch_bounds__(64 + kBwdEpi, 1)
    k_attn_bwd(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
               const __grid_constant__ CUtensorMap mv, const __grid_constant__ CUtensorMap mdo,
               const __grid_constant__ CUtensorMap mqn, const __grid_constant__ CUtensorMap mkn,
               const __grid_constant__ CUtensorMap mdon, float *__restrict__ dq, float *__restrict__ dk,
               float *__restrict__ dv, int64_t ldg, int seq, int heads, float scale, int flags, int *err) {
  extern __shared__ uint8_t raw[];
  uint8_t *sm = (uint8_t *)(((uintptr_t)raw + 1023) & ~(uintptr_t)1023);
  uint8_t *R0 = sm, *R2 = sm + 2 * kTile, *R4 = sm + 4 * kTile, *R5 = sm + 5 * kTile;
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + 6 * kTile);
  uint64_t *b_ld1 = bars, *b_ld2 = bars + 1, *b_ld3 = bars + 2, *b_cv = bars + 3, *b_cv3 = bars + 4,
           *b_s = bars + 5, *b_pt = bars + 6, *b_ds = bars + 7, *b_dv = bars + 8, *b_dq = bars + 9,
           *b_dst = bars + 10, *b_dk = bars + 11;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 16);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);
  float *xmax = reinterpret_cast<float *>(sm + 6 * kTile + 1024);  // [2][128] per half
  float *xsum = xmax + 2 * kRows, *xd = xsum + 2 * kRows;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x / heads, h = blockIdx.x % heads;
  const int row0 = b * seq, col0 = h * kDim;
  const bool rounded = flags & 1, acc = flags & 2, rnd = flags & 4;

  if (threadIdx.x == 0) {
    bar_init(b_ld1, 1);
    bar_init(b_ld2, 1);
    bar_init(b_ld3, 1);
    bar_init(b_cv, kBwdEpi);
    bar_init(b_cv3, kBwdEpi);
    bar_init(b_s, 1);
    bar_init(b_pt, kBwdEpi);
    bar_init(b_ds, kBwdEpi);
    bar_init(b_dv, 1);
    bar_init(b_dq, 1);
    bar_init(b_dst, kBwdEpi);
    bar_init(b_dk, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_holder)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      bool issued3 = false;
      bar_expect(b_ld1, 4 * kTile);
      for (int j = 0; j < kDim / 32; ++j) {
        tma_2d(su32(R0 + j * 16384), &mq, b_ld1, col0 + 32 * j, row0);
        tma_2d(su32(R0 + kTile + j * 16384), &mk, b_ld1, col0 + 32 * j, row0);
        tma_2d(su32(R2 + j * 16384), &mdo, b_ld1, col0 + 32 * j, row0);
        tma_2d(su32(R2 + kTile + j * 16384), &mv, b_ld1, col0 + 32 * j, row0);
      }
      bar_expect(b_ld2, 2 * kTile);
      for (int kb = 0; kb < 4; ++kb)
        for (int j = 0; j < kDim / 32; ++j) {
          const int off = (kb * (kDim / 32) + j) * 4096;
          tma_2d(su32(R4 + off), &mdon, b_ld2, col0 + 32 * j, row0 + 32 * kb);
          tma_2d(su32(R5 + off), &mkn, b_ld2, col0 + 32 * j, row0 + 32 * kb);
        }
      const uint32_t id_sq = idesc(128, 128, false, false), id_d = idesc(128, kDim, false, true);
      bool ok = rounded ? (bar_wait(b_ld1, abort_flag, err, 11) && bar_wait(b_ld2, abort_flag, err, 12))
                        : bar_wait(b_cv, abort_flag, err, 13);
      if (ok) {
        fence_after();
        for (int j = 0; j < kDim / 32; ++j)
          for (int k = 0; k < 4; ++k) {
            const uint32_t a = (j | k) ? 1u : 0u;
            mma_tf32(tmem, kdesc(su32(R0 + j * 16384), k), kdesc(su32(R0 + kTile + j * 16384), k), id_sq, a);
            mma_tf32(tmem + 128, kdesc(su32(R2 + j * 16384), k), kdesc(su32(R2 + kTile + j * 16384), k), id_sq,
                     a);
          }
        mma_commit(b_s);
      }
      ok = ok && bar_wait(b_pt, abort_flag, err, 14);
      if (ok) {  // dV = P^T dO: rows are keys, K = queries
        fence_after();
        for (int kb = 0; kb < 4; ++kb)
          for (int k = 0; k < 4; ++k)
            mma_tf32(tmem + 256, kdesc(su32(R0 + kb * 16384), k), ndesc(su32(R4 + kb * (kDim / 32) * 4096), k),
                     id_d, (kb | k) ? 1u : 0u);
        mma_commit(b_dv);
      }
      ok = ok && bar_wait(b_ds, abort_flag, err, 15);
      if (ok) {  // dQ = dS K: rows are queries, K = keys
        fence_after();
        for (int kb = 0; kb < 4; ++kb)
          for (int k = 0; k < 4; ++k)
            mma_tf32(tmem + 320, kdesc(su32(R2 + kb * 16384), k), ndesc(su32(R5 + kb * (kDim / 32) * 4096), k),
                     id_d, (kb | k) ? 1u : 0u);
        mma_commit(b_dq);
      }
      ok = ok && bar_wait(b_dv, abort_flag, err, 16);  // R4 (dO) is free again
      if (ok) {
        fence_after();
        bar_expect(b_ld3, kTile);
        for (int kb = 0; kb < 4; ++kb)
          for (int j = 0; j < kDim / 32; ++j)
            tma_2d(su32(R4 + (kb * (kDim / 32) + j) * 4096), &mqn, b_ld3, col0 + 32 * j, row0 + 32 * kb);
        issued3 = true;
      }
      ok = ok && bar_wait(rounded ? b_ld3 : b_cv3, abort_flag, err, 17) && bar_wait(b_dst, abort_flag, err, 18);
      if (ok) {  // dK = dS^T Q: rows are keys, K = queries
        fence_after();
        for (int kb = 0; kb < 4; ++kb)
          for (int k = 0; k < 4; ++k)
            mma_tf32(tmem + 384, kdesc(su32(R0 + kb * 16384), k), ndesc(su32(R4 + kb * (kDim / 32) * 4096), k),
                     id_d, (kb | k) ? 1u : 0u);
        mma_commit(b_dk);
      }
      bar_drain(b_ld1);
      bar_drain(b_ld2);
      if (issued3) bar_drain(b_ld3);
    }
  } else if (warp >= 2) {
    const int t = threadIdx.x - 64;     // 0 .. kBwdEpi - 1
    const int half = (warp - 2) >> 2;   // key columns 64 * half ..
    const int quad = warp & 3, r = quad * 32 + lane;
    const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16);
    const bool live = r < seq;
    if (!rounded) {
      if (bar_wait(b_ld1, abort_flag, err, 21)) round_region(sm, 4 * kTile, t, kBwdEpi);
      if (bar_wait(b_ld2, abort_flag, err, 22)) round_region(R4, 2 * kTile, t, kBwdEpi);
      fence_async_smem();
      bar_arrive(b_cv);
    }
    bool ok = __all_sync(0xffffffffu, bar_wait(b_s, abort_flag, err, 23));
    fence_after();
    // Softmax of this half's 64 keys against the row's max and sum (every
    // pair barrier below is reached by both warps whatever `ok` says).
    float p[64];
    float m = -INFINITY;
    if (ok) {
      uint32_t r0[32], r1[32];
      tld32_issue(trow + half * 64, r0);
      tld32_issue(trow + half * 64 + 32, r1);
      tld_wait();
      regs_after_wait(r0);
      regs_after_wait(r1);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        p[j] = __uint_as_float(r0[j]) * scale;
        p[32 + j] = __uint_as_float(r1[j]) * scale;
      }
#pragma unroll
      for (int j = 0; j < 64; ++j)
        if (half * 64 + j < seq) m = fmaxf(m, p[j]);
    }
    xmax[half * kRows + r] = m;
    pair_sync(quad);
    m = fmaxf(xmax[r], xmax[kRows + r]);
    float sum = 0.f;
    if (ok) {
#pragma unroll
      for (int j = 0; j < 64; ++j) {
        p[j] = half * 64 + j < seq ? __expf(p[j] - m) : 0.f;
        sum += p[j];
      }
    }
    xsum[half * kRows + r] = sum;
    pair_sync(quad);
    sum = xsum[r] + xsum[kRows + r];
    const float inv = live ? 1.0f / sum : 0.f;
    float dsum = 0.f;
    if (ok) {
#pragma unroll
      for (int j = 0; j < 64; ++j) p[j] *= inv;
      // P^T for dV, and this half's share of D = rowsum(P * dP)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float g[32], q[32];
        tld32(trow + 128 + (2 * half + c) * 32, g);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          dsum += p[c * 32 + j] * g[j];
          q[j] = rn_tf32(p[c * 32 + j]);
        }
        put_col(R0, r, 2 * half + c, q);
      }
    }
    xd[half * kRows + r] = dsum;
    fence_async_smem();
    bar_arrive(b_pt);
    pair_sync(quad);
    dsum = xd[r] + xd[kRows + r];
    if (ok) {  // dS rows for dQ; dS also replaces dP in TMEM for the dS^T pass
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int cc = 2 * half + c;
        float g[32];
        tld32(trow + 128 + cc * 32, g);
#pragma unroll
        for (int j = 0; j < 32; ++j) g[j] = rn_tf32(p[c * 32 + j] * (g[j] - dsum) * scale);
        put_row(R2 + cc * 16384, r, g);
        tst32(trow + 128 + cc * 32, g);
      }
      tst_wait();
    }
    fence_async_smem();
    bar_arrive(b_ds);
    // dV rows (lane = key) while dQ runs
    ok = __all_sync(0xffffffffu, ok && bar_wait(b_dv, abort_flag, err, 24));
    fence_after();
    if (ok) {
      store_chunk(trow + 256 + half * 32, dv + (int64_t)(row0 + r) * ldg + col0 + half * 32, live, acc, rnd);
      // dS^T into the P^T region for dK
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        float g[32];
        tld32(trow + 128 + (2 * half + c) * 32, g);
        put_col(R0, r, 2 * half + c, g);
      }
    }
    fence_async_smem();
    bar_arrive(b_dst);
    if (!rounded) {
      if (ok && bar_wait(b_ld3, abort_flag, err, 25)) round_region(R4, kTile, t, kBwdEpi);
      fence_async_smem();
      bar_arrive(b_cv3);
    }
    ok = __all_sync(0xffffffffu, ok && bar_wait(b_dq, abort_flag, err, 26));
    fence_after();
    if (ok) store_chunk(trow + 320 + half * 32, dq + (int64_t)(row0 + r) * ldg + col0 + half * 32, live, acc, rnd);
    ok = __all_sync(0xffffffffu, ok && bar_wait(b_dk, abort_flag, err, 27));
    fence_after();
    if (ok) store_chunk(trow + 384 + half * 32, dk + (int64_t)(row0 + r) * ldg + col0 + half * 32, live, acc, rnd);
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
}

// ---- host -----------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 g_enc = nullptr;
std::once_flag g_enc_once;

bool encoder() {
  std::call_once(g_enc_once, [] {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_enc = (PFN_cuTensorMapEncodeTiled_v12000)fn;
  });
  return g_enc != nullptr;
}

// 2-D map over a [rows x cols] fp32 row-major matrix with row stride ld:
// K-major boxes {32, 128} (128-byte swizzle) or MN-major boxes {32, 32}
// (128-byte swizzle, 32-byte atoms)
bool map2d(CUtensorMap *m, const float *base, int64_t rows, int64_t ld, bool mn) {
  cuuint64_t dims[2] = {(cuuint64_t)ld, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 4)};
  cuuint32_t box[2] = {32u, mn ? 32u : 128u};
  cuuint32_t es[2] = {1u, 1u};
  return g_enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)base, dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE,
               mn ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int check_args(tx_ctx *ctx, std::initializer_list<const float *> ptrs, int64_t ld, int64_t batch, int64_t seq,
               int64_t heads, int64_t dim) {
  if (dim != kDim) return tx_fail(ctx, TX_ERR_UNSUPPORTED, "fused attention: head dimension must be 64");
  if (seq < 1 || seq > kRows) return tx_fail(ctx, TX_ERR_UNSUPPORTED, "fused attention: sequence length 1..128");
  if (batch < 1 || heads < 1 || batch * heads > 0x7fffffff || batch * seq > 0x7fffffff)
    return tx_fail(ctx, TX_ERR_INVALID, "fused attention: bad batch or head count");
  if (ld < heads * dim || (ld & 3)) return tx_fail(ctx, TX_ERR_INVALID, "fused attention: row stride");
  for (const float *p : ptrs)
    if (!p || ((uintptr_t)p & 15)) return tx_fail(ctx, TX_ERR_INVALID, "fused attention: 16-byte aligned buffers");
  if (!encoder()) return tx_fail(ctx, TX_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
  return TX_OK;
}

}  // namespace

extern "C" int tx_attention_fwd(tx_ctx *ctx, const float *q, const float *k, const float *v, int64_t ld_in,
                                float *out, int64_t ld_out, int64_t batch, int64_t seq, int64_t heads,
                                int64_t head_dim, float scale, int flags) {
  if (!ctx) return TX_ERR_INVALID;
  TX_TRY(check_args(ctx, {q, k, v, out}, ld_in, batch, seq, heads, head_dim));
  if (ld_out < heads * head_dim || (ld_out & 3)) return tx_fail(ctx, TX_ERR_INVALID, "fused attention: output row stride");
  CUtensorMap mq, mk, mv;
  const int64_t rows = batch * seq;
  if (!map2d(&mq, q, rows, ld_in, false) || !map2d(&mk, k, rows, ld_in, false) || !map2d(&mv, v, rows, ld_in, true))
    return tx_fail(ctx, TX_ERR_UNSUPPORTED, "fused attention: tensor map");
  static bool attr = false;
  if (!attr) {
    TX_CUDA(ctx, cudaFuncSetAttribute(k_attn_fwd, cudaFuncAttributeMaxDynamicSharedMemorySize, kFwdSmem));
    attr = true;
  }
  k_attn_fwd<<<(unsigned)(batch * heads), 192, kFwdSmem, ctx->stream>>>(mq, mk, mv, out, ld_out, (int)seq,
                                                                       (int)heads, scale, flags & 3, ctx->d_err);
  TX_LAUNCHED(ctx, "k_attn_fwd");
  return TX_OK;
}

extern "C" int tx_attention_bwd(tx_ctx *ctx, const float *q, const float *k, const float *v, int64_t ld_in,
                                const float *dout, int64_t ld_dout, float *dq, float *dk, float *dv,
                                int64_t ld_grad, int64_t batch, int64_t seq, int64_t heads, int64_t head_dim,
                                float scale, int flags) {
  if (!ctx) return TX_ERR_INVALID;
  TX_TRY(check_args(ctx, {q, k, v, dout, dq, dk, dv}, ld_in, batch, seq, heads, head_dim));
  if (ld_dout < heads * head_dim || (ld_dout & 3) || ld_grad < heads * head_dim || (ld_grad & 3))
    return tx_fail(ctx, TX_ERR_INVALID, "fused attention: gradient row stride");
  const int64_t rows = batch * seq;
  CUtensorMap mq, mk, mv, mdo, mqn, mkn, mdon;
  if (!map2d(&mq, q, rows, ld_in, false) || !map2d(&mk, k, rows, ld_in, false) ||
      !map2d(&mv, v, rows, ld_in, false) || !map2d(&mdo, dout, rows, ld_dout, false) ||
      !map2d(&mqn, q, rows, ld_in, true) || !map2d(&mkn, k, rows, ld_in, true) ||
      !map2d(&mdon, dout, rows, ld_dout, true))
    return tx_fail(ctx, TX_ERR_UNSUPPORTED, "fused attention: tensor map");
  static bool attr = false;
  if (!attr) {
    TX_CUDA(ctx, cudaFuncSetAttribute(k_attn_bwd, cudaFuncAttributeMaxDynamicSharedMemorySize, kBwdSmem));
    attr = true;
  }
  k_attn_bwd<<<(unsigned)(batch * heads), 64 + kBwdEpi, kBwdSmem, ctx->stream>>>(
      mq, mk, mv, mdo, mqn, mkn, mdon, dq, dk, dv, ld_grad, (int)seq, (int)heads, scale, flags & 7, ctx->d_err);
  TX_LAUNCHED(ctx, "k_attn_bwd");
  return TX_OK;
}
