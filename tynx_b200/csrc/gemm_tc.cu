// Host side of the tcgen05 contraction: tensor maps, tile and split choice,
// and the dispatch between the one-tile, CTA-pair and persistent kernels
// (kernels in gemm_tc_kern.cuh, instantiated by gemm_tc_m0/m1/m2/pair/pers.cu).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "common.h"
#include "gemm_tc.cuh"

using namespace tx_tc;

namespace {

int launch_any(tx_ctx *ctx, int mode, int bn, const tx_gemm_desc &d, const Maps &m, int64_t z,
               int kb_per_cta) {
  switch (mode) {
    case 0: return launch_mode0(ctx, bn, d, m, z, kb_per_cta);
    case 2: return launch_mode2(ctx, bn, d, m, z, kb_per_cta);
    default: return launch_mode1(ctx, bn, d, m, z, kb_per_cta);
  }
}

// ---- host side ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

bool load_encode() {
  std::call_once(g_encode_once, [] {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
  });
  return g_encode != nullptr;
}

// 3-D fp32 tensor map: dims {inner, outer, batch}; box {32, box_outer, 1}; 128-byte
// swizzle (32-byte atomicity for MN-major operands, see smem_desc).
bool make_map(CUtensorMap *map, const float *base, int64_t inner, int64_t outer, int64_t ld,
              int64_t batch, int64_t batch_stride, int box_outer, bool mn_major) {
  cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)outer, (cuuint64_t)batch};
  int64_t bs = batch > 1 ? batch_stride : ld * outer;
  cuuint64_t strides[2] = {(cuuint64_t)(ld * 4), (cuuint64_t)(((bs * 4) + 15) & ~int64_t(15))};
  cuuint32_t box[3] = {32u, (cuuint32_t)box_outer, 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void *)base, dims, strides, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 4-D map of an MN-major operand stored [batch][outer = K][ld] with inner = MN
// a multiple of 32: dims {32, K, MN / 32, batch}, so a box {32, 32, nblk, 1}
// brings nblk consecutive 32-column blocks in one copy (the 128-byte swizzle
// with 32-byte atoms, as the per-block boxes).
bool make_map_mn4(CUtensorMap *map, const float *base, int64_t inner, int64_t outer, int64_t ld, int64_t batch,
                  int64_t batch_stride, int nblk) {
  if (inner % 32 || nblk < 1 || nblk > 8) return false;
  cuuint64_t dims[4] = {32u, (cuuint64_t)outer, (cuuint64_t)(inner / 32), (cuuint64_t)batch};
  int64_t bs = batch > 1 ? batch_stride : ld * outer;
  cuuint64_t strides[3] = {(cuuint64_t)(ld * 4), 128u, (cuuint64_t)(((bs * 4) + 15) & ~int64_t(15))};
  cuuint32_t box[4] = {32u, 32u, (cuuint32_t)nblk, 1u};
  cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (void *)base, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 4-D map over a channels-last [n][h][w][c] tensor (dims {c, w, h, n}) whose
// boxes step estr_w / estr_h elements along w / h: the operand tiles of an
// implicit-GEMM convolution.  Coordinates outside the tensor read zeros.
bool make_map_4d(CUtensorMap *map, const ConvTensor &t, const uint32_t box[4], uint32_t estr_w, uint32_t estr_h,
                 bool mn_major) {
  if (!t.base || ((uintptr_t)t.base & 15) || (t.c & 3)) return false;
  cuuint64_t dims[4] = {(cuuint64_t)t.c, (cuuint64_t)t.w, (cuuint64_t)t.h, (cuuint64_t)t.n};
  cuuint64_t strides[3] = {(cuuint64_t)(t.c * 4), (cuuint64_t)(t.w * t.c * 4), (cuuint64_t)(t.h * t.w * t.c * 4)};
  cuuint32_t bx[4] = {box[0], box[1], box[2], box[3]};
  cuuint32_t estr[4] = {1u, estr_w, estr_h, 1u};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (void *)t.base, dims, strides, bx, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Output-side 3-D view [rows][wsplit][N] (element strides sw, sr) with
// 32 x 32-element boxes: an output chunk of 32 GEMM rows is min(wsplit, 32)
// view columns by 32 / that many view rows.
bool make_view_map(CUtensorMap *map, const float *base, int64_t N, int wsplit, int64_t rows, int64_t sw,
                   int64_t sr) {
  if (!base || ((uintptr_t)base & 15) || (sw & 3) || (sr & 3)) return false;
  const uint32_t bw = wsplit < 32 ? (uint32_t)wsplit : 32u;
  cuuint64_t dims[3] = {(cuuint64_t)N, (cuuint64_t)wsplit, (cuuint64_t)rows};
  cuuint64_t strides[2] = {(cuuint64_t)(sw * 4), (cuuint64_t)(sr * 4)};
  cuuint32_t box[3] = {32u, bw, 32u / bw};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void *)base, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// A row-major [batch][M][N] fp32 tensor TMA can tile: 16-byte aligned base,
// row and batch strides that are 16-byte multiples.
bool tma_tileable(const float *p, int64_t ld, int64_t batch, int64_t stride) {
  return p && ((uintptr_t)p & 15) == 0 && (ld & 3) == 0 && (batch <= 1 || (stride & 3) == 0);
}

// Output-side maps (32 x 32 boxes, 128-byte swizzle); false: use the
// register epilogue instead.
bool make_epilogue_maps(Maps &m, const tx_gemm_desc &d, int64_t z) {
  if (!tma_tileable(d.C, d.ldc, z, d.stride_c)) return false;
  if (d.dact && !tma_tileable(d.dact_src, d.ld_dact, z, d.stride_c)) return false;
  if (d.preact && !tma_tileable(d.preact, d.ld_preact, z, d.stride_c)) return false;
  if (!make_map(&m.c, d.C, d.N, d.M, d.ldc, z, d.stride_c, 32, false)) return false;
  if (d.dact && !make_map(&m.s, d.dact_src, d.N, d.M, d.ld_dact, z, d.stride_c, 32, false)) return false;
  if (d.preact && !make_map(&m.p, d.preact, d.N, d.M, d.ld_preact, z, d.stride_c, 32, false)) return false;
  m.tma_epi = 1;
  return true;
}

struct Tiling {
  int bn = 128;
  int splits = 1;
};


// Pick the tile width and the K split from a small cost model: waves of CTAs
// times the per-CTA k-block work (one 128 x BN x 32 step costs about BN + 96
// "column units" including the fixed TMA/commit latency), plus the traffic of
// the split reduction.  1 unit ~ 1.5 ns at the TF32 rate of one SM.
Tiling pick_tiling(tx_ctx *ctx, int64_t M, int64_t N, int64_t K, int64_t batch, int max_bn) {
  Tiling best;
  double best_cost = 1e300;
  const int total_kb = (int)((K + TC_BK - 1) / TC_BK);
  const int cands[3] = {256, 128, 64};
  for (int bn : cands) {
    if (bn > max_bn) continue;
    if (bn > 64 && N <= bn / 2) continue;  // mostly-empty tiles
    const int64_t tiles = ((M + TC_BM - 1) / TC_BM) * ((N + bn - 1) / bn) * batch;
    int max_split = 1;
    if (batch == 1 && tiles < ctx->num_sms && total_kb >= 16) {
      int64_t want = (ctx->num_sms + tiles - 1) / tiles;
      int64_t most = total_kb / 8;  // at least 8 k-blocks (K = 256) per split
      max_split = (int)(want < most ? want : most);
      // many splits only while their partial tiles stay small (a weight
      // gradient with a tiny output and a reduction over every pixel)
      const int cap = (double)M * N * 4 * 128 <= 64.0 * (1 << 20) ? 128 : 32;
      if (max_split > cap) max_split = cap;
    }
    for (int s = 1; s <= max_split; s = s < 4 ? s + 1 : s * 2) {
      const int kb_per = (total_kb + s - 1) / s;
      const int64_t ctas = tiles * s;
      const int64_t waves = (ctas + ctx->num_sms - 1) / ctx->num_sms;
      double cost = (double)waves * kb_per * (bn + 96) * 1.5e-3;  // microseconds
      if (s > 1) cost += 2.0 + (double)(s + 1) * M * N * 4 / 5.0e6;  // reduce: ~5 TB/s
      if (cost < best_cost) {
        best_cost = cost;
        best.bn = bn;
        best.splits = s;
      }
    }
  }
  return best;
}

}  // namespace

namespace {

// mode: 0 raw fp32 operands (hardware truncation), 1 TF32 round-to-nearest, 2 3xTF32.
// cv (or null): gathered operands of an implicit-GEMM convolution.
int tc_product(tx_ctx *ctx, const tx_gemm_desc &desc, int mode, FusedSum *fs, const ConvGemm *cv) {
  tx_gemm_desc d = desc;
  if (d.K <= 0 || d.M <= 0 || d.N <= 0) return TX_ERR_UNSUPPORTED;
  const int64_t batch = d.batch > 1 ? d.batch : 1;
  if (d.M >= (1ll << 31) || d.N >= (1ll << 31) || d.K >= (1ll << 31) || batch > 65535)
    return TX_ERR_UNSUPPORTED;
  // TMA: 16-byte aligned bases and row strides that are 16-byte multiples
  if (((uintptr_t)d.A & 15) || ((uintptr_t)d.B & 15) || (d.lda & 3) || (d.ldb & 3))
    return TX_ERR_UNSUPPORTED;
  if (batch > 1 && ((d.stride_a & 3) || (d.stride_b & 3))) return TX_ERR_UNSUPPORTED;
  // one A for every batch entry: its tensor map has a single batch entry and
  // the kernels load it at batch 0
  const bool a_shared = (d.flags & TX_GEMM_A_SHARED) && batch > 1;
  if ((d.flags & TX_GEMM_A_SHARED) && batch > 1 && d.stride_a != 0) return TX_ERR_INVALID;
  const int64_t a_batch = a_shared ? 1 : batch;
  // rows shorter than half a swizzle row waste most of each tile; SIMT is better
  const int64_t a_inner = d.trans_a ? d.M : d.K;
  const int64_t b_inner = d.trans_b ? d.K : d.N;
  if (a_inner < 16 || b_inner < 16) return TX_ERR_UNSUPPORTED;
  if (!load_encode()) return TX_ERR_UNSUPPORTED;

  Maps m;
  memset(&m, 0, sizeof m);
  if (mode == 1) {
    // round-to-nearest: only operands that do not already hold TF32 values
    // are converted; with none left the plain pipeline is exact
    m.conv_mask = ((d.flags & TX_GEMM_A_TF32) ? 0 : 1) | ((d.flags & TX_GEMM_B_TF32) ? 0 : 2);
    if (m.conv_mask == 0) mode = 0;
  }
  Tiling tiling = pick_tiling(ctx, d.M, d.N, d.K, batch, mode == 2 ? 128 : 256);
  // A conversion-mode GEMM with enough tiles for the persistent kernel, whose
  // unconverted operands are small next to its output (at most half its
  // elements), rounds them once into scratch (one read and one write, the same
  // round-to-nearest the conversion applies) and runs without conversion, so
  // each tile's epilogue overlaps the next tile's main loop.  Measured on the
  // transformer's 32768x1024x256 dgrad with GELU': 180 us in 1024 one-tile CTAs.
  int64_t pre_na = 0, pre_nb = 0;
  if (cv) {
    // the gathered operands are no dense matrices to pre-round; a view
    // output takes neither split partials nor fused column sums
    if (d.B_lo || (cv->op.wsplit && (fs || d.preact || batch > 1))) return TX_ERR_UNSUPPORTED;
    if (cv->op.wsplit) tiling.splits = 1;
  }
  if (!cv && !a_shared && mode == 1 && tiling.splits == 1 && tma_tileable(d.C, d.ldc, batch, d.stride_c) &&
      (!d.dact || tma_tileable(d.dact_src, d.ld_dact, batch, d.stride_c)) &&
      (!d.preact || tma_tileable(d.preact, d.ld_preact, batch, d.stride_c))) {
    const int pbn = d.N > 128 ? 256 : d.N > 64 ? 128 : 64;
    const int64_t tiles = ((d.M + TC_BM - 1) / TC_BM) * ((d.N + pbn - 1) / pbn) * batch;
    const int64_t a_rows = d.trans_a ? d.K : d.M, a_inner = d.trans_a ? d.M : d.K;
    const int64_t b_rows = d.trans_b ? d.N : d.K, b_inner = d.trans_b ? d.K : d.N;
    const bool a_dense = d.lda == a_inner && (batch == 1 || d.stride_a == a_rows * d.lda);
    const bool b_dense = d.ldb == b_inner && (batch == 1 || d.stride_b == b_rows * d.ldb);
    const int64_t na = (m.conv_mask & 1) ? batch * a_rows * a_inner : 0;
    const int64_t nb = (m.conv_mask & 2) ? batch * b_rows * b_inner : 0;
    if (tiles > (pbn == 256 ? 1 : 2) * (int64_t)ctx->num_sms && (!na || a_dense) && (!nb || b_dense) &&
        2 * (na + nb) <= d.M * d.N * batch) {
      pre_na = na;
      pre_nb = nb;
    }
  }
  Scratch pre_a(ctx, (size_t)pre_na * sizeof(float)), pre_b(ctx, (size_t)pre_nb * sizeof(float));
  if ((pre_na || pre_nb) && (!pre_na || pre_a.ptr) && (!pre_nb || pre_b.ptr)) {
    if (pre_na) {
      TX_TRY(tx_round_tf32(ctx, d.A, pre_a.as<float>(), pre_na));
      d.A = pre_a.as<float>();
    }
    if (pre_nb) {
      TX_TRY(tx_round_tf32(ctx, d.B, pre_b.as<float>(), pre_nb));
      d.B = pre_b.as<float>();
    }
    d.flags |= TX_GEMM_A_TF32 | TX_GEMM_B_TF32;
    m.conv_mask = 0;
    mode = 0;
  }
  // Shapes with more tiles than SMs run persistently: the epilogue of one tile
  // overlaps the next tile's main loop (measured without conversion:
  // 32768x1024x256 100 -> 70 us, 32768x256x256 33 -> 27 us).  One wave gains
  // nothing and keeps two interleaved accumulators.  With operand conversion
  // the one-tile kernel keeps every stage and the epilogue in one CTA per SM,
  // so its setup (barriers, TMEM, tensor-map fetches) and epilogue are paid
  // once per tile with nothing overlapping them: products of three or more
  // waves, or of two waves of short tiles (at most 16 k-blocks: the implicit
  // convolutions), run persistently too, on tiles at most 128 wide (64 for
  // 3xTF32) that keep the one-tile kernel's accumulator count.
  bool persistent = false;
  if (tiling.splits == 1) {
    if (mode == 0) {
      // narrow outputs (batched attention products) need more waves to pay off
      const int pbn = d.N > 128 ? 256 : d.N > 64 ? 128 : 64;
      const int64_t tiles = ((d.M + TC_BM - 1) / TC_BM) * ((d.N + pbn - 1) / pbn) * batch;
      if (tiles > (pbn == 256 ? 1 : 2) * (int64_t)ctx->num_sms) {
        persistent = true;
        tiling.bn = pbn;
      } else if (d.B_lo) {
        // split weights in one launch at any size (the head and tail products
        // share one main loop and one epilogue, where the one-tile kernel
        // would run a second product through beta * C; transformer step at
        // batch 32: 1.66 -> 1.42 ms); narrower tiles while a wave would leave
        // a quarter of the SMs idle
        int qbn = pbn;
        while (qbn > 64 && ((d.M + TC_BM - 1) / TC_BM) * ((d.N + qbn - 1) / qbn) * batch * 4 <
                               3 * (int64_t)ctx->num_sms)
          qbn /= 2;
        persistent = true;
        tiling.bn = qbn;
      }
    } else {
      const int64_t tiles = ((d.M + TC_BM - 1) / TC_BM) * ((d.N + tiling.bn - 1) / tiling.bn) * batch;
      const int64_t waves = (tiles + ctx->num_sms - 1) / ctx->num_sms;
      const int64_t kblocks = (d.K + TC_BK - 1) / TC_BK;
      if (waves >= 3 || (waves >= 2 && kblocks <= 16)) {
        persistent = true;
        tiling.bn = mode == 2 || d.N <= 64 ? 64 : 128;
      }
    }
  }
  const int bn = tiling.bn;
  // One-tile launches of 256-wide tiles without conversion and an MN-major B
  // (the dgrad and wgrad products) run as CTA pairs when there are at least
  // two row tiles: each SM stages half of B (eight 32-column boxes become
  // four).  Measured main loops: 4096x1024x1024 dgrad 14.6 -> 12.4 us,
  // 1024x1024x4096 wgrad (4 splits) 17.6 -> 14.4 us; with a K-major B the pair
  // is slower (11.1 -> 12.2 us) and the single-CTA tile stays.
  const bool pair = mode == 0 && bn == 256 && !persistent && d.M > TC_BM && !d.trans_b && !cv;
  bool ok;
  if (cv && cv->op.a)  // 128 pixels of the activation per tile: K-major, 128-byte swizzle
    ok = make_map_4d(&m.a, cv->src, cv->box, cv->estr_w, cv->estr_h, false);
  else if (d.trans_a)  // A stored K x M (MN-major): box 32(M) x 32(K)
    ok = make_map(&m.a, d.A, d.M, d.K, d.lda, a_batch, d.stride_a, 32, true);
  else  // A stored M x K (K-major): box 32(K) x 128(M)
    ok = make_map(&m.a, d.A, d.K, d.M, d.lda, a_batch, d.stride_a, TC_BM, false);
  if (!ok) return TX_ERR_UNSUPPORTED;
  if (cv && cv->op.b == 1)  // 32 pixels by 32 channels per sub-tile: MN-major
    ok = make_map_4d(&m.b, cv->src, cv->box, cv->estr_w, cv->estr_h, true);
  else if (cv && cv->op.b == 2)  // a tap's weight rows, K-major
    ok = make_map(&m.b, d.B, cv->b_inner, cv->b_rows, d.ldb, 1, 0, bn, false);
  else if (d.trans_b)  // B stored N x K (K-major): box 32(K) x BN(N), BN / 2 per CTA of a pair
    ok = make_map(&m.b, d.B, d.K, d.N, d.ldb, batch, d.stride_b, pair ? bn / 2 : bn, false);
  else  // B stored K x N (MN-major): box 32(N) x 32(K)
    ok = make_map(&m.b, d.B, d.N, d.K, d.ldb, batch, d.stride_b, 32, true);
  if (!ok) return TX_ERR_UNSUPPORTED;
  if (cv) m.g = cv->op;
  m.g.ashared = a_shared ? 1 : 0;
  // dense MN-major operands whose MN extent is a multiple of 32: one box per
  // tile instead of one per 32-column block (the per-block maps stay when the
  // 4-D map is refused)
  CUtensorMap mn4;
  if (d.trans_a && !(cv && cv->op.a) && make_map_mn4(&mn4, d.A, d.M, d.K, d.lda, a_batch, d.stride_a, TC_BM / 32)) {
    m.a = mn4;
    m.g.amn = 1;
  }
  if (!d.trans_b && !(cv && cv->op.b) &&
      make_map_mn4(&mn4, d.B, d.N, d.K, d.ldb, batch, d.stride_b, (pair ? bn / 2 : bn) / 32)) {
    m.b = mn4;
    m.g.bmn = 1;
  }
  // split weights (B head + tail) run on the persistent kernel only; other
  // shapes report unsupported and the dispatcher runs two products instead
  if (d.B_lo) {
    if (!persistent || tiling.splits > 1 || d.trans_a || ((uintptr_t)d.B_lo & 15)) return TX_ERR_UNSUPPORTED;
    if (d.trans_b)
      ok = make_map(&m.b2, d.B_lo, d.K, d.N, d.ldb, batch, d.stride_b, bn, false);
    else if (m.g.bmn)  // the same 4-D form as B
      ok = make_map_mn4(&m.b2, d.B_lo, d.N, d.K, d.ldb, batch, d.stride_b, bn / 32);
    else
      ok = make_map(&m.b2, d.B_lo, d.N, d.K, d.ldb, batch, d.stride_b, 32, true);
    if (!ok) return TX_ERR_UNSUPPORTED;
  }

  // Split K across CTAs when the output has fewer tiles than SMs (the weight
  // gradients of small layers, whose reduction runs over the whole batch):
  // raw partial tiles go to scratch and a fixed-order reduction applies the
  // epilogue.  Shorter accumulation chains are also more accurate.
  const int total_kb = (int)((d.K + TC_BK - 1) / TC_BK);
  int splits = tiling.splits;
  if (splits <= 1) {
    if (cv && cv->op.wsplit) {
      const int ws = cv->op.wsplit;
      if (!make_view_map(&m.c, d.C, d.N, ws, cv->out_rows, cv->out_sw, cv->out_sr)) return TX_ERR_UNSUPPORTED;
      if (d.dact && !make_view_map(&m.s, d.dact_src, d.N, ws, cv->out_rows, cv->out_sw, cv->out_sr))
        return TX_ERR_UNSUPPORTED;
      m.tma_epi = 1;
    } else {
      make_epilogue_maps(m, d, batch);
    }
    if (fs) {
      // the TMA epilogue sums columns as it stores; otherwise C stays unrounded
      // and the caller sums it
      if (m.tma_epi && batch == 1) {
        m.col_part = fs->part;
        fs->rows = (d.M + 31) / 32;
        fs->fused = true;
      } else {
        d.flags &= ~TX_GEMM_ROUND_OUT;
      }
    }
    if (persistent && m.tma_epi) {
      const int rc = mode == 0   ? launch_persistent(ctx, bn, d, m, batch, 0)
                     : mode == 1 ? launch_persistent_round(ctx, bn, d, m, batch, 0)
                                 : launch_persistent_split(ctx, bn, d, m, batch, 0);
      if (rc != TX_ERR_UNSUPPORTED || d.B_lo) return rc;
    } else if (d.B_lo) {
      return TX_ERR_UNSUPPORTED;
    }
    if (pair) return launch_pair(ctx, d, m, batch, 0);
    return launch_any(ctx, mode, bn, d, m, batch, 0);
  }
  const int kb_per = (total_kb + splits - 1) / splits;
  splits = (total_kb + kb_per - 1) / kb_per;
  if (fs) d.flags &= ~TX_GEMM_ROUND_OUT;  // the split reduction does not sum columns
  Scratch part(ctx, (size_t)splits * d.M * d.N * sizeof(float));
  if (!part.ptr) return TX_ERR_OOM;
  tx_gemm_desc raw = d;
  raw.C = part.as<float>();
  raw.ldc = d.N;
  raw.stride_c = d.M * d.N;
  raw.alpha = 1.f;
  raw.beta = 0.f;
  raw.bias = nullptr;
  raw.act = TX_ACT_NONE;
  raw.preact = nullptr;
  raw.dact = TX_ACT_NONE;
  raw.dact_src = nullptr;
  raw.flags = d.flags & ~TX_GEMM_ROUND_OUT;  // partials stay exact; the reduction rounds
  make_epilogue_maps(m, raw, splits);
  int rc = TX_ERR_UNSUPPORTED;
  if (persistent && mode == 0 && m.tma_epi) rc = launch_persistent(ctx, bn, raw, m, splits, kb_per);
  if (rc == TX_ERR_UNSUPPORTED) rc = pair ? launch_pair(ctx, raw, m, splits, kb_per)
                                          : launch_any(ctx, mode, bn, raw, m, splits, kb_per);
  TX_TRY(rc);
  return gemm_split_reduce(ctx, d, part.as<float>(), splits);
}

}  // namespace

int gemm_tcgen05(tx_ctx *ctx, const tx_gemm_desc &d, int mode, FusedSum *fs) {
  return tc_product(ctx, d, mode, fs, nullptr);
}

int gemm_conv_tc(tx_ctx *ctx, const tx_gemm_desc &d, int mode, const ConvGemm &cv) {
  if (d.K <= 0 || d.M <= 0 || d.N <= 0) return TX_ERR_UNSUPPORTED;
  if (cv.op.cblocks <= 0 || cv.op.ntaps <= 0 || cv.op.ntaps > kGatherTaps || cv.op.ohw <= 0 || cv.op.ow <= 0)
    return TX_ERR_UNSUPPORTED;
  if (!load_encode()) return TX_ERR_UNSUPPORTED;
  return tc_product(ctx, d, mode, nullptr, &cv);
}
