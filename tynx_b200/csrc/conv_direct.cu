// Direct convolution for short filters (C * KH * KW < 32 taps x channels, at
// most 64 output channels): the first convolution of an image network (3
// channels, 3 x 3 taps).  Its im2col columns would be 28 floats per output
// pixel against 32 output floats, and the tensor core gains nothing at K = 27,
// so each thread gathers its pixel's patch from the NCHW input into registers
// (independent loads through a per-block table of tap offsets) and runs the
// whole filter bank in fp32 FMAs (products to full fp32 accuracy in every math
// mode, like the 3xTF32 split).
//
//   forward   y[n][o][oh][ow] = act(sum_k patch(p)[k] w[o][k] + b[o]), the
//             output NCHW or channels-last [pixel][o] (staged through shared
//             memory so each block writes one contiguous run);
//   wgrad     dW[o][k] = sum_p dz[p][o] patch(p)[k] and db[o] = sum_p dz[p][o]
//             (the patch's column K is 1): blocks walk tiles of 128 pixels,
//             keep their partial sums in registers and write one partial
//             each; a fixed-order reduction finishes them.
// k = (c * KH + kh) * KW + kw, the weight's own memory order.  The reference
// computes the same sums (DynTensor::conv2d_padded, crates/tynx/src/tensor.rs:1080-1180).
#include <cstring>

#include "common.h"
#include "epilogue.cuh"

namespace {

constexpr int kDirectK = 32;   // patch length bound (C * KH * KW < 32)
constexpr int kDirectOC = 64;  // output channel bound
constexpr int kPix = 128;      // pixels per forward block tile
constexpr int kWPix = 64;      // pixels per weight-gradient tile
constexpr int kPartLd = kDirectK;  // floats per output channel in a wgrad partial

struct DirectGeom {
  int N, C, H, W, KH, KW, OH, OW, sh, sw, pt, pl, dh, dw, OC, K;
};

// Per patch slot k: the input offset relative to the window's corner
// (c H W + kh dh W + kw dw) and the corner-relative row / column (kh dh, kw dw).
struct PatchTable {
  int off[kDirectK];
  short dy[kDirectK], dx[kDirectK];
};

__device__ void build_table(const DirectGeom &g, PatchTable &t) {
  for (int k = threadIdx.x; k < kDirectK; k += blockDim.x) {
    int off = 0, dy = 0, dx = 0;
    if (k < g.K) {
      const int c = k / (g.KH * g.KW), r = k % (g.KH * g.KW), kh = r / g.KW, kw = r % g.KW;
      dy = kh * g.dh;
      dx = kw * g.dw;
      off = c * g.H * g.W + dy * g.W + dx;
    }
    t.off[k] = off;
    t.dy[k] = (short)dy;
    t.dx[k] = (short)dx;
  }
}

// Slots [k0, k0 + NK) of pixel p's patch (zeros outside the image and past
// K).  The loads are independent and all issued before their first use.
template <int NK>
__device__ __forceinline__ void load_patch(const float *__restrict__ x, const DirectGeom &g, const PatchTable &t,
                                           int64_t p, int k0, float (&v)[NK]) {
  const int ow = (int)(p % g.OW);
  const int64_t q = p / g.OW;
  const int oh = (int)(q % g.OH);
  const int64_t n = q / g.OH;
  const int ih0 = oh * g.sh - g.pt, iw0 = ow * g.sw - g.pl;
  const float *base = x + n * g.C * (int64_t)g.H * g.W + (int64_t)ih0 * g.W + iw0;
#pragma unroll
  for (int j = 0; j < NK; ++j) {
    const int k = k0 + j;
    const int ih = ih0 + t.dy[k], iw = iw0 + t.dx[k];
    const bool in = k < g.K && ih >= 0 && ih < g.H && iw >= 0 && iw < g.W;
    v[j] = in ? __ldg(base + t.off[k]) : 0.f;
  }
}

// A block tile is kPix pixels x OCP channels in 32 x (OCP / 8) work items of
// four consecutive pixels x eight channels (item it: pixels 4 (it % 32) ..,
// channels 8 (it / 32) ..), so each k step reads one float4 of patch values
// and two of weights for 32 FMAs.  Patches are staged k-major (pt[k][pixel])
// by one thread per pixel with independent loads.
template <int OCP>
__global__ void __launch_bounds__(kPix) k_conv_direct_fwd(const float *__restrict__ x, const float *__restrict__ w,
                                                          const float *__restrict__ bias, float *__restrict__ y,
                                                          DirectGeom g, int act, int nhwc_out) {
  constexpr int OG = OCP / 8;  // channel groups of eight
  __shared__ __align__(16) float ws[kDirectK][OCP];   // ws[k][o] = w[o][k]
  __shared__ __align__(16) float pt[kDirectK][kPix + 4];  // pt[k][pixel]
  __shared__ float bs[OCP];
  __shared__ PatchTable tab;
  for (int e = threadIdx.x; e < kDirectK * OCP; e += blockDim.x) {
    const int k = e / OCP, o = e % OCP;
    ws[k][o] = (k < g.K && o < g.OC) ? w[(int64_t)o * g.K + k] : 0.f;
  }
  for (int o = threadIdx.x; o < OCP; o += blockDim.x) bs[o] = (bias && o < g.OC) ? bias[o] : 0.f;
  build_table(g, tab);
  const int64_t M = (int64_t)g.N * g.OH * g.OW;
  const int64_t hw = (int64_t)g.OH * g.OW;
  // kPix / 4 = 32 pixel quads x OG channel groups = 32 OG work items per tile,
  // kPix threads: each thread takes items it, it + kPix, ...
  for (int64_t p0 = (int64_t)blockIdx.x * kPix; p0 < M; p0 += (int64_t)gridDim.x * kPix) {
    __syncthreads();  // the table is built / the previous tile's patches are consumed
    {
      const int64_t p = p0 + threadIdx.x;
      float v[kDirectK];
      if (p < M) {
        load_patch<kDirectK>(x, g, tab, p, 0, v);
      } else {
#pragma unroll
        for (int k = 0; k < kDirectK; ++k) v[k] = 0.f;
      }
#pragma unroll
      for (int k = 0; k < kDirectK; ++k) pt[k][threadIdx.x] = v[k];
    }
    __syncthreads();
    for (int it = threadIdx.x; it < 32 * OG; it += blockDim.x) {
      const int q = it % 32, og = it / 32;
      const int px = 4 * q, o0 = 8 * og;
      float acc[4][8];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
#pragma unroll 8
      for (int k = 0; k < kDirectK; ++k) {
        const float4 pv = *reinterpret_cast<const float4 *>(&pt[k][px]);
        const float4 w0 = *reinterpret_cast<const float4 *>(&ws[k][o0]);
        const float4 w1 = *reinterpret_cast<const float4 *>(&ws[k][o0 + 4]);
        const float pa[4] = {pv.x, pv.y, pv.z, pv.w};
        const float wa[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(pa[i], wa[j], acc[i][j]);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int64_t p = p0 + px + i;
        if (p >= M) break;
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = tx_epi::act(act, acc[i][j] + bs[o0 + j]);
        if (nhwc_out) {
          float *dst = y + p * g.OC + o0;
          if (o0 + 8 <= g.OC && (g.OC & 3) == 0) {
            reinterpret_cast<float4 *>(dst)[0] = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
            reinterpret_cast<float4 *>(dst)[1] = make_float4(acc[i][4], acc[i][5], acc[i][6], acc[i][7]);
          } else {
            for (int j = 0; j < 8 && o0 + j < g.OC; ++j) dst[j] = acc[i][j];
          }
        } else {
          const int64_t n = p / hw, r = p - n * hw;
          for (int j = 0; j < 8 && o0 + j < g.OC; ++j) y[(n * g.OC + o0 + j) * hw + r] = acc[i][j];
        }
      }
    }
  }
}

// Block partial sums of the weight and bias gradients: part[block][o][k],
// k < K the weight, k == K the bias (the patch's slot K is 1).  256 threads in
// G = 256 / (2 OCT) groups; in a group, thread j owns the 4 x 4 outputs
// (o = 4 (j / 8) .., k = 4 (j % 8) ..) and walks the tile's pixels r = group
// (mod G): one float4 of dZ and one of the patch feed 16 FMAs.  The groups'
// sums are added in a fixed order at the end.
template <int OCT>
__global__ void __launch_bounds__(256) k_conv_direct_wgrad(const float *__restrict__ x,
                                                           const float *__restrict__ dz, DirectGeom g,
                                                           float *__restrict__ part) {
  constexpr int GT = OCT * 2;      // threads per group: OCT / 4 x 8
  constexpr int G = 256 / GT;      // groups
  __shared__ __align__(16) float pt[kWPix][kDirectK + 4];  // patch (+ the bias slot) per pixel
  __shared__ __align__(16) float dzt[kWPix][OCT + 4];
  __shared__ float red[G][OCT][kDirectK + 1];
  __shared__ PatchTable tab;
  build_table(g, tab);
  const int t = threadIdx.x;
  const int grp = t / GT, j = t % GT;
  const int o0 = 4 * (j / 8), k0 = 4 * (j % 8);
  float acc[4][4];
#pragma unroll
  for (int a = 0; a < 4; ++a) acc[a][0] = acc[a][1] = acc[a][2] = acc[a][3] = 0.f;
  const int64_t M = (int64_t)g.N * g.OH * g.OW;
  // patch loads: four threads per pixel, eight slots each
  const int lp = t >> 2, lk = (t & 3) * 8;
  for (int64_t p0 = (int64_t)blockIdx.x * kWPix; p0 < M; p0 += (int64_t)gridDim.x * kWPix) {
    __syncthreads();  // the table is built / the previous tile is consumed
    {
      const int64_t p = p0 + lp;
      float v[8];
      if (p < M) {
        load_patch<8>(x, g, tab, p, lk, v);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) pt[lp][lk + i] = (lk + i == g.K && p < M) ? 1.f : v[i];
    }
    const int rows = M - p0 < kWPix ? (int)(M - p0) : kWPix;
    for (int e = t; e < kWPix * OCT; e += blockDim.x) {
      const int r = e / OCT, oo = e % OCT;
      dzt[r][oo] = (r < rows && oo < g.OC) ? dz[(p0 + r) * g.OC + oo] : 0.f;
    }
    __syncthreads();
#pragma unroll 4
    for (int r = grp; r < kWPix; r += G) {
      const float4 dv = *reinterpret_cast<const float4 *>(&dzt[r][o0]);
      const float4 pv = *reinterpret_cast<const float4 *>(&pt[r][k0]);
      const float d4[4] = {dv.x, dv.y, dv.z, dv.w}, p4[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) acc[a][b] = fmaf(d4[a], p4[b], acc[a][b]);
    }
  }
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) red[grp][o0 + a][k0 + b] = acc[a][b];
  __syncthreads();
  // k in [0, 32) covers the weights and the bias slot (K < 32)
  float *pb = part + (int64_t)blockIdx.x * kDirectOC * kPartLd;
  for (int e = t; e < OCT * kDirectK; e += blockDim.x) {
    const int o = e / kDirectK, k = e % kDirectK;
    float s = red[0][o][k];
#pragma unroll
    for (int q = 1; q < G; ++q) s += red[q][o][k];
    pb[o * kPartLd + k] = s;
  }
}

// dW[o][k] (+)= sum_b part[b][o][k], db[o] (+)= sum_b part[b][o][K]: one warp
// per output, lanes over blocks, then a fixed shuffle tree (deterministic).
__global__ void k_conv_direct_wgrad_finish(const float *__restrict__ part, int blocks, DirectGeom g,
                                           float *__restrict__ dw, float *__restrict__ db, int acc_w,
                                           int acc_b) {
  const int e = (int)((blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
  if (e >= g.OC * (g.K + 1)) return;
  const int o = e / (g.K + 1), k = e % (g.K + 1);
  float s = 0.f;
  for (int b = lane; b < blocks; b += 32) s += part[(int64_t)b * kDirectOC * kPartLd + o * kPartLd + k];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (lane) return;
  if (k < g.K) {
    float *q = dw + (int64_t)o * g.K + k;
    *q = acc_w ? *q + s : s;
  } else if (db) {
    db[o] = acc_b ? db[o] + s : s;
  }
}

DirectGeom direct_geom(const int *gi, int OC) {
  DirectGeom g;
  g.N = gi[0]; g.C = gi[1]; g.H = gi[2]; g.W = gi[3]; g.KH = gi[4]; g.KW = gi[5]; g.OH = gi[6]; g.OW = gi[7];
  g.sh = gi[8]; g.sw = gi[9]; g.pt = gi[10]; g.pl = gi[11]; g.dh = gi[12]; g.dw = gi[13];
  g.OC = OC;
  g.K = g.C * g.KH * g.KW;
  return g;
}

}  // namespace

bool conv_direct_ok(int C, int KH, int KW, int OC) {
  return C * KH * KW <= kDirectK - 1 && OC >= 1 && OC <= kDirectOC;
}

int conv_direct_fwd(tx_ctx *ctx, const float *x, const float *w, const float *bias, float *y, const int *geom, int OC,
                    int act, bool nhwc_out) {
  const DirectGeom g = direct_geom(geom, OC);
  if (!conv_direct_ok(g.C, g.KH, g.KW, OC)) return TX_ERR_UNSUPPORTED;
  const int64_t M = (int64_t)g.N * g.OH * g.OW;
  if (M <= 0) return TX_OK;
  int64_t blocks = (M + kPix - 1) / kPix;
  if (blocks > (int64_t)ctx->num_sms * 8) blocks = (int64_t)ctx->num_sms * 8;
  if (OC <= 16)
    k_conv_direct_fwd<16><<<(unsigned)blocks, kPix, 0, ctx->stream>>>(x, w, bias, y, g, act, nhwc_out);
  else if (OC <= 32)
    k_conv_direct_fwd<32><<<(unsigned)blocks, kPix, 0, ctx->stream>>>(x, w, bias, y, g, act, nhwc_out);
  else
    k_conv_direct_fwd<64><<<(unsigned)blocks, kPix, 0, ctx->stream>>>(x, w, bias, y, g, act, nhwc_out);
  TX_LAUNCHED(ctx, "k_conv_direct_fwd");
  return TX_OK;
}

int conv_direct_wgrad(tx_ctx *ctx, const float *x, const float *dz, const int *geom, int OC, float *dw, float *db,
                      int acc_w, int acc_b) {
  const DirectGeom g = direct_geom(geom, OC);
  if (!conv_direct_ok(g.C, g.KH, g.KW, OC)) return TX_ERR_UNSUPPORTED;
  const int64_t M = (int64_t)g.N * g.OH * g.OW;
  int64_t blocks = (M + kWPix - 1) / kWPix;
  if (blocks > (int64_t)ctx->num_sms * 4) blocks = (int64_t)ctx->num_sms * 4;
  if (blocks < 1) blocks = 1;
  Scratch part(ctx, (size_t)blocks * kDirectOC * kPartLd * sizeof(float));
  if (!part.ptr) return TX_ERR_OOM;
  if (OC <= 32)
    k_conv_direct_wgrad<32><<<(unsigned)blocks, 256, 0, ctx->stream>>>(x, dz, g, part.as<float>());
  else
    k_conv_direct_wgrad<64><<<(unsigned)blocks, 256, 0, ctx->stream>>>(x, dz, g, part.as<float>());
  TX_LAUNCHED(ctx, "k_conv_direct_wgrad");
  const int warps = OC * (g.K + 1);
  k_conv_direct_wgrad_finish<<<(warps + 7) / 8, 256, 0, ctx->stream>>>(part.as<float>(), (int)blocks, g, dw, db,
                                                                       acc_w, acc_b);
  TX_LAUNCHED(ctx, "k_conv_direct_wgrad_finish");
  return TX_OK;
}
