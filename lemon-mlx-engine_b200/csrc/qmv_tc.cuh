// qmv_tc.cuh -- K1 for small batches on the tensor cores: the quantized
// GEMV for 4 <= M <= 16 below the tcgen05 threshold (speculative drafts
// M = B, short verify blocks M = B(K+1)) in tensor-core mode.  On B200 the
// CUDA cores run out of FMA throughput before HBM does once M >= ~4 (M FMAs
// per weight element), so the products run on mma.sync.m16n8k16 (bf16 in,
// fp32 accumulate) with swap-AB: 16 weight rows are the A operand, up to 8
// (NT=1) or 16 (NT=2) tokens the B operand.
//
// Numerics: MLX's qmv form (the reference's kernel for these M), per 64-k
// group  e = s * sum_k q_k x_k + b * sum_k x_k,  summed over the groups.  The
// codes q (0..255) are exact bf16 values, so the tensor cores take A = q and
// B = x and the only difference from the canonical GEMV is the fp32
// summation order; sum_k x_k comes from a second mma with an all-ones A.
// Results are compared with a tolerance (exact mode keeps the canonical
// GEMV for every M).
//
// CTA = one 16-row tile (PLAIN / RESID: of the concatenated matrices;
// SWIGLU: 16 gate rows and the same 16 up rows), 8 warps each owning a
// contiguous range of the K groups (SWIGLU: 4 + 4); tiles too few to fill
// the GPU are split along K over a cluster of 2 or 4 CTAs whose partial
// tiles are summed through distributed shared memory in rank order.
//
// Per group, lane (q, c) = (lane/4, lane%4) owns the 16 k values
// 16c .. 16c+15: it loads them contiguously for weight rows q and q+8 (4-bit:
// 8 bytes, 8-bit: 16 bytes) and for its token rows (32 bytes), and maps them
// onto its mma k slots (2c, 2c+1, 2c+8, 2c+9 of each 16-k step) under one
// permutation shared by A and B, so every load is a full sector and nothing
// is loaded twice.  4-bit codes become bf16 pairs (q_i, q_{i+4}) of a word
// through the exact 128 + q bf16 trick; 8-bit codes through the fp32 magic
// 2^23 + q and one bf16x2 convert.
//
// With norm_w set (the layer's input / post-attention RMSNorm fused into the
// prologue, as the CUDA-core GEMV does), the CTA forms each token row's
// factor r in the canonical warp order (rms_factor_warp) after the wait on
// the producing kernel and normalises every activation value as it is
// loaded: x' = bf16((x r) w) -- the values the separate RMSNorm kernel would
// have written.
#pragma once
#include <cooperative_groups.h>

#include "attn_mma.cuh"
#include "qmm_mma.cuh"

namespace lmx {

static constexpr int kTcgRows = 16;

// Tile -> (matrix, first row) over the concatenated matrices (16-row tiles).
LMX_DEV bool tcg_tile(const QmmArgs& a, int tile, int& mi, int& row0) {
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    if (i < a.nmat) {
      const int nt = (a.mat[i].rows + kTcgRows - 1) / kTcgRows;
      if (tile < nt) {
        mi = i;
        row0 = tile * kTcgRows;
        return true;
      }
      tile -= nt;
    }
  }
  return false;
}

// 8-bit code j of word w as an exact fp32 value
LMX_DEV float tcg_code8(uint32_t w, int j) {
  return __fsub_rn(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540 + j)), 8388608.0f);
}

template <int BITS, int NT>
__global__ void __launch_bounds__(256) qmv_tc_kernel(QmmArgs a, int ks) {
  namespace cg = cooperative_groups;
  constexpr int RS = 8 * NT + 1;  // padded token stride of the partial tiles
  __shared__ float red[8][kTcgRows][RS];
  __shared__ float fnorm[kTcgRows];  // RMSNorm factor per token row (norm_w set)
  extern __shared__ uint32_t sbm[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, q = lane >> 2, c = lane & 3;
  const int rank = ks > 1 ? (int)(blockIdx.x % ks) : 0, tile = (int)blockIdx.x / ks;
  const bool sw = a.mode == QMM_SWIGLU;
  const int nslice = sw ? 4 : 8, slice = sw ? (warp & 3) : warp;
  int mi = 0, row0 = 0;
  if (sw) {
    mi = warp >> 2;
    row0 = tile * kTcgRows;
  } else if (!tcg_tile(a, tile, mi, row0)) {
    return;  // (the whole cluster shares the tile, so no CTA waits on this one)
  }
  const QmmMat& W = mi == 0 ? a.mat[0] : (mi == 1 ? a.mat[1] : a.mat[2]);
  const int G = a.K / 64, rows = sw ? a.N : W.rows;
  const int S = nslice * ks, sl = rank * nslice + slice;
  const int g0 = sl * G / S, g1 = (sl + 1) * G / S;
  const int ra = row0 + q, rb = row0 + q + 8;
  const bool va = ra < rows, vb = rb < rows;
  constexpr int WPG = 2 * BITS;  // words per group and row
  constexpr int LW = BITS / 2;   // words per group, row and lane
  const uint32_t* wa = W.w + (size_t)(va ? ra : 0) * G * WPG + LW * c;
  const uint32_t* wb = W.w + (size_t)(vb ? rb : 0) * G * WPG + LW * c;
  // this CTA's (scale, bias) pairs, one bf16x2 word per (row, group), staged
  // in shared memory once (row stride GS + 1 words: conflict-free reads)
  const int glo = rank * G / ks, GS = (rank + 1) * G / ks - glo, nrt = sw ? 2 * kTcgRows : kTcgRows;
  for (int idx = tid; idx < nrt * GS; idx += blockDim.x) {
    const int r = idx / GS, gi = idx - r * GS;
    const QmmMat& Wr = sw ? (r < kTcgRows ? a.mat[0] : a.mat[1]) : W;
    const int row = row0 + (r & (kTcgRows - 1));
    uint32_t v = 0;
    if (row < rows) {
      const size_t o = (size_t)row * G + glo + gi;
      v = (uint32_t)Wr.s[o] | ((uint32_t)Wr.b[o] << 16);
    }
    sbm[r * (GS + 1) + gi] = v;
  }
  const uint32_t* sbq = sbm + ((sw ? mi * kTcgRows : 0) + q) * (GS + 1);
  const uint32_t* sbq8 = sbq + 8 * (GS + 1);
  const bf16_t* xr[NT];
  bool xv[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    const int n = t * 8 + q;
    xv[t] = n < a.M;
    xr[t] = a.x + (size_t)(xv[t] ? n : 0) * a.ldx + 16 * c;
  }
  float acc[NT][4];
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[t][e] = 0.0f;
  const uint32_t one2 = 0x3F803F80u, m128 = 0xC300C300u;
  const uint32_t ones[4] = {one2, one2, one2, one2};
  // software pipeline over the groups: the next group's weights are loaded
  // while this one's products run; the first group's before the wait on the
  // previous kernel, since weights do not depend on it
  uint32_t A[2][LW], B[2][LW];
  auto load_w = [&](int g, int u) {
    const bool ua = va && g < g1, ub = vb && g < g1;
    if constexpr (BITS == 4) {
      const uint2 x0 = ua ? *reinterpret_cast<const uint2*>(wa + (size_t)g * WPG) : make_uint2(0, 0);
      const uint2 x1 = ub ? *reinterpret_cast<const uint2*>(wb + (size_t)g * WPG) : make_uint2(0, 0);
      A[u][0] = x0.x, A[u][1] = x0.y, B[u][0] = x1.x, B[u][1] = x1.y;
    } else {
      const uint4 x0 = ua ? *reinterpret_cast<const uint4*>(wa + (size_t)g * WPG) : make_uint4(0, 0, 0, 0);
      const uint4 x1 = ub ? *reinterpret_cast<const uint4*>(wb + (size_t)g * WPG) : make_uint4(0, 0, 0, 0);
      A[u][0] = x0.x, A[u][1] = x0.y, A[u][2] = x0.z, A[u][3] = x0.w;
      B[u][0] = x1.x, B[u][1] = x1.y, B[u][2] = x1.z, B[u][3] = x1.w;
    }
  };
  load_w(g0, 0);
  __syncthreads();  // the (scale, bias) table
  grid_wait();
  grid_launch_dependents();
  const bool nrm = a.norm_w != nullptr;
  float fr[NT];
  // activations of group g into buffer u (double-buffered like the weights:
  // group g+1's loads are in flight while group g's products run)
  uint32_t XB[2][NT][8];
  auto load_x = [&](int g, int u) {
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      uint4 lo = make_uint4(0, 0, 0, 0), hi = make_uint4(0, 0, 0, 0);
      if (xv[t] && g < g1) {
        lo = __ldg(reinterpret_cast<const uint4*>(xr[t] + (size_t)g * 64));
        hi = __ldg(reinterpret_cast<const uint4*>(xr[t] + (size_t)g * 64 + 8));
      }
      XB[u][t][0] = lo.x, XB[u][t][1] = lo.y, XB[u][t][2] = lo.z, XB[u][t][3] = lo.w;
      XB[u][t][4] = hi.x, XB[u][t][5] = hi.y, XB[u][t][6] = hi.z, XB[u][t][7] = hi.w;
    }
  };
  load_x(g0, 0);
  if (nrm) {
    for (int m = warp; m < a.M; m += 8) {
      const float f = rms_factor_warp(a.x + (size_t)m * a.ldx, a.K, a.eps, lane);
      if (lane == 0) fnorm[m] = f;
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < NT; ++t) fr[t] = xv[t] ? fnorm[t * 8 + q] : 0.0f;
  }
  // one group: prefetch group g+1 into buffer u^1, then the products of
  // group g from buffer u (u is a literal at each call, so the buffers stay
  // in registers)
  auto step = [&](const int g, const int u) {
    if (g + 1 < g1) {
      load_w(g + 1, u ^ 1);
      load_x(g + 1, u ^ 1);
    }
    {
      uint32_t X[NT][8];
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int i = 0; i < 8; ++i) X[t][i] = XB[u][t][i];
      if (nrm) {
        const uint4 n0 = __ldg(reinterpret_cast<const uint4*>(a.norm_w + (size_t)g * 64 + 16 * c));
        const uint4 n1 = __ldg(reinterpret_cast<const uint4*>(a.norm_w + (size_t)g * 64 + 16 * c + 8));
        const uint32_t nw[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const bf16_t lo = f2bf(__fmul_rn(__fmul_rn(lo_bf(X[t][i]), fr[t]), lo_bf(nw[i])));
            const bf16_t hi = f2bf(__fmul_rn(__fmul_rn(hi_bf(X[t][i]), fr[t]), hi_bf(nw[i])));
            X[t][i] = (uint32_t)lo | ((uint32_t)hi << 16);
          }
      }
      float dot[NT][4], xs[NT][4];
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) dot[t][e] = xs[t][e] = 0.0f;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t af[4], bfr[NT][2];
        if constexpr (BITS == 4) {
          // step kk: word h = kk/2 of the lane's two (k = 16c + 8h + j),
          // nibble pairs (i, i+4) and (i+1, i+5), i = 2(kk%2); x pairs to match
          const int h = kk >> 1, i = (kk & 1) * 2;
          af[0] = bf2_fma(((A[u][h] >> (4 * i)) & 0x000F000Fu) | 0x43004300u, one2, m128);
          af[1] = bf2_fma(((B[u][h] >> (4 * i)) & 0x000F000Fu) | 0x43004300u, one2, m128);
          af[2] = bf2_fma(((A[u][h] >> (4 * i + 4)) & 0x000F000Fu) | 0x43004300u, one2, m128);
          af[3] = bf2_fma(((B[u][h] >> (4 * i + 4)) & 0x000F000Fu) | 0x43004300u, one2, m128);
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            const uint32_t x0 = X[t][4 * h + (i >> 1)], x1 = X[t][4 * h + 2 + (i >> 1)];
            bfr[t][0] = __byte_perm(x0, x1, 0x5410);
            bfr[t][1] = __byte_perm(x0, x1, 0x7632);
          }
        } else {
          // step kk: word kk of the lane's four (k = 16c + 4kk + j), code
          // pairs (0, 1) and (2, 3); the x pairs are the lane's x words 2kk, 2kk+1
          af[0] = bf2_pack(tcg_code8(A[u][kk], 0), tcg_code8(A[u][kk], 1));
          af[1] = bf2_pack(tcg_code8(B[u][kk], 0), tcg_code8(B[u][kk], 1));
          af[2] = bf2_pack(tcg_code8(A[u][kk], 2), tcg_code8(A[u][kk], 3));
          af[3] = bf2_pack(tcg_code8(B[u][kk], 2), tcg_code8(B[u][kk], 3));
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            bfr[t][0] = X[t][2 * kk];
            bfr[t][1] = X[t][2 * kk + 1];
          }
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          mma_16816(dot[t], af, bfr[t][0], bfr[t][1]);
          mma_16816(xs[t], ones, bfr[t][0], bfr[t][1]);
        }
      }
      // the group's term s * dot + b * xsum (rows q: e = 0, 1; q+8: e = 2, 3)
      const uint32_t pa = sbq[g - glo], pb = sbq8[g - glo];
      const float sa = __uint_as_float(pa << 16), ba = __uint_as_float(pa & 0xFFFF0000u);
      const float sb = __uint_as_float(pb << 16), bb = __uint_as_float(pb & 0xFFFF0000u);
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        acc[t][0] = __fadd_rn(acc[t][0], __fmaf_rn(sa, dot[t][0], __fmul_rn(ba, xs[t][0])));
        acc[t][1] = __fadd_rn(acc[t][1], __fmaf_rn(sa, dot[t][1], __fmul_rn(ba, xs[t][1])));
        acc[t][2] = __fadd_rn(acc[t][2], __fmaf_rn(sb, dot[t][2], __fmul_rn(bb, xs[t][2])));
        acc[t][3] = __fadd_rn(acc[t][3], __fmaf_rn(sb, dot[t][3], __fmul_rn(bb, xs[t][3])));
      }
    }
  };
  for (int g = g0; g < g1; g += 2) {
    step(g, 0);
    if (g + 1 < g1) step(g + 1, 1);
  }
  // partial tile: rows (q, q+8), tokens t*8 + 2c, +1
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    red[warp][q][t * 8 + 2 * c] = acc[t][0];
    red[warp][q][t * 8 + 2 * c + 1] = acc[t][1];
    red[warp][q + 8][t * 8 + 2 * c] = acc[t][2];
    red[warp][q + 8][t * 8 + 2 * c + 1] = acc[t][3];
  }
  cg::cluster_group cluster = cg::this_cluster();
  if (ks > 1) cluster.sync();
  else __syncthreads();
  // each rank finishes a share of the tile's outputs, summing the partial
  // tiles in (rank, warp) order
  const int total = kTcgRows * a.M, per = (total + ks - 1) / ks;
  const int i0 = rank * per, i1 = min(total, i0 + per);
  for (int e = i0 + tid; e < i1; e += blockDim.x) {
    const int r = e % kTcgRows, m = e / kTcgRows;
    const int row = row0 + r;
    if (row >= rows) continue;
    float s0 = 0.0f, s1 = 0.0f;
    for (int k = 0; k < ks; ++k) {
      const float* rr = ks > 1 ? cluster.map_shared_rank(&red[0][0][0], k) : &red[0][0][0];
      for (int w = 0; w < nslice; ++w) s0 = __fadd_rn(s0, rr[(w * kTcgRows + r) * RS + m]);
      if (sw)
        for (int w = 4; w < 8; ++w) s1 = __fadd_rn(s1, rr[(w * kTcgRows + r) * RS + m]);
    }
    if (sw) {
      a.y[(size_t)m * a.ldy + row] = swiglu_c(f2bf(s0), f2bf(s1));
    } else {
      const int col = (mi == 0 ? 0 : (mi == 1 ? a.mat[0].rows : a.mat[0].rows + a.mat[1].rows)) + row;
      bf16_t yv = f2bf(s0);
      if (a.mode == QMM_RESID) yv = f2bf(__fadd_rn(bf2f(yv), bf2f(a.res[(size_t)m * a.ldy + col])));
      a.y[(size_t)m * a.ldy + col] = yv;
    }
  }
  if (ks > 1) cluster.sync();  // peers may still read this CTA's partial tile
}

// The same products for matrices with many tiles (the lm_head: 151936 /
// 16 tiles): each warp owns one whole 16-row tile over the full K -- no
// split across warps, no shared-memory reduction, no per-CTA scale table --
// so a CTA's fixed costs are spread over 8 tiles.  Scales and biases are
// loaded with the weights, two groups ahead.  PLAIN / RESID only; the fused
// RMSNorm as above.  Per row the groups are summed in ascending order by one
// warp (fp32, tensor-core order within a group).
template <int BITS, int NT>
__global__ void __launch_bounds__(256) qmv_tc_rows_kernel(QmmArgs a) {
  __shared__ float fnorm[kTcgRows];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, q = lane >> 2, c = lane & 3;
  int mi = 0, row0 = 0;
  const bool have = tcg_tile(a, (int)blockIdx.x * 8 + warp, mi, row0);
  const QmmMat& W = mi == 0 ? a.mat[0] : (mi == 1 ? a.mat[1] : a.mat[2]);
  const int G = a.K / 64, rows = W.rows;
  const int ra = row0 + q, rb = row0 + q + 8;
  const bool va = have && ra < rows, vb = have && rb < rows;
  constexpr int WPG = 2 * BITS;
  constexpr int LW = BITS / 2;
  const uint32_t* wa = W.w + (size_t)(va ? ra : 0) * G * WPG + LW * c;
  const uint32_t* wb = W.w + (size_t)(vb ? rb : 0) * G * WPG + LW * c;
  const bf16_t* sa_p = W.s + (size_t)(va ? ra : 0) * G;
  const bf16_t* ba_p = W.b + (size_t)(va ? ra : 0) * G;
  const bf16_t* sb_p = W.s + (size_t)(vb ? rb : 0) * G;
  const bf16_t* bb_p = W.b + (size_t)(vb ? rb : 0) * G;
  uint32_t A[2][LW], B[2][LW], SB[2][2];  // SB: (scale | bias << 16) of rows ra, rb
  auto load_w = [&](int g, int u) {
    const bool ua = va && g < G, ub = vb && g < G;
    if constexpr (BITS == 4) {
      const uint2 x0 = ua ? *reinterpret_cast<const uint2*>(wa + (size_t)g * WPG) : make_uint2(0, 0);
      const uint2 x1 = ub ? *reinterpret_cast<const uint2*>(wb + (size_t)g * WPG) : make_uint2(0, 0);
      A[u][0] = x0.x, A[u][1] = x0.y, B[u][0] = x1.x, B[u][1] = x1.y;
    } else {
      const uint4 x0 = ua ? *reinterpret_cast<const uint4*>(wa + (size_t)g * WPG) : make_uint4(0, 0, 0, 0);
      const uint4 x1 = ub ? *reinterpret_cast<const uint4*>(wb + (size_t)g * WPG) : make_uint4(0, 0, 0, 0);
      A[u][0] = x0.x, A[u][1] = x0.y, A[u][2] = x0.z, A[u][3] = x0.w;
      B[u][0] = x1.x, B[u][1] = x1.y, B[u][2] = x1.z, B[u][3] = x1.w;
    }
    SB[u][0] = ua ? ((uint32_t)sa_p[g] | ((uint32_t)ba_p[g] << 16)) : 0u;
    SB[u][1] = ub ? ((uint32_t)sb_p[g] | ((uint32_t)bb_p[g] << 16)) : 0u;
  };
  load_w(0, 0);
  grid_wait();
  grid_launch_dependents();
  const bf16_t* xr[NT];
  bool xv[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    const int n = t * 8 + q;
    xv[t] = n < a.M;
    xr[t] = a.x + (size_t)(xv[t] ? n : 0) * a.ldx + 16 * c;
  }
  uint32_t XB[2][NT][8];
  auto load_x = [&](int g, int u) {
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      uint4 lo = make_uint4(0, 0, 0, 0), hi = make_uint4(0, 0, 0, 0);
      if (xv[t] && g < G) {
        lo = __ldg(reinterpret_cast<const uint4*>(xr[t] + (size_t)g * 64));
        hi = __ldg(reinterpret_cast<const uint4*>(xr[t] + (size_t)g * 64 + 8));
      }
      XB[u][t][0] = lo.x, XB[u][t][1] = lo.y, XB[u][t][2] = lo.z, XB[u][t][3] = lo.w;
      XB[u][t][4] = hi.x, XB[u][t][5] = hi.y, XB[u][t][6] = hi.z, XB[u][t][7] = hi.w;
    }
  };
  load_x(0, 0);
  const bool nrm = a.norm_w != nullptr;
  float fr[NT];
  if (nrm) {
    for (int m = warp; m < a.M; m += 8) {
      const float f = rms_factor_warp(a.x + (size_t)m * a.ldx, a.K, a.eps, lane);
      if (lane == 0) fnorm[m] = f;
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < NT; ++t) fr[t] = xv[t] ? fnorm[t * 8 + q] : 0.0f;
  }
  if (!have) return;
  float acc[NT][4];
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[t][e] = 0.0f;
  const uint32_t one2 = 0x3F803F80u, m128 = 0xC300C300u;
  const uint32_t ones[4] = {one2, one2, one2, one2};
  auto step = [&](const int g, const int u) {
    if (g + 1 < G) {
      load_w(g + 1, u ^ 1);
      load_x(g + 1, u ^ 1);
    }
    uint32_t X[NT][8];
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int i = 0; i < 8; ++i) X[t][i] = XB[u][t][i];
    if (nrm) {
      const uint4 n0 = __ldg(reinterpret_cast<const uint4*>(a.norm_w + (size_t)g * 64 + 16 * c));
      const uint4 n1 = __ldg(reinterpret_cast<const uint4*>(a.norm_w + (size_t)g * 64 + 16 * c + 8));
      const uint32_t nw[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const bf16_t lo = f2bf(__fmul_rn(__fmul_rn(lo_bf(X[t][i]), fr[t]), lo_bf(nw[i])));
          const bf16_t hi = f2bf(__fmul_rn(__fmul_rn(hi_bf(X[t][i]), fr[t]), hi_bf(nw[i])));
          X[t][i] = (uint32_t)lo | ((uint32_t)hi << 16);
        }
    }
    float dot[NT][4], xs[NT][4];
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int e = 0; e < 4; ++e) dot[t][e] = xs[t][e] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t af[4], bfr[NT][2];
      if constexpr (BITS == 4) {
        const int h = kk >> 1, i = (kk & 1) * 2;
        af[0] = bf2_fma(((A[u][h] >> (4 * i)) & 0x000F000Fu) | 0x43004300u, one2, m128);
        af[1] = bf2_fma(((B[u][h] >> (4 * i)) & 0x000F000Fu) | 0x43004300u, one2, m128);
        af[2] = bf2_fma(((A[u][h] >> (4 * i + 4)) & 0x000F000Fu) | 0x43004300u, one2, m128);
        af[3] = bf2_fma(((B[u][h] >> (4 * i + 4)) & 0x000F000Fu) | 0x43004300u, one2, m128);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const uint32_t x0 = X[t][4 * h + (i >> 1)], x1 = X[t][4 * h + 2 + (i >> 1)];
          bfr[t][0] = __byte_perm(x0, x1, 0x5410);
          bfr[t][1] = __byte_perm(x0, x1, 0x7632);
        }
      } else {
        af[0] = bf2_pack(tcg_code8(A[u][kk], 0), tcg_code8(A[u][kk], 1));
        af[1] = bf2_pack(tcg_code8(B[u][kk], 0), tcg_code8(B[u][kk], 1));
        af[2] = bf2_pack(tcg_code8(A[u][kk], 2), tcg_code8(A[u][kk], 3));
        af[3] = bf2_pack(tcg_code8(B[u][kk], 2), tcg_code8(B[u][kk], 3));
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          bfr[t][0] = X[t][2 * kk];
          bfr[t][1] = X[t][2 * kk + 1];
        }
      }
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        mma_16816(dot[t], af, bfr[t][0], bfr[t][1]);
        mma_16816(xs[t], ones, bfr[t][0], bfr[t][1]);
      }
    }
    const uint32_t pa = SB[u][0], pb = SB[u][1];
    const float sa = __uint_as_float(pa << 16), ba = __uint_as_float(pa & 0xFFFF0000u);
    const float sb = __uint_as_float(pb << 16), bb = __uint_as_float(pb & 0xFFFF0000u);
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      acc[t][0] = __fadd_rn(acc[t][0], __fmaf_rn(sa, dot[t][0], __fmul_rn(ba, xs[t][0])));
      acc[t][1] = __fadd_rn(acc[t][1], __fmaf_rn(sa, dot[t][1], __fmul_rn(ba, xs[t][1])));
      acc[t][2] = __fadd_rn(acc[t][2], __fmaf_rn(sb, dot[t][2], __fmul_rn(bb, xs[t][2])));
      acc[t][3] = __fadd_rn(acc[t][3], __fmaf_rn(sb, dot[t][3], __fmul_rn(bb, xs[t][3])));
    }
  };
  for (int g = 0; g < G; g += 2) {
    step(g, 0);
    if (g + 1 < G) step(g + 1, 1);
  }
  // rows (q, q+8) x tokens t*8 + 2c, +1 straight from the fragments
  const int cbase = mi == 0 ? 0 : (mi == 1 ? a.mat[0].rows : a.mat[0].rows + a.mat[1].rows);
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int m = t * 8 + 2 * c + (e & 1), row = (e < 2) ? ra : rb;
      if (m >= a.M || row >= rows) continue;
      const size_t o = (size_t)m * a.ldy + cbase + row;
      bf16_t yv = f2bf(acc[t][e]);
      if (a.mode == QMM_RESID) yv = f2bf(__fadd_rn(bf2f(yv), bf2f(a.res[o])));
      a.y[o] = yv;
    }
}

}  // namespace lmx
