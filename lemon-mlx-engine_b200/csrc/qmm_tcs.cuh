// qmm_tcs.cuh -- K1 for mid-size batches on the tensor cores: the quantized
// matmul for 16 <= M <= 64 rows in tensor-core mode (the batched verify
// pass: config 3 runs M = 8 sequences x 6 tokens = 48).
//
// The tcgen05 path (qmm_mma.cuh) dequantizes every weight to bf16 before the
// MMA; at these M its eight dequantizer warps per CTA are bound by their
// dependent unpack / TMEM-store chains (~2.5 instructions per weight) and the
// tensor pipe idles.  Here the weights never become bf16 values: as in the
// small-batch GEMV (qmv_tc.cuh) the codes q (exact in bf16) are the mma.sync
// A operand and every 64-k group contributes  s * sum_k q_k x_k + b * sum_k x_k
// (MLX's qmv math); the group sums of x are formed once per CTA.
//
// CTA: 8 warps; warp w owns one 16-row weight tile (PLAIN / RESID: tiles of
// the concatenated matrices; SWIGLU: 16 gate rows (w < 4) or the same 16 up
// rows (w >= 4) of the CTA's 64 output rows) over the CTA's range of K
// groups.  A cluster of `ks` CTAs splits K; the partial tiles [128 rows][M]
// are summed in rank order through distributed shared memory.
//
// Activations: per block of 2 groups (128 k) every thread loads its 16-byte
// chunks of x [M][128] into registers one block ahead, then stores them into
// a double-buffered shared tile (16-byte chunks XOR-swizzled by row % 8) and
// forms the per-(token, group) sums with 8-lane shuffles; one __syncthreads
// per block.  For 4-bit weights each 8-value chunk is stored in the order
// (k0,k4,k1,k5,k2,k6,k3,k7), the order in which a word's nibble pairs come
// out, so that lane (q, c) loads its 16 k of a token as two 16-byte words and
// uses them as mma B fragments unchanged; 8-bit chunks stay in k order.
//
// Numerics: fp32 tensor-core products of exact codes, per group the term
// s * dot + b * xsum added into the row's accumulator in ascending group
// order, ranks summed in order; compared with the canonical GEMV within a
// tolerance (exact mode never takes this path).
#pragma once
#include <cooperative_groups.h>

#include "qmv_tc.cuh"

namespace lmx {

static constexpr int kTcsWarps = 8;
static constexpr int kTcsRows = 16 * kTcsWarps;  // weight rows per CTA
static constexpr int kTcsMaxSplit = 8;

// Dynamic shared memory: two activation blocks [2 groups][R rows][128 B]
// (the [128][R + 1] fp32 partial tile reuses them after the main loop), then
// two group-sum blocks [2 groups][R] floats.
__host__ __device__ constexpr size_t tcs_tile_bytes(int R) {
  return (size_t)2 * 2 * R * 128 > (size_t)kTcsRows * (R + 1) * 4 ? (size_t)2 * 2 * R * 128
                                                                   : (size_t)kTcsRows * (R + 1) * 4;
}
__host__ __device__ constexpr size_t tcs_smem(int R) { return tcs_tile_bytes(R) + (size_t)2 * 2 * R * 4; }

template <int BITS, int NT>
__global__ void __launch_bounds__(256) qmm_tcs_kernel(QmmArgs a, int ks) {
  namespace cg = cooperative_groups;
  constexpr int R = NT * 8;      // token rows of the tile (M padded to 8)
  constexpr int WPG = 2 * BITS;  // words per group and weight row
  constexpr int LW = BITS / 2;   // words per group, row and lane
  constexpr int RS = R + 1;      // padded token stride of the partial tile
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* xs_tile = smem;                                              // [2][2][R][128 B]
  float* red = reinterpret_cast<float*>(smem);                         // [128][RS] after the loop
  float* xsum = reinterpret_cast<float*>(smem + tcs_tile_bytes(R));    // [2][2][R]
  __shared__ int tile_mi[kTcsWarps], tile_row0[kTcsWarps];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, q = lane >> 2, c = lane & 3;
  const int rank = ks > 1 ? (int)(blockIdx.x % ks) : 0, ctile = (int)blockIdx.x / ks;
  const bool sw = a.mode == QMM_SWIGLU;
  int mi = 0, row0 = 0;
  bool have;
  if (sw) {
    mi = warp >> 2;
    row0 = ctile * (kTcsRows / 2) + 16 * (warp & 3);
    have = row0 < a.N;
  } else {
    have = tcg_tile(a, ctile * kTcsWarps + warp, mi, row0);
  }
  if (lane == 0) {
    tile_mi[warp] = have ? mi : -1;
    tile_row0[warp] = row0;
  }
  const QmmMat& W = mi == 0 ? a.mat[0] : (mi == 1 ? a.mat[1] : a.mat[2]);
  const int G = a.K / 64, rows = sw ? a.N : W.rows;
  const int g0 = rank * G / ks, g1 = (rank + 1) * G / ks;
  const int nblk = (g1 - g0 + 1) / 2;
  const int ra = row0 + q, rb = row0 + q + 8;
  const bool va = have && ra < rows, vb = have && rb < rows;
  const uint32_t* wa = W.w + (size_t)(va ? ra : 0) * G * WPG + LW * c;
  const uint32_t* wb = W.w + (size_t)(vb ? rb : 0) * G * WPG + LW * c;
  const bf16_t* sa_p = W.s + (size_t)(va ? ra : 0) * G;
  const bf16_t* ba_p = W.b + (size_t)(va ? ra : 0) * G;
  const bf16_t* sb_p = W.s + (size_t)(vb ? rb : 0) * G;
  const bf16_t* bb_p = W.b + (size_t)(vb ? rb : 0) * G;

  // weights of a block (2 groups) for rows q, q+8, double-buffered by block
  uint32_t WA[2][2][LW], WB[2][2][LW], SBa[2][2], SBb[2][2];
  auto load_w = [&](int blk, int u) {
#pragma unroll
    for (int gg = 0; gg < 2; ++gg) {
      const int g = g0 + 2 * blk + gg;
      const bool ua = va && blk < nblk && g < g1, ub = vb && blk < nblk && g < g1;
      if constexpr (BITS == 4) {
        const uint2 x0 = ua ? *reinterpret_cast<const uint2*>(wa + (size_t)g * WPG) : make_uint2(0, 0);
        const uint2 x1 = ub ? *reinterpret_cast<const uint2*>(wb + (size_t)g * WPG) : make_uint2(0, 0);
        WA[u][gg][0] = x0.x, WA[u][gg][1] = x0.y, WB[u][gg][0] = x1.x, WB[u][gg][1] = x1.y;
      } else {
        const uint4 x0 = ua ? *reinterpret_cast<const uint4*>(wa + (size_t)g * WPG) : make_uint4(0, 0, 0, 0);
        const uint4 x1 = ub ? *reinterpret_cast<const uint4*>(wb + (size_t)g * WPG) : make_uint4(0, 0, 0, 0);
        WA[u][gg][0] = x0.x, WA[u][gg][1] = x0.y, WA[u][gg][2] = x0.z, WA[u][gg][3] = x0.w;
        WB[u][gg][0] = x1.x, WB[u][gg][1] = x1.y, WB[u][gg][2] = x1.z, WB[u][gg][3] = x1.w;
      }
      SBa[u][gg] = ua ? ((uint32_t)sa_p[g] | ((uint32_t)ba_p[g] << 16)) : 0u;
      SBb[u][gg] = ub ? ((uint32_t)sb_p[g] | ((uint32_t)bb_p[g] << 16)) : 0u;
    }
  };

  // activations: item e = (group gg, token row n, 16-byte chunk j) of a block
  constexpr int NITEM = 2 * R * 8;
  constexpr int NI = (NITEM + 255) / 256;
  uint4 XR[NI];
  auto load_x = [&](int blk) {
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const int e = tid + 256 * i, gg = e / (R * 8), n = (e >> 3) % R, j = e & 7;
      const int g = g0 + 2 * blk + gg;
      XR[i] = make_uint4(0u, 0u, 0u, 0u);
      if (e < NITEM && blk < nblk && g < g1 && n < a.M)
        XR[i] = __ldg(reinterpret_cast<const uint4*>(a.x + (size_t)n * a.ldx + (size_t)g * 64 + 8 * j));
    }
  };
  // store block `u` (swizzled, 4-bit: nibble-pair order) and its group sums
  auto store_x = [&](int u) {
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const int e = tid + 256 * i, gg = e / (R * 8), n = (e >> 3) % R, j = e & 7;
      const uint4 v = XR[i];
      float sum = 0.0f;
      sum = __fadd_rn(sum, lo_bf(v.x)), sum = __fadd_rn(sum, hi_bf(v.x));
      sum = __fadd_rn(sum, lo_bf(v.y)), sum = __fadd_rn(sum, hi_bf(v.y));
      sum = __fadd_rn(sum, lo_bf(v.z)), sum = __fadd_rn(sum, hi_bf(v.z));
      sum = __fadd_rn(sum, lo_bf(v.w)), sum = __fadd_rn(sum, hi_bf(v.w));
      // the 8 chunks of a (group, token) sit on 8 consecutive lanes
      sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 1));
      sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 2));
      sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 4));
      if (e < NITEM) {
        uint4 o = v;
        if constexpr (BITS == 4) {
          o.x = __byte_perm(v.x, v.z, 0x5410);  // (k0, k4)
          o.y = __byte_perm(v.x, v.z, 0x7632);  // (k1, k5)
          o.z = __byte_perm(v.y, v.w, 0x5410);  // (k2, k6)
          o.w = __byte_perm(v.y, v.w, 0x7632);  // (k3, k7)
        }
        *reinterpret_cast<uint4*>(xs_tile + ((size_t)(u * 2 + gg) * R + n) * 128 + ((j ^ (n & 7)) << 4)) = o;
        if (j == 0) xsum[(u * 2 + gg) * R + n] = sum;
      }
    }
  };

  float acc[NT][4];
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[t][e] = 0.0f;
  const uint32_t one2 = 0x3F803F80u, m128 = 0xC300C300u;

  // one group: codes -> exact bf16 A fragments, products per token tile,
  // then acc += s * dot + b * xsum for rows q (e = 0, 1) and q + 8 (e = 2, 3)
  auto group = [&](const uint8_t* xt, const float* xsm, const uint32_t (&A)[LW], const uint32_t (&B)[LW],
                   uint32_t pa, uint32_t pb) {
    uint32_t af[4][4];
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      if constexpr (BITS == 4) {
        const int h = kk >> 1, i = (kk & 1) * 2;
        af[kk][0] = bf2_fma(((A[h] >> (4 * i)) & 0x000F000Fu) | 0x43004300u, one2, m128);
        af[kk][1] = bf2_fma(((B[h] >> (4 * i)) & 0x000F000Fu) | 0x43004300u, one2, m128);
        af[kk][2] = bf2_fma(((A[h] >> (4 * i + 4)) & 0x000F000Fu) | 0x43004300u, one2, m128);
        af[kk][3] = bf2_fma(((B[h] >> (4 * i + 4)) & 0x000F000Fu) | 0x43004300u, one2, m128);
      } else {
        af[kk][0] = bf2_pack(tcg_code8(A[kk], 0), tcg_code8(A[kk], 1));
        af[kk][1] = bf2_pack(tcg_code8(B[kk], 0), tcg_code8(B[kk], 1));
        af[kk][2] = bf2_pack(tcg_code8(A[kk], 2), tcg_code8(A[kk], 3));
        af[kk][3] = bf2_pack(tcg_code8(B[kk], 2), tcg_code8(B[kk], 3));
      }
    }
    const float sa = __uint_as_float(pa << 16), ba = __uint_as_float(pa & 0xFFFF0000u);
    const float sb = __uint_as_float(pb << 16), bb = __uint_as_float(pb & 0xFFFF0000u);
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const uint8_t* rp = xt + (size_t)(t * 8 + q) * 128;
      const uint4 lo = *reinterpret_cast<const uint4*>(rp + (((2 * c) ^ q) << 4));
      const uint4 hi = *reinterpret_cast<const uint4*>(rp + (((2 * c + 1) ^ q) << 4));
      const uint32_t X[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
      float dot[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) mma_16816(dot, af[kk], X[2 * kk], X[2 * kk + 1]);
      const float2 xs = *reinterpret_cast<const float2*>(xsm + t * 8 + 2 * c);
      acc[t][0] = __fmaf_rn(sa, dot[0], __fmaf_rn(ba, xs.x, acc[t][0]));
      acc[t][1] = __fmaf_rn(sa, dot[1], __fmaf_rn(ba, xs.y, acc[t][1]));
      acc[t][2] = __fmaf_rn(sb, dot[2], __fmaf_rn(bb, xs.x, acc[t][2]));
      acc[t][3] = __fmaf_rn(sb, dot[3], __fmaf_rn(bb, xs.y, acc[t][3]));
    }
  };

  // block blk from buffer u (a literal at each call): stage it, one barrier,
  // prefetch the next block's activations and weights, run its groups
  auto step = [&](const int blk, const int u) {
    store_x(u);
    __syncthreads();
    if (blk + 1 < nblk) {
      load_x(blk + 1);
      load_w(blk + 1, u ^ 1);
    }
    if (have) {
#pragma unroll
      for (int gg = 0; gg < 2; ++gg)
        if (g0 + 2 * blk + gg < g1)
          group(xs_tile + (size_t)(u * 2 + gg) * R * 128, xsum + (u * 2 + gg) * R, WA[u][gg], WB[u][gg], SBa[u][gg],
                SBb[u][gg]);
    }
  };

  load_w(0, 0);  // weights do not depend on the previous kernel
  grid_wait();
  grid_launch_dependents();
  load_x(0);
  for (int blk = 0; blk < nblk; blk += 2) {
    step(blk, 0);
    if (blk + 1 < nblk) step(blk + 1, 1);
  }

  // partial tile [128 rows][R tokens] over the activation blocks (every warp
  // is past its last read of them after this barrier)
  __syncthreads();
  if (have) {
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const int m = t * 8 + 2 * c;
      red[(warp * 16 + q) * RS + m] = acc[t][0];
      red[(warp * 16 + q) * RS + m + 1] = acc[t][1];
      red[(warp * 16 + q + 8) * RS + m] = acc[t][2];
      red[(warp * 16 + q + 8) * RS + m + 1] = acc[t][3];
    }
  }
  cg::cluster_group cluster = cg::this_cluster();
  if (ks > 1) cluster.sync();
  else __syncthreads();
  // each rank finishes a share of the tile's outputs, summing the partial
  // tiles in rank order
  const int rows_out = sw ? kTcsRows / 2 : kTcsRows;
  const int total = rows_out * a.M, per = (total + ks - 1) / ks;
  const int i0 = rank * per, i1 = min(total, i0 + per);
  for (int e = i0 + tid; e < i1; e += blockDim.x) {
    const int r = e % rows_out, m = e / rows_out;
    const int w = r >> 4, wm = tile_mi[w];
    if (wm < 0) continue;
    const int row = tile_row0[w] + (r & 15);
    if (row >= (sw ? a.N : (wm == 0 ? a.mat[0].rows : (wm == 1 ? a.mat[1].rows : a.mat[2].rows)))) continue;
    float s0 = 0.0f, s1 = 0.0f;
    for (int k = 0; k < ks; ++k) {
      const float* rr = ks > 1 ? cluster.map_shared_rank(red, k) : red;
      s0 = __fadd_rn(s0, rr[r * RS + m]);
      if (sw) s1 = __fadd_rn(s1, rr[(r + kTcsRows / 2) * RS + m]);
    }
    if (sw) {
      a.y[(size_t)m * a.ldy + row] = swiglu_c(f2bf(s0), f2bf(s1));
    } else {
      const int col = (wm == 0 ? 0 : (wm == 1 ? a.mat[0].rows : a.mat[0].rows + a.mat[1].rows)) + row;
      bf16_t yv = f2bf(s0);
      if (a.mode == QMM_RESID) yv = f2bf(__fadd_rn(bf2f(yv), bf2f(a.res[(size_t)m * a.ldy + col])));
      a.y[(size_t)m * a.ldy + col] = yv;
    }
  }
  if (ks > 1) cluster.sync();  // peers may still read this CTA's partial tile
}

}  // namespace lmx
