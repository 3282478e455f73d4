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
// Memory pipeline, per block of 2 groups (128 k): the CTA's packed weight
// rows and the activations x [M][128] stream into a kTcsStages-deep ring in
// shared memory by cp.async (16-byte copies, no multicast), kTcsStages - 1
// blocks ahead; scales and biases come through registers one block ahead.
// Per block one pass moves the activations from the ring into a
// double-buffered compute tile (16-byte chunks XOR-swizzled by row % 8) and
// forms the per-(token, group) sums with 8-lane shuffles; for 4-bit weights
// each 8-value chunk is stored in the order (k0,k4,k1,k5,k2,k6,k3,k7), the
// order in which a word's nibble pairs come out, so that lane (q, c) loads its
// 16 k of a token as two 16-byte words and uses them as mma B fragments
// unchanged (8-bit chunks stay in k order).  Two barriers per block.
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
static constexpr int kTcsStages = 4;             // ring depth (blocks of 2 groups)

LMX_DEV void tcs_cp16(uint32_t dst, const void* src, uint32_t bytes) {
  // bytes 0: the 16 bytes are zero-filled and nothing is read
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}
LMX_DEV void tcs_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
LMX_DEV void tcs_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Shared-memory layout (bytes) for R token rows and BITS-bit weights:
//   ring[kTcsStages]: weights [8 tiles][2 groups][16 rows][8 BITS bytes],
//                     activations [2 groups][R rows][128 B]
//   compute tile [2][2 groups][R rows][128 B]  (the [128][R + 1] fp32 partial
//                     tile reuses ring + compute tile after the main loop)
//   group sums [2][2 groups][R] fp32, scales / biases [kTcsStages][8][2][16] u32
__host__ __device__ constexpr size_t tcs_w_stage(int bits) { return (size_t)kTcsRows * 2 * 8 * bits; }
__host__ __device__ constexpr size_t tcs_x_stage(int R) { return (size_t)2 * R * 128; }
__host__ __device__ constexpr size_t tcs_ring_bytes(int R, int bits) {
  return (size_t)kTcsStages * (tcs_w_stage(bits) + tcs_x_stage(R));
}
__host__ __device__ constexpr size_t tcs_main_bytes(int R, int bits) {
  return tcs_ring_bytes(R, bits) + (size_t)2 * tcs_x_stage(R);
}
__host__ __device__ constexpr size_t tcs_smem(int R, int bits) {
  return (tcs_main_bytes(R, bits) > (size_t)kTcsRows * (R + 1) * 4 ? tcs_main_bytes(R, bits)
                                                                  : (size_t)kTcsRows * (R + 1) * 4) +
         (size_t)2 * 2 * R * 4 + (size_t)kTcsStages * kTcsRows * 2 * 4;
}

template <int BITS, int NT>
__global__ void __launch_bounds__(256) qmm_tcs_kernel(QmmArgs a, int ks) {
  namespace cg = cooperative_groups;
  constexpr int R = NT * 8;      // token rows of the tile (M padded to 8)
  constexpr int WPG = 2 * BITS;  // words per group and weight row
  constexpr int LW = BITS / 2;   // words per group, row and lane
  constexpr int RS = R + 1;      // padded token stride of the partial tile
  constexpr size_t WST = tcs_w_stage(BITS), XST = tcs_x_stage(R);
  constexpr size_t MAINB = tcs_main_bytes(R, BITS);
  constexpr size_t TAIL = MAINB > (size_t)kTcsRows * RS * 4 ? MAINB : (size_t)kTcsRows * RS * 4;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* wring = smem;                                       // [S][WST]
  uint8_t* xring = smem + kTcsStages * WST;                    // [S][XST]
  uint8_t* xtile = smem + tcs_ring_bytes(R, BITS);             // [2][XST]
  float* red = reinterpret_cast<float*>(smem);                 // [128][RS] after the loop
  float* xsum = reinterpret_cast<float*>(smem + TAIL);         // [2][2][R]
  uint32_t* sbring = reinterpret_cast<uint32_t*>(xsum + 2 * 2 * R);  // [S][8 tiles][2][16]
  __shared__ int tile_mi[kTcsWarps], tile_row0[kTcsWarps];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, q = lane >> 2, c = lane & 3;
  const int rank = ks > 1 ? (int)(blockIdx.x % ks) : 0, ctile = (int)blockIdx.x / ks;
  const bool sw = a.mode == QMM_SWIGLU;
  if (tid < kTcsWarps) {
    int mi = 0, row0 = 0;
    bool have;
    if (sw) {
      mi = tid >> 2;
      row0 = ctile * (kTcsRows / 2) + 16 * (tid & 3);
      have = row0 < a.N;
    } else {
      have = tcg_tile(a, ctile * kTcsWarps + tid, mi, row0);
    }
    tile_mi[tid] = have ? mi : -1;
    tile_row0[tid] = row0;
  }
  __syncthreads();
  const int G = a.K / 64;
  const int g0 = rank * G / ks, g1 = (rank + 1) * G / ks;
  const int nblk = (g1 - g0 + 1) / 2;
  const bool have = tile_mi[warp] >= 0;
  auto mat_of = [&](int mi) -> const QmmMat& { return mi == 0 ? a.mat[0] : (mi == 1 ? a.mat[1] : a.mat[2]); };
  auto rows_of = [&](int mi) { return sw ? a.N : mat_of(mi).rows; };

  // ---- staging of block blk into ring stage st ----
  // Each thread's copies are fixed for the whole K range: its weight chunks
  // (tile, group, row, 16-byte part) and activation chunks (group, token,
  // 16-byte part) differ between blocks only by the group offset, so the row
  // addresses and validity are formed once here.
  constexpr int CH16 = WPG * 4 / 16;  // 16-byte chunks per weight row and group
  constexpr int WITEM = kTcsWarps * 2 * 16 * CH16;
  constexpr int XITEM = 2 * R * 8;
  constexpr int NWI = (WITEM + 255) / 256, NXI = (XITEM + 255) / 256;
  const uint32_t* wsrc[NWI];  // row start + the chunk's word offset, nullptr when invalid
  uint32_t wdst[NWI];
  int wgg[NWI];
#pragma unroll
  for (int i = 0; i < NWI; ++i) {
    const int e = tid + 256 * i;
    const int h = e % CH16, r = (e / CH16) & 15, gg = (e / (CH16 * 16)) & 1, w = e / (CH16 * 32);
    wsrc[i] = nullptr;
    wdst[i] = (uint32_t)((((w * 2 + gg) * 16 + r) * WPG * 4) + 16 * h);
    wgg[i] = gg;
    if (e < WITEM) {
      const int mi = tile_mi[w], row = tile_row0[w] + r;
      if (mi >= 0 && row < rows_of(mi)) wsrc[i] = mat_of(mi).w + (size_t)row * G * WPG + 4 * h;
    } else {
      wdst[i] = 0xFFFFFFFFu;
    }
  }
  const bf16_t* xsrc[NXI];  // token row + the chunk's offset, nullptr when the token is padding
  uint32_t xdst[NXI];
  int xgg[NXI];
#pragma unroll
  for (int i = 0; i < NXI; ++i) {
    const int e = tid + 256 * i, gg = e / (R * 8), n = (e >> 3) % R, j = e & 7;
    xsrc[i] = (e < XITEM && n < a.M) ? a.x + (size_t)n * a.ldx + 8 * j : nullptr;
    xdst[i] = e < XITEM ? (uint32_t)((gg * R + n) * 128 + 16 * j) : 0xFFFFFFFFu;
    xgg[i] = gg;
  }
  auto issue_w = [&](int blk, int st) {
    const uint32_t base = smem_u32(wring + (size_t)st * WST);
#pragma unroll
    for (int i = 0; i < NWI; ++i) {
      if (wdst[i] == 0xFFFFFFFFu) continue;
      const int g = g0 + 2 * blk + wgg[i];
      const bool v = wsrc[i] != nullptr && g < g1;
      tcs_cp16(base + wdst[i], v ? wsrc[i] + (size_t)g * WPG : a.mat[0].w, v ? 16u : 0u);
    }
  };
  auto issue_x = [&](int blk, int st) {
    const uint32_t base = smem_u32(xring + (size_t)st * XST);
#pragma unroll
    for (int i = 0; i < NXI; ++i) {
      if (xdst[i] == 0xFFFFFFFFu) continue;
      const int g = g0 + 2 * blk + xgg[i];
      const bool v = xsrc[i] != nullptr && g < g1;
      tcs_cp16(base + xdst[i], v ? xsrc[i] + (size_t)g * 64 : a.x, v ? 16u : 0u);
    }
  };
  auto issue = [&](int blk, int st) {
    if (blk < nblk) {  // past the CTA's range: an empty group keeps the count
      issue_w(blk, st);
      issue_x(blk, st);
    }
    tcs_commit();
  };
  // scale | bias << 16 of one (tile, group, row) per thread
  const bf16_t *sbs = nullptr, *sbb = nullptr;
  {
    const int w = tid >> 5, r = tid & 15, mi = tile_mi[w], row = tile_row0[w] + r;
    if (mi >= 0 && row < rows_of(mi)) {
      sbs = mat_of(mi).s + (size_t)row * G;
      sbb = mat_of(mi).b + (size_t)row * G;
    }
  }
  const int sbgg = (tid >> 4) & 1;
  auto load_sb = [&](int blk) -> uint32_t {
    const int g = g0 + 2 * blk + sbgg;
    if (!sbs || g >= g1 || blk >= nblk) return 0u;
    return (uint32_t)sbs[g] | ((uint32_t)sbb[g] << 16);
  };
  auto store_sb = [&](int st, uint32_t v) { sbring[(st * kTcsWarps + (tid >> 5)) * 32 + (tid & 31)] = v; };

  // ring stage st -> compute tile u (swizzled, 4-bit: nibble-pair order) and
  // the per-(group, token) sums of x
  auto stage_x = [&](int st, int u) {
    const uint8_t* xr = xring + (size_t)st * XST;
#pragma unroll
    for (int i = 0; i < (XITEM + 255) / 256; ++i) {
      const int e = tid + 256 * i, gg = e / (R * 8), n = (e >> 3) % R, j = e & 7;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (e < XITEM) v = *reinterpret_cast<const uint4*>(xr + (gg * R + n) * 128 + 16 * j);
      float sum = 0.0f;
      sum = __fadd_rn(sum, lo_bf(v.x)), sum = __fadd_rn(sum, hi_bf(v.x));
      sum = __fadd_rn(sum, lo_bf(v.y)), sum = __fadd_rn(sum, hi_bf(v.y));
      sum = __fadd_rn(sum, lo_bf(v.z)), sum = __fadd_rn(sum, hi_bf(v.z));
      sum = __fadd_rn(sum, lo_bf(v.w)), sum = __fadd_rn(sum, hi_bf(v.w));
      // the 8 chunks of a (group, token) sit on 8 consecutive lanes
      sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 1));
      sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 2));
      sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 4));
      if (e < XITEM) {
        uint4 o = v;
        if constexpr (BITS == 4) {
          o.x = __byte_perm(v.x, v.z, 0x5410);  // (k0, k4)
          o.y = __byte_perm(v.x, v.z, 0x7632);  // (k1, k5)
          o.z = __byte_perm(v.y, v.w, 0x5410);  // (k2, k6)
          o.w = __byte_perm(v.y, v.w, 0x7632);  // (k3, k7)
        }
        *reinterpret_cast<uint4*>(xtile + (size_t)u * XST + (gg * R + n) * 128 + ((j ^ (n & 7)) << 4)) = o;
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

  // one group of this warp's tile: codes -> exact bf16 A fragments, products
  // per token tile, acc += s * dot + b * xsum (rows q: e = 0, 1; q+8: e = 2, 3)
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
  auto compute = [&](int blk, int u, int st) {
#pragma unroll
    for (int gg = 0; gg < 2; ++gg) {
      if (g0 + 2 * blk + gg >= g1) break;
      const uint8_t* wr = wring + (size_t)st * WST + (size_t)(warp * 2 + gg) * 16 * WPG * 4 + 4 * LW * c;
      uint32_t A[LW], B[LW];
      if constexpr (BITS == 4) {
        const uint2 x0 = *reinterpret_cast<const uint2*>(wr + q * WPG * 4);
        const uint2 x1 = *reinterpret_cast<const uint2*>(wr + (q + 8) * WPG * 4);
        A[0] = x0.x, A[1] = x0.y, B[0] = x1.x, B[1] = x1.y;
      } else {
        const uint4 x0 = *reinterpret_cast<const uint4*>(wr + q * WPG * 4);
        const uint4 x1 = *reinterpret_cast<const uint4*>(wr + (q + 8) * WPG * 4);
        A[0] = x0.x, A[1] = x0.y, A[2] = x0.z, A[3] = x0.w;
        B[0] = x1.x, B[1] = x1.y, B[2] = x1.z, B[3] = x1.w;
      }
      const uint32_t* sbp = sbring + (st * kTcsWarps + warp) * 32 + gg * 16;
      group(xtile + (size_t)u * XST + (size_t)gg * R * 128, xsum + (u * 2 + gg) * R, A, B, sbp[q], sbp[q + 8]);
    }
  };

  // prologue: the first blocks' weights and scales do not depend on the
  // previous kernel and are requested before waiting for it
  uint32_t sb0[kTcsStages - 1];
#pragma unroll
  for (int b = 0; b < kTcsStages - 1; ++b) {
    if (b < nblk) issue_w(b, b);
    sb0[b] = load_sb(b);
  }
  grid_wait();
  grid_launch_dependents();
#pragma unroll
  for (int b = 0; b < kTcsStages - 1; ++b) {
    if (b < nblk) issue_x(b, b);
    tcs_commit();
    store_sb(b, sb0[b]);
  }
  uint32_t sbv = 0u;
  for (int blk = 0; blk < nblk; ++blk) {
    const int st = blk % kTcsStages, u = blk & 1;
    tcs_wait<kTcsStages - 2>();  // this thread's copies of block blk have landed
    __syncthreads();             // everyone's have; every warp is done with block blk - 1
    if (blk > 0) store_sb((blk + kTcsStages - 2) % kTcsStages, sbv);
    sbv = load_sb(blk + kTcsStages - 1);
    issue(blk + kTcsStages - 1, (blk + kTcsStages - 1) % kTcsStages);
    stage_x(st, u);
    __syncthreads();
    if (have) compute(blk, u, st);
  }
  tcs_wait<0>();  // no copy may land on the partial tile below

  // partial tile [128 rows][R tokens] over the shared memory used above
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
    if (row >= rows_of(wm)) continue;
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
