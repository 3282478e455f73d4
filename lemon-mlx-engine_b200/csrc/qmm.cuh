// qmm.cuh -- K1: quantized GEMV for the verify / draft pass (M < 16).
//
// Replaces mx::quantized_matmul (include/mlx-lm/common/quantized_linear.h:82-85)
// for skinny M.  HBM-bound: every weight byte is read once, unpack and
// dequant are fused, activations stay in registers for the whole row sweep.
//
// Work decomposition (block = 256 threads, one CTA per SM):
//   * A "segment" is 512 consecutive k (8 groups of 64).  Warp w owns segment
//     w % NSEG of the rows of row-slot w / NSEG; lane l owns quarter l (16 k)
//     of that segment, so a warp reads one contiguous 256 B (4-bit) / 512 B
//     (8-bit) run per row.
//   * Weights stream HBM -> shared memory through cp.async.bulk (the TMA
//     engine) into an NST-deep per-warp ring completed on mbarriers; the first
//     NST stages are issued before griddepcontrol.wait, overlapping the
//     previous kernel's tail (weights never depend on it).
//   * Activations for up to MT rows are loaded once into registers
//     (16 values per m per lane), optionally RMS-normalised on the way in,
//     and pre-scaled by 16^-(j%4) (4-bit) / 256^-(j%2) (8-bit) so the nibble /
//     byte can be used in place inside a 2^23 "magic" float without shifting.
//     (q*16^r)*(x*16^-r) == q*x exactly for normal x.
//   * Per batch of RB rows each lane forms RB*MT quarter dot-products, then a
//     reduce-scatter shuffle tree (one shuffle per two values per level)
//     produces the group and segment sums in the canonical order below.
//
// Canonical fp32 order (identical to oracle/oracle.cpp orc_qmm):
//   Q_c  = fma chain over the 16 k of quarter c, ascending, from 0
//   X_c  = add chain of x over quarter c, ascending, from 0
//   d_g  = (Q_4g + Q_4g+1) + (Q_4g+2 + Q_4g+3);  xs_g likewise
//   e_g  = fma(s_g, d_g, b_g * xs_g)
//   t    = ((e0+e1)+(e2+e3)) + ((e4+e5)+(e6+e7))   per segment
//   y    = bf16(t_0 + t_1 + ... )                  segments left to right
#pragma once
#include <cooperative_groups.h>
#include "lmx_common.cuh"
namespace cg = cooperative_groups;

namespace lmx {

struct QmmMat {
  const uint32_t* w;
  const bf16_t* s;
  const bf16_t* b;
  int rows;
};

enum { QMM_PLAIN = 0, QMM_RESID = 1, QMM_SWIGLU = 2 };

struct QmmArgs {
  const bf16_t* x;       // [M, K]
  const bf16_t* norm_w;  // optional RMSNorm weight [K] applied to x in the prologue
  float eps;
  QmmMat mat[3];         // PLAIN/RESID: virtual rows = concatenation; SWIGLU: gate, up
  int nmat;
  int N;                 // virtual rows (PLAIN/RESID) or rows per matrix (SWIGLU)
  bf16_t* y;             // [M, ldy]
  int ldy;
  const bf16_t* res;     // RESID: y = bf16(bf16(acc) + res), res [M, ldy] (may alias y)
  int M, K;
  int mode;
  unsigned* err;         // device error word (bounded-wait timeouts)
};

static constexpr int kQmmThreads = 256;
static constexpr int kQmmMaxNormRows = 64;

LMX_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

LMX_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
LMX_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
LMX_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
LMX_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: gives up after ~2^22 polls (seconds), flags the error word.
LMX_DEV bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, unsigned* err, unsigned code) {
  for (uint32_t i = 0; i < (1u << 22); ++i)
    if (mbar_try_wait(bar, parity)) return true;
  if (err) atomicExch(err, code);
  return false;
}

LMX_DEV bool qmm_item_row(const QmmArgs& a, int item, int& mi, int& row) {
  if (a.mode == QMM_SWIGLU) {
    mi = item & 1;
    row = item >> 1;
    return row < a.N;
  }
  int r = item;
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    if (i < a.nmat) {
      if (r < a.mat[i].rows) {
        mi = i;
        row = r;
        return true;
      }
      r -= a.mat[i].rows;
    }
  }
  return false;
}

LMX_DEV const QmmMat& qmm_mat(const QmmArgs& a, int mi) {
  return mi == 0 ? a.mat[0] : (mi == 1 ? a.mat[1] : a.mat[2]);
}

// One reduce-scatter level over N (compile-time) values: the lane keeps the
// upper half if `up`, adding the partner's copy of the same items (a+b == b+a,
// so both lanes of a pair form the same canonical sum).  N == 1 is a plain
// butterfly step (value replicated in both lanes).
template <int N, int CAP>
LMX_DEV void rs_level(float (&v)[CAP], int off, bool up, int& base) {
  if constexpr (N >= 2) {
#pragma unroll
    for (int k = 0; k < N / 2; ++k) {
      float send = up ? v[k] : v[k + N / 2];
      float keep = up ? v[k + N / 2] : v[k];
      v[k] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, off));
    }
    if (up) base += N / 2;
  } else {
    v[0] = __fadd_rn(v[0], __shfl_xor_sync(0xffffffffu, v[0], off));
  }
}
__host__ __device__ constexpr int cmax1(int a) { return a < 1 ? 1 : a; }

template <int BITS>
LMX_DEV void unpack_quarter(const uint8_t* p, float (&q)[16]) {
  const float kMagic = 8388608.0f;  // 2^23
  if (BITS == 4) {
    uint2 w = *reinterpret_cast<const uint2*>(p);
    const uint32_t src[4] = {w.x, w.x >> 16, w.y, w.y >> 16};
#pragma unroll
    for (int h = 0; h < 4; ++h) {
#pragma unroll
      for (int r = 0; r < 4; ++r)
        q[4 * h + r] = __fsub_rn(__uint_as_float((src[h] & (0xFu << (4 * r))) | 0x4B000000u), kMagic);
    }
  } else {
    uint4 w = *reinterpret_cast<const uint4*>(p);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t lo = ws[k], hi = ws[k] >> 16;
      q[4 * k + 0] = __fsub_rn(__uint_as_float((lo & 0xFFu) | 0x4B000000u), kMagic);
      q[4 * k + 1] = __fsub_rn(__uint_as_float((lo & 0xFF00u) | 0x4B000000u), kMagic);
      q[4 * k + 2] = __fsub_rn(__uint_as_float((hi & 0xFFu) | 0x4B000000u), kMagic);
      q[4 * k + 3] = __fsub_rn(__uint_as_float((hi & 0xFF00u) | 0x4B000000u), kMagic);
    }
  }
}

template <int BITS>
LMX_DEV float quarter_prescale(int j) {
  if (BITS == 4) return (j & 3) == 0 ? 1.0f : ((j & 3) == 1 ? 0.0625f : ((j & 3) == 2 ? 0.00390625f : 0.000244140625f));
  return (j & 1) ? 0.00390625f : 1.0f;
}

// Shared-memory layout of qmv_kernel (per CTA, 8 warps):
//   [warp][nst][RB][SEGB] weight ring | [warp][nst] mbarriers |
//   [2][rs][8][V] segment partials | [kQmmMaxNormRows] RMSNorm factors
// K <= 4096: one CTA covers a row (rs = 8 / nseg row slots per CTA).
// K  > 4096: a cluster of ceil(nseg/8) CTAs covers a row (rs = 1); rank 0
//            sums the segment partials of all ranks through DSMEM.
template <int BITS, int MT, int RB>
__global__ void __launch_bounds__(kQmmThreads, 1) qmv_kernel(QmmArgs a, int nst) {
  constexpr int V = RB * MT;
  constexpr int QB = 16 * BITS / 8;
  constexpr int SEGB = 32 * QB;
  constexpr int N1 = cmax1(V / 2), N2 = cmax1(V / 4), N3 = cmax1(V / 8), N4 = cmax1(V / 16),
                N5 = cmax1(V / 32);
  constexpr int NW = kQmmThreads / 32;
  extern __shared__ __align__(128) uint8_t smem[];
  cg::cluster_group cluster = cg::this_cluster();
  const int csize = (int)cluster.num_blocks(), crank = (int)cluster.block_rank();

  const int K = a.K, M = a.M;
  const int nseg = (K + 511) >> 9;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int rs, seg, slot, lseg;
  if (csize == 1) {
    rs = NW / nseg;
    seg = warp % nseg;
    slot = warp / nseg;
    lseg = seg;
  } else {
    rs = 1;
    seg = crank * NW + warp;
    slot = 0;
    lseg = warp;
  }
  const bool wactive = slot < rs && seg < nseg;

  uint8_t* wst = smem + (size_t)warp * nst * RB * SEGB;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)NW * nst * RB * SEGB) + warp * nst;
  float* red = reinterpret_cast<float*>(smem + (size_t)NW * nst * RB * SEGB + (size_t)NW * nst * 8);
  float* fnorm = red + 2 * NW * V;

  const int k0 = seg * 512 + 16 * lane;
  const bool qvalid = wactive && k0 < K;
  const uint32_t segbytes = wactive ? (uint32_t)(min(512, K - seg * 512) * BITS / 8) : 0u;
  const int G = K >> 6;
  const int g = k0 >> 6;
  const int KWB = K * BITS / 8;
  const int items = a.mode == QMM_SWIGLU ? 2 * a.N : a.N;
  const int nbatch = (items + RB - 1) / RB;
  const int cid = blockIdx.x / csize, ncl = gridDim.x / csize;
  const int bstride = ncl * rs;
  const int niter = (nbatch - cid * rs + bstride - 1) / bstride;
  const int nmt = (M + MT - 1) / MT;
  const int ntask = niter > 0 ? niter * nmt : 0;

  auto batch_of = [&](int t) { return cid * rs + slot + (t % niter) * bstride; };
  auto issue = [&](int t) {
    if (!wactive || t >= ntask) return;
    const int st = t % nst, batch = batch_of(t);
    uint32_t bytes = 0;
    int mi, row;
#pragma unroll
    for (int i = 0; i < RB; ++i)
      if (batch < nbatch && qmm_item_row(a, batch * RB + i, mi, row)) bytes += segbytes;
    mbar_arrive_expect_tx(&bars[st], bytes);
#pragma unroll
    for (int i = 0; i < RB; ++i)
      if (batch < nbatch && qmm_item_row(a, batch * RB + i, mi, row)) {
        const uint8_t* src = reinterpret_cast<const uint8_t*>(qmm_mat(a, mi).w) + (size_t)row * KWB +
                             (size_t)seg * SEGB;
        bulk_g2s(wst + (size_t)(st * RB + i) * SEGB, src, segbytes, &bars[st]);
      }
  };

  if (lane == 0 && wactive) {
    for (int s = 0; s < nst; ++s) mbar_init(&bars[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  if (lane == 0)
    for (int t = 0; t < nst; ++t) issue(t);

  grid_wait();
  grid_launch_dependents();

  if (a.norm_w) {
    for (int m = warp; m < M; m += NW) {
      const bf16_t* xrow = a.x + (size_t)m * K;
      float p = 0.0f;
      for (int i = lane; i < K; i += 32) {
        float v = bf2f(xrow[i]);
        p = __fmaf_rn(v, v, p);
      }
      p = warp_sum_xor(p, 16, 1);
      if (lane == 0) fnorm[m] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(p, (float)K), a.eps)));
    }
  }
  __syncthreads();

  float nw[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) nw[j] = (a.norm_w && qvalid) ? bf2f(a.norm_w[k0 + j]) : 1.0f;

  float xr[MT][16];
  float xg[MT];
  bool abort_ = false;

  for (int t = 0; t < ntask; ++t) {
    const int st = t % nst;
    const int it = t % niter;
    const int mt0 = (t / niter) * MT;
    const int mcnt = min(MT, M - mt0);
    const int batch = batch_of(t);

    if (it == 0) {
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        float X = 0.0f;
        if (m < mcnt && qvalid) {
          const bf16_t* src = a.x + (size_t)(mt0 + m) * K + k0;
          uint4 r0 = *reinterpret_cast<const uint4*>(src);
          uint4 r1 = *reinterpret_cast<const uint4*>(src + 8);
          const uint32_t rw[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
          const float f = a.norm_w ? fnorm[mt0 + m] : 1.0f;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float v = (j & 1) ? hi_bf(rw[j >> 1]) : lo_bf(rw[j >> 1]);
            if (a.norm_w) v = bf2f(f2bf(__fmul_rn(__fmul_rn(v, f), nw[j])));
            X = __fadd_rn(X, v);
            xr[m][j] = __fmul_rn(v, quarter_prescale<BITS>(j));
          }
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) xr[m][j] = 0.0f;
        }
        X = __fadd_rn(X, __shfl_xor_sync(0xffffffffu, X, 1));
        X = __fadd_rn(X, __shfl_xor_sync(0xffffffffu, X, 2));
        xg[m] = X;
      }
    }

    float sv[RB], bv[RB];
#pragma unroll
    for (int i = 0; i < RB; ++i) {
      int mi, row;
      sv[i] = 0.0f;
      bv[i] = 0.0f;
      if (qvalid && batch < nbatch && qmm_item_row(a, batch * RB + i, mi, row)) {
        const QmmMat& mm = qmm_mat(a, mi);
        sv[i] = bf2f(mm.s[(size_t)row * G + g]);
        bv[i] = bf2f(mm.b[(size_t)row * G + g]);
      }
    }

    if (wactive && !abort_)
      if (!mbar_wait_bounded(&bars[st], (uint32_t)((t / nst) & 1), a.err, 0x51u)) abort_ = true;

    float v[V];
#pragma unroll
    for (int i = 0; i < RB; ++i) {
      float q[16];
      if (qvalid) {
        unpack_quarter<BITS>(wst + (size_t)(st * RB + i) * SEGB + lane * QB, q);
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) q[j] = 0.0f;
      }
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        float Q = 0.0f;
        if (m < mcnt) {
#pragma unroll
          for (int j = 0; j < 16; ++j) Q = __fmaf_rn(q[j], xr[m][j], Q);
        }
        v[i * MT + m] = Q;
      }
    }
    __syncwarp();
    if (lane == 0 && !abort_) issue(t + nst);

    // group level (lane bits 0,1): d = (Q0+Q1)+(Q2+Q3)
    int base = 0;
    bool owner = true;
    rs_level<V>(v, 1, lane & 1, base);
    if (V < 2) owner = owner && !(lane & 1);
    rs_level<N1>(v, 2, (lane >> 1) & 1, base);
    if (N1 < 2) owner = owner && !((lane >> 1) & 1);
    // e = fma(s, d, b * xs) on the N2 items this lane holds
#pragma unroll
    for (int k = 0; k < N2; ++k) {
      const int idx = base + k, i = idx / MT, m = idx % MT;
      float s = sv[0], b = bv[0], xs = xg[0];
#pragma unroll
      for (int r = 1; r < RB; ++r)
        if (i == r) { s = sv[r]; b = bv[r]; }
#pragma unroll
      for (int r = 1; r < MT; ++r)
        if (m == r) xs = xg[r];
      v[k] = __fmaf_rn(s, v[k], __fmul_rn(b, xs));
    }
    // segment tree over 8 groups (lane bits 2,3,4)
    rs_level<N2>(v, 4, (lane >> 2) & 1, base);
    if (N2 < 2) owner = owner && !((lane >> 2) & 1);
    rs_level<N3>(v, 8, (lane >> 3) & 1, base);
    if (N3 < 2) owner = owner && !((lane >> 3) & 1);
    rs_level<N4>(v, 16, (lane >> 4) & 1, base);
    if (N4 < 2) owner = owner && !((lane >> 4) & 1);

    float* rb = red + (size_t)(t & 1) * NW * V;
    if (wactive && owner) {
#pragma unroll
      for (int k = 0; k < N5; ++k) rb[(size_t)warp * V + base + k] = v[k];
    }
    if (csize == 1) __syncthreads();
    else cluster.sync();

    // epilogue: segment partials left to right, then the fused op
    const bool epi = (csize == 1) ? (slot < rs && seg == 0) : (crank == 0 && warp == 0);
    if (epi) {
      for (int idx = lane; idx < V; idx += 32) {
        const int i = idx / MT, m = idx % MT;
        int mi, row;
        if (m >= mcnt || batch >= nbatch || !qmm_item_row(a, batch * RB + i, mi, row)) continue;
        const int item = batch * RB + i;
        float tot = 0.0f, tu = 0.0f;
        for (int s = 0; s < nseg; ++s) {
          const float* src;
          if (csize == 1) src = rb + (size_t)(slot * nseg + s) * V;
          else src = cluster.map_shared_rank(rb, s / NW) + (size_t)(s % NW) * V;
          tot = s == 0 ? src[idx] : __fadd_rn(tot, src[idx]);
          if (a.mode == QMM_SWIGLU) tu = s == 0 ? src[idx + MT] : __fadd_rn(tu, src[idx + MT]);
        }
        const size_t orow = (size_t)(mt0 + m) * a.ldy;
        if (a.mode == QMM_SWIGLU) {
          if (mi == 0) a.y[orow + row] = swiglu_c(f2bf(tot), f2bf(tu));
        } else {
          bf16_t yv = f2bf(tot);
          if (a.mode == QMM_RESID) yv = f2bf(__fadd_rn(bf2f(yv), bf2f(a.res[orow + item])));
          a.y[orow + item] = yv;
        }
      }
    }
  }
  if (csize > 1) cluster.sync();  // keep every rank's shared memory alive until rank 0 is done
}

}  // namespace lmx
