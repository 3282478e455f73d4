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
#include <cuda.h>
#include "lmx_common.cuh"
#include "norm_argmax.cuh"
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
  const bf16_t* x;       // [M, ldx]
  int ldx;               // row stride of x (elements, multiple of 8)
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
  int pstart[3];         // PLAIN/RESID: first virtual row of each matrix (multiple of RB)
  int cstart[3];         // PLAIN/RESID: first output column of each matrix
  int items;             // virtual rows (incl. padding) / swiglu items
};

// TMA descriptors: weights as uint32 [rows][K*bits/32], scales and biases as
// bf16 [rows][K/64]; box = one 512-k segment x (RB or RB/2 for SWIGLU) rows.
struct QmmMaps {
  CUtensorMap w[3], s[3], b[3];
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
#ifdef LMX_MBAR_POLL
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
#else
  // suspend-time hint 1 ms: the thread sleeps in hardware until the phase
  // completes (or the hint expires) instead of spinning on issue slots
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
      : "memory");
#endif
  return ok != 0;
}
LMX_DEV uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait: gives up after 4 s of wall time or 2^26 polls, whichever
// comes first, and flags the error word.  The polling loop is out of line so
// that the common case (phase already complete) stays a few instructions,
// and it backs off with nanosleep (32 ns doubling to 256 ns): warps that run
// ahead of a pipeline would otherwise spin and take issue slots from the
// warps whose work they are waiting for.
__device__ __noinline__ bool mbar_wait_slow(uint64_t* bar, uint32_t parity, unsigned* err, unsigned code) {
  const uint64_t t0 = global_ns();
  uint32_t ns = 32;
  for (uint32_t i = 1; i < (1u << 26); ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    __nanosleep(ns);
    if (ns < 256) ns <<= 1;
    if (global_ns() - t0 > 4000000000ull) break;
  }
  if (err) atomicExch(err, code);
  return false;
}
LMX_DEV bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, unsigned* err, unsigned code) {
  if (mbar_try_wait(bar, parity)) return true;
  return mbar_wait_slow(bar, parity, err, code);
}

// Item -> (matrix, row).  PLAIN/RESID: items are the concatenated rows of
// mat[0..nmat).  SWIGLU: a batch of RB items holds RB/2 gate rows followed by
// the same RB/2 up rows, so both runs are contiguous in memory and in smem.
template <int RB>
LMX_DEV bool qmm_item_row(const QmmArgs& a, int item, int& mi, int& row) {
  if (a.mode == QMM_SWIGLU) {
    const int bt = item / RB, w = item % RB;
    mi = w / (RB / 2);
    row = bt * (RB / 2) + w % (RB / 2);
    return row < a.N;
  }
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    if (i < a.nmat && item >= a.pstart[i] && item < a.pstart[i] + a.mat[i].rows) {
      mi = i;
      row = item - a.pstart[i];
      return true;
    }
  }
  return false;
}

LMX_DEV void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
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

// Two independent IEEE fp32 FMAs / adds in one sm_100 instruction.  Each
// lane of the pair rounds exactly like __fmaf_rn / __fadd_rn.
LMX_DEV void fma2(float& d0, float& d1, float a0, float a1, float b) {
  asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %4};\n"
      " mov.b64 rd, {%0, %1};\n fma.rn.f32x2 rd, ra, rb, rd;\n mov.b64 {%0, %1}, rd;\n}\n"
      : "+f"(d0), "+f"(d1)
      : "f"(a0), "f"(a1), "f"(b));
}
LMX_DEV void sub_magic2(float& a0, float& a1) {
  asm("{\n .reg .b64 ra, rc;\n mov.b64 ra, {%0, %1};\n mov.b64 rc, {%2, %2};\n"
      " add.rn.f32x2 ra, ra, rc;\n mov.b64 {%0, %1}, ra;\n}\n"
      : "+f"(a0), "+f"(a1)
      : "f"(-8388608.0f));
}

// Quarter unpack into "magic" floats 2^23 + q*scale_j (the 2^23 is removed
// by sub_magic2 on row pairs).
template <int BITS>
LMX_DEV void unpack_quarter_raw(const uint8_t* p, float (&q)[16]) {
  if (BITS == 4) {
    uint2 w = *reinterpret_cast<const uint2*>(p);
    const uint32_t src[4] = {w.x, w.x >> 16, w.y, w.y >> 16};
#pragma unroll
    for (int h = 0; h < 4; ++h) {
#pragma unroll
      for (int r = 0; r < 4; ++r) q[4 * h + r] = __uint_as_float((src[h] & (0xFu << (4 * r))) | 0x4B000000u);
    }
  } else {
    uint4 w = *reinterpret_cast<const uint4*>(p);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t lo = ws[k], hi = ws[k] >> 16;
      q[4 * k + 0] = __uint_as_float((lo & 0xFFu) | 0x4B000000u);
      q[4 * k + 1] = __uint_as_float((lo & 0xFF00u) | 0x4B000000u);
      q[4 * k + 2] = __uint_as_float((hi & 0xFFu) | 0x4B000000u);
      q[4 * k + 3] = __uint_as_float((hi & 0xFF00u) | 0x4B000000u);
    }
  }
}

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

// Launch plan (computed on the host by qmv_plan(), identical for every CTA).
struct QmvPlan {
  int W;          // warps per row slot inside one CTA
  int SPW;        // segments (512 k) per warp
  int rs;         // row slots per CTA
  int nst;        // TMA ring depth per warp
  int RP, SP;     // smem bytes of one stage's weight rows / of its scale rows
  int SPH;        // offset of the second (SWIGLU up-rows) scale box, 128-aligned
  int stage;      // bytes per warp stage
  int red_off, vbuf_off, bar_off, stage_off;
  int sb_bulk;    // scales / biases come through the TMA ring
};

LMX_DEV void named_barrier(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// qmv_kernel.  Each warp owns SPW consecutive segments of the rows of its row
// slot and streams them through its own cp.async.bulk ring (no block-wide
// barrier in the main loop).  When a row needs more than one warp (W > 1) or
// more than one CTA (cluster), the first warp continues the left-to-right
// segment chain with the other warps' per-segment sums (named barrier / DSMEM).
// Row pairs share one fma.rn.f32x2; the fp32 op sequence of every output is
// still the canonical one above.
template <int BITS, int MT, int RB>
__global__ void __launch_bounds__(kQmmThreads, MT <= 2 ? 2 : 1) qmv_kernel(const __grid_constant__ QmmMaps mp, QmmArgs a, QmvPlan p) {
  constexpr int V = RB * MT;
  constexpr int QB = 2 * BITS;
  constexpr int SEGB = 32 * QB;
  constexpr int NW = kQmmThreads / 32;
  constexpr int SPWMAX = 1;
  constexpr int N1 = cmax1(V / 2), N2 = cmax1(V / 4), N3 = cmax1(V / 8), N4 = cmax1(V / 16),
                N5 = cmax1(V / 32);
  static_assert(RB >= 4 && RB % 4 == 0, "RB");
  extern __shared__ __align__(128) uint8_t smem[];
  cg::cluster_group cluster = cg::this_cluster();
  const int csize = (int)cluster.num_blocks(), crank = (int)cluster.block_rank();

  const int K = a.K, M = a.M;
  const int nseg = (K + 511) >> 9, G = K >> 6;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slot = csize == 1 ? warp / p.W : 0;
  const int widx = csize == 1 ? warp % p.W : warp;
  const bool inslot = slot < p.rs;
  const int gw = (csize == 1 ? 0 : crank * NW) + widx;  // warp rank along the row
  const int seg0 = gw * p.SPW;
  const int nsw = inslot ? max(0, min(p.SPW, nseg - seg0)) : 0;
  const int nwr = csize == 1 ? p.W : NW * csize;  // warps along a row (incl. idle ones)

  float* fnorm = reinterpret_cast<float*>(smem);
  float* red = reinterpret_cast<float*>(smem + p.red_off);
  float* vbuf = reinterpret_cast<float*>(smem + p.vbuf_off) + (size_t)warp * V * 32;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.bar_off) + warp * p.nst;
  uint8_t* stages = smem + p.stage_off + (size_t)warp * p.nst * p.stage;

  const int nbatch = (a.items + RB - 1) / RB;
  const int cid = blockIdx.x / csize, ncl = gridDim.x / csize;
  const int bstride = ncl * p.rs;
  const int niter = (nbatch - cid * p.rs + bstride - 1) / bstride;
  const int nmt = (M + MT - 1) / MT;
  const int ntask = niter > 0 ? niter * nmt : 0;
  auto batch_of = [&](int t) { return cid * p.rs + slot + (t % niter) * bstride; };

  // issuer (lane 0 of each warp): one 2D tensor copy per tensor and stage
  // (two for SWIGLU: the gate rows and the up rows of the batch)
  auto issue = [&](int t) {
    if (nsw == 0 || t >= ntask) return;
    const int st = t % p.nst, batch = batch_of(t);
    uint8_t* dst = stages + (size_t)st * p.stage;
    uint64_t* bar = &bars[st];
    int mi = 0, row = 0;
    const bool valid = batch < nbatch && qmm_item_row<RB>(a, batch * RB, mi, row);
    if (!valid) {
      mbar_arrive_expect_tx(bar, 0);
      return;
    }
    const int nbox = a.mode == QMM_SWIGLU ? 2 : 1;
    const int bh = RB / nbox;
    mbar_arrive_expect_tx(bar, (uint32_t)(nbox * bh * (SEGB + (p.sb_bulk ? 32 : 0))));
    // every TMA destination is 128-byte aligned: weight boxes at multiples of
    // bh*SEGB (>= 512 B), the up-rows' scale / bias boxes at p.SPH
    for (int k = 0; k < nbox; ++k) {
      const int m = a.mode == QMM_SWIGLU ? k : mi;
      tma_load_2d(dst + (size_t)k * bh * SEGB, &mp.w[m], seg0 * (SEGB / 4), row, bar);
      if (p.sb_bulk) {
        tma_load_2d(dst + (size_t)RB * SEGB + (size_t)k * p.SPH, &mp.s[m], seg0 * 8, row, bar);
        tma_load_2d(dst + (size_t)RB * SEGB + p.SP + (size_t)k * p.SPH, &mp.b[m], seg0 * 8, row, bar);
      }
    }
  };

  if (lane == 0 && nsw > 0) {
    for (int s = 0; s < p.nst; ++s) mbar_init(&bars[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int t = 0; t < p.nst; ++t) issue(t);
  }

  grid_wait();
  grid_launch_dependents();

  if (a.norm_w) {
    for (int m = warp; m < M; m += NW) {
      const float f = rms_factor_warp(a.x + (size_t)m * a.ldx, K, a.eps, lane);
      if (lane == 0) fnorm[m] = f;
    }
  }
  __syncthreads();

  // which rows of a batch this lane scales after the group-level reduction
  const int q2 = ((lane & 1) << 1) | ((lane >> 1) & 1);
  float xr[SPWMAX][MT][16];
  float xg[SPWMAX][MT];
  bool abort_ = false;

  for (int t = 0; t < ntask; ++t) {
    const int st = t % p.nst;
    const int it = t % niter;
    const int mt0 = (t / niter) * MT;
    const int mcnt = min(MT, M - mt0);
    const int batch = batch_of(t);
    const uint8_t* sb = stages + (size_t)st * p.stage;

    if (it == 0) {
#pragma unroll
      for (int si = 0; si < SPWMAX; ++si) {
        const int k0 = (seg0 + si) * 512 + 16 * lane;
        const bool qv = si < nsw && k0 < K;
        float nwv[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) nwv[j] = (a.norm_w && qv) ? bf2f(a.norm_w[k0 + j]) : 1.0f;
        // every row's loads first (one L2 round trip for the tile), then the
        // conversions
        uint4 raw[MT][2];
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          if (m < mcnt && qv) {
            const bf16_t* src = a.x + (size_t)(mt0 + m) * a.ldx + k0;
            raw[m][0] = *reinterpret_cast<const uint4*>(src);
            raw[m][1] = *reinterpret_cast<const uint4*>(src + 8);
          }
        }
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          float X = 0.0f;
          if (m < mcnt && qv) {
            const uint4 r0 = raw[m][0], r1 = raw[m][1];
            const uint32_t rw[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
            const float f = a.norm_w ? fnorm[mt0 + m] : 1.0f;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              float v = (j & 1) ? hi_bf(rw[j >> 1]) : lo_bf(rw[j >> 1]);
              if (a.norm_w) v = bf2f(f2bf(__fmul_rn(__fmul_rn(v, f), nwv[j])));
              X = __fadd_rn(X, v);
              xr[si][m][j] = __fmul_rn(v, quarter_prescale<BITS>(j));
            }
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) xr[si][m][j] = 0.0f;
          }
          X = __fadd_rn(X, __shfl_xor_sync(0xffffffffu, X, 1));
          X = __fadd_rn(X, __shfl_xor_sync(0xffffffffu, X, 2));
          xg[si][m] = X;
        }
      }
    }

    if (nsw > 0 && !abort_)
      if (!mbar_wait_bounded(&bars[st], (uint32_t)((t / p.nst) & 1), a.err, 0x51u)) abort_ = true;

    float tot[N5];
    int base = 0;
    bool owner = true;
#pragma unroll
    for (int si = 0; si < SPWMAX; ++si) {
      if (si < nsw) {
        const int k0 = (seg0 + si) * 512 + 16 * lane;
        const bool qv = k0 < K;
        const int lg = si * 8 + (lane >> 2);  // group index inside this warp's portion
        // quarter dot-products of the RB rows, a row pair per iteration (one
        // fma.rn.f32x2 per k); the loop is rolled to keep the kernel small, so
        // the sums are parked in shared memory (vbuf[item][lane])
#pragma unroll 1
        for (int i = 0; i < RB; i += 2) {
          float qa[16], qb[16];
          if (qv) {
            unpack_quarter_raw<BITS>(sb + (size_t)i * SEGB + lane * QB, qa);
            unpack_quarter_raw<BITS>(sb + (size_t)(i + 1) * SEGB + lane * QB, qb);
#pragma unroll
            for (int j = 0; j < 16; ++j) sub_magic2(qa[j], qb[j]);
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) { qa[j] = 0.0f; qb[j] = 0.0f; }
          }
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            float A = 0.0f, B = 0.0f;
            if (m < mcnt) {
#pragma unroll
              for (int j = 0; j < 16; ++j) fma2(A, B, qa[j], qb[j], xr[si][m][j]);
            }
            vbuf[(i * MT + m) * 32 + lane] = A;
            vbuf[((i + 1) * MT + m) * 32 + lane] = B;
          }
        }
        __syncwarp();
        float v[V];
#pragma unroll
        for (int k = 0; k < V; ++k) v[k] = vbuf[k * 32 + lane];
        base = 0;
        owner = true;
        rs_level<V>(v, 1, lane & 1, base);
        rs_level<N1>(v, 2, (lane >> 1) & 1, base);
        // e = fma(s, d, b * xs) for the RB/4 rows x MT columns this lane holds
#pragma unroll
        for (int c = 0; c < RB / 4; ++c) {
          const int i = q2 * (RB / 4) + c;
          float s = 0.0f, b = 0.0f;
          if (qv) {
            if (p.sb_bulk) {
              const size_t so = (a.mode == QMM_SWIGLU && i >= RB / 2) ? (size_t)p.SPH + (size_t)(i - RB / 2) * 16
                                                                      : (size_t)i * 16;
              s = bf2f(reinterpret_cast<const bf16_t*>(sb + (size_t)RB * SEGB + so)[lg]);
              b = bf2f(reinterpret_cast<const bf16_t*>(sb + (size_t)RB * SEGB + p.SP + so)[lg]);
            } else {
              int mi, row;
              if (batch < nbatch && qmm_item_row<RB>(a, batch * RB + i, mi, row)) {
                const QmmMat& mm = qmm_mat(a, mi);
                s = bf2f(mm.s[(size_t)row * G + (k0 >> 6)]);
                b = bf2f(mm.b[(size_t)row * G + (k0 >> 6)]);
              }
            }
          }
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            const int k = c * MT + m;
            v[k] = __fmaf_rn(s, v[k], __fmul_rn(b, xg[si][m]));
          }
        }
        rs_level<N2>(v, 4, (lane >> 2) & 1, base);
        if (N2 < 2) owner = owner && !((lane >> 2) & 1);
        rs_level<N3>(v, 8, (lane >> 3) & 1, base);
        if (N3 < 2) owner = owner && !((lane >> 3) & 1);
        rs_level<N4>(v, 16, (lane >> 4) & 1, base);
        if (N4 < 2) owner = owner && !((lane >> 4) & 1);
        if (gw == 0) {
#pragma unroll
          for (int k = 0; k < N5; ++k) tot[k] = si == 0 ? v[k] : __fadd_rn(tot[k], v[k]);
        } else if (owner) {
          float* dst = red + ((size_t)((t & 1) * NW + warp) * p.SPW + si) * V;
#pragma unroll
          for (int k = 0; k < N5; ++k) dst[base + k] = v[k];
        }
      }
    }
    __syncwarp();
    if (lane == 0 && !abort_) issue(t + p.nst);  // this warp is done with stage st

    if (csize > 1) cluster.sync();
    else if (p.W > 1 && inslot) named_barrier(1 + slot, p.W * 32);

    if (gw == 0 && inslot) {
      // continue the segment chain with the other warps' sums (in row order)
      if (owner) {
        for (int w2 = 1; w2 < nwr; ++w2) {
          const int n2 = max(0, min(p.SPW, nseg - w2 * p.SPW));
          const float* src;
          if (csize == 1) src = red + ((size_t)((t & 1) * NW + slot * p.W + w2) * p.SPW) * V;
          else src = cluster.map_shared_rank(red, w2 / NW) + ((size_t)((t & 1) * NW + w2 % NW) * p.SPW) * V;
          for (int s2 = 0; s2 < n2; ++s2)
#pragma unroll
            for (int k = 0; k < N5; ++k) tot[k] = __fadd_rn(tot[k], src[(size_t)s2 * V + base + k]);
        }
      }
      float tu[N5];
#pragma unroll
      for (int k = 0; k < N5; ++k) tu[k] = __shfl_xor_sync(0xffffffffu, tot[k], 1);
      if (owner) {
#pragma unroll
        for (int k = 0; k < N5; ++k) {
          const int idx = base + k, i = idx / MT, m = idx % MT;
          int mi, row;
          if (m >= mcnt || batch >= nbatch || !qmm_item_row<RB>(a, batch * RB + i, mi, row)) continue;
          const size_t orow = (size_t)(mt0 + m) * a.ldy;
          if (a.mode == QMM_SWIGLU) {
            if (mi == 0) a.y[orow + row] = swiglu_c(f2bf(tot[k]), f2bf(tu[k]));
          } else {
            const int col = (mi == 0 ? a.cstart[0] : (mi == 1 ? a.cstart[1] : a.cstart[2])) + row;
            bf16_t yv = f2bf(tot[k]);
            if (a.mode == QMM_RESID) yv = f2bf(__fadd_rn(bf2f(yv), bf2f(a.res[orow + col])));
            a.y[orow + col] = yv;
          }
        }
      }
    }
  }
  if (csize > 1) cluster.sync();
}

}  // namespace lmx
