// qmm_mma.cuh -- K1 tensor-core path for M >= 16 (batched verify, prefill):
// dequantize-to-shared-memory + tcgen05.mma with a TMEM accumulator.
//
// Swap-AB: D[n, m] = sum_k W[n, k] * X[m, k].  The weight tile is the MMA's A
// operand (128 weight rows = UMMA M), the activations are B (the token count
// padded to 16 = UMMA N), both K-major in the 128-byte-swizzled canonical
// layout (8-row x 128-byte atoms, 16-byte chunk index XOR row % 8).  Per CTA
// and 64-k chunk (one quantization group):
//   warp 0      TMA producer: packed weight tile [128 (or 2 x 64) rows x 64 k]
//               on `wfull`, activation tile [Mpad x 64 k] (TMA 128B swizzle)
//               on `xfull`.  Weight loads for the first stages are issued
//               before the programmatic-launch wait (weights are constant).
//   warps 2..5  one weight row per thread: bf16(fma(scale, q, bias)) written
//               into the swizzled A tile, then a proxy fence and `deq` arrive.
//   warp 1      allocates TMEM; one lane issues 4 x tcgen05.mma (K = 16) per
//               chunk and commits each stage back to `empty`, the whole
//               accumulation to `accf`.
// Split-K: a cluster of `ks` CTAs shares one output tile, each accumulating a
// contiguous range of chunks; the fp32 tiles meet in shared memory and each
// rank reduces a slice of the outputs over the ranks in rank order (DSMEM).
// Epilogue: tcgen05.ld (warps 2..5, one TMEM lane quarter each) -> fp32 tile
// [m][row] in shared memory -> coalesced PLAIN / RESID / SWIGLU stores.
// Every mbarrier wait is bounded and sets the device error word on timeout.
// No TMA multicast.  Numerics: bf16 dequantized weights, fp32 tensor-core
// accumulation in the hardware's order (compared with a tolerance).
#pragma once
#include "qmm.cuh"

namespace lmx {

static constexpr int kMmaRows = 128;  // weight rows per tile (UMMA M)
static constexpr int kMmaK = 64;      // k per pipeline stage (one group)
static constexpr int kMmaThreads = 192;
static constexpr int kMmaMaxStages = 8;
static constexpr int kMmaMaxSplit = 8;

struct MmaMaps {
  CUtensorMap w[3];  // uint32 [rows][K*bits/32], box {2*bits words, 128 (SWIGLU: 64) rows}
  CUtensorMap x;     // bf16 [M][ldx], box {64, Mpad}, 128-byte swizzle
};

struct MmaArgs {
  QmmMat mat[3];
  int nmat;
  int tstart[3];  // PLAIN/RESID: first tile of each matrix
  int cstart[3];  // PLAIN/RESID: first output column of each matrix
  int N;          // SWIGLU: rows per matrix
  int M, Mpad, K, mode;
  int stages, ks;
  bf16_t* y;
  int ldy;
  const bf16_t* res;
  unsigned* err;
};

// UMMA shared-memory descriptor, K-major, 128-byte swizzle: start address,
// leading byte offset 16 B (unused inside one swizzle atom), stride byte
// offset 1024 B (between 8-row groups), descriptor version 1, base offset 0
// (atoms are 1024-byte aligned), layout type 2 = SWIZZLE_128B.
LMX_DEV uint64_t umma_desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor, kind::f16: D fp32 (bit 4), A and B bf16 (bits 7,
// 10), both K-major, N >> 3 at bit 17, M >> 4 at bit 24 (M = 128).
LMX_DEV uint32_t umma_idesc_bf16(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kMmaRows >> 4) << 24);
}

LMX_DEV void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

LMX_DEV void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

LMX_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

LMX_DEV void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

LMX_DEV uint32_t bf2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Eight 4-bit codes of one word (k = 8c .. 8c+7) -> eight bf16 weights
// bf16(s*q + b) in k order.  Codes become exact bf16 values 128 + q by OR-ing
// the exponent of 128 (0x4300) over a nibble; subtracting 128 is exact; the
// bf16x2 fma rounds s*q + b once.  That equals bf16(fmaf(s, q, b)) whenever
// fmaf is exact, i.e. whenever s*q + b fits 24 significant bits (always the
// case unless |bias| and |scale| lie more than ~2^12 apart).
LMX_DEV uint4 deq8_b4(uint32_t w, uint32_t s2, uint32_t b2) {
  const uint32_t one = 0x3F803F80u, m128 = 0xC300C300u;
  uint32_t v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t x = ((w >> (4 * i)) & 0x000F000Fu) | 0x43004300u;  // (q_i, q_{i+4})
    v[i] = bf2_fma(s2, bf2_fma(x, one, m128), b2);
  }
  return make_uint4(__byte_perm(v[0], v[1], 0x5410), __byte_perm(v[2], v[3], 0x5410),
                    __byte_perm(v[0], v[1], 0x7632), __byte_perm(v[2], v[3], 0x7632));
}

// Eight 8-bit codes (two words) -> bf16(fmaf(s, q, b)) in k order: the code
// becomes an exact fp32 (2^23 + q) - 2^23, the fma runs in fp32.
LMX_DEV uint4 deq8_b8(uint32_t w0, uint32_t w1, float s, float b) {
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t w = i < 2 ? w0 : w1;
    const int e = (i & 1) * 2;
    const float q0 = __fsub_rn(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540 + e)), 8388608.0f);
    const float q1 = __fsub_rn(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7541 + e)), 8388608.0f);
    o[i] = (uint32_t)f2bf(__fmaf_rn(s, q0, b)) | ((uint32_t)f2bf(__fmaf_rn(s, q1, b)) << 16);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

LMX_DEV const QmmMat& mma_mat(const MmaArgs& a, int mi) {
  return mi == 0 ? a.mat[0] : (mi == 1 ? a.mat[1] : a.mat[2]);
}

// Tile -> (matrix, first row) for PLAIN/RESID.
LMX_DEV bool mma_tile(const MmaArgs& a, int tile, int& mi, int& row0) {
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    if (i < a.nmat) {
      const int nt = (a.mat[i].rows + kMmaRows - 1) / kMmaRows;
      if (tile >= a.tstart[i] && tile < a.tstart[i] + nt) {
        mi = i;
        row0 = (tile - a.tstart[i]) * kMmaRows;
        return true;
      }
    }
  }
  return false;
}

// Bounded wait by every lane of a warp; the result is made warp-uniform.
LMX_DEV bool warp_wait(uint64_t* bar, uint32_t parity, unsigned* err, unsigned code) {
  const bool ok = mbar_wait_bounded(bar, parity, err, code);
  return __all_sync(0xffffffffu, ok);
}

// Shared memory (base rounded up to 1024 bytes):
//   A[stages][16 KB]  B[stages][Mpad * 128 B]  P[stages][128 * 64 * BITS / 8 B]
//   barriers: wfull, xfull, deq, empty [stages] + accf;  tmem slot;  fail flag
//   red = fp32 [Mpad][128] over the A/B/P region once the MMAs are done
template <int BITS>
__global__ void __launch_bounds__(kMmaThreads, 1) qmm_mma_kernel(const __grid_constant__ MmaMaps mp, MmaArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  constexpr int ABYTES = kMmaRows * kMmaK * 2;
  constexpr int PBYTES = kMmaRows * kMmaK * BITS / 8;
  constexpr int PROW = kMmaK * BITS / 8;  // packed bytes of one row per chunk
  const int NS = a.stages;
  const int BBYTES = a.Mpad * kMmaK * 2;
  uint8_t* As = smem;
  uint8_t* Bs = As + NS * ABYTES;
  uint8_t* Ps = Bs + NS * BBYTES;
  uint64_t* wfull = reinterpret_cast<uint64_t*>(Ps + NS * PBYTES);
  uint64_t* xfull = wfull + NS;
  uint64_t* deq = xfull + NS;
  uint64_t* empty = deq + NS;
  uint64_t* accf = empty + NS;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accf + 1);
  int* s_fail = reinterpret_cast<int*>(tmem_slot + 1);
  float* red = reinterpret_cast<float*>(smem);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ks = a.ks;
  const int tile = blockIdx.x / ks, rank = blockIdx.x % ks;
  const int m0 = blockIdx.y * a.Mpad;
  const int nk = a.K / kMmaK;
  const int kc0 = (int)((long)rank * nk / ks), kc1 = (int)((long)(rank + 1) * nk / ks);
  const int nloc = kc1 - kc0;
  const int G = a.K / 64;
  const bool swiglu = a.mode == QMM_SWIGLU;
  int mi = 0, row0 = 0;
  if (swiglu) row0 = tile * (kMmaRows / 2);
  else mma_tile(a, tile, mi, row0);
  const uint32_t ncols = a.Mpad <= 32 ? 32u : (a.Mpad <= 64 ? 64u : (a.Mpad <= 128 ? 128u : 256u));

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&xfull[s], 1);
      mbar_init(&deq[s], 4);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accf, 1);
    *s_fail = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  grid_launch_dependents();
  bool ok = true;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const int wx_step = kMmaK * BITS / 32;
      auto load_w = [&](int j) {
        const int s = j % NS, kc = kc0 + j;
        mbar_arrive_expect_tx(&wfull[s], (uint32_t)PBYTES);
        if (swiglu) {
          tma_load_2d(Ps + s * PBYTES, &mp.w[0], kc * wx_step, row0, &wfull[s]);
          tma_load_2d(Ps + s * PBYTES + PBYTES / 2, &mp.w[1], kc * wx_step, row0, &wfull[s]);
        } else {
          tma_load_2d(Ps + s * PBYTES, &mp.w[mi], kc * wx_step, row0, &wfull[s]);
        }
      };
      auto load_x = [&](int j) {
        const int s = j % NS, kc = kc0 + j;
        mbar_arrive_expect_tx(&xfull[s], (uint32_t)BBYTES);
        tma_load_2d(Bs + s * BBYTES, &mp.x, kc * kMmaK, m0, &xfull[s]);
      };
      const int npre = nloc < NS ? nloc : NS;
      for (int j = 0; j < npre; ++j) load_w(j);
      grid_wait();
      for (int j = 0; j < npre; ++j) load_x(j);
      for (int j = npre; j < nloc; ++j) {
        if (!mbar_wait_bounded(&empty[j % NS], (uint32_t)(((j / NS) - 1) & 1), a.err, 0x61u)) {
          ok = false;
          break;
        }
        load_w(j);
        load_x(j);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(a.Mpad);
      for (int j = 0; j < nloc; ++j) {
        const int s = j % NS;
        const uint32_t par = (uint32_t)((j / NS) & 1);
        if (!mbar_wait_bounded(&deq[s], par, a.err, 0x62u) || !mbar_wait_bounded(&xfull[s], par, a.err, 0x63u)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t abase = smem_u32(As + s * ABYTES), bbase = smem_u32(Bs + s * BBYTES);
#pragma unroll
        for (int k16 = 0; k16 < kMmaK / 16; ++k16)
          umma_bf16(tmem, umma_desc_sw128(abase + 32 * k16), umma_desc_sw128(bbase + 32 * k16), idesc,
                    (j > 0 || k16 > 0) ? 1u : 0u);
        umma_commit(&empty[s]);
      }
      // arrives once every MMA issued above has completed
      umma_commit(accf);
    }
  } else {
    // ---------------- dequantizers: thread r owns weight row r of the tile ----------------
    const int r = threadIdx.x - 64;
    int wmi = mi, wrow = row0 + r;
    if (swiglu) {
      wmi = r < 64 ? 0 : 1;
      wrow = row0 + (r & 63);
    }
    const QmmMat& wm = mma_mat(a, wmi);
    const bool rvalid = wrow < (swiglu ? a.N : wm.rows);
    const bf16_t* srow = wm.s + (size_t)(rvalid ? wrow : 0) * G;
    const bf16_t* brow = wm.b + (size_t)(rvalid ? wrow : 0) * G;
    bf16_t sc = rvalid && nloc > 0 ? srow[kc0] : (bf16_t)0, bi = rvalid && nloc > 0 ? brow[kc0] : (bf16_t)0;
    uint8_t* arow0 = As + (r >> 3) * 1024 + (r & 7) * 128;
    for (int j = 0; j < nloc; ++j) {
      const int s = j % NS, kc = kc0 + j;
      const bf16_t sn = (rvalid && j + 1 < nloc) ? srow[kc + 1] : (bf16_t)0;
      const bf16_t bn = (rvalid && j + 1 < nloc) ? brow[kc + 1] : (bf16_t)0;
      if (j >= NS && !warp_wait(&empty[s], (uint32_t)(((j / NS) - 1) & 1), a.err, 0x64u)) {
        ok = false;
        break;
      }
      if (!warp_wait(&wfull[s], (uint32_t)((j / NS) & 1), a.err, 0x65u)) {
        ok = false;
        break;
      }
      const uint4* prow = reinterpret_cast<const uint4*>(Ps + s * PBYTES + r * PROW);
      uint8_t* arow = arow0 + s * ABYTES;
      if (BITS == 4) {
        const uint4 p0 = prow[0], p1 = prow[1];
        const uint32_t wv[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
        const uint32_t s2 = (uint32_t)sc | ((uint32_t)sc << 16), b2 = (uint32_t)bi | ((uint32_t)bi << 16);
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<uint4*>(arow + ((c ^ (r & 7)) << 4)) = deq8_b4(wv[c], s2, b2);
      } else {
        uint32_t wv[16];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint4 p = prow[i];
          wv[4 * i] = p.x;
          wv[4 * i + 1] = p.y;
          wv[4 * i + 2] = p.z;
          wv[4 * i + 3] = p.w;
        }
        const float sf = bf2f(sc), bf = bf2f(bi);
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<uint4*>(arow + ((c ^ (r & 7)) << 4)) = deq8_b8(wv[2 * c], wv[2 * c + 1], sf, bf);
      }
      // generic-proxy stores -> visible to the tensor core, then signal
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&deq[s]);
      sc = sn;
      bi = bn;
    }
    // accumulator -> red[m][row] (fp32), lane quarter q = warp % 4
    if (ok) ok = warp_wait(accf, 0u, a.err, 0x66u);
    if (ok) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int q = warp & 3, rr = 32 * q + lane;
      for (int c0 = 0; c0 < a.Mpad; c0 += 16) {
        float v[16];
        tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0, v);
#pragma unroll
        for (int i = 0; i < 16; ++i) red[(c0 + i) * kMmaRows + rr] = v[i];
      }
    }
  }
  if (!ok) atomicOr(s_fail, 1);

  // ---------------- split-K reduction and stores ----------------
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  cg::cluster_group cluster = cg::this_cluster();
  if (ks > 1) cluster.sync();
  else __syncthreads();
  grid_wait();
  if (*s_fail == 0) {
    const int rows_out = swiglu ? kMmaRows / 2 : kMmaRows;
    const int mcount = min(a.Mpad, a.M - m0);
    const int total = mcount * rows_out;
    const int per = (total + ks - 1) / ks;
    const int i0 = rank * per, i1 = min(total, i0 + per);
    for (int idx = i0 + (int)threadIdx.x; idx < i1; idx += kMmaThreads) {
      const int m = idx / rows_out, rr = idx % rows_out;
      float acc = 0.0f, acc2 = 0.0f;
      for (int k = 0; k < ks; ++k) {
        const float* rb = ks > 1 ? cluster.map_shared_rank(red, k) : red;
        acc = __fadd_rn(acc, rb[m * kMmaRows + rr]);
        if (swiglu) acc2 = __fadd_rn(acc2, rb[m * kMmaRows + 64 + rr]);
      }
      const size_t orow = (size_t)(m0 + m) * a.ldy;
      if (swiglu) {
        const int col = row0 + rr;
        if (col < a.N) a.y[orow + col] = swiglu_c(f2bf(acc), f2bf(acc2));
      } else {
        const int row = row0 + rr;
        if (row < mma_mat(a, mi).rows) {
          const size_t o = orow + a.cstart[mi] + row;
          bf16_t yv = f2bf(acc);
          if (a.mode == QMM_RESID) yv = f2bf(__fadd_rn(bf2f(yv), bf2f(a.res[o])));
          a.y[o] = yv;
        }
      }
    }
  }
  if (ks > 1) cluster.sync();  // peers may still read this CTA's red tile
  // the accumulator must be idle before TMEM is released
  if (warp == 1) {
    if (lane == 0 && *s_fail) mbar_wait_bounded(accf, 0u, a.err, 0x67u);
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols) : "memory");
  }
}

}  // namespace lmx
