// qmm_mma.cuh -- K1 tensor-core path for M >= 16 (batched verify, prefill):
// dequantize into tensor memory + tcgen05.mma with a TMEM accumulator.
//
// Swap-AB: D[n, m] = sum_k W[n, k] * X[m, k].  The dequantized weight tile is
// the MMA's A operand, held in TMEM (128 weight rows = 128 lanes, two bf16 k
// per 32-bit column); the activations are B, TMA-loaded into shared memory in
// the 128-byte-swizzled K-major layout (8-row x 128-byte atoms); the fp32
// accumulator [128 rows x Mpad tokens] sits in TMEM.  Per 64-k chunk (one
// quantization group):
//   warp 0      W producer: packed weight tile [128 (or 2 x 64) rows x 64 k]
//               into a deep ring of `NP` stages (`pfull` / `pfree`); weights
//               are constant, so it runs ahead of the programmatic-launch
//               wait, and the first NP stages are issued right after the
//               barrier initialisation, before the TMEM allocation and the
//               CTA-wide set-up barrier.
//   warp 10     X producer: activation tiles [Mpad x 64 k] of a step (two
//               chunks) into the `na`-stage ring shared with the A stages
//               (`xfull` / `mdone`).
//   warps 2..9  dequantizers, two threads per weight row (k halves of 32):
//               packed words -> bf16(fma(scale, q, bias)) -> tcgen05.st into
//               the A stage (`afull`); they free a packed stage once its
//               last words are consumed.
//   warp 1      allocates TMEM; one lane issues 4 x tcgen05.mma (K = 16, A
//               from TMEM, B from shared memory) per chunk and commits each
//               step's stage to `mdone`, the whole accumulation to `accf`.
// A and X stages hold one step = kMmaStep chunks, so the per-stage
// synchronisation (waits, arrives, TMEM store fences) is paid once per 128 k.
// Split-K: a cluster of `ks` CTAs shares one output tile, each accumulating a
// contiguous range of chunks; the fp32 tiles meet in shared memory and each
// rank reduces a slice of the outputs over the ranks in rank order (DSMEM).
// Epilogue: tcgen05.ld (lane quarter = warp % 4) -> fp32 tile [m][row] in
// shared memory -> coalesced PLAIN / RESID / SWIGLU stores.
// Every mbarrier wait is bounded and sets the device error word on timeout.
// Each TMA load fills only its own CTA's shared memory.  Numerics: bf16
// dequantized weights, fp32 tensor-core accumulation in the hardware's order
// (compared with a tolerance).
#pragma once
#include "qmm.cuh"

namespace lmx {

static constexpr int kMmaRows = 128;  // weight rows per tile (UMMA M)
static constexpr int kMmaK = 64;      // k per pipeline stage (one group)
static constexpr int kMmaWarps = 11;  // W producer, MMA, 8 dequantizers, X producer
static constexpr int kMmaThreads = 32 * kMmaWarps;
static constexpr int kMmaDeqWarps = 8;
static constexpr int kMmaStep = 2;        // chunks per A (TMEM) / X (shared) stage
static constexpr int kMmaMaxAStages = 4;
static constexpr int kMmaMaxPStages = 16;
static constexpr int kMmaMaxSplit = 8;

struct MmaMaps {
  CUtensorMap w[3];  // uint32 [rows][K*bits/32], box {32 words, 128 (SWIGLU: 64) rows}, 128B swizzle
  CUtensorMap x;     // bf16 [M][ldx], box {64, Mpad}, 128-byte swizzle
};

struct MmaArgs {
  QmmMat mat[3];
  int nmat;
  int tstart[3];  // PLAIN/RESID: first tile of each matrix
  int cstart[3];  // PLAIN/RESID: first output column of each matrix
  int N;          // SWIGLU: rows per matrix
  int M, Mpad, K, mode;
  int np, na, ks;      // packed-weight stages, A/X stages, split-K factor (cluster size)
  int acc_cols, tmem_cols;
  int sb_vec;          // scales / biases readable as 16-byte vectors (K % 512 == 0, aligned)
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

// D[tmem] (+)= A[tmem] * B[smem]^T, 128 x N x 16.
LMX_DEV void umma_ts_bf16(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
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

// 32 lanes x 16 columns of 32 bits: lane i of the warp's quarter gets v[0..15].
LMX_DEV void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

LMX_DEV uint32_t bf2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Eight 4-bit codes of one word (k = 8c .. 8c+7) -> eight bf16 weights
// bf16(s*q + b) in k order, two per word of `o`.  Codes become exact bf16
// values 128 + q by OR-ing the exponent of 128 (0x4300) over a nibble;
// subtracting 128 is exact; the bf16x2 fma rounds s*q + b once.  That equals
// bf16(fmaf(s, q, b)) whenever fmaf is exact, i.e. whenever s*q + b fits 24
// significant bits (always, unless |bias| and |scale| lie more than ~2^12
// apart).
LMX_DEV void deq8_b4(uint32_t w, uint32_t s2, uint32_t b2, uint32_t* o) {
  const uint32_t one = 0x3F803F80u, m128 = 0xC300C300u;
  uint32_t v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t x = ((w >> (4 * i)) & 0x000F000Fu) | 0x43004300u;  // (q_i, q_{i+4})
    v[i] = bf2_fma(s2, bf2_fma(x, one, m128), b2);
  }
  o[0] = __byte_perm(v[0], v[1], 0x5410);
  o[1] = __byte_perm(v[2], v[3], 0x5410);
  o[2] = __byte_perm(v[0], v[1], 0x7632);
  o[3] = __byte_perm(v[2], v[3], 0x7632);
}

// Eight 8-bit codes (two words) -> bf16(fmaf(s, q, b)) in k order: the code
// becomes an exact fp32 (2^23 + q) - 2^23, the fma runs in fp32.
LMX_DEV void deq8_b8(uint32_t w0, uint32_t w1, float s, float b, uint32_t* o) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t w = i < 2 ? w0 : w1;
    const int e = (i & 1) * 2;
    const float q0 = __fsub_rn(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540 + e)), 8388608.0f);
    const float q1 = __fsub_rn(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7541 + e)), 8388608.0f);
    o[i] = (uint32_t)f2bf(__fmaf_rn(s, q0, b)) | ((uint32_t)f2bf(__fmaf_rn(s, q1, b)) << 16);
  }
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

LMX_DEV uint32_t u4_word(const uint4& v, int i) {
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

// Shared memory (base rounded up to 1024 bytes):
//   X[na][2 x Mpad * 128 B]  P[np][128 rows * 128 B] (16/BITS chunks per
//   stage, 16-byte units swizzled by row % 8, as TMA's 128-byte swizzle
//   writes them)
//   barriers: pfull, pfree [np]; xfull, afull, mdone [na]; accf;  tmem slot;  fail flag
//   red = fp32 [Mpad][128] over the X/P region once the MMAs are done
// TMEM: accumulator columns [0, acc_cols), A stage s at acc_cols + 64 s
// (chunk u of the step at + 32 u, k half h of a chunk at + 16 h).
template <int BITS>
__global__ void __launch_bounds__(kMmaThreads, 2) qmm_mma_kernel(const __grid_constant__ MmaMaps mp, MmaArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  constexpr int PBYTES = kMmaRows * 128;
  constexpr int CH = 16 / BITS;  // chunks per packed stage (128 bytes of a row)
  const int NP = a.np, NA = a.na;
  const int XBYTES = a.Mpad * kMmaK * 2;  // one chunk's activation tile
  const int XSTAGE = kMmaStep * XBYTES;
  uint8_t* Xs = smem;
  uint8_t* Ps = Xs + NA * XSTAGE;
  uint64_t* pfull = reinterpret_cast<uint64_t*>(Ps + NP * PBYTES);
  uint64_t* pfree = pfull + NP;
  uint64_t* xfull = pfree + NP;
  uint64_t* afull = xfull + NA;
  uint64_t* mdone = afull + NA;
  uint64_t* accf = mdone + NA;
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
  const int nsteps = (nloc + kMmaStep - 1) / kMmaStep;
  const int G = a.K / 64;
  const bool swiglu = a.mode == QMM_SWIGLU;
  int mi = 0, row0 = 0;
  if (swiglu) row0 = tile * (kMmaRows / 2);
  else mma_tile(a, tile, mi, row0);

  // packed stage t of this CTA's k range into ring slot st (weights do not
  // depend on earlier kernels)
  const int nst = (nloc + CH - 1) / CH;
  auto issue_w = [&](int t, int st) {
    const int wx = (kc0 + t * CH) * 2 * BITS;  // word column of the stage's first chunk
    mbar_arrive_expect_tx(&pfull[st], (uint32_t)PBYTES);
    if (swiglu) {
      tma_load_2d(Ps + st * PBYTES, &mp.w[0], wx, row0, &pfull[st]);
      tma_load_2d(Ps + st * PBYTES + PBYTES / 2, &mp.w[1], wx, row0, &pfull[st]);
    } else {
      tma_load_2d(Ps + st * PBYTES, &mp.w[mi], wx, row0, &pfull[st]);
    }
  };
  const int npre = min(NP, nst);  // stages issued before the CTA-wide set-up barrier
  if (threadIdx.x == 0) {
    for (int s = 0; s < NP; ++s) {
      mbar_init(&pfull[s], 1);
      mbar_init(&pfree[s], kMmaDeqWarps);
    }
    for (int s = 0; s < NA; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&afull[s], kMmaDeqWarps);
      mbar_init(&mdone[s], 1);
    }
    mbar_init(accf, 1);
    *s_fail = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    // the first weight stages start streaming before the TMEM allocation
    // and the set-up barrier (thread 0 is the W producer's lane)
    for (int t = 0; t < npre; ++t) issue_w(t, t);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"((uint32_t)a.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_a = tmem + (uint32_t)a.acc_cols;
  grid_launch_dependents();
  bool ok = true;

  if (warp == 0) {
    // ---------------- W producer (no dependency on earlier kernels) ----------------
    if (lane == 0) {
      int s = npre == NP ? 0 : npre;
      uint32_t ph = 0;  // parity of the pfree phase that frees stage s
      for (int t = npre; t < nst; ++t) {
        if (t >= NP && !mbar_wait_bounded(&pfree[s], ph, a.err, 0x61u)) {
          ok = false;
          break;
        }
        issue_w(t, s);
        if (++s == NP) {
          s = 0;
          if (t >= NP) ph ^= 1u;
        }
      }
    }
  } else if (warp == kMmaWarps - 1) {
    // ---------------- X producer (after the programmatic-launch wait) ----------------
    if (lane == 0) {
      grid_wait();
      int s = 0;
      uint32_t ph = 0;  // parity of the mdone phase that frees stage s
      for (int t = 0; t < nsteps; ++t) {
        const int kc = kc0 + kMmaStep * t, cnt = min(kMmaStep, nloc - kMmaStep * t);
        if (t >= NA && !mbar_wait_bounded(&mdone[s], ph, a.err, 0x62u)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&xfull[s], (uint32_t)(cnt * XBYTES));
        for (int u = 0; u < cnt; ++u)
          tma_load_2d(Xs + s * XSTAGE + u * XBYTES, &mp.x, (kc + u) * kMmaK, m0, &xfull[s]);
        if (++s == NA) {
          s = 0;
          if (t >= NA) ph ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(a.Mpad);
      int s = 0;
      uint32_t ph = 0;  // parity of the afull / xfull phase of stage s
      for (int t = 0; t < nsteps; ++t) {
        if (!mbar_wait_bounded(&afull[s], ph, a.err, 0x63u) || !mbar_wait_bounded(&xfull[s], ph, a.err, 0x64u)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const int cnt = min(kMmaStep, nloc - kMmaStep * t);
        const uint32_t bbase = smem_u32(Xs + s * XSTAGE);
        for (int u = 0; u < cnt; ++u) {
#pragma unroll
          for (int k16 = 0; k16 < kMmaK / 16; ++k16)
            umma_ts_bf16(tmem, tmem_a + (uint32_t)(64 * s + 32 * u + 8 * k16),
                         umma_desc_sw128(bbase + u * XBYTES + 32 * k16), idesc, (t > 0 || u > 0 || k16 > 0) ? 1u : 0u);
        }
        umma_commit(&mdone[s]);
        if (++s == NA) {
          s = 0;
          ph ^= 1u;
        }
      }
      // arrives once every MMA issued above has completed
      umma_commit(accf);
    }
  } else {
    // ---------------- dequantizers: row rr of the tile, k half h ----------------
    const int q = warp & 3, h = (warp - 2) >> 2;
    const int rr = 32 * q + lane;
    int wmi = mi, wrow = row0 + rr;
    if (swiglu) {
      wmi = rr < 64 ? 0 : 1;
      wrow = row0 + (rr & 63);
    }
    const QmmMat& wm = mma_mat(a, wmi);
    const bool rvalid = wrow < (swiglu ? a.N : wm.rows);
    const bf16_t* srow = wm.s + (size_t)(rvalid ? wrow : 0) * G;
    const bf16_t* brow = wm.b + (size_t)(rvalid ? wrow : 0) * G;
    const bool vec = a.sb_vec != 0;
    // scales / biases: 8-group blocks as 16-byte vectors (current and next)
    uint4 cs = make_uint4(0, 0, 0, 0), cb = cs, ns = cs, nb = cs;
    if (vec && nloc > 0) {
      const int blk = kc0 >> 3;
      cs = *reinterpret_cast<const uint4*>(srow + 8 * blk);
      cb = *reinterpret_cast<const uint4*>(brow + 8 * blk);
      if (8 * (blk + 1) < G) {
        ns = *reinterpret_cast<const uint4*>(srow + 8 * (blk + 1));
        nb = *reinterpret_cast<const uint4*>(brow + 8 * (blk + 1));
      }
    }
    const uint32_t tlane = (uint32_t)(32 * q) << 16;
    const uint32_t prow0 = smem_u32(Ps) + (uint32_t)rr * 128u;
    const int sw = rr & 7;
    int sp = 0;
    uint32_t pph = 0;  // parity of the pfull phase of stage sp
    int s = 0;
    uint32_t aph = 0;  // parity of the mdone phase that frees A stage s
    if constexpr (BITS == 4) {
      // 4-bit: a packed stage holds four chunks, i.e. exactly two steps, so
      // a step takes at most one wait per ring, two 16-byte shared loads
      // (16-byte units 2c+h of the row for its chunks c) and the two groups'
      // scale / bias words, which are loaded a step ahead
      const uint32_t pbase = smem_u32(Ps) + (uint32_t)rr * 128u;
      const uint32_t offs[4] = {(uint32_t)((h ^ sw) << 4), (uint32_t)(((2 + h) ^ sw) << 4),
                                (uint32_t)(((4 + h) ^ sw) << 4), (uint32_t)(((6 + h) ^ sw) << 4)};
      const uint32_t tbase = tlane + tmem_a + (uint32_t)(16 * h);
      const unsigned short* s16 = reinterpret_cast<const unsigned short*>(srow);
      const unsigned short* b16 = reinterpret_cast<const unsigned short*>(brow);
      uint32_t ns0 = 0, ns1 = 0, nb0 = 0, nb1 = 0;
      auto load_sb = [&](int t) {
        const int kc = kc0 + 2 * t;
        const bool two = 2 * t + 1 < nloc;
        ns0 = rvalid ? (uint32_t)__ldg(s16 + kc) : 0u;
        nb0 = rvalid ? (uint32_t)__ldg(b16 + kc) : 0u;
        ns1 = rvalid && two ? (uint32_t)__ldg(s16 + kc + 1) : 0u;
        nb1 = rvalid && two ? (uint32_t)__ldg(b16 + kc + 1) : 0u;
      };
      if (nsteps > 0) load_sb(0);
      for (int t = 0; t < nsteps; ++t) {
        const uint32_t s20 = ns0 | (ns0 << 16), b20 = nb0 | (nb0 << 16);
        const uint32_t s21 = ns1 | (ns1 << 16), b21 = nb1 | (nb1 << 16);
        if (t + 1 < nsteps) load_sb(t + 1);
        const bool two = 2 * t + 1 < nloc;
        if (t >= NA && !warp_wait(&mdone[s], aph, a.err, 0x66u)) {
          ok = false;
          break;
        }
        const int half = t & 1;  // which two chunks of the packed stage
        if (half == 0 && !warp_wait(&pfull[sp], pph, a.err, 0x65u)) {
          ok = false;
          break;
        }
        const uint32_t pst = pbase + (uint32_t)(sp * PBYTES);
        const uint32_t off0 = half ? offs[2] : offs[0], off1 = half ? offs[3] : offs[1];
        uint32_t w0[4], w1[4] = {0u, 0u, 0u, 0u};
        asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(w0[0]), "=r"(w0[1]), "=r"(w0[2]), "=r"(w0[3])
                     : "r"(pst + off0));
        if (two)
          asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
                       : "=r"(w1[0]), "=r"(w1[1]), "=r"(w1[2]), "=r"(w1[3])
                       : "r"(pst + off1));
        const uint32_t ta = tbase + (uint32_t)(64 * s);
        {
          uint32_t o[16];
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) deq8_b4(w0[cc], s20, b20, &o[4 * cc]);
          tmem_st16(ta, o);
        }
        if (two) {
          uint32_t o[16];
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) deq8_b4(w1[cc], s21, b21, &o[4 * cc]);
          tmem_st16(ta + 32u, o);
        }
        // a stage whose last words are consumed (used above) may be refilled
        if (half == 1 || t == nsteps - 1) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&pfree[sp]);
          if (++sp == NP) {
            sp = 0;
            pph ^= 1u;
          }
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&afull[s]);
        if (++s == NA) {
          s = 0;
          if (t >= NA) aph ^= 1u;
        }
      }
    } else {
    // one step (kMmaStep chunks) at a time: every wait and shared-memory load
    // of the step first, then dequantization and TMEM stores chunk by chunk
    // (the loads of the second chunk overlap the first one's work)
    for (int t = 0; t < nsteps && ok; ++t) {
      const int cnt = min(kMmaStep, nloc - kMmaStep * t);
      if (t >= NA && !warp_wait(&mdone[s], aph, a.err, 0x66u)) {
        ok = false;
        break;
      }
      uint32_t wv[kMmaStep][BITS];  // this thread's 32 k of row rr per chunk (4 or 8 words)
      bf16_t scu[kMmaStep], biu[kMmaStep];
      int spu[kMmaStep];
      bool endu[kMmaStep];
#pragma unroll
      for (int u = 0; u < kMmaStep; ++u) {
        endu[u] = false;
        spu[u] = sp;
        if (u >= cnt || !ok) continue;
        const int j = kMmaStep * t + u, kc = kc0 + j, c = j % CH;
        if (vec) {
          if (j > 0 && (kc & 7) == 0) {
            cs = ns;
            cb = nb;
            if (8 * ((kc >> 3) + 1) < G) {
              ns = *reinterpret_cast<const uint4*>(srow + 8 * ((kc >> 3) + 1));
              nb = *reinterpret_cast<const uint4*>(brow + 8 * ((kc >> 3) + 1));
            }
          }
          const int g = kc & 7, sh = 16 * (g & 1);
          scu[u] = (bf16_t)(u4_word(cs, g >> 1) >> sh);
          biu[u] = (bf16_t)(u4_word(cb, g >> 1) >> sh);
        } else {
          scu[u] = srow[kc];
          biu[u] = brow[kc];
        }
        if (c == 0 && !warp_wait(&pfull[sp], pph, a.err, 0x65u)) {
          ok = false;
          continue;
        }
        // 16-byte units 2c+h (4-bit) or 4c+2h, 4c+2h+1 (8-bit) of the packed row
        const uint32_t pst = prow0 + (uint32_t)(sp * PBYTES);
#pragma unroll
        for (int i = 0; i < BITS / 4; ++i) {
          const int un = (BITS == 4) ? (2 * c + h) : (4 * c + 2 * h + i);
          asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
                       : "=r"(wv[u][4 * i]), "=r"(wv[u][4 * i + 1]), "=r"(wv[u][4 * i + 2]), "=r"(wv[u][4 * i + 3])
                       : "r"(pst + (uint32_t)((un ^ sw) << 4)));
        }
        endu[u] = c == CH - 1 || j == nloc - 1;
        if (endu[u] && ++sp == NP) {
          sp = 0;
          pph ^= 1u;
        }
      }
      if (!ok) break;
#pragma unroll
      for (int u = 0; u < kMmaStep; ++u) {
        if (u >= cnt) continue;
        uint32_t o[16];
        if (BITS == 4) {
          const bf16_t sc = rvalid ? scu[u] : (bf16_t)0, bi = rvalid ? biu[u] : (bf16_t)0;
          const uint32_t s2 = (uint32_t)sc | ((uint32_t)sc << 16), b2 = (uint32_t)bi | ((uint32_t)bi << 16);
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) deq8_b4(wv[u][cc], s2, b2, &o[4 * cc]);
        } else {
          const float sf = rvalid ? bf2f(scu[u]) : 0.0f, bf = rvalid ? bf2f(biu[u]) : 0.0f;
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) deq8_b8(wv[u][2 * cc], wv[u][2 * cc + 1], sf, bf, &o[4 * cc]);
        }
        tmem_st16(tlane + tmem_a + (uint32_t)(64 * s + 32 * u + 16 * h), o);
      }
      // a packed stage whose last chunk has been consumed (its loads are
      // complete: their values are used above) may be refilled; an arrive
      // right after the loads could let the TMA overwrite words in flight
      __syncwarp();
#pragma unroll
      for (int u = 0; u < kMmaStep; ++u)
        if (u < cnt && endu[u] && lane == 0) mbar_arrive(&pfree[spu[u]]);
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[s]);
      if (++s == NA) {
        s = 0;
        if (t >= NA) aph ^= 1u;
      }
    }
    }
    // accumulator -> red[m][row] (fp32); the two warps of a lane quarter
    // take alternate 16-column blocks
    if (ok) ok = warp_wait(accf, 0u, a.err, 0x67u);
    if (ok) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      for (int c0 = 16 * h; c0 < a.Mpad; c0 += 32) {
        float v[16];
        tmem_ld16(tlane + tmem + (uint32_t)c0, v);
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
    // four consecutive rows of one token per thread: the ranks' float4s are
    // requested four at a time before any is added (the remote reads
    // overlap), and the partial tiles are summed in rank order
    const int rows_out = swiglu ? kMmaRows / 2 : kMmaRows;
    const int mcount = min(a.Mpad, a.M - m0);
    const int total = mcount * rows_out / 4;
    const int per = (total + ks - 1) / ks;
    const int i0 = rank * per, i1 = min(total, i0 + per);
    for (int idx = i0 + (int)threadIdx.x; idx < i1; idx += kMmaThreads) {
      const int m = (4 * idx) / rows_out, r2 = (4 * idx) % rows_out;
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f}, acc2[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int k0 = 0; k0 < kMmaMaxSplit; k0 += 4) {
        float4 v[4], v2[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (k0 + k < ks) {
            const float* rb = ks > 1 ? cluster.map_shared_rank(red, k0 + k) : red;
            v[k] = *reinterpret_cast<const float4*>(rb + m * kMmaRows + r2);
            if (swiglu) v2[k] = *reinterpret_cast<const float4*>(rb + m * kMmaRows + 64 + r2);
          }
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (k0 + k < ks) {
            acc[0] = __fadd_rn(acc[0], v[k].x), acc[1] = __fadd_rn(acc[1], v[k].y);
            acc[2] = __fadd_rn(acc[2], v[k].z), acc[3] = __fadd_rn(acc[3], v[k].w);
            if (swiglu) {
              acc2[0] = __fadd_rn(acc2[0], v2[k].x), acc2[1] = __fadd_rn(acc2[1], v2[k].y);
              acc2[2] = __fadd_rn(acc2[2], v2[k].z), acc2[3] = __fadd_rn(acc2[3], v2[k].w);
            }
          }
        }
      }
      const size_t orow = (size_t)(m0 + m) * a.ldy;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (swiglu) {
          const int col = row0 + r2 + e;
          if (col < a.N) a.y[orow + col] = swiglu_c(f2bf(acc[e]), f2bf(acc2[e]));
        } else {
          const int row = row0 + r2 + e;
          if (row < mma_mat(a, mi).rows) {
            const size_t o = orow + a.cstart[mi] + row;
            bf16_t yv = f2bf(acc[e]);
            if (a.mode == QMM_RESID) yv = f2bf(__fadd_rn(bf2f(yv), bf2f(a.res[o])));
            a.y[o] = yv;
          }
        }
      }
    }
  }
  if (ks > 1) cluster.sync();  // peers may still read this CTA's red tile
  // the accumulator must be idle before TMEM is released
  if (warp == 1) {
    if (lane == 0 && *s_fail) mbar_wait_bounded(accf, 0u, a.err, 0x68u);
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)a.tmem_cols)
                 : "memory");
  }
}

}  // namespace lmx
