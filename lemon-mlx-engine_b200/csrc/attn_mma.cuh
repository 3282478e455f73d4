// attn_mma.cuh -- K2 on the tensor cores: verify-block SDPA when a KV head
// serves many query rows (G*T >= the tensor-core threshold; e.g. G=8 q heads
// per KV head x T=5 verify tokens = 40 rows).  At long contexts the
// CUDA-core kernel (attn.cuh) spends 2*rows*128 fp32 FMAs per cached key and
// becomes compute-bound; here the two products run on mma.sync (bf16 in,
// fp32 accumulate).
//
// One CTA of 16 warps per (sequence, KV head, row tile of <= 64 rows,
// split): the split covers cpc = ceil(chunks / nsplit) of the 128-key chunks
// the tile reaches at the current cache length, with an online softmax:
//   stage K, V chunk -> bf16 smem (dequantized on the way, rows past the
//   visible range zero-filled).  Affine (4/8-bit) caches: the packed rows of
//   the next chunk stream into a two-stage raw ring by cp.async.bulk (one
//   copy for K, one for V; bounded mbarrier waits) and its scales / biases
//   into registers while the current chunk is computed; the rows are then
//   dequantized shared -> shared.  bf16 caches load directly.
//   S = (Q K^T) * scale (fp32; warp w: keys [8w, 8w+8));
//   per row, in base 2 (s' = s * scale * log2 e, hardware ex2): running max
//   m, rescale alpha = 2^(m_old - m_new), p = 2^(s' - m_new) (masked keys
//   0), l = l*alpha + sum(p);
//   O = O*alpha + P V (warp w: head dims [8w, 8w+8)), with p carried as two
//   bf16 terms p_hi = bf16(p), p_lo = bf16(p - p_hi) (two products), so P
//   keeps ~16 significant bits instead of bf16's 8.
// The split's (m, l, O) go to the scratch partials; the last CTA of the
// (sequence, KV head, tile) combines them: out = sum_s 2^(m_s-M) O_s /
// sum_s 2^(m_s-M) l_s.  All rows of a KV head share one pass over its cache.
//
// Numerics differ from the canonical order: products accumulate in the
// tensor core's order, exponentials come from the hardware ex2 (a few ulp)
// and p is represented to ~2^-17; results are compared with a tolerance
// (the canonical kernel stays the exact path).
#pragma once
#include "attn.cuh"
#include "qmm.cuh"

namespace lmx {

static constexpr int kAttnMmaRows = 64;         // rows per tile (partials layout)
static constexpr int kAttnChunk = 128;          // keys per chunk
static constexpr int kAttnKP = kHeadDim + 8;    // bf16 pitch of Q / K / V rows
static constexpr int kAttnSP = kAttnChunk + 4;  // fp32 pitch of S rows (P hi | lo bf16 in place)
static constexpr int kAttnThreads = 512;
static constexpr int kAttnWarps = kAttnThreads / 32;
static constexpr int kAttnItems = kAttnChunk * 8 / kAttnThreads;  // (key, 16 dims) items per thread

LMX_DEV void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
LMX_DEV void ldsm_x4(uint32_t (&r)[4], const void* p) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(p);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(s));
}
LMX_DEV void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(p);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(s));
}

// bf16x2 of (lo, hi), each rounded to nearest even (one cvt for the pair)
LMX_DEV uint32_t bf2_pack(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// 2^x (the hardware approximation; the softmax below works in base 2)
LMX_DEV float ex2(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// raw ring: per stage the packed K rows then the packed V rows of one chunk
template <int BITS>
__host__ __device__ constexpr size_t sdpa_raw_stage() {
  return BITS == 16 ? 0 : (size_t)2 * kAttnChunk * kHeadDim * BITS / 8;
}
template <int MT, int BITS>
constexpr size_t sdpa_mma_smem() {
  return (size_t)16 * MT * kAttnKP * 2 + (size_t)2 * kAttnChunk * kAttnKP * 2 + (size_t)16 * MT * kAttnSP * 4 +
         (size_t)3 * 16 * MT * 4 + 2 * sdpa_raw_stage<BITS>() + 64;
}

// Scales / biases of this thread's items of one chunk (rows >= jn: 0), as
// loaded: sr[4i .. 4i+3] = K scale, K bias, V scale, V bias of item i.  Nothing
// here uses the values, so the loads stay in flight until sdpa_pack_scales
// (a chunk later in the loop).
LMX_DEV void sdpa_load_scales(const KvDesc& kv, size_t row0, int jn, int tid, uint32_t (&sr)[4 * kAttnItems]) {
#pragma unroll
  for (int i = 0; i < kAttnItems; ++i) {
    const int e = tid + kAttnThreads * i, j = e >> 3, g = (e & 7) >> 2;
    sr[4 * i] = sr[4 * i + 1] = sr[4 * i + 2] = sr[4 * i + 3] = 0u;
    if (j < jn) {
      const size_t r = (row0 + j) * 2 + g;
      sr[4 * i] = __ldg(kv.ks + r);
      sr[4 * i + 1] = __ldg(kv.kb + r);
      sr[4 * i + 2] = __ldg(kv.vs + r);
      sr[4 * i + 3] = __ldg(kv.vb + r);
    }
  }
}

// -> bf16 pairs: sb[i] = (scale, bias) of K, sb[items + i] of V.
LMX_DEV void sdpa_pack_scales(const uint32_t (&sr)[4 * kAttnItems], uint32_t (&sb)[2 * kAttnItems]) {
#pragma unroll
  for (int i = 0; i < kAttnItems; ++i) {
    sb[i] = sr[4 * i] | (sr[4 * i + 1] << 16);
    sb[kAttnItems + i] = sr[4 * i + 2] | (sr[4 * i + 3] << 16);
  }
}

// Dequantize one chunk from the raw stage into the bf16 tiles: item = (key
// j, 16 head dims); bf16(fma(scale, q, bias)) as kv_chunk8.  Rows >= jn zero.
template <int BITS>
LMX_DEV void sdpa_stage_raw(int jn, const uint8_t* raw, const uint32_t (&sb)[2 * kAttnItems], bf16_t* Ks,
                            bf16_t* Vs, int tid) {
  constexpr int RB = kHeadDim * BITS / 8;  // packed bytes per row
#pragma unroll
  for (int i = 0; i < kAttnItems; ++i) {
    const int e = tid + kAttnThreads * i, j = e >> 3, c16 = e & 7;
#pragma unroll
    for (int h = 0; h < 2; ++h) {  // 0: K, 1: V
      const uint8_t* src = raw + (size_t)h * kAttnChunk * RB + (size_t)j * RB + c16 * (16 * BITS / 8);
      // code -> float exactly: the code as the low mantissa bits of
      // 2^23 (0x4B000000), minus 2^23
      float q[16];
      if (BITS == 8) {
        const uint4 w = *reinterpret_cast<const uint4*>(src);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int k = 0; k < 16; ++k)
          q[k] = __fsub_rn(__uint_as_float(__byte_perm(ws[k >> 2], 0x4B000000u, (k & 3) | 0x7650)), 8388608.0f);
      } else {
        const uint2 w = *reinterpret_cast<const uint2*>(src);
        const uint32_t ws[2] = {w.x, w.y};
#pragma unroll
        for (int k = 0; k < 16; ++k)
          q[k] = __fsub_rn(__uint_as_float(((ws[k >> 3] >> (4 * (k & 7))) & 0xFu) | 0x4B000000u), 8388608.0f);
      }
      const uint32_t p = sb[h * kAttnItems + i];
      const float sc = lo_bf(p), bi = hi_bf(p);
      uint32_t o[8];
#pragma unroll
      for (int k = 0; k < 8; ++k)
        o[k] = j < jn ? bf2_pack(__fmaf_rn(sc, q[2 * k], bi), __fmaf_rn(sc, q[2 * k + 1], bi)) : 0u;
      bf16_t* dst = (h ? Vs : Ks) + j * kAttnKP + c16 * 16;
      *reinterpret_cast<uint4*>(dst) = make_uint4(o[0], o[1], o[2], o[3]);
      *reinterpret_cast<uint4*>(dst + 8) = make_uint4(o[4], o[5], o[6], o[7]);
    }
  }
}

// MT = m16 row tiles (rows padded to 16*MT <= 64).  a.tiles row tiles of
// 16*MT rows, a.nsplit splits of the reached chunks; partials [b][kvh][tile][split]
// [kAttnMmaRows][kPartStride], counters [b][kvh][tile].
// One-tile blocks (single-token decode, short verify blocks) fit two CTAs per
// SM (<= 64 registers, ~113 KB of shared memory for a 4-bit or bf16 cache),
// which doubles the key splits the plan gives them (engine.cuh sdpa_mma_plan).
template <int MT, int BITS>
__global__ void __launch_bounds__(kAttnThreads, MT == 1 ? 2 : 1) sdpa_mma_kernel(SdpaArgs a) {
  constexpr int MP = 16 * MT;
  constexpr size_t RAW = sdpa_raw_stage<BITS>(), RB = (size_t)kHeadDim * BITS / 8;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* raw = smem;                                                   // [2][RAW]
  bf16_t* Qs = reinterpret_cast<bf16_t*>(smem + 2 * RAW);                // [MP][KP]
  bf16_t* Ks = Qs + MP * kAttnKP;                                        // [128][KP]
  bf16_t* Vs = Ks + kAttnChunk * kAttnKP;                                // [128][KP]
  float* S = reinterpret_cast<float*>(Vs + kAttnChunk * kAttnKP);        // [MP][SP]
  float* m_run = S + MP * kAttnSP;
  float* l_run = m_run + MP;
  float* alpha = l_run + MP;
  uint64_t* full = reinterpret_cast<uint64_t*>(alpha + MP);              // [2]
  __shared__ bool is_last;
  __shared__ int s_fail;

  grid_wait();
  grid_launch_dependents();
  const int split = blockIdx.x % a.nsplit, tile = blockIdx.x / a.nsplit;
  const int kvh = blockIdx.y, b = blockIdx.z;
  const int G = a.Hq / a.kv.Hk, rows = G * a.T;
  const int r0 = tile * MP, nr = min(MP, rows - r0);
  if (nr <= 0) return;
  const int off = a.kv.len[b];
  const int jmax = off + (r0 + nr - 1) / G + 1;
  const int nchunks = (jmax + kAttnChunk - 1) / kAttnChunk;
  const int cpc = (nchunks + a.nsplit - 1) / a.nsplit;  // this block's chunks, evenly over the splits
  const int tile_splits = (nchunks + cpc - 1) / cpc;
  if (split >= tile_splits) return;
  const int c_begin = split * cpc, c_end = min(nchunks, c_begin + cpc);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const size_t kvrow = ((size_t)b * a.kv.Hk + kvh) * a.kv.cap;
  auto chunk_rows = [&](int ch) { return min(kAttnChunk, jmax - ch * kAttnChunk); };

  // packed rows [j0, j0+jn) of chunk ch -> raw stage (ch - c_begin) & 1
  auto issue = [&](int ch) {
    const int j0 = ch * kAttnChunk, jn = chunk_rows(ch);
    uint8_t* dst = raw + (size_t)((ch - c_begin) & 1) * RAW;
    uint64_t* bar = &full[(ch - c_begin) & 1];
    const uint32_t bytes = (uint32_t)(jn * RB);
    mbar_arrive_expect_tx(bar, 2 * bytes);
    bulk_g2s(dst, reinterpret_cast<const uint8_t*>(a.kv.kq) + (kvrow + j0) * RB, bytes, bar);
    bulk_g2s(dst + kAttnChunk * RB, reinterpret_cast<const uint8_t*>(a.kv.vq) + (kvrow + j0) * RB, bytes, bar);
  };
  uint32_t sb[2 * kAttnItems], sr[4 * kAttnItems];
  if (BITS != 16) {
    if (tid == 0) {
      mbar_init(&full[0], 1);
      mbar_init(&full[1], 1);
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
      issue(c_begin);
    }
    sdpa_load_scales(a.kv, kvrow + (size_t)c_begin * kAttnChunk, chunk_rows(c_begin), tid, sr);
  }
  if (tid == 0) s_fail = 0;

  // queries (bf16, unscaled); padding rows zero
  for (int e = tid; e < MP * 16; e += kAttnThreads) {
    const int rr = e >> 4, c = e & 15;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (rr < nr) {
      const int r = r0 + rr, t = r / G, g = r % G;
      v = *reinterpret_cast<const uint4*>(a.q + ((size_t)b * a.T + t) * a.Hq * kHeadDim +
                                          (size_t)(kvh * G + g) * kHeadDim + c * 8);
    }
    *reinterpret_cast<uint4*>(Qs + rr * kAttnKP + c * 8) = v;
  }
  if (tid < MP) {
    m_run[tid] = -INFINITY;
    l_run[tid] = 0.0f;
    alpha[tid] = 1.0f;  // padding rows keep it
  }
  const float sl2 = __fmul_rn(a.scale, 1.4426950408889634f);  // scale * log2(e)
  // P V split: warp w owns head dims [16 (w % 8), +16) (two n8 tiles) over
  // the keys [64 (w / 8), +64) of each chunk, so a warp reads half of P; the
  // two key halves' partial outputs are added after the last chunk
  const int kh = warp >> 3, ds = warp & 7;
  float o[MT][2][4];
#pragma unroll
  for (int mi = 0; mi < MT; ++mi)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[mi][nt][e] = 0.0f;

  int ch = c_begin;
  for (; ch < c_end; ++ch) {
    const int j0 = ch * kAttnChunk, jn = chunk_rows(ch);
    __syncthreads();  // the previous chunk's reads of the tiles / raw stage are done
    if (BITS == 16) {
      for (int e = tid; e < kAttnChunk * 16; e += kAttnThreads) {
        const int j = e >> 4, c = e & 15;
        uint4 kc = make_uint4(0, 0, 0, 0), vc = make_uint4(0, 0, 0, 0);
        if (j < jn) {
          kc = kv_chunk8(a.kv, true, kvrow + j0 + j, c);
          vc = kv_chunk8(a.kv, false, kvrow + j0 + j, c);
        }
        *reinterpret_cast<uint4*>(Ks + j * kAttnKP + c * 8) = kc;
        *reinterpret_cast<uint4*>(Vs + j * kAttnKP + c * 8) = vc;
      }
    } else {
      if (tid == 0 && ch + 1 < c_end) issue(ch + 1);  // its stage was freed by the sync above
      // this chunk's scales (loaded a chunk ago), then the next chunk's loads
      sdpa_pack_scales(sr, sb);
      if (ch + 1 < c_end) sdpa_load_scales(a.kv, kvrow + j0 + kAttnChunk, chunk_rows(ch + 1), tid, sr);
      const int k = ch - c_begin;
      if (!mbar_wait_bounded(&full[k & 1], (uint32_t)((k >> 1) & 1), a.err, 0x42u)) s_fail = 1;
      sdpa_stage_raw<BITS>(jn, raw + (size_t)(k & 1) * RAW, sb, Ks, Vs, tid);
    }
    __syncthreads();
    if (s_fail) break;

    // S = Q K^T: warp w owns keys [8w, 8w+8); one x4 load covers two k16 steps
    {
      float s[MT][4];
#pragma unroll
      for (int mi = 0; mi < MT; ++mi)
#pragma unroll
        for (int e = 0; e < 4; ++e) s[mi][e] = 0.0f;
#pragma unroll
      for (int kk = 0; kk < kHeadDim / 32; ++kk) {
        uint32_t bf[4];
        ldsm_x4(bf, Ks + (8 * warp + (lane & 7)) * kAttnKP + kk * 32 + (lane >> 3) * 8);
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int mi = 0; mi < MT; ++mi) {
            uint32_t af[4];
            ldsm_x4(af, Qs + (mi * 16 + (lane & 15)) * kAttnKP + kk * 32 + h * 16 + (lane >> 4) * 8);
            mma_16816(s[mi], af, bf[2 * h], bf[2 * h + 1]);
          }
      }
#pragma unroll
      for (int mi = 0; mi < MT; ++mi) {
        const int row = mi * 16 + (lane >> 2), col = 8 * warp + 2 * (lane & 3);
        *reinterpret_cast<float2*>(S + row * kAttnSP + col) =
            make_float2(__fmul_rn(s[mi][0], sl2), __fmul_rn(s[mi][1], sl2));
        *reinterpret_cast<float2*>(S + (row + 8) * kAttnSP + col) =
            make_float2(__fmul_rn(s[mi][2], sl2), __fmul_rn(s[mi][3], sl2));
      }
    }
    __syncthreads();

    // online softmax in base 2 (S holds s * scale * log2 e), one warp per
    // valid row, lane l owns keys 4l..4l+3; P (bf16 hi at [0,128), lo at
    // [128,256) of the row's storage) overwrites the row's S.  Padding rows
    // are skipped: their P rows only feed output rows that are never stored.
    for (int rr = warp; rr < nr; rr += kAttnWarps) {
      const int vis = min(jn, off + (r0 + rr) / G + 1 - j0);
      const float4 s4 = *reinterpret_cast<const float4*>(S + rr * kAttnSP + 4 * lane);
      float v[4] = {s4.x, s4.y, s4.z, s4.w};
      float cmax = -INFINITY;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (4 * lane + k >= vis) v[k] = -INFINITY;
        cmax = fmaxf(cmax, v[k]);
      }
      for (int x = 16; x >= 1; x >>= 1) cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, x));
      const float m_old = m_run[rr];
      const float m_new = fmaxf(m_old, cmax);
      const bool none = m_new == -INFINITY;
      float pv[4], lo[4];
      float psum = 0.0f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        pv[k] = (!none && 4 * lane + k < vis) ? ex2(__fsub_rn(v[k], m_new)) : 0.0f;
        psum = __fadd_rn(psum, pv[k]);
      }
      const uint32_t h01 = bf2_pack(pv[0], pv[1]), h23 = bf2_pack(pv[2], pv[3]);
      lo[0] = __fsub_rn(pv[0], lo_bf(h01));
      lo[1] = __fsub_rn(pv[1], hi_bf(h01));
      lo[2] = __fsub_rn(pv[2], lo_bf(h23));
      lo[3] = __fsub_rn(pv[3], hi_bf(h23));
      psum = warp_sum_xor(psum, 16, 1);
      __syncwarp();
      bf16_t* prow = reinterpret_cast<bf16_t*>(S + rr * kAttnSP);
      *reinterpret_cast<uint2*>(prow + 4 * lane) = make_uint2(h01, h23);
      *reinterpret_cast<uint2*>(prow + kAttnChunk + 4 * lane) =
          make_uint2(bf2_pack(lo[0], lo[1]), bf2_pack(lo[2], lo[3]));
      if (lane == 0) {
        const float al = none ? 1.0f : ex2(__fsub_rn(m_old, m_new));
        alpha[rr] = al;
        l_run[rr] = __fadd_rn(__fmul_rn(l_run[rr], al), psum);
        m_run[rr] = m_new;
      }
    }
    __syncthreads();

    // O = O * alpha + P V over this warp's key half; one transposed x4 load
    // covers two k16 steps (32 keys) of 8 head dims
    {
      const bf16_t* P = reinterpret_cast<const bf16_t*>(S);
#pragma unroll
      for (int mi = 0; mi < MT; ++mi) {
        const float fa = alpha[mi * 16 + (lane >> 2)], fb = alpha[mi * 16 + (lane >> 2) + 8];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          o[mi][nt][0] = __fmul_rn(o[mi][nt][0], fa);
          o[mi][nt][1] = __fmul_rn(o[mi][nt][1], fa);
          o[mi][nt][2] = __fmul_rn(o[mi][nt][2], fb);
          o[mi][nt][3] = __fmul_rn(o[mi][nt][3], fb);
        }
      }
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        const int kb = 64 * kh + 32 * kk;
        uint32_t bf[2][4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
          ldsm_x4_t(bf[nt], Vs + (kb + (lane & 7) + (lane >> 3) * 8) * kAttnKP + 16 * ds + 8 * nt);
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int mi = 0; mi < MT; ++mi) {
            uint32_t af[4];
            const bf16_t* prow = P + (mi * 16 + (lane & 15)) * (2 * kAttnSP) + kb + h * 16 + (lane >> 4) * 8;
            ldsm_x4(af, prow + kAttnChunk);  // lo terms first: the smaller addend
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) mma_16816(o[mi][nt], af, bf[nt][2 * h], bf[nt][2 * h + 1]);
            ldsm_x4(af, prow);
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) mma_16816(o[mi][nt], af, bf[nt][2 * h], bf[nt][2 * h + 1]);
          }
      }
    }
  }
  __syncthreads();
  if (s_fail) {  // a copy never landed: wait (bounded) for what was issued, report
    if (BITS != 16 && tid == 0)
      for (int k = ch - c_begin; k <= ch + 1 - c_begin && c_begin + k < c_end; ++k)
        mbar_wait_bounded(&full[k & 1], (uint32_t)((k >> 1) & 1), a.err, 0x43u);
    return;
  }

  // the key halves' partial outputs: half 1 parks its tile in S (free now,
  // MP x 128 fp32 <= MP x kAttnSP), half 0 adds it
  float* Op = S;
#pragma unroll
  for (int mi = 0; mi < MT; ++mi)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int row = mi * 16 + (lane >> 2), d = 16 * ds + 8 * nt + 2 * (lane & 3);
      if (kh == 1) {
        *reinterpret_cast<float2*>(Op + row * kHeadDim + d) = make_float2(o[mi][nt][0], o[mi][nt][1]);
        *reinterpret_cast<float2*>(Op + (row + 8) * kHeadDim + d) = make_float2(o[mi][nt][2], o[mi][nt][3]);
      }
    }
  __syncthreads();
  float* part = a.part + ((((size_t)b * a.kv.Hk + kvh) * a.tiles + tile) * a.nsplit + split) *
                             (size_t)kAttnMmaRows * kPartStride;
  if (tid < nr) {
    part[tid * kPartStride + 0] = m_run[tid];
    part[tid * kPartStride + 1] = l_run[tid];
  }
  if (kh == 0) {
#pragma unroll
    for (int mi = 0; mi < MT; ++mi)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int row = mi * 16 + (lane >> 2), d = 16 * ds + 8 * nt + 2 * (lane & 3);
        const float2 u = *reinterpret_cast<const float2*>(Op + row * kHeadDim + d);
        const float2 w = *reinterpret_cast<const float2*>(Op + (row + 8) * kHeadDim + d);
        if (row < nr) {
          part[row * kPartStride + 2 + d] = __fadd_rn(o[mi][nt][0], u.x);
          part[row * kPartStride + 3 + d] = __fadd_rn(o[mi][nt][1], u.y);
        }
        if (row + 8 < nr) {
          part[(row + 8) * kPartStride + 2 + d] = __fadd_rn(o[mi][nt][2], w.x);
          part[(row + 8) * kPartStride + 3 + d] = __fadd_rn(o[mi][nt][3], w.y);
        }
      }
  }

  __threadfence();
  __syncthreads();
  unsigned* ctr = a.counters + ((size_t)b * a.kv.Hk + kvh) * a.tiles + tile;
  if (tid == 0) {
    const unsigned prev = atomicAdd(ctr, 1u);
    is_last = prev + 1 == (unsigned)tile_splits;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  const float* pb = a.part + (((size_t)b * a.kv.Hk + kvh) * a.tiles + tile) * a.nsplit *
                                 (size_t)kAttnMmaRows * kPartStride;
  for (int e = tid; e < nr * kHeadDim; e += kAttnThreads) {
    const int rr = e / kHeadDim, d = e % kHeadDim;
    float M = -INFINITY;
    for (int s = 0; s < tile_splits; ++s) M = fmaxf(M, __ldcg(pb + ((size_t)s * kAttnMmaRows + rr) * kPartStride));
    float L = 0.0f, O = 0.0f;
    for (int s = 0; s < tile_splits; ++s) {
      const float* ps = pb + ((size_t)s * kAttnMmaRows + rr) * kPartStride;
      const float ms = __ldcg(ps);
      if (ms == -INFINITY) continue;  // the row saw no key in this split
      const float w = ex2(__fsub_rn(ms, M));
      L = __fmaf_rn(w, __ldcg(ps + 1), L);
      O = __fmaf_rn(w, __ldcg(ps + 2 + d), O);
    }
    const int r = r0 + rr, t = r / G, g = r % G;
    a.out[((size_t)b * a.T + t) * a.Hq * kHeadDim + (size_t)(kvh * G + g) * kHeadDim + d] = f2bf(__fdiv_rn(O, L));
  }
  if (tid == 0) *ctr = 0u;
}

}  // namespace lmx
