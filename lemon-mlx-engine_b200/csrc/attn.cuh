// attn.cuh -- K4 (q/k RMSNorm + RoPE + KV-cache append / quantize) and
// K2 (split-K decode / verify SDPA over a bf16 or 4/8-bit affine KV cache).
//
// Reference: Qwen3Attention::operator() (src/llm/models/qwen3.cpp:69-99):
// q/k rms_norm per head, NeoX rope at the cache offset, cache->update
// (KVCacheSimple::update_impl src/common/kv_cache.cpp:34-110, or
// QuantizedKVCache::update_impl :271-298 which quantizes on append and
// dequantizes the whole cache for SDPA), then
// mx::fast::scaled_dot_product_attention with the [T, offset+T] causal mask
// (src/common/kv_cache.cpp:15-30).  Here the dequantize is fused into the
// SDPA tile loads and the append into the norm/rope kernel.
#pragma once
#include "lmx_common.cuh"

namespace lmx {

static constexpr int kHeadDim = 128;
static constexpr int kSplit = 128;   // keys per SDPA split (canonical constant)
static constexpr int kRowTile = 32;  // query rows per SDPA block

struct KvDesc {
  int B, Hk, cap, bits;        // bits: 16 (bf16) or 4 / 8 (affine, group 64)
  bf16_t* k;                   // bf16: [B][Hk][cap][D]
  bf16_t* v;
  uint32_t* kq;                // quantized: [B][Hk][cap][D*bits/32]
  uint32_t* vq;
  bf16_t *ks, *kb, *vs, *vb;   // [B][Hk][cap][D/64]
  int* len;                    // [B] valid rows per sequence (device)
};

// ---------------------------------------------------------------------------
// K4: one warp per (token row, head).  Lane l < 16 holds the 8-element chunk
// d = 8l..8l+7 of the head (lanes 16..31 hold nothing): the canonical RMSNorm
// partition (norm_argmax.cuh), rope pairs (d, d+64) sit in lanes l and l+8,
// and for the affine cache lane l packs exactly its own word(s).
// Quantize rule (per group of 64, group 0 = lanes 0..7, group 1 = lanes
// 8..15): scale = bf16((max-min)/(2^bits-1)) (1 if zero), bias = bf16(min),
// q = clamp(rint((x - bias)/scale)).
// ---------------------------------------------------------------------------
struct PrepArgs {
  const bf16_t* qkv;      // [R, ldq]: q heads, k heads, v heads
  int ldq;
  int R, T, Hq, Hk;
  const bf16_t* qn;       // q_norm weight [D] or null (no q/k norm)
  const bf16_t* kn;
  float eps;
  const float* cos_t;     // [max_pos][D/2]
  const float* sin_t;
  int max_pos;
  bf16_t* q_out;          // [R, Hq*D]
  KvDesc kv;
  unsigned* err;
};

LMX_DEV void unpack8(const uint4 v, float (&x)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int e = 0; e < 8; ++e) x[e] = (e & 1) ? hi_bf(w[e >> 1]) : lo_bf(w[e >> 1]);
}
LMX_DEV uint4 pack8(const float (&x)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) w[k] = (uint32_t)f2bf(x[2 * k]) | ((uint32_t)f2bf(x[2 * k + 1]) << 16);
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__global__ void __launch_bounds__(256) attn_prep_kernel(PrepArgs a) {
  grid_wait();
  grid_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nh = a.Hq + 2 * a.Hk;
  const int task = blockIdx.x * 8 + warp;
  if (task >= a.R * nh) return;
  const int r = task / nh, h = task % nh;
  const int b = r / a.T, t = r % a.T;
  const int pos = a.kv.len[b] + t;
  if (pos >= a.kv.cap || pos >= a.max_pos) {
    if (lane == 0 && a.err) atomicExch(a.err, 0x41u);
    return;
  }
  const bool has = lane < 16;
  float x[8];
  if (has) unpack8(*reinterpret_cast<const uint4*>(a.qkv + (size_t)r * a.ldq + (size_t)h * kHeadDim + 8 * lane), x);
  else
#pragma unroll
    for (int e = 0; e < 8; ++e) x[e] = 0.0f;
  const bool is_q = h < a.Hq, is_k = !is_q && h < a.Hq + a.Hk;
  if (is_q || is_k) {
    const bf16_t* nw = is_q ? a.qn : a.kn;
    if (nw) {
      float p = 0.0f;
#pragma unroll
      for (int e = 0; e < 8; ++e) p = __fmaf_rn(x[e], x[e], p);
      p = warp_sum_xor(p, 16, 1);
      const float f = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(p, (float)kHeadDim), a.eps)));
      if (has) {
        float w8[8];
        unpack8(*reinterpret_cast<const uint4*>(nw + 8 * lane), w8);
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = bf2f(f2bf(__fmul_rn(__fmul_rn(x[e], f), w8[e])));
      }
    }
    // NeoX rope: lane l < 8 holds d = 8l+e, its partner lane l+8 holds d+64
    float y[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) y[e] = __shfl_xor_sync(0xffffffffu, x[e], 8);
    if (has) {
      const int i0 = 8 * (lane & 7);
      const float* ct = a.cos_t + (size_t)pos * (kHeadDim / 2) + i0;
      const float* st = a.sin_t + (size_t)pos * (kHeadDim / 2) + i0;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float c = ct[e], s = st[e];
        if (lane < 8) x[e] = bf2f(f2bf(__fsub_rn(__fmul_rn(x[e], c), __fmul_rn(y[e], s))));
        else x[e] = bf2f(f2bf(__fadd_rn(__fmul_rn(x[e], c), __fmul_rn(y[e], s))));
      }
    }
  }
  if (is_q) {
    if (has)
      *reinterpret_cast<uint4*>(a.q_out + (size_t)r * a.Hq * kHeadDim + (size_t)h * kHeadDim + 8 * lane) = pack8(x);
    return;
  }
  const int hk = is_k ? h - a.Hq : h - a.Hq - a.Hk;
  const size_t row = ((size_t)b * a.kv.Hk + hk) * a.kv.cap + pos;
  if (a.kv.bits == 16) {
    if (has) *reinterpret_cast<uint4*>((is_k ? a.kv.k : a.kv.v) + row * kHeadDim + 8 * lane) = pack8(x);
    return;
  }
  // group-64 min / max over the 8 lanes of each group (lanes 16..31 mirror lanes 0..15)
  float mn = x[0], mx = x[0];
#pragma unroll
  for (int e = 1; e < 8; ++e) { mn = fminf(mn, x[e]); mx = fmaxf(mx, x[e]); }
  for (int off = 4; off >= 1; off >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, off));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  }
  if (!has) return;
  const int bits = a.kv.bits, nb = (1 << bits) - 1;
  bf16_t sb = f2bf(__fdiv_rn(__fsub_rn(mx, mn), (float)nb));
  float sc = bf2f(sb);
  if (sc == 0.0f) { sb = f2bf(1.0f); sc = 1.0f; }
  const bf16_t bb = f2bf(mn);
  const float bi = bf2f(bb);
  uint32_t q[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    int v = (int)rintf(__fdiv_rn(__fsub_rn(x[e], bi), sc));
    q[e] = (uint32_t)(v < 0 ? 0 : (v > nb ? nb : v));
  }
  uint32_t* words = (is_k ? a.kv.kq : a.kv.vq) + row * (kHeadDim * bits / 32);
  if (bits == 4) {
    uint32_t w = 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) w |= q[e] << (4 * e);
    words[lane] = w;
  } else {
    words[2 * lane] = q[0] | (q[1] << 8) | (q[2] << 16) | (q[3] << 24);
    words[2 * lane + 1] = q[4] | (q[5] << 8) | (q[6] << 16) | (q[7] << 24);
  }
  if ((lane & 7) == 0) {
    (is_k ? a.kv.ks : a.kv.vs)[row * 2 + (lane >> 3)] = sb;
    (is_k ? a.kv.kb : a.kv.vb)[row * 2 + (lane >> 3)] = bb;
  }
}

// ---------------------------------------------------------------------------
// K2: split-K SDPA.  Grid (nsplit_max * row_tiles, Hk, B); 256 threads.
// Query rows of one (b, kv head): r = t*G + g (head kvh*G + g), tiled by 32.
// Canonical order (identical to oracle orc_sdpa):
//   qs = q * scale; score = fma chain over d ascending from 0
//   m_s = max over visible keys of the split; p = exp(score - m_s)
//   l_s = butterfly of 32 lane partials (lane l: keys j0+l+32k ascending)
//   o_s[d] = fma chain of p_j v_j[d] over the split's keys ascending from 0
//   combine (last block of the tile, splits ascending):
//     M = max m_s, w = exp(m_s - M), L = fma(w, l_s, L), O = fma(w, o_s, O)
//   out = bf16(O / L)
// Scratch (caller-owned): partials [B][Hk][tiles][nsplit][32][130] floats and
// counters [B][Hk][tiles] (zero at rest; the combining block resets its own).
// ---------------------------------------------------------------------------
struct SdpaArgs {
  const bf16_t* q;        // [B*T, Hq*D] roped queries
  KvDesc kv;
  int T, Hq;
  float scale;
  int nsplit;             // splits per row tile in the grid (>= ceil(max len / 128))
  int tiles;
  float* part;            // scratch partials
  unsigned* counters;     // scratch counters
  bf16_t* out;            // [B*T, Hq*D]
  size_t part_floats;     // capacity of part (floats), checked by the launcher
  size_t n_counters;      // capacity of counters
  unsigned* err;          // device error word (bounded waits of the tensor-core path)
};

static constexpr int kPartStride = kHeadDim + 2;  // m, l, o[128]

// Dequantize (or copy) 8 consecutive K/V values d = 8c..8c+7 of one cache
// row into packed bf16 (bf16(fma(s, q, b)) for the affine cache).
// Chunk c (8 values) of a K or V row in two halves, so a caller can issue
// every load of a tile before converting any of it: kv_raw8 loads the raw
// words (bf16: the 8 values; 4 / 8-bit: the packed word(s) and the group's
// scale | bias << 16), kv_cvt8 dequantizes them, bf16(fma(s, q, b)).
LMX_DEV void kv_raw8(const KvDesc& kv, bool is_k, size_t row, int c, uint4& w, uint32_t& sb) {
  if (kv.bits == 16) {
    w = *reinterpret_cast<const uint4*>((is_k ? kv.k : kv.v) + row * kHeadDim + c * 8);
    sb = 0u;
    return;
  }
  sb = (uint32_t)(is_k ? kv.ks : kv.vs)[row * 2 + c / 8] | ((uint32_t)(is_k ? kv.kb : kv.vb)[row * 2 + c / 8] << 16);
  const uint32_t* p = (is_k ? kv.kq : kv.vq) + row * (kHeadDim * kv.bits / 32);
  w = make_uint4(0u, 0u, 0u, 0u);
  if (kv.bits == 4) {
    w.x = p[c];
  } else {
    w.x = p[2 * c];
    w.y = p[2 * c + 1];
  }
}

LMX_DEV uint4 kv_cvt8(int bits, const uint4& w, uint32_t sb) {
  if (bits == 16) return w;
  const float s = __uint_as_float(sb << 16), b = __uint_as_float(sb & 0xffff0000u);
  uint32_t q[8];
  if (bits == 4) {
#pragma unroll
    for (int e = 0; e < 8; ++e) q[e] = (w.x >> (4 * e)) & 0xFu;
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      q[e] = (w.x >> (8 * e)) & 0xFFu;
      q[4 + e] = (w.y >> (8 * e)) & 0xFFu;
    }
  }
  uint32_t o[4];
#pragma unroll
  for (int e = 0; e < 4; ++e)
    o[e] = (uint32_t)f2bf(__fmaf_rn(s, (float)q[2 * e], b)) |
           ((uint32_t)f2bf(__fmaf_rn(s, (float)q[2 * e + 1], b)) << 16);
  return make_uint4(o[0], o[1], o[2], o[3]);
}

LMX_DEV uint4 kv_chunk8(const KvDesc& kv, bool is_k, size_t row, int c) {
  uint4 w;
  uint32_t sb;
  kv_raw8(kv, is_k, row, c, w, sb);
  return kv_cvt8(kv.bits, w, sb);
}

static constexpr int kKPitch = kHeadDim + 8;  // bf16 elements per staged K row (16 B pad)

// RPT = query rows per thread (rows of the tile are split by parity between
// the two halves of the block), a template parameter so the row loops are
// short and unrolled.
template <int RPT>
__global__ void __launch_bounds__(256) sdpa_split_kernel(SdpaArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  bf16_t* Ks = reinterpret_cast<bf16_t*>(smem);                   // [kSplit][kKPitch]
  bf16_t* Vs = Ks + kSplit * kKPitch;                              // [kSplit][D]
  float* Qs = reinterpret_cast<float*>(Vs + kSplit * kHeadDim);    // [32][D]
  float* S = Qs + kRowTile * kHeadDim;                             // [32][kSplit]
  __shared__ bool is_last;

  grid_wait();
  grid_launch_dependents();
  const int split = blockIdx.x % a.nsplit, tile = blockIdx.x / a.nsplit;
  const int kvh = blockIdx.y, b = blockIdx.z;
  const int G = a.Hq / a.kv.Hk, rows = G * a.T;
  const int r0 = tile * kRowTile, nr = min(kRowTile, rows - r0);
  if (nr <= 0) return;
  const int off = a.kv.len[b];
  const int t_last = (r0 + nr - 1) / G;
  const int jmax = off + t_last + 1;
  const int tile_splits = (jmax + kSplit - 1) / kSplit;
  if (split >= tile_splits) return;
  const int j0 = split * kSplit, jn = min(kSplit, jmax - j0);
  const int jn4 = (jn + 3) & ~3;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const size_t kvrow0 = ((size_t)b * a.kv.Hk + kvh) * a.kv.cap + j0;

  // stage K, V rows [0, jn) as bf16 (16-byte chunks), zero V rows [jn, jn4):
  // every raw load of the tile first (one memory round trip), then the
  // conversions and shared-memory stores
  constexpr int kStageIters = kSplit * 16 / 256;
  uint4 kw[kStageIters], vw[kStageIters];
  uint32_t ksb[kStageIters], vsb[kStageIters];
#pragma unroll
  for (int i = 0; i < kStageIters; ++i) {
    const int e = tid + 256 * i, j = e >> 4, c = e & 15;
    kw[i] = vw[i] = make_uint4(0u, 0u, 0u, 0u);
    ksb[i] = vsb[i] = 0u;
    if (j < jn) {
      kv_raw8(a.kv, true, kvrow0 + j, c, kw[i], ksb[i]);
      kv_raw8(a.kv, false, kvrow0 + j, c, vw[i], vsb[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < kStageIters; ++i) {
    const int e = tid + 256 * i, j = e >> 4, c = e & 15;
    if (j < jn4) {
      uint4 kc = make_uint4(0u, 0u, 0u, 0u), vc = kc;
      if (j < jn) {
        kc = kv_cvt8(a.kv.bits, kw[i], ksb[i]);
        vc = kv_cvt8(a.kv.bits, vw[i], vsb[i]);
      }
      *reinterpret_cast<uint4*>(Ks + j * kKPitch + c * 8) = kc;
      *reinterpret_cast<uint4*>(Vs + j * kHeadDim + c * 8) = vc;
    }
  }
  for (int e = tid; e < nr * kHeadDim; e += 256) {
    const int rr = e / kHeadDim, d = e % kHeadDim;
    const int r = r0 + rr, t = r / G, g = r % G;
    Qs[e] = __fmul_rn(bf2f(a.q[((size_t)b * a.T + t) * a.Hq * kHeadDim + (size_t)(kvh * G + g) * kHeadDim + d]),
                      a.scale);
  }
  __syncthreads();

  // scores: thread (key j, row parity rp) holds RPT rows' accumulators; each
  // accumulator is an fma chain over d ascending
  {
    const int j = tid & (kSplit - 1), rp = tid >> 7;
    if (j < jn) {
      float acc[RPT];
#pragma unroll
      for (int i = 0; i < RPT; ++i) acc[i] = 0.0f;
      const bf16_t* kr = Ks + j * kKPitch;
#pragma unroll 2
      for (int dc = 0; dc < kHeadDim / 8; ++dc) {
        const uint4 kw = *reinterpret_cast<const uint4*>(kr + dc * 8);
        const float k8[8] = {lo_bf(kw.x), hi_bf(kw.x), lo_bf(kw.y), hi_bf(kw.y),
                             lo_bf(kw.z), hi_bf(kw.z), lo_bf(kw.w), hi_bf(kw.w)};
#pragma unroll
        for (int i = 0; i < RPT; ++i) {
          const int rr = rp + 2 * i;
          if (rr < nr) {
            const float4 qa = *reinterpret_cast<const float4*>(Qs + rr * kHeadDim + dc * 8);
            const float4 qb = *reinterpret_cast<const float4*>(Qs + rr * kHeadDim + dc * 8 + 4);
            float x = acc[i];
            x = __fmaf_rn(qa.x, k8[0], x);
            x = __fmaf_rn(qa.y, k8[1], x);
            x = __fmaf_rn(qa.z, k8[2], x);
            x = __fmaf_rn(qa.w, k8[3], x);
            x = __fmaf_rn(qb.x, k8[4], x);
            x = __fmaf_rn(qb.y, k8[5], x);
            x = __fmaf_rn(qb.z, k8[6], x);
            x = __fmaf_rn(qb.w, k8[7], x);
            acc[i] = x;
          }
        }
      }
#pragma unroll
      for (int i = 0; i < RPT; ++i)
        if (rp + 2 * i < nr) S[(rp + 2 * i) * kSplit + j] = acc[i];
    }
  }
  __syncthreads();

  float* part_base = a.part + ((((size_t)b * a.kv.Hk + kvh) * a.tiles + tile) * a.nsplit + split) *
                                  (size_t)kRowTile * kPartStride;
  for (int rr = warp; rr < nr; rr += 8) {
    const int t = (r0 + rr) / G;
    const int vis = min(jn, off + t + 1 - j0);
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < kSplit / 32; ++k) {
      const int j = lane + 32 * k;
      if (j < vis) m = fmaxf(m, S[rr * kSplit + j]);
    }
    for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float lp = 0.0f;
#pragma unroll
    for (int k = 0; k < kSplit / 32; ++k) {
      const int j = lane + 32 * k;
      float p = 0.0f;
      if (j < vis) p = exp_c(__fsub_rn(S[rr * kSplit + j], m));
      S[rr * kSplit + j] = p;
      lp = __fadd_rn(lp, p);
    }
    lp = warp_sum_xor(lp, 16, 1);
    if (lane == 0) {
      part_base[rr * kPartStride + 0] = m;
      part_base[rr * kPartStride + 1] = lp;
    }
  }
  __syncthreads();

  // o[d] for the thread's rows: fma chains over keys ascending.  Keys past a
  // row's visible range have p = 0 and the V rows past jn are zero-filled, so
  // the extra fma(0, v, acc) terms leave every chain exactly unchanged.
  {
    const int d = tid & (kHeadDim - 1), rp = tid >> 7;
    float acc[RPT];
#pragma unroll
    for (int i = 0; i < RPT; ++i) acc[i] = 0.0f;
#pragma unroll 2
    for (int j = 0; j < jn4; j += 4) {
      const float v0 = bf2f(Vs[j * kHeadDim + d]), v1 = bf2f(Vs[(j + 1) * kHeadDim + d]);
      const float v2 = bf2f(Vs[(j + 2) * kHeadDim + d]), v3 = bf2f(Vs[(j + 3) * kHeadDim + d]);
#pragma unroll
      for (int i = 0; i < RPT; ++i) {
        const int rr = rp + 2 * i;
        if (rr < nr) {
          const float4 p4 = *reinterpret_cast<const float4*>(S + rr * kSplit + j);
          float x = acc[i];
          x = __fmaf_rn(p4.x, v0, x);
          x = __fmaf_rn(p4.y, v1, x);
          x = __fmaf_rn(p4.z, v2, x);
          x = __fmaf_rn(p4.w, v3, x);
          acc[i] = x;
        }
      }
    }
#pragma unroll
    for (int i = 0; i < RPT; ++i)
      if (rp + 2 * i < nr) part_base[(rp + 2 * i) * kPartStride + 2 + d] = acc[i];
  }

  __threadfence();
  __syncthreads();
  unsigned* ctr = a.counters + ((size_t)b * a.kv.Hk + kvh) * a.tiles + tile;
  if (tid == 0) {
    unsigned prev = atomicAdd(ctr, 1u);
    is_last = prev + 1 == (unsigned)tile_splits;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  const float* pbase = a.part + (((size_t)b * a.kv.Hk + kvh) * a.tiles + tile) * a.nsplit *
                                    (size_t)kRowTile * kPartStride;
  for (int e = tid; e < nr * kHeadDim; e += 256) {
    const int rr = e / kHeadDim, d = e % kHeadDim;
    float M = -INFINITY;
    // other CTAs' partials: L2 loads (__ldcg), never a possibly stale L1 line
    for (int s = 0; s < tile_splits; ++s) M = fmaxf(M, __ldcg(pbase + ((size_t)s * kRowTile + rr) * kPartStride));
    float L = 0.0f, O = 0.0f;
    for (int s = 0; s < tile_splits; ++s) {
      const float* ps = pbase + ((size_t)s * kRowTile + rr) * kPartStride;
      const float w = exp_c(__fsub_rn(__ldcg(ps), M));
      L = __fmaf_rn(w, __ldcg(ps + 1), L);
      O = __fmaf_rn(w, __ldcg(ps + 2 + d), O);
    }
    const int r = r0 + rr, t = r / G, g = r % G;
    a.out[((size_t)b * a.T + t) * a.Hq * kHeadDim + (size_t)(kvh * G + g) * kHeadDim + d] =
        f2bf(__fdiv_rn(O, L));
  }
  if (tid == 0) *ctr = 0u;
}

static constexpr size_t kSdpaSmem = (size_t)kSplit * kKPitch * 2 + (size_t)kSplit * kHeadDim * 2 +
                                    (size_t)kRowTile * kHeadDim * 4 + (size_t)kRowTile * kSplit * 4;

}  // namespace lmx
