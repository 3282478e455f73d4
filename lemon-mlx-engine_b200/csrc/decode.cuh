// decode.cuh -- the fused small-batch decode forward: the whole decoder stack
// of a dense Qwen3 / Llama model for R = B*T <= 16 token rows (speculative
// draft tokens, short verify blocks) in ONE persistent cooperative launch.
//
// Why: at R <= 16 every op of a layer moves only a few MB, so as separate
// launches (RMSNorm, q|k|v, q/k norm + RoPE + KV append, SDPA, o_proj,
// RMSNorm, gate|up, down: 8 per layer) each one is bound by its own launch,
// ramp and memory latency, not by HBM.  Here one CTA per SM walks the same
// ops as five phases per layer separated by grid barriers:
//   A  q|k|v GEMV of rms_norm(h)                       -> qkv
//   B  attention: one CTA per (sequence, KV head): q norm + RoPE, the new
//      K/V rows (norm, RoPE, quantize, append to the cache), the 128-key
//      splits over its warps, their partials combined in order    -> o
//   C  o_proj GEMV + residual                           -> h
//   D  gate|up GEMV of rms_norm(h) + SwiGLU             -> act
//   E  down GEMV + residual                             -> h
// A producer warp per CTA streams each GEMV work item's bytes (packed weight
// rows with their scales / biases) into a ring in shared memory with
// cp.async.bulk (no multicast), completion on one mbarrier per item.
// Weights do not depend on the previous phase, so the producer runs ahead
// across the grid barriers and the HBM stream does not wait for them.  The
// attention phase reads the cached rows with coalesced loads, each lane its
// own keys (scores) or dims (P V).  Sixteen consumer warps compute.
//
// Numerics.  GEMV: MLX's qmv form per 64-k group, e = s * sum q x + b * sum x,
// with the codes exact on the tensor cores (mma.sync.m16n8k16, swap-AB:
// weight rows are the A operand, tokens B, sum x from an all-ones A) as the
// small-batch tensor-core GEMV (qmv_tc.cuh): within the tensor-core
// tolerance of the canonical order and deterministic (fixed warp and k-slice
// order).  RMSNorm, q/k norm, RoPE, quantize-on-append and the SDPA (splits
// of 128 keys, per-split max / exp / sums, ordered combine) execute the
// canonical CUDA-core order exactly (attn.cuh, norm_argmax.cuh).  Runs only in
// tensor-core mode; exact mode keeps the per-op kernels.
//
// Every wait is bounded: grid barriers give up after 2 s (device error word
// 0x72), ring-space waits after 4 s (0x73), item waits after 4 s (0x74); the
// CTA then drains the copies it issued and returns.
#pragma once
#include <cooperative_groups.h>

#include "attn.cuh"
#include "attn_mma.cuh"
#include "norm_argmax.cuh"
#include "qmm.cuh"
#include "qmm_mma.cuh"
#include "qmv_tc.cuh"

namespace lmx {

static constexpr int kDecWarps = 16;                       // consumer warps
static constexpr int kDecCons = kDecWarps * 32;            // consumer threads
static constexpr int kDecThreads = kDecCons + 32;          // + the producer warp
static constexpr int kDecSlots = 8;                        // items in flight
static constexpr int kDecMaxRows = 16;                     // R = B*T
static constexpr int kDecMaxSlice = 1024;                  // k per GEMV item
static constexpr int kDecPhases = 5;
static constexpr uint32_t kDecRing = 112 * 1024;           // staging ring bytes
static constexpr int kDecXP = kDecMaxSlice + 8;            // bf16 pitch of the staged x rows
static constexpr int kDecRedP = kDecMaxRows + 1;           // float pitch of the partial tiles
// union region: GEMV (x rows + per-warp partial tiles) or attention staging
static constexpr size_t kDecXBytes = (size_t)kDecMaxRows * kDecXP * 2;
static constexpr size_t kDecRedBytes = (size_t)kDecWarps * 32 * kDecRedP * 4;
static constexpr int kDecAttnRows = 8;  // query rows per KV head (G*T) the attention phase takes
static constexpr size_t kDecAttnBytes = (size_t)kDecAttnRows * kHeadDim * 4 + (size_t)2 * 8 * kHeadDim * 2 +
                                        (size_t)kDecWarps * kDecAttnRows * kSplit * 4;
static constexpr size_t kDecUnion = kDecXBytes + kDecRedBytes > kDecAttnBytes ? kDecXBytes + kDecRedBytes
                                                                              : kDecAttnBytes;
static constexpr size_t kDecSmem = kDecRing + kDecUnion;

struct DecLayer {
  QMat m[7];  // q k v o gate up down
  const bf16_t *in_norm, *post_norm, *q_norm, *k_norm;  // q/k norm null: none
  KvDesc kv;
};

struct DecArgs {
  const DecLayer* L;
  int nl, B, T, R, H, Hq, Hk, I;
  int ks[kDecPhases];  // k-slices per tile of the GEMV phases (index = phase)
  int nsplit;          // 128-key splits of the capacity (stride of the partials)
  float eps, scale;
  const float *cos_t, *sin_t;
  int max_pos;
  bf16_t *h, *qkv, *o, *act;
  float* gpart;        // split-K partial tiles [tiles][ks][32][R]
  unsigned* gcnt;      // per-tile arrival counters (zero at rest)
  float* apart;        // attention split partials [B][Hk][nsplit][32][130]
  unsigned* acnt;      // per (sequence, KV head) counters (zero at rest)
  unsigned* bar;       // [0] barrier arrivals, [1] exits (zero at rest)
  unsigned* err;
};

// ---- item geometry (identical in the producer and the consumers) ----------
struct DecGemv {
  int tiles, ks, K, kslice, nrows;  // nrows: weight rows per tile (16, SwiGLU 32)
};

LMX_DEV DecGemv dec_gemv(const DecArgs& a, int ph) {
  DecGemv g;
  g.ks = a.ks[ph];
  g.nrows = 16;
  if (ph == 0) { g.tiles = (a.Hq + 2 * a.Hk) * kHeadDim / 16; g.K = a.H; }
  else if (ph == 2) { g.tiles = a.H / 16; g.K = a.Hq * kHeadDim; }
  else if (ph == 3) { g.tiles = a.I / 16; g.K = a.H; g.nrows = 32; }
  else { g.tiles = a.H / 16; g.K = a.I; }
  g.kslice = g.K / g.ks;
  return g;
}

LMX_DEV int dec_items(const DecArgs& a, int ph) {  // GEMV phases (0, 2, 3, 4)
  const DecGemv g = dec_gemv(a, ph);
  return g.tiles * g.ks;
}

// Weight row `r` (0 .. nrows-1) of tile `tile`: matrix and row within it.
LMX_DEV const QMat& dec_row(const DecArgs& a, const DecLayer& L, int ph, int tile, int r, int& row) {
  if (ph == 0) {
    int v = tile * 16 + r;
    const int nq = a.Hq * kHeadDim, nk = a.Hk * kHeadDim;
    if (v < nq) { row = v; return L.m[0]; }
    v -= nq;
    if (v < nk) { row = v; return L.m[1]; }
    row = v - nk;
    return L.m[2];
  }
  if (ph == 2) { row = tile * 16 + r; return L.m[3]; }
  if (ph == 3) { row = tile * 16 + (r & 15); return r < 16 ? L.m[4] : L.m[5]; }
  row = tile * 16 + r;
  return L.m[6];
}

// Staged layout of a GEMV item: [nrows][wpitch] packed words, then scales and
// biases [nrows][spitch] bytes each.  The pitches keep the fragment loads free
// of bank conflicts (4-bit rows: 8 words mod 32; 8-bit: 16 words mod 32).
LMX_DEV int dec_wpitch(int kslice, int bits) { return bits == 4 ? kslice / 2 + 32 : kslice + 64; }
LMX_DEV int dec_spitch(int kslice) { return kslice / 32 + 16; }
LMX_DEV uint32_t dec_gemv_bytes(const DecGemv& g, int bits) {
  return (uint32_t)(g.nrows * (dec_wpitch(g.kslice, bits) + 2 * dec_spitch(g.kslice)));
}

struct DecCtl {
  uint64_t full[kDecSlots];
  unsigned long long head;          // producer: next free ring byte (virtual)
  unsigned long long tail;          // consumers: end of the last finished item (virtual)
  unsigned long long vend[kDecSlots];
  uint32_t off[kDecSlots];          // ring offset of the item in each slot
  int done_items;                   // items the consumers finished
  int issued;                       // items the producer issued (final when prod_done)
  int prod_done;
  int abort_;
  float fac[kDecMaxRows];           // RMSNorm factors of the phase's rows
  int is_last;
};

// ---- small device helpers ---------------------------------------------------
LMX_DEV uint32_t ld_acquire_gpu(const unsigned* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

LMX_DEV void dec_sync() { named_barrier(1, kDecCons); }

// Canonical RMSNorm factor (rms_factor_warp) reading x through L2: rows
// rewritten by other CTAs in an earlier phase must not come from L1.
LMX_DEV float dec_rms_factor(const bf16_t* x, int dim, float eps, int lane) {
  float p = 0.0f;
  const int nch = dim >> 3;
  for (int c0 = lane; c0 < nch; c0 += 256) {
    uint4 buf[8];
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (c0 + 32 * k < nch) buf[k] = __ldcg(reinterpret_cast<const uint4*>(x + 8 * (c0 + 32 * k)));
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (c0 + 32 * k < nch) {
        const uint32_t w[4] = {buf[k].x, buf[k].y, buf[k].z, buf[k].w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float v = (e & 1) ? hi_bf(w[e >> 1]) : lo_bf(w[e >> 1]);
          p = __fmaf_rn(v, v, p);
        }
      }
    }
  }
  p = warp_sum_xor(p, 16, 1);
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(p, (float)dim), eps)));
}

// Consumer-side grid barrier (every consumer thread calls it).
LMX_DEV bool dec_grid_sync(const DecArgs& a, DecCtl& c, unsigned target) {
  dec_sync();
  if (threadIdx.x == 0 && !c.abort_) {
    __threadfence();
    atomicAdd(a.bar, 1u);
    const uint64_t t0 = global_ns();
    uint32_t ns = 32;
    while (ld_acquire_gpu(a.bar) < target) {
      __nanosleep(ns);
      if (ns < 256) ns <<= 1;
      if (global_ns() - t0 > 2000000000ull) {
        atomicExch(a.err, 0x72u);
        c.abort_ = 1;
        break;
      }
    }
  }
  dec_sync();
  return !*(volatile int*)&c.abort_;
}

// q / k / v head `h` of row `r` from the q|k|v buffer: q/k RMSNorm (when the
// layer has the weights) and NeoX RoPE at `pos`, exactly as attn_prep_kernel;
// lanes < 16 return their 8 values (d = 8 lane ..).
LMX_DEV void dec_prep_head(const DecArgs& a, const DecLayer& L, int r, int h, int pos, int lane, float (&x)[8]) {
  const int ldq = (a.Hq + 2 * a.Hk) * kHeadDim;
  const bool has = lane < 16;
  if (has) unpack8(__ldcg(reinterpret_cast<const uint4*>(a.qkv + (size_t)r * ldq + (size_t)h * kHeadDim + 8 * lane)), x);
  else
#pragma unroll
    for (int e = 0; e < 8; ++e) x[e] = 0.0f;
  const bool is_q = h < a.Hq, is_k = !is_q && h < a.Hq + a.Hk;
  if (!(is_q || is_k)) return;
  const bf16_t* nw = is_q ? L.q_norm : L.k_norm;
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
  float y[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) y[e] = __shfl_xor_sync(0xffffffffu, x[e], 8);
  if (has) {
    const int i0 = 8 * (lane & 7);
    const float* ct = a.cos_t + (size_t)pos * (kHeadDim / 2) + i0;
    const float* st = a.sin_t + (size_t)pos * (kHeadDim / 2) + i0;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float cs = ct[e], sn = st[e];
      if (lane < 8) x[e] = bf2f(f2bf(__fsub_rn(__fmul_rn(x[e], cs), __fmul_rn(y[e], sn))));
      else x[e] = bf2f(f2bf(__fadd_rn(__fmul_rn(x[e], cs), __fmul_rn(y[e], sn))));
    }
  }
}

// Append one prepared K or V row (lanes < 16 hold d = 8 lane ..) to the cache
// at `row` -- quantize-on-append exactly as attn_prep_kernel -- and return in
// `deq` the values an SDPA read of that row sees.
LMX_DEV void dec_append(const KvDesc& kv, bool is_k, size_t row, int lane, const float (&x)[8], uint4& deq) {
  const bool has = lane < 16;
  if (kv.bits == 16) {
    if (has) {
      deq = pack8(x);
      *reinterpret_cast<uint4*>((is_k ? kv.k : kv.v) + row * kHeadDim + 8 * lane) = deq;
    }
    return;
  }
  float mn = x[0], mx = x[0];
#pragma unroll
  for (int e = 1; e < 8; ++e) { mn = fminf(mn, x[e]); mx = fmaxf(mx, x[e]); }
  for (int off = 4; off >= 1; off >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, off));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  }
  if (!has) return;
  const int bits = kv.bits, nb = (1 << bits) - 1;
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
  uint32_t* words = (is_k ? kv.kq : kv.vq) + row * (kHeadDim * bits / 32);
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
    (is_k ? kv.ks : kv.vs)[row * 2 + (lane >> 3)] = sb;
    (is_k ? kv.kb : kv.vb)[row * 2 + (lane >> 3)] = bb;
  }
  uint32_t o[4];
#pragma unroll
  for (int e = 0; e < 4; ++e)
    o[e] = (uint32_t)f2bf(__fmaf_rn(sc, (float)q[2 * e], bi)) | ((uint32_t)f2bf(__fmaf_rn(sc, (float)q[2 * e + 1], bi)) << 16);
  deq = make_uint4(o[0], o[1], o[2], o[3]);
}

// ---- producer (warp kDecWarps) ------------------------------------------------
// Walks this CTA's items in consumer order and issues their bulk copies: lane
// 0 reserves the slot and the ring bytes and arms the slot's mbarrier with the
// item's byte count, then the lanes issue the copies.
template <int BITS>
LMX_DEV void dec_producer(const DecArgs& a, DecCtl& c, uint8_t* ring) {
  const int lane = threadIdx.x & 31;
  int n = 0;
  bool stop = false;
  for (int l = 0; l < a.nl && !stop; ++l) {
    const DecLayer& L = a.L[l];
    for (int ph = 0; ph < kDecPhases && !stop; ++ph) {
      if (ph == 1) continue;  // the attention phase reads the cache directly
      const int items = dec_items(a, ph);
      for (int it = blockIdx.x; it < items && !stop; it += gridDim.x) {
        const DecGemv g = dec_gemv(a, ph);
        const uint32_t bytes = dec_gemv_bytes(g, BITS);
        const uint32_t tx = (uint32_t)g.nrows * (uint32_t)(g.kslice * BITS / 8 + 2 * (g.kslice / 32));
        const int slot = n % kDecSlots;
        int ok = 1;
        if (lane == 0) {
          const uint64_t t0 = global_ns();
          unsigned long long pos = 0;
          for (;;) {
            pos = c.head;
            if ((pos % kDecRing) + bytes > kDecRing) pos += kDecRing - pos % kDecRing;
            const int done = *(volatile int*)&c.done_items;
            const unsigned long long tail = *(volatile unsigned long long*)&c.tail;
            // free when the item's bytes stay clear of the unconsumed items
            // [tail, head); a drained ring (tail == head) takes any placement,
            // including one after skipping the ring's end
            if (done > n - kDecSlots && (tail == c.head || pos + bytes - tail <= kDecRing)) break;
            if (*(volatile int*)&c.abort_) { ok = 0; break; }
            __nanosleep(64);
            if (global_ns() - t0 > 4000000000ull) {
              atomicExch(a.err, 0x73u);
              c.abort_ = 1;
              ok = 0;
              break;
            }
          }
          if (ok) {
            c.head = pos + bytes;
            c.off[slot] = (uint32_t)(pos % kDecRing);
            c.vend[slot] = pos + bytes;
            mbar_arrive_expect_tx(&c.full[slot], tx);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) { stop = true; break; }
        __syncwarp();
        uint8_t* dst = ring + *(volatile uint32_t*)&c.off[slot];
        {
          const int tile = it / g.ks, k0 = (it % g.ks) * g.kslice;
          const int wp = dec_wpitch(g.kslice, BITS), spb = dec_spitch(g.kslice), G64 = g.K / 64;
          for (int r = lane; r < g.nrows; r += 32) {
            int row = 0;
            const QMat& M = dec_row(a, L, ph, tile, r, row);
            bulk_g2s(dst + r * wp, M.w + (size_t)row * (g.K * BITS / 32) + (size_t)k0 * BITS / 32,
                     (uint32_t)(g.kslice * BITS / 8), &c.full[slot]);
            bulk_g2s(dst + g.nrows * wp + r * spb, M.s + (size_t)row * G64 + k0 / 64, (uint32_t)(g.kslice / 32),
                     &c.full[slot]);
            bulk_g2s(dst + g.nrows * (wp + spb) + r * spb, M.b + (size_t)row * G64 + k0 / 64,
                     (uint32_t)(g.kslice / 32), &c.full[slot]);
          }
        }
        ++n;
      }
    }
  }
  if (lane == 0) {
    c.issued = n;
    __threadfence_block();
    *(volatile int*)&c.prod_done = 1;
  }
}

// ---- consumer: one GEMV item -------------------------------------------------
LMX_DEV void dec_epilogue(const DecArgs& a, int ph, int tile, int r, int m, float s0, float s1) {
  const int col = tile * 16 + r;
  if (ph == 0) {
    a.qkv[(size_t)m * (a.Hq + 2 * a.Hk) * kHeadDim + col] = f2bf(s0);
  } else if (ph == 3) {
    a.act[(size_t)m * a.I + col] = swiglu_c(f2bf(s0), f2bf(s1));
  } else {  // residual into h (o_proj, down)
    bf16_t* hp = a.h + (size_t)m * a.H + col;
    *hp = f2bf(__fadd_rn(bf2f(f2bf(s0)), bf2f(__ldcg(hp))));
  }
}

template <int BITS, int NT>
LMX_DEV void dec_gemv_item(const DecArgs& a, const DecLayer& L, DecCtl& c, int ph, int it, const uint8_t* st,
                           uint8_t* U, int& xk0) {
  const DecGemv g = dec_gemv(a, ph);
  const int tile = it / g.ks, ksl = it % g.ks, k0 = ksl * g.kslice;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, q = lane >> 2, cc = lane & 3;
  bf16_t* X = reinterpret_cast<bf16_t*>(U);
  float* red = reinterpret_cast<float*>(U + kDecXBytes);
  const int R = a.R;
  // 1. x[:, k0 .. k0+kslice) into shared memory (normalised for q|k|v and
  // gate|up), once per (phase, slice); rows R .. 8 NT-1 are zero
  if (xk0 != k0) {
    const bf16_t* src = ph == 2 ? a.o : (ph == 4 ? a.act : a.h);
    const int ld = ph == 2 ? a.Hq * kHeadDim : (ph == 4 ? a.I : a.H);
    const bf16_t* nw = ph == 0 ? L.in_norm : (ph == 3 ? L.post_norm : nullptr);
    const int cpr = g.kslice / 8;
    for (int e = tid; e < 8 * NT * cpr; e += kDecCons) {
      const int m = e / cpr, ch = e - m * cpr;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (m < R) {
        v = __ldcg(reinterpret_cast<const uint4*>(src + (size_t)m * ld + k0 + 8 * ch));
        if (nw) v = rms_apply8(v, *reinterpret_cast<const uint4*>(nw + k0 + 8 * ch), c.fac[m]);
      }
      *reinterpret_cast<uint4*>(X + m * kDecXP + 8 * ch) = v;
    }
    dec_sync();
    xk0 = k0;
  }
  // 2. products: warps split into nsub row subtiles, each warp takes every
  // wps-th group of the slice
  const int nsub = g.nrows / 16, wps = kDecWarps / nsub, sub = warp / wps, wi = warp % wps;
  const int ngr = g.kslice / 64, wp = dec_wpitch(g.kslice, BITS), spb = dec_spitch(g.kslice);
  const uint8_t* wa = st + (size_t)(sub * 16 + q) * wp;
  const uint8_t* wb = wa + 8 * wp;
  const bf16_t* sa = reinterpret_cast<const bf16_t*>(st + (size_t)g.nrows * wp + (size_t)(sub * 16 + q) * spb);
  const bf16_t* sbp = reinterpret_cast<const bf16_t*>(reinterpret_cast<const uint8_t*>(sa) + 8 * spb);
  const bf16_t* ba = reinterpret_cast<const bf16_t*>(reinterpret_cast<const uint8_t*>(sa) + (size_t)g.nrows * spb);
  const bf16_t* bbp = reinterpret_cast<const bf16_t*>(reinterpret_cast<const uint8_t*>(ba) + 8 * spb);
  float acc[NT][4];
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[t][e] = 0.0f;
  const uint32_t one2 = 0x3F803F80u, m128 = 0xC300C300u;
  const uint32_t ones[4] = {one2, one2, one2, one2};
  for (int gi = wi; gi < ngr; gi += wps) {
    constexpr int LW = BITS / 2;
    uint32_t A[LW], B[LW];
    if constexpr (BITS == 4) {
      const uint2 x0 = *reinterpret_cast<const uint2*>(wa + gi * 32 + 8 * cc);
      const uint2 x1 = *reinterpret_cast<const uint2*>(wb + gi * 32 + 8 * cc);
      A[0] = x0.x, A[1] = x0.y, B[0] = x1.x, B[1] = x1.y;
    } else {
      const uint4 x0 = *reinterpret_cast<const uint4*>(wa + gi * 64 + 16 * cc);
      const uint4 x1 = *reinterpret_cast<const uint4*>(wb + gi * 64 + 16 * cc);
      A[0] = x0.x, A[1] = x0.y, A[2] = x0.z, A[3] = x0.w;
      B[0] = x1.x, B[1] = x1.y, B[2] = x1.z, B[3] = x1.w;
    }
    uint32_t Xf[NT][8];
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const bf16_t* xr = X + (t * 8 + q) * kDecXP + gi * 64 + 16 * cc;
      const uint4 lo = *reinterpret_cast<const uint4*>(xr), hi = *reinterpret_cast<const uint4*>(xr + 8);
      Xf[t][0] = lo.x, Xf[t][1] = lo.y, Xf[t][2] = lo.z, Xf[t][3] = lo.w;
      Xf[t][4] = hi.x, Xf[t][5] = hi.y, Xf[t][6] = hi.z, Xf[t][7] = hi.w;
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
        af[0] = bf2_fma(((A[h] >> (4 * i)) & 0x000F000Fu) | 0x43004300u, one2, m128);
        af[1] = bf2_fma(((B[h] >> (4 * i)) & 0x000F000Fu) | 0x43004300u, one2, m128);
        af[2] = bf2_fma(((A[h] >> (4 * i + 4)) & 0x000F000Fu) | 0x43004300u, one2, m128);
        af[3] = bf2_fma(((B[h] >> (4 * i + 4)) & 0x000F000Fu) | 0x43004300u, one2, m128);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const uint32_t x0 = Xf[t][4 * h + (i >> 1)], x1 = Xf[t][4 * h + 2 + (i >> 1)];
          bfr[t][0] = __byte_perm(x0, x1, 0x5410);
          bfr[t][1] = __byte_perm(x0, x1, 0x7632);
        }
      } else {
        af[0] = bf2_pack(tcg_code8(A[kk], 0), tcg_code8(A[kk], 1));
        af[1] = bf2_pack(tcg_code8(B[kk], 0), tcg_code8(B[kk], 1));
        af[2] = bf2_pack(tcg_code8(A[kk], 2), tcg_code8(A[kk], 3));
        af[3] = bf2_pack(tcg_code8(B[kk], 2), tcg_code8(B[kk], 3));
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          bfr[t][0] = Xf[t][2 * kk];
          bfr[t][1] = Xf[t][2 * kk + 1];
        }
      }
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        mma_16816(dot[t], af, bfr[t][0], bfr[t][1]);
        mma_16816(xs[t], ones, bfr[t][0], bfr[t][1]);
      }
    }
    const float s_a = bf2f(sa[gi]), b_a = bf2f(ba[gi]), s_b = bf2f(sbp[gi]), b_b = bf2f(bbp[gi]);
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      acc[t][0] = __fadd_rn(acc[t][0], __fmaf_rn(s_a, dot[t][0], __fmul_rn(b_a, xs[t][0])));
      acc[t][1] = __fadd_rn(acc[t][1], __fmaf_rn(s_a, dot[t][1], __fmul_rn(b_a, xs[t][1])));
      acc[t][2] = __fadd_rn(acc[t][2], __fmaf_rn(s_b, dot[t][2], __fmul_rn(b_b, xs[t][2])));
      acc[t][3] = __fadd_rn(acc[t][3], __fmaf_rn(s_b, dot[t][3], __fmul_rn(b_b, xs[t][3])));
    }
  }
  // 3. per-warp partial tiles: rows (q, q+8) of the subtile, tokens t*8+2cc, +1
  float* rw = red + (size_t)warp * 32 * kDecRedP;
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    rw[(sub * 16 + q) * kDecRedP + t * 8 + 2 * cc] = acc[t][0];
    rw[(sub * 16 + q) * kDecRedP + t * 8 + 2 * cc + 1] = acc[t][1];
    rw[(sub * 16 + q + 8) * kDecRedP + t * 8 + 2 * cc] = acc[t][2];
    rw[(sub * 16 + q + 8) * kDecRedP + t * 8 + 2 * cc + 1] = acc[t][3];
  }
  dec_sync();
  // 4. sum the warps of each subtile in warp order; epilogue, or this slice's
  // partial tile (split K: the last slice to arrive sums the slices in order)
  const bool sw = ph == 3;
  for (int e = tid; e < 16 * R; e += kDecCons) {
    const int r = e & 15, m = e >> 4;
    float s0 = 0.0f, s1 = 0.0f;
    for (int w = 0; w < wps; ++w) s0 = __fadd_rn(s0, red[((size_t)w * 32 + r) * kDecRedP + m]);
    if (sw)
      for (int w = wps; w < 2 * wps; ++w) s1 = __fadd_rn(s1, red[((size_t)w * 32 + 16 + r) * kDecRedP + m]);
    if (g.ks == 1) {
      dec_epilogue(a, ph, tile, r, m, s0, s1);
    } else {
      float* gp = a.gpart + ((size_t)(tile * g.ks + ksl) * 32) * R;
      gp[r * R + m] = s0;
      if (sw) gp[(16 + r) * R + m] = s1;
    }
  }
  if (g.ks > 1) {
    __threadfence();
    dec_sync();
    if (tid == 0) c.is_last = atomicAdd(a.gcnt + tile, 1u) + 1u == (unsigned)g.ks;
    dec_sync();
    if (c.is_last) {
      __threadfence();
      for (int e = tid; e < 16 * R; e += kDecCons) {
        const int r = e & 15, m = e >> 4;
        float s0 = 0.0f, s1 = 0.0f;
        for (int k = 0; k < g.ks; ++k) {
          const float* gp = a.gpart + ((size_t)(tile * g.ks + k) * 32) * R;
          s0 = __fadd_rn(s0, __ldcg(gp + r * R + m));
          if (sw) s1 = __fadd_rn(s1, __ldcg(gp + (16 + r) * R + m));
        }
        dec_epilogue(a, ph, tile, r, m, s0, s1);
      }
      if (tid == 0) a.gcnt[tile] = 0u;
    }
  }
}

// ---- consumer: the attention of one (sequence, KV head) ---------------------
// The canonical split SDPA (sdpa_split_kernel's order) with the splits of 128
// keys spread over the CTA's warps: warp w takes splits w, w + 16, ...; lane l
// scores keys l, l+32, l+64, l+96 of a split (each an fma chain over d
// ascending, K dequantized on the fly from the cached codes as kv_chunk8),
// the warp forms the split's max / exp / lane-ordered sum, then lane l
// accumulates o[d] for d = 4l .. 4l+3 as fma chains over the split's keys
// ascending.  Split partials (m, l, o) go to global scratch and are combined
// in split order by the CTA -- no cross-CTA hand-off.  The block's new K / V
// rows are prepared (norm, RoPE, quantize), appended to the cache and kept in
// shared memory as the values a cache read returns.  NR >= G*T query rows.
static constexpr int kDecSP = kSplit;  // keys per split
LMX_DEV float dec_deq(float s, uint32_t q, float b) { return bf2f(f2bf(__fmaf_rn(s, (float)q, b))); }

template <int NR>
LMX_DEV void dec_attn_seq(const DecArgs& a, const DecLayer& L, int b, int kvh, uint8_t* U) {
  const KvDesc& kv = L.kv;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = a.Hq / a.Hk, T = a.T, nr = G * T;
  const int len = __ldcg(kv.len + b), jmax = len + T;
  const int nsp = (jmax + kDecSP - 1) / kDecSP;
  float* Qs = reinterpret_cast<float*>(U);                          // [NR][128]
  bf16_t* Nk = reinterpret_cast<bf16_t*>(Qs + NR * kHeadDim);       // [8][128] new K rows
  bf16_t* Nv = Nk + 8 * kHeadDim;                                   // [8][128] new V rows
  float* S = reinterpret_cast<float*>(Nv + 8 * kHeadDim) + warp * NR * kDecSP;  // this warp's [NR][128]
  if (jmax > kv.cap || jmax > a.max_pos) {  // the block does not fit the cache: report, write nothing
    if (tid == 0) atomicExch(a.err, 0x41u);
    return;
  }
  // (a) query rows (q norm + RoPE, scaled) and the new K / V rows
  for (int task = warp; task < nr + 2 * T; task += kDecWarps) {
    float x[8];
    if (task < nr) {
      const int t = task / G, gq = task % G;
      dec_prep_head(a, L, b * T + t, kvh * G + gq, len + t, lane, x);
      if (lane < 16)
#pragma unroll
        for (int e = 0; e < 8; ++e) Qs[task * kHeadDim + 8 * lane + e] = __fmul_rn(x[e], a.scale);
    } else {
      const int u = task - nr, t = u >> 1;
      const bool is_k = (u & 1) == 0;
      dec_prep_head(a, L, b * T + t, is_k ? a.Hq + kvh : a.Hq + a.Hk + kvh, len + t, lane, x);
      uint4 deq = make_uint4(0, 0, 0, 0);
      dec_append(kv, is_k, ((size_t)b * kv.Hk + kvh) * kv.cap + len + t, lane, x, deq);
      if (lane < 16) *reinterpret_cast<uint4*>((is_k ? Nk : Nv) + t * kHeadDim + 8 * lane) = deq;
    }
  }
  for (int e = tid; e < (NR - nr) * kHeadDim; e += kDecCons) Qs[nr * kHeadDim + e] = 0.0f;
  dec_sync();
  const size_t base = ((size_t)b * kv.Hk + kvh) * kv.cap;
  const int bits = kv.bits;
  float* part = a.apart + ((size_t)b * a.Hk + kvh) * a.nsplit * (size_t)kRowTile * kPartStride;
  for (int sp = warp; sp < nsp; sp += kDecWarps) {
    const int j0 = sp * kDecSP, jn = min(kDecSP, jmax - j0);
    // scores
#pragma unroll 1
    for (int k = 0; k < 4; ++k) {
      const int j = lane + 32 * k;
      if (j >= jn) break;
      const int row = j0 + j;
      float acc[NR];
#pragma unroll
      for (int r = 0; r < NR; ++r) acc[r] = 0.0f;
      if (row >= len) {  // a new row of this block
        const bf16_t* kr = Nk + (row - len) * kHeadDim;
#pragma unroll 4
        for (int d = 0; d < kHeadDim; ++d) {
          const float kv_ = bf2f(kr[d]);
#pragma unroll
          for (int r = 0; r < NR; ++r) acc[r] = __fmaf_rn(Qs[r * kHeadDim + d], kv_, acc[r]);
        }
      } else if (bits == 16) {
        const uint4* kr = reinterpret_cast<const uint4*>(kv.k + (base + row) * kHeadDim);
#pragma unroll 2
        for (int c8 = 0; c8 < kHeadDim / 8; ++c8) {
          const uint4 w = kr[c8];
          const float k8[8] = {lo_bf(w.x), hi_bf(w.x), lo_bf(w.y), hi_bf(w.y),
                               lo_bf(w.z), hi_bf(w.z), lo_bf(w.w), hi_bf(w.w)};
#pragma unroll
          for (int e = 0; e < 8; ++e)
#pragma unroll
            for (int r = 0; r < NR; ++r) acc[r] = __fmaf_rn(Qs[r * kHeadDim + 8 * c8 + e], k8[e], acc[r]);
        }
      } else {
        const uint32_t* kr = kv.kq + (base + row) * (kHeadDim * bits / 32);
#pragma unroll 1
        for (int g = 0; g < 2; ++g) {
          const float s = bf2f(kv.ks[(base + row) * 2 + g]), bb = bf2f(kv.kb[(base + row) * 2 + g]);
          const int nw = 64 * bits / 32;  // words of one 64-d group
#pragma unroll 2
          for (int wi = 0; wi < nw; ++wi) {
            const uint32_t w = kr[g * nw + wi];
            const int per = 32 / bits;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              if (e >= per) break;
              const float kv_ = dec_deq(s, (w >> (bits * e)) & ((1u << bits) - 1u), bb);
              const int d = 64 * g + wi * per + e;
#pragma unroll
              for (int r = 0; r < NR; ++r) acc[r] = __fmaf_rn(Qs[r * kHeadDim + d], kv_, acc[r]);
            }
          }
        }
      }
#pragma unroll
      for (int r = 0; r < NR; ++r) S[r * kDecSP + j] = acc[r];
    }
    __syncwarp();
    // split softmax per row (canonical: lane l owns keys l + 32k)
    for (int r = 0; r < nr; ++r) {
      const int t = r / G;
      const int vis = min(jn, len + t + 1 - j0);
      float m = -INFINITY;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int j = lane + 32 * k;
        if (j < vis) m = fmaxf(m, S[r * kDecSP + j]);
      }
      for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      float lp = 0.0f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int j = lane + 32 * k;
        float p = 0.0f;
        if (j < vis) p = exp_c(__fsub_rn(S[r * kDecSP + j], m));
        S[r * kDecSP + j] = p;
        lp = __fadd_rn(lp, p);
      }
      lp = warp_sum_xor(lp, 16, 1);
      if (lane == 0) {
        float* pb = part + ((size_t)sp * kRowTile + r) * kPartStride;
        pb[0] = m;
        pb[1] = lp;
      }
    }
    __syncwarp();
    // o[d], d = 4 lane .. 4 lane + 3: fma chains over the split's keys ascending
    float o[NR][4];
#pragma unroll
    for (int r = 0; r < NR; ++r)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[r][e] = 0.0f;
    const int g = lane >> 4;
#pragma unroll 2
    for (int j = 0; j < jn; ++j) {
      const int row = j0 + j;
      float v[4];
      if (row >= len) {
        const uint2 w = *reinterpret_cast<const uint2*>(Nv + (row - len) * kHeadDim + 4 * lane);
        v[0] = lo_bf(w.x), v[1] = hi_bf(w.x), v[2] = lo_bf(w.y), v[3] = hi_bf(w.y);
      } else if (bits == 16) {
        const uint2 w = *reinterpret_cast<const uint2*>(kv.v + (base + row) * kHeadDim + 4 * lane);
        v[0] = lo_bf(w.x), v[1] = hi_bf(w.x), v[2] = lo_bf(w.y), v[3] = hi_bf(w.y);
      } else {
        const float s = bf2f(kv.vs[(base + row) * 2 + g]), bb = bf2f(kv.vb[(base + row) * 2 + g]);
        const uint32_t* vr = kv.vq + (base + row) * (kHeadDim * bits / 32);
        if (bits == 4) {
          const uint32_t w = vr[lane >> 1] >> ((lane & 1) * 16);
#pragma unroll
          for (int e = 0; e < 4; ++e) v[e] = dec_deq(s, (w >> (4 * e)) & 0xFu, bb);
        } else {
          const uint32_t w = vr[lane];
#pragma unroll
          for (int e = 0; e < 4; ++e) v[e] = dec_deq(s, (w >> (8 * e)) & 0xFFu, bb);
        }
      }
#pragma unroll
      for (int r = 0; r < NR; ++r) {
        const float p = S[r * kDecSP + j];
#pragma unroll
        for (int e = 0; e < 4; ++e) o[r][e] = __fmaf_rn(p, v[e], o[r][e]);
      }
    }
    // (rows of kPartStride = 130 floats: the o[] part is 8-byte aligned)
#pragma unroll
    for (int r = 0; r < NR; ++r)
      if (r < nr) {
        float2* po = reinterpret_cast<float2*>(part + ((size_t)sp * kRowTile + r) * kPartStride + 2 + 4 * lane);
        po[0] = make_float2(o[r][0], o[r][1]);
        po[1] = make_float2(o[r][2], o[r][3]);
      }
    __syncwarp();
  }
  dec_sync();
  // combine the splits in order (canonical), this CTA's own partials
  for (int e = tid; e < nr * kHeadDim; e += kDecCons) {
    const int rr = e / kHeadDim, d = e % kHeadDim;
    float M = -INFINITY;
    for (int s = 0; s < nsp; ++s) M = fmaxf(M, __ldcg(part + ((size_t)s * kRowTile + rr) * kPartStride));
    float Lsum = 0.0f, O = 0.0f;
    for (int s = 0; s < nsp; ++s) {
      const float* ps = part + ((size_t)s * kRowTile + rr) * kPartStride;
      const float w = exp_c(__fsub_rn(__ldcg(ps), M));
      Lsum = __fmaf_rn(w, __ldcg(ps + 1), Lsum);
      O = __fmaf_rn(w, __ldcg(ps + 2 + d), O);
    }
    const int t = rr / G, gq = rr % G;
    a.o[((size_t)b * T + t) * a.Hq * kHeadDim + (size_t)(kvh * G + gq) * kHeadDim + d] = f2bf(__fdiv_rn(O, Lsum));
  }
}

// ---- the kernel ----------------------------------------------------------------
template <int BITS, int NT>
__global__ void __launch_bounds__(kDecThreads, 1) decode_fwd_kernel(DecArgs a) {
  extern __shared__ __align__(128) uint8_t dsm[];
  __shared__ DecCtl c;
  uint8_t* ring = dsm;
  uint8_t* U = dsm + kDecRing;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < kDecSlots; ++s) mbar_init(&c.full[s], 1);
    c.head = c.tail = 0;
    c.done_items = 0;
    c.issued = 0;
    c.prod_done = 0;
    c.abort_ = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (warp == kDecWarps) {
    dec_producer<BITS>(a, c, ring);
    return;
  }
  grid_wait();  // h from the embedding, lengths and cache rows from earlier kernels
  int n = 0;
  unsigned nbar = 0;
  bool ok = true;
  for (int l = 0; l < a.nl && ok; ++l) {
    const DecLayer& L = a.L[l];
    for (int ph = 0; ph < kDecPhases && ok; ++ph) {
      if (ph == 0 || ph == 3) {  // RMSNorm factors of the rows of h
        if (warp < a.R) {
          const float f = dec_rms_factor(a.h + (size_t)warp * a.H, a.H, a.eps, lane);
          if (lane == 0) c.fac[warp] = f;
        }
        dec_sync();
      }
      int xk0 = -1;
      if (ph == 1) {  // attention: one (sequence, KV head) per CTA, no staged bytes
        const int nr = (a.Hq / a.Hk) * a.T;
        for (int it = blockIdx.x; it < a.B * a.Hk; it += gridDim.x) {
          if (nr <= 2) dec_attn_seq<2>(a, L, it / a.Hk, it % a.Hk, U);
          else if (nr <= 4) dec_attn_seq<4>(a, L, it / a.Hk, it % a.Hk, U);
          else dec_attn_seq<8>(a, L, it / a.Hk, it % a.Hk, U);
          dec_sync();
        }
      }
      const int items = ph == 1 ? 0 : dec_items(a, ph);
      for (int it = blockIdx.x; it < items && ok; it += gridDim.x) {
        const int slot = n % kDecSlots;
        if (!mbar_wait_bounded(&c.full[slot], (uint32_t)((n / kDecSlots) & 1), a.err, 0x74u)) c.abort_ = 1;
        dec_sync();
        if (*(volatile int*)&c.abort_) { ok = false; break; }
        const uint8_t* st = ring + c.off[slot];
        if (NT == 1) dec_gemv_item<BITS, 1>(a, L, c, ph, it, st, U, xk0);
        else dec_gemv_item<BITS, 2>(a, L, c, ph, it, st, U, xk0);
        dec_sync();  // every consumer is done with the stage (and with U)
        if (tid == 0) {
          *(volatile unsigned long long*)&c.tail = c.vend[slot];
          __threadfence_block();
          *(volatile int*)&c.done_items = n + 1;
        }
        ++n;
      }
      if (!ok) break;
      if (l + 1 < a.nl || ph + 1 < kDecPhases) ok = dec_grid_sync(a, c, ++nbar * gridDim.x);
    }
  }
  // drain: on an early exit wait (bounded) for the copies already issued
  if (tid == 0) {
    const uint64_t t0 = global_ns();
    while (!*(volatile int*)&c.prod_done && global_ns() - t0 < 4000000000ull) __nanosleep(128);
    const int issued = *(volatile int*)&c.issued;
    for (int i = n; i < issued; ++i) mbar_wait_bounded(&c.full[i % kDecSlots], (uint32_t)((i / kDecSlots) & 1), a.err, 0x74u);
    // the last CTA out resets the barrier counters for the next launch
    __threadfence();
    if (atomicAdd(a.bar + 1, 1u) + 1u == gridDim.x) {
      a.bar[0] = 0u;
      a.bar[1] = 0u;
      __threadfence();
    }
  }
}

}  // namespace lmx

// ---- host side -------------------------------------------------------------------
namespace lmx {

struct DecPlan {
  int ks[kDecPhases] = {};
  size_t gpart_floats = 0;  // split-K partial tiles
  int max_tiles = 0;        // per-tile counters
};

// k-slices of a GEMV phase: slices are multiples of 512 dividing K (the bulk
// copies of the scale / bias rows then start and end on 16-byte boundaries)
// and at most kDecMaxSlice; the fewest whose items fill the grid.
static int dec_ks_choice(int tiles, int K, int grid) {
  int best = -1;
  for (int ks = 1; ks <= K / 512; ++ks) {
    if (K % ks || (K / ks) % 512 || K / ks > kDecMaxSlice) continue;
    best = ks;
    if (tiles * ks >= grid) break;
  }
  return best;
}

static bool dec_plan(int H, int Hq, int Hk, int I, int R, int grid, DecPlan& p) {
  const int tiles[kDecPhases] = {(Hq + 2 * Hk) * kHeadDim / 16, 0, H / 16, I / 16, H / 16};
  const int Ks[kDecPhases] = {H, 0, Hq * kHeadDim, H, I};
  p.gpart_floats = 0;
  p.max_tiles = 0;
  for (int ph = 0; ph < kDecPhases; ++ph) {
    if (ph == 1) { p.ks[ph] = 1; continue; }
    p.ks[ph] = dec_ks_choice(tiles[ph], Ks[ph], grid);
    if (p.ks[ph] < 1) return false;
    p.gpart_floats = std::max(p.gpart_floats, (size_t)tiles[ph] * p.ks[ph] * 32 * R);
    p.max_tiles = std::max(p.max_tiles, tiles[ph]);
  }
  return true;
}

template <int BITS, int NT>
static int dec_occupancy() {
  static int occ[64] = {};
  int d = 0;
  cudaGetDevice(&d);
  if (!occ[d & 63]) {
    int n = 0;
    if (cudaFuncSetAttribute(decode_fwd_kernel<BITS, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kDecSmem) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_fwd_kernel<BITS, NT>, kDecThreads, kDecSmem) !=
            cudaSuccess) {
      (void)cudaGetLastError();
      n = 0;
    }
    occ[d & 63] = n > 0 ? n : -1;
  }
  return occ[d & 63];
}

template <int BITS, int NT>
static int dec_launch_t(const DecArgs& a, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(device_sms());
  cfg.blockDim = dim3(kDecThreads);
  cfg.dynamicSmemBytes = kDecSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_check(lmx_counted(cudaLaunchKernelEx(&cfg, decode_fwd_kernel<BITS, NT>, a)), "decode: launch");
}

static int dec_launch(const DecArgs& a, int bits, cudaStream_t st) {
  const bool two = a.R > 8;
  if (bits == 4) return two ? dec_launch_t<4, 2>(a, st) : dec_launch_t<4, 1>(a, st);
  return two ? dec_launch_t<8, 2>(a, st) : dec_launch_t<8, 1>(a, st);
}

static int dec_occupancy_for(int bits, int R) {
  const bool two = R > 8;
  if (bits == 4) return two ? dec_occupancy<4, 2>() : dec_occupancy<4, 1>();
  return two ? dec_occupancy<8, 2>() : dec_occupancy<8, 1>();
}

}  // namespace lmx
