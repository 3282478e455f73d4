// tp.cuh -- tensor-parallel collectives over NVLink peer memory.
//
// Megatron-style split of a decoder across n ranks (one GPU each): q/k/v and
// gate/up are split by output rows (heads, FFN columns), o_proj and down_proj
// by input columns, the lm_head by vocabulary rows.  Two exchanges remain:
//   * after o_proj and down_proj every rank holds a bf16 partial [R, H]; the
//     sum, the residual add and the following RMSNorm are one kernel here
//     (tp_allreduce_norm_kernel), which pulls the peers' partials over NVLink
//     with plain loads and sums them in rank order -- the same result on every
//     rank and for every run, which is what keeps greedy streams reproducible;
//   * the vocab-parallel argmax exchanges one (value, index) pair per row
//     (tp_argmax_exchange_kernel).
//
// Every rank owns one device block, mapped into the peers through CUDA IPC:
//   [slot 0 | slot 1]  partial buffers, bf16 [max_rows][max_hidden] each
//   pairs              argmax (value, index) pairs, [max_rows]
//   flags              [kTpSlots][kTpMaxRanks] u32 arrival epochs
// Barrier slot c (c < kTpArCtas) belongs to CTA c of the all-reduce kernel,
// slot kTpArCtas to the argmax exchange.  Arrival at a slot: one thread bumps
// the local epoch of that slot, stores it (release, system scope) into the
// slot's flag of every peer, then waits (acquire) until each peer's flag in
// its own block has reached the epoch.  Each wait is bounded (2 s of
// %globaltimer); a timeout sets the device error word and the kernel returns
// without touching its outputs.
//
// Reuse: partial slots alternate per exchange.  A rank rewrites slot s only
// two exchanges later, after it passed the barrier of the exchange in
// between, which every peer reaches only once its earlier kernels (the reads
// of slot s included) completed; every kernel here waits on its predecessor
// (griddepcontrol.wait) before it signals.  The pairs buffer is rewritten
// only after at least one all-reduce barrier.
#pragma once
#include "attn.cuh"
#include "lmx_common.cuh"
#include "norm_argmax.cuh"
#include "qmm.cuh"

namespace lmx {

static constexpr int kTpMaxRanks = 8;
static constexpr int kTpArCtas = 128;
static constexpr int kTpSlots = kTpArCtas + 1;
static constexpr int kTpArgSlot = kTpArCtas;
static constexpr uint64_t kTpWaitNs = 2000000000ull;

struct TpPeers {
  int n = 1, rank = 0;
  uint8_t* base[kTpMaxRanks] = {};  // every rank's block (base[rank] is local)
  size_t slot_bytes = 0;            // one partial slot
  size_t pairs_off = 0, flags_off = 0;
  uint32_t* epoch = nullptr;        // local [kTpSlots], never shared
};

LMX_DEV uint32_t* tp_flags(const TpPeers& t, int p) { return reinterpret_cast<uint32_t*>(t.base[p] + t.flags_off); }

LMX_DEV uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
LMX_DEV void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
LMX_DEV uint4 ld_cg16(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
LMX_DEV uint2 ld_cg8(const void* p) {
  uint2 v;
  asm volatile("ld.global.cg.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}

// One thread: arrive at barrier `slot` and wait for every peer (bounded).
LMX_DEV bool tp_barrier(const TpPeers& t, int slot, unsigned* err) {
  const uint32_t e = t.epoch[slot] + 1u;
  t.epoch[slot] = e;
  __threadfence_system();
  for (int p = 0; p < t.n; ++p)
    if (p != t.rank) st_release_sys(tp_flags(t, p) + slot * kTpMaxRanks + t.rank, e);
  const uint32_t* mine = tp_flags(t, t.rank) + slot * kTpMaxRanks;
  const uint64_t t0 = global_ns();
  uint32_t ns = 32;
  for (int p = 0; p < t.n; ++p) {
    if (p == t.rank) continue;
    while ((int32_t)(ld_acquire_sys(mine + p) - e) < 0) {
      __nanosleep(ns);
      if (ns < 512) ns <<= 1;
      if (global_ns() - t0 > kTpWaitNs) {
        if (err) atomicExch(err, 0x71u);
        return false;
      }
    }
  }
  return true;
}

// h[r] = bf16(h[r] + bf16(sum_p partial_p[r]))   (fp32 sum in rank order)
// xn[r] = RMSNorm(h[r]) * w                         (canonical warp order)
// One CTA per row (rows strided over the grid); the row's new h is staged in
// shared memory for the norm.  H % 8 == 0, H <= the comm's max_hidden.
__global__ void __launch_bounds__(256) tp_allreduce_norm_kernel(TpPeers t, int sel, int R, int H, bf16_t* h,
                                                                const bf16_t* w, float eps, bf16_t* xn,
                                                                unsigned* err) {
  extern __shared__ __align__(16) uint8_t tp_smem[];
  bf16_t* srow = reinterpret_cast<bf16_t*>(tp_smem);
  __shared__ int s_ok;
  __shared__ float s_fac;
  grid_wait();
  if (threadIdx.x == 0) s_ok = tp_barrier(t, blockIdx.x, err) ? 1 : 0;
  __syncthreads();
  grid_launch_dependents();
  if (!s_ok) return;
  const int nch = H >> 3, n = t.n;
  const size_t soff = (size_t)sel * t.slot_bytes;
  for (int r = blockIdx.x; r < R; r += gridDim.x) {
    const size_t roff = soff + (size_t)r * H * sizeof(bf16_t);
    for (int c = threadIdx.x; c < nch; c += blockDim.x) {
      uint4 v[kTpMaxRanks];
#pragma unroll
      for (int p = 0; p < kTpMaxRanks; ++p)
        if (p < n) v[p] = ld_cg16(t.base[p] + roff + (size_t)c * 16);
      float s[8];
      unpack8(v[0], s);
#pragma unroll
      for (int p = 1; p < kTpMaxRanks; ++p)
        if (p < n) {
          float x[8];
          unpack8(v[p], x);
#pragma unroll
          for (int e = 0; e < 8; ++e) s[e] = __fadd_rn(s[e], x[e]);
        }
      const uint4 hv = *reinterpret_cast<const uint4*>(h + (size_t)r * H + 8 * c);
      float hf[8];
      unpack8(hv, hf);
#pragma unroll
      for (int e = 0; e < 8; ++e) hf[e] = __fadd_rn(bf2f(f2bf(s[e])), hf[e]);
      const uint4 o = pack8(hf);
      *reinterpret_cast<uint4*>(h + (size_t)r * H + 8 * c) = o;
      *reinterpret_cast<uint4*>(srow + 8 * c) = o;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      const float f = rms_factor_warp(srow, H, eps, threadIdx.x);
      if (threadIdx.x == 0) s_fac = f;
    }
    __syncthreads();
    const float f = s_fac;
    for (int c = threadIdx.x; c < nch; c += blockDim.x) {
      const uint4 xv = *reinterpret_cast<const uint4*>(srow + 8 * c);
      const uint4 wv = *reinterpret_cast<const uint4*>(w + 8 * c);
      const uint32_t xa[4] = {xv.x, xv.y, xv.z, xv.w}, wa[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const bf16_t lo = f2bf(__fmul_rn(__fmul_rn(lo_bf(xa[k]), f), lo_bf(wa[k])));
        const bf16_t hi = f2bf(__fmul_rn(__fmul_rn(hi_bf(xa[k]), f), hi_bf(wa[k])));
        o[k] = (uint32_t)lo | ((uint32_t)hi << 16);
      }
      *reinterpret_cast<uint4*>(xn + (size_t)r * H + 8 * c) = make_uint4(o[0], o[1], o[2], o[3]);
    }
    __syncthreads();
  }
}

// Local half of the vocab-parallel argmax: per row of this rank's logits
// slice [rows][ld] (V valid columns, global index base + j), the best
// (value, index) pair -- a cluster of kArgmaxCluster CTAs per row, lowest
// index winning ties -- stored into this rank's pairs buffer.
__global__ void __launch_bounds__(512) tp_argmax_local_kernel(const bf16_t* logits, int V, int ld, int base,
                                                              uint2* pairs) {
  __shared__ float sv[32];
  __shared__ int si[32];
  __shared__ float cv;
  __shared__ int ci;
  grid_wait();
  grid_launch_dependents();
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank(), cs = (int)cluster.num_blocks();
  const int row = blockIdx.x / cs;
  const int chunk = (V + cs - 1) / cs;
  const int j0 = rank * chunk, j1 = min(V, j0 + chunk);
  const bf16_t* l = logits + (size_t)row * ld;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int j = j0 + threadIdx.x; j < j1; j += blockDim.x) {
    const float v = bf2f(l[j]);
    if (v == v && am_better(v, base + j, bv, bi)) { bv = v; bi = base + j; }
  }
  am_block(bv, bi, sv, si);
  if (threadIdx.x == 0) { cv = bv; ci = bi; }
  cluster.sync();
  if (rank == 0 && threadIdx.x == 0) {
    float rv = cv;
    int ri = ci;
    for (int r = 1; r < cs; ++r) {
      const float ov = *cluster.map_shared_rank(&cv, r);
      const int oi = *cluster.map_shared_rank(&ci, r);
      if (am_better(ov, oi, rv, ri)) { rv = ov; ri = oi; }
    }
    pairs[row] = make_uint2(__float_as_uint(rv), (uint32_t)ri);
  }
  cluster.sync();
}

// Exchange half: after the barrier, every rank reads all ranks' pairs in rank
// order and keeps the best; out[row] = its index (0 if the row had no finite
// logit).  One CTA, one thread per row.
__global__ void __launch_bounds__(1024) tp_argmax_exchange_kernel(TpPeers t, int rows, int32_t* out,
                                                                  unsigned* err) {
  __shared__ int s_ok;
  grid_wait();
  if (threadIdx.x == 0) s_ok = tp_barrier(t, kTpArgSlot, err) ? 1 : 0;
  __syncthreads();
  grid_launch_dependents();
  if (!s_ok) return;
  for (int r = threadIdx.x; r < rows; r += blockDim.x) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int p = 0; p < t.n; ++p) {
      const uint2 q = ld_cg8(reinterpret_cast<const uint2*>(t.base[p] + t.pairs_off) + r);
      const float v = __uint_as_float(q.x);
      const int i = (int)q.y;
      if (am_better(v, i, bv, bi)) { bv = v; bi = i; }
    }
    out[r] = bi == 0x7fffffff ? 0 : bi;
  }
}

// Expert parallelism: the combine of the routed experts across ranks.  Rank
// p wrote the bf16 down output of every slot whose expert it holds (experts
// [p*per, (p+1)*per)) into its partial slot `sel` as [M][k][H]; after the
// barrier every rank forms y[m] = bf16(fma chain over slots j in order of
// w[m][j] * v[m][j]), pulling v from the slot's owner over NVLink -- the
// single-GPU moe_down_kernel's order, so every rank and every rank count
// computes the same bits.  One CTA per row (rows strided), 8 outputs per
// thread, 16-byte L2 loads.
__global__ void __launch_bounds__(256) ep_combine_kernel(TpPeers t, int sel, int M, int k, int H, const int32_t* idx,
                                                         const float* w, int per, bf16_t* y, unsigned* err) {
  __shared__ int s_ok;
  grid_wait();
  if (threadIdx.x == 0) s_ok = tp_barrier(t, blockIdx.x, err) ? 1 : 0;
  __syncthreads();
  grid_launch_dependents();
  if (!s_ok) return;
  const size_t soff = (size_t)sel * t.slot_bytes;
  for (int m = blockIdx.x; m < M; m += gridDim.x) {
    for (int c = threadIdx.x; c < H / 8; c += blockDim.x) {
      float acc[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = 0.0f;
      for (int j = 0; j < k; ++j) {
        const int ex = idx[(size_t)m * k + j];
        const int owner = min(max(ex, 0) / per, t.n - 1);
        const uint4 v = ld_cg16(t.base[owner] + soff + (((size_t)m * k + j) * H + 8 * c) * sizeof(bf16_t));
        float x[8];
        unpack8(v, x);
        const float wj = w[(size_t)m * k + j];
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = __fmaf_rn(wj, x[e], acc[e]);
      }
      *reinterpret_cast<uint4*>(y + (size_t)m * H + 8 * c) = pack8(acc);
    }
  }
}

}  // namespace lmx
