// sample.cuh -- K3: temperature / top-p sampling and speculative rejection
// sampling (Leviathan et al. 2023; Chen et al. 2023) in exact integer
// arithmetic, one thread-block cluster of kSampCluster CTAs per sequence.
//
// The reference samples with mx::random::categorical (Gumbel noise from
// MLX's RNG, src/common/generate.cpp:83-120) and has no rejection sampler;
// here both the draft and the acceptance consume caller-side Philox uniforms
// and every decision is an integer comparison, so the result is identical to
// any implementation of the same rule (oracle/oracle.cpp make_dist /
// draw_dist / orc_accept_stochastic):
//   w_j  = rint(exp((l_j - max) * (1/T)) * 2^32)                (uint64)
//   top-p: smallest prefix in (w desc, index asc) order with
//          2^24 * mass >= rint(top_p * 2^24) * Z
//   draw:  smallest index t with 2^24 * cumsum_t(kept w) > u24 * Z_kept
//   accept d iff u24 * q(d) * Zp < 2^24 * p(d) * Zq; on rejection draw from
//   r_j = max(0, p_j Zq - q_j Zp); after K acceptances draw from p_K.
//
// Work split: CTA rank r of the cluster owns the index slice [v0, v1) of the
// row; inside it, thread t owns a contiguous chunk, so (rank, thread) order
// is index order.  Reductions and exclusive scans run per CTA, then across
// the cluster: each CTA publishes its block result in one of two alternating
// shared slots, one cluster barrier, and every CTA combines the ranks' values
// in rank order through distributed shared memory (all CTAs hold identical
// results afterwards, so they take identical control flow).
#pragma once
#include <cooperative_groups.h>

#include "lmx_common.cuh"

namespace lmx {

typedef unsigned __int128 u128;
static constexpr int kSampThreads = 1024;
static constexpr int kSampCluster = 8;

struct Dist {
  float mx, inv_t;
  int topp;
  uint64_t Z;        // total mass
  uint64_t tau;      // top-p threshold weight
  uint64_t mass_gt;  // mass of weights > tau
  uint64_t kties;    // tokens with weight == tau kept (lowest indices)
  uint64_t Zk;       // kept mass
};

struct SampScratch {
  float fred[32];
  uint64_t ured[32];
  uint64_t tscan[32];  // warp totals of the block scans
  u128 mscan[32];
  uint64_t tscan2[32];
  uint64_t hmass[2048];  // this CTA's radix histogram (mass per bucket)
  uint64_t tmass[2048];  // the cluster's histogram
  float xf[2];           // cluster exchange slots (alternating)
  uint64_t xu[2];
  u128 xw[2];
  int xi[2], xj[2];
  int selb;        // radix level result: bucket and the mass above it
  uint64_t sela;
};

// Cluster context of one row: rank, size, slice, exchange-slot counter.
struct Cl {
  int rank, cs, v0, v1, gen;
};

LMX_DEV Cl cl_make(int V) {
  namespace cg = cooperative_groups;
  Cl c;
  cg::cluster_group cl = cg::this_cluster();
  c.rank = (int)cl.block_rank();
  c.cs = (int)cl.num_blocks();
  const int per = (V + c.cs - 1) / c.cs;
  c.v0 = min(V, c.rank * per);
  c.v1 = min(V, c.v0 + per);
  c.gen = 0;
  return c;
}

LMX_DEV void cl_sync() { cooperative_groups::this_cluster().sync(); }

template <typename T>
LMX_DEV T* cl_peer(T* p, int rank) {
  return cooperative_groups::this_cluster().map_shared_rank(p, rank);
}

// A row of logits as a CTA reads it: its own slice [v0, v1) staged once in
// shared memory (every pass over the slice reads it from there), any other
// index from global memory.
struct Row {
  const bf16_t* g;
  const bf16_t* s;
  int v0, v1;
};

LMX_DEV float row_at(const Row& r, int j) { return bf2f(j >= r.v0 && j < r.v1 ? r.s[j - r.v0] : r.g[j]); }

// Bytes of shared memory for `n` staged row slices of a V-wide row.
__host__ __device__ inline size_t samp_row_bytes(int V, int n) {
  const size_t per = (size_t)(V + kSampCluster - 1) / kSampCluster;
  return ((per * 2 + 15) / 16 * 16) * (size_t)n;
}

// Stage this CTA's slice of row g into s (every load of a batch in flight
// before the stores); a barrier before (the previous row in s may still be
// read) and after.
LMX_DEV Row stage_row(const bf16_t* g, bf16_t* s, const Cl& c) {
  constexpr int U = 20;
  const int n = c.v1 - c.v0;
  __syncthreads();
  for (int base = 0; base < n; base += U * kSampThreads) {
    uint16_t r[U];
#pragma unroll
    for (int i = 0; i < U; ++i) {
      const int k = base + (int)threadIdx.x + i * kSampThreads;
      r[i] = k < n ? reinterpret_cast<const uint16_t*>(g)[c.v0 + k] : (uint16_t)0;
    }
#pragma unroll
    for (int i = 0; i < U; ++i) {
      const int k = base + (int)threadIdx.x + i * kSampThreads;
      if (k < n) reinterpret_cast<uint16_t*>(s)[k] = r[i];
    }
  }
  __syncthreads();
  Row row;
  row.g = g;
  row.s = s;
  row.v0 = c.v0;
  row.v1 = c.v1;
  return row;
}

LMX_DEV uint64_t dist_w(const Row& l, int j, float mx, float inv_t) {
  const float v = row_at(l, j);
  if (v != v) return 0;
  const float e = exp_c(__fmul_rn(__fsub_rn(v, mx), inv_t));
  return __float2ull_rn(__fmul_rn(e, 4294967296.0f));
}

LMX_DEV float block_max(float v, SampScratch& sm) {
  for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sm.fred[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = sm.fred[0];
  for (int i = 1; i < kSampThreads / 32; ++i) r = fmaxf(r, sm.fred[i]);
  return r;
}

LMX_DEV uint64_t block_sum64(uint64_t v, SampScratch& sm) {
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sm.ured[threadIdx.x >> 5] = v;
  __syncthreads();
  uint64_t r = 0;
  for (int i = 0; i < kSampThreads / 32; ++i) r += sm.ured[i];
  return r;
}

// Exclusive prefix over threads in thread order: warp shuffle scans plus a
// 32-entry table of warp totals.
LMX_DEV uint64_t shfl_up64(uint64_t v, int d) {
  const uint32_t lo = __shfl_up_sync(0xffffffffu, (uint32_t)v, d);
  const uint32_t hi = __shfl_up_sync(0xffffffffu, (uint32_t)(v >> 32), d);
  return ((uint64_t)hi << 32) | lo;
}
LMX_DEV u128 shfl_up128(u128 v, int d) {
  return ((u128)shfl_up64((uint64_t)(v >> 64), d) << 64) | shfl_up64((uint64_t)v, d);
}

LMX_DEV uint64_t block_exscan64(uint64_t v, uint64_t* wt /* [32] */, uint64_t* total = nullptr) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint64_t inc = v;
  for (int d = 1; d < 32; d <<= 1) {
    const uint64_t t = shfl_up64(inc, d);
    if (lane >= d) inc += t;
  }
  __syncthreads();
  if (lane == 31) wt[warp] = inc;
  __syncthreads();
  uint64_t base = 0, all = 0;
  for (int w = 0; w < kSampThreads / 32; ++w) {
    if (w < warp) base += wt[w];
    all += wt[w];
  }
  __syncthreads();
  if (total) *total = all;
  return base + inc - v;
}

LMX_DEV u128 block_exscan128(u128 v, u128* wt /* [32] */, u128* total = nullptr) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  u128 inc = v;
  for (int d = 1; d < 32; d <<= 1) {
    const u128 t = shfl_up128(inc, d);
    if (lane >= d) inc += t;
  }
  __syncthreads();
  if (lane == 31) wt[warp] = inc;
  __syncthreads();
  u128 base = 0, all = 0;
  for (int w = 0; w < kSampThreads / 32; ++w) {
    if (w < warp) base += wt[w];
    all += wt[w];
  }
  __syncthreads();
  if (total) *total = all;
  return base + inc - v;
}

// ---- cluster reductions (identical result in every CTA) ----
LMX_DEV float cl_max(float v, Cl& c, SampScratch& sm) {
  const float m = block_max(v, sm);
  const int slot = c.gen++ & 1;
  if (threadIdx.x == 0) sm.xf[slot] = m;
  cl_sync();
  float r = -INFINITY;
  for (int k = 0; k < c.cs; ++k) r = fmaxf(r, *cl_peer(&sm.xf[slot], k));
  return r;
}

LMX_DEV uint64_t cl_sum64(uint64_t v, Cl& c, SampScratch& sm) {
  const uint64_t s = block_sum64(v, sm);
  const int slot = c.gen++ & 1;
  if (threadIdx.x == 0) sm.xu[slot] = s;
  cl_sync();
  uint64_t r = 0;
  for (int k = 0; k < c.cs; ++k) r += *cl_peer(&sm.xu[slot], k);
  return r;
}

// Exclusive prefix in index order across the whole row; *total = row sum.
LMX_DEV uint64_t cl_exscan64(uint64_t v, Cl& c, SampScratch& sm, uint64_t* wt, uint64_t* total = nullptr) {
  uint64_t bt;
  const uint64_t pre = block_exscan64(v, wt, &bt);
  const int slot = c.gen++ & 1;
  if (threadIdx.x == 0) sm.xu[slot] = bt;
  cl_sync();
  uint64_t base = 0, all = 0;
  for (int k = 0; k < c.cs; ++k) {
    const uint64_t t = *cl_peer(&sm.xu[slot], k);
    if (k < c.rank) base += t;
    all += t;
  }
  if (total) *total = all;
  return base + pre;
}

LMX_DEV u128 cl_exscan128(u128 v, Cl& c, SampScratch& sm, u128* total) {
  u128 bt;
  const u128 pre = block_exscan128(v, sm.mscan, &bt);
  const int slot = c.gen++ & 1;
  if (threadIdx.x == 0) sm.xw[slot] = bt;
  cl_sync();
  u128 base = 0, all = 0;
  for (int k = 0; k < c.cs; ++k) {
    const u128 t = *cl_peer(&sm.xw[slot], k);
    if (k < c.rank) base += t;
    all += t;
  }
  *total = all;
  return base + pre;
}

// One index per row found by at most one thread of the cluster (`mine` >= 0
// there, -1 elsewhere), returned in every CTA; when no thread found one, the
// largest `fall` over the row (-1 if none).
LMX_DEV int cl_pick(int mine, int fall, Cl& c, SampScratch& sm) {
  const int slot = c.gen++ & 1;
  __syncthreads();
  if (threadIdx.x == 0) {
    sm.xi[slot] = -1;
    sm.xj[slot] = -1;
  }
  __syncthreads();
  if (mine >= 0) sm.xi[slot] = mine;
  if (fall >= 0) atomicMax(&sm.xj[slot], fall);
  cl_sync();
  int hit = -1, fb = -1;
  for (int k = 0; k < c.cs; ++k) {
    hit = max(hit, *cl_peer(&sm.xi[slot], k));
    fb = max(fb, *cl_peer(&sm.xj[slot], k));
  }
  return hit >= 0 ? hit : fb;
}

// Build the (temperature, top-p) distribution of one logits row.
LMX_DEV void make_dist_dev(const Row& l, int V, float temperature, float top_p, Dist& D, Cl& c,
                           SampScratch& sm) {
  const int tid = threadIdx.x;
  float mx = -INFINITY;
  for (int j = c.v0 + tid; j < c.v1; j += kSampThreads) {
    const float v = row_at(l, j);
    if (v == v) mx = fmaxf(mx, v);
  }
  D.mx = cl_max(mx, c, sm);
  D.inv_t = __fdiv_rn(1.0f, temperature);
  uint64_t z = 0;
  for (int j = c.v0 + tid; j < c.v1; j += kSampThreads) z += dist_w(l, j, D.mx, D.inv_t);
  D.Z = cl_sum64(z, c, sm);
  D.topp = top_p > 0.0f && top_p < 1.0f;
  if (!D.topp) {
    D.tau = 0;
    D.mass_gt = 0;
    D.kties = 0;
    D.Zk = D.Z;
    return;
  }
  const uint64_t P24 = __float2ull_rn(__fmul_rn(top_p, 16777216.0f));
  const u128 target = (u128)P24 * D.Z;  // keep until 2^24 * mass >= target
  // radix select over the 33-bit weights, 11 bits per level, high to low
  uint64_t prefix = 0, above = 0;
  for (int level = 0; level < 3; ++level) {
    const int shift = 22 - 11 * level;
    for (int i = tid; i < 2048; i += kSampThreads) sm.hmass[i] = 0;
    __syncthreads();
    // warp-aggregated updates: lanes hitting the same bucket are grouped with
    // match_any; the group's mass is summed exactly as two 16-bit-split halves
    // (each < 2^22 over 32 lanes) and one lane issues the atomic, so the few
    // buckets holding most tokens see one update per warp, not 32
    for (int base = c.v0; base < c.v1; base += kSampThreads) {
      const int j = base + tid;
      int bkt = -1;
      uint64_t w = 0;
      if (j < c.v1) {
        w = dist_w(l, j, D.mx, D.inv_t);
        if ((w >> (shift + 11)) == (prefix >> (shift + 11)))  // level 0: every w < 2^33 matches
          bkt = (int)((w >> shift) & 2047u);
      }
      const unsigned peers = __match_any_sync(0xffffffffu, bkt);
      if (bkt >= 0) {
        const unsigned hi = __reduce_add_sync(peers, (unsigned)(w >> 16));
        const unsigned lo = __reduce_add_sync(peers, (unsigned)(w & 0xFFFFu));
        if ((int)(tid & 31) == __ffs(peers) - 1)
          atomicAdd((unsigned long long*)&sm.hmass[bkt], ((unsigned long long)hi << 16) + lo);
      }
    }
    cl_sync();  // every CTA's histogram complete
    for (int i = tid; i < 2048; i += kSampThreads) {
      uint64_t m = 0;
      for (int k = 0; k < c.cs; ++k) m += cl_peer(sm.hmass, k)[i];
      sm.tmass[i] = m;
    }
    cl_sync();  // peers done reading this CTA's histogram (it is reset next level)
    // Largest bucket b in [0, 2047] whose suffix mass (from 2047 down to b,
    // plus `above`) reaches the target, else 0; acc = above + the mass of the
    // buckets above b.  Thread t owns buckets 2047 - 2t and 2046 - 2t.
    const int bh = 2047 - 2 * tid, bl = bh - 1;
    const uint64_t mh = sm.tmass[bh], ml = sm.tmass[bl];
    uint64_t tot;
    const uint64_t ex = block_exscan64(mh + ml, sm.tscan, &tot);  // mass of buckets > bh
    const uint64_t sh = ex + mh, sl = sh + ml;                    // suffix sums from bh, bl
    const bool ph = ((u128)(above + sh) << 24) >= target, pl = ((u128)(above + sl) << 24) >= target;
    const bool pabove = ((u128)(above + ex) << 24) >= target;   // predicate at bucket bh + 1
    if (tid == 0) {
      sm.selb = 0;
      sm.sela = above + (tot - sm.tmass[0]);  // b = 0: everything above bucket 0
    }
    __syncthreads();
    if (ph && (bh == 2047 || !pabove)) {
      sm.selb = bh;
      sm.sela = above + ex;
    } else if (pl && !ph && bl >= 1) {
      sm.selb = bl;
      sm.sela = above + sh;
    }
    __syncthreads();
    prefix |= (uint64_t)sm.selb << shift;
    above = sm.sela;
    __syncthreads();
  }
  D.tau = prefix;
  D.mass_gt = above;
  const u128 need = target - ((u128)above << 24);  // > 0
  const u128 per = (u128)D.tau << 24;
  D.kties = per ? (uint64_t)((need + per - 1) / per) : 0;
  D.Zk = above + D.kties * D.tau;
}

LMX_DEV bool kept_w(const Dist& D, uint64_t w, uint64_t tie_rank) {
  return !D.topp || w > D.tau || (w == D.tau && tie_rank < D.kties);
}

// Index range [c0, c1) of this thread's contiguous chunk of the CTA's slice.
LMX_DEV void chunk_of(const Cl& c, int& c0, int& c1) {
  const int n = c.v1 - c.v0;
  const int per = (n + kSampThreads - 1) / kSampThreads;
  c0 = min(c.v1, c.v0 + (int)threadIdx.x * per);
  c1 = min(c.v1, c0 + per);
}

// Exclusive count of weight-tau ties before each thread's chunk (row order).
LMX_DEV uint64_t tie_prefix(const Row& l, const Dist& D, Cl& c, SampScratch& sm, uint64_t* buf) {
  int c0, c1;
  chunk_of(c, c0, c1);
  uint64_t n = 0;
  if (D.topp)
    for (int j = c0; j < c1; ++j) n += dist_w(l, j, D.mx, D.inv_t) == D.tau;
  return cl_exscan64(n, c, sm, buf);
}

// Draw by inverse CDF over kept weights in index order.
LMX_DEV int draw_dev(const Row& l, const Dist& D, uint32_t u24, Cl& c, SampScratch& sm) {
  int c0, c1;
  chunk_of(c, c0, c1);
  uint64_t ties = tie_prefix(l, D, c, sm, sm.tscan);
  uint64_t local = 0, tr = ties;
  int last = -1;
  for (int j = c0; j < c1; ++j) {
    const uint64_t w = dist_w(l, j, D.mx, D.inv_t);
    const bool k = kept_w(D, w, tr);
    if (D.topp && w == D.tau) ++tr;
    if (k && w) {
      local += w;
      last = j;
    }
  }
  const uint64_t pre = cl_exscan64(local, c, sm, sm.tscan2);
  const u128 target = (u128)u24 * D.Zk;
  int mine = -1;
  // the crossing lies in this thread's chunk iff 2^24*pre <= target < 2^24*(pre+local)
  if (local && ((u128)pre << 24) <= target && ((u128)(pre + local) << 24) > target) {
    uint64_t cum = pre;
    tr = ties;
    for (int j = c0; j < c1; ++j) {
      const uint64_t w = dist_w(l, j, D.mx, D.inv_t);
      const bool k = kept_w(D, w, tr);
      if (D.topp && w == D.tau) ++tr;
      if (!k || !w) continue;
      cum += w;
      if (((u128)cum << 24) > target) {
        mine = j;
        break;
      }
    }
  }
  // unreachable for a consistent distribution: the last kept positive token
  const int r = cl_pick(mine, last, c, sm);
  return r < 0 ? 0 : r;
}

// Kept weight of token d (0 if outside the top-p set).
LMX_DEV uint64_t kept_weight_of(const Row& l, const Dist& D, int d, Cl& c, SampScratch& sm) {
  const uint64_t w = dist_w(l, d, D.mx, D.inv_t);
  if (!D.topp || w > D.tau) return w;
  if (w < D.tau) return 0;
  uint64_t n = 0;
  for (int j = c.v0 + threadIdx.x; j < min(c.v1, d); j += kSampThreads) n += dist_w(l, j, D.mx, D.inv_t) == D.tau;
  n = cl_sum64(n, c, sm);
  return n < D.kties ? w : 0;
}

// Residual draw r_j = max(0, p_j Zq - q_j Zp) by inverse CDF with u24;
// returns -1 if R == 0.
LMX_DEV int residual_draw_dev(const Row& lp, const Dist& P, const Row& lq, const Dist& Q, uint32_t u24,
                              Cl& c, SampScratch& sm) {
  int c0, c1;
  chunk_of(c, c0, c1);
  const uint64_t tp = tie_prefix(lp, P, c, sm, sm.tscan);
  const uint64_t tq = tie_prefix(lq, Q, c, sm, sm.tscan2);
  u128 local = 0;
  uint64_t rp = tp, rq = tq;
  for (int j = c0; j < c1; ++j) {
    const uint64_t wp = dist_w(lp, j, P.mx, P.inv_t), wq = dist_w(lq, j, Q.mx, Q.inv_t);
    const bool kp = kept_w(P, wp, rp), kq = kept_w(Q, wq, rq);
    if (P.topp && wp == P.tau) ++rp;
    if (Q.topp && wq == Q.tau) ++rq;
    const u128 a = kp ? (u128)wp * Q.Zk : 0, b = kq ? (u128)wq * P.Zk : 0;
    if (a > b) local += a - b;
  }
  u128 R;
  const u128 pre = cl_exscan128(local, c, sm, &R);
  if (R == 0) return -1;
  const u128 target = (u128)u24 * R;
  int mine = -1;
  if (local && (pre << 24) <= target && ((pre + local) << 24) > target) {
    u128 cum = pre;
    rp = tp;
    rq = tq;
    for (int j = c0; j < c1; ++j) {
      const uint64_t wp = dist_w(lp, j, P.mx, P.inv_t), wq = dist_w(lq, j, Q.mx, Q.inv_t);
      const bool kp = kept_w(P, wp, rp), kq = kept_w(Q, wq, rq);
      if (P.topp && wp == P.tau) ++rp;
      if (Q.topp && wq == Q.tau) ++rq;
      const u128 a = kp ? (u128)wp * Q.Zk : 0, b = kq ? (u128)wq * P.Zk : 0;
      if (a <= b) continue;
      cum += a - b;
      if ((cum << 24) > target) {
        mine = j;
        break;
      }
    }
  }
  return cl_pick(mine, -1, c, sm);
}

// ---------------------------------------------------------------------------
// kernels (grid = rows x kSampCluster, cluster = kSampCluster, block = 1024)
// ---------------------------------------------------------------------------
struct StochParams {
  float temperature, top_p;
  uint64_t seed;
  uint32_t seq_base = 0;  // global id of row 0: uniforms are keyed by global sequence
};

// Cluster launch of a sampling kernel over `rows` rows, with programmatic
// dependent launch like every other kernel of the library.
// nrow: row slices staged at once (2 for the acceptance kernels).
template <typename Kern, typename... Args>
static inline cudaError_t samp_launch(Kern kern, int rows, int V, int nrow, cudaStream_t st, Args... args) {
  const size_t dyn = samp_row_bytes(V, nrow);
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, size_t> set;  // (kernel, device) -> bytes allowed
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    size_t& have = set[{(const void*)kern, dev}];
    // static scratch + staged rows may exceed the 48 KB default: always
    // raise the kernel's dynamic limit to what this launch needs
    if (dyn > have) {
      const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn);
      if (e != cudaSuccess) return e;
      have = dyn;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(rows * kSampCluster);
  cfg.blockDim = dim3(kSampThreads);
  cfg.dynamicSmemBytes = dyn;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = kSampCluster;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return lmx_counted(cudaLaunchKernelEx(&cfg, kern, args...));
}

LMX_DEV bool cl_lead(const Cl& c) { return c.rank == 0 && threadIdx.x == 0; }

// Sample one token per row from logits [rows][ld] with uniform
// (seed, row, step, slot, stream); writes out[row].
__global__ void __launch_bounds__(kSampThreads) sample_rows_kernel(const bf16_t* logits, int ld, int V,
                                                                   StochParams sp, uint32_t step,
                                                                   uint32_t slot, uint32_t stream,
                                                                   int32_t* out) {
  __shared__ SampScratch sm;
  extern __shared__ __align__(128) uint8_t smem[];
  grid_wait();
  grid_launch_dependents();
  const int b = blockIdx.x / kSampCluster;
  Cl c = cl_make(V);
  const Row l = stage_row(logits + (size_t)b * ld, reinterpret_cast<bf16_t*>(smem), c);
  Dist D;
  make_dist_dev(l, V, sp.temperature, sp.top_p, D, c, sm);
  const int t = draw_dev(l, D, uniform24(sp.seed, sp.seq_base + b, step, slot, stream), c, sm);
  if (cl_lead(c)) out[b] = t;
  cl_sync();
}

}  // namespace lmx

#include "engine_kernels.cuh"

namespace lmx {

// Draft token i of every sequence, drawn from q_i = dist(draft logits):
// uniform (seed, b, step_b, i, 0).  Bookkeeping as draft_argmax_kernel.
__global__ void __launch_bounds__(kSampThreads) draft_sample_kernel(const bf16_t* qlog, int V, SpecState s,
                                                                    StochParams sp, int i, int adv) {
  __shared__ SampScratch sm;
  extern __shared__ __align__(128) uint8_t smem[];
  grid_wait();
  grid_launch_dependents();
  const int b = blockIdx.x / kSampCluster;
  Cl c = cl_make(V);
  const Row l = stage_row(qlog + ((size_t)b * s.K + i) * V, reinterpret_cast<bf16_t*>(smem), c);
  Dist D;
  make_dist_dev(l, V, sp.temperature, sp.top_p, D, c, sm);
  const int tok = draw_dev(l, D, uniform24(sp.seed, sp.seq_base + b, (uint32_t)s.ustep[b], i, 0), c, sm);
  if (cl_lead(c)) {
    s.drafts[b * s.K + i] = tok;
    if (s.emitted[b] < s.max_tokens) s.dlen[b] += adv;
    if (i == s.K - 1) {
      s.vt[b * (s.K + 1)] = s.tok2[2 * b + 1];
      for (int k = 0; k < s.K; ++k) s.vt[b * (s.K + 1) + 1 + k] = s.drafts[b * s.K + k];
    }
  }
  cl_sync();
}

// Rejection sampling against the verify pass (target logits [B][K+1][V]) and
// the stored draft logits, then commit / rollback (commit_step).  Uniforms:
// accept test i -> (b, step, i, 1), residual / bonus draw -> (b, step, 0, 2).
__global__ void __launch_bounds__(kSampThreads) accept_stochastic_kernel(const bf16_t* tlog, int V, SpecState s,
                                                                         StochParams sp) {
  __shared__ SampScratch sm;
  extern __shared__ __align__(128) uint8_t smem[];
  bf16_t* rp_s = reinterpret_cast<bf16_t*>(smem);
  bf16_t* rq_s = reinterpret_cast<bf16_t*>(smem + samp_row_bytes(V, 1));
  grid_wait();
  grid_launch_dependents();
  const int b = blockIdx.x / kSampCluster, K = s.K;
  Cl c = cl_make(V);
  const uint32_t step = (uint32_t)s.ustep[b];
  const bool finished = s.emitted[b] >= s.max_tokens;
  cl_sync();  // every CTA has read the step counter before it advances
  if (cl_lead(c)) s.ustep[b] = (int)step + 1;
  if (finished) {  // frozen
    if (cl_lead(c)) s.dlen[b] = s.tlen[b] - 1;
    cl_sync();
    return;
  }
  const uint32_t uf = uniform24(sp.seed, sp.seq_base + b, step, 0, 2);
  int acc = K, next = -1;
  for (int i = 0; i < K; ++i) {
    const Row lp = stage_row(tlog + ((size_t)b * (K + 1) + i) * V, rp_s, c);
    const Row lq = stage_row(s.qlog + ((size_t)b * K + i) * V, rq_s, c);
    Dist P, Q;
    make_dist_dev(lp, V, sp.temperature, sp.top_p, P, c, sm);
    make_dist_dev(lq, V, sp.temperature, sp.top_p, Q, c, sm);
    const int d = s.drafts[b * K + i];
    const uint64_t pd = kept_weight_of(lp, P, d, c, sm), qd = kept_weight_of(lq, Q, d, c, sm);
    const uint32_t ua = uniform24(sp.seed, sp.seq_base + b, step, i, 1);
    if ((u128)ua * qd * P.Zk < (((u128)pd * Q.Zk) << 24)) continue;
    acc = i;
    next = residual_draw_dev(lp, P, lq, Q, uf, c, sm);
    if (next < 0) next = draw_dev(lp, P, uf, c, sm);
    break;
  }
  if (acc == K) {
    const Row lp = stage_row(tlog + ((size_t)b * (K + 1) + K) * V, rp_s, c);
    Dist P;
    make_dist_dev(lp, V, sp.temperature, sp.top_p, P, c, sm);
    next = draw_dev(lp, P, uf, c, sm);
  }
  if (cl_lead(c)) commit_step(s, b, acc, next);
  cl_sync();
}

}  // namespace lmx

namespace lmx {

// Standalone forms with caller-supplied 24-bit uniforms (the C-ABI ops).
__global__ void __launch_bounds__(kSampThreads) sample_u_kernel(const bf16_t* logits, int V, float temperature,
                                                                float top_p, const uint32_t* u24, int32_t* out) {
  __shared__ SampScratch sm;
  extern __shared__ __align__(128) uint8_t smem[];
  grid_wait();
  grid_launch_dependents();
  const int b = blockIdx.x / kSampCluster;
  Cl c = cl_make(V);
  const Row l = stage_row(logits + (size_t)b * V, reinterpret_cast<bf16_t*>(smem), c);
  Dist D;
  make_dist_dev(l, V, temperature, top_p, D, c, sm);
  const int t = draw_dev(l, D, u24[b] & 0xFFFFFFu, c, sm);
  if (cl_lead(c)) out[b] = t;
  cl_sync();
}

__global__ void __launch_bounds__(kSampThreads) accept_u_kernel(const bf16_t* tlog, const bf16_t* qlog,
                                                                const int32_t* drafts, int K, int V,
                                                                float temperature, float top_p,
                                                                const uint32_t* u_accept, const uint32_t* u_final,
                                                                int32_t* n_accepted, int32_t* out_tokens) {
  __shared__ SampScratch sm;
  extern __shared__ __align__(128) uint8_t smem[];
  bf16_t* rp_s = reinterpret_cast<bf16_t*>(smem);
  bf16_t* rq_s = reinterpret_cast<bf16_t*>(smem + samp_row_bytes(V, 1));
  grid_wait();
  grid_launch_dependents();
  const int b = blockIdx.x / kSampCluster;
  Cl c = cl_make(V);
  const uint32_t uf = u_final[b] & 0xFFFFFFu;
  int acc = K, next = -1;
  for (int i = 0; i < K; ++i) {
    const Row lp = stage_row(tlog + ((size_t)b * (K + 1) + i) * V, rp_s, c);
    const Row lq = stage_row(qlog + ((size_t)b * K + i) * V, rq_s, c);
    Dist P, Q;
    make_dist_dev(lp, V, temperature, top_p, P, c, sm);
    make_dist_dev(lq, V, temperature, top_p, Q, c, sm);
    const int d = drafts[b * K + i];
    const uint64_t pd = kept_weight_of(lp, P, d, c, sm), qd = kept_weight_of(lq, Q, d, c, sm);
    const uint32_t ua = u_accept[b * K + i] & 0xFFFFFFu;
    if ((u128)ua * qd * P.Zk < (((u128)pd * Q.Zk) << 24)) {
      if (cl_lead(c)) out_tokens[b * (K + 1) + i] = d;
      continue;
    }
    acc = i;
    next = residual_draw_dev(lp, P, lq, Q, uf, c, sm);
    if (next < 0) next = draw_dev(lp, P, uf, c, sm);
    break;
  }
  if (acc == K) {
    const Row lp = stage_row(tlog + ((size_t)b * (K + 1) + K) * V, rp_s, c);
    Dist P;
    make_dist_dev(lp, V, temperature, top_p, P, c, sm);
    next = draw_dev(lp, P, uf, c, sm);
  }
  if (cl_lead(c)) {
    out_tokens[b * (K + 1) + acc] = next;
    n_accepted[b] = acc;
  }
  cl_sync();
}

}  // namespace lmx
