// sample.cuh -- K3: temperature / top-p sampling and speculative rejection
// sampling (Leviathan et al. 2023; Chen et al. 2023) in exact integer
// arithmetic, one 1024-thread CTA per sequence.
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
#pragma once
#include "lmx_common.cuh"

namespace lmx {

typedef unsigned __int128 u128;
static constexpr int kSampThreads = 1024;

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
  u128 wred[32];
  uint32_t hcnt[2048];
  uint64_t hmass[2048];
  uint64_t tscan[32];   // warp totals of the block scans
  u128 mscan[32];
  uint64_t tscan2[32];
  int result;
};

LMX_DEV uint64_t dist_w(const bf16_t* l, int j, float mx, float inv_t) {
  const float v = bf2f(l[j]);
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

// Exclusive prefix over threads in thread order (= index order of the
// contiguous chunks): warp shuffle scans plus a 32-entry table of warp totals.
LMX_DEV uint64_t shfl_up64(uint64_t v, int d) {
  const uint32_t lo = __shfl_up_sync(0xffffffffu, (uint32_t)v, d);
  const uint32_t hi = __shfl_up_sync(0xffffffffu, (uint32_t)(v >> 32), d);
  return ((uint64_t)hi << 32) | lo;
}
LMX_DEV u128 shfl_up128(u128 v, int d) {
  return ((u128)shfl_up64((uint64_t)(v >> 64), d) << 64) | shfl_up64((uint64_t)v, d);
}

LMX_DEV uint64_t block_exscan64(uint64_t v, uint64_t* wt /* [32] */) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint64_t inc = v;
  for (int d = 1; d < 32; d <<= 1) {
    const uint64_t t = shfl_up64(inc, d);
    if (lane >= d) inc += t;
  }
  __syncthreads();
  if (lane == 31) wt[warp] = inc;
  __syncthreads();
  uint64_t base = 0;
  for (int w = 0; w < warp; ++w) base += wt[w];
  __syncthreads();
  return base + inc - v;
}

LMX_DEV u128 block_exscan128(u128 v, u128* wt /* [32] */) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  u128 inc = v;
  for (int d = 1; d < 32; d <<= 1) {
    const u128 t = shfl_up128(inc, d);
    if (lane >= d) inc += t;
  }
  __syncthreads();
  if (lane == 31) wt[warp] = inc;
  __syncthreads();
  u128 base = 0;
  for (int w = 0; w < warp; ++w) base += wt[w];
  __syncthreads();
  return base + inc - v;
}

// Build the (temperature, top-p) distribution of one logits row.
LMX_DEV void make_dist_dev(const bf16_t* l, int V, float temperature, float top_p, Dist& D, SampScratch& sm) {
  const int tid = threadIdx.x;
  float mx = -INFINITY;
  for (int j = tid; j < V; j += kSampThreads) {
    const float v = bf2f(l[j]);
    if (v == v) mx = fmaxf(mx, v);
  }
  D.mx = block_max(mx, sm);
  D.inv_t = __fdiv_rn(1.0f, temperature);
  uint64_t z = 0;
  for (int j = tid; j < V; j += kSampThreads) z += dist_w(l, j, D.mx, D.inv_t);
  D.Z = block_sum64(z, sm);
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
    __syncthreads();
    for (int i = tid; i < 2048; i += kSampThreads) { sm.hcnt[i] = 0; sm.hmass[i] = 0; }
    __syncthreads();
    for (int j = tid; j < V; j += kSampThreads) {
      const uint64_t w = dist_w(l, j, D.mx, D.inv_t);
      if ((w >> (shift + 11)) == (prefix >> (shift + 11))) {  // level 0: every w < 2^33 matches
        const int bkt = (int)((w >> shift) & 2047u);
        atomicAdd(&sm.hcnt[bkt], 1u);
        atomicAdd((unsigned long long*)&sm.hmass[bkt], (unsigned long long)w);
      }
    }
    __syncthreads();
    if (tid == 0) {
      int b = 2047;
      uint64_t acc = above;
      for (; b > 0; --b) {
        if (((u128)(acc + sm.hmass[b]) << 24) >= target) break;
        acc += sm.hmass[b];
      }
      sm.result = b;
      sm.ured[0] = acc;
    }
    __syncthreads();
    prefix |= (uint64_t)sm.result << shift;
    above = sm.ured[0];
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

// Index range [c0, c1) of this thread's contiguous chunk.
LMX_DEV void chunk_of(int V, int& c0, int& c1) {
  const int per = (V + kSampThreads - 1) / kSampThreads;
  c0 = min(V, (int)threadIdx.x * per);
  c1 = min(V, c0 + per);
}

// Exclusive count of weight-tau ties before each thread's chunk.
LMX_DEV uint64_t tie_prefix(const bf16_t* l, const Dist& D, int V, uint64_t* buf) {
  int c0, c1;
  chunk_of(V, c0, c1);
  uint64_t n = 0;
  if (D.topp)
    for (int j = c0; j < c1; ++j) n += dist_w(l, j, D.mx, D.inv_t) == D.tau;
  return block_exscan64(n, buf);
}

// Draw by inverse CDF over kept weights in index order.
LMX_DEV int draw_dev(const bf16_t* l, const Dist& D, int V, uint32_t u24, SampScratch& sm) {
  int c0, c1;
  chunk_of(V, c0, c1);
  uint64_t ties = tie_prefix(l, D, V, sm.tscan);
  uint64_t local = 0, tr = ties;
  int last = -1;
  for (int j = c0; j < c1; ++j) {
    const uint64_t w = dist_w(l, j, D.mx, D.inv_t);
    const bool k = kept_w(D, w, tr);
    if (D.topp && w == D.tau) ++tr;
    if (k && w) { local += w; last = j; }
  }
  const uint64_t pre = block_exscan64(local, sm.tscan2);
  const u128 target = (u128)u24 * D.Zk;
  if (threadIdx.x == 0) sm.result = -1;
  __syncthreads();
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
      if (((u128)cum << 24) > target) { sm.result = j; break; }
    }
  }
  __syncthreads();
  int r = sm.result;
  if (r < 0) {  // unreachable for a consistent distribution: last kept positive token
    __syncthreads();
    if (threadIdx.x == 0) sm.result = -1;
    __syncthreads();
    atomicMax(&sm.result, last);
    __syncthreads();
    r = sm.result < 0 ? 0 : sm.result;
  }
  __syncthreads();
  return r;
}

// Kept weight of token d (0 if outside the top-p set).
LMX_DEV uint64_t kept_weight_of(const bf16_t* l, const Dist& D, int d, SampScratch& sm) {
  const uint64_t w = dist_w(l, d, D.mx, D.inv_t);
  if (!D.topp || w > D.tau) return w;
  if (w < D.tau) return 0;
  uint64_t n = 0;
  for (int j = threadIdx.x; j < d; j += kSampThreads) n += dist_w(l, j, D.mx, D.inv_t) == D.tau;
  n = block_sum64(n, sm);
  return n < D.kties ? w : 0;
}

// Residual draw r_j = max(0, p_j Zq - q_j Zp) by inverse CDF with u24;
// returns -1 if R == 0.
LMX_DEV int residual_draw_dev(const bf16_t* lp, const Dist& P, const bf16_t* lq, const Dist& Q, int V,
                              uint32_t u24, SampScratch& sm) {
  int c0, c1;
  chunk_of(V, c0, c1);
  const uint64_t tp = tie_prefix(lp, P, V, sm.tscan);
  const uint64_t tq = tie_prefix(lq, Q, V, sm.tscan2);
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
  const u128 pre = block_exscan128(local, sm.mscan);
  // total R = pre + local of the last thread
  __syncthreads();
  if (threadIdx.x == kSampThreads - 1) sm.wred[0] = pre + local;
  if (threadIdx.x == 0) sm.result = -1;
  __syncthreads();
  const u128 R = sm.wred[0];
  if (R == 0) return -1;
  const u128 target = (u128)u24 * R;
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
      if ((cum << 24) > target) { sm.result = j; break; }
    }
  }
  __syncthreads();
  const int r = sm.result;
  __syncthreads();
  return r;
}

// ---------------------------------------------------------------------------
// kernels (grid = batch, block = 1024)
// ---------------------------------------------------------------------------
struct StochParams {
  float temperature, top_p;
  uint64_t seed;
};

// Sample one token per row from logits [rows][ld] with uniform
// (seed, row, step, slot, stream); writes out[row].
__global__ void __launch_bounds__(kSampThreads) sample_rows_kernel(const bf16_t* logits, int ld, int V,
                                                                   StochParams sp, uint32_t step,
                                                                   uint32_t slot, uint32_t stream,
                                                                   int32_t* out) {
  __shared__ SampScratch sm;
  grid_wait();
  grid_launch_dependents();
  const int b = blockIdx.x;
  const bf16_t* l = logits + (size_t)b * ld;
  Dist D;
  make_dist_dev(l, V, sp.temperature, sp.top_p, D, sm);
  const int t = draw_dev(l, D, V, uniform24(sp.seed, b, step, slot, stream), sm);
  if (threadIdx.x == 0) out[b] = t;
}

}  // namespace lmx

#include "engine_kernels.cuh"

namespace lmx {

// Draft token i of every sequence, drawn from q_i = dist(draft logits):
// uniform (seed, b, step_b, i, 0).  Bookkeeping as draft_argmax_kernel.
__global__ void __launch_bounds__(kSampThreads) draft_sample_kernel(const bf16_t* qlog, int V, SpecState s,
                                                                    StochParams sp, int i, int adv) {
  __shared__ SampScratch sm;
  grid_wait();
  grid_launch_dependents();
  const int b = blockIdx.x;
  const bf16_t* l = qlog + ((size_t)b * s.K + i) * V;
  Dist D;
  make_dist_dev(l, V, sp.temperature, sp.top_p, D, sm);
  const int tok = draw_dev(l, D, V, uniform24(sp.seed, b, (uint32_t)s.ustep[b], i, 0), sm);
  if (threadIdx.x == 0) {
    s.drafts[b * s.K + i] = tok;
    if (s.emitted[b] < s.max_tokens) s.dlen[b] += adv;
    if (i == s.K - 1) {
      s.vt[b * (s.K + 1)] = s.tok2[2 * b + 1];
      for (int k = 0; k < s.K; ++k) s.vt[b * (s.K + 1) + 1 + k] = s.drafts[b * s.K + k];
    }
  }
}

// Rejection sampling against the verify pass (target logits [B][K+1][V]) and
// the stored draft logits, then commit / rollback (commit_step).  Uniforms:
// accept test i -> (b, step, i, 1), residual / bonus draw -> (b, step, 0, 2).
__global__ void __launch_bounds__(kSampThreads) accept_stochastic_kernel(const bf16_t* tlog, int V, SpecState s,
                                                                         StochParams sp) {
  __shared__ SampScratch sm;
  grid_wait();
  grid_launch_dependents();
  const int b = blockIdx.x, K = s.K;
  const uint32_t step = (uint32_t)s.ustep[b];
  __syncthreads();
  if (threadIdx.x == 0) s.ustep[b] = (int)step + 1;
  if (s.emitted[b] >= s.max_tokens) {  // finished: frozen
    if (threadIdx.x == 0) s.dlen[b] = s.tlen[b] - 1;
    return;
  }
  const uint32_t uf = uniform24(sp.seed, b, step, 0, 2);
  int acc = K, next = -1;
  for (int i = 0; i < K; ++i) {
    const bf16_t* lp = tlog + ((size_t)b * (K + 1) + i) * V;
    const bf16_t* lq = s.qlog + ((size_t)b * K + i) * V;
    Dist P, Q;
    make_dist_dev(lp, V, sp.temperature, sp.top_p, P, sm);
    make_dist_dev(lq, V, sp.temperature, sp.top_p, Q, sm);
    const int d = s.drafts[b * K + i];
    const uint64_t pd = kept_weight_of(lp, P, d, sm), qd = kept_weight_of(lq, Q, d, sm);
    const uint32_t ua = uniform24(sp.seed, b, step, i, 1);
    if ((u128)ua * qd * P.Zk < (((u128)pd * Q.Zk) << 24)) continue;
    acc = i;
    next = residual_draw_dev(lp, P, lq, Q, V, uf, sm);
    if (next < 0) next = draw_dev(lp, P, V, uf, sm);
    break;
  }
  if (acc == K) {
    const bf16_t* lp = tlog + ((size_t)b * (K + 1) + K) * V;
    Dist P;
    make_dist_dev(lp, V, sp.temperature, sp.top_p, P, sm);
    next = draw_dev(lp, P, V, uf, sm);
  }
  if (threadIdx.x == 0) commit_step(s, b, acc, next);
}

}  // namespace lmx

namespace lmx {

// Standalone forms with caller-supplied 24-bit uniforms (the C-ABI ops).
__global__ void __launch_bounds__(kSampThreads) sample_u_kernel(const bf16_t* logits, int V, float temperature,
                                                                float top_p, const uint32_t* u24, int32_t* out) {
  __shared__ SampScratch sm;
  grid_wait();
  grid_launch_dependents();
  const int b = blockIdx.x;
  const bf16_t* l = logits + (size_t)b * V;
  Dist D;
  make_dist_dev(l, V, temperature, top_p, D, sm);
  const int t = draw_dev(l, D, V, u24[b] & 0xFFFFFFu, sm);
  if (threadIdx.x == 0) out[b] = t;
}

__global__ void __launch_bounds__(kSampThreads) accept_u_kernel(const bf16_t* tlog, const bf16_t* qlog,
                                                                const int32_t* drafts, int K, int V,
                                                                float temperature, float top_p,
                                                                const uint32_t* u_accept, const uint32_t* u_final,
                                                                int32_t* n_accepted, int32_t* out_tokens) {
  __shared__ SampScratch sm;
  grid_wait();
  grid_launch_dependents();
  const int b = blockIdx.x;
  const uint32_t uf = u_final[b] & 0xFFFFFFu;
  int acc = K, next = -1;
  for (int i = 0; i < K; ++i) {
    const bf16_t* lp = tlog + ((size_t)b * (K + 1) + i) * V;
    const bf16_t* lq = qlog + ((size_t)b * K + i) * V;
    Dist P, Q;
    make_dist_dev(lp, V, temperature, top_p, P, sm);
    make_dist_dev(lq, V, temperature, top_p, Q, sm);
    const int d = drafts[b * K + i];
    const uint64_t pd = kept_weight_of(lp, P, d, sm), qd = kept_weight_of(lq, Q, d, sm);
    const uint32_t ua = u_accept[b * K + i] & 0xFFFFFFu;
    if ((u128)ua * qd * P.Zk < (((u128)pd * Q.Zk) << 24)) {
      if (threadIdx.x == 0) out_tokens[b * (K + 1) + i] = d;
      continue;
    }
    acc = i;
    next = residual_draw_dev(lp, P, lq, Q, V, uf, sm);
    if (next < 0) next = draw_dev(lp, P, V, uf, sm);
    break;
  }
  if (acc == K) {
    const bf16_t* lp = tlog + ((size_t)b * (K + 1) + K) * V;
    Dist P;
    make_dist_dev(lp, V, temperature, top_p, P, sm);
    next = draw_dev(lp, P, V, uf, sm);
  }
  if (threadIdx.x == 0) {
    out_tokens[b * (K + 1) + acc] = next;
    n_accepted[b] = acc;
  }
}

}  // namespace lmx
