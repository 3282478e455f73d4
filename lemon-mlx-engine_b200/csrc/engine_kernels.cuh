// engine_kernels.cuh -- small kernels of the speculative loop: synthetic
// weights, embedding lookup, draft-token selection and greedy acceptance with
// all bookkeeping kept on the device (so a whole step replays as one graph).
#pragma once
#include <cooperative_groups.h>

#include "lmx_common.cuh"
#include "attn.cuh"
#include "norm_argmax.cuh"
namespace cg = cooperative_groups;

namespace lmx {

// ---------------------------------------------------------------------------
// Synthetic weights, bit-identical to the oracle's orc_gen_normal_bf16 +
// orc_quantize: element e of tensor tid is Irwin-Hall(4) of 22-bit Philox
// uniforms (counter (e_lo, e_hi, tid, 0x243F6A88)), bf16(z * C); each group of
// 64 is quantized with scale = bf16((max-min)/(2^bits-1)), bias = bf16(min).
// One thread per group.  A tensor-parallel shard is the block of rows
// [row0, row0+N) and columns [col0, col0+K) of the full [*, Kfull] matrix:
// element (n, k) keeps its full-matrix index (row0+n)*Kfull + col0+k, so a
// shard holds exactly the values of that block of the unsharded weight.
// ---------------------------------------------------------------------------
LMX_DEV bf16_t gen_normal(uint64_t seed, uint32_t tid, uint64_t e, float C) {
  uint32_t c[4] = {(uint32_t)e, (uint32_t)(e >> 32), tid, 0x243F6A88u};
  philox10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
  int32_t S = (int32_t)((c[0] >> 10) + (c[1] >> 10) + (c[2] >> 10) + (c[3] >> 10));
  return f2bf(__fmul_rn((float)(S - (1 << 23)), C));
}

// One group of 64 values quantized as above into `bits`-bit codes.
LMX_DEV void quantize_group64(const float (&v)[64], int bits, uint32_t* wout, bf16_t* s_out, bf16_t* b_out) {
  float mn = v[0], mx = v[0];
  for (int j = 1; j < 64; ++j) {
    mn = fminf(mn, v[j]);
    mx = fmaxf(mx, v[j]);
  }
  const int nb = (1 << bits) - 1;
  bf16_t sb = f2bf(__fdiv_rn(__fsub_rn(mx, mn), (float)nb));
  float sc = bf2f(sb);
  if (sc == 0.0f) { sb = f2bf(1.0f); sc = 1.0f; }
  const bf16_t bb = f2bf(mn);
  const float bi = bf2f(bb);
  const int per = 32 / bits;
  for (int w = 0; w < 64 / per; ++w) {
    uint32_t word = 0;
    for (int j = 0; j < per; ++j) {
      int q = (int)rintf(__fdiv_rn(__fsub_rn(v[w * per + j], bi), sc));
      q = q < 0 ? 0 : (q > nb ? nb : q);
      word |= (uint32_t)q << (j * bits);
    }
    wout[w] = word;
  }
  *s_out = sb;
  *b_out = bb;
}

__global__ void gen_qweight_kernel(uint64_t seed, uint32_t tid, int N, int K, int bits, float C,
                                   int64_t row0, int64_t col0, int64_t Kfull,
                                   uint32_t* wq, bf16_t* scales, bf16_t* biases) {
  const int G = K / 64;
  const int64_t grp = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (grp >= (int64_t)N * G) return;
  const int n = (int)(grp / G), g = (int)(grp % G);
  const uint64_t e0 = (uint64_t)(row0 + n) * (uint64_t)Kfull + (uint64_t)col0 + (uint64_t)g * 64;
  float v[64];
#pragma unroll 4
  for (int j = 0; j < 64; ++j) v[j] = bf2f(gen_normal(seed, tid, e0 + j, C));
  quantize_group64(v, bits, wq + (size_t)n * (K * bits / 32) + (size_t)g * (64 * bits / 32), &scales[grp],
                   &biases[grp]);
}

// Synthetic context (a stand-in for prefilling a long random-token prefix):
// rows [0, n) of one layer's K or V cache hold N(0, std) values from the same
// Philox normal, tensor id tid, element ((b*Hk_total + hk0+hk)*n + j)*128 + d
// (hk0 = the first KV head of this tensor-parallel shard), quantized per
// group of 64 exactly like an append.  One thread per (b, hk, j, group).
__global__ void fill_kv_kernel(uint64_t seed, uint32_t tid, KvDesc kv, int is_v, int n, int hk0, int Hk_total,
                               float C) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int gpr = kHeadDim / 64;
  if (t >= (int64_t)kv.B * kv.Hk * n * gpr) return;
  const int g = (int)(t % gpr);
  const int64_t rowi = t / gpr;  // (b, hk, j)
  const int j = (int)(rowi % n);
  const int hk = (int)((rowi / n) % kv.Hk), b = (int)(rowi / ((int64_t)n * kv.Hk));
  const uint64_t e0 = (((uint64_t)b * Hk_total + hk0 + hk) * (uint64_t)n + j) * kHeadDim + (uint64_t)g * 64;
  const size_t row = ((size_t)b * kv.Hk + hk) * kv.cap + j;
  if (kv.bits == 16) {
    bf16_t* dst = (is_v ? kv.v : kv.k) + row * kHeadDim + g * 64;
    for (int d = 0; d < 64; ++d) dst[d] = gen_normal(seed, tid, e0 + d, C);
    return;
  }
  float v[64];
#pragma unroll 4
  for (int d = 0; d < 64; ++d) v[d] = bf2f(gen_normal(seed, tid, e0 + d, C));
  const int wpr = kHeadDim * kv.bits / 32;
  quantize_group64(v, kv.bits, (is_v ? kv.vq : kv.kq) + row * wpr + g * (64 * kv.bits / 32),
                   (is_v ? kv.vs : kv.ks) + row * gpr + g, (is_v ? kv.vb : kv.kb) + row * gpr + g);
}

__global__ void fill_bf16_kernel(bf16_t* p, int64_t n, bf16_t v) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = v;
}

// ---------------------------------------------------------------------------
// Embedding lookup from the packed (tied) table: h = bf16(fma(s, q, b)).
// Token of row r: tok[(r / T) * ld + off + r % T].
// ---------------------------------------------------------------------------
__global__ void embed_kernel(const int32_t* tok, int T, int ld, int off, const uint32_t* wq,
                             const bf16_t* s, const bf16_t* b, int H, int bits, bf16_t* h, int R) {
  grid_wait();
  grid_launch_dependents();
  const int r = blockIdx.x;
  if (r >= R) return;
  const int t = tok[(r / T) * ld + off + r % T];
  const int per = 32 / bits, G = H / 64;
  const uint32_t* row = wq + (size_t)t * (H * bits / 32);
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const int q = (int)((row[i / per] >> ((i % per) * bits)) & ((1u << bits) - 1u));
    h[(size_t)r * H + i] =
        f2bf(__fmaf_rn(bf2f(s[(size_t)t * G + i / 64]), (float)q, bf2f(b[(size_t)t * G + i / 64])));
  }
}

// ---------------------------------------------------------------------------
// Device-side state of the speculative loop (one entry per sequence).
// ---------------------------------------------------------------------------
struct SpecState {
  int B, K, max_tokens;
  int32_t* tok2;     // [B][2]: token at position p-1, token y at position p
  int32_t* drafts;   // [B][K]
  int32_t* vt;       // [B][K+1]: verify input y, d1..dK
  int32_t* pred;     // [B][K+1]: target argmax of the verify pass
  int* tlen;         // [B] target cache length (= p)
  int* dlen;         // [B] draft cache length
  int* emitted;      // [B]
  int* accepted;     // [B] accepted drafts (sum)
  int* steps;        // [B] speculative steps taken while unfinished
  int32_t* out;      // [B][max_tokens]
  bf16_t* qlog;      // stochastic: draft logits [B][K][V]
  int* ustep;        // stochastic: per-sequence step index of the uniform draws
};

// Greedy draft token i of every sequence: cluster argmax of the draft logits
// (rows [B][V]), then rank 0 records d_{i+1}, advances the draft length by the
// forward's token count and, after the last draft, assembles the verify input.
__global__ void __launch_bounds__(512) draft_argmax_kernel(const bf16_t* logits, int V, SpecState s,
                                                          int i, int adv) {
  __shared__ float sv[32];
  __shared__ int si[32];
  __shared__ float cv;
  __shared__ int ci;
  grid_wait();
  grid_launch_dependents();
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank(), cs = (int)cluster.num_blocks();
  const int b = blockIdx.x / cs;
  const int chunk = (V + cs - 1) / cs;
  const int j0 = rank * chunk, j1 = min(V, j0 + chunk);
  const bf16_t* l = logits + (size_t)b * V;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int j = j0 + threadIdx.x; j < j1; j += blockDim.x) {
    float v = bf2f(l[j]);
    if (v == v && am_better(v, j, bv, bi)) { bv = v; bi = j; }
  }
  am_block(bv, bi, sv, si);
  if (threadIdx.x == 0) { cv = bv; ci = bi; }
  cluster.sync();
  if (rank == 0 && threadIdx.x == 0) {
    float rv = cv;
    int ri = ci;
    for (int r = 1; r < cs; ++r) {
      float ov = *cluster.map_shared_rank(&cv, r);
      int oi = *cluster.map_shared_rank(&ci, r);
      if (am_better(ov, oi, rv, ri)) { rv = ov; ri = oi; }
    }
    const int tok = ri == 0x7fffffff ? 0 : ri;
    s.drafts[b * s.K + i] = tok;
    const bool done = s.emitted[b] >= s.max_tokens;
    if (!done) s.dlen[b] += adv;
    if (i == s.K - 1) {
      s.vt[b * (s.K + 1)] = s.tok2[2 * b + 1];
      for (int k = 0; k < s.K; ++k) s.vt[b * (s.K + 1) + 1 + k] = s.drafts[b * s.K + k];
    }
  }
  cluster.sync();
}

// The same bookkeeping for a tensor-parallel draft, whose greedy token per
// sequence comes from the vocab-parallel argmax (tok[b]): records d_{i+1},
// advances the draft length and, after the last draft, assembles the verify
// input.  One thread per sequence.
__global__ void __launch_bounds__(128) draft_commit_kernel(SpecState s, const int32_t* tok, int i, int adv) {
  grid_wait();
  grid_launch_dependents();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= s.B) return;
  s.drafts[b * s.K + i] = tok[b];
  if (s.emitted[b] < s.max_tokens) s.dlen[b] += adv;
  if (i == s.K - 1) {
    s.vt[b * (s.K + 1)] = s.tok2[2 * b + 1];
    for (int k = 0; k < s.K; ++k) s.vt[b * (s.K + 1) + 1 + k] = s.drafts[b * s.K + k];
  }
}

// Emit / commit / rollback shared by the greedy and stochastic acceptance:
// emit y, d1..d_acc; next y = `next`; target length p+acc+1, draft p+acc.
LMX_DEV void commit_step(const SpecState& s, int b, int acc, int next) {
  const int p = s.tlen[b];
  const int32_t* d = s.drafts + b * s.K;
  const int y = s.tok2[2 * b + 1];
  int e = s.emitted[b];
  int32_t* o = s.out + (size_t)b * s.max_tokens;
  if (e < s.max_tokens) o[e++] = y;
  for (int k = 0; k < acc; ++k)
    if (e < s.max_tokens) o[e++] = d[k];
  s.emitted[b] = e;
  s.accepted[b] += acc;
  s.steps[b] += 1;
  s.tok2[2 * b] = acc > 0 ? d[acc - 1] : y;
  s.tok2[2 * b + 1] = next;
  s.vt[b * (s.K + 1)] = next;  // the next verify input starts with it (K = 0: it is the whole input)
  s.tlen[b] = p + acc + 1;
  s.dlen[b] = p + acc;
}

// Greedy acceptance (src/common/generate.cpp:800-823) and commit/rollback
// (:850-888): accept while pred[i] == d_{i+1}; emit y, d1..d_acc; the next y
// is the correction or bonus token; target length p+acc+1, draft length p+acc.
// Finished sequences are frozen (nothing emitted, lengths unchanged).
__global__ void accept_greedy_kernel(SpecState s) {
  grid_wait();
  grid_launch_dependents();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= s.B) return;
  const int K = s.K;
  const int p = s.tlen[b];
  if (s.emitted[b] >= s.max_tokens) {
    s.dlen[b] = p - 1;
    return;
  }
  const int32_t* pr = s.pred + b * (K + 1);
  const int32_t* d = s.drafts + b * K;
  int acc = 0;
  while (acc < K && pr[acc] == d[acc]) ++acc;
  commit_step(s, b, acc, pr[acc]);
}

// Prefill bookkeeping: y = the first token from the last prompt position,
// tok2 = (prompt[P-1], y), the target / draft cache lengths (ctx+P and
// ctx+P-1, ctx synthetic context rows before the prompt; with the KV pad
// quirk, the reference allocations).
__global__ void prefill_done_kernel(SpecState s, const int32_t* prompts, int P, const int32_t* y, int tlen,
                                    int dlen) {
  grid_wait();
  grid_launch_dependents();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= s.B) return;
  s.tok2[2 * b] = prompts[(size_t)b * P + P - 1];
  s.tok2[2 * b + 1] = y[b];
  s.vt[b * (s.K + 1)] = y[b];
  s.tlen[b] = tlen;
  s.dlen[b] = dlen;
  s.emitted[b] = 0;
  s.accepted[b] = 0;
  s.steps[b] = 0;
  if (s.ustep) s.ustep[b] = 1;
}

__global__ void add_len_kernel(int* len, int B, int n) {
  grid_wait();
  grid_launch_dependents();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) len[b] += n;
}

}  // namespace lmx
