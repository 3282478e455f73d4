// hybrid.cuh -- configuration 4: a Qwen3-Next-style hybrid decoder (gated
// full attention every attn_every-th layer, Gated DeltaNet elsewhere, a
// sparse MoE block after each mixer) and its MTP speculative decoder.
//
// Reference: Qwen3NextModel / decoder layers (src/llm/models/
// qwen3_next.cpp:118-167 gated attention, 216-403 Gated DeltaNet, 452-490
// sparse MoE with shared expert), MTPHead (src/llm/models/mtp_head.cpp:
// 146-178), TokenIterator::mtp_speculative_step (src/common/generate.cpp:
// 669-933).  Built from the library's kernels: K1 GEMV / tcgen05 matmuls,
// the attention prep + SDPA, the Gated DeltaNet verify / commit and the MoE
// router / experts (gdn_moe.cuh), plus the small kernels below.
#pragma once
#include "gdn_moe.cuh"

namespace lmx {

// o = bf16(o * bf16(sigmoid(g))) (gated attention output, MLX materialises
// sigmoid then the product); o [R][n], g rows ldg apart.
__global__ void gate_mul_kernel(bf16_t* o, const bf16_t* g, int R, int n, int ldg) {
  grid_wait();
  grid_launch_dependents();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)R * n) return;
  const int r = (int)(i / n), c = (int)(i % n);
  const float sg = bf2f(f2bf(sigmoid_c(bf2f(g[(size_t)r * ldg + c]))));
  o[i] = f2bf(__fmul_rn(bf2f(o[i]), sg));
}

// h = bf16(h + bf16(y_moe + bf16(bf16(sigmoid(sg)) * y_sh)))   (shared
// expert gate, qwen3_next.cpp:480-489, then the decoder residual)
__global__ void moe_combine_kernel(bf16_t* h, const bf16_t* ymoe, const bf16_t* ysh, const bf16_t* sg, int R,
                                   int H) {
  grid_wait();
  grid_launch_dependents();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)R * H) return;
  const int r = (int)(i / H);
  const float gs = bf2f(f2bf(sigmoid_c(bf2f(sg[r]))));
  const float t = bf2f(f2bf(__fmul_rn(gs, bf2f(ysh[i]))));
  const float m = bf2f(f2bf(__fadd_rn(bf2f(ymoe[i]), t)));
  h[i] = f2bf(__fadd_rn(bf2f(h[i]), m));
}

// MTP input: cat[r] = [rms(e[r]) * we | rms(hid[r]) * wh] (embedding first,
// mtp_head.cpp:160-167); one warp per (row, half), canonical RMSNorm.
__global__ void __launch_bounds__(256) mtp_prep_kernel(const bf16_t* e, const bf16_t* hid, int ldh,
                                                       const bf16_t* we, const bf16_t* wh, float eps, bf16_t* cat,
                                                       int R, int H) {
  grid_wait();
  grid_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int task = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (task >= 2 * R) return;
  const int r = task >> 1, part = task & 1;
  const bf16_t* x = part ? hid + (size_t)r * ldh : e + (size_t)r * H;
  const bf16_t* w = part ? wh : we;
  const float f = rms_factor_warp(x, H, eps, lane);
  bf16_t* y = cat + (size_t)r * 2 * H + (size_t)part * H;
  for (int c = lane; c < (H >> 3); c += 32) {
    const uint4 xv = *reinterpret_cast<const uint4*>(x + 8 * c);
    const uint4 wv = *reinterpret_cast<const uint4*>(w + 8 * c);
    const uint32_t xa[4] = {xv.x, xv.y, xv.z, xv.w}, wa[4] = {wv.x, wv.y, wv.z, wv.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const bf16_t lo = f2bf(__fmul_rn(__fmul_rn(lo_bf(xa[k]), f), lo_bf(wa[k])));
      const bf16_t hi = f2bf(__fmul_rn(__fmul_rn(hi_bf(xa[k]), f), hi_bf(wa[k])));
      o[k] = (uint32_t)lo | ((uint32_t)hi << 16);
    }
    *reinterpret_cast<uint4*>(y + 8 * c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

__global__ void set_int_kernel(int32_t* p, int n, int v) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = v;
}

// copy rows: dst[b] = src[b * T + idx[b]] (H bf16 each); idx < 0: unchanged
__global__ void gather_rows_kernel(bf16_t* dst, const bf16_t* src, const int32_t* idx, int T, int H) {
  grid_wait();
  grid_launch_dependents();
  const int b = blockIdx.x;
  const int t = idx[b];
  if (t < 0) return;
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x)
    reinterpret_cast<uint4*>(dst + (size_t)b * H)[c] = reinterpret_cast<const uint4*>(src + ((size_t)b * T + t) * H)[c];
}

// ---------------------------------------------------------------------------
// model
// ---------------------------------------------------------------------------
struct HybLayer {
  bool attn = false;
  QWeight q, k, v, qg, o;                    // gated attention
  QWeight wqkv, wz, wb, wa, wout;            // Gated DeltaNet
  bf16_t *conv_w = nullptr, *dt_bias = nullptr, *gnorm = nullptr;
  float* a_log = nullptr;
  QWeight router, eg, eu, ed, sg, su, sd, sgate;  // MoE (eg / eu: E*I rows, ed: E*H rows)
  bf16_t *in_norm = nullptr, *post_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
};

struct HybModel {
  lmx_hybrid_config c;
  std::vector<HybLayer> L;
  HybLayer mtp;  // the MTP decoder layer (attention + MoE)
  QWeight embed, lm_head, mtp_fc;
  bf16_t *final_norm = nullptr, *mtp_norm_e = nullptr, *mtp_norm_h = nullptr, *mtp_norm = nullptr;
  float *cos_t = nullptr, *sin_t = nullptr;
  int max_pos = 16384;
  int n_attn = 0, n_gdn = 0;
  // expert parallelism: this rank's experts [e_lo, e_lo + per) of every MoE
  // block (router, shared expert, attention / GDN, heads replicated); comm
  // not owned
  int ep = 1, ep_rank = 0, per = 0, e_lo = 0;
  TpComm* comm = nullptr;
  Arena ar;
  int CD() const { return 2 * c.lin_k_heads * kGdnD + c.lin_v_heads * kGdnD; }
};

// Seeded bf16 N(0, std) vector (tensor id tid, the weights' Philox normal).
__global__ void gen_bf16_kernel(uint64_t seed, uint32_t tid, int64_t n, float C, bf16_t* out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = gen_normal(seed, tid, (uint64_t)i, C);
}
__global__ void bf16_to_f32_kernel(const bf16_t* in, float* out, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = bf2f(in[i]);
}
static int gen_bf16(Arena& ar, bf16_t** p, int64_t n, uint64_t seed, uint32_t tid, float std_dev, cudaStream_t st) {
  int rc = ar.alloc(p, (size_t)n, false);
  if (rc) return rc;
  const float C = (float)((double)std_dev * std::sqrt(3.0) / 4194304.0);
  gen_bf16_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(seed, tid, n, C, *p);
  return cuda_check(cudaGetLastError(), "gen_bf16");
}

// Tensor ids: layer l (0..layers-1; the MTP layer is l = layers), base
// (l+1)*64: attention q 0, k 1, v 2, q-gate 3, o 4; GDN qkv 8, z 9, b 10,
// a 11, out 12, conv_w 13 (N(0,0.3)), dt_bias 14 (N(0,0.5)), a_log 15
// (N(0,0.5), fp32 of the bf16); MoE router 16, experts gate 17, up 18, down
// 19, shared gate 20, up 21, down 22, shared-expert gate 23; embed 1,
// lm_head 2, MTP fc 3.  Norm weights are ones.
static int hyb_layer_create(HybModel& m, int l, bool attn, uint64_t seed, cudaStream_t st) {
  const lmx_hybrid_config& c = m.c;
  Arena& ar = m.ar;
  HybLayer& L = l < c.layers ? m.L[l] : m.mtp;
  L.attn = attn;
  const int H = c.hidden, NQ = c.heads * kHeadDim, NK = c.kv_heads * kHeadDim;
  const uint32_t base = (uint32_t)(l + 1) * 64;
  int rc = LMX_OK;
  auto gq = [&](QWeight& q, uint32_t k, int N, int K) {
    if (!rc) rc = gen_qweight(ar, q, seed, base + k, N, K, c.bits, st);
  };
  if (attn) {
    gq(L.q, 0, NQ, H);
    gq(L.k, 1, NK, H);
    gq(L.v, 2, NK, H);
    gq(L.qg, 3, NQ, H);
    gq(L.o, 4, H, NQ);
    if (!rc) rc = fill_ones(ar, &L.q_norm, kHeadDim, st);
    if (!rc) rc = fill_ones(ar, &L.k_norm, kHeadDim, st);
  } else {
    const int CD = m.CD(), Z = c.lin_v_heads * kGdnD;
    gq(L.wqkv, 8, CD, H);
    gq(L.wz, 9, Z, H);
    gq(L.wb, 10, c.lin_v_heads, H);
    gq(L.wa, 11, c.lin_v_heads, H);
    gq(L.wout, 12, H, Z);
    if (!rc) rc = gen_bf16(ar, &L.conv_w, (int64_t)CD * kGdnKS, seed, base + 13, 0.3f, st);
    if (!rc) rc = gen_bf16(ar, &L.dt_bias, c.lin_v_heads, seed, base + 14, 0.5f, st);
    bf16_t* al = nullptr;
    if (!rc) rc = gen_bf16(ar, &al, c.lin_v_heads, seed, base + 15, 0.5f, st);
    if (!rc) rc = ar.alloc(&L.a_log, c.lin_v_heads, false);
    if (!rc) {
      bf16_to_f32_kernel<<<(c.lin_v_heads + 255) / 256, 256, 0, st>>>(al, L.a_log, c.lin_v_heads);
      rc = cuda_check(cudaGetLastError(), "a_log");
    }
    if (!rc) rc = fill_ones(ar, &L.gnorm, kGdnD, st);
  }
  gq(L.router, 16, c.experts, H);
  // this rank's experts as row blocks of the stacked expert matrices, with
  // their full-matrix element indices (the same values as unsharded)
  const int per = m.per, e0 = m.e_lo;
  if (!rc) rc = gen_qweight(ar, L.eg, seed, base + 17, per * c.expert_inter, H, c.bits, st, (int64_t)e0 * c.expert_inter, 0, H);
  if (!rc) rc = gen_qweight(ar, L.eu, seed, base + 18, per * c.expert_inter, H, c.bits, st, (int64_t)e0 * c.expert_inter, 0, H);
  if (!rc)
    rc = gen_qweight(ar, L.ed, seed, base + 19, per * H, c.expert_inter, c.bits, st, (int64_t)e0 * H, 0, c.expert_inter);
  gq(L.sg, 20, c.shared_inter, H);
  gq(L.su, 21, c.shared_inter, H);
  gq(L.sd, 22, H, c.shared_inter);
  gq(L.sgate, 23, 1, H);
  if (!rc) rc = fill_ones(ar, &L.in_norm, H, st);
  if (!rc) rc = fill_ones(ar, &L.post_norm, H, st);
  return rc;
}

static int hyb_create(const lmx_hybrid_config& c, uint64_t seed, TpComm* comm, HybModel** out) {
  if ((c.bits != 4 && c.bits != 8) || c.hidden % 512 || c.layers < 1 || c.attn_every < 1 || c.heads < 1 ||
      c.kv_heads < 1 || c.heads % c.kv_heads || c.lin_k_heads < 1 || c.lin_v_heads % c.lin_k_heads ||
      c.experts < 1 || c.top_k < 1 || c.top_k > 16 || c.top_k > c.experts || c.expert_inter % 512 ||
      c.shared_inter % 512 || c.vocab < 1 || c.experts > 16384)
    return set_error(LMX_ERR_UNSUPPORTED, "hybrid config not supported (hidden / FFNs %% 512, top_k <= 16, 4/8-bit)");
  const int ep = comm ? comm->n : 1;
  if (ep > 1) {
    if (!comm->opened) return set_error(LMX_ERR_INVALID, "hybrid_create: ep comm not opened");
    if (c.experts % ep || c.hidden > comm->max_hidden)
      return set_error(LMX_ERR_UNSUPPORTED, "hybrid_create: experts %% ep == 0 and hidden <= comm max_hidden needed");
  }
  auto m = std::make_unique<HybModel>();
  m->c = c;
  m->ep = ep;
  m->ep_rank = comm ? comm->rank : 0;
  m->per = c.experts / ep;
  m->e_lo = m->ep_rank * m->per;
  m->comm = ep > 1 ? comm : nullptr;
  m->L.resize(c.layers);
  cudaStream_t st = 0;
  int rc = LMX_OK;
  for (int l = 0; l < c.layers && !rc; ++l) {
    const bool attn = l % c.attn_every == c.attn_every - 1;
    (attn ? m->n_attn : m->n_gdn)++;
    rc = hyb_layer_create(*m, l, attn, seed, st);
  }
  if (!rc) rc = hyb_layer_create(*m, c.layers, true, seed, st);
  if (!rc) rc = gen_qweight(m->ar, m->embed, seed, 1, c.vocab, c.hidden, c.bits, st);
  if (!rc) rc = gen_qweight(m->ar, m->lm_head, seed, 2, c.vocab, c.hidden, c.bits, st);
  if (!rc) rc = gen_qweight(m->ar, m->mtp_fc, seed, 3, c.hidden, 2 * c.hidden, c.bits, st);
  for (bf16_t** p : {&m->final_norm, &m->mtp_norm_e, &m->mtp_norm_h, &m->mtp_norm})
    if (!rc) rc = fill_ones(m->ar, p, c.hidden, st);
  if (rc) return rc;
  // RoPE table: period_i = theta^(2i/128), angle = pos / period (double)
  const int D = kHeadDim;
  std::vector<float> ct((size_t)m->max_pos * D / 2), stt(ct.size());
  for (int i = 0; i < D / 2; ++i) {
    const double pd = std::pow((double)c.rope_theta, 2.0 * (double)i / (double)D);
    for (int p = 0; p < m->max_pos; ++p) {
      const double th = (double)p / pd;
      ct[(size_t)p * D / 2 + i] = (float)std::cos(th);
      stt[(size_t)p * D / 2 + i] = (float)std::sin(th);
    }
  }
  rc = m->ar.alloc(&m->cos_t, ct.size(), false);
  if (!rc) rc = m->ar.alloc(&m->sin_t, stt.size(), false);
  if (!rc) rc = cuda_check(cudaMemcpy(m->cos_t, ct.data(), ct.size() * 4, cudaMemcpyHostToDevice), "rope");
  if (!rc) rc = cuda_check(cudaMemcpy(m->sin_t, stt.data(), stt.size() * 4, cudaMemcpyHostToDevice), "rope");
  if (!rc) rc = cuda_check(cudaDeviceSynchronize(), "hybrid init");
  if (rc) return rc;
  *out = m.release();
  return LMX_OK;
}

// ---------------------------------------------------------------------------
// state: attention KV caches, recurrent states, activations
// ---------------------------------------------------------------------------
struct HybGdnLayer {
  bf16_t* qkv = nullptr;   // [B][Tmax][CD] this layer's pre-conv inputs (kept for the commit)
  bf16_t* conv = nullptr;  // [B][3][CD]
  float* state = nullptr;  // [B][Hv][128][128]
  float* snap = nullptr;   // [B][Tsnap][Hv][128][128]
};

struct HybState {
  int B = 0, cap = 0, Tmax = 0, Tsnap = 0, Rmax = 0;
  std::unique_ptr<Cache> kv;      // attention layers, in layer order
  std::unique_ptr<Cache> mtp_kv;  // the MTP layer
  std::vector<HybGdnLayer> gdn;
  Arena ar;
  // activations [Rmax][...]
  bf16_t *h = nullptr, *xn = nullptr, *qkv = nullptr, *qg = nullptr, *q = nullptr, *o = nullptr;
  bf16_t *gz = nullptr, *gb = nullptr, *ga = nullptr, *gout = nullptr;
  uint8_t* gscr = nullptr;
  bf16_t *rl = nullptr, *acte = nullptr, *ymoe = nullptr, *acts = nullptr, *ysh = nullptr, *sgl = nullptr;
  int32_t* idx = nullptr;
  float* wts = nullptr;
  bf16_t *hid = nullptr, *logits = nullptr, *cat = nullptr, *emb = nullptr;
  float* part = nullptr;
  unsigned* counters = nullptr;
  size_t part_floats = 0, n_counters = 0;
  int32_t* tlast = nullptr;  // [B] = T-1 (commit-all index), set per forward
  size_t state_floats = 0, conv_elems = 0;  // per GDN layer, whole batch
};

static int hyb_state_create(const HybModel& m, int B, int cap, int kv_bits, int Tmax, int Tsnap, int logit_rows,
                            HybState** out) {
  const lmx_hybrid_config& c = m.c;
  if (B < 1 || cap < 1 || cap > m.max_pos || Tmax < 1 || Tsnap < 1)
    return set_error(LMX_ERR_INVALID, "hybrid state: bad arguments");
  auto s = std::make_unique<HybState>();
  s->B = B;
  s->cap = cap;
  s->Tmax = Tmax;
  s->Tsnap = Tsnap;
  const int R = B * Tmax, H = c.hidden, NQ = c.heads * kHeadDim, NK = c.kv_heads * kHeadDim;
  s->Rmax = R;
  Model shape;  // cache geometry only
  shape.c.kv_heads = c.kv_heads;
  shape.hk = c.kv_heads;
  shape.n_layers = std::max(m.n_attn, 1);
  shape.max_pos = m.max_pos;
  Cache* kc = nullptr;
  int rc = LMX_OK;
  if (m.n_attn > 0) {
    rc = cache_create(shape, m.n_attn, B, cap, kv_bits, &kc);
    if (rc) return rc;
    s->kv.reset(kc);
  }
  rc = cache_create(shape, 1, B, 8, kv_bits, &kc);  // MTP: two draft rows per step
  if (rc) return rc;
  s->mtp_kv.reset(kc);
  const int CD = m.CD(), Z = c.lin_v_heads * kGdnD, Hv = c.lin_v_heads;
  s->state_floats = (size_t)B * Hv * kGdnD * kGdnD;
  s->conv_elems = (size_t)B * (kGdnKS - 1) * CD;
  s->gdn.resize(m.n_gdn);
  for (auto& g : s->gdn) {
    if (!rc) rc = s->ar.alloc(&g.qkv, (size_t)R * CD, false);
    if (!rc) rc = s->ar.alloc(&g.conv, (size_t)B * (kGdnKS - 1) * CD);
    if (!rc) rc = s->ar.alloc(&g.state, (size_t)B * Hv * kGdnD * kGdnD);
    if (!rc) rc = s->ar.alloc(&g.snap, (size_t)B * Tsnap * Hv * kGdnD * kGdnD, false);
  }
  Arena& ar = s->ar;
  if (!rc) rc = ar.alloc(&s->h, (size_t)R * H);
  if (!rc) rc = ar.alloc(&s->xn, (size_t)R * H);
  if (!rc) rc = ar.alloc(&s->qkv, (size_t)R * (NQ + 2 * NK));
  if (!rc) rc = ar.alloc(&s->qg, (size_t)R * NQ);
  if (!rc) rc = ar.alloc(&s->q, (size_t)R * NQ);
  if (!rc) rc = ar.alloc(&s->o, (size_t)R * NQ);
  if (!rc) rc = ar.alloc(&s->gz, (size_t)R * Z);
  if (!rc) rc = ar.alloc(&s->gb, (size_t)R * Hv);
  if (!rc) rc = ar.alloc(&s->ga, (size_t)R * Hv);
  if (!rc) rc = ar.alloc(&s->gout, (size_t)R * Z);
  if (!rc) rc = ar.alloc(&s->gscr, gdn_scratch_bytes(B, Tmax, c.lin_k_heads, Hv));
  if (!rc) rc = ar.alloc(&s->rl, (size_t)R * c.experts);
  // routing of every MoE block of the last forward (layers, then the MTP
  // layer), kept for counting the experts a pass touches
  if (!rc) rc = ar.alloc(&s->idx, (size_t)(c.layers + 1) * R * c.top_k);
  if (!rc) rc = ar.alloc(&s->wts, (size_t)R * c.top_k);
  if (!rc) rc = ar.alloc(&s->acte, (size_t)R * c.top_k * c.expert_inter);
  if (!rc) rc = ar.alloc(&s->ymoe, (size_t)R * H);
  if (!rc) rc = ar.alloc(&s->acts, (size_t)R * c.shared_inter);
  if (!rc) rc = ar.alloc(&s->ysh, (size_t)R * H);
  if (!rc) rc = ar.alloc(&s->sgl, (size_t)R);
  if (!rc) rc = ar.alloc(&s->hid, (size_t)R * H);
  if (!rc) rc = ar.alloc(&s->logits, (size_t)logit_rows * c.vocab);
  if (!rc) rc = ar.alloc(&s->cat, (size_t)B * 2 * H);
  if (!rc) rc = ar.alloc(&s->emb, (size_t)B * H);
  if (!rc) rc = ar.alloc(&s->tlast, (size_t)B);
  sdpa_scratch_need(B, Tmax, c.heads / c.kv_heads, c.kv_heads, cap, s->part_floats, s->n_counters);
  if (!rc) rc = ar.alloc(&s->part, s->part_floats, false);
  if (!rc) rc = ar.alloc(&s->counters, s->n_counters);
  if (rc) return rc;
  *out = s.release();
  return LMX_OK;
}

static int hyb_qmm(const bf16_t* x, const QWeight* w, int nmat, int N, bf16_t* y, int ldy, int M, int K, int bits,
                   QmmMode mode, const bf16_t* res, cudaStream_t st) {
  QmmCall c;
  c.x = x;
  for (int i = 0; i < nmat; ++i) c.mat[i] = w[i].mat();
  c.nmat = nmat;
  c.N = N;
  c.y = y;
  c.ldy = ldy;
  c.M = M;
  c.K = K;
  c.bits = bits;
  c.mode = mode;
  c.res = res;
  return launch_qmm(c, st);
}

static int launch_elem(void (*k)(bf16_t*, const bf16_t*, int, int, int), int64_t n, cudaStream_t st, bf16_t* a,
                       const bf16_t* b, int R, int c, int d) {
  return cuda_check(lmx_launch(k, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, true, a, b, R, c, d), "elem");
}

// Attention mixer of layer L on s.xn (R = B*T rows) with cache layer kvd;
// the output is added to s.h.
static int hyb_attention(const HybModel& m, HybState& s, const HybLayer& L, const KvDesc& kvd, int B, int T,
                         cudaStream_t st) {
  const lmx_hybrid_config& c = m.c;
  const int R = B * T, H = c.hidden, NQ = c.heads * kHeadDim, NK = c.kv_heads * kHeadDim;
  const QWeight qkv3[3] = {L.q, L.k, L.v};
  int rc = hyb_qmm(s.xn, qkv3, 3, NQ + 2 * NK, s.qkv, NQ + 2 * NK, R, H, c.bits, kPlain, nullptr, st);
  if (!rc) rc = hyb_qmm(s.xn, &L.qg, 1, NQ, s.qg, NQ, R, H, c.bits, kPlain, nullptr, st);
  PrepArgs pa;
  pa.qkv = s.qkv;
  pa.ldq = NQ + 2 * NK;
  pa.R = R;
  pa.T = T;
  pa.Hq = c.heads;
  pa.Hk = c.kv_heads;
  pa.qn = L.q_norm;
  pa.kn = L.k_norm;
  pa.eps = c.eps;
  pa.cos_t = m.cos_t;
  pa.sin_t = m.sin_t;
  pa.max_pos = m.max_pos;
  pa.q_out = s.q;
  pa.kv = kvd;
  pa.err = device_error_word();
  if (!rc) rc = launch_attn_prep(pa, st);
  const int G = c.heads / c.kv_heads;
  SdpaArgs sa;
  sa.q = s.q;
  sa.kv = kvd;
  sa.T = T;
  sa.Hq = c.heads;
  sa.scale = (float)(1.0 / std::sqrt((double)kHeadDim));
  sa.nsplit = (kvd.cap + kSplit - 1) / kSplit;
  sa.tiles = (G * T + kRowTile - 1) / kRowTile;
  sa.part = s.part;
  sa.counters = s.counters;
  sa.out = s.o;
  sa.part_floats = s.part_floats;
  sa.n_counters = s.n_counters;
  sa.err = device_error_word();
  if (!rc) rc = launch_sdpa(sa, B, st);
  if (!rc) rc = launch_elem(gate_mul_kernel, (int64_t)R * NQ, st, s.o, s.qg, R, NQ, NQ);
  if (!rc) rc = hyb_qmm(s.o, &L.o, 1, H, s.h, H, R, NQ, c.bits, kResid, s.h, st);
  return rc;
}

// Gated DeltaNet mixer of layer L with recurrent state g; commit_idx != null:
// commit right away at that device index (prefill), else leave the
// per-token snapshots for a later commit.
static int hyb_gdn(const HybModel& m, HybState& s, const HybLayer& L, HybGdnLayer& g, int B, int T, int snap_T,
                   const int32_t* commit_idx, cudaStream_t st) {
  const lmx_hybrid_config& c = m.c;
  const int R = B * T, H = c.hidden, CD = m.CD(), Hv = c.lin_v_heads, Z = Hv * kGdnD;
  int rc = hyb_qmm(s.xn, &L.wqkv, 1, CD, g.qkv, CD, R, H, c.bits, kPlain, nullptr, st);
  if (!rc) rc = hyb_qmm(s.xn, &L.wz, 1, Z, s.gz, Z, R, H, c.bits, kPlain, nullptr, st);
  if (!rc) rc = hyb_qmm(s.xn, &L.wb, 1, Hv, s.gb, Hv, R, H, c.bits, kPlain, nullptr, st);
  if (!rc) rc = hyb_qmm(s.xn, &L.wa, 1, Hv, s.ga, Hv, R, H, c.bits, kPlain, nullptr, st);
  if (rc) return rc;
  GdnArgs a;
  a.state_bf16 = g_gdn_state_bf16;
  a.B = B;
  a.T = T;
  a.Hk = c.lin_k_heads;
  a.Hv = Hv;
  a.qkv = g.qkv;
  a.z = s.gz;
  a.b = s.gb;
  a.a = s.ga;
  a.conv_w = L.conv_w;
  a.a_log = L.a_log;
  a.dt_bias = L.dt_bias;
  a.norm_w = L.gnorm;
  a.eps = c.eps;
  a.conv_state = g.conv;
  a.state = g.state;
  a.snap = g.snap;
  a.snap_T = snap_T;
  a.out = s.gout;
  auto up = [](size_t x) { return (x + 255) / 256 * 256; };
  const size_t bt = (size_t)B * T;
  uint8_t* p = s.gscr;
  a.qn = (bf16_t*)p;
  p += up(bt * a.Hk * kGdnD * 2);
  a.kn = (bf16_t*)p;
  p += up(bt * a.Hk * kGdnD * 2);
  a.vc = (bf16_t*)p;
  p += up(bt * Hv * kGdnD * 2);
  a.beta = (float*)p;
  p += up(bt * Hv * 4);
  a.gdecay = (float*)p;
  const long long tasks = (long long)B * T * (2 * a.Hk + Hv);
  rc = cuda_check(lmx_launch(gdn_prep_kernel, dim3((unsigned)((tasks + 7) / 8)), dim3(256), 0, st, true, a), "gdn_prep");
  if (!rc) rc = cuda_check(lmx_launch(gdn_recur_kernel, dim3(Hv, B), dim3(256), 0, st, true, a), "gdn_recur");
  if (!rc && commit_idx)
    rc = cuda_check(lmx_launch(gdn_commit_kernel, dim3(B, Hv + 1), dim3(256), 0, st, true, a, commit_idx, g.state, g.conv),
                    "gdn_commit");
  if (!rc) rc = hyb_qmm(s.gout, &L.wout, 1, H, s.h, H, R, Z, c.bits, kResid, s.h, st);
  return rc;
}

// The commit of every GDN layer at device index acc (per sequence; < 0:
// unchanged) after a forward that kept all T snapshots.
static int hyb_gdn_commit_all(const HybModel& m, HybState& s, int B, int T, const int32_t* acc, cudaStream_t st) {
  int rc = LMX_OK;
  for (size_t i = 0; i < s.gdn.size() && !rc; ++i) {
    HybGdnLayer& g = s.gdn[i];
    GdnArgs a;
    a.state_bf16 = g_gdn_state_bf16;
  a.state_bf16 = g_gdn_state_bf16;
    std::memset(&a, 0, sizeof(a));
    a.B = B;
    a.T = T;
    a.Hk = m.c.lin_k_heads;
    a.Hv = m.c.lin_v_heads;
    a.qkv = g.qkv;
    a.conv_state = g.conv;
    a.snap = g.snap;
    a.snap_T = T;
    rc = cuda_check(lmx_launch(gdn_commit_kernel, dim3(B, a.Hv + 1), dim3(256), 0, st, true, a, acc, g.state, g.conv),
                    "gdn_commit");
  }
  return rc;
}

// MoE block of layer L on s.h: xn = rms(h), y = experts + gated shared expert,
// h += y.
static int hyb_moe(const HybModel& m, HybState& s, const HybLayer& L, int l, int R, cudaStream_t st) {
  const lmx_hybrid_config& c = m.c;
  const int H = c.hidden;
  int32_t* idx = s.idx + (size_t)l * s.Rmax * c.top_k;
  int rc = launch_rms_norm(s.h, L.post_norm, s.xn, R, H, c.eps, st);
  if (!rc) rc = hyb_qmm(s.xn, &L.router, 1, c.experts, s.rl, c.experts, R, H, c.bits, kPlain, nullptr, st);
  if (!rc)
    rc = cuda_check(lmx_launch(moe_route_kernel, dim3((R + 7) / 8), dim3(256), 0, st, true, (const bf16_t*)s.rl, R,
                               c.experts, c.top_k, idx, s.wts),
                    "moe_route");
  if (rc) return rc;
  MoeArgs a;
  a.M = R;
  a.H = H;
  a.I = c.expert_inter;
  a.E = c.experts;
  a.k = c.top_k;
  a.x = s.xn;
  a.idx = idx;
  a.w = s.wts;
  a.gw = L.eg.w;
  a.uw = L.eu.w;
  a.dw = L.ed.w;
  a.gs = L.eg.s;
  a.gb = L.eg.b;
  a.us = L.eu.s;
  a.ub = L.eu.b;
  a.ds = L.ed.s;
  a.db = L.ed.b;
  a.act = s.acte;
  a.y = s.ymoe;
  a.err = device_error_word();
  if (m.ep > 1) {  // this rank's experts, then the exchange-combine across ranks
    TpComm& cm = *m.comm;
    if ((int64_t)R * c.top_k > cm.max_rows || H > cm.max_hidden)
      return set_error(LMX_ERR_INVALID, "hybrid ep: %d x %d slot rows exceed the comm", R, c.top_k);
    a.e_lo = m.e_lo;
    a.e_hi = m.e_lo + m.per;
    a.slot_out = tp_slot(cm, cm.sel);
  }
  rc = c.bits == 4 ? launch_moe_t<4>(a, st) : launch_moe_t<8>(a, st);
  if (!rc && m.ep > 1) {
    TpComm& cm = *m.comm;
    const int grid = R < kTpArCtas ? R : kTpArCtas;
    rc = cuda_check(lmx_launch(ep_combine_kernel, dim3(grid), dim3(256), 0, st, true, cm.t, cm.sel, R, c.top_k, H,
                               (const int32_t*)idx, (const float*)s.wts, m.per, s.ymoe, device_error_word()),
                    "ep_combine");
    cm.sel ^= 1;
  }
  const QWeight gu[2] = {L.sg, L.su};
  if (!rc) rc = hyb_qmm(s.xn, gu, 2, c.shared_inter, s.acts, c.shared_inter, R, H, c.bits, kSwiglu, nullptr, st);
  if (!rc) rc = hyb_qmm(s.acts, &L.sd, 1, H, s.ysh, H, R, c.shared_inter, c.bits, kPlain, nullptr, st);
  if (!rc) rc = hyb_qmm(s.xn, &L.sgate, 1, 1, s.sgl, 1, R, H, c.bits, kPlain, nullptr, st);
  if (!rc)
    rc = cuda_check(lmx_launch(moe_combine_kernel, dim3((unsigned)(((int64_t)R * H + 255) / 256)), dim3(256), 0, st,
                               true, s.h, (const bf16_t*)s.ymoe, (const bf16_t*)s.ysh, (const bf16_t*)s.sgl, R, H),
                    "moe_combine");
  return rc;
}

// Trunk forward of tokens tok[(r/T)*ld + off + r%T], R = B*T rows: layers,
// final norm into s.hid (every row), logits of every row (or each
// sequence's last) into `logits` (ld V) when non-null.  GDN layers commit
// at commit_idx (device, per sequence) when non-null (snap_T = 1), else
// keep all T snapshots.  The caller advances the attention lengths.
static int hyb_forward(const HybModel& m, HybState& s, const int32_t* tok, int ld, int off, int B, int T,
                       bf16_t* logits, bool last_only, const int32_t* commit_idx, cudaStream_t st) {
  const lmx_hybrid_config& c = m.c;
  const int R = B * T, H = c.hidden;
  if (R > s.Rmax || B != s.B || (!commit_idx && T > s.Tsnap))
    return set_error(LMX_ERR_INVALID, "hybrid forward: %d x %d exceeds the state", B, T);
  int rc = cuda_check(lmx_launch(embed_kernel, dim3(R), dim3(256), 0, st, true, tok, T, ld, off,
                                 (const uint32_t*)m.embed.w, (const bf16_t*)m.embed.s, (const bf16_t*)m.embed.b, H,
                                 c.bits, s.h, R),
                      "embed");
  int ia = 0, ig = 0;
  for (int l = 0; l < c.layers && !rc; ++l) {
    const HybLayer& L = m.L[l];
    rc = launch_rms_norm(s.h, L.in_norm, s.xn, R, H, c.eps, st);
    if (rc) break;
    if (L.attn) rc = hyb_attention(m, s, L, s.kv->kv[ia++], B, T, st);
    else rc = hyb_gdn(m, s, L, s.gdn[ig++], B, T, commit_idx ? 1 : T, commit_idx, st);
    if (!rc) rc = hyb_moe(m, s, L, l, R, st);
  }
  if (!rc) rc = launch_rms_norm(s.h, m.final_norm, s.hid, R, H, c.eps, st);
  if (rc || !logits) return rc;
  QmmCall hc;
  hc.x = last_only ? s.hid + (size_t)(T - 1) * H : s.hid;
  hc.ldx = last_only ? T * H : H;
  hc.mat[0] = m.lm_head.mat();
  hc.N = c.vocab;
  hc.y = logits;
  hc.ldy = c.vocab;
  hc.M = last_only ? B : R;
  hc.K = H;
  hc.bits = c.bits;
  return launch_qmm(hc, st);
}

// ---------------------------------------------------------------------------
// MTP speculative decoding (TokenIterator::mtp_speculative_step): per step
// d0 (the trunk's next token) is known; the MTP head drafts d1 from (the
// trunk hidden at d0's predicting position, embed(d0)) and d2 from (its own
// output hidden, embed(d1)), with its attention cache reset to 0 every step;
// the trunk verifies [d0, d1, d2]; the accepted prefix is emitted, the
// attention lengths advance by acc + 1, every Gated DeltaNet state takes
// the snapshot after token acc, and the trunk hidden at acc seeds the next
// step.  Finished sequences keep their state (acc = -1).
// ---------------------------------------------------------------------------
static constexpr int kHybN = 3;  // verify tokens (d0 + 2 drafts)

__global__ void hyb_accept_kernel(int B, int MT, int32_t* vt, const int32_t* pred, int32_t* acc_out, int* tlen,
                                  int* emitted, int* accepted, int* steps, int32_t* out) {
  grid_wait();
  grid_launch_dependents();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  int e = emitted[b];
  if (e >= MT) {
    acc_out[b] = -1;
    return;
  }
  int32_t* v = vt + (size_t)b * kHybN;
  const int32_t* p = pred + (size_t)b * kHybN;
  int acc = 0;
  while (acc < kHybN - 1 && p[acc] == v[acc + 1]) ++acc;
  for (int i = 0; i <= acc && e < MT; ++i) out[(size_t)b * MT + e++] = v[i];
  emitted[b] = e;
  accepted[b] += acc;
  steps[b] += 1;
  tlen[b] += acc + 1;
  v[0] = p[acc];  // correction, or the bonus token after a full accept
  acc_out[b] = acc;
}

struct HybSpec {
  HybModel* m = nullptr;
  int B = 0, MT = 0, P = 0;
  std::unique_ptr<HybState> s;
  Arena ar;
  int32_t *prompts = nullptr, *vt = nullptr, *pred = nullptr, *acc = nullptr, *out = nullptr;
  int *emitted = nullptr, *accepted = nullptr, *steps = nullptr;
  bf16_t *capt = nullptr, *mtp_hid = nullptr;
  cudaStream_t st = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  bool prefilled = false;
  int64_t replays = 0;
  ~HybSpec() {
    if (exec) cudaGraphExecDestroy(exec);
    if (graph) cudaGraphDestroy(graph);
    if (st) cudaStreamDestroy(st);
  }
};

// One MTP draft: hidden_in [B][H] (trunk capture or the previous MTP output),
// token vt[b][i-1] -> MTP layer -> hidden out (pre-norm) in mtp_hid ->
// output norm -> lm_head -> argmax into vt[b][i].
static int hyb_mtp_draft(HybSpec& sp, int i, const bf16_t* hidden_in, cudaStream_t st) {
  HybModel& m = *sp.m;
  HybState& s = *sp.s;
  const lmx_hybrid_config& c = m.c;
  const int B = sp.B, H = c.hidden;
  int rc = cuda_check(lmx_launch(embed_kernel, dim3(B), dim3(256), 0, st, true, (const int32_t*)sp.vt, 1, kHybN, i - 1,
                                 (const uint32_t*)m.embed.w, (const bf16_t*)m.embed.s, (const bf16_t*)m.embed.b, H,
                                 c.bits, s.emb, B),
                      "mtp embed");
  if (!rc)
    rc = cuda_check(lmx_launch(mtp_prep_kernel, dim3((2 * B + 7) / 8), dim3(256), 0, st, true, (const bf16_t*)s.emb,
                               hidden_in, H, (const bf16_t*)m.mtp_norm_e, (const bf16_t*)m.mtp_norm_h, c.eps, s.cat, B,
                               H),
                    "mtp prep");
  if (!rc) rc = hyb_qmm(s.cat, &m.mtp_fc, 1, H, s.h, H, B, 2 * H, c.bits, kPlain, nullptr, st);
  if (!rc) rc = launch_rms_norm(s.h, m.mtp.in_norm, s.xn, B, H, c.eps, st);
  if (!rc) rc = hyb_attention(m, s, m.mtp, s.mtp_kv->kv[0], B, 1, st);
  if (!rc) rc = hyb_moe(m, s, m.mtp, m.c.layers, B, st);
  if (!rc) rc = add_len(s.mtp_kv->len, B, 1, st);
  if (!rc) rc = cuda_check(cudaMemcpyAsync(sp.mtp_hid, s.h, (size_t)B * H * 2, cudaMemcpyDeviceToDevice, st), "mtp hid");
  if (!rc) rc = launch_rms_norm(s.h, m.mtp_norm, s.xn, B, H, c.eps, st);
  QmmCall hc;
  hc.x = s.xn;
  hc.mat[0] = m.lm_head.mat();
  hc.N = c.vocab;
  hc.y = s.logits;
  hc.ldy = c.vocab;
  hc.M = B;
  hc.K = H;
  hc.bits = c.bits;
  if (!rc) rc = launch_qmm(hc, st);
  // argmax of each row into vt[b][i]
  if (!rc) rc = launch_argmax(s.logits, B, c.vocab, sp.pred, st);
  if (!rc)
    rc = cuda_check(cudaMemcpy2DAsync(sp.vt + i, kHybN * 4, sp.pred, 4, 4, B, cudaMemcpyDeviceToDevice, st), "draft");
  return rc;
}

static int hyb_spec_step(HybSpec& sp) {
  HybModel& m = *sp.m;
  HybState& s = *sp.s;
  const int B = sp.B;
  cudaStream_t st = sp.st;
  int rc = cuda_check(cudaMemsetAsync(s.mtp_kv->len, 0, B * 4, st), "mtp reset");
  if (!rc) rc = hyb_mtp_draft(sp, 1, sp.capt, st);
  if (!rc) rc = hyb_mtp_draft(sp, 2, sp.mtp_hid, st);
  if (!rc) rc = hyb_forward(m, s, sp.vt, kHybN, 0, B, kHybN, s.logits, false, nullptr, st);
  if (!rc) rc = launch_argmax(s.logits, B * kHybN, m.c.vocab, sp.pred, st);
  if (!rc)
    rc = cuda_check(lmx_launch(hyb_accept_kernel, dim3((B + 127) / 128), dim3(128), 0, st, true, B, sp.MT, sp.vt,
                               (const int32_t*)sp.pred, sp.acc, s.kv ? s.kv->len : s.mtp_kv->len, sp.emitted,
                               sp.accepted, sp.steps, sp.out),
                    "hyb accept");
  if (!rc) rc = hyb_gdn_commit_all(m, s, B, kHybN, sp.acc, st);
  if (!rc)
    rc = cuda_check(lmx_launch(gather_rows_kernel, dim3(B), dim3(128), 0, st, true, sp.capt, (const bf16_t*)s.hid,
                               (const int32_t*)sp.acc, kHybN, m.c.hidden),
                    "capture hidden");
  return rc;
}

static int hyb_spec_create(HybModel* m, int B, int MT, int P, int kv_bits, HybSpec** out) {
  if (B < 1 || MT < 1 || P < 1) return set_error(LMX_ERR_INVALID, "hybrid spec: bad config");
  auto sp = std::make_unique<HybSpec>();
  sp->m = m;
  sp->B = B;
  sp->MT = MT;
  sp->P = P;
  const int cap = P + MT + kHybN + 8, Tmax = std::max(kHybN, kPrefillChunk);
  HybState* s = nullptr;
  int rc = hyb_state_create(*m, B, cap, kv_bits, Tmax, kHybN, B * kHybN, &s);
  if (rc) return rc;
  sp->s.reset(s);
  Arena& ar = sp->ar;
  const int H = m->c.hidden;
  if (!rc) rc = ar.alloc(&sp->prompts, (size_t)B * P);
  if (!rc) rc = ar.alloc(&sp->vt, (size_t)B * kHybN);
  if (!rc) rc = ar.alloc(&sp->pred, (size_t)B * kHybN);
  if (!rc) rc = ar.alloc(&sp->acc, (size_t)B);
  if (!rc) rc = ar.alloc(&sp->out, (size_t)B * MT);
  if (!rc) rc = ar.alloc(&sp->emitted, (size_t)B);
  if (!rc) rc = ar.alloc(&sp->accepted, (size_t)B);
  if (!rc) rc = ar.alloc(&sp->steps, (size_t)B);
  if (!rc) rc = ar.alloc(&sp->capt, (size_t)B * H);
  if (!rc) rc = ar.alloc(&sp->mtp_hid, (size_t)B * H);
  if (!rc) rc = cuda_check(cudaStreamCreateWithFlags(&sp->st, cudaStreamNonBlocking), "stream");
  if (rc) return rc;
  *out = sp.release();
  return LMX_OK;
}

static int hyb_reset(HybState& s, cudaStream_t st) {
  int rc = LMX_OK;
  if (s.kv) rc = cuda_check(cudaMemsetAsync(s.kv->len, 0, s.B * 4, st), "len");
  if (!rc) rc = cuda_check(cudaMemsetAsync(s.mtp_kv->len, 0, s.B * 4, st), "len");
  for (auto& g : s.gdn) {
    if (!rc) rc = cuda_check(cudaMemsetAsync(g.state, 0, s.state_floats * 4, st), "state");
    if (!rc) rc = cuda_check(cudaMemsetAsync(g.conv, 0, s.conv_elems * 2, st), "conv");
  }
  return rc;
}

// Run a [B, T] block (device tokens, row stride ld) through the trunk in
// chunks of kPrefillChunk, committing every token and advancing the
// attention lengths; the last chunk's last-position logits go to `logits`
// ([B][V]) when non-null and its hidden rows stay in s.hid.
static int hyb_prefill_tokens(const HybModel& m, HybState& s, const int32_t* tok, int ld, int T, bf16_t* logits,
                              int* last_tn, cudaStream_t st) {
  int rc = LMX_OK;
  for (int t0 = 0; t0 < T && !rc; t0 += kPrefillChunk) {
    const int tn = std::min(kPrefillChunk, T - t0);
    const bool last = t0 + tn >= T;
    rc = cuda_check(lmx_launch(set_int_kernel, dim3((s.B + 127) / 128), dim3(128), 0, st, false, s.tlast, s.B, tn - 1),
                    "tlast");
    if (!rc) rc = hyb_forward(m, s, tok, ld, t0, s.B, tn, last ? logits : nullptr, true, s.tlast, st);
    if (!rc && s.kv) rc = add_len(s.kv->len, s.B, tn, st);
    if (last && last_tn) *last_tn = tn;
  }
  return rc;
}

static int hyb_spec_prefill(HybSpec& sp, const int32_t* prompts_host) {
  HybModel& m = *sp.m;
  HybState& s = *sp.s;
  const int B = sp.B, P = sp.P;
  cudaStream_t st = sp.st;
  int rc = cuda_check(cudaMemcpyAsync(sp.prompts, prompts_host, (size_t)B * P * 4, cudaMemcpyHostToDevice, st),
                      "prompts");
  if (!rc) rc = hyb_reset(s, st);
  int tn = 0;
  if (!rc) rc = hyb_prefill_tokens(m, s, sp.prompts, P, P, s.logits, &tn, st);
  if (!rc) rc = launch_argmax(s.logits, B, m.c.vocab, sp.pred, st);
  if (!rc)  // d0 into vt[b][0]
    rc = cuda_check(cudaMemcpy2DAsync(sp.vt, kHybN * 4, sp.pred, 4, 4, B, cudaMemcpyDeviceToDevice, st), "d0");
  if (!rc)  // the trunk hidden at the last prompt position
    rc = cuda_check(lmx_launch(gather_rows_kernel, dim3(B), dim3(128), 0, st, true, sp.capt, (const bf16_t*)s.hid,
                               (const int32_t*)s.tlast, tn, m.c.hidden),
                    "capture hidden");
  for (int* p : {sp.emitted, sp.accepted, sp.steps})
    if (!rc) rc = cuda_check(cudaMemsetAsync(p, 0, B * 4, st), "counters");
  if (!rc) rc = cuda_check(cudaStreamSynchronize(st), "prefill");
  if (!rc) sp.prefilled = true;
  return rc;
}

static int hyb_spec_decode(HybSpec& sp, int use_graph, double* seconds) {
  if (!sp.prefilled) return set_error(LMX_ERR_INVALID, "hybrid spec: decode before prefill");
  cudaStream_t st = sp.st;
  int rc = LMX_OK;
  if (use_graph && !sp.exec) {
    rc = cuda_check(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal), "capture begin");
    if (rc) return rc;
    const int rc2 = hyb_spec_step(sp);
    cudaGraph_t g = nullptr;
    rc = cuda_check(cudaStreamEndCapture(st, &g), "capture end");
    if (rc2) {
      if (g) cudaGraphDestroy(g);
      return rc2;
    }
    if (rc) return rc;
    sp.graph = g;
    rc = cuda_check(cudaGraphInstantiate(&sp.exec, g, 0), "graph instantiate");
    if (rc) return rc;
  }
  std::vector<int> em(sp.B);
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaEventRecord(e0, st);
  sp.replays = 0;
  for (int it = 0; it < sp.MT + 1 && !rc; it += 4) {
    for (int k = 0; k < 4 && !rc; ++k, ++sp.replays)
      rc = use_graph ? cuda_check(cudaGraphLaunch(sp.exec, st), "graph launch") : hyb_spec_step(sp);
    if (rc) break;
    rc = cuda_check(cudaMemcpyAsync(em.data(), sp.emitted, sp.B * 4, cudaMemcpyDeviceToHost, st), "emitted");
    if (!rc) rc = cuda_check(cudaStreamSynchronize(st), "decode step");
    bool all = true;
    for (int b = 0; b < sp.B; ++b) all = all && em[b] >= sp.MT;
    if (all) break;
  }
  cudaEventRecord(e1, st);
  cudaEventSynchronize(e1);
  float ms = 0.0f;
  cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (seconds) *seconds = ms * 1e-3;
  if (!rc) {
    unsigned code = 0;
    cudaMemcpyFromSymbol(&code, g_lmx_kernel_error, sizeof(code));
    if (code) rc = set_error(LMX_ERR_CUDA, "kernel reported error 0x%x", code);
  }
  return rc;
}

// Time `iters` verify passes (the trunk over the current [d0, d1, d2], no
// commit) on the spec's stream after a prefill; bytes = algorithmic bytes of
// one pass: every layer's projections, router, shared expert and the
// experts its routing touched (counted from the pass's own routing), the
// lm_head, KV rows read and written, Gated DeltaNet states read and their
// 3 snapshots written.
static double qw_bytes(const QWeight& w, int bits) { return (double)w.N * w.K * bits / 8 + (double)w.N * (w.K / 64) * 4; }

static int hyb_spec_profile(HybSpec& sp, int iters, double* seconds, double* bytes) {
  if (!sp.prefilled) return set_error(LMX_ERR_INVALID, "hybrid profile before prefill");
  HybModel& m = *sp.m;
  HybState& s = *sp.s;
  const lmx_hybrid_config& c = m.c;
  const int B = sp.B, R = B * kHybN, bits = c.bits;
  cudaStream_t st = sp.st;
  auto once = [&]() { return hyb_forward(m, s, sp.vt, kHybN, 0, B, kHybN, s.logits, false, nullptr, st); };
  int rc = once();
  if (!rc) rc = cuda_check(cudaStreamSynchronize(st), "profile");
  if (rc) return rc;
  std::vector<int32_t> idx((size_t)c.layers * s.Rmax * c.top_k);
  rc = cuda_check(cudaMemcpy(idx.data(), s.idx, idx.size() * 4, cudaMemcpyDeviceToHost), "idx");
  std::vector<int> lens(B, 0);
  if (!rc && s.kv) rc = cuda_check(cudaMemcpy(lens.data(), s.kv->len, B * 4, cudaMemcpyDeviceToHost), "len");
  if (rc) return rc;
  double by = qw_bytes(m.lm_head, bits) + (double)R * c.hidden * 2;
  // (expert parallelism: this rank's experts only)
  const double per_expert = qw_bytes(m.L[0].eg, bits) / m.per * 2 + qw_bytes(m.L[0].ed, bits) / m.per;
  for (int l = 0; l < c.layers; ++l) {
    const HybLayer& L = m.L[l];
    for (const QWeight* q : {&L.q, &L.k, &L.v, &L.qg, &L.o, &L.wqkv, &L.wz, &L.wb, &L.wa, &L.wout, &L.router, &L.sg,
                             &L.su, &L.sd, &L.sgate})
      if (q->w) by += qw_bytes(*q, bits);
    std::vector<char> seen(c.experts, 0);
    int uniq = 0;
    for (int r = 0; r < R * c.top_k; ++r) {
      const int e = idx[(size_t)l * s.Rmax * c.top_k + r];
      if (e >= m.e_lo && e < m.e_lo + m.per && !seen[e]) { seen[e] = 1; ++uniq; }
    }
    by += uniq * per_expert;
    if (L.attn) {
      const double row = (double)c.kv_heads * kHeadDim * (s.kv->bits == 16 ? 2.0 : s.kv->bits / 8.0 + 4.0 / 64) * 2;
      for (int b = 0; b < B; ++b) by += row * (lens[b] + kHybN);
    } else {
      by += (double)B * c.lin_v_heads * kGdnD * kGdnD * 4 * (1 + kHybN);
    }
  }
  for (int i = 0; i < 2 && !rc; ++i) rc = once();
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaEventRecord(e0, st);
  nvtxRangePushA("lmx_verify_pass");
  for (int i = 0; i < iters && !rc; ++i) rc = once();
  nvtxRangePop();
  cudaEventRecord(e1, st);
  if (!rc) rc = cuda_check(cudaEventSynchronize(e1), "profile");
  float ms = 0;
  cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (seconds) *seconds = ms * 1e-3 / (iters > 0 ? iters : 1);
  if (bytes) *bytes = by;
  return rc;
}

struct HybStateHandle {
  HybModel* m = nullptr;
  std::unique_ptr<HybState> s;
  int T = 0;
};

}  // namespace lmx

using namespace lmx;

extern "C" int lmx_hybrid_create(const lmx_hybrid_config* cfg, uint64_t seed, void** model) {
  if (!cfg || !model) return set_error(LMX_ERR_INVALID, "hybrid_create: null argument");
  HybModel* m = nullptr;
  int rc = hyb_create(*cfg, seed, nullptr, &m);
  if (!rc) *model = m;
  return rc;
}

extern "C" int lmx_hybrid_create_ep(const lmx_hybrid_config* cfg, uint64_t seed, void* comm, void** model) {
  if (!cfg || !model) return set_error(LMX_ERR_INVALID, "hybrid_create_ep: null argument");
  HybModel* m = nullptr;
  int rc = hyb_create(*cfg, seed, (TpComm*)comm, &m);
  if (!rc) *model = m;
  return rc;
}

extern "C" int lmx_hybrid_free(void* model) {
  delete (HybModel*)model;
  return LMX_OK;
}

extern "C" int lmx_hybrid_state_create(void* model, int batch, int capacity, int kv_bits, int max_tokens_per_forward,
                                       void** state) {
  HybModel* m = (HybModel*)model;
  if (!m || !state || max_tokens_per_forward < 1) return set_error(LMX_ERR_INVALID, "hybrid_state_create: bad arguments");
  auto h = std::make_unique<HybStateHandle>();
  h->m = m;
  h->T = max_tokens_per_forward;
  HybState* s = nullptr;
  int rc = hyb_state_create(*m, batch, capacity, kv_bits, std::max(max_tokens_per_forward, kPrefillChunk),
                            kHybN, batch * max_tokens_per_forward, &s);
  if (rc) return rc;
  h->s.reset(s);
  rc = hyb_reset(*s, 0);
  if (!rc) rc = cuda_check(cudaDeviceSynchronize(), "hybrid state");
  if (rc) return rc;
  *state = h.release();
  return LMX_OK;
}

extern "C" int lmx_hybrid_state_free(void* state) {
  delete (HybStateHandle*)state;
  return LMX_OK;
}

extern "C" int lmx_hybrid_forward(void* model, void* state, const int32_t* tokens_host, int B, int T,
                                  void* logits_host) {
  HybModel* m = (HybModel*)model;
  HybStateHandle* h = (HybStateHandle*)state;
  if (!m || !h || h->m != m || !tokens_host || T < 1 || T > h->T || B != h->s->B)
    return set_error(LMX_ERR_INVALID, "hybrid_forward: bad arguments");
  HybState& s = *h->s;
  int32_t* tok = nullptr;
  Arena ar;
  int rc = ar.alloc(&tok, (size_t)B * T);
  if (!rc) rc = cuda_check(cudaMemcpy(tok, tokens_host, (size_t)B * T * 4, cudaMemcpyHostToDevice), "tokens");
  if (!rc) rc = cuda_check(lmx_launch(set_int_kernel, dim3((B + 127) / 128), dim3(128), 0, (cudaStream_t)0, false,
                                      s.tlast, B, T - 1),
                           "tlast");
  if (!rc) rc = hyb_forward(*m, s, tok, T, 0, B, T, logits_host ? s.logits : nullptr, false, s.tlast, 0);
  if (!rc && s.kv) rc = add_len(s.kv->len, B, T, 0);
  if (!rc) rc = cuda_check(cudaDeviceSynchronize(), "hybrid forward");
  if (!rc && logits_host)
    rc = cuda_check(cudaMemcpy(logits_host, s.logits, (size_t)B * T * m->c.vocab * 2, cudaMemcpyDeviceToHost), "logits");
  if (!rc) {
    unsigned code = 0;
    cudaMemcpyFromSymbol(&code, g_lmx_kernel_error, sizeof(code));
    if (code) rc = set_error(LMX_ERR_CUDA, "kernel reported error 0x%x", code);
  }
  return rc;
}

extern "C" int lmx_hybrid_spec_create(void* model, int batch, int max_tokens, int prompt_len, int kv_bits,
                                      void** spec) {
  if (!model || !spec) return set_error(LMX_ERR_INVALID, "hybrid_spec_create: null argument");
  HybSpec* sp = nullptr;
  int rc = hyb_spec_create((HybModel*)model, batch, max_tokens, prompt_len, kv_bits, &sp);
  if (!rc) *spec = sp;
  return rc;
}

extern "C" int lmx_hybrid_spec_prefill(void* spec, const int32_t* prompts_host) {
  if (!spec || !prompts_host) return set_error(LMX_ERR_INVALID, "hybrid_spec_prefill: null argument");
  return hyb_spec_prefill(*(HybSpec*)spec, prompts_host);
}

extern "C" int lmx_hybrid_spec_decode(void* spec, int use_graph, double* seconds) {
  if (!spec) return set_error(LMX_ERR_INVALID, "hybrid_spec_decode: null argument");
  return hyb_spec_decode(*(HybSpec*)spec, use_graph, seconds);
}

extern "C" int lmx_hybrid_spec_result(void* spec, int32_t* out_host, int64_t* stats_host) {
  HybSpec* sp = (HybSpec*)spec;
  if (!sp) return set_error(LMX_ERR_INVALID, "hybrid_spec_result: null argument");
  const int B = sp->B;
  int rc = LMX_OK;
  if (out_host)
    rc = cuda_check(cudaMemcpy(out_host, sp->out, (size_t)B * sp->MT * 4, cudaMemcpyDeviceToHost), "out");
  if (!rc && stats_host) {
    std::vector<int> st(B), ac(B), em(B);
    rc = cuda_check(cudaMemcpy(st.data(), sp->steps, B * 4, cudaMemcpyDeviceToHost), "stats");
    if (!rc) rc = cuda_check(cudaMemcpy(ac.data(), sp->accepted, B * 4, cudaMemcpyDeviceToHost), "stats");
    if (!rc) rc = cuda_check(cudaMemcpy(em.data(), sp->emitted, B * 4, cudaMemcpyDeviceToHost), "stats");
    int64_t a = 0, b2 = 0, c = 0;
    for (int b = 0; b < B; ++b) { a += st[b]; b2 += ac[b]; c += em[b]; }
    stats_host[0] = a;
    stats_host[1] = a * (kHybN - 1);
    stats_host[2] = b2;
    stats_host[3] = c;
    stats_host[4] = sp->replays;
  }
  return rc;
}

extern "C" int lmx_hybrid_spec_free(void* spec) {
  delete (HybSpec*)spec;
  return LMX_OK;
}

extern "C" int lmx_hybrid_spec_profile(void* spec, int iters, double* seconds, double* bytes) {
  if (!spec) return set_error(LMX_ERR_INVALID, "hybrid_spec_profile: null argument");
  return hyb_spec_profile(*(HybSpec*)spec, iters, seconds, bytes);
}

extern "C" int lmx_hybrid_spec_step_launches(void* spec, int64_t* launches) {
  HybSpec* sp = (HybSpec*)spec;
  if (!sp || !launches || !sp->graph) return set_error(LMX_ERR_INVALID, "hybrid_spec_step_launches: no graph yet");
  size_t nodes = 0;
  int rc = cuda_check(cudaGraphGetNodes(sp->graph, nullptr, &nodes), "graph nodes");
  *launches = (int64_t)nodes;
  return rc;
}
