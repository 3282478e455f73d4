// gdn_moe.cuh -- configuration 4's hot ops (Qwen3-Next-style hybrid
// decoder): the Gated DeltaNet verify step with per-token state snapshots
// and its rollback, the MoE router and the routed SwiGLU experts.
//
// Reference: Qwen3NextGatedDeltaNet::operator() (src/llm/models/
// qwen3_next.cpp:216-403): in_proj_qkvz / in_proj_ba -> depthwise causal
// conv1d (kernel 4) over q|k|v with a 3-row state, SiLU -> q, k RMSNorm with
// weights 1/Dk and 1/sqrt(Dk) -> beta = sigmoid(b), g = exp(-exp(A_log) *
// softplus(a + dt_bias)) (gated_delta.cpp:603-633) -> recurrence per value
// head (gated_delta.cpp:634-650, gated_delta_ops_seq :1067-1118):
//   S = S * g;  kv = S k;  delta = (v - kv) * beta;  S += delta k^T;  y = S q
// -> gated RMSNorm rms_norm(y, w) * silu(z) (gated_delta.cpp:948-971) ->
// out_proj.  MambaCache rollback keeps the state after the last accepted
// token (kv_cache.h:178-288).  MoE: Qwen3NextSparseMoeBlock (qwen3_next.cpp:
// 452-490): top-k of softmax(router logits), scores renormalised over the k
// (= softmax over the k selected logits, moe_route gated_delta.cpp:973-999),
// SwitchGLU experts (switch_layers.cpp:200-245), score-weighted sum.
//
// Canonical orders (shared with the oracle, bit-exact):
//  * expert dot products (qd_dot below): K in 16-element chunks, lane l of a
//    warp owns chunks l, l+32, ...; per chunk p = fma chain of q_j * x_j,
//    xs = add chain of x_j, e = fma(scale, p, bias * xs); lane sum in chunk
//    order from 0; xor butterfly 16, 8, 4, 2, 1.
//  * recurrence: the state is fp32 (the reference keeps it in bf16); two
//    threads per state row dv, each owning 64 dk; every reduction over dk is
//    an fma chain over the thread's 64 (ascending) plus one add of the
//    partner's partial (lower half first).
#pragma once
#include "attn.cuh"
#include "lmx_common.cuh"
#include "norm_argmax.cuh"

namespace lmx {

static constexpr int kGdnD = 128;  // Dk = Dv
static constexpr int kGdnKS = 4;   // conv kernel

// Process-wide: Gated DeltaNet state snapshots (and hence committed states)
// rounded to bf16 as the reference stores them (1, default) or kept fp32 (0).
static int g_gdn_state_bf16 = 1;

struct GdnArgs {
  int B, T, Hk, Hv;
  const bf16_t* qkv;      // [B][T][CD], CD = 2*Hk*128 + Hv*128
  const bf16_t* z;        // [B][T][Hv*128]
  const bf16_t* b;        // [B][T][Hv]
  const bf16_t* a;        // [B][T][Hv]
  const bf16_t* conv_w;   // [CD][4]
  const float* a_log;     // [Hv]
  const bf16_t* dt_bias;  // [Hv]
  const bf16_t* norm_w;   // [128]
  float eps;
  const bf16_t* conv_state;  // [B][3][CD]
  const float* state;        // [B][Hv][128][128]
  float* snap;               // [B][snap_T][Hv][128][128]: states after the last snap_T tokens
  int snap_T;                // T (every token) or 1 (only the last, e.g. a prefill chunk)
  int state_bf16 = 1;        // snapshots rounded to bf16, as the reference stores its states
  bf16_t* out;               // [B][T][Hv*128]
  bf16_t* qn;                // scratch [B][T][Hk][128] normalised q
  bf16_t* kn;                // scratch [B][T][Hk][128] normalised k
  bf16_t* vc;                // scratch [B][T][Hv][128] conv'd v
  float* beta;               // scratch [B][T][Hv]
  float* gdecay;             // scratch [B][T][Hv]
};

// log(x) for normal x > 0: x = m 2^e with m in [sqrt(1/2), sqrt(2)),
// log m = 2 atanh(u), u = (m-1)/(m+1), by its odd series to u^11 (Horner in
// u^2), plus e ln 2 (ln 2 split in a 16-bit head and a tail).
LMX_DEV float log_c(float x) {
  const uint32_t bits = __float_as_uint(x);
  int e = (int)(bits >> 23) - 127;
  float m = __uint_as_float((bits & 0x7FFFFFu) | 0x3F800000u);
  if (m > 1.41421356f) {
    m = __fmul_rn(m, 0.5f);
    e += 1;
  }
  const float u = __fdiv_rn(__fsub_rn(m, 1.0f), __fadd_rn(m, 1.0f));
  const float u2 = __fmul_rn(u, u);
  float p = 0.0909090909f;  // 1/11
  p = __fmaf_rn(p, u2, 0.111111111f);
  p = __fmaf_rn(p, u2, 0.142857143f);
  p = __fmaf_rn(p, u2, 0.2f);
  p = __fmaf_rn(p, u2, 0.333333333f);
  p = __fmaf_rn(p, u2, 1.0f);
  const float r = __fmul_rn(__fmul_rn(2.0f, u), p);
  const float fe = (float)e;
  return __fmaf_rn(fe, 0.693145752f, __fmaf_rn(fe, 1.42860677e-06f, r));
}

// softplus(x) = log(1 + exp(x)) (x > 20: x)
LMX_DEV float softplus_c(float x) { return x > 20.0f ? x : log_c(__fadd_rn(1.0f, exp_c(x))); }

// Depthwise causal conv + SiLU over one 8-channel chunk of token t.
// window rows: conv_state[0..2] then tokens 0..T-1; y = sum_i w[c][i]*row[t+i]
// (fma chain i = 0..3), out = bf16(silu) with bf16 after the conv sum,
// after sigmoid and after the product (MLX materialises each op).
LMX_DEV void gdn_conv8(const GdnArgs& a, int b, int t, int c0, int CD, float (&o)[8]) {
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int c = c0 + e;
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < kGdnKS; ++i) {
      const int r = t + i;  // window row: < 3 from the state, else token r - 3
      const float x = r < kGdnKS - 1 ? bf2f(a.conv_state[((size_t)b * (kGdnKS - 1) + r) * CD + c])
                                     : bf2f(a.qkv[((size_t)b * a.T + (r - (kGdnKS - 1))) * CD + c]);
      acc = __fmaf_rn(bf2f(a.conv_w[(size_t)c * kGdnKS + i]), x, acc);
    }
    const float y = bf2f(f2bf(acc));
    const float sg = bf2f(f2bf(sigmoid_c(y)));
    o[e] = bf2f(f2bf(__fmul_rn(y, sg)));
  }
}

// Prep: one warp per (b, t, head slot): slots [0, Hk) -> q head, [Hk, 2Hk)
// -> k head (conv, SiLU, RMSNorm with weight 1/Dk resp. 1/sqrt(Dk), eps
// 1e-6), [2Hk, 2Hk+Hv) -> v head (conv, SiLU) plus beta / g of that head.
__global__ void __launch_bounds__(256) gdn_prep_kernel(GdnArgs a) {
  grid_wait();
  grid_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int slots = 2 * a.Hk + a.Hv;
  const long long task = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (task >= (long long)a.B * a.T * slots) return;
  const int slot = (int)(task % slots);
  const int bt = (int)(task / slots), b = bt / a.T, t = bt % a.T;
  const int CD = 2 * a.Hk * kGdnD + a.Hv * kGdnD;
  const int c0 = slot * kGdnD + 8 * (lane & 15);  // lanes 16..31 mirror 0..15
  float o[8];
  gdn_conv8(a, b, t, c0, CD, o);
  if (slot < 2 * a.Hk) {
    // canonical RMSNorm factor over the 128 values (chunks of 8 by lane)
    float p = 0.0f;
    if (lane < 16)
#pragma unroll
      for (int e = 0; e < 8; ++e) p = __fmaf_rn(o[e], o[e], p);
    p = warp_sum_xor(p, 16, 1);
    const float f = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(p, (float)kGdnD), 1e-6f)));
    // weights: q 1/Dk, k 1/sqrt(Dk), as bf16
    const float w = slot < a.Hk ? bf2f(f2bf(1.0f / kGdnD)) : bf2f(f2bf(0.08838834764831845f));
    if (lane < 16) {
      float r[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) r[e] = __fmul_rn(__fmul_rn(o[e], f), w);
      bf16_t* dst = (slot < a.Hk ? a.qn + (((size_t)b * a.T + t) * a.Hk + slot) * kGdnD
                                 : a.kn + (((size_t)b * a.T + t) * a.Hk + slot - a.Hk) * kGdnD) +
                    8 * lane;
      *reinterpret_cast<uint4*>(dst) = pack8(r);
    }
  } else {
    const int h = slot - 2 * a.Hk;
    if (lane < 16)
      *reinterpret_cast<uint4*>(a.vc + (((size_t)b * a.T + t) * a.Hv + h) * kGdnD + 8 * lane) = pack8(o);
    if (lane == 0) {
      const size_t i = ((size_t)b * a.T + t) * a.Hv + h;
      const float bv = bf2f(a.b[i]), av = bf2f(a.a[i]);
      a.beta[i] = bf2f(f2bf(sigmoid_c(bv)));
      const float sp = softplus_c(__fadd_rn(av, bf2f(a.dt_bias[h])));
      a.gdecay[i] = bf2f(f2bf(exp_c(-__fmul_rn(exp_c(a.a_log[h]), sp))));
    }
  }
}

// Recurrence + gated RMSNorm: one CTA of 256 threads per (b, value head);
// thread 2*dv + half owns S[dv][64*half .. 64*half+63] in registers.
__global__ void __launch_bounds__(256) gdn_recur_kernel(GdnArgs a) {
  __shared__ float qs[kGdnD], ks[kGdnD];
  __shared__ __align__(16) bf16_t yb[kGdnD];
  __shared__ float s_f;
  grid_wait();
  grid_launch_dependents();
  const int h = blockIdx.x, b = blockIdx.y, hk = h / (a.Hv / a.Hk);
  const int tid = threadIdx.x, dv = tid >> 1, half = tid & 1;
  float S[64];
  const float* s0 = a.state + (((size_t)b * a.Hv + h) * kGdnD + dv) * kGdnD + 64 * half;
#pragma unroll
  for (int j = 0; j < 64; j += 4) {
    const float4 v = *reinterpret_cast<const float4*>(s0 + j);
    S[j] = v.x; S[j + 1] = v.y; S[j + 2] = v.z; S[j + 3] = v.w;
  }
  for (int t = 0; t < a.T; ++t) {
    const size_t bt = (size_t)b * a.T + t;
    __syncthreads();
    if (tid < kGdnD) {
      qs[tid] = bf2f(a.qn[(bt * a.Hk + hk) * kGdnD + tid]);
      ks[tid] = bf2f(a.kn[(bt * a.Hk + hk) * kGdnD + tid]);
    }
    __syncthreads();
    const float g = a.gdecay[bt * a.Hv + h], be = a.beta[bt * a.Hv + h];
    const float v = bf2f(a.vc[(bt * a.Hv + h) * kGdnD + dv]);
    // S *= g;  kv = S k
    float kv = 0.0f;
#pragma unroll
    for (int j = 0; j < 64; ++j) {
      S[j] = __fmul_rn(S[j], g);
      kv = __fmaf_rn(S[j], ks[64 * half + j], kv);
    }
    const float other = __shfl_xor_sync(0xffffffffu, kv, 1);
    kv = half ? __fadd_rn(other, kv) : __fadd_rn(kv, other);
    const float delta = __fmul_rn(__fsub_rn(v, kv), be);
    // S += delta k^T;  y = S q
    float y = 0.0f;
#pragma unroll
    for (int j = 0; j < 64; ++j) {
      S[j] = __fmaf_rn(delta, ks[64 * half + j], S[j]);
      y = __fmaf_rn(S[j], qs[64 * half + j], y);
    }
    const float oy = __shfl_xor_sync(0xffffffffu, y, 1);
    y = half ? __fadd_rn(oy, y) : __fadd_rn(y, oy);
    const int ts = t - (a.T - a.snap_T);  // snapshot slot of token t
    if (a.snap && ts >= 0) {
      float* sn = a.snap + (((((size_t)b * a.snap_T + ts) * a.Hv + h) * kGdnD + dv) * kGdnD) + 64 * half;
      // the reference keeps the state in fp32 within a block and stores it
      // (the per-token states and the block's final state) as bf16
      // (src/common/gated_delta.cpp:93, :162-172): state_bf16 rounds the
      // snapshots the same way; the running state stays fp32
      if (a.state_bf16) {
#pragma unroll
        for (int j = 0; j < 64; j += 4)
          *reinterpret_cast<float4*>(sn + j) = make_float4(bf2f(f2bf(S[j])), bf2f(f2bf(S[j + 1])),
                                                           bf2f(f2bf(S[j + 2])), bf2f(f2bf(S[j + 3])));
      } else {
#pragma unroll
        for (int j = 0; j < 64; j += 4)
          *reinterpret_cast<float4*>(sn + j) = make_float4(S[j], S[j + 1], S[j + 2], S[j + 3]);
      }
    }
    // gated RMSNorm of the head's y (bf16), canonical warp factor
    if (!half) yb[dv] = f2bf(y);
    __syncthreads();
    if (tid < 32) {
      const float f = rms_factor_warp(yb, kGdnD, a.eps, tid);
      if (tid == 0) s_f = f;
    }
    __syncthreads();
    if (!half) {
      const float nv = bf2f(f2bf(__fmul_rn(__fmul_rn(bf2f(yb[dv]), s_f), bf2f(a.norm_w[dv]))));
      const float zv = bf2f(a.z[(bt * a.Hv + h) * kGdnD + dv]);
      const float sz = bf2f(f2bf(__fmul_rn(zv, bf2f(f2bf(sigmoid_c(zv))))));
      a.out[(bt * a.Hv + h) * kGdnD + dv] = f2bf(__fmul_rn(sz, nv));
    }
  }
}

// MambaCache rollback_spec: state[b] = snap[b][acc[b]]; conv_state[b] =
// the 3 window rows ending at token acc[b] (old state rows, then tokens);
// acc[b] < 0 leaves sequence b unchanged (a finished sequence).
// Grid (B, Hv + 1): blocks y < Hv copy one head's state, y == Hv the conv rows.
__global__ void __launch_bounds__(256) gdn_commit_kernel(GdnArgs a, const int32_t* acc, float* state,
                                                         bf16_t* conv_state_out) {
  grid_wait();
  grid_launch_dependents();
  const int b = blockIdx.x, h = blockIdx.y;
  if (acc[b] < 0) return;
  const int t = min(acc[b], a.T - 1);
  const int ts = max(t - (a.T - a.snap_T), 0);  // snapshot slot of token t
  if (h < a.Hv) {
    const float4* src = reinterpret_cast<const float4*>(a.snap + ((((size_t)b * a.snap_T + ts) * a.Hv + h) * kGdnD) * kGdnD);
    float4* dst = reinterpret_cast<float4*>(state + (((size_t)b * a.Hv + h) * kGdnD) * kGdnD);
    for (int i = threadIdx.x; i < kGdnD * kGdnD / 4; i += blockDim.x) dst[i] = src[i];
    return;
  }
  const int CD = 2 * a.Hk * kGdnD + a.Hv * kGdnD;
  // new window row r (0..2) = combined row t + 1 + r of [state rows, tokens];
  // one thread per channel writes rows in increasing order, so an in-place
  // update (conv_state_out == conv_state) reads each source row before it is
  // overwritten (the source index is always above the destination)
  for (int c = threadIdx.x; c < CD; c += blockDim.x)
    for (int r = 0; r < kGdnKS - 1; ++r) {
      const int src = t + 1 + r;
      const bf16_t v = src < kGdnKS - 1 ? a.conv_state[((size_t)b * (kGdnKS - 1) + src) * CD + c]
                                        : a.qkv[((size_t)b * a.T + src - (kGdnKS - 1)) * CD + c];
      conv_state_out[((size_t)b * (kGdnKS - 1) + r) * CD + c] = v;
    }
}

// ---------------------------------------------------------------------------
// MoE router: one warp per row; k rounds of a warp argmax over the row's
// logits (highest value, lowest index on ties) excluding the experts already
// picked; w_j = exp(l_j - l_0) / sum (slot order, fma-free adds from 0).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) moe_route_kernel(const bf16_t* logits, int rows, int E, int k, int32_t* idx,
                                                        float* w) {
  grid_wait();
  grid_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const bf16_t* l = logits + (size_t)row * E;
  uint32_t taken[16] = {};  // bit i of word j: expert lane + 32*(32*j + i) picked (E <= 16384)
  float lv[16];
  int li[16];
  for (int j = 0; j < k; ++j) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int e = lane, n = 0; e < E; e += 32, ++n)
      if (!((taken[n >> 5] >> (n & 31)) & 1u)) {
        const float v = bf2f(l[e]);
        if (v == v && am_better(v, e, bv, bi)) { bv = v; bi = e; }
      }
    am_warp(bv, bi);
    if (bi != 0x7fffffff && (bi & 31) == lane) {
      const int n = bi >> 5;
      taken[n >> 5] |= 1u << (n & 31);
    }
    lv[j] = bv;
    li[j] = bi == 0x7fffffff ? 0 : bi;
  }
  if (lane == 0) {
    float e0[16], z = 0.0f;
    for (int j = 0; j < k; ++j) {
      e0[j] = exp_c(__fsub_rn(lv[j], lv[0]));
      z = __fadd_rn(z, e0[j]);
    }
    for (int j = 0; j < k; ++j) {
      idx[(size_t)row * k + j] = li[j];
      w[(size_t)row * k + j] = __fdiv_rn(e0[j], z);
    }
  }
}

// Canonical quantized dot (see the header) of packed row `wr` (K values,
// `bits`-bit, group 64, scales / biases sr / br) with x (fp32, K) by one warp.
// x is staged transposed in shared memory: element 16c + j at xt[j*(K/16) + c]
// (consecutive lanes read consecutive words).
template <int BITS>
LMX_DEV float qd_dot(const uint32_t* wr, const bf16_t* sr, const bf16_t* br, const float* xt, int K, int lane) {
  constexpr int WPC = 16 * BITS / 32;  // words per 16-element chunk
  const int NC = K / 16;
  float acc = 0.0f;
  for (int c = lane; c < NC; c += 32) {
    uint32_t wv[WPC];
    if (BITS == 4) {
      const uint2 v = *reinterpret_cast<const uint2*>(wr + c * WPC);
      wv[0] = v.x;
      wv[WPC - 1] = v.y;
    } else {
      const uint4 v = *reinterpret_cast<const uint4*>(wr + c * WPC);
      wv[0] = v.x; wv[1 % WPC] = v.y; wv[2 % WPC] = v.z; wv[3 % WPC] = v.w;
    }
    float p = 0.0f, xs = 0.0f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint32_t q = (wv[j * BITS / 32] >> ((j * BITS) & 31)) & ((1u << BITS) - 1u);
      const float xv = xt[j * NC + c];
      p = __fmaf_rn((float)q, xv, p);
      xs = __fadd_rn(xs, xv);
    }
    const int g = c >> 2;
    acc = __fadd_rn(acc, __fmaf_rn(bf2f(sr[g]), p, __fmul_rn(bf2f(br[g]), xs)));
  }
  return warp_sum_xor(acc, 16, 1);
}

struct MoeArgs {
  int M, H, I, E, k;
  const bf16_t* x;       // [M][H]
  const int32_t* idx;    // [M][k]
  const float* w;        // [M][k]
  const uint32_t *gw, *uw, *dw;  // [E][I][H*b/32], [E][I][H*b/32], [E][H][I*b/32]
  const bf16_t *gs, *gb, *us, *ub, *ds, *db;
  bf16_t* act;           // [M][k][I]
  bf16_t* y;             // [M][H]
  unsigned* err;         // device error word (expert index out of range)
  // expert parallelism: this rank holds experts [e_lo, e_hi) (the weight
  // pointers start at expert e_lo) and writes each owned slot's down output
  // bf16 [M][k][H] to slot_out instead of combining (ep_combine_kernel)
  int e_lo = 0, e_hi = 1 << 30;
  bf16_t* slot_out = nullptr;
};

// Local expert of slot s (index into this rank's weights), or -1 when it is
// out of range (the error word set) or, expert-parallel (EP), another rank's
// expert.  EP is a template switch so that the one-GPU kernels carry none of
// the sharding logic (measured: with the range test and the slot-output
// branch compiled in, the one-GPU routed experts took 334 instead of 223 us
// at configuration 4's verify shape).
template <bool EP>
LMX_DEV int moe_expert(const MoeArgs& a, size_t s) {
  const int e = a.idx[s];
  if (e < 0 || e >= a.E) {
    if (a.err) atomicExch(a.err, 0x81u);
    return -1;
  }
  if (!EP) return e;
  if (e < a.e_lo || e >= a.e_hi) return -1;
  return e - a.e_lo;
}

// gate / up: CTA = (slot m*k+j, block of 64 expert rows); warp per row pair
// (gate row i, up row i); act = swiglu(bf16(gate), bf16(up)).
template <int BITS, bool EP>
__global__ void __launch_bounds__(256) moe_gateup_kernel(MoeArgs a) {
  extern __shared__ float mx_smem[];  // x of the slot's token, fp32 [H]
  grid_wait();
  grid_launch_dependents();
  const int slot = blockIdx.y, m = slot / a.k;
  const int e = moe_expert<EP>(a, slot);
  if (e < 0) return;
  const int NC = a.H / 16;
  for (int i = threadIdx.x; i < a.H; i += blockDim.x) mx_smem[(i & 15) * NC + (i >> 4)] = bf2f(a.x[(size_t)m * a.H + i]);
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const size_t wpr = (size_t)a.H * BITS / 32, gpr = a.H / 64;
  for (int r = blockIdx.x * 64 + warp; r < min(a.I, (int)blockIdx.x * 64 + 64); r += 8) {
    const size_t row = (size_t)e * a.I + r;
    const float gv = qd_dot<BITS>(a.gw + row * wpr, a.gs + row * gpr, a.gb + row * gpr, mx_smem, a.H, lane);
    const float uv = qd_dot<BITS>(a.uw + row * wpr, a.us + row * gpr, a.ub + row * gpr, mx_smem, a.H, lane);
    if (lane == 0) a.act[(size_t)slot * a.I + r] = swiglu_c(f2bf(gv), f2bf(uv));
  }
}

// down + combine: CTA = (token m, block of 64 output rows); for each slot j
// in order, warp per output row: v = bf16(down_e row . act[m][j]);
// y = bf16(fma chain over j of w[m][j] * v from 0).
template <int BITS, bool EP>
__global__ void __launch_bounds__(256) moe_down_kernel(MoeArgs a) {
  extern __shared__ float mx_smem[];  // act of the token's k slots, fp32 [k][I]
  grid_wait();
  grid_launch_dependents();
  const int m = blockIdx.y;
  const int NC = a.I / 16;
  for (int i = threadIdx.x; i < a.k * a.I; i += blockDim.x) {
    const int j = i / a.I, r = i % a.I;  // slot, element
    mx_smem[(size_t)j * a.I + (r & 15) * NC + (r >> 4)] = bf2f(a.act[(size_t)m * a.k * a.I + i]);
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const size_t wpr = (size_t)a.I * BITS / 32, gpr = a.I / 64;
  for (int r = blockIdx.x * 64 + warp; r < min(a.H, (int)blockIdx.x * 64 + 64); r += 8) {
    float acc = 0.0f;
    for (int j = 0; j < a.k; ++j) {
      const int e = moe_expert<EP>(a, (size_t)m * a.k + j);
      if (e < 0) continue;
      const size_t row = (size_t)e * a.H + r;
      const bf16_t v = f2bf(qd_dot<BITS>(a.dw + row * wpr, a.ds + row * gpr, a.db + row * gpr,
                                         mx_smem + (size_t)j * a.I, a.I, lane));
      if (EP) {
        if (lane == 0) a.slot_out[((size_t)m * a.k + j) * a.H + r] = v;
      } else {
        acc = __fmaf_rn(a.w[(size_t)m * a.k + j], bf2f(v), acc);
      }
    }
    if (lane == 0 && !EP) a.y[(size_t)m * a.H + r] = f2bf(acc);
  }
}

}  // namespace lmx
