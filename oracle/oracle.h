/*
 * oracle.h -- CPU restatement of lemon-mlx-engine's speculative-decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (the lemon-mlx-engine_b200
 * package, include/lmx.h, the C ABI) links, loads or calls this code.  It is
 * used by tests/, by __graft_entry__.smoke() and by bench.py's cpu_baseline /
 * `--impl reference` leg, always as the checker or the timed CPU baseline,
 * never as the thing measured or shipped.
 *
 * Parity status: the reference's arithmetic lives in MLX (fetched from an
 * unpinned branch, CMakeLists.txt:32-40), which is not present here and cannot
 * be built, so parity against MLX itself is UNPINNED for the fp32 reduction
 * order, the quantize() rounding rule, exp/sin/cos and argmax tie-breaking.
 * What IS pinned against the reference's own files:
 *   - 4/8-bit affine packing order (LSB-first) and w = q*scale + bias:
 *       debug_numerical_trace.py:67-100, debug_layer0_reference.py:53-82
 *     (golden vectors made by importing those functions: tests/golden/)
 *   - rms_norm formula: debug_numerical_trace.py:103-108
 *   - NeoX RoPE definition: examples/test_device_rope.cpp:15-46
 *   - SDPA = fp32 softmax(q k^T * scale + causal offset mask) v:
 *       examples/test_sdpa_ref.cpp:81-100, src/common/kv_cache.cpp:15-30
 *   - ArgMax known answers: tests/test_generate.cpp:21-36,162-172
 *   - greedy MTP/speculative accept rule and emission order:
 *       src/common/generate.cpp:669-933, :968-1045
 *   - KV set_position rollback: src/common/kv_cache.cpp:112-142,301-377
 *
 * Where MLX leaves the order of fp32 operations open, this file fixes one
 * canonical order (documented per function below) that the CUDA-core kernels
 * follow operation for operation, so GPU and oracle results are bit-identical
 * on those paths.  Tensor-core (tcgen05) paths are compared with a tolerance.
 *
 * All bf16 tensors are passed as uint16_t bit patterns.
 */
#ifndef LMX_ORACLE_H
#define LMX_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- scalar numerics ---- */
float orc_exp(float x);                 /* Cody-Waite + degree-7 Taylor, exact op order */
uint16_t orc_f32_to_bf16(float x);      /* round to nearest even */
float orc_bf16_to_f32(uint16_t h);

/* ---- deterministic synthetic data (Philox4x32-10 counter RNG) ---- */
void orc_philox(uint64_t seed, const uint32_t ctr_in[4], uint32_t out[4]);
/* N(0,std) approximated by the Irwin-Hall sum of four 22-bit uniforms. */
void orc_gen_normal_bf16(uint64_t seed, uint32_t tensor_id, float std_dev,
                         int64_t n, uint16_t* out);
float orc_normal_scale(float std_dev);  /* the fp32 multiplier used above */
void orc_gen_words(uint64_t seed, uint32_t tensor_id, int64_t n_words, uint32_t* out);
void orc_gen_tokens(uint64_t seed, uint32_t tensor_id, int64_t n, int vocab, int32_t* out);
uint32_t orc_uniform24(uint64_t seed, uint32_t seq, uint32_t step, uint32_t slot,
                       uint32_t stream);

/* ---- affine quantization (group-wise, min/max rule) ---- */
int orc_quantize(const uint16_t* w, int N, int K, int group, int bits,
                 uint32_t* wq, uint16_t* scales, uint16_t* biases);
int orc_dequantize(const uint32_t* wq, const uint16_t* scales, const uint16_t* biases,
                   int N, int K, int group, int bits, uint16_t* out);
/* Op-sweep weights: uniform codes, scales = |N(0,0.02)|/7.5, biases = -8*scale. */
int orc_gen_sweep_weights(uint64_t seed, uint32_t tensor_id, int N, int K, int bits,
                          uint32_t* wq, uint16_t* scales, uint16_t* biases);

/* ---- ops ---- */
int orc_qmm(const uint16_t* x, const uint32_t* wq, const uint16_t* scales,
            const uint16_t* biases, uint16_t* y, int M, int N, int K, int group, int bits);
/* M >= threshold: dequantize-then-dot (the tensor-core path); 0 = never */
void orc_set_mma_min_m(int m);
int orc_mma_min_m(void);
/* M in [the threshold, this bound] (default 0 = none) use the canonical GEMV form
 * (the device's mid-batch tensor-core GEMM keeps MLX's qmv math). */
void orc_set_tcs_max_m(int m);
int orc_tcs_max_m(void);
void orc_rms_norm(const uint16_t* x, const uint16_t* w, uint16_t* y, int rows, int dim,
                  float eps);
void orc_rope_table(int max_pos, int dims, float base, float* cos_t, float* sin_t);
void orc_rope_table_scaled(int max_pos, int dims, float base, float factor, float low_freq,
                           float high_freq, float orig_max_pos, float* cos_t, float* sin_t);
void orc_rope(uint16_t* x, const int32_t* pos, int rows, int heads, int dim,
              const float* cos_t, const float* sin_t);
void orc_swiglu(const uint16_t* g, const uint16_t* u, uint16_t* y, int64_t n);
void orc_add(const uint16_t* a, const uint16_t* b, uint16_t* y, int64_t n);
void orc_argmax(const uint16_t* logits, int rows, int V, int32_t* out);

/* SDPA over a bf16 cache for one sequence.  q [T, Hq, D] bf16 (already roped),
 * k/v [Hkv, cap, D] bf16.  Query row t sees keys 0..offset+t.  out [T, Hq, D]. */
void orc_sdpa(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out,
              int T, int Hq, int Hkv, int D, int cap, int offset, float scale);

/* ---- sampling / acceptance (exact integer arithmetic) ---- */
int orc_sample(const uint16_t* logits, int V, float temperature, float top_p, uint32_t u24);
/* Greedy: n_accepted and the K+1 emitted-or-next tokens.
 * target_logits [K+1, V], drafts [K] (d1..dK).  Returns accepted count;
 * out_tokens[0..acc-1] = accepted drafts, out_tokens[acc] = correction/bonus. */
int orc_accept_greedy(const uint16_t* target_logits, const int32_t* drafts, int K, int V,
                      int32_t* out_tokens);
int orc_accept_stochastic(const uint16_t* target_logits, const uint16_t* draft_logits,
                          const int32_t* drafts, int K, int V, float temperature,
                          float top_p, const uint32_t* u_accept, uint32_t u_final,
                          int32_t* out_tokens);

/* ---- model + KV cache + speculative loop ---- */
typedef struct {
  int hidden, layers, inter, heads, kv_heads, head_dim, vocab;
  float rope_theta, eps;
  int qk_norm;   /* Qwen3: 1, Llama: 0 */
  int tied;      /* lm_head shares the packed embedding */
  int bits, group;
  /* Llama-3 RoPE frequency scaling; factor <= 1: none */
  float rope_factor, rope_low_freq, rope_high_freq, rope_orig_max_pos;
} orc_model_cfg;

void* orc_model_create(const orc_model_cfg* cfg, uint64_t seed);
void orc_model_free(void* m);
/* Copy a generated weight out (for bit-exactness checks vs the GPU generator).
 * kind: 0 q,1 k,2 v,3 o,4 gate,5 up,6 down,7 embed,8 lm_head. */
int orc_model_weight(void* m, int layer, int kind, uint32_t* wq, uint16_t* s, uint16_t* b);
/* Install a checkpoint's weight at `bits` (its own quantization) / a norm
 * vector (which: 0 input, 1 post-attention, 2 q, 3 k of `layer`; 4 final). */
int orc_model_set_weight(void* m, int layer, int kind, int bits, const uint32_t* wq, const uint16_t* s,
                         const uint16_t* b);
int orc_model_set_norm(void* m, int layer, int which, const uint16_t* v);

/* kv_bits: 16 = bf16 cache, 4/8 = affine group-64 quantized cache. */
void* orc_cache_create(void* model, int n_layers, int batch, int capacity, int kv_bits);
int orc_cache_fill_synthetic(void* cache, int rows, uint64_t seed, uint32_t tid_base);
/* Hybrid-model ops (configuration 4), canonical orders of gdn_moe.cuh. */
float orc_log(float x);
int orc_gdn_verify(int B, int T, int Hk, int Hv, const uint16_t* qkv, const uint16_t* z, const uint16_t* b,
                   const uint16_t* a, const uint16_t* conv_w, const float* a_log, const uint16_t* dt_bias,
                   const uint16_t* norm_w, float eps, const uint16_t* conv_state, const float* state, float* snap,
                   uint16_t* out);
int orc_gdn_commit(int B, int T, int Hk, int Hv, const uint16_t* qkv, const float* snap, const int32_t* acc,
                   float* state, uint16_t* conv_state);
int orc_moe_route(const uint16_t* logits, int rows, int E, int k, int32_t* idx, float* w);
int orc_moe_experts(const uint16_t* x, int M, int H, int I, int E, int k, const int32_t* idx, const float* w,
                    const uint32_t* gw, const uint16_t* gs, const uint16_t* gb, const uint32_t* uw,
                    const uint16_t* us, const uint16_t* ub, const uint32_t* dw, const uint16_t* ds,
                    const uint16_t* db, int bits, uint16_t* y);
/* Hybrid (Qwen3-Next-style) model + MTP speculative loop (hybrid.cuh). */
typedef struct {
  int hidden, layers, attn_every, heads, kv_heads, lin_k_heads, lin_v_heads;
  int experts, top_k, expert_inter, shared_inter, vocab;
  float rope_theta, eps;
  int bits;
} orc_hybrid_cfg;
void* orc_hybrid_create(const orc_hybrid_cfg* cfg, uint64_t seed);
void orc_hybrid_free(void* model);
void* orc_hybrid_state_create(void* model, int batch, int capacity, int kv_bits);
void orc_hybrid_state_free(void* state);
int orc_hybrid_forward(void* model, void* state, const int32_t* tokens, int B, int T, uint16_t* logits);
int orc_hybrid_spec_generate(void* model, const int32_t* prompts, int B, int P, int max_tokens, int kv_bits,
                             int32_t* out, int64_t* stats);
/* Emulate a tp-rank tensor-parallel split of o_proj / down_proj (partials
 * over column slices summed in fp32 in rank order); 0 = ok. */
int orc_model_set_tp(void* model, int tp);
void orc_cache_free(void* c);
int orc_cache_len(void* c, int b);
void orc_cache_set_position(void* c, int b, int pos);

/* Forward T tokens per sequence through layers [0, n_layers) with final norm
 * and lm_head.  tokens [B, T].  logits [B, T, V] (may be NULL). */
int orc_forward(void* model, void* cache, int n_layers, const int32_t* tokens, int B, int T,
                uint16_t* logits);

typedef struct {
  int K;              /* draft tokens per step (verify pass has K+1) */
  int max_tokens;     /* tokens emitted per sequence */
  float temperature;  /* 0 = greedy */
  float top_p;
  uint64_t seed;      /* uniforms */
  int draft_layers;   /* >0: draft = first draft_layers of target (self-draft) */
  int context_len;    /* synthetic context rows before the prompt (0: none) */
  uint64_t context_seed;
} orc_spec_params;

/* Speculative decode with a separate draft model (draft may be the target
 * itself with draft_layers > 0).  prompts [B, P].  out [B, max_tokens].
 * stats[0]=steps, [1]=proposed, [2]=accepted (summed over sequences),
 * [3]=prefill ns, [4]=decode ns (wall clock). */
int orc_spec_generate(void* target, void* draft, const int32_t* prompts, int B, int P,
                      const orc_spec_params* prm, int kv_bits, int32_t* out, int64_t* stats);
/* The same loop as a session: prefill once, then run steps (CPU baseline). */
void* orc_spec_session(void* target, void* draft, const int32_t* prompts, int B, int P,
                       const orc_spec_params* prm, int kv_bits);
int orc_spec_session_step(void* session, int n_steps);
void orc_spec_session_result(void* session, int32_t* out, int64_t* stats);
void orc_spec_session_free(void* session);
int orc_threads(void);
/* OpenMP threads for later calls (n <= 0: every online host core); returns the count. */
int orc_set_threads(int n);
/* Gated DeltaNet state snapshots rounded to bf16 as the reference stores
 * them (1, default) or kept fp32 (0); the device's lmx_set_gdn_state_bf16. */
void orc_set_gdn_state_bf16(int on);
/* REF_KV_PAD_QUIRK mode for quantized KV caches (the reference's
 * maybe_quantize_kv_cache): the prompt is prefilled into a bf16 cache, then
 * the whole reference allocation (orc_kv_quirk_alloc rows, zero rows past the
 * prompt included) is quantized and decoding continues at that offset.  Off:
 * the intended semantics (rows quantized on append, offset = tokens). */
void orc_set_kv_quirk(int on);
int orc_kv_quirk_alloc(int n_tokens);
/* Plain (non-speculative) greedy decode, same emission contract. */
int orc_generate(void* target, const int32_t* prompts, int B, int P, int max_tokens,
                 int kv_bits, int32_t* out);

#ifdef __cplusplus
}
#endif
#endif
