/*
 * lmx.h -- C ABI of the B200-native speculative-decode hot path.
 *
 * Drop-in for lemon-mlx-engine's MLX op surface on the speculative / MTP
 * decode path (reference interfaces cited per entry point) and for its
 * generate / TokenIterator contract.  Plain pointers and sizes only.
 *
 * Conventions
 *   - bf16 tensors are `void*` to 16-bit bf16 values (bit pattern), row-major.
 *   - Every pointer argument is a DEVICE pointer unless the name says `host`.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy stream).
 *   - Functions return lmx_status (0 = OK) and never throw; no entry point
 *     on the decode path allocates device memory.
 *   - Asynchronous: results are ready when the stream is.
 */
#ifndef LMX_H
#define LMX_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  LMX_OK = 0,
  LMX_ERR_INVALID = 1,      /* bad shape / pointer / alignment            */
  LMX_ERR_UNSUPPORTED = 2,  /* valid for the reference, not implemented   */
  LMX_ERR_CUDA = 3,         /* CUDA runtime error (see lmx_last_error)    */
  LMX_ERR_OOM = 4,          /* device allocation failed (setup calls only) */
  LMX_ERR_CAPACITY = 5,     /* KV cache capacity exceeded                 */
  LMX_ERR_IO = 6            /* checkpoint file missing / malformed         */
} lmx_status;

/* Human-readable text of the last error on this thread. */
const char* lmx_last_error(void);
/* Library version, e.g. "lmx-b200 0.1". */
const char* lmx_version(void);
/* Select the CUDA device for this thread's subsequent calls (one process per
 * GPU: the rank's local device). */
int lmx_set_device(int device);

/* ---------------------------------------------------------------------------
 * quantized_matmul
 * Replaces mx::quantized_matmul(x, w, scales, biases, transpose=true,
 * group_size, bits) as called by linear_forward()
 * (include/mlx-lm/common/quantized_linear.h:82-85).
 *   x [M,K] bf16;  w [N, K*bits/32] uint32, MLX affine packing (value j of a
 *   row in word j/(32/bits), bits (j%(32/bits))*bits, LSB first);
 *   scales, biases [N, K/group_size] bf16;  y [M,N] bf16.
 * Supported: bits 4 or 8, group_size 64, K % 64 == 0, K <= 16384.
 * M below the tensor-core threshold runs the fused-dequant GEMV (bit-exact
 * canonical order); M at or above it runs the tcgen05 path (weights
 * dequantized to bf16 in shared memory, fp32 accumulation: within tolerance).
 * ------------------------------------------------------------------------- */
int lmx_quantized_matmul(const void* x, const uint32_t* w, const void* scales,
                         const void* biases, void* y, int M, int N, int K,
                         int group_size, int bits, void* stream);

/* Smallest M routed to the tcgen05 path (default 16, as MLX switches from
 * its qmv to its tiled qmm for batched rows); 0 = never (every M runs the
 * canonical GEMV order).  Process-wide; no reference counterpart. */
int lmx_set_mma_min_m(int m);
int lmx_mma_min_m(void);

/* Smallest M routed to the small-batch tensor-core GEMV (mma.sync with the
 * weights dequantized into register fragments; default 4) for M below the
 * tcgen05 threshold; 0 = off.  Only in tensor-core mode: with
 * lmx_set_mma_min_m(0) every M runs the canonical GEMV order whatever this
 * is.  Results are within the tensor-core tolerance.  Process-wide; no
 * reference counterpart. */
int lmx_set_gemv_tc_min_m(int m);
int lmx_gemv_tc_min_m(void);
/* Matrices with at least this many 16-row tiles (default 1024: an lm_head)
 * run the small-batch tensor-core GEMV with one warp per tile over the whole
 * K instead of eight warps splitting K; 0 = never.  Same math, groups summed
 * by one warp (within the same tolerance).  Process-wide; no reference
 * counterpart. */
/* M from the tcgen05 threshold up to this bound (at most 64; default 0) run
 * the mid-batch tensor-core GEMM (mma.sync on the exact codes, MLX's qmv math
 * per group: s * sum q x + b * sum x) instead of the tcgen05 kernel
 * (dequantize-then-MMA); 0 = never.  Within the same tolerance of the
 * canonical order as the small-batch GEMV.  Process-wide; no reference
 * counterpart. */
int lmx_set_gemm_tcs_max_m(int m);
int lmx_gemm_tcs_max_m(void);
int lmx_set_gemv_tc_rows_min_tiles(int t);
int lmx_gemv_tc_rows_min_tiles(void);

/* The fused small-batch decode forward (default off): in tensor-core mode a
 * model forward of at most 16 token rows (B*T, at most 8 query rows per KV
 * head) runs its whole decoder stack as one persistent kernel (one CTA per
 * SM, grid barriers between the dependent phases, weights streamed ahead into
 * shared memory) instead of eight kernels per layer.  Results are within the
 * tensor-core tolerance; exact mode never uses it.  Off by default because
 * the per-op kernels are faster today.  Process-wide; no reference
 * counterpart. */
int lmx_set_fused_decode(int on);
int lmx_fused_decode(void);

/* Cache capacity (rows) from which, in tensor-core mode, every attention
 * block takes the tensor-core SDPA -- also single-token decode, whose few
 * query rows per KV head would otherwise take the CUDA-core kernel (default
 * 1: every block); 0 = only blocks of at least the tensor-core threshold's
 * rows per KV head.  Results
 * are within the tensor-core tolerance.  Process-wide; no reference
 * counterpart. */
int lmx_set_sdpa_tc_min_cache(int rows);
int lmx_sdpa_tc_min_cache(void);

/* mx::fast::rms_norm(x, w, eps) over the last axis (e.g. qwen3.cpp:78,145).
 * x, y [rows, dim] bf16 (may alias), w [dim] bf16. */
int lmx_rms_norm(const void* x, const void* w, void* y, int rows, int dim, float eps,
                 void* stream);

/* Read (and optionally clear) the device error word that bounded waits in
 * kernels set when they give up (0 = none). */
int lmx_device_error(unsigned* code, int clear);

/* Kernel launches this library has issued so far in the process (eager
 * launches plus launches recorded into captured graphs; a graph replay adds
 * nothing here: lmx_spec_step_launches gives the kernels per replayed step).
 * No reference counterpart (measurement hook). */
long long lmx_launch_count(void);

/* argmax over the last axis, first maximum wins (mx::argmax,
 * src/common/generate.cpp:43,801).  logits [rows, V] bf16 -> out [rows] int32. */
int lmx_argmax(const void* logits, int rows, int V, int32_t* out, void* stream);


/* ---------------------------------------------------------------------------
 * Sampling and speculative acceptance (K3).  The reference samples with
 * mx::random::categorical (temperature-scaled Gumbel, src/common/generate.cpp:
 * 83-120; TopPSampler leaves top-p unapplied) and has no rejection sampler.
 * Here both take caller-supplied 24-bit uniforms and decide in exact integer
 * arithmetic: w_j = rint(exp((l_j - max)/T) * 2^32); top-p keeps the smallest
 * prefix by (w desc, index asc) with 2^24*mass >= rint(top_p*2^24)*Z; a draw
 * is the smallest index t with 2^24*cumsum_t > u24*Z_kept.
 * ------------------------------------------------------------------------- */
/* logits [rows, V] bf16 -> out [rows]; temperature <= 0 is argmax (u24 unused). */
int lmx_sample(const void* logits, int rows, int V, float temperature, float top_p, const uint32_t* u24,
               int32_t* out, void* stream);
/* Rejection sampling (Leviathan et al. 2023): target_logits [B, K+1, V],
 * draft_logits [B, K, V], drafts [B, K] (d1..dK), u_accept [B, K], u_final [B].
 * Accept d_i iff u*q(d_i)*Zp < 2^24*p(d_i)*Zq; on the first rejection draw from
 * max(0, p*Zq - q*Zp); after K acceptances draw the bonus from p_K.
 * n_accepted [B]; out_tokens [B, K+1]: accepted drafts then the correction /
 * bonus token.  temperature must be > 0 (greedy acceptance is in
 * lmx_spec_decode). */
int lmx_spec_accept(const void* target_logits, const void* draft_logits, const int32_t* drafts, int B, int K,
                    int V, float temperature, float top_p, const uint32_t* u_accept, const uint32_t* u_final,
                    int32_t* n_accepted, int32_t* out_tokens, void* stream);

/* ---------------------------------------------------------------------------
 * KV cache view and decode / verify attention.
 * Replaces cache->update + sdpa() -> mx::fast::scaled_dot_product_attention
 * (include/mlx-lm/common/attention_utils.h:60-77, src/common/kv_cache.cpp:
 * 34-110, 271-298) for the speculative step.  lengths[b] is the number of
 * cached rows BEFORE the current block; the block's T rows are already
 * written at rows [lengths[b], lengths[b]+T).  Query row t of sequence b sees
 * keys 0 .. lengths[b]+t (the reference's [T, offset+T] causal mask,
 * src/common/kv_cache.cpp:15-30).  head_dim must be 128, group size 64.
 * ------------------------------------------------------------------------- */
typedef struct {
  int batch, kv_heads, head_dim, capacity;
  int bits;                 /* 16 = bf16 cache, 8 or 4 = affine quantized      */
  void* k;                  /* bits 16: bf16 [batch][kv_heads][capacity][128]  */
  void* v;
  uint32_t* k_packed;       /* bits 4/8: [batch][kv_heads][capacity][128*bits/32],
                             * 16-byte aligned (k, v and the packed arrays)   */
  uint32_t* v_packed;
  void* k_scales;           /* bits 4/8: bf16 [batch][kv_heads][capacity][2]   */
  void* k_biases;
  void* v_scales;
  void* v_biases;
  int32_t* lengths;         /* [batch] rows cached before the current block    */
} lmx_kv;

/* KV append (KVCacheSimple::update_impl, src/common/kv_cache.cpp:34-110;
 * QuantizedKVCache::update_impl + quantize_kv, :271-298, :243-269): rows
 * k_new / v_new bf16 [batch][kv_heads][T][128] (the reference's update
 * layout; keys already normed and roped) go to rows lengths[b] .. +T-1 of
 * each sequence -- quantized on append for a 4/8-bit cache with the rule
 * scale = bf16((max-min)/(2^bits-1)), bias = bf16(min), q = rint((x-bias)/
 * scale) per group of 64 -- and every length advances by T (on the device).
 * A block past the capacity is written nowhere and sets the device error
 * word to 0x42 (lmx_device_error). */
int lmx_kv_append(const lmx_kv* kv, const void* k_new, const void* v_new, int T, void* stream);
/* KVCache::set_position (kv_cache.cpp:135-142, :301-377): roll sequence seq
 * back to pos rows (no-op when pos >= its length); on the device, in stream
 * order. */
int lmx_kv_set_position(const lmx_kv* kv, int seq, int pos, void* stream);

/* Scratch bytes lmx_sdpa_decode needs for this shape (split partials and
 * per-tile counters).  The scratch must be zero-filled before its first use;
 * every call leaves it ready for the next. */
size_t lmx_sdpa_scratch_bytes(int batch, int T, int heads, int kv_heads, int capacity);
/* q, out: bf16 [batch*T, heads*128] (q already normed and roped). */
int lmx_sdpa_decode(const void* q, const lmx_kv* kv, int T, int heads, float scale, void* scratch,
                    size_t scratch_bytes, void* out, void* stream);
/* lmx_sdpa_decode for callers that cannot allocate device memory (a host
 * framework that owns every device allocation and forbids cudaMalloc in its
 * callbacks, or a caller that must not enter the allocator).  It has no
 * counterpart in the reference.  Instead of caller scratch it uses one
 * built-in device array of 16 MiB that every GPU loading this library holds
 * until exit; shapes whose lmx_sdpa_scratch_bytes exceeds 16 MiB are rejected
 * with LMX_ERR_CAPACITY.  It allocates nothing (no cudaMalloc / cudaFree).
 * The first call on each device looks up the array's device address (one-time
 * set-up); make that first call before any stream capture.  All calls share
 * the array and it keeps the last call's contents: calls that overlap on the
 * GPU race, so serialise them.  Results equal lmx_sdpa_decode's. */
int lmx_sdpa_decode_noalloc(const void* q, const lmx_kv* kv, int T, int heads, float scale, void* out,
                            void* stream);

/* ---------------------------------------------------------------------------
 * Hybrid-model ops (configuration 4, Qwen3-Next-style decoder).
 *
 * Gated DeltaNet verify step: replaces Qwen3NextGatedDeltaNet's core between
 * in_proj and out_proj (src/llm/models/qwen3_next.cpp:252-402) --
 * gdn_conv_step / depthwise conv1d + SiLU with a 3-row state
 * (src/common/gated_delta.cpp:885-921), q/k RMSNorm, beta / g
 * (gated_delta.cpp:603-633), gated_delta_update_seq with per-token states
 * (gated_delta.cpp:1067-1138), gated RMSNorm (gated_delta.cpp:948-971).
 * Head dims 128.  The recurrent state is fp32 [B][Hv][128 (v)][128 (k)]
 * holding bf16-rounded values between blocks (lmx_set_gdn_state_bf16).  lmx_gdn_verify reads state / conv_state and
 * writes the state after every token (state_snap) and the output; it never
 * modifies state or conv_state.  lmx_gdn_commit then keeps the state after
 * token acc[b] of each sequence (MambaCache rollback_spec,
 * include/mlx-lm/common/kv_cache.h:178-288; acc read on the device) and
 * advances conv_state (in place) to the window ending at that token;
 * acc[b] < 0 leaves sequence b unchanged.
 * ------------------------------------------------------------------------- */
typedef struct {
  int batch, T;            /* sequences, tokens per sequence in this block     */
  int k_heads, v_heads;    /* linear_num_key_heads / value_heads (v % k == 0)  */
  const void* qkv;         /* bf16 [batch][T][2*k_heads*128 + v_heads*128] pre-conv q|k|v */
  const void* z;           /* bf16 [batch][T][v_heads*128] output gate         */
  const void* b;           /* bf16 [batch][T][v_heads]                          */
  const void* a;           /* bf16 [batch][T][v_heads]                          */
  const void* conv_w;      /* bf16 [2*k_heads*128 + v_heads*128][4]             */
  const float* a_log;      /* fp32 [v_heads]                                    */
  const void* dt_bias;     /* bf16 [v_heads]                                    */
  const void* norm_w;      /* bf16 [128] gated RMSNorm weight                   */
  float eps;
  void* conv_state;        /* bf16 [batch][3][qkv width]                        */
  float* state;            /* fp32 [batch][v_heads][128][128]                   */
  float* state_snap;       /* fp32 [batch][T][v_heads][128][128]                */
  void* out;               /* bf16 [batch][T][v_heads*128]                      */
  void* scratch;           /* lmx_gdn_scratch_bytes(batch, T, k_heads, v_heads) */
} lmx_gdn;
size_t lmx_gdn_scratch_bytes(int batch, int T, int k_heads, int v_heads);
/* Recurrent-state precision between blocks (process-wide, default 1): the
 * reference keeps the state in fp32 while it runs a block of tokens and
 * stores the per-token states and the block's final state as bf16
 * (src/common/gated_delta.cpp:93, :162-172); with 1 the snapshots (and so
 * every committed state) are rounded to bf16 the same way, the state
 * arrays staying fp32 holding bf16 values; 0 keeps full fp32 states. */
int lmx_set_gdn_state_bf16(int on);
int lmx_gdn_state_bf16(void);
int lmx_gdn_verify(const lmx_gdn* g, void* stream);
int lmx_gdn_commit(const lmx_gdn* g, const int32_t* acc, void* stream);

/* MoE router (moe_route, src/common/gated_delta.cpp:973-999; the top-k and
 * renormalised scores of Qwen3NextSparseMoeBlock, qwen3_next.cpp:452-470):
 * per row the k largest logits (ties: lower index), in descending order, and
 * w = softmax over those k (fp32).  k <= 16, E <= 16384. */
int lmx_moe_route(const void* logits, int rows, int E, int k, int32_t* idx, float* w, void* stream);

/* Routed SwiGLU experts (SwitchGLU + gather_qmm, src/common/switch_layers.cpp:
 * 200-245, and the score-weighted sum of qwen3_next.cpp:471-478):
 * y[m] = sum_j w[m][j] * down_e(swiglu(gate_e x_m, up_e x_m)), e = idx[m][j],
 * over packed affine group-64 expert weights in the MLX SwitchLinear layout:
 * gate / up [E][I][H*bits/32] (scales, biases [E][I][H/64]), down
 * [E][H][I*bits/32] ([E][H][I/64]).  act_scratch: bf16 [M][k][I]. */
typedef struct {
  const uint32_t* w;
  const void* scales;
  const void* biases;
} lmx_qweights;
int lmx_moe_experts(const void* x, int M, int H, int I, int E, int k, const int32_t* idx, const float* w,
                    const lmx_qweights* gate, const lmx_qweights* up, const lmx_qweights* down, int bits,
                    void* act_scratch, void* y, void* stream);

/* Hybrid (Qwen3-Next-style) model and its MTP speculative decoder
 * (configuration 4): Qwen3NextModel (src/llm/models/qwen3_next.cpp) with
 * layer l a gated full-attention layer when l % attn_every == attn_every - 1
 * and a Gated DeltaNet layer otherwise, every layer followed by a sparse MoE
 * block (top_k of experts + a sigmoid-gated shared expert); one MTP head
 * (MTPHead, src/llm/models/mtp_head.cpp:146-178: RMSNorm of the embedding
 * and of the trunk hidden, concat, fc, one attention + MoE decoder layer,
 * output norm) drafting 2 tokens per step through the shared lm_head, the
 * step of TokenIterator::mtp_speculative_step (src/common/generate.cpp:
 * 669-933).  Head dims 128; weights synthetic and seeded (affine group 64). */
typedef struct {
  int hidden, layers, attn_every;
  int heads, kv_heads;            /* gated attention (head_dim 128)        */
  int lin_k_heads, lin_v_heads;   /* Gated DeltaNet (head dims 128)        */
  int experts, top_k, expert_inter, shared_inter;
  int vocab;
  float rope_theta, eps;
  int bits;                       /* 4 or 8                                */
} lmx_hybrid_config;
int lmx_hybrid_create(const lmx_hybrid_config* cfg, uint64_t seed, void** model);
/* Expert parallelism across the GPUs of one node (configuration 4): this
 * rank holds experts [rank*E/n, (rank+1)*E/n) of every MoE block (the same
 * seeded values as the unsharded model); attention, Gated DeltaNet, router,
 * shared expert, embedding, lm_head and the MTP head's other weights are
 * replicated.  Per MoE block every rank runs the gate|up / down of the slots
 * whose expert it holds and writes their outputs into its communicator
 * block; after a bounded barrier every rank combines the k slots of each row
 * in slot order, pulling each slot from its owner over NVLink -- the
 * single-GPU arithmetic, so streams are identical for every rank count.  The
 * communicator (lmx_tp_comm_create, opened on every rank) needs max_rows >=
 * rows per forward x top_k and max_hidden >= hidden.  Every rank must issue
 * the same calls in the same order.  The reference runs on one device and
 * has no counterpart (its SwitchGLU / gather_qmm: src/common/
 * switch_layers.cpp:79-245). */
int lmx_hybrid_create_ep(const lmx_hybrid_config* cfg, uint64_t seed, void* comm, void** model);
int lmx_hybrid_free(void* model);
/* Trunk forward of a [B, T] token block (host ints) over the state's caches
 * (attention KV and recurrent states), committing every token; logits
 * [B, T, vocab] bf16 to logits_host (may be NULL). */
int lmx_hybrid_state_create(void* model, int batch, int capacity, int kv_bits, int max_tokens_per_forward,
                            void** state);
int lmx_hybrid_state_free(void* state);
int lmx_hybrid_forward(void* model, void* state, const int32_t* tokens_host, int B, int T, void* logits_host);
/* MTP speculative decoding: greedy, 2 drafts per step (3-token verify). */
int lmx_hybrid_spec_create(void* model, int batch, int max_tokens, int prompt_len, int kv_bits, void** spec);
int lmx_hybrid_spec_prefill(void* spec, const int32_t* prompts_host);
int lmx_hybrid_spec_decode(void* spec, int use_graph, double* seconds);
int lmx_hybrid_spec_result(void* spec, int32_t* out_host, int64_t* stats_host);
int lmx_hybrid_spec_free(void* spec);
/* Measurement hooks: time `iters` verify passes (trunk over 3 tokens,
 * after a prefill) -> seconds per pass and its algorithmic bytes (the
 * experts counted from the pass's own routing); kernel launches of one
 * captured step. */
int lmx_hybrid_spec_profile(void* spec, int iters, double* seconds, double* bytes);
int lmx_hybrid_spec_step_launches(void* spec, int64_t* launches);

/* ---------------------------------------------------------------------------
 * Models.  Replaces the ModelContext function table of a loaded Qwen3 /
 * Llama model (include/mlx-lm/common/model_container.h:20-51; graphs
 * src/llm/models/qwen3.cpp:69-220, llama.cpp:203-469).  Weights are synthetic
 * and seeded: linear / embedding weights N(0,0.02) (Irwin-Hall of Philox
 * draws) in bf16, affine-quantized (group 64) on the device; norms are ones.
 * ------------------------------------------------------------------------- */
typedef struct {
  int hidden, layers, inter, heads, kv_heads, head_dim, vocab;
  float rope_theta, eps;
  int qk_norm;     /* Qwen3 q/k RMSNorm (1) or none (Llama, 0)           */
  int tied;        /* lm_head shares the packed embedding                 */
  int bits;        /* 4 or 8                                              */
  int group_size;  /* 64                                                  */
  /* Llama-3 RoPE frequency scaling (rope_type "llama3"); factor <= 1: none */
  float rope_factor, rope_low_freq, rope_high_freq, rope_orig_max_pos;
} lmx_model_config;

int lmx_model_create(const lmx_model_config* cfg, uint64_t seed, void** model);
/* A model that runs only the first n_layers of `model` (shares its weights,
 * embedding, final norm and lm_head): the self-draft of the speculative
 * configs.  Free it with lmx_model_free before freeing `model`. */
int lmx_model_view(void* model, int n_layers, void** view);
int lmx_model_free(void* model);
/* Copy one packed weight to host memory (kind: 0 q,1 k,2 v,3 o,4 gate,5 up,
 * 6 down,7 embed,8 lm_head).  For a tensor-parallel shard: the shard. */
int lmx_model_weight(void* model, int layer, int kind, void* w_host, void* s_host, void* b_host);

/* ---------------------------------------------------------------------------
 * Checkpoints: MLX-format model directories (load_llm_from_directory,
 * src/llm/llm_factory.cpp:272-290; load_safetensors_from_directory,
 * src/common/safetensors.cpp:23-75; register_quantized_weights,
 * src/common/quantize_utils.cpp:14-104).  A directory holds config.json and
 * model.safetensors, or the shards named by model.safetensors.index.json
 * (else every *.safetensors in it).  Qwen3 (model_type "qwen3") and Llama
 * ("llama", "mistral", with Llama-3 rope scaling); linear layers and the
 * embedding MLX affine-quantized at 4 or 8 bits, group 64, with per-layer
 * overrides from config.json's "quantization" object ({"bits", "group_size"}
 * keyed by the layer prefix, e.g. "model.layers.3.mlp.down_proj"); q/k/v of a
 * layer share their bits, as do gate/up.  Norms and scales may be BF16, F16 or
 * F32 (rounded to bf16).  lm_head.weight is ignored when the embeddings are
 * tied.  A missing tensor, a shape that disagrees with config.json or an
 * unquantized linear layer fails with LMX_ERR_IO / LMX_ERR_UNSUPPORTED.
 * ------------------------------------------------------------------------- */
/* config.json (path: the file or its directory) -> cfg (bits / group_size:
 * the default quantization) and up to max_eos EOS ids (n_eos: how many the
 * file lists).  Host only: needs no GPU. */
int lmx_model_config_load(const char* path, lmx_model_config* cfg, int32_t* eos_ids, int max_eos, int* n_eos);
/* The quantization config.json gives the layer `prefix` (quantization_for,
 * include/mlx-lm/common/base_config.h:47-54).  Host only. */
int lmx_model_quant_for(const char* path, const char* prefix, int* bits, int* group_size);
/* One safetensors header entry: dtype string (<= 15 chars), shape, absolute
 * data offset in the file.  Host only. */
int lmx_safetensors_tensor(const char* file, const char* name, char* dtype, int64_t* shape, int max_dims, int* ndim,
                           uint64_t* data_offset);
int lmx_model_load(const char* dir, void** model);
/* This rank's tensor-parallel shard of a checkpoint (lmx_model_create_tp's
 * split); only the shard's blocks are copied to the device. */
int lmx_model_load_tp(const char* dir, void* comm, void** model);
/* Write config.json + model.safetensors (MLX names, U32 packed weights, BF16
 * scales / biases / norms); per-layer overrides for weights whose bits differ
 * from the model's.  A tp 1, full-depth model. */
int lmx_model_save(void* model, const char* dir);

/* ---------------------------------------------------------------------------
 * Tensor parallelism across the GPUs of one node (one process per GPU).  The
 * reference runs on one device and has no counterpart; this is the
 * multi-GPU form of the same model calls.  Megatron split: q/k/v by heads,
 * gate/up by FFN rows, o_proj / down_proj by the matching input columns, the
 * lm_head by vocabulary rows; one all-reduce after o_proj and one after
 * down_proj (fused with the residual add and the next RMSNorm), a
 * (value, index) exchange for the vocab-parallel argmax -- all over NVLink
 * peer memory, summed in rank order, so every rank and every run computes
 * the same bits.  Setup: every rank creates its communicator, exports its
 * handle (LMX_TP_HANDLE_BYTES), gathers all handles in rank order (any host
 * transport, e.g. torch.distributed.all_gather_object), opens them, and
 * meets the others at a host barrier before its first forward.
 * lmx_model_create_tp then builds this rank's shard of the same seeded
 * weights (comm NULL or size 1: the whole model).  Every rank must issue the
 * same forwards in the same order; a peer that stops arriving makes the
 * waiting kernels give up after 2 s and report LMX_ERR_CUDA ("kernel
 * reported error 0x71").
 * ------------------------------------------------------------------------- */
#define LMX_TP_HANDLE_BYTES 64
int lmx_tp_comm_create(int rank, int size, int max_rows, int max_hidden, void** comm);
int lmx_tp_comm_handle(void* comm, void* handle_out);
int lmx_tp_comm_open(void* comm, const void* handles);  /* size x LMX_TP_HANDLE_BYTES */
int lmx_tp_comm_free(void* comm);  /* after every model that uses it */
/* Bytes of a communicator's device block.  A caller that maps its peers'
 * memory itself (its own IPC or virtual-memory mapping) attaches each peer's
 * block by a pointer this process can address instead of opening handles;
 * the comm is open once every peer is attached or opened.  Blocks are
 * 256-byte aligned. */
size_t lmx_tp_comm_block_bytes(void* comm);
int lmx_tp_comm_attach(void* comm, int peer, void* peer_block);
/* The all-reduce after o_proj / down_proj as one op (the north star's NCCL
 * all-reduce over NVLink, here fused): h[r] = bf16(h[r] + bf16(sum over
 * ranks of partial_p[r])), the sum in fp32 in rank order; xn[r] =
 * rms_norm(h[r]) * norm_w (mx::fast::rms_norm).  partial [rows][hidden]
 * bf16 is this rank's share; it is staged into the comm's current slot
 * unless it already is that slot (lmx_tp_comm_partial, so a producer can
 * write there directly).  Every rank must call it in the same order.  A peer
 * that does not arrive within 2 s makes the kernel give up: h and xn are left
 * unchanged and the device error word (lmx_device_error) reads 0x71.  The
 * peers' flags are then out of step with this rank's: free and re-create the
 * communicator on every rank before the next exchange.  The reference runs
 * on one device and has no counterpart. */
int lmx_tp_comm_partial(void* comm, void** partial);
int lmx_tp_allreduce_rmsnorm(void* comm, const void* partial, int rows, int hidden, void* h, const void* norm_w,
                             float eps, void* xn, void* stream);
int lmx_model_create_tp(const lmx_model_config* cfg, uint64_t seed, void* comm, void** model);

/* ---------------------------------------------------------------------------
 * KV cache: KVCacheSimple / QuantizedKVCache (src/common/kv_cache.cpp:34-142,
 * :243-377).  kv_bits 16 (bf16), 8 or 4 (affine group 64, quantized on
 * append, dequantized inside SDPA).  Rows are preallocated to `capacity`.
 * ------------------------------------------------------------------------- */
int lmx_cache_create(void* model, int n_layers, int batch, int capacity, int kv_bits,
                     int max_tokens_per_forward, void** cache);
int lmx_cache_free(void* cache);
/* KVCacheSimple::set_position (kv_cache.cpp:135-142): roll sequence `seq`
 * back to `pos` rows (no-op if pos >= its length). */
int lmx_cache_set_position(void* cache, int seq, int pos);
int lmx_cache_len(void* cache, int seq, int* len);
/* Layer `layer` of an engine cache as an lmx_kv descriptor: device pointers
 * into the cache itself (KVCacheSimple::state(), include/mlx-lm/common/
 * kv_cache.h:81-87), for lmx_sdpa_decode, lmx_kv_append and
 * lmx_kv_set_position or for reading the rows.  Valid until the cache is
 * freed; capacity may exceed the one requested (rows are allocated in whole
 * 128-key splits). */
int lmx_cache_kv(void* cache, int layer, lmx_kv* out);
/* Synthetic context: rows [0, rows) of every layer's K and V hold seeded
 * N(0,1) values (Philox normal, tensor id tid_base + 2*layer + (0 K, 1 V),
 * element ((b*kv_heads + head)*rows + row)*128 + d over the whole model's KV
 * heads), quantized like an append; every length becomes `rows`. */
int lmx_cache_fill_synthetic(void* cache, int rows, uint64_t seed, uint32_t tid_base);
/* ModelContext::call_fn for a [B, T] token block (host ints): runs the first
 * n_layers, appends K/V at each sequence's length, writes logits [B, T, V]
 * bf16 to logits_host (may be NULL) and advances the lengths. */
int lmx_forward(void* model, void* cache, int n_layers, const int32_t* tokens_host, int B, int T,
                void* logits_host);

/* ---------------------------------------------------------------------------
 * Speculative decoding: TokenIterator::mtp_speculative_step / next()
 * (src/common/generate.cpp:669-933, :968-1045) generalised to a draft model.
 * Per step and sequence: the draft proposes d1..dK, the target verifies
 * [d0, d1..dK] in one K+1-token pass, the accepted prefix d0..d_acc is
 * emitted (d0 first, as the reference's emission contract), the correction /
 * bonus token becomes the next d0 and both caches roll back.  All
 * bookkeeping runs on the device; one step is replayed as a CUDA graph.
 * ------------------------------------------------------------------------- */
typedef struct {
  int batch;        /* independent sequences decoded together            */
  int K;            /* draft tokens per step (reference n_draft_tokens-1);
                     * 0: plain decoding, one token per step, no draft   */
  int max_tokens;   /* tokens emitted per sequence                       */
  int prompt_len;
  int kv_bits;      /* 16, 8 or 4                                        */
  float temperature;/* 0 = greedy (ArgMaxSampler)                        */
  float top_p;
  uint64_t seed;    /* uniform draws of the stochastic path              */
  /* Synthetic context: context_len cache rows per sequence, before the
   * prompt, filled with seeded N(0,1) K/V (a stand-in for prefilling a long
   * random-token prefix; lmx_cache_fill_synthetic).  0: none.            */
  int context_len;
  uint64_t context_seed;
  /* Global id of this decoder's sequence 0: the uniform draws of sequence b
   * are keyed by seq_base + b, so a batch split across ranks (each rank its
   * slice, seq_base = the slice's first global index) draws exactly what one
   * decoder over the whole batch would.  0 for a single decoder.          */
  int seq_base;
  /* REF_KV_PAD_QUIRK (4/8-bit caches): reproduce the reference's
   * maybe_quantize_kv_cache (src/common/kv_cache.cpp:391-413) -- the prompt
   * is prefilled with a bf16 cache, then the whole reference allocation
   * (max(first 512-token chunk, 256) rows, doubled as the prompt grows;
   * zero rows past the prompt included) is quantized and decoding continues
   * at that offset.  0: the intended semantics (rows quantized on append,
   * the offset counts tokens).                                             */
  int kv_quirk;
} lmx_spec_config;

/* draft may be NULL (self-draft: the first draft_layers of target).  With a
 * tensor-parallel target (lmx_model_create_tp / lmx_model_load_tp) the draft
 * is either replicated (a tp 1 model on every rank) or this rank's shard over
 * the same communicator; both decode greedily. */
int lmx_spec_create(void* target, void* draft, int draft_layers, const lmx_spec_config* cfg,
                    void** spec);
int lmx_spec_prefill(void* spec, const int32_t* prompts_host /* [batch, prompt_len] */);
/* Decode until every sequence has emitted max_tokens; *seconds = device time
 * of the decode loop (prefill excluded). */
int lmx_spec_decode(void* spec, int use_graph, double* seconds);
/* out_host [batch, max_tokens]; stats_host[5] = steps, drafts proposed,
 * drafts accepted, tokens emitted (summed over sequences), steps enqueued
 * (graph replays, including those after every sequence finished). */
int lmx_spec_result(void* spec, int32_t* out_host, int64_t* stats_host);
int lmx_spec_free(void* spec);

/* TokenIterator::next() (src/common/generate.cpp:968-1045, include/mlx-lm/
 * common/generate.h:236-330) after lmx_spec_prefill: the next token of every
 * sequence, in the reference's emission order (d0 first, then the accepted
 * drafts; the correction / bonus token is the next step's d0).  A speculative
 * step runs (one graph replay) only when a sequence that has not reached
 * max_tokens has no token left; with K = 0 in lmx_spec_config the step is
 * one plain decode step, the reference's fallback when no draft is available
 * (generate.cpp:671-686).  tokens_host[b] = -1 once sequence b has produced
 * max_tokens tokens; *n_live counts the other sequences (0: the reference's
 * nullopt).  EOS is the caller's to check, as in the reference. */
int lmx_spec_next(void* spec, int32_t* tokens_host, int* n_live);

/* GenerateCompletionInfo (include/mlx-lm/common/generate.h:170-199), per
 * sequence; times in seconds. */
typedef struct {
  int prompt_token_count;
  int generation_token_count;
  double prompt_time;
  double generation_time;
  int mtp_draft_tokens_proposed;
  int mtp_draft_tokens_accepted;
  int mtp_speculative_steps;
} lmx_completion_info;
/* GenerateCancelPredicate (generate.h:218-228): nonzero aborts. */
typedef int (*lmx_cancel_fn)(void* user);
/* The per-token callback of generate(): nonzero stops sequence `seq`
 * (GenerateDisposition::stop). */
typedef int (*lmx_token_fn)(void* user, int seq, int32_t token);
/* generate() (src/common/generate.cpp:1061-1125): prefill prompts_host
 * [batch, prompt_len], then lmx_spec_next until every sequence has stopped.
 * should_cancel (may be NULL) is polled before every step; a token in
 * eos_ids ends its sequence and is neither counted nor passed to on_token;
 * on_token (may be NULL) returning nonzero ends its sequence.  info [batch]
 * (may be NULL): prompt_time = the prefill's wall time, generation_time from
 * the sequence's first token to its end (the reference restarts its clock
 * at the first token). */
int lmx_spec_generate(void* spec, const int32_t* prompts_host, const int32_t* eos_ids, int n_eos,
                      lmx_cancel_fn should_cancel, void* cancel_user, lmx_token_fn on_token, void* token_user,
                      lmx_completion_info* info);
/* Measurement hooks (no reference counterpart; used by bench.py): time one
 * piece of the step on the decoder's stream with CUDA events: the piece is
 * captured into a CUDA graph (as the decode runs it) and replayed `iters`
 * times, after decode.  what: 0 verify pass, 1 one draft token, 2 lm_head at
 * M = batch*(K+1), 3 lm_head at M = batch.  *bytes = algorithmic HBM bytes of
 * one launch (packed weights + scales/biases + KV rows + activations). */
int lmx_spec_profile(void* spec, int what, int iters, double* seconds, double* bytes);
/* Kernel launches in one captured speculative step (graph node count). */
int lmx_spec_step_launches(void* spec, int64_t* launches);

#ifdef __cplusplus
}
#endif
#endif /* LMX_H */
