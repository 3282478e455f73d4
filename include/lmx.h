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
  LMX_ERR_CAPACITY = 5      /* KV cache capacity exceeded                 */
} lmx_status;

/* Human-readable text of the last error on this thread. */
const char* lmx_last_error(void);
/* Library version, e.g. "lmx-b200 0.1". */
const char* lmx_version(void);

/* ---------------------------------------------------------------------------
 * quantized_matmul
 * Replaces mx::quantized_matmul(x, w, scales, biases, transpose=true,
 * group_size, bits) as called by linear_forward()
 * (include/mlx-lm/common/quantized_linear.h:82-85).
 *   x [M,K] bf16;  w [N, K*bits/32] uint32, MLX affine packing (value j of a
 *   row in word j/(32/bits), bits (j%(32/bits))*bits, LSB first);
 *   scales, biases [N, K/group_size] bf16;  y [M,N] bf16.
 * Supported: bits 4 or 8, group_size 64, K % 64 == 0, K <= 16384.
 * M < 16 runs the fused-dequant GEMV (bit-exact canonical order); M >= 16 may
 * run the tcgen05 path.
 * ------------------------------------------------------------------------- */
int lmx_quantized_matmul(const void* x, const uint32_t* w, const void* scales,
                         const void* biases, void* y, int M, int N, int K,
                         int group_size, int bits, void* stream);

/* mx::fast::rms_norm(x, w, eps) over the last axis (e.g. qwen3.cpp:78,145).
 * x, y [rows, dim] bf16 (may alias), w [dim] bf16. */
int lmx_rms_norm(const void* x, const void* w, void* y, int rows, int dim, float eps,
                 void* stream);

/* Read (and optionally clear) the device error word that bounded waits in
 * kernels set when they give up (0 = none). */
int lmx_device_error(unsigned* code, int clear);

/* argmax over the last axis, first maximum wins (mx::argmax,
 * src/common/generate.cpp:43,801).  logits [rows, V] bf16 -> out [rows] int32. */
int lmx_argmax(const void* logits, int rows, int V, int32_t* out, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* LMX_H */
