// lmx_internal.h -- host-side launch API shared by the library's translation
// parts (the kernels and C ABI in lmx.cu, the speculative engine in
// engine.cuh, the hybrid model in hybrid.cuh).  Not part of the public C ABI.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/lmx.h"

namespace lmx {

typedef uint16_t bf16_t;

struct QMat {
  const uint32_t* w = nullptr;
  const bf16_t* s = nullptr;
  const bf16_t* b = nullptr;
  int rows = 0;
};

enum QmmMode { kPlain = 0, kResid = 1, kSwiglu = 2 };

struct QmmCall {
  const bf16_t* x = nullptr;
  int ldx = 0;                     // 0 = K
  const bf16_t* norm_w = nullptr;  // fused RMSNorm of x (M <= 64)
  float eps = 1e-6f;
  QMat mat[3];
  int nmat = 1;
  int N = 0;       // virtual rows (plain/resid) or rows per matrix (swiglu)
  bf16_t* y = nullptr;
  int ldy = 0;
  const bf16_t* res = nullptr;
  int M = 0, K = 0, bits = 4;
  QmmMode mode = kPlain;
};

// Device / error plumbing (lmx.cu)
int set_error(int code, const char* fmt, ...);
int cuda_check(cudaError_t e, const char* what);
int device_sms();
unsigned* device_error_word();

// Kernel launchers (lmx.cu).  All launch with programmatic dependent launch.
int launch_qmm(const QmmCall& c, cudaStream_t st);
// Tensor-core path for M >= the threshold (un-normalised x only).
bool qmm_uses_mma(int M);
bool qmm_uses_tcg(int M);
int qmm_mma_min_m();
int launch_rms_norm(const bf16_t* x, const bf16_t* w, bf16_t* y, int rows, int dim, float eps,
                    cudaStream_t st);
int launch_argmax(const bf16_t* logits, int rows, int V, int32_t* out, cudaStream_t st);

}  // namespace lmx
