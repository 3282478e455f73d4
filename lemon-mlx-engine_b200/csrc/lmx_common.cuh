// lmx_common.cuh -- device helpers shared by the sm_100a kernels.
//
// Numerics contract: every kernel on the CUDA-core path executes the same
// sequence of IEEE fp32 operations as the canonical order documented beside
// each kernel (explicit __fmaf_rn / __fadd_rn / __fmul_rn, no contraction:
// the library is built with --fmad=false), so its results are bit-identical
// to any implementation of that order.
#pragma once
#include <atomic>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/lmx.h"

#define LMX_DEV __device__ __forceinline__

namespace lmx {

typedef uint16_t bf16_t;  // raw bf16 bits in device buffers

LMX_DEV float bf2f(bf16_t h) { return __uint_as_float((uint32_t)h << 16); }
LMX_DEV bf16_t f2bf(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}
LMX_DEV float lo_bf(uint32_t w) { return __uint_as_float(w << 16); }
LMX_DEV float hi_bf(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// exp(x) by Cody-Waite reduction and a degree-7 Taylor polynomial (Horner),
// followed by exact scaling with 2^n.  x > 88 -> +inf, x < -87 -> 0.
LMX_DEV float exp_c(float x) {
  if (x != x) return x;
  if (x > 88.0f) return __int_as_float(0x7f800000);
  if (x < -87.0f) return 0.0f;
  const float kLog2e = 0x1.715476p+0f;
  const float kLn2Hi = 0x1.62e4p-1f;
  const float kLn2Lo = 0x1.7f7d1cp-20f;
  float n = rintf(__fmul_rn(x, kLog2e));
  float r = __fmaf_rn(-n, kLn2Hi, x);
  r = __fmaf_rn(-n, kLn2Lo, r);
  float p = 0x1.a01a02p-13f;
  p = __fmaf_rn(p, r, 0x1.6c16c2p-10f);
  p = __fmaf_rn(p, r, 0x1.111112p-7f);
  p = __fmaf_rn(p, r, 0x1.555556p-5f);
  p = __fmaf_rn(p, r, 0x1.555556p-3f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  int ni = (int)n;
  return __fmul_rn(p, __uint_as_float((uint32_t)(ni + 127) << 23));
}

LMX_DEV float sigmoid_c(float g) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_c(-g))); }

// silu(g) * u with bf16 materialisation after every op (MLX compiled swiglu).
LMX_DEV bf16_t swiglu_c(bf16_t g, bf16_t u) {
  float gf = bf2f(g);
  float sg = bf2f(f2bf(sigmoid_c(gf)));
  float a = bf2f(f2bf(__fmul_rn(gf, sg)));
  return f2bf(__fmul_rn(a, bf2f(u)));
}

// Philox4x32-10 (Salmon et al., SC'11).
LMX_DEV void philox10(uint32_t c[4], uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int i = 0; i < 10; ++i) {
    uint32_t hi0 = __umulhi(0xD2511F53u, c[0]), lo0 = 0xD2511F53u * c[0];
    uint32_t hi1 = __umulhi(0xCD9E8D57u, c[2]), lo1 = 0xCD9E8D57u * c[2];
    uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
    c[0] = n0; c[1] = lo1; c[2] = n2; c[3] = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
}

LMX_DEV uint32_t uniform24(uint64_t seed, uint32_t seq, uint32_t step, uint32_t slot,
                           uint32_t stream) {
  uint32_t c[4] = {seq, step, slot, stream};
  uint64_t k = seed ^ 0x9E3779B97F4A7C15ull;
  philox10(c, (uint32_t)k, (uint32_t)(k >> 32));
  return c[0] >> 8;
}

// Programmatic dependent launch (sm_90+): a kernel may start its prologue
// (constant-weight loads) while its predecessor drains; grid_wait() blocks
// until the predecessor's results are visible.
LMX_DEV void grid_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
LMX_DEV void grid_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

LMX_DEV float warp_sum_xor(float v, int first, int last) {
  for (int off = first; off >= last; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

}  // namespace lmx

// Kernel launches issued by this library (eager launches and launches being
// captured into a graph), for the host-side launch accounting.
static std::atomic<long long> g_lmx_launches{0};
static inline cudaError_t lmx_counted(cudaError_t e) {
  if (e == cudaSuccess) g_lmx_launches.fetch_add(1, std::memory_order_relaxed);
  return e;
}

// Launch helper: every kernel is launched with the programmatic-stream-
// serialization attribute so it can overlap its predecessor's tail.
template <typename Kern, typename... Args>
static inline cudaError_t lmx_launch(Kern kern, dim3 grid, dim3 block, size_t smem,
                                     cudaStream_t st, bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return lmx_counted(cudaLaunchKernelEx(&cfg, kern, args...));
}
