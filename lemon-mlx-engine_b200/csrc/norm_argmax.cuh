// norm_argmax.cuh -- standalone RMSNorm and the cluster argmax.
#pragma once
#include <cooperative_groups.h>

#include "lmx_common.cuh"
namespace cg = cooperative_groups;

namespace lmx {

// Canonical RMSNorm factor of one row, computed by a whole warp:
//   chunk c = elements [8c, 8c+8); lane l owns chunks l, l+32, l+64, ...
//   p_l = fma chain of x^2 over its chunks ascending, elements ascending;
//   butterfly (16,8,4,2,1); factor = 1 / sqrt(ss / dim + eps).
// Chunks are read as 16-byte vectors, up to 8 per lane in flight.  Needs x
// 16-byte aligned and dim % 8 == 0.
LMX_DEV float rms_factor_warp(const bf16_t* x, int dim, float eps, int lane) {
  float p = 0.0f;
  const int nch = dim >> 3;
  for (int c0 = lane; c0 < nch; c0 += 256) {
    uint4 buf[8];
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (c0 + 32 * k < nch) buf[k] = *reinterpret_cast<const uint4*>(x + 8 * (c0 + 32 * k));
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (c0 + 32 * k < nch) {
        const uint32_t w[4] = {buf[k].x, buf[k].y, buf[k].z, buf[k].w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float v = (e & 1) ? hi_bf(w[e >> 1]) : lo_bf(w[e >> 1]);
          p = __fmaf_rn(v, v, p);
        }
      }
    }
  }
  p = warp_sum_xor(p, 16, 1);
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(p, (float)dim), eps)));
}

// RMSNorm (mx::fast::rms_norm, e.g. src/llm/models/qwen3.cpp:78,145): one
// CTA per row.  Warp 0 forms the factor as above while every thread loads its
// chunks of x and w (chunk c = threadIdx.x + 256 i); after the barrier (which
// also makes in-place use safe: all of x is read before any y is written)
// each thread writes y = bf16((x * r) * w) for its chunks.
static constexpr int kNormChunks = 4;  // chunks per thread held in registers (dim <= 8192)

LMX_DEV uint4 rms_apply8(const uint4& xv, const uint4& wv, float f) {
  const uint32_t xa[4] = {xv.x, xv.y, xv.z, xv.w}, wa[4] = {wv.x, wv.y, wv.z, wv.w};
  uint32_t o[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const bf16_t lo = f2bf(__fmul_rn(__fmul_rn(lo_bf(xa[k]), f), lo_bf(wa[k])));
    const bf16_t hi = f2bf(__fmul_rn(__fmul_rn(hi_bf(xa[k]), f), hi_bf(wa[k])));
    o[k] = (uint32_t)lo | ((uint32_t)hi << 16);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__global__ void __launch_bounds__(256) rms_norm_kernel(const bf16_t* x, const bf16_t* w, bf16_t* y,
                                                       int rows, int dim, float eps) {
  __shared__ float s_f;
  grid_wait();
  grid_launch_dependents();
  const int tid = threadIdx.x, lane = tid & 31, row = blockIdx.x;
  if (row >= rows) return;
  const bf16_t* xr = x + (size_t)row * dim;
  bf16_t* yr = y + (size_t)row * dim;
  const int nch = dim >> 3;
  uint4 xv[kNormChunks], wv[kNormChunks];
#pragma unroll
  for (int i = 0; i < kNormChunks; ++i) {
    const int c = tid + 256 * i;
    if (c < nch) {
      xv[i] = *reinterpret_cast<const uint4*>(xr + 8 * c);
      wv[i] = *reinterpret_cast<const uint4*>(w + 8 * c);
    }
  }
  if (tid < 32) {
    const float f = rms_factor_warp(xr, dim, eps, lane);
    if (lane == 0) s_f = f;
  }
  __syncthreads();
  const float f = s_f;
  if (nch <= 256 * kNormChunks) {
#pragma unroll
    for (int i = 0; i < kNormChunks; ++i) {
      const int c = tid + 256 * i;
      if (c < nch) *reinterpret_cast<uint4*>(yr + 8 * c) = rms_apply8(xv[i], wv[i], f);
    }
  } else {
    // rows longer than the register tile: x may equal y, so every thread
    // first holds its values (the loop writes only chunks it has read)
    for (int c = tid; c < nch; c += 256) {
      const uint4 a = *reinterpret_cast<const uint4*>(xr + 8 * c);
      const uint4 b = *reinterpret_cast<const uint4*>(w + 8 * c);
      *reinterpret_cast<uint4*>(yr + 8 * c) = rms_apply8(a, b, f);
    }
  }
}

// (value, index) max with the lowest index winning ties; NaN never wins.
LMX_DEV bool am_better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

LMX_DEV void am_warp(float& bv, int& bi) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, bv, off);
    int oi = __shfl_xor_sync(0xffffffffu, bi, off);
    if (am_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
  }
}

// Block-level argmax of a slice; returns the result in thread 0.
LMX_DEV void am_block(float& bv, int& bi, float* sv, int* si) {
  am_warp(bv, bi);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (lane == 0) { sv[warp] = bv; si[warp] = bi; }
  __syncthreads();
  if (warp == 0) {
    bv = lane < nw ? sv[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : 0x7fffffff;
    am_warp(bv, bi);
  }
}

// argmax over V per row: a cluster of kArgmaxCluster CTAs per row, each
// reducing a contiguous slice; rank 0 combines the partials through DSMEM
// (no global scratch).
static constexpr int kArgmaxCluster = 8;
__global__ void __launch_bounds__(512) argmax_kernel(const bf16_t* logits, int V, int32_t* out) {
  __shared__ float sv[32];
  __shared__ int si[32];
  __shared__ float cv;
  __shared__ int ci;
  grid_wait();
  grid_launch_dependents();
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank(), cs = (int)cluster.num_blocks();
  const int row = blockIdx.x / cs;
  const int chunk = (V + cs - 1) / cs;
  const int j0 = rank * chunk, j1 = min(V, j0 + chunk);
  const bf16_t* l = logits + (size_t)row * V;
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
    out[row] = ri == 0x7fffffff ? 0 : ri;
  }
  cluster.sync();
}

}  // namespace lmx
