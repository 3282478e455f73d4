// oracle.cpp -- CPU restatement of the reference's speculative-decode hot path.
//
// TEST INFRASTRUCTURE ONLY (see oracle.h for the scope, the pinned/unpinned
// split and the rule that nothing in the product may use this file).
//
// Build: oracle/Makefile (g++ -O3 -fopenmp -ffp-contract=off).  Contraction is
// off so every fp32 multiply/add below is its own IEEE operation; every fused
// multiply-add is written as std::fma, exactly where the CUDA kernels use
// __fmaf_rn, so both sides execute the same operations in the same order.
#include "oracle.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

typedef unsigned __int128 u128;

// ---------------------------------------------------------------------------
// scalar numerics
// ---------------------------------------------------------------------------
static inline float bf2f(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}
static inline uint16_t f2bf(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);  // quiet NaN
  u += 0x7fffu + ((u >> 16) & 1u);                                              // RNE
  return (uint16_t)(u >> 16);
}
static inline float u2f(uint32_t u) {
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

extern "C" float orc_bf16_to_f32(uint16_t h) { return bf2f(h); }
extern "C" uint16_t orc_f32_to_bf16(float x) { return f2bf(x); }

// exp(x): Cody-Waite reduction x = n*ln2 + r (ln2 split hi/lo, hi with 16
// significant bits so n*ln2_hi is exact), e^r by the degree-7 Taylor
// polynomial in Horner form, then an exact scaling by 2^n.  Domain clamps:
// x > 88 -> +inf, x < -87 -> 0.  Every operation is a single IEEE fp32
// operation so the CUDA kernels reproduce the result bit for bit.
extern "C" float orc_exp(float x) {
  if (x != x) return x;
  if (x > 88.0f) return INFINITY;
  if (x < -87.0f) return 0.0f;
  const float kLog2e = 0x1.715476p+0f;
  const float kLn2Hi = 0x1.62e4p-1f;
  const float kLn2Lo = 0x1.7f7d1cp-20f;
  float n = std::rint(x * kLog2e);
  float r = std::fma(-n, kLn2Hi, x);
  r = std::fma(-n, kLn2Lo, r);
  float p = 0x1.a01a02p-13f;            // 1/5040
  p = std::fma(p, r, 0x1.6c16c2p-10f);  // 1/720
  p = std::fma(p, r, 0x1.111112p-7f);   // 1/120
  p = std::fma(p, r, 0x1.555556p-5f);   // 1/24
  p = std::fma(p, r, 0x1.555556p-3f);   // 1/6
  p = std::fma(p, r, 0.5f);
  p = std::fma(p, r, 1.0f);
  p = std::fma(p, r, 1.0f);
  int ni = (int)n;
  return p * u2f((uint32_t)(ni + 127) << 23);
}

static inline float sigmoid_f(float g) { return 1.0f / (1.0f + orc_exp(-g)); }

// ---------------------------------------------------------------------------
// Philox4x32-10 (Salmon et al., SC'11) and the synthetic-data generators
// ---------------------------------------------------------------------------
static inline void philox10(uint32_t c[4], uint32_t k0, uint32_t k1) {
  for (int i = 0; i < 10; ++i) {
    uint64_t p0 = (uint64_t)0xD2511F53u * c[0];
    uint64_t p1 = (uint64_t)0xCD9E8D57u * c[2];
    uint32_t n0 = (uint32_t)(p1 >> 32) ^ c[1] ^ k0;
    uint32_t n1 = (uint32_t)p1;
    uint32_t n2 = (uint32_t)(p0 >> 32) ^ c[3] ^ k1;
    uint32_t n3 = (uint32_t)p0;
    c[0] = n0; c[1] = n1; c[2] = n2; c[3] = n3;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
}

extern "C" void orc_philox(uint64_t seed, const uint32_t ctr_in[4], uint32_t out[4]) {
  uint32_t c[4] = {ctr_in[0], ctr_in[1], ctr_in[2], ctr_in[3]};
  philox10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
  std::memcpy(out, c, 16);
}

// Element e of tensor `tid`: counter (e_lo, e_hi, tid, 0x243F6A88).
static inline void gen_block(uint64_t seed, uint32_t tid, uint64_t e, uint32_t out[4]) {
  out[0] = (uint32_t)e;
  out[1] = (uint32_t)(e >> 32);
  out[2] = tid;
  out[3] = 0x243F6A88u;
  philox10(out, (uint32_t)seed, (uint32_t)(seed >> 32));
}

extern "C" float orc_normal_scale(float std_dev) {
  return (float)((double)std_dev * std::sqrt(3.0) / 4194304.0);
}

// Irwin-Hall(4) of 22-bit uniforms: S in [0, 2^24), z = S - 2^23 is exact in
// fp32, w = bf16(z * C) with C = std*sqrt(3)/2^22 (variance of the sum of four
// U(0,1) is 1/3).
static inline uint16_t normal_bf16(uint64_t seed, uint32_t tid, uint64_t e, float C) {
  uint32_t r[4];
  gen_block(seed, tid, e, r);
  int32_t S = (int32_t)((r[0] >> 10) + (r[1] >> 10) + (r[2] >> 10) + (r[3] >> 10));
  float z = (float)(S - (1 << 23));
  return f2bf(z * C);
}

extern "C" void orc_gen_normal_bf16(uint64_t seed, uint32_t tid, float std_dev, int64_t n,
                                    uint16_t* out) {
  const float C = orc_normal_scale(std_dev);
#pragma omp parallel for schedule(static)
  for (int64_t e = 0; e < n; ++e) out[e] = normal_bf16(seed, tid, (uint64_t)e, C);
}

extern "C" void orc_gen_words(uint64_t seed, uint32_t tid, int64_t n_words, uint32_t* out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < (n_words + 3) / 4; ++i) {
    uint32_t r[4];
    gen_block(seed, tid, (uint64_t)i, r);
    for (int j = 0; j < 4 && 4 * i + j < n_words; ++j) out[4 * i + j] = r[j];
  }
}

extern "C" void orc_gen_tokens(uint64_t seed, uint32_t tid, int64_t n, int vocab, int32_t* out) {
  for (int64_t e = 0; e < n; ++e) {
    uint32_t r[4];
    gen_block(seed, tid, (uint64_t)e, r);
    out[e] = (int32_t)(((uint64_t)r[0] * (uint64_t)vocab) >> 32);
  }
}

// Uniform draws for sampling: counter (seq, step, slot, stream), key seed^golden.
extern "C" uint32_t orc_uniform24(uint64_t seed, uint32_t seq, uint32_t step, uint32_t slot,
                                  uint32_t stream) {
  uint32_t c[4] = {seq, step, slot, stream};
  uint64_t k = seed ^ 0x9E3779B97F4A7C15ull;
  philox10(c, (uint32_t)k, (uint32_t)(k >> 32));
  return c[0] >> 8;
}

// ---------------------------------------------------------------------------
// Affine group quantization.  Packing (pinned by the reference's
// debug_layer0_reference.py:53-82): value j of a row sits in word j/(32/bits)
// at bit offset (j % (32/bits))*bits, LSB first; w = q*scale + bias.
// The quantize rule (MLX's is unpinned): scale = bf16((max-min)/(2^bits-1)),
// bias = bf16(min), q = clamp(rint((w - bias)/scale)).  A constant group gets
// scale 1.  Dequantized value: bf16(fma(scale, q, bias)).
// ---------------------------------------------------------------------------
static inline void quantize_group(const uint16_t* w, int n, int bits, uint32_t* words,
                                  uint16_t* s_out, uint16_t* b_out) {
  float mn = bf2f(w[0]), mx = bf2f(w[0]);
  for (int j = 1; j < n; ++j) {
    float v = bf2f(w[j]);
    mn = std::min(mn, v);
    mx = std::max(mx, v);
  }
  const int nb = (1 << bits) - 1;
  uint16_t sb = f2bf((mx - mn) / (float)nb);
  float sc = bf2f(sb);
  if (sc == 0.0f) { sb = f2bf(1.0f); sc = 1.0f; }
  uint16_t bb = f2bf(mn);
  float bi = bf2f(bb);
  const int per = 32 / bits;
  for (int j = 0; j < n / per; ++j) words[j] = 0;
  for (int j = 0; j < n; ++j) {
    float qf = std::rint((bf2f(w[j]) - bi) / sc);
    int q = (int)qf;
    q = q < 0 ? 0 : (q > nb ? nb : q);
    words[j / per] |= (uint32_t)q << ((j % per) * bits);
  }
  *s_out = sb;
  *b_out = bb;
}

static inline int qcode(const uint32_t* row_words, int j, int bits) {
  const int per = 32 / bits;
  return (int)((row_words[j / per] >> ((j % per) * bits)) & ((1u << bits) - 1u));
}

extern "C" int orc_quantize(const uint16_t* w, int N, int K, int group, int bits, uint32_t* wq,
                            uint16_t* scales, uint16_t* biases) {
  if ((bits != 4 && bits != 8) || group <= 0 || K % group || group % (32 / bits)) return 1;
  const int G = K / group, KW = K * bits / 32;
#pragma omp parallel for schedule(static)
  for (int n = 0; n < N; ++n)
    for (int g = 0; g < G; ++g)
      quantize_group(w + (size_t)n * K + (size_t)g * group, group, bits,
                     wq + (size_t)n * KW + (size_t)g * group * bits / 32,
                     scales + (size_t)n * G + g, biases + (size_t)n * G + g);
  return 0;
}

extern "C" int orc_dequantize(const uint32_t* wq, const uint16_t* scales, const uint16_t* biases,
                              int N, int K, int group, int bits, uint16_t* out) {
  if ((bits != 4 && bits != 8) || group <= 0 || K % group) return 1;
  const int G = K / group, KW = K * bits / 32;
#pragma omp parallel for schedule(static)
  for (int n = 0; n < N; ++n)
    for (int k = 0; k < K; ++k) {
      float s = bf2f(scales[(size_t)n * G + k / group]);
      float b = bf2f(biases[(size_t)n * G + k / group]);
      out[(size_t)n * K + k] = f2bf(std::fma(s, (float)qcode(wq + (size_t)n * KW, k, bits), b));
    }
  return 0;
}

extern "C" int orc_gen_sweep_weights(uint64_t seed, uint32_t tid, int N, int K, int bits,
                                     uint32_t* wq, uint16_t* scales, uint16_t* biases) {
  if ((bits != 4 && bits != 8) || K % 64) return 1;
  orc_gen_words(seed, tid, (int64_t)N * K * bits / 32, wq);
  const int64_t G = (int64_t)N * (K / 64);
  const float C = orc_normal_scale(0.02f);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < G; ++i) {
    uint16_t z = normal_bf16(seed, tid + 1, (uint64_t)i, C);
    uint16_t s = f2bf(std::fabs(bf2f(z)) / 7.5f);
    scales[i] = s;
    biases[i] = f2bf(-8.0f * bf2f(s));
  }
  return 0;
}

// ---------------------------------------------------------------------------
// quantized_matmul  y[M,N] = x[M,K] . dequant(W[N,K])^T
// (reference call site: include/mlx-lm/common/quantized_linear.h:82-85).
// Uses MLX's affine identity  sum_j x_j (s q_j + b) = s sum_j q_j x_j + b sum_j x_j.
// Canonical fp32 order (group size 64, any bits, independent of M):
//   quarter c (16 consecutive k):  Q_c = fma chain over j ascending from 0
//                                  X_c = add chain over j ascending from 0
//   group g:   d_g  = (Q_4g + Q_4g+1) + (Q_4g+2 + Q_4g+3);   xs_g likewise from X
//              e_g  = fma(s_g, d_g, b_g * xs_g)
//   segment (8 groups, missing groups = 0):
//              t = ((e0+e1)+(e2+e3)) + ((e4+e5)+(e6+e7))
//   row total: segments added left to right;  y = bf16(total)
// ---------------------------------------------------------------------------
static void qmm_block8(const float* xf, const float* xsum, int M, int K, const uint32_t* wq,
                       const uint16_t* sc, const uint16_t* bi, int n0, int nr, int N,
                       int bits, uint16_t* y) {
  const int KW = K * bits / 32, G = K / 64, NSEG = (G + 7) / 8;
  std::vector<float> qv((size_t)K * 8, 0.0f);
  float s8[8], b8[8];
  for (int r = 0; r < nr; ++r) {
    const uint32_t* row = wq + (size_t)(n0 + r) * KW;
    for (int k = 0; k < K; ++k) qv[(size_t)k * 8 + r] = (float)qcode(row, k, bits);
  }
  for (int m = 0; m < M; ++m) {
    const float* xr = xf + (size_t)m * K;
    float tot[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int seg = 0; seg < NSEG; ++seg) {
      float e[8][8];
      for (int gi = 0; gi < 8; ++gi) {
        const int g = seg * 8 + gi;
        if (g >= G) {
          for (int r = 0; r < 8; ++r) e[gi][r] = 0.0f;
          continue;
        }
        float Q[4][8];
        for (int c = 0; c < 4; ++c) {
          for (int r = 0; r < 8; ++r) Q[c][r] = 0.0f;
          for (int j = 0; j < 16; ++j) {
            const int k = 64 * g + 16 * c + j;
            const float xv = xr[k];
            const float* qk = &qv[(size_t)k * 8];
            for (int r = 0; r < 8; ++r) Q[c][r] = std::fma(qk[r], xv, Q[c][r]);
          }
        }
        for (int r = 0; r < 8; ++r) {
          s8[r] = r < nr ? bf2f(sc[(size_t)(n0 + r) * G + g]) : 0.0f;
          b8[r] = r < nr ? bf2f(bi[(size_t)(n0 + r) * G + g]) : 0.0f;
        }
        const float xs = xsum[(size_t)m * G + g];
        for (int r = 0; r < 8; ++r) {
          float d = (Q[0][r] + Q[1][r]) + (Q[2][r] + Q[3][r]);
          e[gi][r] = std::fma(s8[r], d, b8[r] * xs);
        }
      }
      for (int r = 0; r < 8; ++r) {
        float t = ((e[0][r] + e[1][r]) + (e[2][r] + e[3][r])) +
                  ((e[4][r] + e[5][r]) + (e[6][r] + e[7][r]));
        tot[r] = seg == 0 ? t : tot[r] + t;
      }
    }
    for (int r = 0; r < nr; ++r) y[(size_t)m * N + n0 + r] = f2bf(tot[r]);
  }
}

// Tensor-core path (batched verify, prefill): for M >= the threshold the
// product is taken over dequantized weights, as MLX's tiled qmm does
// (dequantize the tile to the activation type, then MMA with fp32
// accumulation):  y = bf16( sum_k bf16(fma(s, q, b)) * x_k ).  The sum is
// formed in double here; the device accumulates in fp32 on the tensor cores
// in an order the hardware chooses, so this path is compared with a
// tolerance.  threshold 0 = never (canonical order for every M).
static int g_mma_min_m = 16;
extern "C" void orc_set_mma_min_m(int m) { g_mma_min_m = m < 0 ? 0 : m; }
extern "C" int orc_mma_min_m(void) { return g_mma_min_m; }
// The device's mid-batch tensor-core GEMM (M from the threshold up to this
// bound, default 64) keeps MLX's qmv form, s * sum q x + b * sum x per group,
// like its GEMV: the oracle then takes its canonical GEMV for those M, and the
// dequantize-then-dot form above the bound.  0 (default, as the device) = the
// dequantize form for every M at or above the threshold.
static int g_tcs_max_m = 0;
extern "C" void orc_set_tcs_max_m(int m) { g_tcs_max_m = m < 0 ? 0 : m; }
extern "C" int orc_tcs_max_m(void) { return g_tcs_max_m; }

static void qmm_dequant_rows(const float* xf, int M, int K, const uint32_t* wq, const uint16_t* sc,
                             const uint16_t* bi, int n0, int nr, int N, int bits, uint16_t* y) {
  const int KW = K * bits / 32, G = K / 64;
  std::vector<double> wd((size_t)K);
  for (int r = 0; r < nr; ++r) {
    const int n = n0 + r;
    const uint32_t* row = wq + (size_t)n * KW;
    for (int k = 0; k < K; ++k) {
      const float s = bf2f(sc[(size_t)n * G + k / 64]), b = bf2f(bi[(size_t)n * G + k / 64]);
      wd[k] = (double)bf2f(f2bf(std::fma(s, (float)qcode(row, k, bits), b)));
    }
    for (int m = 0; m < M; ++m) {
      const float* xr = xf + (size_t)m * K;
      double acc = 0.0;
      for (int k = 0; k < K; ++k) acc += wd[k] * (double)xr[k];
      y[(size_t)m * N + n] = f2bf((float)acc);
    }
  }
}

extern "C" int orc_qmm(const uint16_t* x, const uint32_t* wq, const uint16_t* scales,
                       const uint16_t* biases, uint16_t* y, int M, int N, int K, int group,
                       int bits) {
  if (group != 64 || (bits != 4 && bits != 8) || K % 64 || M < 0 || N < 0) return 1;
  if (M == 0 || N == 0) return 0;
  if (g_mma_min_m > 0 && M >= g_mma_min_m && M > g_tcs_max_m) {
    std::vector<float> xf((size_t)M * K);
    for (size_t i = 0; i < xf.size(); ++i) xf[i] = bf2f(x[i]);
    const int nblk = (N + 7) / 8;
#pragma omp parallel for schedule(dynamic, 4)
    for (int blk = 0; blk < nblk; ++blk) {
      const int n0 = blk * 8, nr = std::min(8, N - n0);
      qmm_dequant_rows(xf.data(), M, K, wq, scales, biases, n0, nr, N, bits, y);
    }
    return 0;
  }
  const int G = K / 64;
  std::vector<float> xf((size_t)M * K), xsum((size_t)M * G);
  for (size_t i = 0; i < xf.size(); ++i) xf[i] = bf2f(x[i]);
  for (int m = 0; m < M; ++m)
    for (int g = 0; g < G; ++g) {
      float X[4];
      for (int c = 0; c < 4; ++c) {
        float a = 0.0f;
        for (int j = 0; j < 16; ++j) a = a + xf[(size_t)m * K + 64 * g + 16 * c + j];
        X[c] = a;
      }
      xsum[(size_t)m * G + g] = (X[0] + X[1]) + (X[2] + X[3]);
    }
  const int nblk = (N + 7) / 8;
#pragma omp parallel for schedule(dynamic, 4)
  for (int blk = 0; blk < nblk; ++blk) {
    const int n0 = blk * 8, nr = std::min(8, N - n0);
    qmm_block8(xf.data(), xsum.data(), M, K, wq, scales, biases, n0, nr, N, bits, y);
  }
  return 0;
}

// ---------------------------------------------------------------------------
// rms_norm (mx::fast::rms_norm; formula debug_numerical_trace.py:103-108)
//   chunk c = elements [8c, 8c+8); lane l (0..31) owns chunks l, l+32, l+64, ...
//   p_l = fma chain of x_i^2 over its chunks ascending, elements ascending, from 0
//   butterfly: for off in 16,8,4,2,1: p_l = p_l + p_(l^off);  ss = p_0
//   r = 1 / sqrt(ss / dim + eps);   y_i = bf16((x_i * r) * w_i)
// (dim is a multiple of 8.)
static float rms_factor(const float* xr, int dim, float eps) {
  float p[32];
  for (int l = 0; l < 32; ++l) {
    float a = 0.0f;
    for (int c = l; c * 8 < dim; c += 32)
      for (int e = 0; e < 8; ++e) a = std::fma(xr[8 * c + e], xr[8 * c + e], a);
    p[l] = a;
  }
  for (int off = 16; off >= 1; off >>= 1) {
    float q[32];
    for (int l = 0; l < 32; ++l) q[l] = p[l] + p[l ^ off];
    std::memcpy(p, q, sizeof(p));
  }
  return 1.0f / std::sqrt(p[0] / (float)dim + eps);
}

extern "C" void orc_rms_norm(const uint16_t* x, const uint16_t* w, uint16_t* y, int rows, int dim,
                             float eps) {
#pragma omp parallel for schedule(static) if (rows > 64)
  for (int r = 0; r < rows; ++r) {
    std::vector<float> xr(dim);
    for (int i = 0; i < dim; ++i) xr[i] = bf2f(x[(size_t)r * dim + i]);
    const float f = rms_factor(xr.data(), dim, eps);
    for (int i = 0; i < dim; ++i) y[(size_t)r * dim + i] = f2bf((xr[i] * f) * bf2f(w[i]));
  }
}

// ---------------------------------------------------------------------------
// RoPE, NeoX half-split (traditional = false), examples/test_device_rope.cpp:15-46:
//   inv_freq_i = base^(-2i/dims); theta = pos * inv_freq_i  (double, then fp32
//   cos/sin table);  rx1 = x1*c - x2*s;  rx2 = x2*c + x1*s  (products rounded
//   separately, one bf16 rounding at the end)
// ---------------------------------------------------------------------------
extern "C" void orc_rope_table(int max_pos, int dims, float base, float* cos_t, float* sin_t) {
  orc_rope_table_scaled(max_pos, dims, base, 0.0f, 1.0f, 4.0f, 8192.0f, cos_t, sin_t);
}

// Period of rotation pair i: base^(2i/dims), with the Llama-3 frequency
// scaling of LlamaDynamicNTKScalingRoPE::compute_freqs
// (src/llm/models/llama.cpp:122-183) when factor > 1: wavelength 2*pi*period
// above old/low_freq -> period * factor; strictly between old/high_freq and
// old/low_freq -> period / ((1 - s)/factor + s), s = (old/wavelength -
// low_freq) / (high_freq - low_freq); shorter wavelengths unchanged.
extern "C" void orc_rope_table_scaled(int max_pos, int dims, float base, float factor, float low_freq,
                                      float high_freq, float orig_max_pos, float* cos_t, float* sin_t) {
  const int half = dims / 2;
  std::vector<double> period(half);
  for (int i = 0; i < half; ++i) {
    double pd = std::pow((double)base, 2.0 * (double)i / (double)dims);
    if (factor > 1.0f) {
      const double wl = 2.0 * M_PI * pd;
      const double low_wl = (double)orig_max_pos / (double)low_freq;
      const double high_wl = (double)orig_max_pos / (double)high_freq;
      if (wl > low_wl) {
        pd = pd * (double)factor;
      } else if (wl > high_wl) {
        const double s = ((double)orig_max_pos / wl - (double)low_freq) / ((double)high_freq - (double)low_freq);
        pd = pd / ((1.0 - s) / (double)factor + s);
      }
    }
    period[i] = pd;
  }
  for (int p = 0; p < max_pos; ++p)
    for (int i = 0; i < half; ++i) {
      const double th = (double)p / period[i];
      cos_t[(size_t)p * half + i] = (float)std::cos(th);
      sin_t[(size_t)p * half + i] = (float)std::sin(th);
    }
}

extern "C" void orc_rope(uint16_t* x, const int32_t* pos, int rows, int heads, int dim,
                         const float* cos_t, const float* sin_t) {
  const int half = dim / 2;
  for (int r = 0; r < rows; ++r)
    for (int h = 0; h < heads; ++h) {
      uint16_t* v = x + ((size_t)r * heads + h) * dim;
      const float* c = cos_t + (size_t)pos[r] * half;
      const float* s = sin_t + (size_t)pos[r] * half;
      for (int i = 0; i < half; ++i) {
        float a = bf2f(v[i]), b = bf2f(v[i + half]);
        float t1 = a * c[i], t2 = b * s[i], t3 = b * c[i], t4 = a * s[i];
        v[i] = f2bf(t1 - t2);
        v[i + half] = f2bf(t3 + t4);
      }
    }
}

// swiglu (include/mlx-lm/common/activations.h:24-33): silu(g) * u with every
// MLX op materialised in bf16: sg = bf16(sigmoid(g)), a = bf16(g*sg), y = bf16(a*u).
static inline uint16_t swiglu1(uint16_t g, uint16_t u) {
  float gf = bf2f(g);
  float sg = bf2f(f2bf(sigmoid_f(gf)));
  float a = bf2f(f2bf(gf * sg));
  return f2bf(a * bf2f(u));
}
extern "C" void orc_swiglu(const uint16_t* g, const uint16_t* u, uint16_t* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = swiglu1(g[i], u[i]);
}
extern "C" void orc_add(const uint16_t* a, const uint16_t* b, uint16_t* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = f2bf(bf2f(a[i]) + bf2f(b[i]));
}

// argmax over the last axis, first maximum wins (NaN never wins).
extern "C" void orc_argmax(const uint16_t* logits, int rows, int V, int32_t* out) {
  for (int r = 0; r < rows; ++r) {
    const uint16_t* l = logits + (size_t)r * V;
    int best = 0;
    float bv = -INFINITY;
    bool any = false;
    for (int j = 0; j < V; ++j) {
      float v = bf2f(l[j]);
      if (v != v) continue;
      if (!any || v > bv) { bv = v; best = j; any = true; }
    }
    out[r] = best;
  }
}

// ---------------------------------------------------------------------------
// SDPA for decode / verify (mx::fast::scaled_dot_product_attention with the
// [T, offset+T] causal mask of src/common/kv_cache.cpp:15-30).  Canonical order:
//   qs_d = q_d * scale;  keys are taken in splits of 128 (split s = keys
//   [128s, 128s+128) clipped to the row's visible range 0..offset+t):
//     score_j = fma chain over d ascending from 0
//     m_s = max score;  p_j = exp(score_j - m_s)
//     l_s: lane partials  a_l = add chain of p_j over keys j = j0+l, j0+l+32, ...
//          (l = 0..31, ascending, from 0), then butterfly (16,8,4,2,1) -> a_0
//     o_s[d] = fma chain of p_j * v_j[d] over j ascending from 0
//   combine over splits ascending: M = max m_s, w_s = exp(m_s - M),
//     L = fma(w_s, l_s, L), O[d] = fma(w_s, o_s[d], O[d]) from 0
//   out[d] = bf16(O[d] / L)
// ---------------------------------------------------------------------------
static const int kSdpaSplit = 128;

extern "C" void orc_sdpa(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out,
                         int T, int Hq, int Hkv, int D, int cap, int offset, float scale) {
  const int G = Hq / Hkv;
#pragma omp parallel for collapse(2) schedule(dynamic) if (T * Hq > 8)
  for (int t = 0; t < T; ++t)
    for (int h = 0; h < Hq; ++h) {
      const int kvh = h / G, L = offset + t + 1, nsp = (L + kSdpaSplit - 1) / kSdpaSplit;
      const uint16_t* kb = k + (size_t)kvh * cap * D;
      const uint16_t* vb = v + (size_t)kvh * cap * D;
      std::vector<float> qs(D), ms(nsp), ls(nsp), os((size_t)nsp * D), sc(kSdpaSplit);
      for (int d = 0; d < D; ++d) qs[d] = bf2f(q[((size_t)t * Hq + h) * D + d]) * scale;
      for (int s = 0; s < nsp; ++s) {
        const int j0 = s * kSdpaSplit, j1 = std::min(L, j0 + kSdpaSplit);
        float m = -INFINITY;
        for (int j = j0; j < j1; ++j) {
          float a = 0.0f;
          for (int d = 0; d < D; ++d) a = std::fma(qs[d], bf2f(kb[(size_t)j * D + d]), a);
          sc[j - j0] = a;
          m = std::max(m, a);
        }
        float lp[32] = {0};
        for (int j = j0; j < j1; ++j) {
          sc[j - j0] = orc_exp(sc[j - j0] - m);
          lp[(j - j0) & 31] = lp[(j - j0) & 31] + sc[j - j0];
        }
        for (int off = 16; off >= 1; off >>= 1) {
          float t2[32];
          for (int i = 0; i < 32; ++i) t2[i] = lp[i] + lp[i ^ off];
          std::memcpy(lp, t2, sizeof(lp));
        }
        const float l = lp[0];
        for (int d = 0; d < D; ++d) {
          float o = 0.0f;
          for (int j = j0; j < j1; ++j) o = std::fma(sc[j - j0], bf2f(vb[(size_t)j * D + d]), o);
          os[(size_t)s * D + d] = o;
        }
        ms[s] = m;
        ls[s] = l;
      }
      float M = -INFINITY;
      for (int s = 0; s < nsp; ++s) M = std::max(M, ms[s]);
      float Lt = 0.0f;
      std::vector<float> O(D, 0.0f);
      for (int s = 0; s < nsp; ++s) {
        const float w = orc_exp(ms[s] - M);
        Lt = std::fma(w, ls[s], Lt);
        for (int d = 0; d < D; ++d) O[d] = std::fma(w, os[(size_t)s * D + d], O[d]);
      }
      for (int d = 0; d < D; ++d) out[((size_t)t * Hq + h) * D + d] = f2bf(O[d] / Lt);
    }
}

// ---------------------------------------------------------------------------
// Sampling in exact integer arithmetic (the reference's categorical sampler,
// src/common/generate.cpp:83-120, draws Gumbel noise from MLX's RNG, which is
// not reproducible; both sides here consume the same caller-supplied 24-bit
// uniforms instead, and every decision is an exact integer comparison, so the
// result does not depend on any summation order).
//   w_j   = rint(exp((l_j - max l) * (1/T)) * 2^32)            (uint64)
//   top-p: keep the smallest prefix of tokens ordered by (w desc, index asc)
//          whose mass satisfies 2^24 * kept >= rint(top_p * 2^24) * Z
//   draw:  smallest index t with 2^24 * cumsum_t(kept w) > u24 * Z_kept
// Speculative acceptance (Leviathan et al. 2023; Chen et al. 2023):
//   accept d  iff  u24 * q(d) * Zp < 2^24 * p(d) * Zq
//   on the first rejection draw from r_j = max(0, p_j Zq - q_j Zp);
//   after K acceptances draw the bonus token from p_K.
// ---------------------------------------------------------------------------
struct Dist {
  std::vector<uint64_t> w;
  std::vector<uint8_t> keep;
  uint64_t Z = 0;
};

static void make_dist(const uint16_t* l, int V, float temperature, float top_p, Dist& d) {
  float mx = -INFINITY;
  for (int j = 0; j < V; ++j) {
    float v = bf2f(l[j]);
    if (v == v && v > mx) mx = v;
  }
  const float inv_t = 1.0f / temperature;
  d.w.assign(V, 0);
  d.keep.assign(V, 0);
  uint64_t Z = 0;
  for (int j = 0; j < V; ++j) {
    float v = bf2f(l[j]);
    if (v != v) continue;
    float e = orc_exp((v - mx) * inv_t);
    d.w[j] = (uint64_t)std::llrint(e * 4294967296.0f);
    Z += d.w[j];
  }
  if (!(top_p > 0.0f && top_p < 1.0f)) {
    std::fill(d.keep.begin(), d.keep.end(), 1);
    d.Z = Z;
    return;
  }
  const uint64_t P24 = (uint64_t)std::llrint(top_p * 16777216.0f);
  std::vector<int> order(V);
  for (int j = 0; j < V; ++j) order[j] = j;
  std::sort(order.begin(), order.end(), [&](int a, int b) {
    return d.w[a] != d.w[b] ? d.w[a] > d.w[b] : a < b;
  });
  uint64_t cum = 0;
  for (int i = 0; i < V; ++i) {
    d.keep[order[i]] = 1;
    cum += d.w[order[i]];
    if (((u128)cum << 24) >= (u128)P24 * Z) break;
  }
  d.Z = cum;
}

static int draw_dist(const Dist& d, uint32_t u24) {
  const u128 target = (u128)u24 * d.Z;
  u128 cum = 0;
  int last = 0;
  for (size_t j = 0; j < d.w.size(); ++j) {
    if (!d.keep[j] || d.w[j] == 0) continue;
    cum += d.w[j];
    last = (int)j;
    if ((cum << 24) > target) return (int)j;
  }
  return last;
}

extern "C" int orc_sample(const uint16_t* logits, int V, float temperature, float top_p,
                          uint32_t u24) {
  if (temperature <= 0.0f) {
    int32_t t;
    orc_argmax(logits, 1, V, &t);
    return t;
  }
  Dist d;
  make_dist(logits, V, temperature, top_p, d);
  return draw_dist(d, u24);
}

extern "C" int orc_accept_greedy(const uint16_t* target_logits, const int32_t* drafts, int K,
                                 int V, int32_t* out_tokens) {
  std::vector<int32_t> pred(K + 1);
  orc_argmax(target_logits, K + 1, V, pred.data());
  int acc = 0;
  while (acc < K && pred[acc] == drafts[acc]) {
    out_tokens[acc] = drafts[acc];
    ++acc;
  }
  out_tokens[acc] = pred[acc];
  return acc;
}

extern "C" int orc_accept_stochastic(const uint16_t* target_logits, const uint16_t* draft_logits,
                                     const int32_t* drafts, int K, int V, float temperature,
                                     float top_p, const uint32_t* u_accept, uint32_t u_final,
                                     int32_t* out_tokens) {
  if (temperature <= 0.0f) return orc_accept_greedy(target_logits, drafts, K, V, out_tokens);
  Dist p, q;
  for (int i = 0; i < K; ++i) {
    make_dist(target_logits + (size_t)i * V, V, temperature, top_p, p);
    make_dist(draft_logits + (size_t)i * V, V, temperature, top_p, q);
    const int d = drafts[i];
    const uint64_t pd = p.keep[d] ? p.w[d] : 0, qd = q.keep[d] ? q.w[d] : 0;
    if ((u128)u_accept[i] * qd * p.Z < ((u128)pd * q.Z << 24)) {
      out_tokens[i] = d;
      continue;
    }
    // residual max(0, p - q), drawn by inverse CDF in index order
    std::vector<u128> r(V);
    u128 R = 0;
    for (int j = 0; j < V; ++j) {
      u128 a = p.keep[j] ? (u128)p.w[j] * q.Z : 0, b = q.keep[j] ? (u128)q.w[j] * p.Z : 0;
      r[j] = a > b ? a - b : 0;
      R += r[j];
    }
    if (R == 0) {
      out_tokens[i] = draw_dist(p, u_final);
      return i;
    }
    const u128 target = (u128)u_final * R;
    u128 cum = 0;
    int pick = 0;
    for (int j = 0; j < V; ++j) {
      if (r[j] == 0) continue;
      cum += r[j];
      pick = j;
      if ((cum << 24) > target) break;
    }
    out_tokens[i] = pick;
    return i;
  }
  make_dist(target_logits + (size_t)K * V, V, temperature, top_p, p);
  out_tokens[K] = draw_dist(p, u_final);
  return K;
}

// ---------------------------------------------------------------------------
// Hybrid-model ops (configuration 4): the device engine's gdn_moe.cuh in the
// same canonical orders.  Reference math: Qwen3NextGatedDeltaNet
// (src/llm/models/qwen3_next.cpp:216-403), gated_delta.cpp:603-650,
// 885-921, 948-999, 1067-1138; Qwen3NextSparseMoeBlock (qwen3_next.cpp:
// 452-490), SwitchGLU (src/common/switch_layers.cpp:200-245).
// ---------------------------------------------------------------------------
// log(x), x > 0 normal: x = m 2^e, m in [sqrt(1/2), sqrt(2)); log m =
// 2 atanh((m-1)/(m+1)) by its odd series to u^11; + e ln 2 (split).
extern "C" float orc_log(float x) {
  uint32_t bits;
  std::memcpy(&bits, &x, 4);
  int e = (int)(bits >> 23) - 127;
  float m = u2f((bits & 0x7FFFFFu) | 0x3F800000u);
  if (m > 1.41421356f) {
    m = m * 0.5f;
    e += 1;
  }
  const float u = (m - 1.0f) / (m + 1.0f);
  const float u2 = u * u;
  float p = 0.0909090909f;
  p = std::fma(p, u2, 0.111111111f);
  p = std::fma(p, u2, 0.142857143f);
  p = std::fma(p, u2, 0.2f);
  p = std::fma(p, u2, 0.333333333f);
  p = std::fma(p, u2, 1.0f);
  const float r = (2.0f * u) * p;
  const float fe = (float)e;
  return std::fma(fe, 0.693145752f, std::fma(fe, 1.42860677e-06f, r));
}
static inline float softplus_f(float x) { return x > 20.0f ? x : orc_log(1.0f + orc_exp(x)); }

namespace {
const int kGD = 128, kKS = 4;
}

// Gated DeltaNet verify step (lmx_gdn_verify): reads state / conv_state,
// writes the state after each token to snap [B][T][Hv][128][128] and the
// gated-normed output [B][T][Hv*128].
static int g_gdn_state_bf16 = 1;
extern "C" void orc_set_gdn_state_bf16(int on) { g_gdn_state_bf16 = on ? 1 : 0; }

extern "C" int orc_gdn_verify(int B, int T, int Hk, int Hv, const uint16_t* qkv, const uint16_t* z,
                              const uint16_t* bb, const uint16_t* aa, const uint16_t* conv_w,
                              const float* a_log, const uint16_t* dt_bias, const uint16_t* norm_w, float eps,
                              const uint16_t* conv_state, const float* state, float* snap, uint16_t* out) {
  if (B < 1 || T < 1 || Hk < 1 || Hv % Hk) return 1;
  const int CD = 2 * Hk * kGD + Hv * kGD, rep = Hv / Hk;
  const float wq = bf2f(f2bf(1.0f / kGD)), wk = bf2f(f2bf(0.08838834764831845f));
  for (int b = 0; b < B; ++b) {
    // conv + SiLU for every token and channel, q/k norms, v, beta, g
    std::vector<float> cv((size_t)T * CD), qn((size_t)T * Hk * kGD), kn((size_t)T * Hk * kGD);
    std::vector<float> beta((size_t)T * Hv), gd((size_t)T * Hv);
    for (int t = 0; t < T; ++t) {
      for (int c = 0; c < CD; ++c) {
        float acc = 0.0f;
        for (int i = 0; i < kKS; ++i) {
          const int r = t + i;
          const float x = r < kKS - 1 ? bf2f(conv_state[((size_t)b * (kKS - 1) + r) * CD + c])
                                      : bf2f(qkv[((size_t)b * T + (r - (kKS - 1))) * CD + c]);
          acc = std::fma(bf2f(conv_w[(size_t)c * kKS + i]), x, acc);
        }
        const float y = bf2f(f2bf(acc));
        const float sg = bf2f(f2bf(sigmoid_f(y)));
        cv[(size_t)t * CD + c] = bf2f(f2bf(y * sg));
      }
      for (int s = 0; s < 2 * Hk; ++s) {
        const float* src = &cv[(size_t)t * CD + s * kGD];
        const float f = rms_factor(src, kGD, 1e-6f);
        const float w = s < Hk ? wq : wk;
        float* dst = s < Hk ? &qn[((size_t)t * Hk + s) * kGD] : &kn[((size_t)t * Hk + s - Hk) * kGD];
        for (int d = 0; d < kGD; ++d) dst[d] = bf2f(f2bf((src[d] * f) * w));
      }
      for (int h = 0; h < Hv; ++h) {
        const size_t i = ((size_t)b * T + t) * Hv + h;
        beta[(size_t)t * Hv + h] = bf2f(f2bf(sigmoid_f(bf2f(bb[i]))));
        const float sp = softplus_f(bf2f(aa[i]) + bf2f(dt_bias[h]));
        gd[(size_t)t * Hv + h] = bf2f(f2bf(orc_exp(-(orc_exp(a_log[h]) * sp))));
      }
    }
#pragma omp parallel for schedule(static)
    for (int h = 0; h < Hv; ++h) {
      const int hk = h / rep;
      std::vector<float> S((size_t)kGD * kGD);
      std::memcpy(S.data(), state + (((size_t)b * Hv + h) * kGD) * kGD, S.size() * 4);
      std::vector<float> y(kGD);
      for (int t = 0; t < T; ++t) {
        const float* q = &qn[((size_t)t * Hk + hk) * kGD];
        const float* k = &kn[((size_t)t * Hk + hk) * kGD];
        const float g = gd[(size_t)t * Hv + h], be = beta[(size_t)t * Hv + h];
        for (int dv = 0; dv < kGD; ++dv) {
          float* row = &S[(size_t)dv * kGD];
          float part[2];
          for (int hf = 0; hf < 2; ++hf) {
            float kv = 0.0f;
            for (int j = 0; j < 64; ++j) {
              row[64 * hf + j] = row[64 * hf + j] * g;
              kv = std::fma(row[64 * hf + j], k[64 * hf + j], kv);
            }
            part[hf] = kv;
          }
          const float kv = part[0] + part[1];
          const float v = cv[(size_t)t * CD + 2 * Hk * kGD + h * kGD + dv];
          const float delta = (v - kv) * be;
          float yp[2];
          for (int hf = 0; hf < 2; ++hf) {
            float a = 0.0f;
            for (int j = 0; j < 64; ++j) {
              row[64 * hf + j] = std::fma(delta, k[64 * hf + j], row[64 * hf + j]);
              a = std::fma(row[64 * hf + j], q[64 * hf + j], a);
            }
            yp[hf] = a;
          }
          y[dv] = bf2f(f2bf(yp[0] + yp[1]));
        }
        {
          // the reference stores its per-token / final states as bf16
          // (gated_delta.cpp:93, :162-172); the running state stays fp32
          float* sn = snap + ((((size_t)b * T + t) * Hv + h) * kGD) * kGD;
          if (g_gdn_state_bf16)
            for (size_t i = 0; i < S.size(); ++i) sn[i] = bf2f(f2bf(S[i]));
          else
            std::memcpy(sn, S.data(), S.size() * 4);
        }
        const float f = rms_factor(y.data(), kGD, eps);
        for (int dv = 0; dv < kGD; ++dv) {
          const float nv = bf2f(f2bf((y[dv] * f) * bf2f(norm_w[dv])));
          const float zv = bf2f(z[(((size_t)b * T + t) * Hv + h) * kGD + dv]);
          const float sz = bf2f(f2bf(zv * bf2f(f2bf(sigmoid_f(zv)))));
          out[(((size_t)b * T + t) * Hv + h) * kGD + dv] = f2bf(sz * nv);
        }
      }
    }
  }
  return 0;
}

// lmx_gdn_commit: state[b] = snap[b][acc[b]]; conv_state[b] = the window
// ending at token acc[b] (in place).
extern "C" int orc_gdn_commit(int B, int T, int Hk, int Hv, const uint16_t* qkv, const float* snap,
                              const int32_t* acc, float* state, uint16_t* conv_state) {
  const int CD = 2 * Hk * kGD + Hv * kGD;
  for (int b = 0; b < B; ++b) {
    if (acc[b] < 0) continue;  // finished sequence: unchanged
    const int t = std::min(acc[b], T - 1);
    std::memcpy(state + ((size_t)b * Hv * kGD) * kGD, snap + (((size_t)b * T + t) * Hv * kGD) * kGD,
                (size_t)Hv * kGD * kGD * 4);
    std::vector<uint16_t> win((size_t)(kKS - 1) * CD);
    for (int r = 0; r < kKS - 1; ++r)
      for (int c = 0; c < CD; ++c) {
        const int src = t + 1 + r;
        win[(size_t)r * CD + c] = src < kKS - 1 ? conv_state[((size_t)b * (kKS - 1) + src) * CD + c]
                                                : qkv[((size_t)b * T + src - (kKS - 1)) * CD + c];
      }
    std::memcpy(conv_state + (size_t)b * (kKS - 1) * CD, win.data(), win.size() * 2);
  }
  return 0;
}

// lmx_moe_route: k largest logits (ties: lower index) in descending order,
// w_j = exp(l_j - l_0) / sum (slot order).
extern "C" int orc_moe_route(const uint16_t* logits, int rows, int E, int k, int32_t* idx, float* w) {
  for (int r = 0; r < rows; ++r) {
    const uint16_t* l = logits + (size_t)r * E;
    std::vector<char> taken(E, 0);
    std::vector<float> lv(k);
    for (int j = 0; j < k; ++j) {
      float bv = -INFINITY;
      int bi = -1;
      for (int e = 0; e < E; ++e) {
        const float v = bf2f(l[e]);
        if (taken[e] || v != v) continue;
        if (bi < 0 || v > bv) { bv = v; bi = e; }
      }
      if (bi >= 0) taken[bi] = 1;
      lv[j] = bv;
      idx[(size_t)r * k + j] = bi < 0 ? 0 : bi;
    }
    std::vector<float> e0(k);
    float z = 0.0f;
    for (int j = 0; j < k; ++j) {
      e0[j] = orc_exp(lv[j] - lv[0]);
      z = z + e0[j];
    }
    for (int j = 0; j < k; ++j) w[(size_t)r * k + j] = e0[j] / z;
  }
  return 0;
}

namespace {
// canonical expert dot product (gdn_moe.cuh qd_dot)
float qd_dot(const uint32_t* wr, const uint16_t* sr, const uint16_t* br, const float* x, int K, int bits) {
  const int NC = K / 16;
  float lane[32];
  for (int l = 0; l < 32; ++l) {
    float acc = 0.0f;
    for (int c = l; c < NC; c += 32) {
      float p = 0.0f, xs = 0.0f;
      for (int j = 0; j < 16; ++j) {
        const float q = (float)qcode(wr, 16 * c + j, bits);
        p = std::fma(q, x[16 * c + j], p);
        xs = xs + x[16 * c + j];
      }
      const int g = c >> 2;
      acc = acc + std::fma(bf2f(sr[g]), p, bf2f(br[g]) * xs);
    }
    lane[l] = acc;
  }
  for (int off = 16; off >= 1; off >>= 1) {
    float q[32];
    for (int l = 0; l < 32; ++l) q[l] = lane[l] + lane[l ^ off];
    std::memcpy(lane, q, sizeof(lane));
  }
  return lane[0];
}
}  // namespace

// lmx_moe_experts: y[m] = bf16(fma chain over j of w[m][j] *
// bf16(down_e . swiglu(bf16(gate_e . x), bf16(up_e . x)))).
extern "C" int orc_moe_experts(const uint16_t* x, int M, int H, int I, int E, int k, const int32_t* idx,
                               const float* w, const uint32_t* gw, const uint16_t* gs, const uint16_t* gb,
                               const uint32_t* uw, const uint16_t* us, const uint16_t* ub, const uint32_t* dw,
                               const uint16_t* ds, const uint16_t* db, int bits, uint16_t* y) {
  const size_t wpr_h = (size_t)H * bits / 32, gpr_h = H / 64, wpr_i = (size_t)I * bits / 32, gpr_i = I / 64;
  std::vector<uint16_t> act((size_t)M * k * I);
#pragma omp parallel for schedule(dynamic)
  for (int s = 0; s < M * k; ++s) {
    const int m = s / k, e = idx[s];
    if (e < 0 || e >= E) continue;
    std::vector<float> xf(H);
    for (int i = 0; i < H; ++i) xf[i] = bf2f(x[(size_t)m * H + i]);
    for (int r = 0; r < I; ++r) {
      const size_t row = (size_t)e * I + r;
      const float g = qd_dot(gw + row * wpr_h, gs + row * gpr_h, gb + row * gpr_h, xf.data(), H, bits);
      const float u = qd_dot(uw + row * wpr_h, us + row * gpr_h, ub + row * gpr_h, xf.data(), H, bits);
      act[(size_t)s * I + r] = swiglu1(f2bf(g), f2bf(u));
    }
  }
#pragma omp parallel for schedule(dynamic)
  for (int m = 0; m < M; ++m) {
    std::vector<float> af((size_t)k * I);
    for (size_t i = 0; i < af.size(); ++i) af[i] = bf2f(act[(size_t)m * k * I + i]);
    for (int r = 0; r < H; ++r) {
      float acc = 0.0f;
      for (int j = 0; j < k; ++j) {
        const int e = idx[(size_t)m * k + j];
        if (e < 0 || e >= E) continue;
        const size_t row = (size_t)e * H + r;
        const float v = bf2f(f2bf(qd_dot(dw + row * wpr_i, ds + row * gpr_i, db + row * gpr_i, &af[(size_t)j * I],
                                         I, bits)));
        acc = std::fma(w[(size_t)m * k + j], v, acc);
      }
      y[(size_t)m * H + r] = f2bf(acc);
    }
  }
  return 0;
}

// ---------------------------------------------------------------------------
// Model (Qwen3 / Llama decoder, src/llm/models/qwen3.cpp:69-220,
// src/llm/models/llama.cpp:203-469) with synthetic weights:
// linear and embedding weights N(0,0.02) (Irwin-Hall) in bf16, quantized with
// the rule above; norm weights are ones (the reference's initialisers,
// qwen3.cpp:51-52,129-131,159).  Tensor ids: embed 1, lm_head 2,
// layer l kind k -> (l+1)*16 + k.
// ---------------------------------------------------------------------------
namespace {
struct QW {
  int N = 0, K = 0;
  int bits = 4;  // per weight: a checkpoint's per-layer override may differ from the model's
  std::vector<uint32_t> w;
  std::vector<uint16_t> s, b;
};
struct Layer {
  QW w[7];  // q k v o gate up down
  std::vector<uint16_t> in_norm, post_norm, q_norm, k_norm;
};
struct Model {
  orc_model_cfg c;
  int bits, group;
  std::vector<Layer> L;
  QW embed, lm_head;
  std::vector<uint16_t> final_norm;
  int max_pos = 16384;
  std::vector<float> cos_t, sin_t;
  int tp = 1;  // tensor-parallel emulation of o_proj / down_proj
  const QW& head() const { return c.tied ? embed : lm_head; }
};
struct Cache {
  int L, B, cap, Hk, D, bits;
  std::vector<std::vector<uint16_t>> k, v;             // bf16 [B][Hk][cap][D]
  std::vector<std::vector<uint32_t>> kq, vq;           // packed [B][Hk][cap][D*bits/32]
  std::vector<std::vector<uint16_t>> ks, kb, vs, vb;   // [B][Hk][cap][D/64]
  std::vector<int> len;
};

void gen_qw(QW& q, uint64_t seed, uint32_t tid, int N, int K, int bits, int group) {
  q.N = N;
  q.K = K;
  q.bits = bits;
  std::vector<uint16_t> tmp((size_t)N * K);
  orc_gen_normal_bf16(seed, tid, 0.02f, (int64_t)tmp.size(), tmp.data());
  q.w.resize((size_t)N * K * bits / 32);
  q.s.resize((size_t)N * (K / group));
  q.b.resize(q.s.size());
  orc_quantize(tmp.data(), N, K, group, bits, q.w.data(), q.s.data(), q.b.data());
}

void qmm(const Model& m, const QW& w, const uint16_t* x, uint16_t* y, int M) {
  orc_qmm(x, w.w.data(), w.s.data(), w.b.data(), y, M, w.N, w.K, m.group, w.bits);
}

// h = h + x W^T for the row-split projections (o_proj, down_proj).  With
// m.tp ranks (the device engine's tensor-parallel all-reduce, tp.cuh): rank
// r's partial p_r = bf16(x[:, r-th K/tp columns] W[:, same]^T) in the
// canonical order for K/tp, the sum s = p_0 + p_1 + ... in fp32 in rank
// order, then h = bf16(h + bf16(s)).  tp == 1 is the plain residual add.
void qmm_resid(const Model& m, const QW& w, const uint16_t* x, uint16_t* h, int M) {
  const int N = w.N, K = w.K, tp = m.tp;
  std::vector<uint16_t> a((size_t)M * N);
  if (tp <= 1) {
    qmm(m, w, x, a.data(), M);
    orc_add(h, a.data(), h, (int64_t)M * N);
    return;
  }
  const int Ks = K / tp, G = K / 64, Gs = Ks / 64, WPR = K * w.bits / 32, WPRs = Ks * w.bits / 32;
  std::vector<float> sum((size_t)M * N);
  std::vector<uint16_t> xs((size_t)M * Ks), ss((size_t)N * Gs), bs((size_t)N * Gs);
  std::vector<uint32_t> ws((size_t)N * WPRs);
  for (int r = 0; r < tp; ++r) {
    for (int i = 0; i < M; ++i) std::memcpy(&xs[(size_t)i * Ks], x + (size_t)i * K + (size_t)r * Ks, Ks * 2);
    for (int n = 0; n < N; ++n) {
      std::memcpy(&ws[(size_t)n * WPRs], &w.w[(size_t)n * WPR + (size_t)r * WPRs], WPRs * 4);
      std::memcpy(&ss[(size_t)n * Gs], &w.s[(size_t)n * G + (size_t)r * Gs], Gs * 2);
      std::memcpy(&bs[(size_t)n * Gs], &w.b[(size_t)n * G + (size_t)r * Gs], Gs * 2);
    }
    orc_qmm(xs.data(), ws.data(), ss.data(), bs.data(), a.data(), M, N, Ks, m.group, w.bits);
    for (size_t i = 0; i < sum.size(); ++i) sum[i] = r == 0 ? bf2f(a[i]) : sum[i] + bf2f(a[i]);
  }
  for (size_t i = 0; i < sum.size(); ++i) h[i] = f2bf(bf2f(f2bf(sum[i])) + bf2f(h[i]));
}
}  // namespace

extern "C" int orc_model_set_tp(void* mp, int tp) {
  Model& m = *(Model*)mp;
  const orc_model_cfg& c = m.c;
  if (tp < 1 || c.heads % tp || c.kv_heads % tp || c.inter % (64 * tp) || c.vocab % tp) return 1;
  m.tp = tp;
  return 0;
}

extern "C" void* orc_model_create(const orc_model_cfg* cfg, uint64_t seed) {
  if (cfg->group != 64 || (cfg->bits != 4 && cfg->bits != 8)) return nullptr;
  Model* m = new Model();
  m->c = *cfg;
  m->bits = cfg->bits;
  m->group = cfg->group;
  const int H = cfg->hidden, D = cfg->head_dim, I = cfg->inter;
  const int NQ = cfg->heads * D, NK = cfg->kv_heads * D;
  m->L.resize(cfg->layers);
  for (int l = 0; l < cfg->layers; ++l) {
    Layer& L = m->L[l];
    const int shp[7][2] = {{NQ, H}, {NK, H}, {NK, H}, {H, NQ}, {I, H}, {I, H}, {H, I}};
    for (int k = 0; k < 7; ++k)
      gen_qw(L.w[k], seed, (uint32_t)((l + 1) * 16 + k), shp[k][0], shp[k][1], m->bits, m->group);
    L.in_norm.assign(H, f2bf(1.0f));
    L.post_norm.assign(H, f2bf(1.0f));
    L.q_norm.assign(D, f2bf(1.0f));
    L.k_norm.assign(D, f2bf(1.0f));
  }
  gen_qw(m->embed, seed, 1, cfg->vocab, H, m->bits, m->group);
  if (!cfg->tied) gen_qw(m->lm_head, seed, 2, cfg->vocab, H, m->bits, m->group);
  m->final_norm.assign(H, f2bf(1.0f));
  m->cos_t.resize((size_t)m->max_pos * D / 2);
  m->sin_t.resize(m->cos_t.size());
  orc_rope_table_scaled(m->max_pos, D, cfg->rope_theta, cfg->rope_factor, cfg->rope_low_freq, cfg->rope_high_freq,
                        cfg->rope_orig_max_pos, m->cos_t.data(), m->sin_t.data());
  return m;
}

extern "C" void orc_model_free(void* m) { delete (Model*)m; }

// Install a checkpoint's tensors (test infrastructure: the tests read the
// safetensors file themselves and hand the arrays over).  kind as
// orc_model_weight; N x K is the weight's own shape, which must match the
// model's for that slot.
extern "C" int orc_model_set_weight(void* mp, int layer, int kind, int bits, const uint32_t* wq, const uint16_t* s,
                                    const uint16_t* b) {
  Model& m = *(Model*)mp;
  QW* q = nullptr;
  if (kind == 7) q = &m.embed;
  else if (kind == 8 && !m.c.tied) q = &m.lm_head;
  else if (layer >= 0 && layer < (int)m.L.size() && kind >= 0 && kind < 7) q = &m.L[layer].w[kind];
  if (!q || (bits != 4 && bits != 8)) return 1;
  q->bits = bits;
  q->w.assign(wq, wq + (size_t)q->N * q->K * bits / 32);
  q->s.assign(s, s + (size_t)q->N * (q->K / 64));
  q->b.assign(b, b + (size_t)q->N * (q->K / 64));
  return 0;
}

// which: 0 input_layernorm, 1 post_attention_layernorm, 2 q_norm, 3 k_norm
// (of `layer`), 4 the final norm.
extern "C" int orc_model_set_norm(void* mp, int layer, int which, const uint16_t* v) {
  Model& m = *(Model*)mp;
  std::vector<uint16_t>* dst = nullptr;
  if (which == 4) dst = &m.final_norm;
  else if (layer >= 0 && layer < (int)m.L.size()) {
    Layer& L = m.L[layer];
    dst = which == 0 ? &L.in_norm : which == 1 ? &L.post_norm : which == 2 ? &L.q_norm : which == 3 ? &L.k_norm : nullptr;
  }
  if (!dst) return 1;
  std::copy(v, v + dst->size(), dst->begin());
  return 0;
}

extern "C" int orc_model_weight(void* mp, int layer, int kind, uint32_t* wq, uint16_t* s,
                                uint16_t* b) {
  Model& m = *(Model*)mp;
  const QW* q = nullptr;
  if (kind == 7) q = &m.embed;
  else if (kind == 8) q = &m.head();
  else if (layer >= 0 && layer < (int)m.L.size() && kind >= 0 && kind < 7) q = &m.L[layer].w[kind];
  if (!q) return 1;
  std::memcpy(wq, q->w.data(), q->w.size() * 4);
  std::memcpy(s, q->s.data(), q->s.size() * 2);
  std::memcpy(b, q->b.data(), q->b.size() * 2);
  return 0;
}

extern "C" void* orc_cache_create(void* mp, int n_layers, int batch, int capacity, int kv_bits) {
  Model& m = *(Model*)mp;
  if (kv_bits != 16 && kv_bits != 4 && kv_bits != 8) return nullptr;
  Cache* c = new Cache();
  c->L = n_layers;
  c->B = batch;
  c->cap = capacity;
  c->Hk = m.c.kv_heads;
  c->D = m.c.head_dim;
  c->bits = kv_bits;
  c->len.assign(batch, 0);
  const size_t rows = (size_t)batch * c->Hk * capacity;
  for (int l = 0; l < n_layers; ++l) {
    if (kv_bits == 16) {
      c->k.emplace_back(rows * c->D, 0);
      c->v.emplace_back(rows * c->D, 0);
    } else {
      c->kq.emplace_back(rows * c->D * kv_bits / 32, 0);
      c->vq.emplace_back(rows * c->D * kv_bits / 32, 0);
      for (auto* a : {&c->ks, &c->kb, &c->vs, &c->vb}) a->emplace_back(rows * (c->D / 64), 0);
    }
  }
  return c;
}
// Synthetic context (the device engine's fill_kv_kernel): rows [0, rows) of
// every layer's K and V are N(0,1) bf16 from the Philox normal, tensor id
// tid_base + 2*layer + (0 K, 1 V), element ((b*Hk + hk)*rows + j)*D + d,
// quantized per group of 64 like an append; every length becomes rows.
extern "C" int orc_cache_fill_synthetic(void* cp, int rows, uint64_t seed, uint32_t tid_base) {
  Cache& c = *(Cache*)cp;
  if (rows < 0 || rows > c.cap) return 1;
  const float C = orc_normal_scale(1.0f);
  const int D = c.D;
  for (int l = 0; l < c.L; ++l)
    for (int v = 0; v < 2; ++v) {
      const uint32_t tid = tid_base + 2u * (uint32_t)l + (uint32_t)v;
#pragma omp parallel for schedule(static)
      for (int64_t t = 0; t < (int64_t)c.B * c.Hk * rows; ++t) {
        const int j = (int)(t % rows);
        const int64_t bh = t / rows;  // b * Hk + hk
        const size_t row = (size_t)bh * c.cap + j;
        uint16_t vals[256];
        for (int d = 0; d < D; ++d) vals[d] = normal_bf16(seed, tid, (uint64_t)t * D + d, C);
        if (c.bits == 16) {
          std::memcpy(&(v ? c.v : c.k)[l][row * D], vals, D * 2);
        } else {
          const int WPR = D * c.bits / 32, gpr = D / 64;
          for (int gi = 0; gi < gpr; ++gi)
            quantize_group(vals + 64 * gi, 64, c.bits, &(v ? c.vq : c.kq)[l][row * WPR + gi * 64 * c.bits / 32],
                           &(v ? c.vs : c.ks)[l][row * gpr + gi], &(v ? c.vb : c.kb)[l][row * gpr + gi]);
        }
      }
    }
  for (int b = 0; b < c.B; ++b) c.len[b] = rows;
  return 0;
}

extern "C" void orc_cache_free(void* c) { delete (Cache*)c; }
extern "C" int orc_cache_len(void* c, int b) { return ((Cache*)c)->len[b]; }
extern "C" void orc_cache_set_position(void* cp, int b, int pos) {
  Cache& c = *(Cache*)cp;
  if (pos < c.len[b]) c.len[b] = pos;  // rows past pos are dead (kv_cache.cpp:135-142)
}

// Forward T tokens per sequence through layers [0, n_layers), then the final
// norm and lm_head (for every position, or only each sequence's last one).
static int forward_impl(Model& m, Cache& c, int n_layers, const int32_t* tokens, int B, int T,
                        uint16_t* logits, bool last_only) {
  const orc_model_cfg& cf = m.c;
  const int H = cf.hidden, D = cf.head_dim, Hq = cf.heads, Hk = cf.kv_heads, R = B * T;
  const int NQ = Hq * D, NK = Hk * D, I = cf.inter, G = H / 64;
  if (n_layers > c.L || B != c.B) return 1;
  for (int b = 0; b < B; ++b)
    if (c.len[b] + T > c.cap || c.len[b] + T > m.max_pos) return 2;
  std::vector<uint16_t> h((size_t)R * H), xn((size_t)R * H), q((size_t)R * NQ), k((size_t)R * NK),
      v((size_t)R * NK), o((size_t)R * NQ), a((size_t)R * H), g((size_t)R * I), u((size_t)R * I);
  // embedding lookup = dequantized row of the packed table
  for (int r = 0; r < R; ++r) {
    const int tok = tokens[r];
    const uint32_t* row = m.embed.w.data() + (size_t)tok * H * m.embed.bits / 32;
    for (int i = 0; i < H; ++i) {
      float s = bf2f(m.embed.s[(size_t)tok * G + i / 64]), bb = bf2f(m.embed.b[(size_t)tok * G + i / 64]);
      h[(size_t)r * H + i] = f2bf(std::fma(s, (float)qcode(row, i, m.embed.bits), bb));
    }
  }
  std::vector<int32_t> pos(R);
  for (int b = 0; b < B; ++b)
    for (int t = 0; t < T; ++t) pos[b * T + t] = c.len[b] + t;
  const float scale = (float)(1.0 / std::sqrt((double)D));
  for (int l = 0; l < n_layers; ++l) {
    Layer& L = m.L[l];
    orc_rms_norm(h.data(), L.in_norm.data(), xn.data(), R, H, cf.eps);
    qmm(m, L.w[0], xn.data(), q.data(), R);
    qmm(m, L.w[1], xn.data(), k.data(), R);
    qmm(m, L.w[2], xn.data(), v.data(), R);
    if (cf.qk_norm) {
      orc_rms_norm(q.data(), L.q_norm.data(), q.data(), R * Hq, D, cf.eps);
      orc_rms_norm(k.data(), L.k_norm.data(), k.data(), R * Hk, D, cf.eps);
    }
    orc_rope(q.data(), pos.data(), R, Hq, D, m.cos_t.data(), m.sin_t.data());
    orc_rope(k.data(), pos.data(), R, Hk, D, m.cos_t.data(), m.sin_t.data());
    // KV append at each sequence's offset (quantize on append for 4/8-bit)
    for (int b = 0; b < B; ++b)
      for (int t = 0; t < T; ++t)
        for (int hk = 0; hk < Hk; ++hk) {
          const size_t row = ((size_t)b * Hk + hk) * c.cap + (size_t)(c.len[b] + t);
          const uint16_t* ks = &k[((size_t)(b * T + t) * Hk + hk) * D];
          const uint16_t* vs = &v[((size_t)(b * T + t) * Hk + hk) * D];
          if (c.bits == 16) {
            std::memcpy(&c.k[l][row * D], ks, D * 2);
            std::memcpy(&c.v[l][row * D], vs, D * 2);
          } else {
            const int WPR = D * c.bits / 32, gpr = D / 64;
            for (int gi = 0; gi < gpr; ++gi) {
              quantize_group(ks + 64 * gi, 64, c.bits, &c.kq[l][row * WPR + gi * 64 * c.bits / 32],
                             &c.ks[l][row * gpr + gi], &c.kb[l][row * gpr + gi]);
              quantize_group(vs + 64 * gi, 64, c.bits, &c.vq[l][row * WPR + gi * 64 * c.bits / 32],
                             &c.vs[l][row * gpr + gi], &c.vb[l][row * gpr + gi]);
            }
          }
        }
    for (int b = 0; b < B; ++b) {
      const uint16_t* kb;
      const uint16_t* vb;
      std::vector<uint16_t> kd, vd;
      const size_t base = (size_t)b * Hk * c.cap;
      if (c.bits == 16) {
        kb = &c.k[l][base * D];
        vb = &c.v[l][base * D];
      } else {  // the reference dequantizes the whole cache (kv_cache.cpp:271-298)
        const int WPR = D * c.bits / 32, gpr = D / 64;
        kd.assign((size_t)Hk * c.cap * D, 0);
        vd.assign(kd.size(), 0);
        for (int hk = 0; hk < Hk; ++hk)
          for (int j = 0; j < c.len[b] + T; ++j) {
            const size_t row = base + (size_t)hk * c.cap + j;
            for (int d = 0; d < D; ++d) {
              const int gi = d / 64;
              kd[((size_t)hk * c.cap + j) * D + d] = f2bf(std::fma(bf2f(c.ks[l][row * gpr + gi]),
                  (float)qcode(&c.kq[l][row * WPR], d, c.bits), bf2f(c.kb[l][row * gpr + gi])));
              vd[((size_t)hk * c.cap + j) * D + d] = f2bf(std::fma(bf2f(c.vs[l][row * gpr + gi]),
                  (float)qcode(&c.vq[l][row * WPR], d, c.bits), bf2f(c.vb[l][row * gpr + gi])));
            }
          }
        kb = kd.data();
        vb = vd.data();
      }
      orc_sdpa(&q[(size_t)b * T * NQ], kb, vb, &o[(size_t)b * T * NQ], T, Hq, Hk, D, c.cap,
               c.len[b], scale);
    }
    qmm_resid(m, L.w[3], o.data(), h.data(), R);
    orc_rms_norm(h.data(), L.post_norm.data(), xn.data(), R, H, cf.eps);
    qmm(m, L.w[4], xn.data(), g.data(), R);
    qmm(m, L.w[5], xn.data(), u.data(), R);
    orc_swiglu(g.data(), u.data(), g.data(), (int64_t)R * I);
    qmm_resid(m, L.w[6], g.data(), h.data(), R);
  }
  for (int b = 0; b < B; ++b) c.len[b] += T;
  if (!logits) return 0;
  if (last_only) {
    std::vector<uint16_t> hl((size_t)B * H);
    for (int b = 0; b < B; ++b)
      std::memcpy(&hl[(size_t)b * H], &h[((size_t)b * T + T - 1) * H], H * 2);
    orc_rms_norm(hl.data(), m.final_norm.data(), hl.data(), B, H, cf.eps);
    qmm(m, m.head(), hl.data(), logits, B);
  } else {
    orc_rms_norm(h.data(), m.final_norm.data(), xn.data(), R, H, cf.eps);
    qmm(m, m.head(), xn.data(), logits, R);
  }
  return 0;
}

// Prefill in chunks of kPrefillChunk tokens per sequence (the device engine's
// prefill chunking), so that every quantized matmul sees the same M on both
// sides and takes the same path; logits of each sequence's last token.
static constexpr int kPrefillChunk = 32;
// REF_KV_PAD_QUIRK (the reference's maybe_quantize_kv_cache, src/common/
// kv_cache.cpp:391-413): the prompt is prefilled into a bf16 KVCacheSimple,
// whose first allocation is max(first chunk, 256) rows and which grows to
// max(2 alloc, offset + n) when a chunk does not fit (kv_cache.cpp:34-110,
// include/mlx-lm/common/kv_cache.h:43); the prompt goes in chunks of 512
// while more than 512 remain, then the rest (llm_model.h:18-60).  After the
// prompt the WHOLE allocation -- zero rows past the prompt included -- is
// quantized and the cache offset becomes the allocation length.
static int g_kv_quirk = 0;
extern "C" void orc_set_kv_quirk(int on) { g_kv_quirk = on ? 1 : 0; }
extern "C" int orc_kv_quirk_alloc(int n) {
  int alloc = 0, off = 0, rem = n;
  while (rem > 0) {
    const int c = rem > 512 ? 512 : rem;
    if (alloc == 0) alloc = std::max(c, 256);
    else if (off + c > alloc) alloc = std::max(2 * alloc, off + c);
    off += c;
    rem -= c;
  }
  return alloc;
}
// Quantize rows [0, rows) of every layer of the bf16 cache `src` into the
// quantized cache `dst` (same geometry) and set every length to rows.
static void quirk_convert(const Cache& src, Cache& dst, int rows) {
  const int D = src.D, WPR = D * dst.bits / 32, gpr = D / 64;
  for (int l = 0; l < dst.L; ++l)
    for (int b = 0; b < dst.B; ++b)
      for (int hk = 0; hk < dst.Hk; ++hk)
        for (int j = 0; j < rows; ++j) {
          const size_t rs = ((size_t)b * src.Hk + hk) * src.cap + j, rd = ((size_t)b * dst.Hk + hk) * dst.cap + j;
          for (int gi = 0; gi < gpr; ++gi) {
            quantize_group(&src.k[l][rs * D + 64 * gi], 64, dst.bits, &dst.kq[l][rd * WPR + gi * 64 * dst.bits / 32],
                           &dst.ks[l][rd * gpr + gi], &dst.kb[l][rd * gpr + gi]);
            quantize_group(&src.v[l][rs * D + 64 * gi], 64, dst.bits, &dst.vq[l][rd * WPR + gi * 64 * dst.bits / 32],
                           &dst.vs[l][rd * gpr + gi], &dst.vb[l][rd * gpr + gi]);
          }
        }
  for (int b = 0; b < dst.B; ++b) dst.len[b] = rows;
}

static int prefill_chunked(Model& m, Cache& c, int n_layers, const int32_t* tokens, int ld, int B, int T,
                           uint16_t* last_logits) {
  std::vector<int32_t> chunk;
  for (int t0 = 0; t0 < T; t0 += kPrefillChunk) {
    const int tn = std::min(kPrefillChunk, T - t0);
    chunk.resize((size_t)B * tn);
    for (int b = 0; b < B; ++b) std::memcpy(&chunk[(size_t)b * tn], tokens + (size_t)b * ld + t0, tn * 4);
    const bool last = t0 + tn >= T;
    const int rc = forward_impl(m, c, n_layers, chunk.data(), B, tn, last ? last_logits : nullptr, true);
    if (rc) return rc;
  }
  return 0;
}

extern "C" int orc_forward(void* model, void* cache, int n_layers, const int32_t* tokens, int B,
                           int T, uint16_t* logits) {
  return forward_impl(*(Model*)model, *(Cache*)cache, n_layers, tokens, B, T, logits, false);
}

// Speculative decode (src/common/generate.cpp:669-933 generalised to a draft
// model).  Per step and sequence, with p = target length and y = the token at
// position p (already decided, emitted first -- "d0"):
//   draft forward over [x_(p-1), y] (re-writes position p-1 so a fully
//   accepted previous step needs no catch-up), then K-1 single-token forwards;
//   each draft token is argmax (greedy) or a draw from q (uniform stream 0);
//   verify: target forward over [y, d1..dK] (K+1 tokens);
//   accept: greedy prefix match, or rejection sampling (streams 1 and 2);
//   emit y, d1..d_acc; the next y is the correction / bonus token;
//   rollback: target length p+acc+1, draft length p+acc.
namespace {
struct Session {
  Model* tm;
  Model* dm;
  int dl, B, P, K, V, MT;
  orc_spec_params prm;
  bool greedy;
  std::unique_ptr<Cache> tc, dc;
  std::vector<int32_t> y, last, out;
  std::vector<int> emitted;
  uint32_t step = 1;
  int64_t steps = 0, proposed = 0, accepted = 0, prefill_ns = 0;
};
}  // namespace

extern "C" void* orc_spec_session(void* target, void* draft, const int32_t* prompts, int B, int P,
                                  const orc_spec_params* prm, int kv_bits) {
  auto ss = std::make_unique<Session>();
  ss->tm = (Model*)target;
  ss->dm = draft ? (Model*)draft : ss->tm;
  ss->dl = draft ? ss->dm->c.layers : prm->draft_layers;
  ss->B = B;
  ss->P = P;
  ss->K = prm->K;
  ss->V = ss->tm->c.vocab;
  ss->MT = prm->max_tokens;
  ss->prm = *prm;
  ss->greedy = !(prm->temperature > 0.0f);
  Model& tm = *ss->tm;
  Model& dm = *ss->dm;
  const int K = ss->K, V = ss->V, dl = ss->dl;
  if (K < 1 || dl < 1 || dl > dm.c.layers || P < 2 || dm.c.vocab != V) return nullptr;
  if (prm->context_len < 0) return nullptr;
  const int ctx = prm->context_len;
  const bool quirk = g_kv_quirk && kv_bits != 16;
  const int at = quirk ? orc_kv_quirk_alloc(ctx + P) : ctx + P, ad = quirk ? orc_kv_quirk_alloc(ctx + P - 1) : ctx + P;
  const int cap = std::max(at, ad) + ss->MT + K + 8;
  ss->tc.reset((Cache*)orc_cache_create(&tm, tm.c.layers, B, cap, kv_bits));
  ss->dc.reset((Cache*)orc_cache_create(&dm, dl, B, cap, kv_bits));
  if (!ss->tc || !ss->dc) return nullptr;
  // quirk: the prompt goes into bf16 caches first (converted below)
  std::unique_ptr<Cache> tq, dq;
  if (quirk) {
    tq.reset((Cache*)orc_cache_create(&tm, tm.c.layers, B, cap, 16));
    dq.reset((Cache*)orc_cache_create(&dm, dl, B, cap, 16));
  }
  Cache& tpre = quirk ? *tq : *ss->tc;
  Cache& dpre = quirk ? *dq : *ss->dc;
  // the synthetic context precedes the prompt in both caches (tensor ids as
  // the device engine: target 0x40000000, draft 0x50000000)
  if (ctx > 0 && (orc_cache_fill_synthetic(&tpre, ctx, prm->context_seed, 0x40000000u) ||
                  orc_cache_fill_synthetic(&dpre, ctx, prm->context_seed, 0x50000000u)))
    return nullptr;
  const auto t0 = std::chrono::steady_clock::now();
  std::vector<uint16_t> lg((size_t)B * V);
  if (prefill_chunked(tm, tpre, tm.c.layers, prompts, P, B, P, lg.data())) return nullptr;
  ss->y.resize(B);
  ss->last.resize(B);
  std::vector<int32_t> pp((size_t)B * (P - 1));
  for (int b = 0; b < B; ++b) {
    ss->y[b] = ss->greedy ? orc_sample(&lg[(size_t)b * V], V, 0.0f, 1.0f, 0)
                          : orc_sample(&lg[(size_t)b * V], V, prm->temperature, prm->top_p,
                                       orc_uniform24(prm->seed, b, 0, 0, 3));
    ss->last[b] = prompts[(size_t)b * P + P - 1];
    std::memcpy(&pp[(size_t)b * (P - 1)], &prompts[(size_t)b * P], (P - 1) * 4);
  }
  if (prefill_chunked(dm, dpre, dl, pp.data(), P - 1, B, P - 1, nullptr)) return nullptr;
  if (quirk) {
    quirk_convert(*tq, *ss->tc, at);
    quirk_convert(*dq, *ss->dc, ad);
  }
  ss->prefill_ns =
      std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0).count();
  ss->emitted.assign(B, 0);
  ss->out.assign((size_t)B * ss->MT, 0);
  return ss.release();
}

// Run up to n speculative steps (stops early once every sequence has
// max_tokens).  Returns the number of steps run, or -1 on error.
extern "C" int orc_spec_session_step(void* sp, int n) {
  Session& ss = *(Session*)sp;
  Model& tm = *ss.tm;
  Model& dm = *ss.dm;
  const int B = ss.B, K = ss.K, V = ss.V, MT = ss.MT, dl = ss.dl;
  const orc_spec_params* prm = &ss.prm;
  const bool greedy = ss.greedy;
  std::vector<int32_t> d((size_t)B * K), tok2((size_t)B * 2), vt((size_t)B * (K + 1)), outt(K + 1);
  std::vector<uint16_t> lg((size_t)B * V), qlog((size_t)B * K * V), tlog((size_t)B * (K + 1) * V);
  int done_steps = 0;
  for (; done_steps < n; ++done_steps) {
    bool any = false;
    for (int b = 0; b < B; ++b) any |= ss.emitted[b] < MT;
    if (!any) break;
    const uint32_t step = ss.step++;
    for (int b = 0; b < B; ++b) {
      tok2[2 * b] = ss.last[b];
      tok2[2 * b + 1] = ss.y[b];
    }
    for (int i = 0; i < K; ++i) {
      int rc;
      if (i == 0) rc = forward_impl(dm, *ss.dc, dl, tok2.data(), B, 2, lg.data(), true);
      else {
        std::vector<int32_t> t1(B);
        for (int b = 0; b < B; ++b) t1[b] = d[(size_t)b * K + i - 1];
        rc = forward_impl(dm, *ss.dc, dl, t1.data(), B, 1, lg.data(), true);
      }
      if (rc) return -1;
      for (int b = 0; b < B; ++b) {
        std::memcpy(&qlog[((size_t)b * K + i) * V], &lg[(size_t)b * V], (size_t)V * 2);
        d[(size_t)b * K + i] =
            greedy ? orc_sample(&lg[(size_t)b * V], V, 0.0f, 1.0f, 0)
                   : orc_sample(&lg[(size_t)b * V], V, prm->temperature, prm->top_p,
                                orc_uniform24(prm->seed, b, step, i, 0));
      }
    }
    for (int b = 0; b < B; ++b) {
      vt[(size_t)b * (K + 1)] = ss.y[b];
      for (int i = 0; i < K; ++i) vt[(size_t)b * (K + 1) + 1 + i] = d[(size_t)b * K + i];
    }
    std::vector<int> p0(B);
    for (int b = 0; b < B; ++b) p0[b] = ss.tc->len[b];
    if (forward_impl(tm, *ss.tc, tm.c.layers, vt.data(), B, K + 1, tlog.data(), false)) return -1;
    for (int b = 0; b < B; ++b) {
      if (ss.emitted[b] >= MT) {  // finished: recompute the same step, never advance
        ss.tc->len[b] = p0[b];
        ss.dc->len[b] = p0[b] - 1;
        continue;
      }
      int acc;
      if (greedy) {
        acc = orc_accept_greedy(&tlog[(size_t)b * (K + 1) * V], &d[(size_t)b * K], K, V, outt.data());
      } else {
        std::vector<uint32_t> ua(K);
        for (int i = 0; i < K; ++i) ua[i] = orc_uniform24(prm->seed, b, step, i, 1);
        acc = orc_accept_stochastic(&tlog[(size_t)b * (K + 1) * V], &qlog[(size_t)b * K * V],
                                    &d[(size_t)b * K], K, V, prm->temperature, prm->top_p,
                                    ua.data(), orc_uniform24(prm->seed, b, step, 0, 2), outt.data());
      }
      ss.out[(size_t)b * MT + ss.emitted[b]++] = ss.y[b];
      for (int i = 0; i < acc; ++i)
        if (ss.emitted[b] < MT) ss.out[(size_t)b * MT + ss.emitted[b]++] = outt[i];
      ss.last[b] = acc > 0 ? outt[acc - 1] : ss.y[b];
      ss.y[b] = outt[acc];
      ss.tc->len[b] = p0[b] + acc + 1;
      ss.dc->len[b] = p0[b] + acc;
      ss.accepted += acc;
      ss.proposed += K;
    }
    ss.steps += 1;
  }
  return done_steps;
}

// out [B, max_tokens]; stats: steps, proposed, accepted, emitted, prefill ns.
extern "C" void orc_spec_session_result(void* sp, int32_t* out, int64_t* stats) {
  Session& ss = *(Session*)sp;
  if (out) std::memcpy(out, ss.out.data(), ss.out.size() * 4);
  if (stats) {
    int64_t e = 0;
    for (int v : ss.emitted) e += v;
    stats[0] = ss.steps;
    stats[1] = ss.proposed;
    stats[2] = ss.accepted;
    stats[3] = e;
    stats[4] = ss.prefill_ns;
  }
}

extern "C" void orc_spec_session_free(void* sp) { delete (Session*)sp; }

// Speculative decode (src/common/generate.cpp:669-933 generalised to a draft
// model).  Per step and sequence, with p = target length and y = the token at
// position p (already decided, emitted first -- "d0"):
//   draft forward over [x_(p-1), y] (re-writes position p-1 so a fully
//   accepted previous step needs no catch-up), then K-1 single-token forwards;
//   each draft token is argmax (greedy) or a draw from q (uniform stream 0);
//   verify: target forward over [y, d1..dK] (K+1 tokens);
//   accept: greedy prefix match, or rejection sampling (streams 1 and 2);
//   emit y, d1..d_acc; the next y is the correction / bonus token;
//   rollback: target length p+acc+1, draft length p+acc.
extern "C" int orc_spec_generate(void* target, void* draft, const int32_t* prompts, int B, int P,
                                 const orc_spec_params* prm, int kv_bits, int32_t* out,
                                 int64_t* stats) {
  void* ss = orc_spec_session(target, draft, prompts, B, P, prm, kv_bits);
  if (!ss) return 1;
  const auto t0 = std::chrono::steady_clock::now();
  int rc = 0;
  while (true) {
    int n = orc_spec_session_step(ss, 1 << 20);
    if (n < 0) { rc = 2; break; }
    if (n < (1 << 20)) break;
  }
  const int64_t dec =
      std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0).count();
  int64_t st[5];
  orc_spec_session_result(ss, out, st);
  if (stats) {
    stats[0] = st[0];
    stats[1] = st[1];
    stats[2] = st[2];
    stats[3] = st[4];
    stats[4] = dec;
  }
  orc_spec_session_free(ss);
  return rc;
}

extern "C" int orc_generate(void* target, const int32_t* prompts, int B, int P, int max_tokens,
                            int kv_bits, int32_t* out) {
  Model& tm = *(Model*)target;
  const int V = tm.c.vocab;
  std::unique_ptr<Cache> tc((Cache*)orc_cache_create(&tm, tm.c.layers, B, P + max_tokens + 8, kv_bits));
  if (!tc) return 1;
  std::vector<uint16_t> lg((size_t)B * V);
  int rc = prefill_chunked(tm, *tc, tm.c.layers, prompts, P, B, P, lg.data());
  if (rc) return rc;
  std::vector<int32_t> y(B);
  orc_argmax(lg.data(), B, V, y.data());
  for (int i = 0; i < max_tokens; ++i) {
    for (int b = 0; b < B; ++b) out[(size_t)b * max_tokens + i] = y[b];
    if (i + 1 == max_tokens) break;
    rc = forward_impl(tm, *tc, tm.c.layers, y.data(), B, 1, lg.data(), true);
    if (rc) return rc;
    orc_argmax(lg.data(), B, V, y.data());
  }
  return 0;
}

// ---------------------------------------------------------------------------
// Hybrid (Qwen3-Next-style) model and its MTP speculative loop: the device
// engine's hybrid.cuh composition, operation for operation (reference:
// src/llm/models/qwen3_next.cpp:118-490, mtp_head.cpp:146-178,
// src/common/generate.cpp:669-933).
// ---------------------------------------------------------------------------
namespace {
struct HLayer {
  bool attn = false;
  QW q, k, v, qg, o, wqkv, wz, wb, wa, wout, router, eg, eu, ed, sg, su, sd, sgate;
  std::vector<uint16_t> conv_w, dt_bias;
  std::vector<float> a_log;
};
struct HModel {
  orc_hybrid_cfg c;
  std::vector<HLayer> L;
  HLayer mtp;
  QW embed, lm_head, mtp_fc;
  int max_pos = 16384, n_attn = 0, n_gdn = 0, CD = 0;
  std::vector<float> cos_t, sin_t;
};
struct HGdn {
  std::vector<uint16_t> conv, qkv;  // conv [B][3][CD]; the last forward's inputs [B][T][CD]
  std::vector<float> state, snap;   // [B][Hv][128][128]; [B][T][Hv][128][128]
};
struct HState {
  int B = 0, cap = 0, T = 0;
  std::unique_ptr<Cache> kv, mtp_kv;
  std::vector<HGdn> gdn;
  std::vector<uint16_t> hid;  // final-normed hidden of the last forward [B*T][H]
};

std::vector<uint16_t> gen_bf16v(uint64_t seed, uint32_t tid, int64_t n, float std_dev) {
  std::vector<uint16_t> v((size_t)n);
  const float C = orc_normal_scale(std_dev);
  for (int64_t i = 0; i < n; ++i) v[(size_t)i] = normal_bf16(seed, tid, (uint64_t)i, C);
  return v;
}

void hqmm(const QW& w, const uint16_t* x, uint16_t* y, int M, int bits) {
  orc_qmm(x, w.w.data(), w.s.data(), w.b.data(), y, M, w.N, w.K, 64, bits);
}

void hyb_layer_gen(HModel& m, HLayer& L, int l, bool attn, uint64_t seed) {
  const orc_hybrid_cfg& c = m.c;
  const int H = c.hidden, NQ = c.heads * kGD, NK = c.kv_heads * kGD, bits = c.bits;
  const uint32_t base = (uint32_t)(l + 1) * 64;
  L.attn = attn;
  if (attn) {
    gen_qw(L.q, seed, base + 0, NQ, H, bits, 64);
    gen_qw(L.k, seed, base + 1, NK, H, bits, 64);
    gen_qw(L.v, seed, base + 2, NK, H, bits, 64);
    gen_qw(L.qg, seed, base + 3, NQ, H, bits, 64);
    gen_qw(L.o, seed, base + 4, H, NQ, bits, 64);
  } else {
    const int Z = c.lin_v_heads * kGD;
    gen_qw(L.wqkv, seed, base + 8, m.CD, H, bits, 64);
    gen_qw(L.wz, seed, base + 9, Z, H, bits, 64);
    gen_qw(L.wb, seed, base + 10, c.lin_v_heads, H, bits, 64);
    gen_qw(L.wa, seed, base + 11, c.lin_v_heads, H, bits, 64);
    gen_qw(L.wout, seed, base + 12, H, Z, bits, 64);
    L.conv_w = gen_bf16v(seed, base + 13, (int64_t)m.CD * kKS, 0.3f);
    L.dt_bias = gen_bf16v(seed, base + 14, c.lin_v_heads, 0.5f);
    const auto al = gen_bf16v(seed, base + 15, c.lin_v_heads, 0.5f);
    L.a_log.resize(al.size());
    for (size_t i = 0; i < al.size(); ++i) L.a_log[i] = bf2f(al[i]);
  }
  gen_qw(L.router, seed, base + 16, c.experts, H, bits, 64);
  gen_qw(L.eg, seed, base + 17, c.experts * c.expert_inter, H, bits, 64);
  gen_qw(L.eu, seed, base + 18, c.experts * c.expert_inter, H, bits, 64);
  gen_qw(L.ed, seed, base + 19, c.experts * H, c.expert_inter, bits, 64);
  gen_qw(L.sg, seed, base + 20, c.shared_inter, H, bits, 64);
  gen_qw(L.su, seed, base + 21, c.shared_inter, H, bits, 64);
  gen_qw(L.sd, seed, base + 22, H, c.shared_inter, bits, 64);
  gen_qw(L.sgate, seed, base + 23, 1, H, bits, 64);
}

void rms_ones(const uint16_t* x, uint16_t* y, int rows, int dim, float eps) {
  std::vector<uint16_t> ones(dim, f2bf(1.0f));
  orc_rms_norm(x, ones.data(), y, rows, dim, eps);
}

// gated attention of layer L over xn (B x T rows), cache layer li of kc;
// adds the output to h
void hyb_attn(HModel& m, Cache& kc, int li, const HLayer& L, const uint16_t* xn, uint16_t* h, int B, int T) {
  const orc_hybrid_cfg& c = m.c;
  const int H = c.hidden, Hq = c.heads, Hk = c.kv_heads, D = kGD, R = B * T, NQ = Hq * D, NK = Hk * D;
  std::vector<uint16_t> q((size_t)R * NQ), k((size_t)R * NK), v((size_t)R * NK), g((size_t)R * NQ),
      o((size_t)R * NQ), a((size_t)R * H);
  hqmm(L.q, xn, q.data(), R, c.bits);
  hqmm(L.k, xn, k.data(), R, c.bits);
  hqmm(L.v, xn, v.data(), R, c.bits);
  hqmm(L.qg, xn, g.data(), R, c.bits);
  rms_ones(q.data(), q.data(), R * Hq, D, c.eps);
  rms_ones(k.data(), k.data(), R * Hk, D, c.eps);
  std::vector<int32_t> pos(R);
  for (int b = 0; b < B; ++b)
    for (int t = 0; t < T; ++t) pos[b * T + t] = kc.len[b] + t;
  orc_rope(q.data(), pos.data(), R, Hq, D, m.cos_t.data(), m.sin_t.data());
  orc_rope(k.data(), pos.data(), R, Hk, D, m.cos_t.data(), m.sin_t.data());
  const float scale = (float)(1.0 / std::sqrt((double)D));
  for (int b = 0; b < B; ++b) {
    for (int t = 0; t < T; ++t)
      for (int hk = 0; hk < Hk; ++hk) {
        const size_t row = ((size_t)b * Hk + hk) * kc.cap + (size_t)(kc.len[b] + t);
        const uint16_t* ks = &k[((size_t)(b * T + t) * Hk + hk) * D];
        const uint16_t* vs = &v[((size_t)(b * T + t) * Hk + hk) * D];
        if (kc.bits == 16) {
          std::memcpy(&kc.k[li][row * D], ks, D * 2);
          std::memcpy(&kc.v[li][row * D], vs, D * 2);
        } else {
          const int WPR = D * kc.bits / 32, gpr = D / 64;
          for (int gi = 0; gi < gpr; ++gi) {
            quantize_group(ks + 64 * gi, 64, kc.bits, &kc.kq[li][row * WPR + gi * 64 * kc.bits / 32],
                           &kc.ks[li][row * gpr + gi], &kc.kb[li][row * gpr + gi]);
            quantize_group(vs + 64 * gi, 64, kc.bits, &kc.vq[li][row * WPR + gi * 64 * kc.bits / 32],
                           &kc.vs[li][row * gpr + gi], &kc.vb[li][row * gpr + gi]);
          }
        }
      }
    std::vector<uint16_t> kd, vd;
    const uint16_t *kb, *vb;
    const size_t base = (size_t)b * Hk * kc.cap;
    if (kc.bits == 16) {
      kb = &kc.k[li][base * D];
      vb = &kc.v[li][base * D];
    } else {
      const int WPR = D * kc.bits / 32, gpr = D / 64;
      kd.assign((size_t)Hk * kc.cap * D, 0);
      vd.assign(kd.size(), 0);
      for (int hk = 0; hk < Hk; ++hk)
        for (int j = 0; j < kc.len[b] + T; ++j) {
          const size_t row = base + (size_t)hk * kc.cap + j;
          for (int d = 0; d < D; ++d) {
            const int gi = d / 64;
            kd[((size_t)hk * kc.cap + j) * D + d] = f2bf(std::fma(bf2f(kc.ks[li][row * gpr + gi]),
                (float)qcode(&kc.kq[li][row * WPR], d, kc.bits), bf2f(kc.kb[li][row * gpr + gi])));
            vd[((size_t)hk * kc.cap + j) * D + d] = f2bf(std::fma(bf2f(kc.vs[li][row * gpr + gi]),
                (float)qcode(&kc.vq[li][row * WPR], d, kc.bits), bf2f(kc.vb[li][row * gpr + gi])));
          }
        }
      kb = kd.data();
      vb = vd.data();
    }
    orc_sdpa(&q[(size_t)b * T * NQ], kb, vb, &o[(size_t)b * T * NQ], T, Hq, Hk, D, kc.cap, kc.len[b], scale);
  }
  for (size_t i = 0; i < o.size(); ++i) o[i] = f2bf(bf2f(o[i]) * bf2f(f2bf(sigmoid_f(bf2f(g[i])))));
  hqmm(L.o, o.data(), a.data(), R, c.bits);
  orc_add(h, a.data(), h, (int64_t)R * H);
}

void hyb_moe(HModel& m, const HLayer& L, uint16_t* h, int R) {
  const orc_hybrid_cfg& c = m.c;
  const int H = c.hidden;
  std::vector<uint16_t> xn((size_t)R * H), rl((size_t)R * c.experts), ym((size_t)R * H), g((size_t)R * c.shared_inter),
      u(g.size()), ys((size_t)R * H), sgl(R);
  rms_ones(h, xn.data(), R, H, c.eps);
  hqmm(L.router, xn.data(), rl.data(), R, c.bits);
  std::vector<int32_t> idx((size_t)R * c.top_k);
  std::vector<float> w((size_t)R * c.top_k);
  orc_moe_route(rl.data(), R, c.experts, c.top_k, idx.data(), w.data());
  orc_moe_experts(xn.data(), R, H, c.expert_inter, c.experts, c.top_k, idx.data(), w.data(), L.eg.w.data(),
                  L.eg.s.data(), L.eg.b.data(), L.eu.w.data(), L.eu.s.data(), L.eu.b.data(), L.ed.w.data(),
                  L.ed.s.data(), L.ed.b.data(), c.bits, ym.data());
  hqmm(L.sg, xn.data(), g.data(), R, c.bits);
  hqmm(L.su, xn.data(), u.data(), R, c.bits);
  orc_swiglu(g.data(), u.data(), g.data(), (int64_t)g.size());
  hqmm(L.sd, g.data(), ys.data(), R, c.bits);
  hqmm(L.sgate, xn.data(), sgl.data(), R, c.bits);
  for (int r = 0; r < R; ++r) {
    const float gs = bf2f(f2bf(sigmoid_f(bf2f(sgl[r]))));
    for (int i = 0; i < H; ++i) {
      const size_t j = (size_t)r * H + i;
      const float t = bf2f(f2bf(gs * bf2f(ys[j])));
      const float mm = bf2f(f2bf(bf2f(ym[j]) + t));
      h[j] = f2bf(bf2f(h[j]) + mm);
    }
  }
}

// trunk forward (tokens [B][T]); commit: every GDN layer keeps the state
// after the last token; else the snapshots stay for hyb_commit.  Leaves the
// final-normed hidden in s.hid; logits (all rows, or each sequence's last)
// when non-null.  Advances the attention lengths only when commit.
void hyb_forward(HModel& m, HState& s, const int32_t* tokens, int B, int T, uint16_t* logits, bool last_only,
                 bool commit) {
  const orc_hybrid_cfg& c = m.c;
  const int H = c.hidden, R = B * T, G = H / 64, Hv = c.lin_v_heads, Z = Hv * kGD;
  std::vector<uint16_t> h((size_t)R * H), xn((size_t)R * H);
  for (int r = 0; r < R; ++r) {
    const int tok = tokens[r];
    const uint32_t* row = m.embed.w.data() + (size_t)tok * H * c.bits / 32;
    for (int i = 0; i < H; ++i)
      h[(size_t)r * H + i] = f2bf(std::fma(bf2f(m.embed.s[(size_t)tok * G + i / 64]), (float)qcode(row, i, c.bits),
                                           bf2f(m.embed.b[(size_t)tok * G + i / 64])));
  }
  int ia = 0, ig = 0;
  for (int l = 0; l < c.layers; ++l) {
    const HLayer& L = m.L[l];
    rms_ones(h.data(), xn.data(), R, H, c.eps);
    if (L.attn) {
      hyb_attn(m, *s.kv, ia++, L, xn.data(), h.data(), B, T);
    } else {
      HGdn& g = s.gdn[ig++];
      g.qkv.resize((size_t)R * m.CD);
      std::vector<uint16_t> z((size_t)R * Z), bb((size_t)R * Hv), aa((size_t)R * Hv), out((size_t)R * Z),
          a((size_t)R * H), gnorm(kGD, f2bf(1.0f));
      hqmm(L.wqkv, xn.data(), g.qkv.data(), R, c.bits);
      hqmm(L.wz, xn.data(), z.data(), R, c.bits);
      hqmm(L.wb, xn.data(), bb.data(), R, c.bits);
      hqmm(L.wa, xn.data(), aa.data(), R, c.bits);
      g.snap.assign((size_t)B * T * Hv * kGD * kGD, 0.0f);
      orc_gdn_verify(B, T, c.lin_k_heads, Hv, g.qkv.data(), z.data(), bb.data(), aa.data(), L.conv_w.data(),
                     L.a_log.data(), L.dt_bias.data(), gnorm.data(), c.eps, g.conv.data(), g.state.data(),
                     g.snap.data(), out.data());
      if (commit) {
        std::vector<int32_t> last(B, T - 1);
        orc_gdn_commit(B, T, c.lin_k_heads, Hv, g.qkv.data(), g.snap.data(), last.data(), g.state.data(),
                       g.conv.data());
      }
      hqmm(L.wout, out.data(), a.data(), R, c.bits);
      orc_add(h.data(), a.data(), h.data(), (int64_t)R * H);
    }
    hyb_moe(m, L, h.data(), R);
  }
  s.hid.resize((size_t)R * H);
  rms_ones(h.data(), s.hid.data(), R, H, c.eps);
  s.T = T;
  if (commit && s.kv)
    for (int b = 0; b < B; ++b) s.kv->len[b] += T;
  if (!logits) return;
  if (last_only) {
    std::vector<uint16_t> hl((size_t)B * H);
    for (int b = 0; b < B; ++b) std::memcpy(&hl[(size_t)b * H], &s.hid[((size_t)b * T + T - 1) * H], H * 2);
    hqmm(m.lm_head, hl.data(), logits, B, c.bits);
  } else {
    hqmm(m.lm_head, s.hid.data(), logits, R, c.bits);
  }
}
}  // namespace

extern "C" void* orc_hybrid_create(const orc_hybrid_cfg* cfg, uint64_t seed) {
  auto m = std::make_unique<HModel>();
  m->c = *cfg;
  const orc_hybrid_cfg& c = *cfg;
  if (c.bits != 4 && c.bits != 8) return nullptr;
  m->CD = 2 * c.lin_k_heads * kGD + c.lin_v_heads * kGD;
  m->L.resize(c.layers);
  for (int l = 0; l < c.layers; ++l) {
    const bool attn = l % c.attn_every == c.attn_every - 1;
    (attn ? m->n_attn : m->n_gdn)++;
    hyb_layer_gen(*m, m->L[l], l, attn, seed);
  }
  hyb_layer_gen(*m, m->mtp, c.layers, true, seed);
  gen_qw(m->embed, seed, 1, c.vocab, c.hidden, c.bits, 64);
  gen_qw(m->lm_head, seed, 2, c.vocab, c.hidden, c.bits, 64);
  gen_qw(m->mtp_fc, seed, 3, c.hidden, 2 * c.hidden, c.bits, 64);
  m->cos_t.resize((size_t)m->max_pos * kGD / 2);
  m->sin_t.resize(m->cos_t.size());
  orc_rope_table(m->max_pos, kGD, c.rope_theta, m->cos_t.data(), m->sin_t.data());
  return m.release();
}
extern "C" void orc_hybrid_free(void* m) { delete (HModel*)m; }

namespace {
HState* hyb_state_new(HModel& m, int B, int cap, int kv_bits) {
  auto s = std::make_unique<HState>();
  s->B = B;
  s->cap = cap;
  Model shape;  // cache geometry
  shape.c.kv_heads = m.c.kv_heads;
  shape.c.head_dim = kGD;
  if (m.n_attn) s->kv.reset((Cache*)orc_cache_create(&shape, m.n_attn, B, cap, kv_bits));
  s->mtp_kv.reset((Cache*)orc_cache_create(&shape, 1, B, 8, kv_bits));
  s->gdn.resize(m.n_gdn);
  for (auto& g : s->gdn) {
    g.conv.assign((size_t)B * (kKS - 1) * m.CD, 0);
    g.state.assign((size_t)B * m.c.lin_v_heads * kGD * kGD, 0.0f);
  }
  return s.release();
}
}  // namespace

extern "C" void* orc_hybrid_state_create(void* mp, int B, int cap, int kv_bits) {
  return hyb_state_new(*(HModel*)mp, B, cap, kv_bits);
}
extern "C" void orc_hybrid_state_free(void* s) { delete (HState*)s; }
extern "C" int orc_hybrid_forward(void* mp, void* sp, const int32_t* tokens, int B, int T, uint16_t* logits) {
  HState& s = *(HState*)sp;
  if (B != s.B) return 1;
  hyb_forward(*(HModel*)mp, s, tokens, B, T, logits, false, true);
  return 0;
}

// MTP speculative decode (greedy, 2 drafts): the device engine's step.
extern "C" int orc_hybrid_spec_generate(void* mp, const int32_t* prompts, int B, int P, int MT, int kv_bits,
                                        int32_t* out, int64_t* stats) {
  HModel& m = *(HModel*)mp;
  const orc_hybrid_cfg& c = m.c;
  const int H = c.hidden, V = c.vocab, N = 3;
  std::unique_ptr<HState> s(hyb_state_new(m, B, P + MT + N + 8, kv_bits));
  std::vector<uint16_t> lg((size_t)B * N * V);
  // prefill in 32-token chunks
  std::vector<int32_t> chunk;
  for (int t0 = 0; t0 < P; t0 += 32) {
    const int tn = std::min(32, P - t0);
    chunk.resize((size_t)B * tn);
    for (int b = 0; b < B; ++b) std::memcpy(&chunk[(size_t)b * tn], prompts + (size_t)b * P + t0, tn * 4);
    hyb_forward(m, *s, chunk.data(), B, tn, t0 + tn >= P ? lg.data() : nullptr, true, true);
  }
  std::vector<int32_t> vt((size_t)B * N), pred((size_t)B * N), emitted(B, 0), acc(B);
  std::vector<uint16_t> capt((size_t)B * H), mhid((size_t)B * H);
  orc_argmax(lg.data(), B, V, pred.data());
  for (int b = 0; b < B; ++b) {
    vt[(size_t)b * N] = pred[b];
    std::memcpy(&capt[(size_t)b * H], &s->hid[((size_t)b * s->T + s->T - 1) * H], H * 2);
  }
  int64_t steps = 0, accepted = 0;
  std::vector<uint16_t> ones(H, f2bf(1.0f));
  for (int it = 0; it < MT + 1; ++it) {
    bool all = true;
    for (int b = 0; b < B; ++b) all = all && emitted[b] >= MT;
    if (all) break;
    // MTP drafts d1, d2 (cache reset to 0)
    for (int b = 0; b < B; ++b) s->mtp_kv->len[b] = 0;
    for (int i = 1; i < N; ++i) {
      const uint16_t* hin = i == 1 ? capt.data() : mhid.data();
      std::vector<uint16_t> e((size_t)B * H), cat((size_t)B * 2 * H), h((size_t)B * H), xn((size_t)B * H),
          l1((size_t)B * V);
      const int G = H / 64;
      for (int b = 0; b < B; ++b) {
        const int tok = vt[(size_t)b * N + i - 1];
        const uint32_t* row = m.embed.w.data() + (size_t)tok * H * c.bits / 32;
        for (int j = 0; j < H; ++j)
          e[(size_t)b * H + j] = f2bf(std::fma(bf2f(m.embed.s[(size_t)tok * G + j / 64]),
                                               (float)qcode(row, j, c.bits), bf2f(m.embed.b[(size_t)tok * G + j / 64])));
      }
      std::vector<uint16_t> en((size_t)B * H), hn((size_t)B * H);
      rms_ones(e.data(), en.data(), B, H, c.eps);
      rms_ones(hin, hn.data(), B, H, c.eps);
      for (int b = 0; b < B; ++b) {
        std::memcpy(&cat[(size_t)b * 2 * H], &en[(size_t)b * H], H * 2);
        std::memcpy(&cat[(size_t)b * 2 * H + H], &hn[(size_t)b * H], H * 2);
      }
      hqmm(m.mtp_fc, cat.data(), h.data(), B, c.bits);
      rms_ones(h.data(), xn.data(), B, H, c.eps);
      hyb_attn(m, *s->mtp_kv, 0, m.mtp, xn.data(), h.data(), B, 1);
      hyb_moe(m, m.mtp, h.data(), B);
      for (int b = 0; b < B; ++b) s->mtp_kv->len[b] += 1;
      mhid = h;
      rms_ones(h.data(), xn.data(), B, H, c.eps);
      hqmm(m.lm_head, xn.data(), l1.data(), B, c.bits);
      std::vector<int32_t> d(B);
      orc_argmax(l1.data(), B, V, d.data());
      for (int b = 0; b < B; ++b) vt[(size_t)b * N + i] = d[b];
    }
    // verify
    hyb_forward(m, *s, vt.data(), B, N, lg.data(), false, false);
    orc_argmax(lg.data(), B * N, V, pred.data());
    for (int b = 0; b < B; ++b) {
      int e = emitted[b];
      if (e >= MT) {
        acc[b] = -1;
        continue;
      }
      int a = 0;
      while (a < N - 1 && pred[(size_t)b * N + a] == vt[(size_t)b * N + a + 1]) ++a;
      for (int i = 0; i <= a && e < MT; ++i) out[(size_t)b * MT + e++] = vt[(size_t)b * N + i];
      emitted[b] = e;
      accepted += a;
      steps += 1;
      if (s->kv) s->kv->len[b] += a + 1;
      vt[(size_t)b * N] = pred[(size_t)b * N + a];
      acc[b] = a;
    }
    for (auto& g : s->gdn)
      orc_gdn_commit(B, N, c.lin_k_heads, c.lin_v_heads, g.qkv.data(), g.snap.data(), acc.data(), g.state.data(),
                     g.conv.data());
    for (int b = 0; b < B; ++b)
      if (acc[b] >= 0) std::memcpy(&capt[(size_t)b * H], &s->hid[((size_t)b * N + acc[b]) * H], H * 2);
  }
  if (stats) {
    int64_t em = 0;
    for (int b = 0; b < B; ++b) em += emitted[b];
    stats[0] = steps;
    stats[1] = steps * (N - 1);
    stats[2] = accepted;
    stats[3] = em;
    stats[4] = 0;
  }
  return 0;
}

extern "C" int orc_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* Set the OpenMP thread count of every later oracle call (n <= 0: one per
 * online host core).  Launchers such as torch.distributed.run export
 * OMP_NUM_THREADS=1, which would leave the CPU baseline single-threaded. */
extern "C" int orc_set_threads(int n) {
#ifdef _OPENMP
  if (n <= 0) n = omp_get_num_procs();
  omp_set_num_threads(n);
  return omp_get_max_threads();
#else
  (void)n;
  return 1;
#endif
}
