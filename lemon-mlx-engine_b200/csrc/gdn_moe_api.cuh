// gdn_moe_api.cuh -- C ABI of the hybrid-model ops (gdn_moe.cuh):
// lmx_gdn_verify / lmx_gdn_commit, lmx_moe_route, lmx_moe_experts.
#pragma once
#include "gdn_moe.cuh"
#include "lmx_internal.h"

namespace lmx {

static size_t gdn_scratch_bytes(int B, int T, int Hk, int Hv) {
  auto up = [](size_t x) { return (x + 255) / 256 * 256; };
  const size_t bt = (size_t)B * T;
  return up(bt * Hk * kGdnD * 2) * 2 + up(bt * Hv * kGdnD * 2) + up(bt * Hv * 4) * 2;
}

static int gdn_args(const lmx_gdn* g, GdnArgs& a) {
  if (!g || g->batch < 1 || g->T < 1 || g->k_heads < 1 || g->v_heads < 1 || g->v_heads % g->k_heads)
    return set_error(LMX_ERR_INVALID, "gdn: bad shape");
  if (!g->qkv || !g->z || !g->b || !g->a || !g->conv_w || !g->a_log || !g->dt_bias || !g->norm_w ||
      !g->conv_state || !g->state || !g->state_snap || !g->out || !g->scratch)
    return set_error(LMX_ERR_INVALID, "gdn: null pointer");
  if (((uintptr_t)g->state | (uintptr_t)g->state_snap | (uintptr_t)g->scratch | (uintptr_t)g->out |
       (uintptr_t)g->norm_w) & 15)
    return set_error(LMX_ERR_INVALID, "gdn: state, state_snap, out, norm_w and scratch must be 16-byte aligned");
  a.B = g->batch;
  a.T = g->T;
  a.Hk = g->k_heads;
  a.Hv = g->v_heads;
  a.qkv = (const bf16_t*)g->qkv;
  a.z = (const bf16_t*)g->z;
  a.b = (const bf16_t*)g->b;
  a.a = (const bf16_t*)g->a;
  a.conv_w = (const bf16_t*)g->conv_w;
  a.a_log = g->a_log;
  a.dt_bias = (const bf16_t*)g->dt_bias;
  a.norm_w = (const bf16_t*)g->norm_w;
  a.eps = g->eps;
  a.conv_state = (const bf16_t*)g->conv_state;
  a.state = g->state;
  a.snap = g->state_snap;
  a.snap_T = g->T;
  a.state_bf16 = g_gdn_state_bf16;
  a.out = (bf16_t*)g->out;
  auto up = [](size_t x) { return (x + 255) / 256 * 256; };
  const size_t bt = (size_t)a.B * a.T;
  uint8_t* p = (uint8_t*)g->scratch;
  a.qn = (bf16_t*)p;
  p += up(bt * a.Hk * kGdnD * 2);
  a.kn = (bf16_t*)p;
  p += up(bt * a.Hk * kGdnD * 2);
  a.vc = (bf16_t*)p;
  p += up(bt * a.Hv * kGdnD * 2);
  a.beta = (float*)p;
  p += up(bt * a.Hv * 4);
  a.gdecay = (float*)p;
  return LMX_OK;
}

}  // namespace lmx

extern "C" size_t lmx_gdn_scratch_bytes(int batch, int T, int k_heads, int v_heads) {
  if (batch < 1 || T < 1 || k_heads < 1 || v_heads < 1) return 0;
  return lmx::gdn_scratch_bytes(batch, T, k_heads, v_heads);
}

extern "C" int lmx_gdn_verify(const lmx_gdn* g, void* stream) {
  using namespace lmx;
  GdnArgs a;
  int rc = gdn_args(g, a);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const long long tasks = (long long)a.B * a.T * (2 * a.Hk + a.Hv);
  rc = cuda_check(lmx_launch(gdn_prep_kernel, dim3((unsigned)((tasks + 7) / 8)), dim3(256), 0, st, true, a),
                  "gdn_prep: launch");
  if (!rc)
    rc = cuda_check(lmx_launch(gdn_recur_kernel, dim3(a.Hv, a.B), dim3(256), 0, st, true, a), "gdn_recur: launch");
  return rc;
}

extern "C" int lmx_gdn_commit(const lmx_gdn* g, const int32_t* acc, void* stream) {
  using namespace lmx;
  GdnArgs a;
  int rc = gdn_args(g, a);
  if (rc) return rc;
  if (!acc) return set_error(LMX_ERR_INVALID, "gdn_commit: null acc");
  return cuda_check(lmx_launch(gdn_commit_kernel, dim3(a.B, a.Hv + 1), dim3(256), 0, (cudaStream_t)stream, true, a,
                               acc, g->state, (bf16_t*)g->conv_state),
                    "gdn_commit: launch");
}

extern "C" int lmx_set_gdn_state_bf16(int on) {
  if (on != 0 && on != 1) return lmx::set_error(LMX_ERR_INVALID, "gdn_state_bf16: 0 or 1");
  lmx::g_gdn_state_bf16 = on;
  return LMX_OK;
}
extern "C" int lmx_gdn_state_bf16(void) { return lmx::g_gdn_state_bf16; }

extern "C" int lmx_moe_route(const void* logits, int rows, int E, int k, int32_t* idx, float* w, void* stream) {
  using namespace lmx;
  if (rows == 0) return LMX_OK;
  if (!logits || !idx || !w || rows < 0 || E < 1 || E > 16384 || k < 1 || k > 16 || k > E)
    return set_error(LMX_ERR_INVALID, "moe_route: bad arguments (k <= 16, E <= 16384)");
  return cuda_check(lmx_launch(moe_route_kernel, dim3((rows + 7) / 8), dim3(256), 0, (cudaStream_t)stream, true,
                               (const bf16_t*)logits, rows, E, k, idx, w),
                    "moe_route: launch");
}

namespace lmx {
template <int BITS, bool EP>
static int launch_moe_tt(const MoeArgs& a, cudaStream_t st) {
  static bool attr_set[64] = {};
  int d = 0;
  cudaGetDevice(&d);
  const size_t s1 = (size_t)a.H * 4, s2 = (size_t)a.k * a.I * 4;
  if (!attr_set[d & 63]) {
    int rc = cuda_check(cudaFuncSetAttribute(moe_gateup_kernel<BITS, EP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             200 * 1024),
                        "moe: smem");
    if (!rc)
      rc = cuda_check(cudaFuncSetAttribute(moe_down_kernel<BITS, EP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           200 * 1024),
                      "moe: smem");
    if (rc) return rc;
    attr_set[d & 63] = true;
  }
  int rc = cuda_check(lmx_launch(moe_gateup_kernel<BITS, EP>, dim3((a.I + 63) / 64, a.M * a.k), dim3(256), s1, st,
                                 true, a),
                      "moe_gateup: launch");
  if (!rc)
    rc = cuda_check(lmx_launch(moe_down_kernel<BITS, EP>, dim3((a.H + 63) / 64, a.M), dim3(256), s2, st, true, a),
                    "moe_down: launch");
  return rc;
}
// Expert-parallel launches (slot outputs for ep_combine_kernel) take the EP
// kernels; everything else the one-GPU kernels.
template <int BITS>
static int launch_moe_t(const MoeArgs& a, cudaStream_t st) {
  return a.slot_out ? launch_moe_tt<BITS, true>(a, st) : launch_moe_tt<BITS, false>(a, st);
}
}  // namespace lmx

extern "C" int lmx_moe_experts(const void* x, int M, int H, int I, int E, int k, const int32_t* idx, const float* w,
                               const lmx_qweights* gate, const lmx_qweights* up, const lmx_qweights* down, int bits,
                               void* act_scratch, void* y, void* stream) {
  using namespace lmx;
  if (M == 0) return LMX_OK;
  if (!x || !idx || !w || !gate || !up || !down || !act_scratch || !y || M < 0 || k < 1 || E < 1)
    return set_error(LMX_ERR_INVALID, "moe_experts: bad arguments");
  if (H % 512 || I % 512 || (bits != 4 && bits != 8))
    return set_error(LMX_ERR_UNSUPPORTED, "moe_experts: H and I multiples of 512, 4/8-bit");
  if ((size_t)H * 4 > 200 * 1024 || (size_t)k * I * 4 > 200 * 1024)
    return set_error(LMX_ERR_UNSUPPORTED, "moe_experts: H or k*I too large for shared memory");
  const lmx_qweights* q3[3] = {gate, up, down};
  for (const lmx_qweights* q : q3)
    if (!q->w || !q->scales || !q->biases || ((uintptr_t)q->w & 15))
      return set_error(LMX_ERR_INVALID, "moe_experts: weights must be 16-byte aligned");
  MoeArgs a;
  a.M = M;
  a.H = H;
  a.I = I;
  a.E = E;
  a.k = k;
  a.x = (const bf16_t*)x;
  a.idx = idx;
  a.w = w;
  a.gw = gate->w;
  a.uw = up->w;
  a.dw = down->w;
  a.gs = (const bf16_t*)gate->scales;
  a.gb = (const bf16_t*)gate->biases;
  a.us = (const bf16_t*)up->scales;
  a.ub = (const bf16_t*)up->biases;
  a.ds = (const bf16_t*)down->scales;
  a.db = (const bf16_t*)down->biases;
  a.act = (bf16_t*)act_scratch;
  a.y = (bf16_t*)y;
  a.err = device_error_word();
  return bits == 4 ? launch_moe_t<4>(a, (cudaStream_t)stream) : launch_moe_t<8>(a, (cudaStream_t)stream);
}
