// lmx.cu -- kernels' host launchers and the op-level C ABI (include/lmx.h).
#include <cudaTypedefs.h>

#include <cstdarg>
#include <map>
#include <tuple>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "lmx_internal.h"
#include "norm_argmax.cuh"
#include "qmm.cuh"
#include "qmm_mma.cuh"
#include "attn.cuh"
#include "attn_mma.cuh"
#include "qmv_tc.cuh"
#include "qmm_tcs.cuh"
#include "engine_kernels.cuh"
#include "sample.cuh"
#include "tp.cuh"
#include "decode.cuh"

// Device error word: bounded waits that give up record a code here.
__device__ unsigned g_lmx_kernel_error;

namespace lmx {

namespace {
thread_local std::string t_last_error;

struct DevInfo {
  bool init = false;
  int sms = 0;
  unsigned* err = nullptr;
};
DevInfo g_dev[64];
std::mutex g_dev_mu;

DevInfo& dev() {
  int d = 0;
  cudaGetDevice(&d);
  DevInfo& di = g_dev[d & 63];
  if (!di.init) {
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (!di.init) {
      cudaDeviceGetAttribute(&di.sms, cudaDevAttrMultiProcessorCount, d);
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_lmx_kernel_error) == cudaSuccess) di.err = (unsigned*)p;
      di.init = true;
    }
  }
  return di;
}
}  // namespace

int set_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

int cuda_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return LMX_OK;
  return set_error(LMX_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int device_sms() { return dev().sms; }
unsigned* device_error_word() { return dev().err; }

// ---------------------------------------------------------------------------
// TMA tensor maps (cuTensorMapEncodeTiled through the runtime's driver entry
// point), cached per (address, shape, box): weights never move, so the maps
// of a model are encoded once.
// ---------------------------------------------------------------------------
namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::mutex g_map_mu;
std::map<std::tuple<const void*, int, uint64_t, uint64_t, int, int, int>, CUtensorMap> g_maps;
}  // namespace

static int tensor_map_2d(const void* base, CUtensorMapDataType dt, int esize, uint64_t cols, uint64_t rows,
                         int box_w, int box_h, CUtensorMap* out,
                         CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_NONE) {
  std::lock_guard<std::mutex> lk(g_map_mu);
  const auto key = std::make_tuple(base, (int)dt, cols, rows, box_w, box_h, (int)swz);
  auto it = g_maps.find(key);
  if (it != g_maps.end()) {
    *out = it->second;
    return LMX_OK;
  }
  if (!g_encode) {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess || !fn)
      return set_error(LMX_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    g_encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
  }
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * (uint64_t)esize};
  cuuint32_t box[2] = {(cuuint32_t)box_w, (cuuint32_t)box_h};
  cuuint32_t estr[2] = {1, 1};
  CUtensorMap m;
  CUresult r = g_encode(&m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(LMX_ERR_INVALID, "tensor map encode failed (%d)", (int)r);
  g_maps[key] = m;
  *out = m;
  return LMX_OK;
}

// ---------------------------------------------------------------------------
// K1 launcher
// ---------------------------------------------------------------------------
// Plan the K1 launch: warps per row, segments per warp, ring depth and the
// shared-memory layout (must match qmv_kernel).
struct QmvShape {
  QmvPlan p;
  int csize, RB;
  size_t smem;
};

static int qmv_plan(int K, int MT, int bits, bool sb_aligned, QmvShape& out) {
  constexpr int NW = kQmmThreads / 32;
  const int SEGB = 64 * bits;
  const int nseg = (K + 511) / 512, G = K / 64, KWB = K * bits / 8;
  QmvPlan& p = out.p;
  // one 512-k segment per warp: W warps per row (a cluster when W > 8)
  if (nseg <= NW) {
    out.csize = 1;
    p.W = nseg;
    p.rs = NW / nseg;
  } else {
    out.csize = (nseg + NW - 1) / NW;
    p.W = NW;
    p.rs = 1;
  }
  p.SPW = 1;
  if (out.csize > 8) return set_error(LMX_ERR_UNSUPPORTED, "qmm: K=%d too large", K);
  p.sb_bulk = (G % 8) == 0 && sb_aligned;
  p.RP = SEGB;
  (void)KWB;
  int RB = MT == 1 ? 16 : (MT == 8 ? 4 : 8);
  int nst = 0;
  for (;; RB /= 2) {
    const int V = RB * MT;
    // scale / bias regions: two halves at 128-byte aligned offsets (TMA
    // destinations must be 128-byte aligned; SWIGLU loads each half apart)
    p.SPH = ((RB / 2) * 16 + 127) / 128 * 128;
    p.SP = p.sb_bulk ? 2 * p.SPH : 0;
    p.stage = ((RB * p.RP + 2 * p.SP) + 127) / 128 * 128;
    p.red_off = kQmmMaxNormRows * 4;
    const int red_size = (p.W > 1 || out.csize > 1) ? 2 * NW * p.SPW * V * 4 : 0;
    p.vbuf_off = (p.red_off + red_size + 127) / 128 * 128;
    const int vbuf_size = NW * V * 32 * 4;
    p.bar_off = p.vbuf_off + vbuf_size;
    const int budget = MT <= 2 ? 110 * 1024 : 200 * 1024;  // two CTAs per SM for MT <= 2
    const int fixed = p.bar_off + NW * 8 * 8 + 128;
    nst = (budget - fixed) / (NW * p.stage);
    if (nst >= 2 || RB <= 4) break;
  }
  out.RB = RB;
  if (nst > 6) nst = 6;
  if (nst < 2) return set_error(LMX_ERR_UNSUPPORTED, "qmm: K=%d stage too large", K);
  p.nst = nst;
  p.stage_off = (p.bar_off + NW * nst * 8 + 127) / 128 * 128;
  out.smem = (size_t)p.stage_off + (size_t)NW * nst * p.stage;
  return LMX_OK;
}

template <int BITS, int MT, int RB>
static int launch_qmv_t(const QmmArgs& a_in, const QmvShape& sh, cudaStream_t st) {
  QmmArgs a = a_in;
  QmmMaps mp;
  std::memset(&mp, 0, sizeof(mp));
  const int boxh = a.mode == QMM_SWIGLU ? RB / 2 : RB;
  const int G = a.K / 64, WPR = a.K * BITS / 32;
  int pv = 0, cv = 0;
  for (int i = 0; i < a.nmat; ++i) {
    a.pstart[i] = pv;
    a.cstart[i] = cv;
    pv += (a.mat[i].rows + RB - 1) / RB * RB;
    cv += a.mat[i].rows;
    int rc = tensor_map_2d(a.mat[i].w, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, WPR, a.mat[i].rows, 16 * BITS, boxh, &mp.w[i]);
    if (!rc && sh.p.sb_bulk)
      rc = tensor_map_2d(a.mat[i].s, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, G, a.mat[i].rows, 8, boxh, &mp.s[i]);
    if (!rc && sh.p.sb_bulk)
      rc = tensor_map_2d(a.mat[i].b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, G, a.mat[i].rows, 8, boxh, &mp.b[i]);
    if (rc) return rc;
  }
  a.items = a.mode == QMM_SWIGLU ? ((a.N + RB / 2 - 1) / (RB / 2)) * RB
                                 : a.pstart[a.nmat - 1] + a.mat[a.nmat - 1].rows;
  static bool attr_set[64] = {};
  int d = 0;
  cudaGetDevice(&d);
  if (!attr_set[d & 63]) {
    int rc = cuda_check(cudaFuncSetAttribute(qmv_kernel<BITS, MT, RB>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024),
                        "qmm: set smem");
    if (rc) return rc;
    cudaFuncSetAttribute(qmv_kernel<BITS, MT, RB>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    attr_set[d & 63] = true;
  }
  const int nbatch = (a.items + RB - 1) / RB;
  int nclusters = (nbatch + sh.p.rs - 1) / sh.p.rs;
  const int max_clusters = device_sms() * (MT <= 2 ? 2 : 1) / sh.csize;
  if (nclusters > max_clusters) nclusters = max_clusters;
  if (nclusters < 1) nclusters = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nclusters * sh.csize);
  cfg.blockDim = dim3(kQmmThreads);
  cfg.dynamicSmemBytes = sh.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  int na = 1;
  if (sh.csize > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = sh.csize;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    na = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cuda_check(lmx_counted(cudaLaunchKernelEx(&cfg, qmv_kernel<BITS, MT, RB>, mp, a, sh.p)), "qmm: launch");
}

template <int BITS>
static int launch_qmv_bits(const QmmArgs& a, cudaStream_t st) {
  const int MT = a.M <= 1 ? 1 : (a.M <= 2 ? 2 : (a.M <= 4 ? 4 : 8));
  QmvShape sh;
  bool sb_aligned = true;
  for (int i = 0; i < a.nmat; ++i)
    sb_aligned = sb_aligned && !((uintptr_t)a.mat[i].s & 15) && !((uintptr_t)a.mat[i].b & 15);
  int rc = qmv_plan(a.K, MT, BITS, sb_aligned, sh);
  if (rc) return rc;
  switch (MT * 100 + sh.RB) {
    case 116: return launch_qmv_t<BITS, 1, 16>(a, sh, st);
    case 108: return launch_qmv_t<BITS, 1, 8>(a, sh, st);
    case 104: return launch_qmv_t<BITS, 1, 4>(a, sh, st);
    case 208: return launch_qmv_t<BITS, 2, 8>(a, sh, st);
    case 204: return launch_qmv_t<BITS, 2, 4>(a, sh, st);
    case 408: return launch_qmv_t<BITS, 4, 8>(a, sh, st);
    case 404: return launch_qmv_t<BITS, 4, 4>(a, sh, st);
    case 804: return launch_qmv_t<BITS, 8, 4>(a, sh, st);
  }
  return set_error(LMX_ERR_UNSUPPORTED, "qmm: no kernel for MT=%d RB=%d", MT, sh.RB);
}

// ---------------------------------------------------------------------------
// K1 tensor-core path (M >= the threshold, default 16; 0 disables it)
// ---------------------------------------------------------------------------
static int g_mma_min_m = 16;
static int g_tcg_min_m = 4;
// M in [the tcgen05 threshold, g_tcs_max_m] runs the mid-batch mma.sync
// GEMM (qmm_tcs.cuh) instead of the tcgen05 kernel; 0 = never (default)
static int g_tcs_max_m = 0;
// matrices of at least this many 16-row tiles take the warp-per-tile form
// of the small-batch GEMV (qmv_tc_rows_kernel); 0 = never
static int g_tcg_rows_min_tiles = 1024;
int qmm_mma_min_m() { return g_mma_min_m; }
bool qmm_uses_mma(int M) { return g_mma_min_m > 0 && M >= g_mma_min_m; }
// the small-batch tensor-core GEMV (qmv_tc.cuh): M in [g_tcg_min_m, the
// tcgen05 threshold), tensor-core mode only (off in exact mode)
bool qmm_uses_tcg(int M) { return g_mma_min_m > 0 && g_tcg_min_m > 0 && M >= g_tcg_min_m && M < g_mma_min_m && M <= 16; }

// Activation map: bf16 [M][ldx], box {64, box_h}, 128-byte swizzle (the UMMA
// K-major canonical layout).  Encoded per launch: activation buffers vary.
static int tensor_map_x(const void* base, uint64_t K, uint64_t M, uint64_t ldx, int box_h, CUtensorMap* out) {
  {
    std::lock_guard<std::mutex> lk(g_map_mu);
    if (!g_encode) {
      cudaDriverEntryPointQueryResult q;
      void* fn = nullptr;
      if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess || !fn)
        return set_error(LMX_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
      g_encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
    }
  }
  cuuint64_t dims[2] = {K, M};
  cuuint64_t strides[1] = {ldx * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_h};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(LMX_ERR_INVALID, "activation tensor map encode failed (%d)", (int)r);
  return LMX_OK;
}

struct MmaShape {
  int Mpad = 0, mtiles = 0, np = 0, na = 0, per_sm = 1, acc_cols = 0, tmem_cols = 0;
  size_t smem = 0;
};

// Token tiles of at most 256 (UMMA N), padded to 16.  TMEM: accumulator
// (power of two >= Mpad, >= 32 columns) + na A stages of 64 columns (one
// step of two chunks each).  Two CTAs per SM (256 TMEM columns, ~112 KB of
// shared memory each) when two or more A stages and three or more packed
// stages fit; else one CTA per SM with the whole TMEM and shared memory.
static int mma_plan(int M, int bits, MmaShape& sh) {
  (void)bits;
  sh.mtiles = (M + 255) / 256;
  const int mper = (M + sh.mtiles - 1) / sh.mtiles;
  sh.Mpad = (mper + 15) / 16 * 16;
  sh.acc_cols = sh.Mpad <= 32 ? 32 : (sh.Mpad <= 64 ? 64 : (sh.Mpad <= 128 ? 128 : 256));
  const int xstage = kMmaStep * sh.Mpad * kMmaK * 2, pstage = kMmaRows * 128;
  const int fixed = 1024 + (2 * kMmaMaxPStages + 3 * kMmaMaxAStages + 1) * 8 + 16;
  for (sh.per_sm = 2; sh.per_sm >= 1; --sh.per_sm) {
    sh.tmem_cols = sh.per_sm == 2 ? 256 : 512;
    const int budget = sh.per_sm == 2 ? 112 * 1024 : 227 * 1024;
    const int min_np = sh.per_sm == 2 ? 3 : 2;
    int na = (sh.tmem_cols - sh.acc_cols) / 64;
    const int na_smem = (budget - fixed - min_np * pstage) / xstage;
    if (na > na_smem) na = na_smem;
    if (na > kMmaMaxAStages) na = kMmaMaxAStages;
    if (na < 2) continue;
    int np = (budget - fixed - na * xstage) / pstage;
    if (np > kMmaMaxPStages) np = kMmaMaxPStages;
    if (np < min_np) continue;
    sh.na = na;
    sh.np = np;
    break;
  }
  if (sh.per_sm < 1) return set_error(LMX_ERR_UNSUPPORTED, "qmm: token tile %d too large", sh.Mpad);
  if ((size_t)sh.Mpad * kMmaRows * 4 > (size_t)sh.na * xstage + (size_t)sh.np * pstage)
    return set_error(LMX_ERR_UNSUPPORTED, "qmm: reduction tile does not fit");
  sh.smem = (size_t)fixed + (size_t)sh.na * xstage + (size_t)sh.np * pstage;
  return LMX_OK;
}

template <int BITS>
static int launch_mma_t(const QmmArgs& q, cudaStream_t st) {
  MmaShape sh;
  int rc = mma_plan(q.M, BITS, sh);
  if (rc) return rc;
  MmaArgs a;
  std::memset(&a, 0, sizeof(a));
  MmaMaps mp;
  std::memset(&mp, 0, sizeof(mp));
  const bool swiglu = q.mode == QMM_SWIGLU;
  const int WPR = q.K * BITS / 32, boxh = swiglu ? kMmaRows / 2 : kMmaRows;
  int ntiles = 0, cv = 0;
  for (int i = 0; i < q.nmat; ++i) {
    a.mat[i] = q.mat[i];
    a.tstart[i] = ntiles;
    a.cstart[i] = cv;
    ntiles += (q.mat[i].rows + kMmaRows - 1) / kMmaRows;
    cv += q.mat[i].rows;
    // 128-byte rows (kMmaPackChunks chunks), 128-byte swizzle
    rc = tensor_map_2d(q.mat[i].w, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, WPR, q.mat[i].rows, 32, boxh, &mp.w[i],
                       CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  if (swiglu) ntiles = (q.N + kMmaRows / 2 - 1) / (kMmaRows / 2);
  rc = tensor_map_x(q.x, q.K, q.M, q.ldx, sh.Mpad, &mp.x);
  if (rc) return rc;
  a.nmat = q.nmat;
  a.N = q.N;
  a.M = q.M;
  a.Mpad = sh.Mpad;
  a.K = q.K;
  a.mode = q.mode;
  a.np = sh.np;
  a.na = sh.na;
  a.sb_vec = (q.K % 512) == 0;
  for (int i = 0; i < q.nmat; ++i)
    a.sb_vec = a.sb_vec && !((uintptr_t)q.mat[i].s & 15) && !((uintptr_t)q.mat[i].b & 15);
  a.acc_cols = sh.acc_cols;
  a.tmem_cols = sh.tmem_cols;
  a.y = q.y;
  a.ldy = q.ldy;
  a.res = q.res;
  a.err = q.err;
  static bool attr_set[64] = {};
  int d = 0;
  cudaGetDevice(&d);
  if (!attr_set[d & 63]) {
    rc = cuda_check(cudaFuncSetAttribute(qmm_mma_kernel<BITS>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024),
                    "qmm_mma: set smem");
    if (rc) return rc;
    attr_set[d & 63] = true;
  }
  // split-K factor: the largest (up to 8, >= 2 chunks per CTA) whose grid
  // fits one wave of two CTAs per SM (each CTA's pipeline is latency-bound,
  // so a second resident CTA adds throughput) on the SMs whole clusters can
  // reach: clusters are placed within a GPC, and a grid of 6-CTA clusters was
  // seen to reach 142 of 148 SMs, so 4% of the SMs are held back
  const int nk = q.K / kMmaK, base = ntiles * sh.mtiles;
  const int slots = sh.per_sm * (device_sms() * 96 / 100);
  int ks = 1;
  for (int k = kMmaMaxSplit; k >= 2; --k) {
    if (k > nk / 2) continue;
    if (base * k <= slots) {
      ks = k;
      break;
    }
  }
  a.ks = ks;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ntiles * ks, sh.mtiles);
  cfg.blockDim = dim3(kMmaThreads);
  cfg.dynamicSmemBytes = sh.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  int na = 1;
  if (ks > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = ks;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    na = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cuda_check(lmx_counted(cudaLaunchKernelEx(&cfg, qmm_mma_kernel<BITS>, mp, a)), "qmm_mma: launch");
}

template <int BITS>
static int launch_tcg_t(const QmmArgs& a, cudaStream_t st) {
  int tiles = 0;
  if (a.mode == QMM_SWIGLU) {
    tiles = (a.N + kTcgRows - 1) / kTcgRows;
  } else {
    for (int i = 0; i < a.nmat; ++i) tiles += (a.mat[i].rows + kTcgRows - 1) / kTcgRows;
  }
  // many tiles (PLAIN / RESID): one warp per tile over the full K
  if (a.mode != QMM_SWIGLU && tiles >= g_tcg_rows_min_tiles && g_tcg_rows_min_tiles > 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((tiles + 7) / 8);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (a.M <= 8)
      return cuda_check(lmx_counted(cudaLaunchKernelEx(&cfg, qmv_tc_rows_kernel<BITS, 1>, a)), "qmv_tc_rows: launch");
    return cuda_check(lmx_counted(cudaLaunchKernelEx(&cfg, qmv_tc_rows_kernel<BITS, 2>, a)), "qmv_tc_rows: launch");
  }
  // split K over a cluster while the tiles fill at most two waves of 148
  // SMs and every warp keeps at least one group: at these sizes a CTA's time
  // is its chain of dependent loads, so more CTAs with fewer groups each win
  const int G = a.K / 64, nslice = a.mode == QMM_SWIGLU ? 4 : 8;
  int ks = 1;
  while (ks < 4 && tiles * (2 * ks) <= 2 * 148 && G >= nslice * (2 * ks)) ks *= 2;
  // the (scale, bias) table: rows of the tile x (groups of one rank + 1) words
  const size_t smem = (size_t)(a.mode == QMM_SWIGLU ? 2 * kTcgRows : kTcgRows) * ((G + ks - 1) / ks + 1) * 4;
  static size_t smem_set[2][64] = {};
  int d = 0;
  cudaGetDevice(&d);
  if (smem > 32 * 1024 && smem > smem_set[a.M > 8][d & 63]) {
    const void* fn = a.M <= 8 ? (const void*)qmv_tc_kernel<BITS, 1> : (const void*)qmv_tc_kernel<BITS, 2>;
    int rc = cuda_check(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                        "qmv_tc: set smem");
    if (rc) return rc;
    smem_set[a.M > 8][d & 63] = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles * ks);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  int na = 1;
  if (ks > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = ks;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    na = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  if (a.M <= 8)
    return cuda_check(lmx_counted(cudaLaunchKernelEx(&cfg, qmv_tc_kernel<BITS, 1>, a, ks)), "qmv_tc: launch");
  return cuda_check(lmx_counted(cudaLaunchKernelEx(&cfg, qmv_tc_kernel<BITS, 2>, a, ks)), "qmv_tc: launch");
}

template <int BITS, int NT>
static int launch_tcs_nt(const QmmArgs& a, cudaStream_t st) {
  static int occ[64] = {};
  int d = 0;
  cudaGetDevice(&d);
  const size_t smem = tcs_smem(NT * 8, BITS);
  if (!occ[d & 63]) {
    int rc = cuda_check(cudaFuncSetAttribute(qmm_tcs_kernel<BITS, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem),
                        "qmm_tcs: set smem");
    if (rc) return rc;
    int n = 0;
    rc = cuda_check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, qmm_tcs_kernel<BITS, NT>, 256, smem),
                    "qmm_tcs: occupancy");
    if (rc) return rc;
    occ[d & 63] = n > 0 ? n : 1;
  }
  int tiles = 0;
  if (a.mode == QMM_SWIGLU) {
    tiles = (a.N + kTcsRows / 2 - 1) / (kTcsRows / 2);
  } else {
    int t16 = 0;
    for (int i = 0; i < a.nmat; ++i) t16 += (a.mat[i].rows + kTcgRows - 1) / kTcgRows;
    tiles = (t16 + kTcsWarps - 1) / kTcsWarps;
  }
  // split K over a cluster: the factor (<= 8, >= 2 groups per CTA) with the
  // fewest waves x groups per CTA (one CTA's time is its groups in sequence);
  // clusters reach about 96% of the SMs
  const int G = a.K / 64, slots = occ[d & 63] * (device_sms() * 96 / 100);
  int ks = 1;
  long best = -1;
  for (int k = 1; k <= kTcsMaxSplit && 2 * k <= G; ++k) {
    const long waves = ((long)tiles * k + slots - 1) / slots, cost = waves * ((G + k - 1) / k);
    if (best < 0 || cost < best) {
      best = cost;
      ks = k;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles * ks);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  int na = 1;
  if (ks > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = ks;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    na = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cuda_check(lmx_counted(cudaLaunchKernelEx(&cfg, qmm_tcs_kernel<BITS, NT>, a, ks)), "qmm_tcs: launch");
}

template <int BITS>
static int launch_tcs_t(const QmmArgs& a, cudaStream_t st) {
  if (a.M <= 24) return launch_tcs_nt<BITS, 3>(a, st);
  if (a.M <= 32) return launch_tcs_nt<BITS, 4>(a, st);
  if (a.M <= 48) return launch_tcs_nt<BITS, 6>(a, st);
  return launch_tcs_nt<BITS, 8>(a, st);
}

int launch_qmm(const QmmCall& c, cudaStream_t st) {
  if (c.M == 0 || c.N == 0) return LMX_OK;
  if (c.M < 0 || c.N < 0 || c.K <= 0 || c.K % 64)
    return set_error(LMX_ERR_INVALID, "qmm: bad shape M=%d N=%d K=%d", c.M, c.N, c.K);
  if (c.bits != 4 && c.bits != 8) return set_error(LMX_ERR_UNSUPPORTED, "qmm: bits=%d", c.bits);
  if (c.norm_w && c.M > kQmmMaxNormRows)
    return set_error(LMX_ERR_INVALID, "qmm: fused norm needs M <= %d", kQmmMaxNormRows);
  if (!c.x || !c.y || ((uintptr_t)c.x & 15))
    return set_error(LMX_ERR_INVALID, "qmm: x must be a 16-byte aligned device pointer");
  const int ldx = c.ldx ? c.ldx : c.K;
  if (ldx < c.K || (ldx & 7))
    return set_error(LMX_ERR_INVALID, "qmm: ldx=%d must be >= K and a multiple of 8", ldx);
  QmmArgs a;
  a.x = c.x;
  a.ldx = ldx;
  a.norm_w = c.norm_w;
  a.eps = c.eps;
  a.nmat = c.nmat;
  for (int i = 0; i < 3; ++i) {
    a.mat[i].w = c.mat[i].w;
    a.mat[i].s = c.mat[i].s;
    a.mat[i].b = c.mat[i].b;
    a.mat[i].rows = c.mat[i].rows;
    if (i < c.nmat && (!c.mat[i].w || ((uintptr_t)c.mat[i].w & 15) || !c.mat[i].s || !c.mat[i].b))
      return set_error(LMX_ERR_INVALID, "qmm: weight %d must be 16-byte aligned", i);
  }
  a.N = c.N;
  a.y = c.y;
  a.ldy = c.ldy;
  a.res = c.res;
  a.M = c.M;
  a.K = c.K;
  a.mode = c.mode;
  a.err = device_error_word();
  if (!c.norm_w && qmm_uses_mma(c.M) && c.M <= g_tcs_max_m && c.M <= 64)
    return c.bits == 4 ? launch_tcs_t<4>(a, st) : launch_tcs_t<8>(a, st);
  if (!c.norm_w && qmm_uses_mma(c.M)) return c.bits == 4 ? launch_mma_t<4>(a, st) : launch_mma_t<8>(a, st);
  if (qmm_uses_tcg(c.M)) return c.bits == 4 ? launch_tcg_t<4>(a, st) : launch_tcg_t<8>(a, st);
  return c.bits == 4 ? launch_qmv_bits<4>(a, st) : launch_qmv_bits<8>(a, st);
}

int launch_rms_norm(const bf16_t* x, const bf16_t* w, bf16_t* y, int rows, int dim, float eps,
                    cudaStream_t st) {
  if (rows == 0) return LMX_OK;
  if (!x || !w || !y || rows < 0 || dim <= 0 || (dim & 7) || ((uintptr_t)x & 15) || ((uintptr_t)w & 15) ||
      ((uintptr_t)y & 15))
    return set_error(LMX_ERR_INVALID, "rms_norm: bad arguments (16-byte aligned rows, dim %% 8 == 0)");
  return cuda_check(lmx_launch(rms_norm_kernel, dim3(rows), dim3(256), 0, st, true, x, w, y,
                               rows, dim, eps),
                    "rms_norm: launch");
}

int launch_argmax(const bf16_t* logits, int rows, int V, int32_t* out, cudaStream_t st) {
  if (rows == 0) return LMX_OK;
  if (!logits || !out || rows < 0 || V <= 0) return set_error(LMX_ERR_INVALID, "argmax: bad arguments");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(rows * kArgmaxCluster);
  cfg.blockDim = dim3(512);
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = kArgmaxCluster;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cuda_check(lmx_counted(cudaLaunchKernelEx(&cfg, argmax_kernel, logits, V, out)), "argmax: launch");
}

}  // namespace lmx

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
using namespace lmx;

extern "C" const char* lmx_last_error(void) { return t_last_error.c_str(); }
extern "C" const char* lmx_version(void) { return "lmx-b200 0.1"; }

extern "C" int lmx_device_error(unsigned* code, int clear) {
  unsigned v = 0;
  int rc = cuda_check(cudaMemcpyFromSymbol(&v, g_lmx_kernel_error, sizeof(v)), "device_error");
  if (rc) return rc;
  if (code) *code = v;
  if (clear && v) {
    unsigned z = 0;
    rc = cuda_check(cudaMemcpyToSymbol(g_lmx_kernel_error, &z, sizeof(z)), "device_error");
  }
  return rc;
}

extern "C" long long lmx_launch_count(void) { return g_lmx_launches.load(); }

extern "C" int lmx_set_mma_min_m(int m) {
  if (m < 0) return set_error(LMX_ERR_INVALID, "mma threshold must be >= 0");
  g_mma_min_m = m;
  return LMX_OK;
}
extern "C" int lmx_mma_min_m(void) { return g_mma_min_m; }

extern "C" int lmx_set_gemv_tc_min_m(int m) {
  if (m < 0 || m > 16) return set_error(LMX_ERR_INVALID, "gemv_tc_min_m %d (0 = off, at most 16)", m);
  g_tcg_min_m = m;
  return LMX_OK;
}

extern "C" int lmx_gemv_tc_min_m(void) { return g_tcg_min_m; }

extern "C" int lmx_set_gemm_tcs_max_m(int m) {
  if (m < 0 || m > 64) return set_error(LMX_ERR_INVALID, "gemm_tcs_max_m %d (0 = off, at most 64)", m);
  g_tcs_max_m = m;
  return LMX_OK;
}

extern "C" int lmx_gemm_tcs_max_m(void) { return g_tcs_max_m; }

extern "C" int lmx_set_gemv_tc_rows_min_tiles(int t) {
  if (t < 0) return set_error(LMX_ERR_INVALID, "gemv_tc_rows_min_tiles %d", t);
  g_tcg_rows_min_tiles = t;
  return LMX_OK;
}

extern "C" int lmx_gemv_tc_rows_min_tiles(void) { return g_tcg_rows_min_tiles; }

extern "C" int lmx_quantized_matmul(const void* x, const uint32_t* w, const void* scales,
                                    const void* biases, void* y, int M, int N, int K, int group_size,
                                    int bits, void* stream) {
  if (group_size != 64)
    return set_error(LMX_ERR_UNSUPPORTED, "quantized_matmul: group_size %d (only 64)", group_size);
  QmmCall c;
  c.x = (const bf16_t*)x;
  c.mat[0].w = w;
  c.mat[0].s = (const bf16_t*)scales;
  c.mat[0].b = (const bf16_t*)biases;
  c.mat[0].rows = N;
  c.nmat = 1;
  c.N = N;
  c.y = (bf16_t*)y;
  c.ldy = N;
  c.M = M;
  c.K = K;
  c.bits = bits;
  return launch_qmm(c, (cudaStream_t)stream);
}

extern "C" int lmx_rms_norm(const void* x, const void* w, void* y, int rows, int dim, float eps,
                            void* stream) {
  return launch_rms_norm((const bf16_t*)x, (const bf16_t*)w, (bf16_t*)y, rows, dim, eps,
                         (cudaStream_t)stream);
}

extern "C" int lmx_argmax(const void* logits, int rows, int V, int32_t* out, void* stream) {
  return launch_argmax((const bf16_t*)logits, rows, V, out, (cudaStream_t)stream);
}
#include "engine.cuh"
#include "loader.cuh"

// ---------------------------------------------------------------------------
// Attention for callers that cannot allocate device memory: a host framework
// that owns every device allocation and forbids cudaMalloc in its callbacks,
// or a latency-critical caller that must not enter the allocator.  Instead of
// caller scratch it uses one file-scope device array of kNoAllocScratchBytes,
// which every GPU that loads this library holds until the process exits.
// All calls share the array and it keeps the last call's contents, so calls
// that overlap on the GPU (different streams, or different host threads on the
// same device) race; the split counters are cleared at the start of each call.
// ---------------------------------------------------------------------------
static constexpr size_t kNoAllocScratchBytes = (size_t)16 << 20;  // 16 MiB
static __device__ __align__(256) unsigned char g_sdpa_noalloc_scratch[kNoAllocScratchBytes];

namespace {
struct NoAllocDevice {
  bool init = false;
  void* ptr = nullptr;  // device address of g_sdpa_noalloc_scratch on this device
};
NoAllocDevice g_noalloc[64];
std::mutex g_noalloc_mu;
}  // namespace

extern "C" int lmx_sdpa_decode_noalloc(const void* q, const lmx_kv* kv, int T, int heads, float scale,
                                       void* out, void* stream) {
  int device = 0;
  int rc = cuda_check(cudaGetDevice(&device), "sdpa_noalloc: device");
  if (rc) return rc;
  if (device < 0 || device >= 64) return set_error(LMX_ERR_UNSUPPORTED, "sdpa_noalloc: device %d", device);
  void* scratch = nullptr;
  {
    // one-time set-up per device (with that device current): in host code the
    // array's name is only a stand-in, so its device address is looked up
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    NoAllocDevice& nd = g_noalloc[device];
    if (!nd.init) {
      void* p = nullptr;
      rc = cuda_check(cudaGetSymbolAddress(&p, g_sdpa_noalloc_scratch), "sdpa_noalloc: symbol address");
      if (rc) return rc;
      nd.ptr = p;
      nd.init = true;
    }
    scratch = nd.ptr;
  }
  KvDesc d;
  rc = kv_from_c(kv, d);
  if (rc) return rc;
  if (T < 1 || heads < 1 || heads % d.Hk) return set_error(LMX_ERR_INVALID, "sdpa_noalloc: bad shape");
  const size_t need = sdpa_scratch_bytes(d.B, T, heads, d.Hk, d.cap);
  if (need > kNoAllocScratchBytes)
    return set_error(LMX_ERR_CAPACITY,
                     "sdpa_noalloc: this shape needs %zu bytes of scratch; the built-in array holds %zu "
                     "(use lmx_sdpa_decode with caller scratch)",
                     need, kNoAllocScratchBytes);
  size_t part_floats = 0, n_counters = 0;
  sdpa_scratch_need(d.B, T, heads / d.Hk, d.Hk, d.cap, part_floats, n_counters);
  const size_t ctr_off = (part_floats * 4 + 255) / 256 * 256;
  rc = cuda_check(cudaMemsetAsync((char*)scratch + ctr_off, 0, n_counters * 4, (cudaStream_t)stream),
                  "sdpa_noalloc: clear counters");
  if (rc) return rc;
  return sdpa_call(q, kv, T, heads, scale, scratch, kNoAllocScratchBytes, out, (cudaStream_t)stream);
}

#include "gdn_moe_api.cuh"
#include "hybrid.cuh"
